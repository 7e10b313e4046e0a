"""SafeTensors checkpoints: manifesto's reader and an FP8 checkpoint writer.

Reader -- weights.IndexFile / IndexReader / ReadTensor (weights/reader.go:23-109):
a file is an 8-byte little-endian header length N, N bytes of JSON mapping each
tensor name to {"dtype", "shape", "data_offsets": [begin, end]} (the
"__metadata__" entry is skipped), then the data section; offsets count from the
start of the data section (byte 8 + N).  Errors carry the reference's messages.

Writer -- write_file lays tensors out back to back in the order given (no holes,
as SafeTensors readers require), the header padded with spaces to a multiple of 8.

quantize_file -- whole-checkpoint FP8 quantisation of a SafeTensors file, the
file-backed form of the per-tensor amax-scaled cast: every selected floating
tensor (default: BF16/F16/F32 with two or more dimensions) becomes an F8_E4M3 (or
F8_E5M2) tensor with the same shape plus a float32 scalar "<name>_scale_inv"
(amax / fp8_max; 1 for an all-zero or non-finite tensor); everything else is
copied through.  Tensors stream through the GPU in batches over two device
slots: while batch i is on the device (upload, two kernel passes, download on
three CUDA streams), host threads write batch i-1's codes and read batch i+1 from
the file straight into page-locked memory.  The codes are the ones
mf_ckpt_quant_fp8 produces, so they are bit-identical to the oracle's
scaled cast of each tensor.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import BinaryIO, Callable, Sequence

from .dtype import DType, parse

FP8_WIRE = {DType.FLOAT8_E4M3: "F8_E4M3", DType.FLOAT8_E5M2: "F8_E5M2"}
QUANTIZABLE = (DType.BFLOAT16, DType.FLOAT16, DType.FLOAT32)


class SafeTensorsError(ValueError):
    """A malformed or incomplete SafeTensors file (the reference returns these as errors)."""


def _q(name: str) -> str:
    return json.dumps(name)  # Go's %q for the names that occur here


@dataclass(frozen=True)
class TensorMeta:
    """weights.TensorMeta (weights/reader.go:13-18)."""
    dtype: str
    shape: tuple[int, ...]
    data_offsets: tuple[int, int]

    @property
    def nbytes(self) -> int:
        return self.data_offsets[1] - self.data_offsets[0]

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


def _meta_from_json(name: str, raw) -> TensorMeta:
    if not isinstance(raw, dict):
        raise SafeTensorsError(f"safetensors tensor {_q(name)}: json: cannot unmarshal {type(raw).__name__} "
                               f"into TensorMeta")
    try:
        dt = raw.get("dtype", "")
        shape = tuple(int(d) for d in raw.get("shape", []) or [])
        offs = raw.get("data_offsets", [0, 0]) or [0, 0]
        if not isinstance(dt, str) or len(offs) != 2:
            raise TypeError("bad field types")
        return TensorMeta(dt, shape, (int(offs[0]), int(offs[1])))
    except (TypeError, ValueError) as e:
        raise SafeTensorsError(f"safetensors tensor {_q(name)}: {e}") from None


def index_reader(reader: BinaryIO) -> tuple[dict[str, TensorMeta], int]:
    """IndexReader: (name -> TensorMeta, byte offset of the data section)."""
    head = reader.read(8)
    if len(head) < 8:
        raise SafeTensorsError("safetensors index: " + ("EOF" if not head else "unexpected EOF"))
    (length,) = struct.unpack("<Q", head)
    body = reader.read(length)
    if len(body) < length:
        raise SafeTensorsError("safetensors index: " + ("EOF" if not body and length else "unexpected EOF"))
    try:
        raw = json.loads(body)
    except (ValueError, UnicodeDecodeError) as e:
        raise SafeTensorsError(f"safetensors index: {e}") from None
    if not isinstance(raw, dict):
        raise SafeTensorsError("safetensors index: json: cannot unmarshal into map")
    index = {name: _meta_from_json(name, m) for name, m in raw.items() if name != "__metadata__"}
    return index, length + 8


def index_file(path: str | os.PathLike) -> tuple[dict[str, TensorMeta], int]:
    """IndexFile: the header of the SafeTensors file at path."""
    with open(path, "rb") as f:
        return index_reader(f)


def read_tensor(path: str | os.PathLike, tensor_name: str) -> tuple[bytes, TensorMeta]:
    """ReadTensor: the raw bytes of one tensor and its entry."""
    index, base = index_file(path)
    meta = index.get(tensor_name)
    if meta is None:
        raise SafeTensorsError(f"safetensors: missing tensor {_q(tensor_name)}")
    with open(path, "rb") as f:
        f.seek(base + meta.data_offsets[0])
        data = f.read(meta.nbytes)
    if len(data) < meta.nbytes:
        raise SafeTensorsError(f"safetensors read {_q(tensor_name)}: EOF")
    return data, meta


def metadata(path: str | os.PathLike) -> dict[str, str]:
    """The header's "__metadata__" string map ({} when absent)."""
    with open(path, "rb") as f:
        (length,) = struct.unpack("<Q", f.read(8))
        raw = json.loads(f.read(length))
    md = raw.get("__metadata__") or {}
    return {str(k): str(v) for k, v in md.items()}


# ------------------------------------------------------------------ writer

@dataclass
class OutEntry:
    name: str
    dtype: str
    shape: tuple[int, ...]
    nbytes: int
    offset: int = 0  # within the data section, filled by layout()


def layout(entries: Sequence[OutEntry], meta: dict[str, str] | None = None) -> tuple[bytes, int]:
    """Assign back-to-back offsets and build the header: (length prefix + padded JSON, data size)."""
    off = 0
    head: dict = {}
    if meta:
        head["__metadata__"] = {str(k): str(v) for k, v in meta.items()}
    for e in entries:
        e.offset = off
        head[e.name] = {"dtype": e.dtype, "shape": list(e.shape), "data_offsets": [off, off + e.nbytes]}
        off += e.nbytes
    js = json.dumps(head, separators=(",", ":")).encode()
    js += b" " * (-len(js) % 8)
    return struct.pack("<Q", len(js)) + js, off


def write_file(path: str | os.PathLike, tensors: Sequence[tuple[str, str, Sequence[int], bytes]],
               meta: dict[str, str] | None = None) -> None:
    """Write (name, dtype, shape, data) tensors, in that order."""
    entries = [OutEntry(n, dt, tuple(int(d) for d in shp), len(memoryview(data).cast("B")))
               for n, dt, shp, data in tensors]
    header, _ = layout(entries, meta)
    with open(path, "wb") as f:
        f.write(header)
        for _, _, _, data in tensors:
            f.write(memoryview(data).cast("B"))


# -------------------------------------------------------- FP8 quantisation

def default_select(name: str, meta: TensorMeta) -> bool:
    """Quantise floating matrices and higher; vectors (norms, biases) stay as they are."""
    try:
        dt = parse(meta.dtype)
    except ValueError:
        return False
    return dt in QUANTIZABLE and len(meta.shape) >= 2 and meta.numel > 0


@dataclass
class QuantizeReport:
    tensors: int = 0
    quantized: int = 0
    params: int = 0                 # elements quantised
    src_bytes: int = 0
    dst_bytes: int = 0
    batches: int = 0
    seconds: float = 0.0
    scale_inv: dict[str, float] = field(default_factory=dict)


_ALIGN = 256  # device and staging offsets of every tensor in a batch (16 needed by the bulk-copy path)


def _up(x: int, a: int = _ALIGN) -> int:
    return (x + a - 1) // a * a


def _view(ptr: int, nbytes: int) -> memoryview:
    return memoryview((ctypes.c_uint8 * nbytes).from_address(ptr)).cast("B") if nbytes else memoryview(b"")


def _pread_into(fd: int, buf: memoryview, offset: int) -> None:
    done = 0
    while done < len(buf):
        n = os.preadv(fd, [buf[done:]], offset + done)
        if n <= 0:
            raise SafeTensorsError(f"safetensors read: EOF at byte {offset + done}")
        done += n


def _pwrite_all(fd: int, buf: memoryview, offset: int) -> None:
    done = 0
    while done < len(buf):
        done += os.pwrite(fd, buf[done:], offset + done)


_IO_PIECE = 64 << 20  # bytes per pread/pwrite job (the calls release the GIL and run in parallel)


def _pieces(buf: memoryview, offset: int) -> list[tuple[memoryview, int]]:
    return [(buf[p: p + _IO_PIECE], offset + p) for p in range(0, len(buf), _IO_PIECE)] or [(buf, offset)]


def quantize_file(src: str | os.PathLike, dst: str | os.PathLike, fp8_dtype: DType = DType.FLOAT8_E4M3,
                  compat: int = 0, select: Callable[[str, TensorMeta], bool] | None = None,
                  batch_bytes: int = 1 << 30, suffix: str = "_scale_inv",
                  io_threads: int = min(8, os.cpu_count() or 2)) -> QuantizeReport:
    """Quantise the SafeTensors checkpoint at src into a new file at dst (see the module text).

    batch_bytes bounds the source bytes per device slot (a larger tensor gets a
    slot of its own size); the device holds two slots.  File reads and writes run
    on io_threads threads in 64 MB pieces.  Needs an initialised backend
    (CUDABackend) on the current device."""
    from ._abi import call
    from .backend import DeviceBuffer, Event, PinnedBuffer, Stream
    from .checkpoint import make_chunks, quantise

    if fp8_dtype not in FP8_WIRE:
        raise ValueError(f"quantize_file: {fp8_dtype!r} is not an FP8 dtype")
    select = select or default_select
    t_start = time.perf_counter()
    index, base = index_file(src)
    names = sorted(index, key=lambda n: index[n].data_offsets)
    size = os.path.getsize(src)
    for n in names:
        m = index[n]
        if m.data_offsets[0] < 0 or m.data_offsets[1] < m.data_offsets[0] or base + m.data_offsets[1] > size:
            raise SafeTensorsError(f"safetensors tensor {_q(n)}: data_offsets {list(m.data_offsets)} "
                                   f"outside the file")

    # output plan: every tensor in file order; a quantised one is followed by its scale
    rep = QuantizeReport(tensors=len(names))
    out: list[OutEntry] = []
    qlist: list[tuple[str, TensorMeta, DType, OutEntry, OutEntry]] = []
    for n in names:
        m = index[n]
        if m.numel > 0 and select(n, m):
            sdt = parse(m.dtype)
            if sdt not in QUANTIZABLE:
                raise SafeTensorsError(f"safetensors tensor {_q(n)}: cannot quantise {m.dtype}")
            if m.nbytes != m.numel * sdt.size:
                raise SafeTensorsError(f"safetensors tensor {_q(n)}: {m.nbytes} bytes for shape "
                                       f"{list(m.shape)} of {m.dtype}")
            e = OutEntry(n, FP8_WIRE[fp8_dtype], m.shape, m.numel)
            es = OutEntry(n + suffix, "F32", (), 4)
            if n + suffix in index:
                raise SafeTensorsError(f"safetensors tensor {_q(n + suffix)}: name taken by the source")
            out += [e, es]
            qlist.append((n, m, sdt, e, es))
        else:
            out.append(OutEntry(n, m.dtype, m.shape, m.nbytes))
    md = {}
    try:
        md = metadata(src)
    except (ValueError, struct.error):
        md = {}
    md["quantization"] = f"per-tensor amax-scaled {FP8_WIRE[fp8_dtype]}, scale_inv = amax / fp8_max"
    header, data_size = layout(out, md)
    obase = len(header)

    # batches of consecutive quantised tensors
    batches: list[list[int]] = []
    cur, cur_bytes = [], 0
    for i, (_, m, _, _, _) in enumerate(qlist):
        b = _up(m.nbytes)
        if cur and cur_bytes + b > batch_bytes:
            batches.append(cur)
            cur, cur_bytes = [], 0
        cur.append(i)
        cur_bytes += b
    if cur:
        batches.append(cur)
    slot_src = max([sum(_up(qlist[i][1].nbytes) for i in bt) for bt in batches] or [0])
    slot_dst = max([sum(_up(qlist[i][1].numel) for i in bt) for bt in batches] or [0])
    slot_t = max([len(bt) for bt in batches] or [0])

    fin = os.open(src, os.O_RDONLY)
    fout = os.open(dst, os.O_RDWR | os.O_CREAT | os.O_TRUNC, 0o644)
    streams = slots = None
    ok = False
    pool = ThreadPoolExecutor(max_workers=max(2, min(io_threads, 32)))
    try:
        os.ftruncate(fout, obase + data_size)
        _pwrite_all(fout, memoryview(header), 0)
        # tensors that are copied through
        qset = {q[0] for q in qlist}
        for e in out:
            if e.name in qset or e.name.endswith(suffix) and e.name[: -len(suffix)] in qset:
                continue
            m = index[e.name]
            pos = 0
            while pos < m.nbytes:
                n = min(m.nbytes - pos, 64 << 20)
                _pwrite_all(fout, memoryview(os.pread(fin, n, base + m.data_offsets[0] + pos)), obase + e.offset + pos)
                pos += n
        if batches:
            up, comp, down = Stream(), Stream(), Stream()
            streams = (up, comp, down)
            slots = []
            for _ in range(min(2, len(batches))):
                slots.append({"hs": PinnedBuffer(slot_src), "hd": PinnedBuffer(slot_dst), "hsi": PinnedBuffer(4 * slot_t),
                              "ds": DeviceBuffer(slot_src), "dd": DeviceBuffer(slot_dst),
                              "da": DeviceBuffer(4 * slot_t), "dsi": DeviceBuffer(4 * slot_t),
                              "up": Event(), "comp": Event(), "down": Event(), "batch": None, "plan": None})

            def write_jobs(s) -> list:
                """The slot's finished batch as write jobs (its download must have completed)."""
                hd = _view(s["hd"].ptr, slot_dst)
                sinv = (ctypes.c_float * slot_t).from_address(s["hsi"].ptr)
                jobs = []
                for k, (i, so, do) in enumerate(s["plan"]):
                    name, m, _, e, es = qlist[i]
                    jobs += _pieces(hd[do: do + m.numel], obase + e.offset)
                    jobs.append((memoryview(struct.pack("<f", sinv[k])), obase + es.offset))
                    rep.scale_inv[name] = float(sinv[k])
                s["batch"] = None
                return [pool.submit(_pwrite_all, fout, buf, off) for buf, off in jobs]

            for bi, bt in enumerate(batches):
                s = slots[bi % len(slots)]
                writes = []
                if s["batch"] is not None:
                    s["down"].sync()
                    writes = write_jobs(s)  # the slot's previous codes go out while its next batch comes in
                plan, so, do, reads = [], 0, 0, []
                hs = _view(s["hs"].ptr, slot_src)
                for i in bt:
                    _, m, _, _, _ = qlist[i]
                    reads += [pool.submit(_pread_into, fin, buf, off)
                              for buf, off in _pieces(hs[so: so + m.nbytes], base + m.data_offsets[0])]
                    plan.append((i, so, do))
                    so += _up(m.nbytes)
                    do += _up(m.numel)
                for f in reads:
                    f.result()
                entries = [(s["ds"].ptr + so_, s["dd"].ptr + do_, qlist[i][1].numel, k, qlist[i][2])
                           for k, (i, so_, do_) in enumerate(plan)]
                call("mf_memcpy_h2d_async", s["ds"].ptr, s["hs"].ptr, so, up.handle)
                s["up"].record(up)
                comp.wait(s["up"])
                quantise(make_chunks(entries), len(entries), len(entries), s["da"].ptr, s["dsi"].ptr, fp8_dtype,
                         compat, None, comp)
                s["comp"].record(comp)
                for f in writes:  # the slot's download buffers are reused next
                    f.result()
                down.wait(s["comp"])
                call("mf_memcpy_d2h_async", s["hd"].ptr, s["dd"].ptr, do, down.handle)
                call("mf_memcpy_d2h_async", s["hsi"].ptr, s["dsi"].ptr, 4 * len(entries), down.handle)
                s["down"].record(down)
                s["batch"], s["plan"] = bi, plan
                rep.batches += 1
                rep.params += sum(qlist[i][1].numel for i in bt)
                rep.src_bytes += sum(qlist[i][1].nbytes for i in bt)
            for s in slots:
                if s["batch"] is not None:
                    s["down"].sync()
                    for f in write_jobs(s):
                        f.result()
        rep.quantized = len(qlist)
        rep.dst_bytes = obase + data_size
        ok = True
    finally:
        if slots:
            for s in slots:
                for st in streams:
                    st.sync()
                for k in ("hs", "hd", "hsi", "ds", "dd", "da", "dsi"):
                    s[k].free()
                for k in ("up", "comp", "down"):
                    s[k].close()
        if streams:
            for st in streams:
                st.close()
        pool.shutdown(wait=True)
        os.close(fin)
        os.close(fout)
        if not ok:
            os.unlink(dst)  # no half-written checkpoint is left behind
    rep.seconds = time.perf_counter() - t_start
    return rep
