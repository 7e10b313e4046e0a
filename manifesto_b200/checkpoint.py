"""Whole-checkpoint FP8 quantisation, sharded over the GPUs of one node.

Each of the N ranks (one process per GPU) owns a contiguous row range of
every tensor (``mf_ckpt_partition``: sizes differ by at most one row).  A
quantisation step is two grouped kernel launches and one collective:

  pass 1  per-tensor amax of this rank's rows          (one grouped launch)
  NCCL    max all-reduce of the amax vector (n_tensors floats, in place)
  pass 2  scaled FP8 cast of this rank's rows           (one grouped launch)

Data never leaves its GPU; the only traffic over NVLink is the amax vector.
The reference has no checkpoint writer or quantiser (it only reads
SafeTensors, weights/reader.go:23-109); the per-tensor amax-scale rule is
the one of mf_fp8_quantize.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

from . import _abi
from ._abi import call
from .backend import stream_handle
from .dtype import DType
from .errors import InvalidArgument


@dataclass(frozen=True)
class TensorSpec:
    name: str
    rows: int
    cols: int

    @property
    def numel(self) -> int:
        return self.rows * self.cols


def llama3_8b_layout(layers: int = 32, hidden: int = 4096, mlp: int = 14336, heads: int = 32, kv_heads: int = 8,
                     vocab: int = 128256) -> list[TensorSpec]:
    """Tensor shapes of a Llama-3-8B checkpoint (291 tensors, 8,030,261,248 params).

    1-D norm weights are treated as [hidden, 1] so they split by element.
    """
    head_dim = hidden // heads
    kv = kv_heads * head_dim
    specs = [TensorSpec("model.embed_tokens.weight", vocab, hidden)]
    for i in range(layers):
        p = f"model.layers.{i}."
        specs += [
            TensorSpec(p + "self_attn.q_proj.weight", hidden, hidden),
            TensorSpec(p + "self_attn.k_proj.weight", kv, hidden),
            TensorSpec(p + "self_attn.v_proj.weight", kv, hidden),
            TensorSpec(p + "self_attn.o_proj.weight", hidden, hidden),
            TensorSpec(p + "mlp.gate_proj.weight", mlp, hidden),
            TensorSpec(p + "mlp.up_proj.weight", mlp, hidden),
            TensorSpec(p + "mlp.down_proj.weight", hidden, mlp),
            TensorSpec(p + "input_layernorm.weight", hidden, 1),
            TensorSpec(p + "post_attention_layernorm.weight", hidden, 1),
        ]
    specs += [TensorSpec("model.norm.weight", hidden, 1), TensorSpec("lm_head.weight", vocab, hidden)]
    return specs


def partition(specs: Sequence[TensorSpec], world: int, rank: int) -> list[tuple[int, int]]:
    """(first_row, n_rows) of every tensor for `rank` (mf_ckpt_partition)."""
    n = len(specs)
    rows = (ctypes.c_int64 * max(1, n))(*[s.rows for s in specs])
    first = (ctypes.c_int64 * max(1, n))()
    count = (ctypes.c_int64 * max(1, n))()
    call("mf_ckpt_partition", rows, n, int(world), int(rank), first, count)
    return [(first[i], count[i]) for i in range(n)]


class Communicator:
    """NCCL communicator of the library (mf_comm_*), used for the amax exchange."""

    def __init__(self, world: int, rank: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise InvalidArgument("NCCL unique id must be 128 bytes")
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, 128)
        call("mf_comm_init", ctypes.byref(h), int(world), int(rank), buf)
        self.handle = h.value
        self.world, self.rank = world, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        call("mf_comm_unique_id", buf)
        return buf.raw

    @classmethod
    def from_store(cls, store, world: int, rank: int, key: str = "mfcuda_nccl_id") -> "Communicator":
        """Exchange the unique id through a torch.distributed Store (any backend)."""
        if rank == 0:
            store.set(key, cls.unique_id())
        uid = store.get(key)
        return cls(world, rank, bytes(uid))

    def allreduce_max(self, d_vec: int, count: int, stream=None) -> None:
        call("mf_comm_allreduce_max_f32", self.handle, int(d_vec), int(count), stream_handle(stream))

    def close(self) -> None:
        if self.handle:
            call("mf_comm_destroy", self.handle)
        self.handle = None


def make_chunks(entries: Sequence[tuple[int, int, int, int, DType]]) -> ctypes.Array:
    """entries: (src_ptr, dst_ptr, n, tensor_index, src_dtype) -> mf_chunk_desc[]."""
    arr = (_abi.ChunkDesc * max(1, len(entries)))()
    for i, (src, dst, n, t, dt) in enumerate(entries):
        arr[i] = _abi.ChunkDesc(int(src), int(dst), int(n), int(t), int(dt))
    return arr


def quantise(chunks: ctypes.Array, n_chunks: int, n_tensors: int, d_amax: int, d_scale_inv: int | None,
             fp8_dtype: DType = DType.FLOAT8_E4M3, compat: int = 0, comm: Communicator | None = None,
             stream=None) -> None:
    """mf_ckpt_quant_fp8: pass 1, optional all-reduce, pass 2 (no host sync)."""
    call("mf_ckpt_quant_fp8", chunks, int(n_chunks), int(n_tensors), int(d_amax), d_scale_inv, int(fp8_dtype),
         int(compat), comm.handle if comm is not None else None, stream_handle(stream))


class QuantPlan:
    """mf_ckpt_plan_*: the quantisation step of one chunk table in one kernel launch.

    The tensors are cut into groups of consecutive tensors (at most ``group_bytes`` of
    this rank's source each); one cooperative kernel runs, per group, an amax phase and
    -- one group later, while the group's source is still in L2 -- the cast phase, with
    the per-group amax exchanged between ranks inside the kernel through CUDA IPC peer
    memory.  Same codes, amax and scale_inv as :func:`quantise` with the same table.

    With ``world > 1`` every rank creates its plan, the ranks' ``ipc_handle`` bytes are
    gathered in rank order and passed to :meth:`connect` on every rank, and all ranks
    run the plan the same number of times; destroy it on every rank after a barrier
    that follows every rank's last run.
    """

    def __init__(self, chunks: ctypes.Array, n_chunks: int, n_tensors: int, tensor_numel: Sequence[int] | None = None,
                 group_bytes: int = 0, world: int = 1, rank: int = 0, fp8_dtype: DType = DType.FLOAT8_E4M3,
                 compat: int = 0):
        h = ctypes.c_void_p()
        ipc = ctypes.create_string_buffer(64)
        numel = (ctypes.c_int64 * max(1, n_tensors))(*[int(x) for x in tensor_numel]) if tensor_numel else None
        call("mf_ckpt_plan_create", chunks, int(n_chunks), int(n_tensors), numel, int(group_bytes), int(world),
             int(rank), int(fp8_dtype), int(compat), ctypes.byref(h), ipc if world > 1 else None)
        self.handle = h.value
        self.world, self.rank, self.n_tensors = int(world), int(rank), int(n_tensors)
        self.ipc_handle = ipc.raw if world > 1 else b""
        self._chunks = chunks  # the plan copied the table; kept only so callers' pointers stay referenced

    def connect(self, handles: Sequence[bytes]) -> None:
        """Open every other rank's exchange buffer (handles: each rank's ipc_handle, rank order)."""
        if self.world == 1:
            return
        if len(handles) != self.world or any(len(h) != 64 for h in handles):
            raise InvalidArgument(f"QuantPlan.connect: need {self.world} handles of 64 bytes")
        buf = ctypes.create_string_buffer(b"".join(handles), 64 * self.world)
        call("mf_ckpt_plan_connect", self.handle, buf)

    def connect_via_store(self, store, key: str = "mfcuda_ckpt_plan") -> None:
        """Gather the handles through a torch.distributed Store and connect."""
        if self.world == 1:
            return
        store.set(f"{key}/{self.rank}", self.ipc_handle)
        self.connect([bytes(store.get(f"{key}/{r}")) for r in range(self.world)])

    def run(self, d_amax: int | None, d_scale_inv: int | None, stream=None) -> None:
        call("mf_ckpt_plan_run", self.handle, d_amax, d_scale_inv, stream_handle(stream))

    def run_passes(self, d_amax: int | None, d_scale_inv: int | None, stream=None, passes: int = 3) -> None:
        """The same step as :meth:`run` in two launches (amax pass, then the cast pass), with the amax exchange
        done by the amax pass's last CTA (peer stores and flags) and waited for inside the cast pass.
        ``passes`` = 1 runs only the amax pass, 2 the pending cast pass, 3 both."""
        call("mf_ckpt_plan_run_passes", self.handle, int(passes), d_amax, d_scale_inv, stream_handle(stream))

    def info(self) -> dict:
        g, grid, n = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        call("mf_ckpt_plan_info", self.handle, ctypes.byref(g), ctypes.byref(grid), ctypes.byref(n))
        return {"groups": g.value, "grid": grid.value, "elements": n.value}

    def close(self) -> None:
        if self.handle:
            call("mf_ckpt_plan_destroy", self.handle)
        self.handle = None


class StreamedQuantiser:
    """Quantise checkpoints that live in (pinned) host memory, one after another.

    A checkpoint shard streams through the device in batches of whole tensors: each
    batch is uploaded, quantised (its tensors' amax, the all-reduce when there is a
    communicator, the cast) and downloaded on three CUDA streams -- upload, compute,
    download -- over two device slots, so a batch's FP8 download runs on the PCIe link
    while the next batch's BF16 upload runs in the other direction, and only the last
    batch's download is left when the last upload ends.  Per-tensor scaling needs a
    whole tensor, never a whole checkpoint, so batching changes no result.
    ``submit`` returns as soon as the work is queued.

    sizes[t] is this rank's element count of tensor t (its row range); the host
    buffers hold the shards back to back in tensor order: source (2 bytes per element
    for BF16/F16, 4 for F32), FP8 destination (1 byte per element) and the float32
    scale_inv vector.  Tensors are cut into batches of at most ``batch_bytes`` of
    source by ``batch_sizes`` (default: sizes); with a communicator every rank must
    pass the same batch_sizes (the global tensor sizes, say), because each batch is one
    all-reduce.
    """

    def __init__(self, sizes: Sequence[int], fp8_dtype: DType = DType.FLOAT8_E4M3, compat: int = 0,
                 comm: Communicator | None = None, src_dtype: DType = DType.BFLOAT16, batch_bytes: int = 1 << 30,
                 batch_sizes: Sequence[int] | None = None):
        from .backend import DeviceBuffer, Event, Stream
        self.sizes = [int(s) for s in sizes]
        self.n_tensors = len(self.sizes)
        self.total = sum(self.sizes)
        self.esize = 2 if src_dtype in (DType.BFLOAT16, DType.FLOAT16) else 4
        self.src_dtype, self.fp8_dtype, self.compat, self.comm = src_dtype, fp8_dtype, compat, comm
        key = [int(s) for s in (batch_sizes if batch_sizes is not None else sizes)]
        if len(key) != self.n_tensors:
            raise ValueError(f"StreamedQuantiser: {len(key)} batch sizes for {self.n_tensors} tensors")
        # batches: consecutive tensor ranges [t0, t1)
        self.batches: list[tuple[int, int]] = []
        t0, acc = 0, 0
        for t in range(self.n_tensors):
            b = self.esize * key[t]
            if t > t0 and acc + b > batch_bytes:
                self.batches.append((t0, t))
                t0, acc = t, 0
            acc += b
        if self.n_tensors:
            self.batches.append((t0, self.n_tensors))
        self.offsets = [0]
        for n in self.sizes:
            self.offsets.append(self.offsets[-1] + n)
        slot_elems = max([self.offsets[b] - self.offsets[a] for a, b in self.batches] or [0])
        slot_t = max([b - a for a, b in self.batches] or [1])
        self.up, self.compute, self.down = Stream(), Stream(), Stream()
        self.slots = []
        for _ in range(2):
            src = DeviceBuffer(max(1, self.esize * slot_elems))
            dst = DeviceBuffer(max(1, slot_elems))
            amax = DeviceBuffer(4 * slot_t)
            sinv = DeviceBuffer(4 * slot_t)
            chunks = []
            for a, b in self.batches:
                entries, off = [], 0
                for t in range(a, b):
                    entries.append((src.ptr + self.esize * off, dst.ptr + off, self.sizes[t], t - a, src_dtype))
                    off += self.sizes[t]
                chunks.append(make_chunks(entries))
            self.slots.append({"src": src, "dst": dst, "amax": amax, "sinv": sinv, "chunks": chunks,
                               "uploaded": Event(), "computed": Event(), "downloaded": Event(), "used": False})
        self.count = 0

    def submit(self, host_src: int, host_dst: int, host_scale_inv: int) -> None:
        """Queue one checkpoint: host_src -> device -> quantise -> host_dst, host_scale_inv."""
        for bi, (a, b) in enumerate(self.batches):
            s = self.slots[self.count % 2]
            if s["used"]:
                self.up.wait(s["downloaded"])  # the slot's previous results have left the device
            e0, e1 = self.offsets[a], self.offsets[b]
            call("mf_memcpy_h2d_async", s["src"].ptr, int(host_src) + self.esize * e0, self.esize * (e1 - e0),
                 self.up.handle)
            s["uploaded"].record(self.up)
            self.compute.wait(s["uploaded"])
            quantise(s["chunks"][bi], b - a, b - a, s["amax"].ptr, s["sinv"].ptr, self.fp8_dtype, self.compat,
                     self.comm, self.compute)
            s["computed"].record(self.compute)
            self.down.wait(s["computed"])
            call("mf_memcpy_d2h_async", int(host_dst) + e0, s["dst"].ptr, e1 - e0, self.down.handle)
            call("mf_memcpy_d2h_async", int(host_scale_inv) + 4 * a, s["sinv"].ptr, 4 * (b - a), self.down.handle)
            s["downloaded"].record(self.down)
            s["used"] = True
            self.count += 1

    def synchronize(self) -> None:
        for st in (self.up, self.compute, self.down):
            st.sync()

    def close(self) -> None:
        self.synchronize()
        for s in self.slots:
            for k in ("src", "dst", "amax", "sinv"):
                s[k].free()
            for k in ("uploaded", "computed", "downloaded"):
                s[k].close()
        for st in (self.up, self.compute, self.down):
            st.close()
