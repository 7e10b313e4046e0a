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


class StreamedQuantiser:
    """Quantise checkpoints that live in (pinned) host memory, one after another.

    A checkpoint shard is uploaded, quantised and downloaded in a pipeline of
    three CUDA streams -- upload, compute, download -- over two device slots,
    so the FP8 download of checkpoint i runs on the PCIe link while the BF16
    upload of checkpoint i+1 runs in the other direction, and the kernels run
    between them.  ``submit`` returns as soon as the work is queued.

    sizes[t] is this rank's element count of tensor t (its row range); the
    host buffers hold the shards back to back in tensor order: BF16 source
    (2 bytes per element), FP8 destination (1 byte per element) and the
    float32 scale_inv vector.
    """

    def __init__(self, sizes: Sequence[int], fp8_dtype: DType = DType.FLOAT8_E4M3, compat: int = 0,
                 comm: Communicator | None = None, src_dtype: DType = DType.BFLOAT16):
        from .backend import DeviceBuffer, Event, Stream
        self.sizes = [int(s) for s in sizes]
        self.n_tensors = len(self.sizes)
        self.total = sum(self.sizes)
        self.esize = 2 if src_dtype in (DType.BFLOAT16, DType.FLOAT16) else 4
        self.src_dtype, self.fp8_dtype, self.compat, self.comm = src_dtype, fp8_dtype, compat, comm
        self.up, self.compute, self.down = Stream(), Stream(), Stream()
        self.slots = []
        for _ in range(2):
            src = DeviceBuffer(max(1, self.esize * self.total))
            dst = DeviceBuffer(max(1, self.total))
            amax = DeviceBuffer(4 * self.n_tensors)
            sinv = DeviceBuffer(4 * self.n_tensors)
            entries, off = [], 0
            for t, n in enumerate(self.sizes):
                entries.append((src.ptr + self.esize * off, dst.ptr + off, n, t, src_dtype))
                off += n
            self.slots.append({"src": src, "dst": dst, "amax": amax, "sinv": sinv,
                               "chunks": make_chunks(entries), "uploaded": Event(), "computed": Event(),
                               "downloaded": Event(), "used": False})
        self.count = 0

    def submit(self, host_src: int, host_dst: int, host_scale_inv: int) -> None:
        """Queue one checkpoint: host_src -> device -> quantise -> host_dst, host_scale_inv."""
        s = self.slots[self.count % 2]
        if s["used"]:
            self.up.wait(s["downloaded"])  # the slot's previous results have left the device
        call("mf_memcpy_h2d_async", s["src"].ptr, int(host_src), self.esize * self.total, self.up.handle)
        s["uploaded"].record(self.up)
        self.compute.wait(s["uploaded"])
        quantise(s["chunks"], self.n_tensors, self.n_tensors, s["amax"].ptr, s["sinv"].ptr, self.fp8_dtype,
                 self.compat, self.comm, self.compute)
        s["computed"].record(self.compute)
        self.down.wait(s["computed"])
        call("mf_memcpy_d2h_async", int(host_dst), s["dst"].ptr, self.total, self.down.handle)
        call("mf_memcpy_d2h_async", int(host_scale_inv), s["sinv"].ptr, 4 * self.n_tensors, self.down.handle)
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
