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
