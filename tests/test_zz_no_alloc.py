"""mf_ckpt_quant_fp8_noalloc: the quantiser that allocates nothing.

Some users of this library cannot hand it a device buffer for the per-tensor
amax scratch (their device memory is owned by another allocator, or
cudaMalloc is off limits after set-up); this entry point keeps that scratch in
a static device array instead.  The test checks, through the C ABI, that it
produces exactly what mf_ckpt_quant_fp8 produces with a caller-provided
buffer, on two calls in a row -- the second with smaller values, so a stale
amax left in the shared array by the first call would show up -- and that it
refuses a tensor count beyond its fixed capacity.  This file is collected
last so a failure here never hides the other tests.
"""
import numpy as np
import pytest

from manifesto_b200 import checkpoint, synthetic
from manifesto_b200._abi import lib
from manifesto_b200.dtype import DType

from .gpu_util import bits_equal, empty, fetch, to_device

pytestmark = pytest.mark.gpu

E4M3 = int(DType.FLOAT8_E4M3)


def _layout():
    return checkpoint.llama3_8b_layout(layers=1, hidden=256, mlp=768, heads=4, kv_heads=2, vocab=1000)


def _quantise_both(host, specs):
    """(fp8 codes, scale_inv) from the existing entry point and from the no-alloc one."""
    srcs = [to_device(h) for h in host]
    ref_dst = [empty(s.numel) for s in specs]
    new_dst = [empty(s.numel) for s in specs]
    n_t = len(specs)
    ref_entries = [(srcs[t].ptr, ref_dst[t].ptr, s.numel, t, DType.BFLOAT16) for t, s in enumerate(specs)]
    new_entries = [(srcs[t].ptr, new_dst[t].ptr, s.numel, t, DType.BFLOAT16) for t, s in enumerate(specs)]
    amax = empty(4 * n_t)
    ref_si = empty(4 * n_t)
    new_si = empty(4 * n_t)
    checkpoint.quantise(checkpoint.make_chunks(ref_entries), n_t, n_t, amax.ptr, ref_si.ptr)
    rc = lib().mf_ckpt_quant_fp8_noalloc(checkpoint.make_chunks(new_entries), n_t, n_t, new_si.ptr, E4M3, 0, None,
                                         None)
    assert rc == 0
    out = ([fetch(b, s.numel) for b, s in zip(ref_dst, specs)], fetch(ref_si, 4 * n_t, np.float32),
           [fetch(b, s.numel) for b, s in zip(new_dst, specs)], fetch(new_si, 4 * n_t, np.float32))
    for b in srcs + ref_dst + new_dst + [amax, ref_si, new_si]:
        b.free()
    return out


def test_noalloc_matches_caller_buffer_twice(backend):
    specs = _layout()
    # call 1: wide values; call 2: values 100x smaller (a stale amax would change every code)
    for call, sigma in ((1, 0.5), (2, 0.005)):
        host = [synthetic.normal_bf16(7000 + 31 * call + i, s.numel, 0.0, sigma) for i, s in enumerate(specs)]
        ref_q, ref_si, new_q, new_si = _quantise_both(host, specs)
        for t in range(len(specs)):
            bits_equal(new_q[t], ref_q[t])
        bits_equal(new_si.view(np.uint32), ref_si.view(np.uint32))


def test_noalloc_rejects_too_many_tensors(backend):
    from manifesto_b200._abi import last_error
    chunks = checkpoint.make_chunks([(1, 1, 16, 0, DType.BFLOAT16)])
    rc = lib().mf_ckpt_quant_fp8_noalloc(chunks, 1, 4097, None, E4M3, 0, None, None)
    assert rc == -9  # MF_ERR_ALLOCATOR_EXHAUSTED
    assert "4096" in last_error()
