"""mf_ckpt_quant_fp8_noalloc: the quantiser that allocates nothing.

Some users of this library cannot hand it a device buffer for the per-tensor
amax scratch (their device memory is owned by another allocator, or
cudaMalloc is off limits after set-up); this entry point keeps that scratch in
a static device array instead.  The test checks, through the C ABI, that it
produces exactly what mf_ckpt_quant_fp8 produces with a caller-provided
buffer, on two calls in a row -- the second with smaller values, so a stale
amax left in the shared array by the first call would show up -- that it
matches the CPU oracle bit for bit on mixed source dtypes, split and
unaligned chunks, more chunks than one launch takes, and exactly its
capacity of 4096 tensors, and that it refuses a tensor count beyond that.
This file is collected last so a failure here never hides the other tests.
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


def _noalloc(entries, n_tensors, si_ptr, fp8):
    rc = lib().mf_ckpt_quant_fp8_noalloc(checkpoint.make_chunks(entries), len(entries), n_tensors, si_ptr, fp8, 0,
                                         None, None)
    assert rc == 0


@pytest.mark.parametrize("fp8", [int(DType.FLOAT8_E4M3), int(DType.FLOAT8_E5M2)])
def test_noalloc_mixed_dtypes_and_many_chunks_match_oracle(backend, ref, fp8):
    """BF16, F16 and F32 tensors in one call, checked bit for bit against the CPU oracle: the
    entry point scans the chunk table once per source dtype, in batches of 512 chunks.  One
    tensor is cut into 700 chunks (so a dtype needs two batches), one is split at an offset
    that leaves its second chunk off 16-byte alignment, sizes are ragged, and one tensor has an
    empty chunk."""
    from oracle.ref import BF16, F16, F32, ITEMSIZE
    specs = [(BF16, 40000), (F16, 33333), (F32, 20001), (BF16, 700 * 48 + 5), (F32, 5 * 8192), (F16, 17)]
    wire = {BF16: DType.BFLOAT16, F16: DType.FLOAT16, F32: DType.FLOAT32}
    raws, srcs, dsts, entries = [], [], [], []
    for t, (dt, n) in enumerate(specs):
        v = synthetic.normal_f32(8800 + t, n, 0.0, 0.05 * (t + 1))
        raw = v.view(np.uint32).copy() if dt == F32 else ref.convert(v, F32, dt)
        src, dst = to_device(raw), empty(n)
        raws.append(raw), srcs.append(src), dsts.append(dst)
        if t == 3:
            cuts = list(range(0, 700 * 48, 48)) + [n]
        elif t == 0:
            cuts = [0, 12345, 12345, n]  # an empty chunk, then an unaligned one
        elif t == 2:
            cuts = [0, 7, n]
        else:
            cuts = [0, n]
        for a, b in zip(cuts, cuts[1:]):
            entries.append((src.ptr + a * ITEMSIZE[dt], dst.ptr + a, b - a, t, wire[dt]))
    assert len(entries) > 512
    si = empty(4 * len(specs))
    _noalloc(entries, len(specs), si.ptr, fp8)
    got_si = fetch(si, 4 * len(specs), np.float32)
    for t, ((dt, n), raw) in enumerate(zip(specs, raws)):
        a = ref.amax(raw, dt)
        assert float(got_si[t]) == ref.fp8_scale_inv(a, fp8), t
        bits_equal(fetch(dsts[t], n), ref.scaled_cast(raw, dt, fp8, a))
    for b in srcs + dsts + [si]:
        b.free()


def test_noalloc_exactly_at_capacity(backend, ref):
    """4096 tensors -- the static scratch's capacity -- is accepted and every tensor is exact."""
    from oracle.ref import BF16
    n_t, n = 4096, 40
    host = synthetic.normal_bf16(9100, n_t * n, 0.0, 1.0).reshape(n_t, n)
    host = (host.astype(np.uint32) ^ (np.arange(n_t, dtype=np.uint32)[:, None] & 0x3)).astype(np.uint16)
    src, dst, si = to_device(host), empty(n_t * n), empty(4 * n_t)
    entries = [(src.ptr + 2 * n * t, dst.ptr + n * t, n, t, DType.BFLOAT16) for t in range(n_t)]
    _noalloc(entries, n_t, si.ptr, E4M3)
    got = fetch(dst, n_t * n).reshape(n_t, n)
    got_si = fetch(si, 4 * n_t, np.float32)
    for t in range(n_t):
        a = ref.amax(host[t], BF16)
        assert float(got_si[t]) == ref.fp8_scale_inv(a, E4M3), t
        bits_equal(got[t], ref.scaled_cast(host[t], BF16, E4M3, a))
    for b in (src, dst, si):
        b.free()
