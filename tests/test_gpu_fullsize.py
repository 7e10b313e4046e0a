"""Full-size checks: the Llama-3-8B checkpoint quantisation at the benchmark's size, and empty inputs."""
import ctypes

import numpy as np
import pytest

from manifesto_b200 import checkpoint
from manifesto_b200._abi import call
from manifesto_b200.dtype import DType
from oracle.ref import BF16, E4M3, F32

from .conftest import host_threads
from .gpu_util import empty, fetch, to_device

pytestmark = pytest.mark.gpu


def test_llama3_8b_checkpoint_full_size(backend, ref):
    """All 291 tensors (8,030,261,248 BF16 params) in one mf_ckpt_quant_fp8 call, as the benchmark
    runs it: every scale_inv against the tensor's amax taken by torch on the device, and the codes
    of the largest tensor (lm_head, 525M params), a layer's MLP tensor and a norm bit-exact
    against the oracle."""
    torch = pytest.importorskip("torch")
    specs = checkpoint.llama3_8b_layout()
    sizes = [s.numel for s in specs]
    total = sum(sizes)
    assert total == 8_030_261_248 and len(specs) == 291
    gen = torch.Generator(device="cuda").manual_seed(1234)
    src = torch.empty(total, dtype=torch.bfloat16, device="cuda")
    step = 1 << 28
    for off in range(0, total, step):
        n = min(step, total - off)
        src[off:off + n] = torch.randn(n, device="cuda", generator=gen).mul_(0.02).to(torch.bfloat16)
    dst = torch.empty(total, dtype=torch.uint8, device="cuda")
    amax = torch.zeros(len(specs), dtype=torch.float32, device="cuda")
    sinv = torch.zeros(len(specs), dtype=torch.float32, device="cuda")
    entries, offs, off = [], [], 0
    for t, n in enumerate(sizes):
        entries.append((src.data_ptr() + 2 * off, dst.data_ptr() + off, n, t, DType.BFLOAT16))
        offs.append(off)
        off += n
    chunks = checkpoint.make_chunks(entries)
    checkpoint.quantise(chunks, len(entries), len(specs), amax.data_ptr(), sinv.data_ptr(), DType.FLOAT8_E4M3, 0,
                        None, None)
    torch.cuda.synchronize()
    want_amax = torch.stack([src[o:o + n].abs().max().float() for o, n in zip(offs, sizes)])
    assert torch.equal(amax, want_amax)
    sinv_h = sinv.cpu().numpy()
    for t in range(len(specs)):
        assert float(sinv_h[t]) == ref.fp8_scale_inv(float(want_amax[t]), E4M3), specs[t].name
    names = [s.name for s in specs]
    for name in ("lm_head.weight", "model.layers.17.mlp.down_proj.weight", "model.layers.31.input_layernorm.weight"):
        t = names.index(name)
        o, n = offs[t], sizes[t]
        raw = src[o:o + n].view(torch.uint16).cpu().numpy()
        got = dst[o:o + n].cpu().numpy()
        want = ref.scaled_cast(raw, BF16, E4M3, float(want_amax[t]), threads=host_threads())
        assert np.array_equal(got, want), name
    del src, dst
    torch.cuda.empty_cache()


def test_empty_inputs_are_no_ops(backend, ref):
    """n = 0 everywhere: nothing is launched that could fail, nothing is written."""
    canary = to_device(np.full(64, 0xA5, np.uint8))
    am = to_device(np.zeros(1, np.float32))
    si = to_device(np.zeros(1, np.float32))
    call("mf_convert", F32, BF16, canary.ptr, canary.ptr + 32, 0, 0, None)
    call("mf_axpy", canary.ptr, canary.ptr + 32, 0, 0.5, F32, 0, None)
    call("mf_scalar_broadcast", canary.ptr, F32, canary.ptr + 32, F32, 0, 2.0, 0, None)
    call("mf_int4_dequant_grouped", canary.ptr, canary.ptr + 16, BF16, canary.ptr + 32, BF16, 0, 128, 128, None)
    call("mf_amax", canary.ptr, BF16, 0, am.ptr, None)
    call("mf_fp8_scaled_cast", canary.ptr, BF16, canary.ptr + 32, E4M3, am.ptr, si.ptr, 0, 0, None)
    call("mf_fp8_quantize", canary.ptr, BF16, canary.ptr + 32, E4M3, am.ptr, si.ptr, 0, 0, None)
    zero = checkpoint.make_chunks([(canary.ptr, canary.ptr + 32, 0, 0, DType.BFLOAT16)])
    checkpoint.quantise(zero, 1, 1, am.ptr, si.ptr, DType.FLOAT8_E4M3, 0, None, None)
    code = ctypes.c_int(0)
    call("mf_device_status", ctypes.byref(code))
    assert (fetch(canary, 64) == 0xA5).all()
    assert float(fetch(am, 4, np.float32)[0]) == 0.0
    assert float(fetch(si, 4, np.float32)[0]) == 1.0  # an all-zero (empty) tensor keeps scale 1
    for b in (canary, am, si):
        b.free()
