"""K7 fused chains, K8 amax-scaled FP8 cast and K9 checkpoint quantisation on the GPU."""
import ctypes

import numpy as np
import pytest

from manifesto_b200 import checkpoint, fusion, synthetic
from manifesto_b200._abi import call, lib
from manifesto_b200.dtype import DType
from manifesto_b200.fusion import NodeType as N
from oracle.ref import BF16, E4M3, E5M2, F16, F32, ITEMSIZE

from .conftest import host_threads
from .gpu_util import bits_equal, empty, fetch, to_device

pytestmark = pytest.mark.gpu


def ulp_diff_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in float32 ulps (ordered integer distance; NaN == NaN)."""
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    oa = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ob = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    d = np.abs(oa - ob)
    both_nan = np.isnan(a.view(np.float32)) & np.isnan(b.view(np.float32))
    return np.where(both_nan, 0, d)


def ulp_diff_16(a: np.ndarray, b: np.ndarray, nan_floor: int = 0x7F80) -> np.ndarray:
    """|a - b| in 16-bit ulps.  Two NaNs compare equal: the sign and payload of a NaN
    created by arithmetic (0/0, log(-1)) are platform-defined (x86 and the GPU differ),
    so tolerance checks compare NaN as a class; input NaNs are checked bit-exactly
    by the conversion tests.  nan_floor is 0x7F80 for BF16 and 0x7C00 for F16."""
    ia = a.astype(np.int64)
    ib = b.astype(np.int64)
    oa = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    ob = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    both_nan = ((ia & 0x7FFF) > nan_floor) & ((ib & 0x7FFF) > nan_floor)
    return np.where(both_nan, 0, np.abs(oa - ob))


def ulp_diff_fp8(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in FP8 codes between sign-magnitude codes (adjacent values differ by 1)."""
    ia = a.astype(np.int64)
    ib = b.astype(np.int64)
    oa = np.where(ia & 0x80, -(ia & 0x7F), ia)
    ob = np.where(ib & 0x80, -(ib & 0x7F), ib)
    return np.abs(oa - ob)


def run_fused(k: fusion.CUDAKernel, inputs, n, out_dt, amax=False):
    bufs = [to_device(a) for a in inputs]
    d = empty(n * ITEMSIZE[out_dt] + 64)
    am = empty(4, fill=0) if amax else None
    k.run([b.ptr for b in bufs], d.ptr, n, amax=am.ptr if am else None)
    out = fetch(d, n * ITEMSIZE[out_dt] + 64)
    assert (out[n * ITEMSIZE[out_dt]:] == 0xA5).all()
    amv = float(fetch(am, 4, np.float32)[0]) if amax else None
    for b in bufs + [d] + ([am] if am else []):
        b.free()
    return out[: n * ITEMSIZE[out_dt]].view({2: np.uint16, 4: np.uint32}[ITEMSIZE[out_dt]]), amv


def test_relu_add_known_answer(backend, golden):
    case = golden["known_answers"]["fused_relu_add"]
    root = fusion.unary(N.RELU, fusion.binary(N.ADD, fusion.input_node(0), fusion.input_node(1)))
    k = fusion.emit_cuda(fusion.FusionAST(root, ["x", "y"], "result"))
    assert k.identifier() == "result" and k.target() == fusion.Target.CUDA
    out, _ = run_fused(k, [np.array(case["x"], np.float32), np.array(case["y"], np.float32)], 4, F32)
    assert out.view(np.float32).tolist() == case["out"]
    with pytest.raises(Exception, match="expects 2 inputs"):
        k.run([1], 1, 2)


@pytest.mark.parametrize("op", [N.SIGMOID, N.TANH, N.GELU, N.SILU, N.EXP, N.LOG, N.SQRT])
def test_activations_within_2ulp(backend, ref, op):
    n = 1 << 16
    x = synthetic.normal_f32(int(op), n, 0.0, 4.0)
    if op in (N.LOG, N.SQRT):
        x = np.abs(x)
    x[:4] = [0.0, 1.0, -1.0, 2.0]
    root = fusion.unary(op, fusion.input_node(0))
    f = fusion.FusionAST(root, ["x"], "o")
    k = fusion.emit_cuda(f)
    got, _ = run_fused(k, [x], n, F32)
    want = ref.fused_eval(fusion.node_table(root), [x], [F32], [0], F32, n)
    assert ulp_diff_f32(got, want).max() <= 2


def random_tree(rng, depth, n_inputs):
    if depth == 0 or rng.random() < 0.25:
        if rng.random() < 0.8:
            return fusion.input_node(int(rng.integers(n_inputs)))
        return fusion.constant_node(float(rng.normal()))
    if rng.random() < 0.5:
        op = N(int(rng.integers(int(N.ADD), int(N.MIN) + 1)))
        return fusion.binary(op, random_tree(rng, depth - 1, n_inputs), random_tree(rng, depth - 1, n_inputs))
    op = N(int(rng.integers(int(N.NEG), int(N.LEAKY_RELU) + 1)))
    return fusion.unary(op, random_tree(rng, depth - 1, n_inputs))


@pytest.mark.parametrize("seed", range(12))
def test_random_chains_f32(backend, ref, seed):
    rng = np.random.default_rng(seed)
    n_in = 3
    root = random_tree(rng, 4, n_in)
    n = 20000
    ins = [synthetic.normal_f32(seed * 10 + j, n) for j in range(n_in)]
    bc = [0, 0, 0]
    if seed % 3 == 0:
        bc[2] = 100
    k = fusion.emit_cuda(fusion.FusionAST(root, ["a", "b", "c"], "o"), in_bcast=bc)
    got, _ = run_fused(k, ins, n, F32)
    want = ref.fused_eval(fusion.node_table(root), ins, [F32] * n_in, bc, F32, n)
    assert ulp_diff_f32(got, want).max() <= 2


@pytest.mark.parametrize("out_dt", [BF16, F16])
def test_random_chains_16bit_io(backend, ref, out_dt):
    rng = np.random.default_rng(77)
    root = random_tree(rng, 4, 2)
    n = 30000
    ins = [synthetic.normal_bf16(5, n), synthetic.normal_f32(6, n).astype(np.float16).view(np.uint16)]
    k = fusion.emit_cuda(fusion.FusionAST(root, ["a", "b"], "o"), in_dtypes=[DType.BFLOAT16, DType.FLOAT16],
                         out_dtype=DType(out_dt))
    got, _ = run_fused(k, ins, n, out_dt)
    want = ref.fused_eval(fusion.node_table(root), ins, [BF16, F16], [0, 0], out_dt, n)
    assert ulp_diff_16(got, want, 0x7F80 if out_dt == BF16 else 0x7C00).max() <= 1


@pytest.mark.parametrize("seed", range(8))
def test_generated_kernel_matches_interpreter(backend, ref, seed, monkeypatch):
    """The CUDA codegen target (source emitted per expression, compiled with NVRTC) against the
    runtime interpreter, bit for bit -- they share the node rules -- on random programs with
    mixed input dtypes, broadcast lengths that are and are not multiples of 8, buffers at
    16-byte and odd offsets, and element counts that are not multiples of 8; and both within
    tolerance of the oracle."""
    rng = np.random.default_rng(100 + seed)
    root = random_tree(rng, 4, 3)
    n = 40003 if seed % 2 else 65536
    dts = [[BF16, F16, F32][int(rng.integers(3))] for _ in range(3)]
    bc = [0, [0, 64, 100][seed % 3], [0, 4096, 24][(seed // 3) % 3]]
    out_dt = [BF16, F16, F32][seed % 3]
    wire = {BF16: DType.BFLOAT16, F16: DType.FLOAT16, F32: DType.FLOAT32}
    ins = []
    for j, dt in enumerate(dts):
        m = bc[j] or n
        v = synthetic.normal_f32(300 + 10 * seed + j, m, 0.0, 2.0)
        ins.append(v.view(np.uint32).copy() if dt == F32 else ref.convert(v, F32, dt))
    f = fusion.FusionAST(root, ["a", "b", "c"], "o")
    kw = dict(in_dtypes=[wire[d] for d in dts], in_bcast=bc, out_dtype=wire[out_dt])
    gen = fusion.emit_cuda(f, **kw)
    assert gen.generated(), "NVRTC codegen unavailable"
    monkeypatch.setenv("MF_FUSED_JIT", "0")
    interp = fusion.emit_cuda(f, **kw)
    assert interp.kind() == 0
    osz = ITEMSIZE[out_dt]
    for shift in (0, 1):
        # shift 1 moves every buffer one element (of its own dtype) off 16-byte alignment
        offs = [shift * ITEMSIZE[dt] for dt in dts]
        off = shift * osz
        bufs = [to_device(np.concatenate([np.zeros(o, np.uint8), a.view(np.uint8)])) for o, a in zip(offs, ins)]
        outs = []
        for k in (gen, interp):
            d = empty(off + n * osz + 64)
            am = empty(4, fill=0)
            k.run([b.ptr + o for b, o in zip(bufs, offs)], d.ptr + off, n, amax=am.ptr)
            o = fetch(d, off + n * osz + 64)
            assert (o[off + n * osz:] == 0xA5).all() and (o[:off] == 0xA5).all()
            outs.append((o[off:off + n * osz], fetch(am, 4, np.uint32)[0]))
            d.free(), am.free()
        if out_dt == F32:
            # float32 outputs: both run evalCPU's rules, bit for bit
            bits_equal(outs[0][0], outs[1][0])
            assert outs[0][1] == outs[1][1]
        else:
            # 16-bit outputs: the generated code may take the float32 forms (within 1 ulp)
            g16, i16 = (o[0].view(np.uint16) for o in outs)
            assert ulp_diff_16(g16, i16, 0x7F80 if out_dt == BF16 else 0x7C00).max() <= 1
        for o, am in outs:  # each kernel's amax is max|stored value| of its own output, NaN ignored
            v = o.view({2: np.uint16, 4: np.uint32}[osz])
            vals = ((v.astype(np.uint32) << 16).view(np.float32) if out_dt == BF16 else
                    v.view(np.float16).astype(np.float32) if out_dt == F16 else v.view(np.float32))
            mags = np.abs(vals[~np.isnan(vals)])
            assert am == np.float32(mags.max() if mags.size else 0.0).view(np.uint32)
        for b in bufs:
            b.free()
    got = outs[0][0].view({2: np.uint16, 4: np.uint32}[osz])
    want = ref.fused_eval(fusion.node_table(root), ins, dts, bc, out_dt, n)
    if out_dt == F32:
        assert ulp_diff_f32(got, want).max() <= 2
    else:
        assert ulp_diff_16(got, want, 0x7F80 if out_dt == BF16 else 0x7C00).max() <= 1
    gen.close(), interp.close()


# (tree seed or None for Gelu(Add(Mul(x, g), b)), input dtypes, broadcast lengths, output dtype, tiles per SM)
PIPELINE_CASES = [
    (None, [BF16, BF16, BF16], [0, 4096, 4096], BF16, 2),
    (17, [BF16, F32, F16], [0, 0, 64], F16, 1),
    (24, [BF16, BF16, F16], [0, 0, 4096], BF16, 1),
    (8, [F32, BF16, BF16], [0, 4096, 0], F32, 1),
    (9, [F32, BF16, F16], [0, 8, 4096], BF16, 1),
]


@pytest.mark.parametrize("case", range(len(PIPELINE_CASES)))
def test_generated_pipeline_matches_interpreter(backend, ref, case, monkeypatch):
    """The generated kernel's bulk-copy pipeline (mf_jit_tma: taken for 16-byte aligned buffers with at
    least one whole tile per SM; the tile is the largest power of two whose stage of full-size inputs
    fits 32 KB) against the interpreter: one or two full-size inputs of mixed dtypes, row-broadcast
    inputs of several lengths, several tiles per CTA, a ragged tail finished element by element, and
    the amax of the output."""
    seed, dts, bc, out_dt, per_sm = PIPELINE_CASES[case]
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = sms * 16384 * per_sm + 12345  # at least one whole tile per SM whatever the tile (2048 .. 16384)
    wire = {BF16: DType.BFLOAT16, F16: DType.FLOAT16, F32: DType.FLOAT32}
    if seed is None:
        f = fusion.gelu_affine_chain()
    else:
        f = fusion.FusionAST(random_tree(np.random.default_rng(seed), 4, 3), ["a", "b", "c"], "o")
    ins = []
    for j, dt in enumerate(dts):
        m = bc[j] or n
        v = synthetic.normal_f32(700 + 10 * case + j, m, 0.0, 2.0)
        ins.append(v.view(np.uint32).copy() if dt == F32 else ref.convert(v, F32, dt))
    kw = dict(in_dtypes=[wire[d] for d in dts], in_bcast=bc, out_dtype=wire[out_dt])
    gen = fusion.emit_cuda(f, **kw)
    assert gen.generated(), "NVRTC codegen unavailable"
    monkeypatch.setenv("MF_FUSED_JIT", "0")
    interp = fusion.emit_cuda(f, **kw)
    assert interp.kind() == 0
    osz = ITEMSIZE[out_dt]
    bufs = [to_device(a) for a in ins]
    outs = []
    for k in (gen, interp):
        d = empty(n * osz + 64)
        am = empty(4, fill=0)
        k.run([b.ptr for b in bufs], d.ptr, n, amax=am.ptr)
        o = fetch(d, n * osz + 64)
        assert (o[n * osz:] == 0xA5).all()
        outs.append((o[:n * osz], fetch(am, 4, np.uint32)[0]))
        d.free(), am.free()
    if out_dt == F32:
        bits_equal(outs[0][0], outs[1][0])
        assert outs[0][1] == outs[1][1]
    else:
        g16, i16 = (o[0].view(np.uint16) for o in outs)
        assert ulp_diff_16(g16, i16, 0x7F80 if out_dt == BF16 else 0x7C00).max() <= 1
    for o, am in outs:
        v = o.view({2: np.uint16, 4: np.uint32}[osz])
        vals = ((v.astype(np.uint32) << 16).view(np.float32) if out_dt == BF16 else
                v.view(np.float16).astype(np.float32) if out_dt == F16 else v.view(np.float32))
        mags = np.abs(vals[~np.isnan(vals)])
        assert am == np.float32(mags.max() if mags.size else 0.0).view(np.uint32)
    for b in bufs:
        b.free()
    gen.close(), interp.close()


@pytest.mark.parametrize("out_dt", [BF16, F16])
@pytest.mark.parametrize("op", [N.SIGMOID, N.TANH, N.GELU, N.SILU, N.EXP, N.LOG, N.SQRT])
def test_activations_16bit_output_within_1ulp(backend, ref, op, out_dt):
    """Each transcendental with a 16-bit output, where the generated code may use its float32 form:
    inputs swept across every guard boundary of that form (-80, 88, GELU's u = -9, tiny and huge
    magnitudes) plus +-0, +-Inf and NaN, all within 1 ulp of evalCPU's float64 rule; and the same
    node under a Sub (no float32 form allowed there) as well."""
    sweep = np.concatenate([np.linspace(-120, 120, 48001, dtype=np.float32),
                            np.linspace(-6, -3.5, 4001, dtype=np.float32),
                            np.float32(10.0) ** np.linspace(-38, 38, 2001, dtype=np.float32),
                            -np.float32(10.0) ** np.linspace(-38, 38, 2001, dtype=np.float32),
                            np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 88.0, 88.72, -80.0, -80.01], np.float32),
                            synthetic.normal_f32(int(op) + 7, 20000, 0.0, 4.0)])
    n = sweep.size
    for root, label in ((fusion.unary(op, fusion.input_node(0)), "plain"),
                        (fusion.binary(N.SUB, fusion.unary(op, fusion.input_node(0)), fusion.input_node(0)), "sub")):
        k = fusion.emit_cuda(fusion.FusionAST(root, ["x"], "o"), out_dtype=DType(out_dt))
        assert k.generated()
        got, _ = run_fused(k, [sweep], n, out_dt)
        want = ref.fused_eval(fusion.node_table(root), [sweep], [F32], [0], out_dt, n)
        d = ulp_diff_16(got, want, 0x7F80 if out_dt == BF16 else 0x7C00)
        assert d.max() <= 1, (label, sweep[np.argmax(d)], got[np.argmax(d)], want[np.argmax(d)])
        k.close()


def swiglu_inputs(n, hidden=4096, seed=synthetic.CONFIG_SEED + 40):
    x = synthetic.normal_bf16(seed, n)
    y = synthetic.normal_bf16(seed + 1, n)
    g = synthetic.normal_bf16(seed + 2, hidden, 1.0, 0.1)
    b = synthetic.normal_bf16(seed + 3, hidden, 0.0, 0.1)
    return [x, g, b, y]


def swiglu_kernel(hidden=4096):
    f = fusion.swiglu_chain()
    return f, fusion.emit_cuda(f, in_dtypes=[DType.BFLOAT16] * 4, in_bcast=[0, hidden, hidden, 0],
                               out_dtype=DType.BFLOAT16)


def test_swiglu_specialised_within_1ulp(backend, ref):
    n = 64 * 4096 * 4
    f, k = swiglu_kernel()
    assert k.specialised()
    ins = swiglu_inputs(n)
    got, amax = run_fused(k, ins, n, BF16, amax=True)
    want = ref.fused_eval(fusion.node_table(f.root), ins, [BF16] * 4, [0, 4096, 4096, 0], BF16, n,
                          threads=host_threads())
    d = ulp_diff_16(got, want)
    assert d.max() <= 1
    # amax folds |BF16 output| exactly
    assert amax == float(np.abs((got.astype(np.uint32) << 16).view(np.float32)).max())


def test_swiglu_row_length_without_stationary_grid(backend, ref):
    """A row of 8191 vectors (prime) admits no grid holding a multiple of the row in threads:
    the kernel that advances the row index per step runs, with the same results."""
    hidden = 8 * 8191
    n = hidden * 5
    f, k = swiglu_kernel(hidden)
    assert k.specialised()
    ins = swiglu_inputs(n, hidden=hidden, seed=77)
    got, amax = run_fused(k, ins, n, BF16, amax=True)
    want = ref.fused_eval(fusion.node_table(f.root), ins, [BF16] * 4, [0, hidden, hidden, 0], BF16, n,
                          threads=host_threads())
    assert ulp_diff_16(got, want).max() <= 1
    assert amax == float(np.abs((got.astype(np.uint32) << 16).view(np.float32)).max())


def test_swiglu_specialised_extreme_inputs(backend, ref):
    """t = x*g + b swept through the range where e^-t leaves float32 (t < -88.7) and
    1/(1 + e^-t) turns subnormal, plus Inf, NaN, zeros and subnormal inputs: the fast
    SiLU's float64 hand-over keeps every output within 1 BF16 ulp of the reference."""
    hidden = 4096
    n = hidden * 64
    rng = np.random.default_rng(2024)
    xf = rng.uniform(-140.0, 140.0, n).astype(np.float32)
    xf[: 4096] = np.linspace(-130.0, -70.0, 4096, dtype=np.float32)
    specials = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38], np.float32)
    xf[5000:5000 + specials.size] = specials
    yf = rng.standard_normal(n).astype(np.float32)
    yf[6000:6000 + specials.size] = specials
    yf[: 4096 : 7] = 3e38  # huge y on tiny silu outputs
    x, y = synthetic.f32_to_bf16_bits(xf), synthetic.f32_to_bf16_bits(yf)
    g = synthetic.normal_bf16(11, hidden, 1.0, 0.1)
    b = synthetic.normal_bf16(12, hidden, 0.0, 0.1)
    g[7] = 0x7F80  # +Inf
    b[9] = 0x7FC0  # NaN
    f, k = swiglu_kernel(hidden)
    assert k.specialised()
    got, amax = run_fused(k, [x, g, b, y], n, BF16, amax=True)
    want = ref.fused_eval(fusion.node_table(f.root), [x, g, b, y], [BF16] * 4, [0, hidden, hidden, 0], BF16, n,
                          threads=host_threads())
    d = ulp_diff_16(got, want)
    assert d.max() <= 1, np.nonzero(d > 1)[0][:8]
    mags = (got.astype(np.uint32) << 16).view(np.float32)
    assert amax == float(np.nanmax(np.abs(mags)))


def test_swiglu_commuted_forms_specialise(backend):
    x, g, b, y = (fusion.input_node(i, DType.BFLOAT16) for i in range(4))
    root = fusion.binary(N.MUL, y, fusion.unary(N.SILU, fusion.binary(N.ADD, b, fusion.binary(N.MUL, g, x))))
    k = fusion.emit_cuda(fusion.FusionAST(root, ["x", "g", "b", "y"], "o", dtype=DType.BFLOAT16),
                         in_bcast=[0, 4096, 4096, 0])
    assert k.specialised()
    k2 = fusion.emit_cuda(fusion.FusionAST(root, ["x", "g", "b", "y"], "o", dtype=DType.BFLOAT16))
    assert not k2.specialised()  # no broadcast inputs -> interpreter


def test_fused_fp8_pipeline(backend, ref):
    """Config 4 at reduced size: chain -> BF16 -> amax -> E4M3, within 1 FP8 code."""
    n = 8 * 2048 * 4096 // 8
    f, k = swiglu_kernel()
    ins = swiglu_inputs(n)
    bufs = [to_device(a) for a in ins]
    pre = empty(n * 2)
    q = empty(n)
    am = empty(4)
    si = empty(4)
    k.run_fp8([b.ptr for b in bufs], pre.ptr, q.ptr, n, am.ptr, si.ptr)
    got_pre = fetch(pre, n * 2, np.uint16)
    got_q = fetch(q, n)
    got_amax = float(fetch(am, 4, np.float32)[0])
    got_si = float(fetch(si, 4, np.float32)[0])
    want_pre = ref.fused_eval(fusion.node_table(f.root), ins, [BF16] * 4, [0, 4096, 4096, 0], BF16, n,
                              threads=host_threads())
    assert ulp_diff_16(got_pre, want_pre).max() <= 1
    want_amax = ref.amax(want_pre, BF16)
    want_q = ref.scaled_cast(want_pre, BF16, E4M3, want_amax, threads=host_threads())
    assert ulp_diff_fp8(got_q, want_q).max() <= 1
    # the GPU's own precast -> its FP8 output is bit-exact under the oracle's cast
    bits_equal(got_q, ref.scaled_cast(got_pre, BF16, E4M3, got_amax, threads=host_threads()))
    assert got_amax == ref.amax(got_pre, BF16)
    assert got_si == ref.fp8_scale_inv(got_amax, E4M3)
    for b in bufs + [pre, q, am, si]:
        b.free()


def test_fused_fp8_pipeline_config4_full_size(backend, ref):
    """Config 4 at its stated size, BF16 [64, 2048, 4096] = 2^29 elements, through the same call the
    benchmark times (CUDAKernel.run_fp8): every pre-cast value within 1 BF16 ulp of evalCPU's
    restatement, every FP8 code within 1 code of the oracle's pipeline, the FP8 codes bit-exact under
    the oracle's cast of the GPU's own pre-cast values, and amax / scale_inv exact.  x, y ~ N(0, 1),
    gamma ~ N(1, 0.1), beta ~ N(0, 0.1), drawn on the device and checked on the host."""
    torch = pytest.importorskip("torch")
    hidden, n = 4096, 64 * 2048 * 4096
    gen = torch.Generator(device="cuda").manual_seed(4040)
    x = torch.empty(n, dtype=torch.bfloat16, device="cuda").normal_(0.0, 1.0, generator=gen)
    y = torch.empty(n, dtype=torch.bfloat16, device="cuda").normal_(0.0, 1.0, generator=gen)
    g = torch.empty(hidden, dtype=torch.bfloat16, device="cuda").normal_(1.0, 0.1, generator=gen)
    b = torch.empty(hidden, dtype=torch.bfloat16, device="cuda").normal_(0.0, 0.1, generator=gen)
    pre = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(n, dtype=torch.uint8, device="cuda")
    am = torch.zeros(1, dtype=torch.float32, device="cuda")
    si = torch.zeros(1, dtype=torch.float32, device="cuda")
    f, k = swiglu_kernel(hidden)
    assert k.specialised()
    k.run_fp8([x.data_ptr(), g.data_ptr(), b.data_ptr(), y.data_ptr()], pre.data_ptr(), q.data_ptr(), n,
              am.data_ptr(), si.data_ptr())
    torch.cuda.synchronize()
    host = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)
    ins = [host(x), host(g), host(b), host(y)]
    got_pre, got_q = host(pre), q.cpu().numpy()
    got_amax, got_si = float(am.item()), float(si.item())
    del x, y, pre, q
    torch.cuda.empty_cache()
    th = host_threads()
    want_pre = ref.fused_eval(fusion.node_table(f.root), ins, [BF16] * 4, [0, hidden, hidden, 0], BF16, n, threads=th)
    step = 1 << 26  # compare in slices: the int64 distance arrays of 2^29 elements would take ~25 GB
    assert max(int(ulp_diff_16(got_pre[i:i + step], want_pre[i:i + step]).max()) for i in range(0, n, step)) <= 1
    want_amax = ref.amax(want_pre, BF16, threads=th)
    want_q = ref.scaled_cast(want_pre, BF16, E4M3, want_amax, threads=th)
    assert max(int(ulp_diff_fp8(got_q[i:i + step], want_q[i:i + step]).max()) for i in range(0, n, step)) <= 1
    del want_pre, want_q
    assert got_amax == ref.amax(got_pre, BF16, threads=th)
    assert got_si == ref.fp8_scale_inv(got_amax, E4M3)
    bits_equal(got_q, ref.scaled_cast(got_pre, BF16, E4M3, got_amax, threads=th))
    k.close()


# --------------------------------------------------------------- quant

@pytest.mark.parametrize("dt", [F32, BF16, F16, E4M3, E5M2])
def test_amax(backend, ref, dt):
    n = 100003
    raw = synthetic.uniform_bytes(dt, n * ITEMSIZE[dt])
    d = to_device(raw)
    am = empty(4, fill=0)
    call("mf_amax", d.ptr, dt, n, am.ptr, None)
    got = float(fetch(am, 4, np.float32)[0])
    assert got == ref.amax(raw, dt)
    d.free()
    am.free()


@pytest.mark.parametrize("src", [F32, BF16, F16])
@pytest.mark.parametrize("fp8", [E4M3, E5M2])
@pytest.mark.parametrize("compat", [0, 1])
def test_fp8_quantize_bit_exact(backend, ref, src, fp8, compat):
    n = (1 << 20) + 7
    if src == F32:
        raw = synthetic.normal_f32(src, n, 0, 2.0)
    elif src == BF16:
        raw = synthetic.normal_bf16(src, n, 0, 2.0)
    else:
        raw = synthetic.normal_f32(src, n, 0, 2.0).astype(np.float16).view(np.uint16)
    raw[5] = {F32: 0x7FC00000, BF16: 0x7FC0, F16: 0x7E00}[src]  # a NaN is ignored by amax
    d = to_device(raw)
    q = empty(n)
    am = empty(4)
    si = empty(4)
    call("mf_fp8_quantize", d.ptr, src, q.ptr, fp8, am.ptr, si.ptr, n, compat, None)
    got_amax = float(fetch(am, 4, np.float32)[0])
    assert got_amax == ref.amax(raw, src)
    bits_equal(fetch(q, n), ref.scaled_cast(raw, src, fp8, got_amax, compat))
    assert float(fetch(si, 4, np.float32)[0]) == ref.fp8_scale_inv(got_amax, fp8)
    for b in (d, q, am, si):
        b.free()


@pytest.mark.parametrize("fp8", [E4M3, E5M2])
@pytest.mark.parametrize("src", [F32, BF16])
def test_scaled_cast_fixup_heavy(backend, ref, src, fp8):
    """Scaled casts where most quads need the exact encoder (subnormal bands, the
    E4M3 2^-10 tie, NaN, E5M2 overflow): whole tiles where every warp parks more
    quads than its queue holds, next to tiles with none, plus a ragged end."""
    rng = np.random.default_rng(int(src) * 16 + int(fp8))
    n = 40 * 8192 + 13
    lo, hi = (2.0 ** -11, 2.0 ** -5) if fp8 == E4M3 else (2.0 ** -18, 2.0 ** -13)
    mag = np.exp2(rng.uniform(np.log2(lo), np.log2(hi), n)).astype(np.float32)
    v = np.where(rng.random(n) < 0.5, -mag, mag).astype(np.float32)
    v[8192 * 3: 8192 * 5] = rng.standard_normal(8192 * 2).astype(np.float32) * 100.0  # tiles with few fix-ups
    v[::97] = 2.0 ** -10
    v[::101] = -(2.0 ** -10)
    v[::389] = np.nan
    v[::211] = 0.0
    v[::503] = 60000.0  # past both formats' maxima: E4M3 saturates, E5M2 gives the reference's Inf
    raw = v if src == F32 else synthetic.f32_to_bf16_bits(v)
    amax = 448.0 if fp8 == E4M3 else 57344.0  # scale exactly 1: the values above land unscaled
    d = to_device(raw)
    q = empty(n)
    am = to_device(np.array([amax], np.float32))
    for compat in (0, 1):
        call("mf_fp8_scaled_cast", d.ptr, src, q.ptr, fp8, am.ptr, None, n, compat, None)
        bits_equal(fetch(q, n), ref.scaled_cast(raw, src, fp8, amax, compat, threads=host_threads()))
    for b in (d, q, am):
        b.free()


def test_quantize_zero_and_tiny(backend, ref):
    n = 4096
    raw = np.zeros(n, np.uint16)
    raw[7] = 0x0001  # BF16 subnormal
    d = to_device(raw)
    q = empty(n)
    am = empty(4)
    call("mf_fp8_quantize", d.ptr, BF16, q.ptr, E4M3, am.ptr, None, n, 0, None)
    got_amax = float(fetch(am, 4, np.float32)[0])
    bits_equal(fetch(q, n), ref.scaled_cast(raw, BF16, E4M3, got_amax))
    raw[:] = 0
    d.upload(raw)
    call("mf_fp8_quantize", d.ptr, BF16, q.ptr, E4M3, am.ptr, None, n, 0, None)
    assert float(fetch(am, 4, np.float32)[0]) == 0.0
    assert (fetch(q, n) == 0).all()
    for b in (d, q, am):
        b.free()


# -------------------------------------------------------- checkpoint

def small_layout():
    return checkpoint.llama3_8b_layout(layers=2, hidden=512, mlp=1792, heads=8, kv_heads=2, vocab=4000)


@pytest.mark.parametrize("world", [1, 3, 8])
def test_ckpt_sharded_emulated_bit_exact(backend, ref, world):
    """All ranks' chunks in one grouped launch (the ranks emulated on one GPU)."""
    specs = small_layout()
    host = [synthetic.normal_bf16(1000 + i, s.numel, 0.0, 0.02) for i, s in enumerate(specs)]
    srcs = [to_device(h) for h in host]
    dsts = [empty(s.numel) for s in specs]
    entries = []
    for r in range(world):
        for t, ((first, rows), s) in enumerate(zip(checkpoint.partition(specs, world, r), specs)):
            off = first * s.cols
            entries.append((srcs[t].ptr + 2 * off, dsts[t].ptr + off, rows * s.cols, t, DType.BFLOAT16))
    chunks = checkpoint.make_chunks(entries)
    am = empty(4 * len(specs))
    si = empty(4 * len(specs))
    checkpoint.quantise(chunks, len(entries), len(specs), am.ptr, si.ptr)
    amax = fetch(am, 4 * len(specs), np.float32)
    sinv = fetch(si, 4 * len(specs), np.float32)
    for t, h in enumerate(host):
        want_amax = ref.amax(h, BF16)
        assert amax[t] == want_amax, specs[t].name
        assert sinv[t] == ref.fp8_scale_inv(want_amax, E4M3)
        bits_equal(fetch(dsts[t], specs[t].numel), ref.scaled_cast(h, BF16, E4M3, want_amax))
    for b in srcs + dsts + [am, si]:
        b.free()


def test_ckpt_many_chunks_and_ragged(backend, ref):
    """More chunks than one launch holds, ragged sizes and unaligned chunk starts."""
    rng = np.random.default_rng(5)
    sizes = [int(v) for v in rng.integers(1, 40000, size=700)]
    host = [synthetic.normal_bf16(i, s, 0, 1.0) for i, s in enumerate(sizes)]
    srcs = [to_device(h, pad=32) for h in host]
    dsts = [empty(s + 32) for s in sizes]
    entries = []
    for t, s in enumerate(sizes):
        off = t % 3  # unaligned starts for some chunks
        entries.append((srcs[t].ptr + 2 * off, dsts[t].ptr + off, s - off, t, DType.BFLOAT16))
    am = empty(4 * len(sizes))
    checkpoint.quantise(checkpoint.make_chunks(entries), len(entries), len(sizes), am.ptr, None)
    amax = fetch(am, 4 * len(sizes), np.float32)
    for t, s in enumerate(sizes):
        off = t % 3
        h = host[t][off:]
        assert amax[t] == ref.amax(h, BF16)
        bits_equal(fetch(dsts[t], s - off, offset=off), ref.scaled_cast(h, BF16, E4M3, float(amax[t])))
    for b in srcs + dsts + [am]:
        b.free()


@pytest.mark.parametrize("batch_bytes", [1 << 30, 300_000])
def test_streamed_quantiser_host_checkpoints(backend, ref, batch_bytes):
    """Three host-resident checkpoints through the upload/compute/download pipeline (two slots):
    one batch per checkpoint, or many batches of whole tensors (a tensor larger than the batch
    gets one of its own)."""
    from manifesto_b200 import PinnedBuffer
    specs = small_layout()
    sizes = [s.numel for s in specs]
    total = sum(sizes)
    q = checkpoint.StreamedQuantiser(sizes, batch_bytes=batch_bytes)
    assert (len(q.batches) == 1) == (batch_bytes == 1 << 30)
    assert [t for a, b in q.batches for t in range(a, b)] == list(range(len(sizes)))
    ins, outs, sis, hosts = [], [], [], []
    for k in range(3):
        host = [synthetic.normal_bf16(4000 + 100 * k + i, n, 0.0, 0.02 * (k + 1)) for i, n in enumerate(sizes)]
        hs = PinnedBuffer(2 * total)
        hs.array[:] = np.concatenate(host).view(np.uint8)
        hd, hsi = PinnedBuffer(total), PinnedBuffer(4 * len(sizes))
        q.submit(hs.ptr, hd.ptr, hsi.ptr)
        ins.append(hs), outs.append(hd), sis.append(hsi), hosts.append(host)
    q.synchronize()
    for k in range(3):
        off = 0
        for t, n in enumerate(sizes):
            a = ref.amax(hosts[k][t], BF16)
            assert float(sis[k].array.view(np.float32)[t]) == ref.fp8_scale_inv(a, E4M3)
            bits_equal(outs[k].array[off:off + n], ref.scaled_cast(hosts[k][t], BF16, E4M3, a))
            off += n
    q.close()
    for b in ins + outs + sis:
        b.free()


def test_ckpt_rejects(backend):
    arr = checkpoint.make_chunks([(1, 1, 10, 5, DType.BFLOAT16)])
    assert lib().mf_ckpt_quant_fp8(arr, 1, 2, 1, None, E4M3, 0, None, None) == -1  # tensor 5 of 2
    arr = checkpoint.make_chunks([(1, 1, 10, 0, DType.FLOAT8_E4M3)])
    assert lib().mf_ckpt_quant_fp8(arr, 1, 1, 1, None, E4M3, 0, None, None) == -3


def test_ckpt_scale_inv_covers_tensors_without_local_elements(backend, ref):
    """A rank that holds no row of a tensor still reports that tensor's scale_inv (from the
    all-reduced amax): here tensor 1 has an empty chunk and tensor 3 no chunk at all."""
    sizes = {0: 5000, 1: 0, 2: 2048}
    raws = {t: synthetic.normal_bf16(600 + t, max(n, 1), 0.0, 0.5)[:n] for t, n in sizes.items()}
    amax_all = np.array([ref.amax(raws[0], BF16), 3.5, ref.amax(raws[2], BF16), 0.0], np.float32)
    srcs = {t: to_device(raws[t], pad=16) for t in sizes}
    dsts = {t: empty(max(n, 1) + 16) for t, n in sizes.items()}
    am = to_device(amax_all)
    si = empty(16)
    chunks = checkpoint.make_chunks([(srcs[t].ptr, dsts[t].ptr, n, t, DType.BFLOAT16) for t, n in sizes.items()])
    call("mf_ckpt_cast_pass", chunks, len(sizes), 4, am.ptr, si.ptr, E4M3, 0, None)
    got = fetch(si, 16, np.float32)
    for t in range(4):
        assert float(got[t]) == ref.fp8_scale_inv(float(amax_all[t]), E4M3), t
    for t, n in sizes.items():
        if n:
            bits_equal(fetch(dsts[t], n), ref.scaled_cast(raws[t], BF16, E4M3, float(amax_all[t])))
    for b in list(srcs.values()) + list(dsts.values()) + [am, si]:
        b.free()


@pytest.mark.parametrize("fp8", [E4M3, E5M2])
def test_ckpt_mixed_source_dtypes(backend, ref, fp8):
    """One checkpoint call over BF16, F16 and F32 tensors: the library launches each source
    dtype's chunks separately (F32 tiles hold 8192 elements, 16-bit ones 16384), sizes are
    ragged, and two tensors are split into two chunks at an element offset that leaves the
    second chunk off 16-byte alignment.  Codes and scale_inv are bit-exact against the oracle."""
    specs = [(BF16, 40000), (F16, 33333), (F32, 20001), (BF16, 3 * 16384 + 5), (F32, 5 * 8192), (F16, 17)]
    splits = {0: 12345, 2: 7}
    wire = {BF16: DType.BFLOAT16, F16: DType.FLOAT16, F32: DType.FLOAT32}
    raws, srcs, dsts, entries = [], [], [], []
    for t, (dt, n) in enumerate(specs):
        v = synthetic.normal_f32(800 + t, n, 0.0, 0.05 * (t + 1))
        raw = v.view(np.uint32).copy() if dt == F32 else ref.convert(v, F32, dt)
        src, dst = to_device(raw), empty(n)
        raws.append(raw), srcs.append(src), dsts.append(dst)
        cuts = [0, splits[t], n] if t in splits else [0, n]
        for a, b in zip(cuts, cuts[1:]):
            entries.append((src.ptr + a * ITEMSIZE[dt], dst.ptr + a, b - a, t, wire[dt]))
    am, si = empty(4 * len(specs)), empty(4 * len(specs))
    checkpoint.quantise(checkpoint.make_chunks(entries), len(entries), len(specs), am.ptr, si.ptr, DType(fp8))
    got_si = fetch(si, 4 * len(specs), np.float32)
    for t, ((dt, n), raw) in enumerate(zip(specs, raws)):
        a = ref.amax(raw, dt)
        assert float(got_si[t]) == ref.fp8_scale_inv(a, fp8), t
        bits_equal(fetch(dsts[t], n), ref.scaled_cast(raw, dt, fp8, a))
    for b in srcs + dsts + [am, si]:
        b.free()


def test_ckpt_quantise_from_several_host_threads(backend, ref):
    """cgo may call from any OS thread: four threads quantise four checkpoints at once, each on
    its own stream, through the grouped launches that share the library's argument blocks."""
    import threading

    from manifesto_b200 import Stream
    specs = small_layout()
    sizes = [s.numel for s in specs]
    jobs = []
    for j in range(4):
        raws = [synthetic.normal_bf16(7000 + 50 * j + t, n, 0.0, 0.01 * (j + 1)) for t, n in enumerate(sizes)]
        srcs = [to_device(r) for r in raws]
        dsts = [empty(n) for n in sizes]
        jobs.append({"raws": raws, "srcs": srcs, "dsts": dsts, "am": empty(4 * len(sizes)),
                     "si": empty(4 * len(sizes)), "stream": Stream(), "err": None})

    def work(job):
        try:
            chunks = checkpoint.make_chunks([(s.ptr, d.ptr, n, t, DType.BFLOAT16)
                                             for t, (s, d, n) in enumerate(zip(job["srcs"], job["dsts"], sizes))])
            for _ in range(5):
                checkpoint.quantise(chunks, len(sizes), len(sizes), job["am"].ptr, job["si"].ptr, DType.FLOAT8_E4M3,
                                    0, None, job["stream"])
            job["stream"].sync()
        except Exception as e:  # reported below
            job["err"] = e

    threads = [threading.Thread(target=work, args=(job,)) for job in jobs]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    for job in jobs:
        assert job["err"] is None, job["err"]
        si = fetch(job["si"], 4 * len(sizes), np.float32)
        for t, (raw, d) in enumerate(zip(job["raws"], job["dsts"])):
            a = ref.amax(raw, BF16)
            assert float(si[t]) == ref.fp8_scale_inv(a, E4M3)
            bits_equal(fetch(d, sizes[t]), ref.scaled_cast(raw, BF16, E4M3, a))
        for b in job["srcs"] + job["dsts"] + [job["am"], job["si"]]:
            b.free()
        job["stream"].close()
