"""The checkpoint plan (mf_ckpt_plan_*, checkpoint.QuantPlan) on one GPU: the step in one launch and in
two launches with the exchange fused into them (mf_ckpt_plan_run_passes).

Every run is checked bit for bit against the CPU oracle (amax, scale_inv and the FP8
codes of every tensor) and against the two-pass mf_ckpt_quant_fp8 on the same table.
Runs follow each other on one plan with different data, so a value left over from the
previous run in the per-run scratch (the kernel alternates two copies by run parity)
would show.  Several runs with an unreachable peer check that the kernel's bounded
wait reports MF_DEVICE_TIMEOUT instead of hanging.
"""
import ctypes
import multiprocessing
import os

import numpy as np
import pytest

from manifesto_b200 import checkpoint, synthetic
from manifesto_b200._abi import call
from manifesto_b200.dtype import DType
from oracle.ref import BF16, E4M3, E5M2, F16, F32, ITEMSIZE

from .gpu_util import bits_equal, empty, fetch, to_device

pytestmark = pytest.mark.gpu

WIRE = {BF16: DType.BFLOAT16, F16: DType.FLOAT16, F32: DType.FLOAT32}


def _layout():
    return checkpoint.llama3_8b_layout(layers=3, hidden=512, mlp=1792, heads=8, kv_heads=2, vocab=4000)


def _raw(seed, n, dt, sigma):
    v = synthetic.normal_f32(seed, n, 0.0, sigma)
    return v.view(np.uint32).copy() if dt == F32 else synthetic.f32_to_bf16_bits(v) if dt == BF16 else \
        v.astype(np.float16).view(np.uint16)


def _check(ref, raws, dts, dsts, ns, amax, sinv, fp8, compat=0):
    got_a = fetch(amax, 4 * len(raws), np.float32)
    got_s = fetch(sinv, 4 * len(raws), np.float32)
    for t, (raw, dt) in enumerate(zip(raws, dts)):
        a = ref.amax(raw, dt)
        assert float(got_a[t]) == a, t
        assert float(got_s[t]) == ref.fp8_scale_inv(a, fp8), t
        if ns[t]:
            bits_equal(fetch(dsts[t], ns[t]), ref.scaled_cast(raw, dt, fp8, a, compat=compat))


def _run(plan, form, run, am, si):
    """One step in the named form: "one" the one-launch kernel, "passes" the two-launch form (passes=3, or
    1 then 2 on odd runs), "mixed" alternating the two forms on one plan."""
    if form == "one" or (form == "mixed" and run % 2 == 0):
        plan.run(am, si)
    elif run % 2:
        plan.run_passes(am, si, passes=1)
        plan.run_passes(am, si, passes=2)
    else:
        plan.run_passes(am, si)


@pytest.mark.parametrize("form", ["one", "passes", "mixed"])
@pytest.mark.parametrize("group_bytes", [0, 200_000, 1])
def test_plan_runs_in_a_row_match_oracle_and_two_pass(backend, ref, group_bytes, form):
    """Three runs on one plan, the data replaced between them (sigma 0.5, 0.005, 0.05): every run
    exact; one group for the whole table, many groups, and one group per tensor; in the one-launch
    form, the two-launch form, and both alternating on one plan (each form clears the other's
    per-run scratch)."""
    specs = _layout()
    n = [s.numel for s in specs]
    srcs = [empty(2 * k) for k in n]
    dsts = [empty(k) for k in n]
    ref_dsts = [empty(k) for k in n]
    chunks = checkpoint.make_chunks([(s.ptr, d.ptr, k, t, DType.BFLOAT16) for t, (s, d, k) in enumerate(zip(srcs, dsts, n))])
    ref_chunks = checkpoint.make_chunks([(s.ptr, d.ptr, k, t, DType.BFLOAT16)
                                         for t, (s, d, k) in enumerate(zip(srcs, ref_dsts, n))])
    plan = checkpoint.QuantPlan(chunks, len(n), len(n), tensor_numel=n, group_bytes=group_bytes)
    info = plan.info()
    assert info["elements"] == sum(n)
    if group_bytes == 1:
        assert info["groups"] == len(n)
    am, si, ram, rsi = empty(4 * len(n)), empty(4 * len(n)), empty(4 * len(n)), empty(4 * len(n))
    for run, sigma in enumerate((0.5, 0.005, 0.05)):
        raws = [_raw(9000 + 100 * run + t, k, BF16, sigma * (1 + t % 5)) for t, k in enumerate(n)]
        for s, r in zip(srcs, raws):
            s.upload(r)
        for d in dsts:
            d.upload(np.zeros(d.nbytes, np.uint8))
        _run(plan, form, run, am.ptr, si.ptr)
        checkpoint.quantise(ref_chunks, len(n), len(n), ram.ptr, rsi.ptr)
        _check(ref, raws, [BF16] * len(n), dsts, n, am, si, E4M3)
        for d, r in zip(dsts, ref_dsts):
            bits_equal(fetch(d, d.nbytes), fetch(r, r.nbytes))
        bits_equal(fetch(si, 4 * len(n)), fetch(rsi, 4 * len(n)))
    plan.close()
    for b in srcs + dsts + ref_dsts + [am, si, ram, rsi]:
        b.free()


@pytest.mark.parametrize("form", ["one", "passes"])
@pytest.mark.parametrize("src_dt,fp8,compat", [(F16, E4M3, 0), (F32, E5M2, 0), (BF16, E5M2, 1), (F32, E4M3, 1)])
def test_plan_source_dtypes_ragged_split_chunks(backend, ref, src_dt, fp8, compat, form):
    """F16 / F32 / BF16 sources, both FP8 formats, both compat modes; ragged sizes, a tensor split
    into chunks that leave the second off 16-byte alignment, an empty chunk, a tensor with no
    chunk at all (its amax 0, scale_inv 1), many small groups."""
    sizes = [40000, 33333, 20001, 3 * 16384 + 5, 5 * 8192, 17, 0, 4096]
    raws, srcs, dsts, entries = [], [], [], []
    for t, k in enumerate(sizes):
        raw = _raw(8100 + t, max(k, 1), src_dt, 0.05 * (t + 1))[:k]
        src, dst = to_device(raw, pad=16), empty(max(k, 1))
        raws.append(raw), srcs.append(src), dsts.append(dst)
        if t == 0:
            cuts = [0, 12345, 12345, k]
        elif t == 2:
            cuts = [0, 7, k]
        elif t == 6:
            continue  # no chunk: this rank holds nothing of tensor 6
        else:
            cuts = [0, k]
        for a, b in zip(cuts, cuts[1:]):
            entries.append((src.ptr + a * ITEMSIZE[src_dt], dst.ptr + a, b - a, t, WIRE[src_dt]))
    plan = checkpoint.QuantPlan(checkpoint.make_chunks(entries), len(entries), len(sizes), tensor_numel=sizes,
                                group_bytes=60_000, fp8_dtype=DType(fp8), compat=compat)
    assert plan.info()["groups"] > 2
    am, si = empty(4 * len(sizes)), empty(4 * len(sizes))
    for run in range(2):
        _run(plan, form, run, am.ptr, si.ptr)
    _check(ref, raws, [src_dt] * len(sizes), dsts, sizes, am, si, fp8, compat)
    plan.close()
    for b in srcs + dsts + [am, si]:
        b.free()


def test_plan_rejects(backend):
    from manifesto_b200.errors import DTypeUnsupported, InvalidArgument
    a, b = empty(64), empty(64)
    mixed = checkpoint.make_chunks([(a.ptr, b.ptr, 8, 0, DType.BFLOAT16), (a.ptr, b.ptr, 8, 1, DType.FLOAT32)])
    with pytest.raises(DTypeUnsupported, match="one source dtype per plan"):
        checkpoint.QuantPlan(mixed, 2, 2)
    one = checkpoint.make_chunks([(a.ptr, b.ptr, 8, 0, DType.BFLOAT16)])
    with pytest.raises(InvalidArgument, match="world"):
        checkpoint.QuantPlan(one, 1, 1, world=9, rank=0)
    with pytest.raises(InvalidArgument, match="names tensor"):
        checkpoint.QuantPlan(checkpoint.make_chunks([(a.ptr, b.ptr, 8, 3, DType.BFLOAT16)]), 1, 2)
    with pytest.raises(InvalidArgument, match="ipc_handle"):
        call("mf_ckpt_plan_create", one, 1, 1, None, 0, 2, 0, int(DType.FLOAT8_E4M3), 0,
             ctypes.byref(ctypes.c_void_p()), None)
    # the two-launch form: a run's amax pass, then its cast pass, before anything else
    plan = checkpoint.QuantPlan(one, 1, 1)
    for bad in (0, 4):
        with pytest.raises(InvalidArgument, match="passes must be"):
            plan.run_passes(None, None, passes=bad)
    with pytest.raises(InvalidArgument, match="no amax pass"):
        plan.run_passes(None, None, passes=2)
    plan.run_passes(None, None, passes=1)
    with pytest.raises(InvalidArgument, match="cast pass has not run"):
        plan.run_passes(None, None, passes=1)
    with pytest.raises(InvalidArgument, match="pending"):
        plan.run(None, None)
    plan.run_passes(None, None, passes=2)
    plan.run(None, None)
    plan.close()
    a.free(), b.free()


def _silent_peer(port: int, ready, done) -> None:
    """Rank 1 of a two-rank plan on the same GPU that connects and never runs."""
    import datetime

    import torch.distributed as dist

    from manifesto_b200 import CUDABackend
    CUDABackend(0)
    store = dist.TCPStore("127.0.0.1", port, 2, False, timeout=datetime.timedelta(seconds=60))
    src, dst = empty(2 * 4096), empty(4096)
    plan = checkpoint.QuantPlan(checkpoint.make_chunks([(src.ptr, dst.ptr, 4096, 0, DType.BFLOAT16)]), 1, 1,
                                tensor_numel=[8192], world=2, rank=1)
    plan.connect_via_store(store)
    ready.set()
    done.wait(120)
    plan.close()


@pytest.mark.parametrize("form", ["one", "passes"])
def test_plan_peer_that_never_runs_times_out(backend, ref, form):
    """A two-rank plan whose other rank connects but never launches: this rank's wait for the
    peer's amax runs out after its bound (~2 s), the run reports MF_DEVICE_TIMEOUT through the
    sticky status instead of hanging, and the context stays usable.  In the two-launch form the
    amax pass publishes into the peer's buffer and the cast pass's waits run out."""
    import datetime
    import socket

    import torch.distributed as dist

    from tests.test_gpu_failure import MF_DEVICE_TIMEOUT, status
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    store = dist.TCPStore("127.0.0.1", port, 2, True, timeout=datetime.timedelta(seconds=60), wait_for_workers=False)
    ctx = multiprocessing.get_context("spawn")
    ready, done = ctx.Event(), ctx.Event()
    peer = ctx.Process(target=_silent_peer, args=(port, ready, done))
    peer.start()
    try:
        raw = synthetic.normal_bf16(5, 4096, 0.0, 1.0)
        src, dst, am, si = to_device(raw), empty(4096), empty(4), empty(4)
        plan = checkpoint.QuantPlan(checkpoint.make_chunks([(src.ptr, dst.ptr, 4096, 0, DType.BFLOAT16)]), 1, 1,
                                    tensor_numel=[8192], world=2, rank=0)
        plan.connect_via_store(store)  # returns once the peer has published its handle
        assert ready.wait(120), "peer did not come up"
        assert status() == 0
        if form == "one":
            plan.run(am.ptr, si.ptr)
        else:
            plan.run_passes(am.ptr, si.ptr)
        assert status() == MF_DEVICE_TIMEOUT
        plan.close()  # unmaps the peer's buffer before the peer frees it
        done.set()
        peer.join(60)
        # the context still works
        from tests.gpu_util import convert
        x = np.arange(4096, dtype=np.float32) * 0.25
        assert np.array_equal(convert(x, F32, BF16, 4096), ref.convert(x, F32, BF16))
        assert status() == 0
        for b in (src, dst, am, si):
            b.free()
    finally:
        done.set()
        peer.join(60)
        if peer.exitcode is None:
            peer.kill()
