"""Sharded checkpoint quantisation on 2 GPUs with the library's NCCL exchange.

One process per GPU; each quantises its row range of every tensor with
mf_ckpt_quant_fp8 and the NCCL max all-reduce of the amax vector between the
two passes.  The shards, put back together, must equal the CPU oracle's
single-process quantisation bit for bit; mf_ckpt_quant_fp8_noalloc over the
same communicator, and the checkpoint plan in both forms (one launch, its
amax exchanged inside the kernel; two launches, the amax published by pass 1
and waited for inside pass 2; both through the two GPUs' exchange buffers),
must give the same bytes.  NCCL runs with its defaults, as
in bench.py.  Skipped with fewer than 2 GPUs.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _specs():
    from manifesto_b200 import checkpoint
    return checkpoint.llama3_8b_layout(layers=2, hidden=512, mlp=1536, heads=8, kv_heads=2, vocab=3001)


def _tensor(i, spec):
    from manifesto_b200 import synthetic
    return synthetic.normal_bf16(900 + i, spec.numel, 0.0, 0.02 * (1 + i % 7))


def _rank_main(rank: int, port: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    from manifesto_b200 import CUDABackend, _abi, checkpoint, sync_device
    from manifesto_b200.dtype import DType
    from tests.gpu_util import empty, fetch, to_device

    CUDABackend(rank)
    store = dist.TCPStore("127.0.0.1", port, WORLD, rank == 0, timeout=datetime.timedelta(seconds=60))
    comm = checkpoint.Communicator.from_store(store, WORLD, rank)
    specs = _specs()
    parts = checkpoint.partition(specs, WORLD, rank)
    srcs, dsts, entries, sizes = [], [], [], []
    for t, ((first, rows), s) in enumerate(zip(parts, specs)):
        shard = _tensor(t, s)[first * s.cols:(first + rows) * s.cols]
        srcs.append(to_device(shard))
        dsts.append(empty(shard.size))
        entries.append((srcs[-1].ptr, dsts[-1].ptr, shard.size, t, DType.BFLOAT16))
        sizes.append(shard.size)
    am = empty(4 * len(specs))
    si = empty(4 * len(specs))
    checkpoint.quantise(checkpoint.make_chunks(entries), len(entries), len(specs), am.ptr, si.ptr, comm=comm)
    sync_device()
    out = [fetch(d, n) for d, n in zip(dsts, sizes)]
    # the allocation-free entry point over the same communicator: the same codes and scales
    na_dsts = [empty(n) for n in sizes]
    na_si = empty(4 * len(specs))
    na_entries = [(e[0], d.ptr, e[2], e[3], e[4]) for e, d in zip(entries, na_dsts)]
    rc = _abi.lib().mf_ckpt_quant_fp8_noalloc(checkpoint.make_chunks(na_entries), len(na_entries), len(specs),
                                              na_si.ptr, int(DType.FLOAT8_E4M3), 0, comm.handle, None)
    assert rc == 0, _abi.last_error()
    sync_device()
    noalloc_same = all(np.array_equal(fetch(d, n), o) for d, n, o in zip(na_dsts, sizes, out)) and np.array_equal(
        fetch(na_si, 4 * len(specs)), fetch(si, 4 * len(specs)))
    # the one-launch plan (amax exchanged inside the kernel over peer memory), small groups, three runs
    pl_dsts = [empty(n) for n in sizes]
    pl_am, pl_si = empty(4 * len(specs)), empty(4 * len(specs))
    pl_entries = [(e[0], d.ptr, e[2], e[3], e[4]) for e, d in zip(entries, pl_dsts)]
    plan = checkpoint.QuantPlan(checkpoint.make_chunks(pl_entries), len(pl_entries), len(specs),
                                tensor_numel=[s.numel for s in specs], group_bytes=300_000, world=WORLD, rank=rank)
    assert plan.info()["groups"] > 3
    plan.connect_via_store(store)
    plan_same = True
    for _ in range(3):
        plan.run(pl_am.ptr, pl_si.ptr)
        sync_device()
        plan_same &= all(np.array_equal(fetch(d, n), o) for d, n, o in zip(pl_dsts, sizes, out))
        plan_same &= np.array_equal(fetch(pl_si, 4 * len(specs)), fetch(si, 4 * len(specs)))
        plan_same &= np.array_equal(fetch(pl_am, 4 * len(specs)), fetch(am, 4 * len(specs)))
    # the plan's two-launch form (amax published by pass 1's last CTA, waited for inside the cast pass):
    # outputs cleared before every run, four runs, the first three in a row with no barrier between ranks
    for k in range(4):
        for d, n in zip(pl_dsts, sizes):
            d.upload(np.zeros(n, np.uint8))
        if k % 2:
            plan.run_passes(pl_am.ptr, pl_si.ptr, passes=1)
            plan.run_passes(pl_am.ptr, pl_si.ptr, passes=2)
        else:
            plan.run_passes(pl_am.ptr, pl_si.ptr)
        sync_device()
        plan_same &= all(np.array_equal(fetch(d, n), o) for d, n, o in zip(pl_dsts, sizes, out))
        plan_same &= np.array_equal(fetch(pl_si, 4 * len(specs)), fetch(si, 4 * len(specs)))
        plan_same &= np.array_equal(fetch(pl_am, 4 * len(specs)), fetch(am, 4 * len(specs)))
    plan.run(pl_am.ptr, pl_si.ptr)  # and the one-launch form again after them
    sync_device()
    plan_same &= all(np.array_equal(fetch(d, n), o) for d, n, o in zip(pl_dsts, sizes, out))
    # every rank's last run has finished before any exchange buffer is freed
    store.add("plan_done", 1)
    deadline = time.time() + 60
    while int(store.add("plan_done", 0)) < WORLD and time.time() < deadline:
        time.sleep(0.01)
    plan.close()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), amax=fetch(am, 4 * len(specs), np.float32),
             scale_inv=fetch(si, 4 * len(specs), np.float32), noalloc_same=np.array([noalloc_same]),
             plan_same=np.array([plan_same]), *out)
    comm.close()


def test_two_gpu_nccl_quantisation(backend, ref, tmp_path):
    from manifesto_b200 import device_count
    if device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.exitcode is None:
            p.kill()
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(WORLD)]
    specs = _specs()
    for t, s in enumerate(specs):
        full = _tensor(t, s)
        want_amax = ref.amax(full, ref.BF16)
        for r in range(WORLD):
            assert bool(res[r]["noalloc_same"][0]), r
            assert bool(res[r]["plan_same"][0]), r
            assert res[r]["amax"][t] == want_amax, (s.name, r)
            assert res[r]["scale_inv"][t] == ref.fp8_scale_inv(want_amax, ref.E4M3)
        got = np.concatenate([res[r][f"arr_{t}"] for r in range(WORLD)])
        assert (got == ref.scaled_cast(full, ref.BF16, ref.E4M3, want_amax)).all(), s.name
