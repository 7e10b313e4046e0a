"""The sharded checkpoint-quantisation protocol with 2 CPU ranks over gloo.

Each rank owns the row range mf_ckpt_partition gives it, folds its per-tensor
amax with the CPU oracle, the ranks max-all-reduce the amax vector (the one
exchange of the GPU path, done there by NCCL), then each rank casts its rows.
The concatenated shards must equal a single-process quantisation bit for bit.
No GPU is involved; this checks the host-side partition and exchange logic.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _specs():
    from manifesto_b200 import checkpoint
    return checkpoint.llama3_8b_layout(layers=2, hidden=64, mlp=192, heads=4, kv_heads=2, vocab=301)


def _tensor(i, spec):
    from manifesto_b200 import synthetic
    return synthetic.normal_bf16(500 + i, spec.numel, 0.0, 0.02 * (1 + i % 5))


def _rank_main(rank: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    from manifesto_b200 import checkpoint
    from oracle import ref

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=__import__("datetime").timedelta(seconds=60))
    specs = _specs()
    parts = checkpoint.partition(specs, WORLD, rank)
    shards = []
    amax = np.zeros(len(specs), np.float32)
    for t, ((first, rows), s) in enumerate(zip(parts, specs)):
        full = _tensor(t, s)
        shard = full[first * s.cols:(first + rows) * s.cols]
        shards.append(shard)
        amax[t] = ref.amax(shard, ref.BF16) if shard.size else 0.0
    a = torch.from_numpy(amax)
    dist.all_reduce(a, op=dist.ReduceOp.MAX)
    amax = a.numpy()
    out = [ref.scaled_cast(sh, ref.BF16, ref.E4M3, float(amax[t])) if sh.size else np.zeros(0, np.uint8)
           for t, sh in enumerate(shards)]
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), amax=amax, *out)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_quantisation_matches_single_process(tmp_path, ref):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(WORLD)]
    specs = _specs()
    assert (res[0]["amax"] == res[1]["amax"]).all()
    for t, s in enumerate(specs):
        full = _tensor(t, s)
        want_amax = ref.amax(full, ref.BF16)
        assert res[0]["amax"][t] == want_amax
        want = ref.scaled_cast(full, ref.BF16, ref.E4M3, want_amax)
        got = np.concatenate([res[r][f"arr_{t}"] for r in range(WORLD)])
        assert (got == want).all(), s.name


def test_rank_failure_is_reported_not_hung(tmp_path):
    """A rank that dies before the exchange ends the other rank's collective with an error."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_lonely_rank, args=(port,))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 3, "the surviving rank must see a timeout, not hang"


def _lonely_rank(port: int) -> None:
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        # rank 1 never joins: the rendezvous itself must time out
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=5))
        t = torch.zeros(4)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    except Exception:
        os._exit(3)
    os._exit(0)
