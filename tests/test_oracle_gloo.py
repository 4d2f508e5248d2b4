"""The oracle's per-rank form over a real gloo all_to_all_single (world 2 and
a TP2 x SP2 world of 4) reproduces the golden vectors: covers the N > 1
exchange path on CPU."""

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

GOLDEN = Path(__file__).resolve().parent / "golden"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.set_num_threads(1)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        sys.path.insert(0, str(GOLDEN.parent.parent))
        from flash_ulysses_b200.workloads import Config, make_world
        from oracle import ulysses_oracle as oracle

        z = np.load(GOLDEN / f"{case}.npz")
        meta = {k[5:]: z[k].item() for k in z.files if k.startswith("meta_")}
        cfg = Config("g", meta["world_size"], meta["sp_size"], meta["hidden_size"],
                     meta["num_heads"], meta["num_kv_heads"], (meta["tokens"],),
                     meta["max_position"])
        xs, pos, params = make_world(cfg, meta["tokens"], seed=meta["seed"])
        topo = oracle.Topology(cfg.world_size, cfg.sp_size, cfg.num_heads, cfg.num_kv_heads,
                               cfg.hidden_size)
        S = cfg.sp_size
        mine = None
        for start in range(0, world, S):
            g = dist.new_group(list(range(start, start + S)), backend="gloo")
            if start <= rank < start + S:
                mine = g
        q, k, v = oracle.rank_forward_gloo(topo, xs[rank], pos[rank], params[rank], mine)
        for t, name in ((q, "q"), (k, "k"), (v, "v")):
            want = torch.from_numpy(z[f"{name}{rank}"])
            if not torch.equal(t.view(torch.int16), want):
                raise AssertionError(f"rank {rank} {name} differs")
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("case,world", [("c0", 2), ("tp2_sp2", 4)])
def test_gloo_exchange_matches_golden(case, world):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), case, errq), nprocs=world,
                       join=True, start_method="spawn")
    assert errq.empty()
