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


def _oproj_worker(rank, world, sp, port, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.set_num_threads(1)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        sys.path.insert(0, str(GOLDEN.parent.parent))
        from oracle import ulysses_oracle as oracle

        heads, H, L = 8, 256, 5
        topo = oracle.Topology(world, sp, heads, heads, H)
        cols = topo.output_q_heads * oracle.HEAD_DIM
        g = torch.Generator().manual_seed(7)
        attn = [torch.randn(sp * L, cols, generator=g).bfloat16() for _ in range(world)]
        w = [(torch.randn(H, topo.local_q_heads * oracle.HEAD_DIM, generator=g) * 0.1)
             .bfloat16() for _ in range(world)]
        mine = None
        for start in range(0, world, sp):
            grp = dist.new_group(list(range(start, start + sp)), backend="gloo")
            if start <= rank < start + sp:
                mine = grp
        got = oracle.rank_o_proj_gloo(topo, attn[rank], w[rank], L, mine)
        want = oracle.o_proj_world(topo, attn, w, L)[rank]
        if not torch.equal(got, want):
            raise AssertionError(f"rank {rank}: inverse exchange differs from all_to_all")
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("world,sp", [(2, 2), (4, 2)])
def test_gloo_inverse_exchange_matches_simulation(world, sp):
    """The oracle's inverse exchange (index shuffle) equals a real gloo
    all_to_all_single of the attention output blocks, also with base TP 2."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_oproj_worker, args=(world, sp, _free_port(), errq), nprocs=world,
                       join=True, start_method="spawn")
    assert errq.empty()


def test_inverse_exchange_undoes_forward_exchange():
    """Forward exchange of Q then the inverse returns every rank's own Q
    (the Q columns of its pre-exchange send buffer), on the golden c0 world."""
    import sys
    sys.path.insert(0, str(GOLDEN.parent.parent))
    from flash_ulysses_b200.workloads import CONFIGS, make_world
    from oracle import ulysses_oracle as oracle

    cfg = CONFIGS["c0"]
    L = 64
    xs, pos, params = make_world(cfg, L, seed=0)
    topo = oracle.Topology(cfg.world_size, cfg.sp_size, cfg.num_heads, cfg.num_kv_heads,
                           cfg.hidden_size)
    outs = oracle.simulate_world(topo, xs, pos, params)
    back = oracle.inverse_exchange_world(topo, [o[0] for o in outs], L)
    qc = topo.output_q_heads * oracle.HEAD_DIM
    for r in range(cfg.world_size):
        send = oracle.rank_send(topo, xs[r], pos[r], params[r])
        own_q = torch.cat([send[d][:, :qc] for d in range(cfg.sp_size)], dim=-1)
        assert torch.equal(back[r], own_q)
