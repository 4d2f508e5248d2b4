"""Generate the golden vectors that pin the CPU oracle.

Runs the reference's own PyTorch path -- ``TorchReference.__call__`` from
joey-shao/flash_ulysses ``tests/torch_base.py:48-76``, imported unmodified from
a checkout of the reference -- over gloo with one process per rank, on inputs
from ``flash_ulysses_b200.workloads`` (seeded, host-independent).  Its
``__init__`` hard-codes NCCL groups (torch_base.py:40-46), so instances are
built with ``object.__new__`` and given the gloo SP group directly.

Writes ``tests/golden/<case>.npz`` holding the outputs of every rank (BF16 as
uint16) and SHA-256 digests of the inputs, so a test can regenerate the inputs,
confirm they are the same, and compare the oracle bit for bit.

Usage (needs the reference checkout; not run by the test suite)::

    python tests/golden/make_golden.py --reference /path/to/flash_ulysses
"""

from __future__ import annotations

import argparse
import hashlib
import os
import socket
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from flash_ulysses_b200.workloads import Config, make_world  # noqa: E402

# name -> (config, tokens per rank, seed)
CASES = {
    # Benchmark configuration 0 exactly: P=S=2, H=1024, Q/KV 8/2, L=64, seed 0.
    "c0": (Config("c0", 2, 2, 1024, 8, 2, (64,), 4096), 64, 0),
    # Base TP 2 x SP 2 with an odd length and two SP groups.
    "tp2_sp2": (Config("tp2_sp2", 4, 2, 256, 8, 4, (5,), 64), 5, 1),
    # L=1, S=2: the last rank's only token is caller padding.
    "l1_sp2": (Config("l1_sp2", 2, 2, 128, 2, 2, (1,), 16), 1, 2),
}


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def input_digests(cfg, tokens, seed):
    xs, pos, params = make_world(cfg, tokens, seed=seed)
    out = {}
    for r in range(cfg.world_size):
        out[f"x{r}"] = digest(xs[r])
        out[f"pos{r}"] = digest(pos[r])
        out[f"w{r}"] = digest(params[r]["qkv_weight"])
    out["q_norm"] = digest(params[0]["q_norm_weight"])
    out["k_norm"] = digest(params[0]["k_norm_weight"])
    out["rope"] = digest(params[0]["rope_cache"])
    return out


def _worker(rank, world, port, reference, case, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, str(Path(reference) / "tests"))
    from torch_base import TorchReference  # the reference's own code, unmodified

    cfg, tokens, seed = CASES[case]
    xs, pos, params = make_world(cfg, tokens, seed=seed)
    S = cfg.sp_size
    my_group = None
    for start in range(0, world, S):
        g = dist.new_group(list(range(start, start + S)), backend="gloo")
        if start <= rank < start + S:
            my_group = g
    ref = object.__new__(TorchReference)
    ref.context = SimpleNamespace(
        local_q_heads=cfg.local_q_heads, local_kv_heads=cfg.local_kv_heads, sp_size=S)
    ref.parameters = params[rank]
    ref.group = my_group
    q, k, v = ref(xs[rank], pos[rank])
    np.savez(Path(outdir) / f"{case}_rank{rank}.npz",
             q=q.view(torch.int16).numpy(), k=k.view(torch.int16).numpy(),
             v=v.view(torch.int16).numpy())
    dist.barrier()
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="checkout of joey-shao/flash_ulysses")
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    args = ap.parse_args()
    import tempfile

    for case in args.cases:
        cfg, tokens, seed = CASES[case]
        with tempfile.TemporaryDirectory() as tmp:
            mp.spawn(_worker, args=(cfg.world_size, free_port(), args.reference, case, tmp),
                     nprocs=cfg.world_size, join=True)
            arrays = {}
            for r in range(cfg.world_size):
                part = np.load(Path(tmp) / f"{case}_rank{r}.npz")
                for c in "qkv":
                    arrays[f"{c}{r}"] = part[c]
        meta = dict(world_size=cfg.world_size, sp_size=cfg.sp_size, hidden_size=cfg.hidden_size,
                    num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, tokens=tokens,
                    max_position=cfg.max_position, seed=seed, torch=torch.__version__)
        for k, v in input_digests(cfg, tokens, seed).items():
            arrays[f"sha_{k}"] = np.array(v)
        for k, v in meta.items():
            arrays[f"meta_{k}"] = np.array(v)
        np.savez_compressed(HERE / f"{case}.npz", **arrays)
        print(f"wrote {case}.npz")


if __name__ == "__main__":
    main()
