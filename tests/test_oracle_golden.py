"""The CPU oracle against golden vectors produced by the reference's own
PyTorch path (``TorchReference.__call__``, tests/torch_base.py:48-76, run
unmodified over gloo by tests/golden/make_golden.py): bit for bit."""

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from flash_ulysses_b200.workloads import Config, make_world
from oracle import ulysses_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(case):
    z = np.load(GOLDEN / f"{case}.npz")
    meta = {k[5:]: z[k].item() for k in z.files if k.startswith("meta_")}
    return z, meta


def digest(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def world_for(meta):
    cfg = Config("golden", meta["world_size"], meta["sp_size"], meta["hidden_size"],
                 meta["num_heads"], meta["num_kv_heads"], (meta["tokens"],),
                 meta["max_position"])
    xs, pos, params = make_world(cfg, meta["tokens"], seed=meta["seed"])
    topo = oracle.Topology(cfg.world_size, cfg.sp_size, cfg.num_heads, cfg.num_kv_heads,
                           cfg.hidden_size)
    return cfg, topo, xs, pos, params


def test_golden_cases_present():
    assert {"c0", "tp2_sp2", "l1_sp2"} <= set(CASES)


@pytest.mark.parametrize("case", CASES)
def test_inputs_regenerate_identically(case):
    z, meta = load(case)
    cfg, _, xs, pos, params = world_for(meta)
    for r in range(cfg.world_size):
        assert digest(xs[r]) == z[f"sha_x{r}"].item()
        assert digest(pos[r]) == z[f"sha_pos{r}"].item()
        assert digest(params[r]["qkv_weight"]) == z[f"sha_w{r}"].item()
    assert digest(params[0]["rope_cache"]) == z["sha_rope"].item()
    assert digest(params[0]["q_norm_weight"]) == z["sha_q_norm"].item()


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_bit_for_bit(case):
    z, meta = load(case)
    cfg, topo, xs, pos, params = world_for(meta)
    outs = oracle.simulate_world(topo, xs, pos, params)
    for r in range(cfg.world_size):
        for c, name in enumerate("qkv"):
            want = torch.from_numpy(z[f"{name}{r}"])
            got = outs[r][c].view(torch.int16)
            assert got.shape == want.shape
            assert torch.equal(got, want), f"{case} rank {r} {name}"


def test_padding_rows_are_zero():
    """The reference zeroes the last global token (benchmark.py:60-62); its
    projection and rotated values are exactly zero on the receiving side."""
    z, meta = load("c0")
    L, S = meta["tokens"], meta["sp_size"]
    for r in range(meta["world_size"]):
        for name in "qkv":
            rows = torch.from_numpy(z[f"{name}{r}"])
            assert torch.all(rows[S * L - 1] == 0)       # last row: last source's last token
            assert torch.any(rows[S * L - 2] != 0)
