"""Seeded synthetic workloads with the shapes and distributions of the
benchmark configurations.

There is no public dataset behind this operator; the benchmark shapes are the
workload.  Distributions follow the reference's harness
(``tests/torch_base.py:7-36``, ``tests/benchmark.py:44-62``) with the
generator settings of the benchmark configurations:

* ``hidden_states`` BF16 ``[L, H]`` ~ N(0, 1)
* ``qkv_weight`` BF16 ``[H, N]`` ~ N(0, H^-1/2), packed Q | K | V, one weight
  per base-TP group
* norm weights FP32 ``[128]`` = 1 + 0.1 N(0, 1)
* positions int64 ``[L]`` ~ U[0, max_position)
* rope cache FP32 ``[max_position, 128]`` = cos | sin of ``pos * 1e6^(-2i/128)``
* the last global token of every SP group is zeroed with position 0, as the
  reference harness does to exercise caller padding (benchmark.py:60-62).

CPU generation uses numpy's PCG64 so that fixtures are reproducible across
hosts; ``device="cuda"`` uses a torch CUDA generator (fast, for benchmarking).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

HEAD_DIM = 128


@dataclass(frozen=True)
class Config:
    name: str
    world_size: int
    sp_size: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    tokens: tuple
    max_position: int
    note: str = ""

    @property
    def base_tp_size(self):
        return self.world_size // self.sp_size

    @property
    def local_q_heads(self):
        return self.num_heads // self.base_tp_size

    @property
    def local_kv_heads(self):
        return self.num_kv_heads // self.base_tp_size

    @property
    def packed_width(self):
        return (self.local_q_heads + 2 * self.local_kv_heads) * HEAD_DIM

    def flops(self, tokens):
        """GEMM-equivalent FLOPs per rank per call, 2 L H N (benchmark.py:243)."""
        return 2 * tokens * self.hidden_size * self.packed_width


# The five benchmark configurations.  c0 is the CPU/gloo plumbing case run
# through the reference PyTorch path; c1-c4 are the GPU shapes.
CONFIGS = {
    "c0": Config("c0", 2, 2, 1024, 8, 2, (64,), 4096, "CPU/gloo plumbing"),
    "c1": Config(
        "c1", 4, 4, 4096, 32, 8,
        (1, 63, 64, 65, 127, 128, 129, 1024, 2048, 4096, 8192), 32768,
        "Qwen3-8B-like attention input",
    ),
    "c2": Config("c2", 8, 8, 4096, 32, 8, (1024, 4096, 8192), 32768,
                 "8xB200, sp=8"),
    "c3": Config("c3", 8, 4, 4096, 32, 8, (1, 16, 64, 129, 512), 32768,
                 "TP2 x SP4 decode-leaning"),
    "c4": Config("c4", 8, 8, 5120, 64, 8, (8192,), 131072,
                 "Qwen3-32B-like large shape"),
}


def rope_cache(max_position, device="cpu"):
    """FP32 ``[max_position, 128]`` cos | sin table, theta = 1e6.

    Angles are formed in float64 and rounded once so that the table is the
    same on every host."""
    inv_freq = 1.0 / (1e6 ** (np.arange(0, HEAD_DIM, 2, dtype=np.float64) / HEAD_DIM))
    angles = np.arange(max_position, dtype=np.float64)[:, None] * inv_freq[None, :]
    table = np.concatenate((np.cos(angles), np.sin(angles)), axis=1).astype(np.float32)
    return torch.from_numpy(table).to(device)


def _bf16(array):
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).bfloat16()


def make_parameters(hidden_size, packed_width, max_position, *, tp_rank=0, seed=0,
                    device="cpu"):
    """Weights for one base-TP group plus the shared norm/RoPE tables."""
    if device == "cpu":
        rng = np.random.default_rng([seed, 1, tp_rank])
        weight = _bf16(rng.standard_normal((hidden_size, packed_width), dtype=np.float32)
                       * np.float32(hidden_size ** -0.5))
        rng_g = np.random.default_rng([seed, 2])
        q_norm = torch.from_numpy(
            (1 + 0.1 * rng_g.standard_normal(HEAD_DIM)).astype(np.float32))
        k_norm = torch.from_numpy(
            (1 + 0.1 * rng_g.standard_normal(HEAD_DIM)).astype(np.float32))
    else:
        gen = torch.Generator(device=device).manual_seed(seed * 1000 + 17 + tp_rank)
        weight = (torch.randn(hidden_size, packed_width, device=device,
                              generator=gen) * hidden_size ** -0.5).bfloat16()
        gen_g = torch.Generator(device=device).manual_seed(seed * 1000 + 3)
        q_norm = 1 + 0.1 * torch.randn(HEAD_DIM, device=device, generator=gen_g)
        k_norm = 1 + 0.1 * torch.randn(HEAD_DIM, device=device, generator=gen_g)
    return dict(
        qkv_weight=weight,
        q_norm_weight=q_norm.float(),
        k_norm_weight=k_norm.float(),
        rope_cache=rope_cache(max_position, device),
        q_epsilon=1e-6,
        k_epsilon=1e-6,
    )


def make_rank_inputs(hidden_size, tokens, max_position, *, rank, sp_size, seed=0,
                     pad_last=True, device="cpu"):
    """``(hidden_states, positions)`` for one rank.

    With ``pad_last`` the last global token of the SP group (which lives on
    the group's last rank) is zeroed with position 0 (benchmark.py:60-62)."""
    sp_rank = rank % sp_size
    if device == "cpu":
        rng = np.random.default_rng([seed, 3, rank])
        x = _bf16(rng.standard_normal((tokens, hidden_size), dtype=np.float32))
        positions = torch.from_numpy(
            rng.integers(0, max_position, size=tokens, dtype=np.int64))
    else:
        gen = torch.Generator(device=device).manual_seed(seed * 1000 + 101 + rank)
        x = torch.randn(tokens, hidden_size, device=device, generator=gen).bfloat16()
        positions = torch.randint(0, max_position, (tokens,), device=device,
                                  generator=gen, dtype=torch.int64)
    if pad_last:
        global_tokens = torch.arange(tokens, device=x.device) + sp_rank * tokens
        pad = global_tokens >= tokens * sp_size - 1
        x[pad] = 0
        positions[pad] = 0
    return x, positions


def make_world(cfg: Config, tokens, *, seed=0, pad_last=True, device="cpu"):
    """Inputs and parameters for every rank of ``cfg`` at ``tokens`` per rank.

    Returns ``(xs, positions, params_by_rank)``; ranks in one base-TP group
    (same ``rank // sp_size``) share their parameter dict."""
    by_tp = {}
    xs, pos, params = [], [], []
    for rank in range(cfg.world_size):
        tp_rank = rank // cfg.sp_size
        if tp_rank not in by_tp:
            by_tp[tp_rank] = make_parameters(
                cfg.hidden_size, cfg.packed_width, cfg.max_position,
                tp_rank=tp_rank, seed=seed, device=device)
        x, p = make_rank_inputs(cfg.hidden_size, tokens, cfg.max_position,
                                rank=rank, sp_size=cfg.sp_size, seed=seed,
                                pad_last=pad_last, device=device)
        xs.append(x)
        pos.append(p)
        params.append(by_tp[tp_rank])
    return xs, pos, params
