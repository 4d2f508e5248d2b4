"""CPU oracle for the fused Ulysses QKV path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.  The shipped path (``flash_ulysses_b200``) never calls into it and fails
loudly when its CUDA library is missing.

It restates, with plain torch CPU operators, the reference's own PyTorch
implementation of ``FlashUlyssesContext.ulysses_qkv_forward``
(joey-shao/flash_ulysses ``tests/torch_base.py:48-76``):

    x @ W (BF16 out)                              torch_base.py:52
    split into Q | K | V widths                   torch_base.py:51-52
    cos, sin = rope_cache[positions].chunk(2)     torch_base.py:53
    FP32 RMSNorm, * gamma, round to BF16          torch_base.py:55-61
    FP32 NeoX rotation, round to BF16             torch_base.py:62-64
    pack [S, L, N/S] per SP group                 torch_base.py:68-69
    all_to_all_single inside the SP group         torch_base.py:71
    unpack rows [S*L] and split Q | K | V         torch_base.py:72-76

Head/rank placement follows the reference's DESIGN.md:20-37 (consecutive SP
groups, ``dst = group_start + head // heads_per_gpu``).

Pinning: the restatement is checked bit-for-bit against golden vectors that
were produced by importing and running the reference's own
``TorchReference.__call__`` over gloo (``tests/golden/make_golden.py``).

Two entry points:

* ``simulate_world`` runs every rank of a world in one process and performs the
  all-to-all as an index shuffle (the exact semantics of
  ``all_to_all_single`` with equal splits).
* ``rank_forward_gloo`` is the per-rank form that calls
  ``torch.distributed.all_to_all_single`` on a (gloo) SP group, as the
  reference does with NCCL.

For the output side (no counterpart in the reference, which stops at the
forward exchange): ``inverse_exchange_world`` / ``o_proj_world`` and the
per-rank ``rank_o_proj_gloo`` return each source's rows for all of its local
heads and apply the output projection with FP32 accumulation.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM = 128


@dataclass(frozen=True)
class Topology:
    """World layout (reference context.py:95-117)."""

    world_size: int
    sp_size: int
    num_heads: int
    num_kv_heads: int
    hidden_size: int

    @property
    def base_tp_size(self) -> int:
        return self.world_size // self.sp_size

    @property
    def local_q_heads(self) -> int:
        return self.num_heads // self.base_tp_size

    @property
    def local_kv_heads(self) -> int:
        return self.num_kv_heads // self.base_tp_size

    @property
    def output_q_heads(self) -> int:
        return self.num_heads // self.world_size

    @property
    def output_kv_heads(self) -> int:
        return self.num_kv_heads // self.world_size

    @property
    def packed_width(self) -> int:
        return (self.local_q_heads + 2 * self.local_kv_heads) * HEAD_DIM

    def widths(self):
        """Local Q, K, V projection widths (torch_base.py:51)."""
        return (
            self.local_q_heads * HEAD_DIM,
            self.local_kv_heads * HEAD_DIM,
            self.local_kv_heads * HEAD_DIM,
        )


def project(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """BF16 projection ``x @ W`` (torch_base.py:52)."""
    return x @ weight


def norm_rope(y, gamma, epsilon, cos, sin):
    """Headwise RMSNorm then NeoX RoPE with the reference's rounding points.

    Follows torch_base.py:55-64: FP32 ``v * rsqrt(mean(v^2) + eps)``,
    ``* gamma``, round to BF16 and back, FP32 rotation
    ``(lo*cos - hi*sin, hi*cos + lo*sin)``, round to BF16.
    ``y`` is BF16 ``[L, heads*128]``; ``cos``/``sin`` are FP32 ``[L, 1, 64]``.
    """
    tokens = y.size(0)
    value = y.reshape(tokens, -1, HEAD_DIM).float()
    value = value * torch.rsqrt(value.square().mean(dim=-1, keepdim=True) + epsilon)
    value = (value * gamma).bfloat16().float()
    lo, hi = value.chunk(2, dim=-1)
    rotated = torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)
    return rotated.bfloat16().flatten(1)


def norm_rope_fp32(y32, gamma, epsilon, cos, sin):
    """Headwise RMSNorm then NeoX RoPE kept in FP32 from the accumulator, one
    BF16 rounding at the end: the numerics of the reference's Hopper kernel
    (flash_ulysses_kernel_hopper.cu:129-152: ``rsqrtf(sum/128 + eps)``,
    ``mul_row``, ``mul_col``, rotation ``lo*c - hi*s`` / ``hi*c + lo*s`` built
    with --fmad=false).  ``y32`` is the FP32 projection ``[L, heads*128]``."""
    tokens = y32.size(0)
    value = y32.reshape(tokens, -1, HEAD_DIM).float()
    value = value * torch.rsqrt(value.square().mean(dim=-1, keepdim=True) + epsilon)
    value = value * gamma
    lo, hi = value.chunk(2, dim=-1)
    rotated = torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)
    return rotated.bfloat16().flatten(1)


def rank_send(topo: Topology, x, positions, params, projection=None, fp32_epilogue=False):
    """Per-rank compute before the exchange: returns the packed ``[S, L, N/S]``
    send buffer (torch_base.py:50-69).

    ``projection`` optionally replaces ``x @ W`` with a given BF16 ``[L, N]``
    tensor, so the epilogue can be checked on exactly the projection another
    implementation produced.  ``fp32_epilogue`` selects the reference Hopper
    kernel's numerics instead of its PyTorch path's (see ``norm_rope_fp32``);
    the FP32 projection is then the exact sum rounded once to FP32."""
    cos, sin = params["rope_cache"][positions].unsqueeze(1).chunk(2, dim=-1)
    if fp32_epilogue:
        y32 = (x.double() @ params["qkv_weight"].double()).float()
        q, k, v = y32.split(topo.widths(), dim=-1)
        q = norm_rope_fp32(q, params["q_norm_weight"], params["q_epsilon"], cos, sin)
        k = norm_rope_fp32(k, params["k_norm_weight"], params["k_epsilon"], cos, sin)
        v = v.bfloat16()
        parts = [t.reshape(x.size(0), topo.sp_size, -1) for t in (q, k, v)]
        return torch.cat(parts, dim=-1).transpose(0, 1).contiguous()
    y = project(x, params["qkv_weight"]) if projection is None else projection
    q, k, v = y.split(topo.widths(), dim=-1)
    q = norm_rope(q, params["q_norm_weight"], params["q_epsilon"], cos, sin)
    k = norm_rope(k, params["k_norm_weight"], params["k_epsilon"], cos, sin)
    parts = [t.reshape(x.size(0), topo.sp_size, -1) for t in (q, k, v)]
    return torch.cat(parts, dim=-1).transpose(0, 1).contiguous()


def unpack(topo: Topology, received, tokens):
    """Split the received ``[S, L, N/S]`` buffer into Q, K, V ``[S*L, ...]``
    (torch_base.py:72-76)."""
    output = received.reshape(tokens * topo.sp_size, -1)
    return tuple(
        t.contiguous()
        for t in output.split([w // topo.sp_size for w in topo.widths()], dim=-1)
    )


def simulate_world(topo: Topology, xs, positions, params_by_rank, projections=None,
                   fp32_epilogue=False):
    """Run every rank in one process.

    ``xs[r]``/``positions[r]`` are rank r's inputs; ``params_by_rank[r]`` its
    parameters (the weight is shared inside a base-TP group).  The exchange is
    ``all_to_all_single`` with equal splits inside each SP group of
    ``sp_size`` consecutive ranks: rank ``g+d`` receives block ``d`` of every
    member's send buffer, stacked by source SP rank (torch_base.py:68-71).
    ``projections`` optionally gives each rank's BF16 projection (see
    ``rank_send``).  Returns a list of ``(q, k, v)`` per rank.
    """
    tokens = xs[0].size(0)
    sends = [
        rank_send(topo, xs[r], positions[r], params_by_rank[r],
                  None if projections is None else projections[r], fp32_epilogue)
        for r in range(topo.world_size)
    ]
    outputs = []
    for r in range(topo.world_size):
        start = r // topo.sp_size * topo.sp_size
        dst = r - start
        received = torch.stack(
            [sends[start + src][dst] for src in range(topo.sp_size)], dim=0
        )
        outputs.append(unpack(topo, received, tokens))
    return outputs


def rank_forward_gloo(topo: Topology, x, positions, params, group):
    """The per-rank form over a process group, as torch_base.py:48-76."""
    send = rank_send(topo, x, positions, params)
    received = torch.empty_like(send)
    torch.distributed.all_to_all_single(received, send, group=group)
    return unpack(topo, received, x.size(0))


def inverse_exchange_world(topo: Topology, attn_outs, tokens):
    """Inverse of the forward exchange for Q-shaped tensors: every rank's
    ``[S*L, output_q_heads*128]`` attention output (rows ``s*L..`` belong to
    source ``s``, the layout ``unpack`` returns for Q) goes back to its
    sources.  Returns, per rank, ``[L, local_q_heads*128]`` with member ``d``'s
    heads in columns ``d*cols..`` -- the local head order of the forward's
    projection (reference torch_base.py:68-76 run backwards; the reference
    itself has no inverse step)."""
    S = topo.sp_size
    out = []
    for r in range(topo.world_size):
        start = r // S * S
        src = r - start
        out.append(torch.cat([attn_outs[start + d][src * tokens:(src + 1) * tokens]
                              for d in range(S)], dim=-1))
    return out


def o_proj(gathered, o_weight):
    """``F.linear(gathered, o_weight)`` with FP32 accumulation and one BF16
    rounding (``o_weight`` is ``[H, local_q_heads*128]``, nn.Linear layout)."""
    return (gathered.float() @ o_weight.float().t()).bfloat16()


def o_proj_world(topo: Topology, attn_outs, o_weights, tokens):
    """Inverse exchange then output projection for every rank of a world."""
    gathered = inverse_exchange_world(topo, attn_outs, tokens)
    return [o_proj(g, o_weights[r]) for r, g in enumerate(gathered)]


def rank_o_proj_gloo(topo: Topology, attn_out, o_weight, tokens, group):
    """Per-rank form over a process group: ``all_to_all_single`` sends block
    ``s`` of the attention output (source ``s``'s rows) to member ``s``."""
    send = attn_out.reshape(topo.sp_size, tokens, -1).contiguous()
    received = torch.empty_like(send)
    torch.distributed.all_to_all_single(received, send, group=group)
    return o_proj(torch.cat(list(received), dim=-1), o_weight)


def placement(topo: Topology, rank: int):
    """Where each local packed head of ``rank`` lands after the exchange.

    Returns a list, indexed by local packed head, of
    ``(component, dst_rank, dst_head_column)`` following the reference's
    mapping (the reference's DESIGN.md:28-37, flash_ulysses_kernel_hopper.cu:211-218).
    """
    start = rank // topo.sp_size * topo.sp_size
    out = []
    for h in range(topo.local_q_heads + 2 * topo.local_kv_heads):
        if h < topo.local_q_heads:
            comp, head, per_gpu = 0, h, topo.output_q_heads
        elif h < topo.local_q_heads + topo.local_kv_heads:
            comp, head, per_gpu = 1, h - topo.local_q_heads, topo.output_kv_heads
        else:
            comp = 2
            head = h - topo.local_q_heads - topo.local_kv_heads
            per_gpu = topo.output_kv_heads
        out.append((comp, start + head // per_gpu, head % per_gpu))
    return out
