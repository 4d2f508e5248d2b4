"""Size-independent properties of the oracle's exchange, on random topologies
(CPU, hypothesis): the head placement covers every receive column of every SP
member exactly once; the inverse exchange undoes the forward exchange; the
output projection is linear in the attention output."""

import torch
from hypothesis import given, settings, strategies as st

from oracle import ulysses_oracle as oracle

H = oracle.HEAD_DIM


@st.composite
def topologies(draw):
    sp = draw(st.sampled_from([1, 2, 4, 8]))
    tp = draw(st.sampled_from([1, 2])) if sp <= 4 else 1
    world = sp * tp
    kv = world * draw(st.integers(1, 2))
    heads = kv * draw(st.sampled_from([1, 2, 4]))
    tokens = draw(st.integers(1, 9))
    return oracle.Topology(world, sp, heads, kv, 128), tokens


@settings(max_examples=40, deadline=None)
@given(topologies())
def test_placement_is_a_bijection_onto_receive_columns(case):
    topo, _ = case
    for start in range(0, topo.world_size, topo.sp_size):
        seen = {}
        for src in range(start, start + topo.sp_size):
            for comp, dst, col in oracle.placement(topo, src):
                assert start <= dst < start + topo.sp_size
                key = (comp, dst, col)
                seen[key] = seen.get(key, 0) + 1
        per = (topo.output_q_heads, topo.output_kv_heads, topo.output_kv_heads)
        # Every (component, member, column) receives from every source exactly once.
        for comp in range(3):
            for dst in range(start, start + topo.sp_size):
                for col in range(per[comp]):
                    assert seen.get((comp, dst, col)) == topo.sp_size


@settings(max_examples=40, deadline=None)
@given(topologies(), st.integers(0, 2**31 - 1))
def test_exchange_then_inverse_is_identity(case, seed):
    topo, tokens = case
    g = torch.Generator().manual_seed(seed)
    # Arbitrary per-rank "sent" Q blocks: rank r's Q heads over its own tokens.
    own_q = [torch.randn(tokens, topo.local_q_heads * H, generator=g).bfloat16()
             for _ in range(topo.world_size)]
    # Forward exchange of Q alone, as the reference lays it out: member d of an SP
    # group receives columns [d*cols, (d+1)*cols) of every source's Q, stacked by
    # source (torch_base.py:68-76).
    cols = topo.output_q_heads * H
    recv = []
    for r in range(topo.world_size):
        start = r // topo.sp_size * topo.sp_size
        d = r - start
        recv.append(torch.cat([own_q[start + s][:, d * cols:(d + 1) * cols]
                               for s in range(topo.sp_size)], dim=0))
    back = oracle.inverse_exchange_world(topo, recv, tokens)
    for r in range(topo.world_size):
        assert torch.equal(back[r], own_q[r])


@settings(max_examples=25, deadline=None)
@given(topologies(), st.integers(0, 2**31 - 1))
def test_o_proj_is_linear_in_the_attention_output(case, seed):
    """o_proj_world(a + b) equals o_proj_world(a) + o_proj_world(b) wherever
    integer-valued inputs keep all three results exact in BF16."""
    topo, tokens = case
    g = torch.Generator().manual_seed(seed)
    cols = topo.output_q_heads * H
    a = [torch.randint(-1, 2, (topo.sp_size * tokens, cols), generator=g).bfloat16()
         for _ in range(topo.world_size)]
    b = [torch.randint(-1, 2, (topo.sp_size * tokens, cols), generator=g).bfloat16()
         for _ in range(topo.world_size)]
    w = [torch.randint(-1, 2, (256, topo.local_q_heads * H), generator=g).bfloat16()
         for _ in range(topo.world_size)]
    ab = [x + y for x, y in zip(a, b)]
    left = oracle.o_proj_world(topo, ab, w, tokens)
    ra = oracle.o_proj_world(topo, a, w, tokens)
    rb = oracle.o_proj_world(topo, b, w, tokens)
    for r in range(topo.world_size):
        # Integer sums are exact in FP32 and BF16 holds every integer below 256,
        # while any sum of 256 or more rounds to 256 or more: compare where all
        # three results are below 256 in magnitude.
        la, lb, lab = ra[r].float(), rb[r].float(), left[r].float()
        exact = (la.abs() < 256) & (lb.abs() < 256) & (lab.abs() < 256)
        assert exact.float().mean() > 0.2
        assert torch.equal(lab[exact], (la + lb)[exact])
