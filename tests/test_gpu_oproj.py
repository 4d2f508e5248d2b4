"""GPU parity of the inverse exchange fused with the output projection
(``fu_oproj_forward``) against the CPU oracle (``o_proj_world``).

SP groups are emulated on one GPU in two phases (every rank's push, then every
rank's GEMM), since kernels that wait for one another must not run as separate
launches on one GPU; a world of one runs the single fused launch through the
public context API.  Tolerance 0.01/0.01 (the reference's), zero violations;
inputs whose products and sums are exact in FP32 must match bit for bit.
"""

import pytest
import torch

from emulation import EmulatedGroup, EmulatedOprojGroup, isclose_stats, to_device
from flash_ulysses_b200 import _C
from oracle import ulysses_oracle as oracle

pytestmark = pytest.mark.gpu

HEAD = 128


def world_inputs(S, H, q_heads, tokens, seed=0, exact=False):
    g = torch.Generator().manual_seed(seed)
    cols = q_heads // S * HEAD
    K = q_heads * HEAD
    if exact:
        attn = [torch.randint(-2, 3, (S * tokens, cols), generator=g).bfloat16()
                for _ in range(S)]
        w = torch.randint(-2, 3, (H, K), generator=g).bfloat16()
    else:
        attn = [torch.randn(S * tokens, cols, generator=g).bfloat16() for _ in range(S)]
        w = (torch.randn(H, K, generator=g) * K ** -0.5).bfloat16()
    return attn, w


def run_emulated(S, H, q_heads, tokens, attn, w, calls=1, variant=0):
    dev = torch.device("cuda", 0)
    group = EmulatedOprojGroup(sp_size=S, hidden_size=H, q_heads=q_heads,
                               max_local_tokens=tokens + 5)
    try:
        gattn = [a.to(dev) for a in attn]
        gw = [w.to(dev)] * S
        outs = [torch.full((tokens, H), float("nan"), dtype=torch.bfloat16, device=dev)
                for _ in range(S)]
        for _ in range(calls):
            group.run(gattn, gw, outs, tokens, variant=variant)
        torch.cuda.synchronize()
        assert group.status.value == 0, _C.decode_status(group.status.value)
        assert group.counters_reset()
        gathered = [g[:tokens].cpu() for g in group.gather]
        return [o.cpu() for o in outs], gathered
    finally:
        group.close()


@pytest.mark.parametrize("S,H,q_heads,tokens", [
    (1, 4096, 32, 1), (1, 4096, 32, 129), (2, 1024, 8, 300), (4, 2048, 16, 1000),
    (8, 1024, 8, 64), (4, 4096, 32, 1024), (2, 512, 2, 1), (8, 4096, 32, 257),
    (2, 4096, 16, 300), (1, 2048, 16, 8192), (1, 4096, 32, 4096), (2, 4096, 32, 2500),
])
def test_oproj_emulated_groups(S, H, q_heads, tokens):
    """Tile widths 64 (small L), 128 (L=300 at H=4096) and 256 (large L);
    L=4096 and 2500 at H=4096 leave a last round that fills 34 and 12 of the
    74 pairs."""
    attn, w = world_inputs(S, H, q_heads, tokens)
    topo = oracle.Topology(S, S, q_heads, q_heads, H)
    got, gathered = run_emulated(S, H, q_heads, tokens, attn, w)
    want_g = oracle.inverse_exchange_world(topo, attn, tokens)
    want = oracle.o_proj_world(topo, attn, [w] * S, tokens)
    cols = q_heads // S * HEAD
    for r in range(S):
        # Peers' columns are pushed into G; the rank's own are read in place.
        for d in range(S):
            if d != r:
                sl = slice(d * cols, (d + 1) * cols)
                assert torch.equal(gathered[r][:, sl], want_g[r][:, sl]), f"rank {r} from {d}"
        bad, err = isclose_stats(got[r], want[r])
        assert bad == 0, f"rank {r}: {bad} violations, max abs err {err}"


@pytest.mark.parametrize("S,H,q_heads,tokens,variant", [
    (2, 1024, 8, 300, "single"), (2, 1024, 8, 300, "pair"), (1, 4096, 32, 2000, "single"),
    (1, 4096, 32, 2000, "pair"), (4, 2048, 16, 129, "pair"), (1, 512, 4, 1, "pair"),
    (1, 4096, 32, 1200, "single"),
])
def test_oproj_variants(S, H, q_heads, tokens, variant):
    """The single-CTA and the CTA-pair GEMM (odd m-block counts leave the last
    pair's second CTA without rows), tile widths 64 to 256."""
    flag = {"single": _C.FU_FWD_SINGLE, "pair": _C.FU_FWD_PAIR}[variant]
    attn, w = world_inputs(S, H, q_heads, tokens, seed=11)
    topo = oracle.Topology(S, S, q_heads, q_heads, H)
    got, _ = run_emulated(S, H, q_heads, tokens, attn, w, variant=flag)
    want = oracle.o_proj_world(topo, attn, [w] * S, tokens)
    for r in range(S):
        bad, err = isclose_stats(got[r], want[r])
        assert bad == 0, f"rank {r}: {bad} violations, max abs err {err}"


@pytest.mark.parametrize("S,H,q_heads,tokens", [
    (1, 1024, 8, 65), (2, 512, 4, 300), (4, 1024, 8, 130), (8, 2048, 16, 17),
    (1, 1024, 8, 600), (1, 4096, 32, 1200),
])
def test_oproj_bit_exact_on_exact_inputs(S, H, q_heads, tokens):
    """Integer-valued operands: every order of the FP32 sums is exact, so the
    result must equal the oracle's bit for bit."""
    attn, w = world_inputs(S, H, q_heads, tokens, seed=3, exact=True)
    topo = oracle.Topology(S, S, q_heads, q_heads, H)
    got, _ = run_emulated(S, H, q_heads, tokens, attn, w, calls=2)
    want = oracle.o_proj_world(topo, attn, [w] * S, tokens)
    for r in range(S):
        assert torch.equal(got[r], want[r]), f"rank {r}"


@pytest.mark.parametrize("S,q_heads,kv_heads,tokens", [(2, 4, 2, 100), (4, 8, 4, 257)])
def test_forward_then_inverse_is_identity(S, q_heads, kv_heads, tokens):
    """Forward exchange of Q, then the inverse exchange with W_o = I, returns
    every rank's own normalised and rotated Q rows bit for bit."""
    from flash_ulysses_b200.workloads import make_world, CONFIGS
    H = q_heads * HEAD
    base = CONFIGS["c0"]
    cfg = base.__class__("rt", S, S, H, q_heads, kv_heads, tokens, base.max_position)
    xs, pos, params = make_world(cfg, tokens, seed=5)
    dev = torch.device("cuda", 0)
    fwd = EmulatedGroup(sp_size=S, hidden_size=H, q_heads=q_heads, kv_heads=kv_heads,
                        max_local_tokens=tokens)
    try:
        fwd.run([x.to(dev) for x in xs], [p.to(dev) for p in pos],
                [to_device(p, dev) for p in params], flags=_C.FU_FWD_NO_PEER_WAIT)
        torch.cuda.synchronize()
        assert fwd.status.value == 0
        q_out = [o[0].clone() for o in fwd.outputs(tokens)]
    finally:
        fwd.close()
    eye = torch.eye(H, dtype=torch.bfloat16)
    got, _ = run_emulated(S, H, q_heads, tokens, [q.cpu() for q in q_out], eye)
    # The Q part of each rank's own send buffer, before the exchange.
    topo = oracle.Topology(S, S, q_heads, kv_heads, H)
    want = oracle.o_proj_world(topo, [q.cpu() for q in q_out], [eye] * S, tokens)
    for r in range(S):
        assert torch.equal(got[r], want[r])
        send = oracle.rank_send(topo, xs[r], pos[r], params[r])    # [S, L, N/S]
        qc = q_heads // S * HEAD
        own_q = torch.cat([send[d][:, :qc] for d in range(S)], dim=-1)
        bad, _ = isclose_stats(got[r], own_q)
        assert bad <= own_q.numel() * 1e-4


def test_context_world_of_one():
    """The single fused launch (push and GEMM in one kernel) through the public
    API, three calls of different lengths."""
    from flash_ulysses_b200 import FlashUlyssesContext
    H, q_heads = 2048, 16
    ctx = FlashUlyssesContext(rank=0, world_size=1, max_local_tokens=600, hidden_size=H,
                              num_heads=q_heads, num_kv_heads=4, sp_size=1,
                              output_projection=True)
    try:
        topo = oracle.Topology(1, 1, q_heads, 4, H)
        for i, tokens in enumerate((600, 1, 129)):
            attn, w = world_inputs(1, H, q_heads, tokens, seed=10 + i)
            out = ctx.ulysses_o_proj_forward(attn[0].cuda(), w.cuda())
            ctx.check()
            want = oracle.o_proj_world(topo, attn, [w], tokens)[0]
            bad, err = isclose_stats(out, want)
            assert bad == 0, f"L={tokens}: {bad} violations, max abs err {err}"
        block = ctx.o_barrier.data_.cpu()
        assert int(block[_C.FU_SYNC_EPOCH]) == 3
        assert not bool((block[_C.FU_OPROJ_READY:] != 0).any())
    finally:
        ctx.close()


def test_context_requires_output_projection():
    from flash_ulysses_b200 import FlashUlyssesContext
    ctx = FlashUlyssesContext(rank=0, world_size=1, max_local_tokens=8, hidden_size=512,
                              num_heads=4, num_kv_heads=2, sp_size=1)
    try:
        with pytest.raises(RuntimeError, match="output_projection"):
            ctx.ulysses_o_proj_forward(torch.zeros(8, 512, dtype=torch.bfloat16, device="cuda"),
                                       torch.zeros(512, 512, dtype=torch.bfloat16, device="cuda"))
    finally:
        ctx.close()


def test_context_rejects_bad_shapes():
    from flash_ulysses_b200 import FlashUlyssesContext
    ctx = FlashUlyssesContext(rank=0, world_size=1, max_local_tokens=16, hidden_size=512,
                              num_heads=4, num_kv_heads=2, sp_size=1, output_projection=True)
    try:
        bf = dict(dtype=torch.bfloat16, device="cuda")
        attn = torch.zeros(16, 512, **bf)
        w = torch.zeros(512, 512, **bf)
        for a, ww, o in ((torch.zeros(16, 384, **bf), w, None),
                         (attn, torch.zeros(512, 256, **bf), None),
                         (attn.float(), w, None),
                         (attn, w.t(), None),
                         (attn, w, torch.zeros(8, 512, **bf)),
                         (torch.zeros(17, 512, **bf), w, None)):
            with pytest.raises(ValueError):
                ctx.ulysses_o_proj_forward(a, ww, out=o)
        ctx.ulysses_o_proj_forward(attn, w)
        ctx.check()
    finally:
        ctx.close()
