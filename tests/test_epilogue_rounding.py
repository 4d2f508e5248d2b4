"""The epilogue's FP32 arithmetic, restated on the CPU, against torch's CPU
operators that the oracle (and the reference's PyTorch path) use.

The kernel's RMSNorm must produce torch's ``value.square().mean(-1)`` and
``torch.rsqrt`` bit for bit, so that its outputs equal the oracle's epilogue
exactly whenever the BF16 projections agree.  Here the two summation orders of
``fu_qkv.cu`` (a thread owning a whole 128-column head row in ``emit_head``,
and 32 lanes owning 4 columns each in ``split_item_emit``) and its
``norm_scale`` are written out step by step in float32 numpy (IEEE
round-to-nearest, like the device's ``__fadd_rn`` / ``__fmul_rn``) and
compared with torch on many random head rows.
"""

import numpy as np
import pytest
import torch


def rows(n, seed, scale=1.3):
    g = torch.Generator().manual_seed(seed)
    v = (torch.randn(n, 128, generator=g) * scale).bfloat16().float()
    # A few rows of tiny and of mixed magnitudes.
    v[: n // 16] *= torch.exp2(torch.randint(-40, 8, (n // 16, 1), generator=g).float())
    v[n // 16: n // 8] *= torch.exp2(torch.randint(-12, 12, (n // 16, 128), generator=g).float())
    return v.bfloat16().float()


def thread_order_sum(v):
    """emit_head: lane[l] = sum over k of (sum over c of sq[32c + 8k + l]), then
    the eight lanes left to right."""
    sq = (v * v).astype(np.float32)
    lane = None
    for k in range(4):
        acc = None
        for c in range(4):
            col = sq[:, 32 * c + 8 * k: 32 * c + 8 * k + 8]
            acc = col.copy() if acc is None else (acc + col).astype(np.float32)
        lane = acc if lane is None else (lane + acc).astype(np.float32)
    ss = lane[:, 0].copy()
    for l in range(1, 8):
        ss = (ss + lane[:, l]).astype(np.float32)
    return ss


def warp_order_sum(v):
    """split_item_emit: lane t holds columns 4t..4t+3; shuffles down by 8, 16,
    24 from the squares, then by 2, 4, 6 from those sums, then lane 1's four
    values after lane 0's."""
    n = v.shape[0]
    sq = (v * v).astype(np.float32).reshape(n, 32, 4)        # [row, lane, e]

    def shfl_down(x, d):
        out = x.copy()
        out[:, : 32 - d] = x[:, d:]
        return out

    acc = sq.copy()
    for step in (8, 16, 24):
        acc = (acc + shfl_down(sq, step)).astype(np.float32)
    a = acc.copy()
    for k in (2, 4, 6):
        a = (a + shfl_down(acc, k)).astype(np.float32)
    hi = shfl_down(a, 1)
    ss = a[:, 0, 0].copy()
    for e in range(1, 4):
        ss = (ss + a[:, 0, e]).astype(np.float32)
    for e in range(4):
        ss = (ss + hi[:, 0, e]).astype(np.float32)
    return ss


def norm_scale(ss, eps):
    """1 / sqrt(sum / 128 + eps) with a correctly rounded square root and a
    correctly rounded reciprocal."""
    mean = (ss * np.float32(1 / 128)).astype(np.float32)
    x = (mean + np.float32(eps)).astype(np.float32)
    return (np.float32(1) / np.sqrt(x)).astype(np.float32)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_sum_of_squares_orders_match_torch(seed):
    v = rows(40000, seed)
    want = v.square().mean(dim=-1).numpy()
    vn = v.numpy()
    got_thread = (thread_order_sum(vn) * np.float32(1 / 128)).astype(np.float32)
    got_warp = (warp_order_sum(vn) * np.float32(1 / 128)).astype(np.float32)
    assert np.array_equal(got_thread.view(np.int32), want.view(np.int32))
    assert np.array_equal(got_warp.view(np.int32), want.view(np.int32))
    # The order matters: a plain left-to-right sum differs on many rows, so
    # the equality above is not a coincidence of exact sums.
    seq = np.zeros(vn.shape[0], np.float32)
    for j in range(128):
        seq = (seq + vn[:, j] * vn[:, j]).astype(np.float32)
    assert (seq / np.float32(128) != want).mean() > 0.05


def test_sum_of_squares_in_the_oracle_layout():
    """The oracle reduces a [L, heads, 128] view; same bits as rows."""
    v = rows(8000, 7)
    want = v.view(-1, 8, 128).square().mean(dim=-1, keepdim=True).reshape(-1).numpy()
    got = (thread_order_sum(v.numpy()) * np.float32(1 / 128)).astype(np.float32)
    assert np.array_equal(got.view(np.int32), want.view(np.int32))


def test_norm_scale_matches_torch_rsqrt():
    v = rows(40000, 3)
    mean = v.square().mean(dim=-1, keepdim=True)
    want = torch.rsqrt(mean + 1e-6).reshape(-1).numpy()
    got = norm_scale(thread_order_sum(v.numpy()), 1e-6)
    assert np.array_equal(got.view(np.int32), want.view(np.int32))
    # torch's rsqrt is not the correctly rounded 1/sqrt on a sizeable share.
    exact = (1 / np.sqrt(mean.reshape(-1).double().numpy() + np.float32(1e-6))).astype(np.float32)
    assert (exact != want).mean() > 0.05
