"""The allocation-free entry point ``fu_qkv_forward_noalloc``, called through
the C ABI.

It exists for callers that cannot allocate device memory where they call the
operator (a server whose own pool owns all free HBM, a C caller that owns only
the buffers it passes in); its scratch is a static array inside the library.
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process,
where the first call performs the per-device set-up.
"""

import ctypes

import pytest
import torch

from emulation import EmulatedGroup, to_device
from flash_ulysses_b200 import _C
from flash_ulysses_b200.workloads import make_parameters, make_rank_inputs
from oracle import ulysses_oracle as oracle

pytestmark = pytest.mark.gpu

H, QH, KVH = 4096, 32, 8


def existing_entry_point(x, pos, params, tokens):
    """Outputs of the context-based entry point (fu_qkv_forward), world of one,
    pinned to the kernel variant the allocation-free entry point runs (one CTA
    per 128 x 256 tile over the full reduction), and that call's BF16
    projection (test instrumentation)."""
    group = EmulatedGroup(sp_size=1, hidden_size=H, q_heads=QH, kv_heads=KVH,
                          max_local_tokens=tokens)
    try:
        proj = torch.empty(tokens, (QH + 2 * KVH) * 128, dtype=torch.bfloat16, device=x.device)
        group.run([x], [pos], [params], gemm_outs=[proj],
                  flags=_C.FU_FWD_NO_PEER_WAIT | _C.FU_FWD_SPLITS(1) | _C.FU_FWD_SINGLE)
        torch.cuda.synchronize()
        assert group.status.value == 0
        return tuple(t.clone() for t in group.outputs(tokens)[0]), proj
    finally:
        group.close()


def noalloc_call(x, pos, params, outs, status):
    p = params
    rc = _C.lib.fu_qkv_forward_noalloc(
        torch.cuda.current_device(), x.data_ptr(), p["qkv_weight"].data_ptr(), pos.data_ptr(),
        p["q_norm_weight"].data_ptr(), p["k_norm_weight"].data_ptr(), p["rope_cache"].data_ptr(),
        x.size(0), H, QH, KVH, p["rope_cache"].size(0), p["q_epsilon"], p["k_epsilon"],
        outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(), status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _C.last_error()


def test_noalloc_matches_existing_entry_point_on_two_calls():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cases = []
    for seed, tokens in ((11, 300), (12, 65)):
        params = to_device(make_parameters(H, (QH + 2 * KVH) * 128, 32768, seed=seed), dev)
        x, pos = make_rank_inputs(H, tokens, 32768, rank=0, sp_size=1, seed=seed)
        cases.append((x.to(dev), pos.to(dev), params, tokens))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    results = []
    for i, (x, pos, params, tokens) in enumerate(cases):
        outs = [torch.full((tokens, c), float("nan"), dtype=torch.bfloat16, device=dev)
                for c in (QH * 128, KVH * 128, KVH * 128)]
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        noalloc_call(x, pos, params, outs, status)
        torch.cuda.synchronize()
        if i == 1:
            # The second call cannot have allocated device memory.
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        assert int(status.item()) == 0
        results.append([o.clone() for o in outs])
    for (x, pos, params, tokens), got in zip(cases, results):
        want, proj = existing_entry_point(x, pos, params, tokens)
        # Same kernel variant, same inputs: the same bits.
        for g, w, name in zip(got, want, "QKV"):
            assert torch.equal(g.view(torch.int16), w.view(torch.int16)), name
        # And that variant against the CPU oracle: projection within one BF16
        # ulp of x @ W, epilogue bit for bit on that projection.
        cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in params.items()}
        xs, ps = [x.cpu()], [pos.cpu()]
        ref = oracle.project(xs[0], cpu["qkv_weight"]).float()
        a = proj.cpu().float()
        assert bool(((a - ref).abs() <= torch.maximum(a.abs(), ref.abs()) * 2.0 ** -7 + 1e-4)
                    .all())
        topo = oracle.Topology(1, 1, QH, KVH, H)
        exp = oracle.simulate_world(topo, xs, ps, [cpu], projections=[proj.cpu()])[0]
        for g, e, name in zip(got, exp, "QKV"):
            assert torch.equal(g.cpu().view(torch.int16), e.view(torch.int16)), name


def test_noalloc_rejects_oversized_and_bad_arguments():
    torch.cuda.set_device(0)
    rc = _C.lib.fu_qkv_forward_noalloc(0, 16, 16, 16, 16, 16, 16, (1 << 30) + 1, H, QH, KVH,
                                       1, 1e-6, 1e-6, 16, 16, 16, None, None)
    assert rc == _C.FU_ERR_INVALID and "local_tokens" in _C.last_error()
    rc = _C.lib.fu_qkv_forward_noalloc(0, 16, 16, 16, 16, 16, 16, 8, 100, QH, KVH,
                                       1, 1e-6, 1e-6, 16, 16, 16, None, None)
    assert rc == _C.FU_ERR_INVALID and "hidden_size" in _C.last_error()
