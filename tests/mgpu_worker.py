"""Multi-GPU worker for tests/test_gpu_multi.py (one process per GPU, launched
with torch.distributed.run).

For every case it builds a FlashUlyssesContext over real CUDA IPC mappings and
checks this rank's outputs against the reference's PyTorch path run on the
GPUs (oracle restatement on CUDA tensors + NCCL all_to_all_single inside the
SP group, tests/torch_base.py:48-76) and, for small cases, against the CPU
oracle.  Placement, padding and untouched capacity are checked bit for bit on
exact inputs.  Then back-to-back calls without a host rendezvous, and finally
a host-side fault: one rank skips a call and its peers' bounded wait must
report it.
"""

from __future__ import annotations

import datetime
import os
import sys
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from flash_ulysses_b200 import FlashUlyssesContext  # noqa: E402
from flash_ulysses_b200.workloads import Config, make_world  # noqa: E402
from oracle import ulysses_oracle as oracle  # noqa: E402

ATOL = RTOL = 0.01


def log(msg):
    if dist.get_rank() == 0:
        print(msg, flush=True)


def sp_groups(world, sp, backend):
    mine = None
    for start in range(0, world, sp):
        g = dist.new_group(list(range(start, start + sp)), backend=backend)
        if start <= dist.get_rank() < start + sp:
            mine = g
    return mine


def reference_gpu(topo, x, pos, params, group):
    """The reference's PyTorch path on this GPU (cuBLAS + NCCL)."""
    send = oracle.rank_send(topo, x, pos, params)
    if topo.sp_size == 1:
        return oracle.unpack(topo, send, x.size(0))
    received = torch.empty_like(send)
    dist.all_to_all_single(received, send, group=group)
    return oracle.unpack(topo, received, x.size(0))


def projection_excess(dump, ref):
    """Elements of ``dump`` farther from ``ref`` than one BF16 ulp + 1e-4."""
    a, b = dump.float(), ref.float()
    bound = torch.maximum(a.abs(), b.abs()) * 2.0 ** -7 + 1e-4
    return int(((a - b).abs() > bound).sum())


def reference_gpu_from_projection(topo, x, pos, params, proj, group):
    """The reference's epilogue and NCCL exchange applied to a given BF16
    projection (this rank's)."""
    send = oracle.rank_send(topo, x, pos, params, projection=proj)
    if topo.sp_size == 1:
        return oracle.unpack(topo, send, x.size(0))
    received = torch.empty_like(send)
    dist.all_to_all_single(received, send, group=group)
    return oracle.unpack(topo, received, x.size(0))


def run_case(cfg, tokens_list, gloo, *, cpu_check_max=256):
    rank, world = dist.get_rank(), dist.get_world_size()
    topo = oracle.Topology(cfg.world_size, cfg.sp_size, cfg.num_heads, cfg.num_kv_heads,
                           cfg.hidden_size)
    nccl_sp = sp_groups(world, cfg.sp_size, "nccl")
    ctx = FlashUlyssesContext(rank=rank, world_size=world, max_local_tokens=max(tokens_list) + 5,
                              hidden_size=cfg.hidden_size, num_heads=cfg.num_heads,
                              num_kv_heads=cfg.num_kv_heads, sp_size=cfg.sp_size,
                              control_group=gloo, timeout_s=10.0)
    failures = []
    try:
        for tokens in tokens_list:
            xs, pos, params = make_world(cfg, tokens, seed=tokens)
            dev = torch.device("cuda", torch.cuda.current_device())
            gp = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in params[rank].items()}
            x, p = xs[rank].to(dev), pos[rank].to(dev)
            for t in (ctx.Q, ctx.K, ctx.V):
                t.data_.fill_(float("nan"))
            proj = torch.empty(tokens, topo.packed_width, dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize()
            dist.barrier(group=gloo)
            got = ctx.ulysses_qkv_forward(x, gp["qkv_weight"], p, gp["q_norm_weight"],
                                          gp["k_norm_weight"], gp["rope_cache"],
                                          q_epsilon=gp["q_epsilon"], k_epsilon=gp["k_epsilon"],
                                          _projection_out=proj)
            ctx.check()
            # (1) our projection within one BF16 ulp (or 1e-4) of x @ W (cuBLAS);
            n_proj = projection_excess(proj, oracle.project(x, gp["qkv_weight"]))
            if n_proj:
                failures.append(f"{cfg.name} L={tokens}: projection off in {n_proj} elements")
            # (2) the reference's epilogue + NCCL exchange on our projection: at most
            #     1e-7 of the elements (the FP32 sum of a head's 128 squares is
            #     reduced in another order than torch's, which very rarely moves a
            #     value across a BF16 rounding boundary -- the criterion of
            #     tests/benchmark.py);
            exact = reference_gpu_from_projection(topo, x, p, gp, proj, nccl_sp)
            # (3) the full reference path: rare one-ulp projection flips only.
            want = reference_gpu(topo, x, p, gp, nccl_sp)
            stats = []
            total_bad = 0
            for g, e, w, name in zip(got, exact, want, "QKV"):
                bad2 = int((~torch.isclose(g.float(), e.float(), atol=ATOL, rtol=RTOL)).sum())
                if bad2 > int(1e-7 * g.numel()):
                    failures.append(f"{cfg.name} L={tokens} {name}: {bad2} violations vs the "
                                    "reference epilogue on our projection")
                bad = int((~torch.isclose(g.float(), w.float(), atol=ATOL, rtol=RTOL)).sum())
                err = float((g.float() - w.float()).abs().max())
                total_bad += bad
                stats.append(f"{name} viol {bad} max {err:.3g}")
                if bad and err > 0.0625:
                    failures.append(f"{cfg.name} L={tokens} {name}: max err {err}")
            numel = sum(g.numel() for g in got)
            if total_bad > max(4, 1e-5 * numel):
                failures.append(f"{cfg.name} L={tokens}: {total_bad} violations vs GPU reference")
            if tokens <= cpu_check_max:
                # Against the CPU oracle, the kernel may be no further off than the
                # reference's own GPU path is (both differ from the CPU only by the
                # FP32 accumulation order of the projection).
                cpu = oracle.simulate_world(topo, xs, pos, params)[rank]
                for g, w, ref, name in zip(got, cpu, want, "QKV"):
                    bad = int((~torch.isclose(g.float().cpu(), w.float(), atol=ATOL,
                                              rtol=RTOL)).sum())
                    ref_bad = int((~torch.isclose(ref.float().cpu(), w.float(), atol=ATOL,
                                                  rtol=RTOL)).sum())
                    stats.append(f"{name} vs CPU {bad} (GPU ref vs CPU {ref_bad})")
                    if bad > ref_bad + max(1, 2e-6 * g.numel()):
                        failures.append(f"{cfg.name} L={tokens} {name}: {bad} vs CPU oracle "
                                        f"(reference GPU path: {ref_bad})")
            rows = tokens * cfg.sp_size
            for t, name in zip((ctx.Q, ctx.K, ctx.V), "QKV"):
                if not bool(torch.isnan(t.data_[rows:].float()).all()):
                    failures.append(f"{cfg.name} L={tokens} {name}: capacity written")
            log(f"  {cfg.name} P={world} S={cfg.sp_size} L={tokens}: " + ", ".join(stats))

        # Back-to-back calls without host rendezvous; the last one is checked.
        tokens = tokens_list[-1]
        xs, pos, params = make_world(cfg, tokens, seed=99)
        gp = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in params[rank].items()}
        x, p = xs[rank].cuda(), pos[rank].cuda()
        dist.barrier(group=gloo)
        for _ in range(20):
            got = ctx.ulysses_qkv_forward(x, gp["qkv_weight"], p, gp["q_norm_weight"],
                                          gp["k_norm_weight"], gp["rope_cache"],
                                          q_epsilon=gp["q_epsilon"], k_epsilon=gp["k_epsilon"])
        ctx.check()
        want = reference_gpu(topo, x, p, gp, nccl_sp)
        for g, w, name in zip(got, want, "QKV"):
            bad = int((~torch.isclose(g.float(), w.float(), atol=ATOL, rtol=RTOL)).sum())
            if bad > max(1, 2e-6 * g.numel()):
                failures.append(f"{cfg.name} back-to-back {name}: {bad} violations")
    finally:
        dist.barrier(group=gloo)
        ctx.close()
    return failures


def graph_replay_case(gloo):
    """Each rank captures calls in a CUDA graph and replays them with no host
    rendezvous in between: device-side epochs and the entry barrier keep the
    ranks in step and keep a fast rank from overwriting data a slow rank's
    stream has not reached."""
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Config("graph", world, world, 4096, 32, 8, (257,), 32768)
    topo = oracle.Topology(world, world, 32, 8, 4096)
    nccl_sp = sp_groups(world, world, "nccl")
    ctx = FlashUlyssesContext(rank=rank, world_size=world, max_local_tokens=257,
                              hidden_size=4096, num_heads=32, num_kv_heads=8, sp_size=world,
                              control_group=gloo, timeout_s=10.0)
    failures = []
    try:
        xs, pos, params = make_world(cfg, 257, seed=11)
        gp = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in params[rank].items()}
        x, p = xs[rank].cuda(), pos[rank].cuda()
        want = reference_gpu(topo, x, p, gp, nccl_sp)
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        ctx.ulysses_qkv_forward(x, gp["qkv_weight"], p, gp["q_norm_weight"],
                                gp["k_norm_weight"], gp["rope_cache"])
        ctx.check()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
            for _ in range(4):
                got = ctx.ulysses_qkv_forward(x, gp["qkv_weight"], p, gp["q_norm_weight"],
                                              gp["k_norm_weight"], gp["rope_cache"])
        torch.cuda.current_stream().wait_stream(s)
        dist.barrier(group=gloo)
        for _ in range(6):
            graph.replay()                     # no rendezvous between replays
        ctx.check()
        epoch = int(ctx.barrier.data_[33].item())
        if epoch != 1 + 4 * 6:
            failures.append(f"rank {rank}: device epoch {epoch}, expected 25")
        for g, w, name in zip(got, want, "QKV"):
            bad = int((~torch.isclose(g.float(), w.float(), atol=ATOL, rtol=RTOL)).sum())
            if bad > max(1, 2e-6 * g.numel()):
                failures.append(f"graph replay {name}: {bad} violations")
        log(f"  CUDA graph replay x6 (4 calls each, no rendezvous): "
            f"{'ok' if not failures else failures}")
        del graph
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        ctx.close()
    return failures


def exact_placement_case(world, sp, gloo):
    """Bit-exact placement/padding/capacity on exact inputs over real peer memory."""
    from test_gpu_kernel import exact_world

    rank = dist.get_rank()
    T = world // sp
    q_local, kv_local, H, tokens = 4 * sp, 2 * sp, 256, 67
    xs, pos, params = exact_world(sp, H, q_local, kv_local, tokens)
    topo = oracle.Topology(sp, sp, q_local, kv_local, H)
    want = oracle.simulate_world(topo, xs, pos, params)
    ctx = FlashUlyssesContext(rank=rank, world_size=world, max_local_tokens=tokens + 9,
                              hidden_size=H, num_heads=q_local * T, num_kv_heads=kv_local * T,
                              sp_size=sp, control_group=gloo)
    failures = []
    try:
        for t in (ctx.Q, ctx.K, ctx.V):
            t.data_.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        r = rank % sp
        gp = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in params[r].items()}
        ctx.ulysses_qkv_forward(xs[r].cuda(), gp["qkv_weight"], pos[r].cuda(),
                                gp["q_norm_weight"], gp["k_norm_weight"], gp["rope_cache"],
                                q_epsilon=gp["q_epsilon"], k_epsilon=gp["k_epsilon"])
        ctx.check()
        rows = tokens * sp
        for c, t in enumerate((ctx.Q, ctx.K, ctx.V)):
            full = t.data_.cpu()
            if not torch.equal(full[:rows].view(torch.int16), want[r][c].view(torch.int16)):
                failures.append(f"exact P={world} S={sp}: component {c} differs")
            if not bool(torch.isnan(full[rows:].float()).all()):
                failures.append(f"exact P={world} S={sp}: capacity written")
        log(f"  exact placement P={world} S={sp}: {'ok' if not failures else failures}")
    finally:
        dist.barrier(group=gloo)
        ctx.close()
    return failures


def oproj_case(world, sp, gloo):
    """Inverse exchange + output projection over real peer memory: calls of
    several lengths back to back (no host rendezvous in between) and a CUDA
    graph replayed without rendezvous, against an NCCL all_to_all of the
    attention-output blocks followed by the FP32-accumulated projection."""
    rank = dist.get_rank()
    T = world // sp
    H, heads = 4096, 32
    topo = oracle.Topology(world, sp, heads, 8, H)
    cols = topo.output_q_heads * oracle.HEAD_DIM
    nccl_sp = sp_groups(world, sp, "nccl")
    ctx = FlashUlyssesContext(rank=rank, world_size=world, max_local_tokens=4096,
                              hidden_size=H, num_heads=heads, num_kv_heads=8, sp_size=sp,
                              control_group=gloo, timeout_s=10.0, output_projection=True)
    failures = []

    def reference(attn, w, L):
        send = attn.reshape(sp, L, cols).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=nccl_sp)
        return oracle.o_proj(torch.cat(list(recv), dim=-1), w)

    try:
        g = torch.Generator(device="cuda").manual_seed(100 + rank // sp)
        w = (torch.randn(H, topo.local_q_heads * oracle.HEAD_DIM, device="cuda", generator=g)
             * (topo.local_q_heads * oracle.HEAD_DIM) ** -0.5).bfloat16()
        gx = torch.Generator(device="cuda").manual_seed(200 + rank)
        lengths = (1, 129, 1024, 4096)
        attns = [torch.randn(sp * L, cols, device="cuda", generator=gx).bfloat16()
                 for L in lengths]
        wants = [reference(a, w, L) for a, L in zip(attns, lengths)]
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        outs = [ctx.ulysses_o_proj_forward(a, w) for a in attns]     # back to back
        ctx.check()
        for L, o, want in zip(lengths, outs, wants):
            bad = int((~torch.isclose(o.float(), want.float(), atol=ATOL, rtol=RTOL)).sum())
            if bad:
                failures.append(f"o_proj P={world} S={sp} L={L}: {bad} violations")
        # CUDA graph of two calls, replayed without rendezvous.
        a, L = attns[2], lengths[2]
        out = torch.empty(L, H, dtype=torch.bfloat16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
            for _ in range(2):
                ctx.ulysses_o_proj_forward(a, w, out=out)
        torch.cuda.current_stream().wait_stream(s)
        dist.barrier(group=gloo)
        for _ in range(5):
            graph.replay()
        ctx.check()
        bad = int((~torch.isclose(out.float(), wants[2].float(), atol=ATOL, rtol=RTOL)).sum())
        if bad:
            failures.append(f"o_proj graph replay P={world} S={sp}: {bad} violations")
        epoch = int(ctx.o_barrier.data_[33].item())
        if epoch != len(lengths) + 10:
            failures.append(f"rank {rank}: o_proj epoch {epoch}, expected {len(lengths) + 10}")
        if bool((ctx.o_barrier.data_[64:] != 0).any()):
            failures.append(f"rank {rank}: ready counters not reset")
        log(f"  o_proj P={world} S={sp} (L {lengths}, back to back, graph x5): "
            f"{'ok' if not failures else failures}")
        del graph
    finally:
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        ctx.close()
    return failures


def fault_case(gloo):
    """A rank that never joins a call: the others' bounded wait reports it and
    the host raises, without hanging or faulting the GPU."""
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = Config("fault", world, world, 1024, 8 * world, 2 * world, (16,), 4096)
    ctx = FlashUlyssesContext(rank=rank, world_size=world, max_local_tokens=16,
                              hidden_size=1024, num_heads=8 * world, num_kv_heads=2 * world,
                              sp_size=world, control_group=gloo, timeout_s=0.2)
    failures = []
    try:
        xs, pos, params = make_world(cfg, 16, seed=5)
        gp = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in params[rank].items()}
        dist.barrier(group=gloo)
        if rank != world - 1:          # the last rank skips this call
            ctx.ulysses_qkv_forward(xs[rank].cuda(), gp["qkv_weight"], pos[rank].cuda(),
                                    gp["q_norm_weight"], gp["k_norm_weight"], gp["rope_cache"])
            try:
                ctx.check()
                failures.append(f"rank {rank}: missing peer not detected")
            except RuntimeError as e:
                if "peer flag wait timed out" not in str(e):
                    failures.append(f"rank {rank}: unexpected error {e}")
        log(f"  fault injection (rank {world - 1} skips a call): "
            f"{'detected' if not failures else failures}")
    finally:
        dist.barrier(group=gloo)
        ctx.close()
    return failures


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=120))
    gloo = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    world = dist.get_world_size()
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    base = (4096, 32, 8)
    cases = [Config(f"P{world}S{world}", world, world, *base, (1, 65, 129, 1024), 32768)]
    if world >= 4:
        cases.append(Config(f"P{world}S{world // 2}", world, world // 2, *base, (1, 129, 512),
                            32768))
    if world == 8:
        cases.append(Config("c3", 8, 4, 4096, 32, 8, (1, 16, 64, 129, 512), 32768))
        cases.append(Config("c4", 8, 8, 5120, 64, 8, (8192,), 131072))
    failures = []
    try:
        for cfg in cases:
            failures += run_case(cfg, list(cfg.tokens), gloo)
        failures += graph_replay_case(gloo)
        failures += exact_placement_case(world, world, gloo)
        if world >= 4:
            failures += exact_placement_case(world, world // 2, gloo)
        failures += oproj_case(world, world, gloo)
        if world >= 4:
            failures += oproj_case(world, world // 2, gloo)
        failures += fault_case(gloo)
    except Exception:
        failures.append(f"rank {dist.get_rank()}: " + traceback.format_exc())
    flag = torch.tensor([len(failures)], device="cuda")
    dist.all_reduce(flag)
    if failures:
        print(f"rank {dist.get_rank()} FAILURES: {failures}", flush=True)
    log(f"MULTI-GPU RESULT world={world}: {'PASS' if int(flag.item()) == 0 else 'FAIL'}")
    dist.destroy_process_group(gloo)
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 0 else 1)


if __name__ == "__main__":
    main()
