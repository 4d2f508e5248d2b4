"""Benchmark of the fused Ulysses QKV path (one JSON line on rank 0).

Workload: the benchmark configurations' model shape (H=4096, Q/KV heads
32/8, head_dim 128, BF16) with ``world = sp = N`` GPUs (N=4 is configuration
c1, N=8 is configuration c2; N=1 is the one-GPU self-exchange point) and
``--tokens`` tokens per GPU (default 4096).  A step is one
``FlashUlyssesContext.ulysses_qkv_forward`` call; the metric is its device
latency (max over ranks) and the GEMM-equivalent TFLOP/s per GPU.

Launch: ``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 under
``torch.distributed.run`` (one process per GPU).  ``--impl reference`` times
the reference's PyTorch path on the host CPU instead (the oracle port of
tests/torch_base.py:48-76, run as N gloo processes with the real all-to-all;
rank 0 alone runs it and the other ranks exit at once).

Every rank makes the same sequence of calls and collectives, on error paths
too: each call is a collective of the SP group, so a rank that made one call
more than its peers would wait for them until its bounded wait gives up.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused QKV+exchange latency ms (max rank) vs L; GEMM TFLOP/s/GPU vs peak"
# Per-rank model shapes of the benchmark configurations: hidden size, query and
# key/value heads of one base-TP group, RoPE table rows.  c1/c2 (Qwen3-8B-like),
# c3 (the same model at base TP 2: half the heads per rank), c4 (Qwen3-32B-like).
SHAPES = {"c1": (4096, 32, 8, 32768), "c3": (4096, 16, 4, 32768), "c4": (5120, 64, 8, 131072)}
HIDDEN, Q_HEADS, KV_HEADS, MAX_POS = SHAPES["c1"]
ROTATE = 4            # distinct input sets cycled per step: 4 x 82 MB > 126 MB L2
SWEEP = (1, 128, 1024, 4096, 8192)


def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shape", choices=sorted(SHAPES), default="c1",
                    help="per-rank model shape (default c1: H=4096, 32/8 heads)")
    ap.add_argument("--nvlink-capture", action="store_true",
                    help="one process drives an SP group of two on GPUs 0 and 1 without peer "
                         "waits, so that a one-GPU ncu capture of rank 0's launch sees the "
                         "exchange's NVLink traffic (prints one JSON line)")
    args = ap.parse_args()
    global HIDDEN, Q_HEADS, KV_HEADS, MAX_POS
    HIDDEN, Q_HEADS, KV_HEADS, MAX_POS = SHAPES[args.shape]
    return args


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    """(burst bf16 TF/s, sustained bf16 TF/s, HBM GB/s, source)."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return (d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"],
                "measured")
    return 1590.0, 1400.0, 6650.0, "fallback"


NVLINK_GBS = 770.0      # measured peer copy per direction on this pool (900 nominal)

# DRAM bytes (read + write) per launch of the fused kernel at the c1 shape,
# world of one, from ncu captures (dram__bytes_read.sum + dram__bytes_write.sum;
# profiles/fused_qkv_exchange_c1shape.md).  Keyed by tokens per rank.
PROFILED_TRAFFIC = {4096: 141881344.0}
PROFILED_TRAFFIC_SOURCE = "ncu capture, profiles/fused_qkv_exchange_c1shape.md"
# NVLink user-data bytes sent by one launch of rank 0 of an SP group of two at
# L=4096 (ncu nvltx__bytes_data_user.sum; profiles/fused_qkv_exchange_nvlink_sp2_L4096.md):
# the algorithmic exchange volume 2*L*N*(S-1)/S plus two 32-byte flag writes.
PROFILED_NVLINK_SP2 = {4096: 25165888}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


class NvlinkCounter:
    """Cumulative NVLink bytes sent/received by this GPU from NVML field
    values (read-only).  Drivers differ in which fields and scopes they
    support, so several are tried in order; ``source`` names the one in use,
    ``errors`` the NVML return codes of those that failed."""

    ALL_LINKS = 0xFFFFFFFF

    def __init__(self, device_index, links=18):
        self.ok = False
        self.source = None
        self.errors = {}
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        except Exception as e:          # no NVML: report why
            self.errors["nvml"] = f"{type(e).__name__}: {e}"[:120]
            return
        n = pynvml
        tx_rx = [("throughput_data", n.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX,
                  n.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX, 1024),       # KiB counters
                 ("count_bytes", n.NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES,
                  n.NVML_FI_DEV_NVLINK_COUNT_RCV_BYTES, 1)]
        self.variants = []
        for name, tx, rx, unit in tx_rx:
            self.variants.append((f"{name} all-links scope", [(tx, self.ALL_LINKS)],
                                  [(rx, self.ALL_LINKS)], unit))
            self.variants.append((f"{name} summed over links 0..{links - 1}",
                                  [(tx, l) for l in range(links)],
                                  [(rx, l) for l in range(links)], unit))
        for v in self.variants:
            if self._read(v) is not None:
                self.variant, self.source, self.ok = v, v[0], True
                break

    def _read(self, variant):
        name, tx, rx, unit = variant
        try:
            vals = self.nvml.nvmlDeviceGetFieldValues(self.handle, tx + rx)
        except Exception as e:
            self.errors[name] = f"{type(e).__name__}: {e}"[:120]
            return None
        codes = sorted({v.nvmlReturn for v in vals})
        if codes != [0]:
            self.errors[name] = f"nvmlReturn {codes}"
            return None
        total = [0, 0]
        for i, v in enumerate(vals):
            total[0 if i < len(tx) else 1] += v.value.ullVal * unit
        return total

    def read(self):
        return self._read(self.variant) if self.ok else None


# ---------------------------------------------------------------- helpers
def max_over_ranks(value, world):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rendezvous(world, group=None):
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=group)


FAILED = []            # host-side errors of guarded steps (see ``guarded``)


def healthy(ctx, world, group, what):
    """Synchronise, then agree over the control group whether any rank's
    context reported a device-side error (or a call raised on the host);
    every rank raises together, so no rank is left waiting in a collective
    for one that gave up."""
    torch.cuda.synchronize()
    bad = torch.tensor([1 if ctx._status.value or FAILED else 0], dtype=torch.int32)
    if world > 1:
        dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=group)
    if int(bad.item()):
        raise RuntimeError(f"{what}: a rank reported an error (this rank: status "
                           f"0x{ctx._status.value:x}, host {FAILED[:1]})")


def guarded(fn, failed):
    """A step that stops issuing calls after its first host-side error but
    keeps every collective of the timing loop (the error is raised by
    ``healthy`` afterwards, on every rank at once)."""
    def step(i):
        if failed:
            return
        try:
            fn(i)
        except RuntimeError as e:
            failed.append(str(e))
    return step


def make_inputs(world, rank, tokens, seed):
    from flash_ulysses_b200.workloads import make_parameters, make_rank_inputs

    sp = world
    packed = (Q_HEADS + 2 * KV_HEADS) * 128
    params = make_parameters(HIDDEN, packed, MAX_POS, tp_rank=0, seed=seed, device="cuda")
    x, pos = make_rank_inputs(HIDDEN, tokens, MAX_POS, rank=rank, sp_size=sp, seed=seed,
                              device="cuda")
    return x, pos, params


def time_steps(fn, steps, world, group):
    """Device time of ``steps`` back-to-back calls bracketed by a barrier and a
    synchronize on both sides; returns ms per step, max over ranks."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    rendezvous(world, group)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    rendezvous(world, group)
    return max_over_ranks(start.elapsed_time(end) / steps, world)


def time_isolated(fn, steps, world, group):
    """The reference harness's method (tests/common.py:45-59): rendezvous
    before every call, CUDA events around one call, mean, max over ranks."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    total = 0.0
    for i in range(steps):
        rendezvous(world, group)
        start.record()
        fn(i)
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return max_over_ranks(total / steps, world)


def torch_reference_step(x, pos, params, sp, group):
    """The reference's PyTorch path on the GPU (tests/torch_base.py:48-76):
    cuBLAS projection, separate norm/RoPE kernels, NCCL all_to_all."""
    widths = (Q_HEADS * 128, KV_HEADS * 128, KV_HEADS * 128)
    q, k, v = (x @ params["qkv_weight"]).split(widths, dim=-1)
    cos, sin = params["rope_cache"][pos].unsqueeze(1).chunk(2, dim=-1)

    def norm_rope(t, gamma, eps):
        value = t.reshape(x.size(0), -1, 128).float()
        value = value * torch.rsqrt(value.square().mean(dim=-1, keepdim=True) + eps)
        value = (value * gamma).bfloat16().float()
        lo, hi = value.chunk(2, dim=-1)
        return torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1).bfloat16().flatten(1)

    q = norm_rope(q, params["q_norm_weight"], params["q_epsilon"])
    k = norm_rope(k, params["k_norm_weight"], params["k_epsilon"])
    parts = [t.reshape(x.size(0), sp, -1) for t in (q, k, v)]
    send = torch.cat(parts, dim=-1).transpose(0, 1).contiguous()
    if sp == 1:
        return send
    received = torch.empty_like(send)
    dist.all_to_all_single(received, send, group=group)
    return received


# ---------------------------------------------------------------- CPU leg
def _free_port():
    import socket

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _cpu_rank_worker(rank, sp, port, shape, tokens, steps, warmup, budget_s, threads, out):
    """One rank of the reference's PyTorch path on host cores (the oracle port
    of tests/torch_base.py:48-76: projection, norm, RoPE, pack, gloo
    all_to_all_single, unpack).  Runs in a spawned process; rank 0 puts
    (per-step seconds at the sample size, sample tokens) on ``out``."""
    import datetime

    torch.set_num_threads(threads)
    # An explicit store: under torch.distributed.run the inherited environment
    # would otherwise point the rendezvous at the launcher's agent store.
    timeout = datetime.timedelta(seconds=600)
    store = dist.TCPStore("127.0.0.1", port, sp, rank == 0, timeout=timeout)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=sp, timeout=timeout)
    from flash_ulysses_b200.workloads import make_parameters, make_rank_inputs
    from oracle import ulysses_oracle as oracle

    hidden, q_heads, kv_heads, max_pos = SHAPES[shape]
    topo = oracle.Topology(sp, sp, q_heads, kv_heads, hidden)
    params = make_parameters(hidden, topo.packed_width, max_pos, seed=0)

    def timed(x, pos):
        dist.barrier()
        t0 = time.perf_counter()
        oracle.rank_forward_gloo(topo, x, pos, params, None)
        t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)           # max over ranks
        return float(t.item())

    # Bounded sample: halve the tokens per rank until the whole run fits the budget.
    sample = tokens
    while True:
        x, pos = make_rank_inputs(hidden, sample, max_pos, rank=rank, sp_size=sp, seed=0)
        first = timed(x, pos)
        if first * (steps + warmup) <= budget_s or sample <= 128:
            break
        sample //= 2
    for _ in range(max(warmup - 1, 0)):
        timed(x, pos)
    times = [timed(x, pos) for _ in range(steps)]
    if rank == 0:
        out.put((times, sample))
    dist.destroy_process_group()


def cpu_reference_time(tokens, sp, steps, warmup, budget_s, shape):
    """The reference's PyTorch path as ``sp`` gloo processes on this host's
    cores with the real all-to-all.  Returns (ms per step at the full
    workload, sample description, threads in total)."""
    import multiprocessing as mp

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    threads = max(1, (cores or 1) // sp)
    ctx = mp.get_context("spawn")          # never fork a process that may hold a CUDA context
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank_worker,
                         args=(r, sp, port, shape, tokens, steps, warmup, budget_s, threads, out))
             for r in range(sp)]
    for proc in procs:
        proc.start()
    try:
        times, sample = out.get(timeout=budget_s * 3 + 600)
    finally:
        for proc in procs:
            proc.join(timeout=120)
            if proc.is_alive():
                proc.kill()
    per = statistics.mean(times) * tokens / sample * 1e3
    desc = (f"{sp} gloo process(es) x {threads} threads (the reference PyTorch path with "
            f"all_to_all_single), {len(times)} steps of {sample} of {tokens} tokens/rank, "
            f"max over ranks, scaled x{tokens / sample:g}")
    return per, desc, threads * sp


def reference_arm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    tokens, sp = args.tokens, max(args.gpus, world)
    per, desc, cores = cpu_reference_time(tokens, sp, args.steps, args.warmup, 120.0,
                                          args.shape)
    flops = 2 * tokens * HIDDEN * (Q_HEADS + 2 * KV_HEADS) * 128
    line = {
        "metric": METRIC, "value": round(per, 4), "unit": "ms", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args.gpus, tokens),
        "tflops_per_gpu": round(flops / (per * 1e-3) / 1e12, 3),
        "cpu_baseline": {"value": round(per, 4), "unit": "ms", "cores": cores,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(per, 4), "unit": "ms", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(n, tokens):
    return {
        "workload": f"H={HIDDEN} Q/KV={Q_HEADS}/{KV_HEADS} (per base-TP group) head_dim=128, "
                    f"world=sp={n} (default c1 shape; N=4 is c1, N=8 is c2), L={tokens} tokens/GPU",
        "hidden_size": HIDDEN, "num_heads": Q_HEADS, "num_kv_heads": KV_HEADS,
        "tokens_per_gpu": tokens, "world_size": n, "sp_size": n, "base_tp": 1,
        "global_tokens": tokens * n,
        "l2": f"{ROTATE} rotating input sets per rank (>{ROTATE * 82} MB) > 126 MB L2",
    }


# ---------------------------------------------------------------- NVLink capture
def nvlink_capture(args):
    """An SP group of two in one process: rank r runs on GPU r and stores its
    peer's heads into the other GPU's receive buffers over NVLink.  Each
    rank's kernel is launched with FU_FWD_NO_PEER_WAIT (the ranks never wait
    for one another, so a profiler may serialise and replay one rank's launch
    on its own); peer access is enabled both ways.  Checks the placement of
    every received row against the oracle's exchange of the kernels' own
    projections, and prints the event-timed launch of rank 0 with the
    algorithmic NVLink bytes it sends."""
    from cuda.bindings import runtime as rt

    from flash_ulysses_b200 import _C
    from oracle import ulysses_oracle as oracle

    if torch.cuda.device_count() < 2:
        raise SystemExit("--nvlink-capture needs two GPUs")
    for d in (0, 1):
        (err,) = rt.cudaSetDevice(d)
        assert err == rt.cudaError_t.cudaSuccess, err
        (err,) = rt.cudaDeviceEnablePeerAccess(1 - d, 0)
        if err not in (rt.cudaError_t.cudaSuccess,
                       rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
            raise SystemExit(f"cudaDeviceEnablePeerAccess({d} -> {1 - d}): {err}")
    S, L = 2, args.tokens
    topo = oracle.Topology(S, S, Q_HEADS, KV_HEADS, HIDDEN)
    widths = [w // S for w in topo.widths()]
    devs = [torch.device("cuda", d) for d in (0, 1)]
    recv = [tuple(torch.full((S * L, w), float("nan"), dtype=torch.bfloat16, device=dev)
                  for w in widths) for dev in devs]
    sync = [torch.zeros(_C.FU_SYNC_WORDS, dtype=torch.int32, device=dev) for dev in devs]
    status = _C.StatusWord()
    ops, inputs, projs = [], [], []
    for r in (0, 1):
        torch.cuda.set_device(r)
        t = _C.Topology()
        t.device, t.sp_size, t.sp_rank = r, S, r
        t.q_heads, t.kv_heads, t.hidden_size, t.capacity_rows = Q_HEADS, KV_HEADS, HIDDEN, S * L
        for d in (0, 1):
            t.q_recv[d], t.k_recv[d], t.v_recv[d] = (b.data_ptr() for b in recv[d])
            t.sync[d] = sync[d].data_ptr()
        t.status, t.status_host = status.device_ptr, status.host_ptr
        ops.append(_C.QkvOp(t))
        inputs.append(make_inputs(S, r, L, seed=0))
        projs.append(torch.empty(L, topo.packed_width, dtype=torch.bfloat16, device=devs[r]))
    events = []
    for i in range(args.warmup + args.steps):
        for r in (0, 1):
            torch.cuda.set_device(r)
            x, pos, p = inputs[r]
            if r == 0 and i >= args.warmup:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            _C.launch(x, p["qkv_weight"], pos, p["q_norm_weight"], p["k_norm_weight"],
                      p["rope_cache"], ops[r], q_epsilon=p["q_epsilon"], k_epsilon=p["k_epsilon"],
                      flags=_C.FU_FWD_NO_PEER_WAIT, gemm_out=projs[r])
            if r == 0 and i >= args.warmup:
                end.record()
                events.append((start, end))
    for d in (0, 1):
        torch.cuda.synchronize(d)
    if status.value:
        raise SystemExit("device status " + _C.decode_status(status.value))
    # Every received row is where the oracle's exchange of these projections puts it.
    cpu = []
    for r in (0, 1):
        x, pos, p = inputs[r]
        cpu.append(({k: (v.cpu() if torch.is_tensor(v) else v) for k, v in p.items()}))
    want = oracle.simulate_world(topo, [inputs[r][0].cpu() for r in (0, 1)],
                                 [inputs[r][1].cpu() for r in (0, 1)], cpu,
                                 projections=[projs[r].cpu() for r in (0, 1)])
    exact = all(torch.equal(recv[d][c].cpu().view(torch.int16), want[d][c].view(torch.int16))
                for d in (0, 1) for c in range(3))
    ms = statistics.median(a.elapsed_time(b) for a, b in events)
    nvl = 2 * L * topo.packed_width * (S - 1) // S
    print(json.dumps({"mode": "nvlink-capture", "tokens_per_rank": L, "sp_size": S,
                      "kernel_ms_rank0": round(ms, 5),
                      "nvlink_bytes_per_launch_algorithmic": nvl,
                      "algorithmic_gbs": round(nvl / (ms * 1e-3) / 1e9, 1),
                      "outputs_bit_exact_vs_oracle_exchange": exact}), flush=True)
    for op in ops:
        op.destroy()
    status.free()
    if not exact:
        raise SystemExit(1)


# ---------------------------------------------------------------- our arm
def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.nvlink_capture:
        nvlink_capture(args)
        return
    world, rank, local = dist_env()
    n = max(world, 1)
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
        group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=180))
    from flash_ulysses_b200 import FlashUlyssesContext

    tokens = args.tokens
    max_tokens = max(tokens, max(SWEEP) if not args.no_sweep else tokens)
    ctx = FlashUlyssesContext(rank=rank, world_size=n, max_local_tokens=max_tokens,
                              hidden_size=HIDDEN, num_heads=Q_HEADS, num_kv_heads=KV_HEADS,
                              sp_size=n, control_group=group, output_projection=True)
    sets = [make_inputs(n, rank, tokens, seed=s) for s in range(ROTATE)]

    failed = FAILED

    def call(i):
        x, pos, p = sets[i % ROTATE]
        return ctx.ulysses_qkv_forward(x, p["qkv_weight"], pos, p["q_norm_weight"],
                                       p["k_norm_weight"], p["rope_cache"],
                                       q_epsilon=p["q_epsilon"], k_epsilon=p["k_epsilon"])

    step = guarded(call, failed)
    for i in range(args.warmup):
        step(i)
    healthy(ctx, n, group, "warm-up")
    # Soak ~0.5 s so the clock record reflects steady load, then time K steps.
    # The number of soak calls is fixed before the soak and equal on every
    # rank (from the max-over-ranks latency of a few timed calls): a loop
    # bounded by each rank's own clock could end after different call counts.
    est_ms = time_steps(step, 5, n, group)
    healthy(ctx, n, group, "calibration")
    soak_calls = int(min(5000, max(50, 500.0 / max(est_ms, 1e-3))))
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    for c0 in range(0, soak_calls, 50):
        for i in range(c0, min(c0 + 50, soak_calls)):
            step(i)
        healthy(ctx, n, group, "soak")
    epoch0 = ctx.epoch
    nvl = NvlinkCounter(torch.cuda.current_device()) if n > 1 else None
    nvl0 = nvl.read() if nvl is not None and nvl.ok else None
    ms = time_steps(step, args.steps, n, group)
    nvl1 = nvl.read() if nvl0 is not None else None
    clocks = sampler.stop()
    launches = ctx.epoch - epoch0
    healthy(ctx, n, group, "timed steps")

    flops = 2 * tokens * HIDDEN * ctx.packed_width
    tflops = flops / (ms * 1e-3) / 1e12
    peak_burst, peak_sust, peak_hbm, peak_src = measured_peaks()
    # The timed region follows a 0.5 s soak under the power cap: the sustained
    # cuBLAS figure is the matching denominator (the burst fraction is reported too).
    peak_tf = peak_sust
    # Exchange: bytes this rank sends to its SP peers per call, and NVLink's share.
    nvl_bytes = 2 * tokens * ctx.packed_width * (n - 1) / n
    t_gemm_us = flops / (peak_tf * 1e12) * 1e6
    t_nvl_us = nvl_bytes / (NVLINK_GBS * 1e9) * 1e6
    nvlink = None
    if n > 1:
        nvlink = {"algorithmic_bytes_per_call": int(nvl_bytes),
                  "algorithmic_gbs": round(nvl_bytes / (ms * 1e-3) / 1e9, 1),
                  "link_gbs_per_direction": NVLINK_GBS,
                  "frac_of_link": round(nvl_bytes / (ms * 1e-3) / 1e9 / NVLINK_GBS, 4)}
        if nvl0 is not None and nvl1 is not None:
            dt = ms * 1e-3 * args.steps
            nvlink["measured_source"] = f"NVML {nvl.source}"
            nvlink["measured_tx_bytes_per_call"] = int((nvl1[0] - nvl0[0]) / args.steps)
            nvlink["measured_rx_bytes_per_call"] = int((nvl1[1] - nvl0[1]) / args.steps)
            nvlink["measured_tx_gbs"] = round((nvl1[0] - nvl0[0]) / dt / 1e9, 1)
            nvlink["measured_rx_gbs"] = round((nvl1[1] - nvl0[1]) / dt / 1e9, 1)
        else:
            nvlink["measured"] = ("unavailable: NVML NVLink byte counters not readable "
                                  f"({nvl.errors if nvl is not None else 'no counter'})")[:400]
        if tokens in PROFILED_NVLINK_SP2 and HIDDEN == 4096 and Q_HEADS == 32:
            nvlink["profiled_sp2"] = {
                "nvltx_user_bytes_per_launch": PROFILED_NVLINK_SP2[tokens],
                "algorithmic_bytes_per_launch": 2 * tokens * ctx.packed_width // 2,
                "source": "ncu capture, profiles/fused_qkv_exchange_nvlink_sp2_L4096.md"}

    # The reference harness's per-call method (rendezvous between calls).
    iso = time_isolated(step, min(args.steps, 20), n, group)
    healthy(ctx, n, group, "isolated calls")

    # e2e: through the public API from pinned host memory, every step's inputs
    # uploaded and its Q/K/V read back inside the timed region.  Uploads run on
    # their own stream into double-buffered inputs and read-backs on another,
    # so step i's read-back overlaps step i+1's upload on the two copy engines.
    # A call's outputs alias its context's receive buffers, so two contexts
    # alternate (step i on context i mod 2): a call waits only for the
    # read-back of the call two steps earlier, and each read-back overlaps the
    # next call's kernel as well.
    ctx_b = FlashUlyssesContext(rank=rank, world_size=n, max_local_tokens=tokens,
                                hidden_size=HIDDEN, num_heads=Q_HEADS, num_kv_heads=KV_HEADS,
                                sp_size=n, control_group=group)
    ctxs = (ctx, ctx_b)
    hx = [s[0].cpu().pin_memory() for s in sets]
    hp = [s[1].cpu().pin_memory() for s in sets]
    dx = [torch.empty_like(sets[0][0]) for _ in range(2)]
    dp = [torch.empty_like(sets[0][1]) for _ in range(2)]
    outs_h = [torch.empty((tokens * n, w), dtype=torch.bfloat16).pin_memory()
              for w in (ctx.output_q_heads * 128, ctx.output_kv_heads * 128,
                        ctx.output_kv_heads * 128)]
    main_stream = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    computed = torch.cuda.Event()
    read_back = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        _, _, p = sets[i % ROTATE]
        up.wait_event(in_free[b])                 # the call of step i-2 consumed dx[b]
        with torch.cuda.stream(up):
            dx[b].copy_(hx[i % ROTATE], non_blocking=True)
            dp[b].copy_(hp[i % ROTATE], non_blocking=True)
        in_ready[b].record(up)
        main_stream.wait_event(in_ready[b])
        main_stream.wait_event(read_back[b])      # outputs alias the receive buffers
        q, k, v = ctxs[b].ulysses_qkv_forward(dx[b], p["qkv_weight"], dp[b],
                                              p["q_norm_weight"], p["k_norm_weight"],
                                              p["rope_cache"], q_epsilon=p["q_epsilon"],
                                              k_epsilon=p["k_epsilon"])
        in_free[b].record(main_stream)
        computed.record(main_stream)
        down.wait_event(computed)
        with torch.cuda.stream(down):
            for h, d in zip(outs_h, (q, k, v)):
                h.copy_(d, non_blocking=True)
        read_back[b].record(down)

    e2e_call = guarded(e2e_step, failed)

    def time_e2e(steps):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        rendezvous(n, group)
        start.record()
        up.wait_stream(main_stream)
        for i in range(steps):
            e2e_call(i)
        for ev in read_back:                      # the last read-backs are inside the region
            main_stream.wait_event(ev)
        end.record()
        rendezvous(n, group)
        return max_over_ranks(start.elapsed_time(end) / steps, n)

    for i in range(2):
        e2e_call(i)
    healthy(ctx, n, group, "e2e warm-up")
    healthy(ctx_b, n, group, "e2e warm-up")
    e2e_ms = time_e2e(args.steps)
    healthy(ctx, n, group, "e2e")
    healthy(ctx_b, n, group, "e2e")
    ctx_b.close()
    h2d = dx[0].numel() * 2 + dp[0].numel() * 8
    d2h = sum(t.numel() * 2 for t in outs_h)

    # The reference's own PyTorch + NCCL path on the same GPUs.
    def torch_step(i):
        x, pos, p = sets[i % ROTATE]
        torch_reference_step(x, pos, p, n, None)

    for i in range(2):
        torch_step(i)
    torch_ms = time_steps(torch_step, min(args.steps, 20), n, group)

    sweep = {}
    if not args.no_sweep:
        for L in SWEEP:
            s_sets = sets if L == tokens else [make_inputs(n, rank, L, seed=s)
                                               for s in range(ROTATE)]

            def s_call(i, s_sets=s_sets, static=False):
                x, pos, p = s_sets[i % ROTATE]
                ctx.ulysses_qkv_forward(x, p["qkv_weight"], pos, p["q_norm_weight"],
                                        p["k_norm_weight"], p["rope_cache"],
                                        q_epsilon=p["q_epsilon"], k_epsilon=p["k_epsilon"],
                                        static_weights=static)

            s_step = guarded(s_call, failed)
            for i in range(3):
                s_step(i)
            # Short calls get more of them, so the first call's start-up (no
            # overlap with a previous kernel) weighs little in the per-call time.
            t = time_steps(s_step, 200 if L <= 128 else 20, n, group)
            healthy(ctx, n, group, f"sweep L={L}")
            f = 2 * L * HIDDEN * ctx.packed_width
            sweep[str(L)] = {"ms": round(t, 5), "tflops_per_gpu": round(f / (t * 1e-3) / 1e12, 1),
                             "grid": ctx._op.last_grid,
                             "weight_read_gbs": round(HIDDEN * ctx.packed_width * 2 / (t * 1e-3)
                                                      / 1e9, 1)}
            if L <= 128:
                # The same calls with static_weights=True (inference: no kernel
                # writes W), whose first weight stages load while the previous
                # call finishes.
                st_step = guarded(lambda i, s_sets=s_sets: s_call(i, s_sets, True), failed)
                for i in range(3):
                    st_step(i)
                ts = time_steps(st_step, 200, n, group)
                healthy(ctx, n, group, f"sweep L={L} static weights")
                sweep[str(L)]["static_weights_ms"] = round(ts, 5)
            del s_sets

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu_baseline:
        per, desc, threads = cpu_reference_time(tokens, 1, 5, 1, 20.0, args.shape)
        cpu = {"value": round(per, 3), "unit": "ms", "cores": threads, "kind": "port",
               "sample": desc}

    # Measured last and fenced off: the headline metric above stands even if
    # this extra measurement fails.
    o_proj_launches = [0]

    def measure_o_proj():
        # The output side (no counterpart in the reference): the inverse exchange
        # fused with the attention output projection, against NCCL all_to_all +
        # cuBLAS on the same GPUs.
        o_cols = ctx.output_q_heads * 128
        o_k = ctx.local_q_heads * 128
        og = torch.Generator(device="cuda").manual_seed(300 + rank)
        o_sets = [(torch.randn(n * tokens, o_cols, device="cuda", generator=og).bfloat16(),
                   (torch.randn(HIDDEN, o_k, device="cuda", generator=og) * o_k ** -0.5).bfloat16())
                  for _ in range(ROTATE)]
        o_out = torch.empty(tokens, HIDDEN, dtype=torch.bfloat16, device="cuda")

        def o_call(i):
            a, w = o_sets[i % ROTATE]
            ctx.ulysses_o_proj_forward(a, w, out=o_out)

        o_step = guarded(o_call, failed)

        def o_torch_step(i):
            a, w = o_sets[i % ROTATE]
            if n > 1:
                recv = torch.empty_like(a)
                dist.all_to_all_single(recv, a)
                a = torch.cat(list(recv.view(n, tokens, o_cols)), dim=-1)
            torch.matmul(a, w.t(), out=o_out)

        for i in range(3):
            o_step(i)
            o_torch_step(i)
        o_launches0 = ctx._oproj.calls
        o_ms = time_steps(o_step, args.steps, n, group)
        o_proj_launches[0] = ctx._oproj.calls - o_launches0
        o_torch_ms = time_steps(o_torch_step, min(args.steps, 20), n, group)
        healthy(ctx, n, group, "o_proj")
        o_flops = 2 * tokens * o_k * HIDDEN
        return {"ms": round(o_ms, 5),
                "tflops_per_gpu": round(o_flops / (o_ms * 1e-3) / 1e12, 1),
                "torch_nccl_cublas_ms": round(o_torch_ms, 5),
                "speedup_vs_torch": round(o_torch_ms / o_ms, 3),
                "nvlink_bytes_per_call": int(2 * tokens * o_k * (n - 1) / n),
                "config": f"attn [{n * tokens}, {o_cols}] -> out [{tokens}, {HIDDEN}], "
                          f"W_o [{HIDDEN}, {o_k}]"}

    try:
        o_proj = measure_o_proj()
    except Exception as e:  # reported in the JSON line instead of aborting it
        o_proj = {"error": f"{type(e).__name__}: {e}"[:300]}

    traffic = PROFILED_TRAFFIC.get(tokens) if HIDDEN == 4096 and Q_HEADS == 32 else None
    traffic_src = PROFILED_TRAFFIC_SOURCE if traffic is not None else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms, 5), "unit": "ms", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, N(0,H^-1/2) "
                                     "weights, random-init; no checkpoint)",
            "config": workload_config(n, tokens),
            "tflops_per_gpu": round(tflops, 1),
            "frac_of_peak_bf16": round(tflops / peak_tf, 4),
            "frac_of_burst_peak_bf16": round(tflops / peak_burst, 4),
            "tokens_per_s_total": round(tokens * n / (ms * 1e-3), 1),
            "latency_ms_isolated": round(iso, 5),
            "torch_gpu_path_ms": round(torch_ms, 5),
            "speedup_vs_torch_gpu_path": round(torch_ms / ms, 3),
            "latency_ms_by_tokens": sweep,
            "roofline": {
                "bound": "tensor" if t_gemm_us >= t_nvl_us else "nvlink",
                "achieved": round(tflops, 1), "peak": peak_tf,
                "unit": "TFLOP/s", "frac": round(tflops / peak_tf, 4),
                "peak_source": f"{peak_src} bf16 sustained (MEASURED_PEAKS.json; "
                               f"burst {peak_burst})",
                "t_gemm_at_peak_us": round(t_gemm_us, 2),
                "t_exchange_at_link_us": round(t_nvl_us, 2),
                "frac_of_roofline_time": round(max(t_gemm_us, t_nvl_us) / (ms * 1e3), 4),
                "traffic": traffic, "traffic_source": traffic_src,
            },
            "nvlink": nvlink,
            "clocks": clocks,
            "e2e": {"value": round(e2e_ms, 5), "unit": "ms", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "method": "public API from pinned host memory; two contexts alternate so "
                              "a call's Q/K/V read-back overlaps the next call"},
            "gpu_launches": launches,
            "o_proj": o_proj,
            "o_proj_gpu_launches": o_proj_launches[0],
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)

    ctx.close()
    if world > 1:
        dist.destroy_process_group(group)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
