"""Test helpers: the ranks of one SP group emulated on a single GPU, driven
through the C ABI.

All "peer" buffers live on the same device, so every rank's kernel is
launched in turn with FU_FWD_NO_PEER_WAIT (kernels that wait on one another
must never run as separate launches on one GPU); the epoch flags each rank
publishes are then checked from the host.
"""

from __future__ import annotations

import torch

from flash_ulysses_b200 import _C

HEAD = 128


class EmulatedGroup:
    def __init__(self, *, sp_size, hidden_size, q_heads, kv_heads, max_local_tokens,
                 device="cuda", timeout_s=2.0):
        """``q_heads``/``kv_heads`` are local (post base-TP) head counts."""
        self.S = sp_size
        self.H = hidden_size
        self.q_heads, self.kv_heads = q_heads, kv_heads
        self.capacity = sp_size * max_local_tokens
        self.device = torch.device(device)
        qc = q_heads // sp_size * HEAD
        kc = kv_heads // sp_size * HEAD
        self.recv = []
        self.sync = []
        for _ in range(sp_size):
            self.recv.append(tuple(
                torch.full((self.capacity, c), float("nan"), dtype=torch.bfloat16,
                           device=self.device) for c in (qc, kc, kc)))
            self.sync.append(torch.zeros(_C.FU_SYNC_WORDS, dtype=torch.int32, device=self.device))
        self.status = _C.StatusWord()
        self.ops = []
        for r in range(sp_size):
            t = _C.Topology()
            t.device = self.device.index or 0
            t.sp_size = sp_size
            t.sp_rank = r
            t.q_heads, t.kv_heads = q_heads, kv_heads
            t.hidden_size = hidden_size
            t.capacity_rows = self.capacity
            for d in range(sp_size):
                t.q_recv[d] = self.recv[d][0].data_ptr()
                t.k_recv[d] = self.recv[d][1].data_ptr()
                t.v_recv[d] = self.recv[d][2].data_ptr()
                t.sync[d] = self.sync[d].data_ptr()
            t.status = self.status.device_ptr
            t.status_host = self.status.host_ptr
            t.timeout_ns = int(timeout_s * 1e9)
            self.ops.append(_C.QkvOp(t))

    def fill_nan(self):
        for bufs in self.recv:
            for b in bufs:
                b.fill_(float("nan"))

    def run(self, xs, positions, params_list, *, gemm_outs=None, flags=_C.FU_FWD_NO_PEER_WAIT,
            ranks=None):
        """Launch the given emulated ranks (default: all) in order."""
        ranks = range(self.S) if ranks is None else ranks
        for r in ranks:
            p = params_list[r]
            _C.launch(xs[r], p["qkv_weight"], positions[r], p["q_norm_weight"],
                      p["k_norm_weight"], p["rope_cache"], self.ops[r],
                      q_epsilon=p["q_epsilon"], k_epsilon=p["k_epsilon"], flags=flags,
                      gemm_out=None if gemm_outs is None else gemm_outs[r])

    def outputs(self, tokens):
        rows = tokens * self.S
        return [tuple(b[:rows] for b in bufs) for bufs in self.recv]

    def flags_ok(self):
        """Every member advanced its epoch to this call's and published it to
        every member (entry and exit flags); completion counters are reset."""
        epoch = self.ops[0].epoch
        for d in range(self.S):
            block = self.sync[d].cpu()
            if int(block[_C.FU_SYNC_EPOCH]) != epoch:
                return False
            if not bool((block[: self.S] == epoch).all()):
                return False
            if self.S > 1 and not bool(
                    (block[_C.FU_SYNC_ENTRY: _C.FU_SYNC_ENTRY + self.S] == epoch).all()):
                return False
            if int(block[_C.FU_SYNC_COUNTER]) != 0:
                return False
        return True

    def close(self):
        for op in self.ops:
            op.destroy()
        self.status.free()


class EmulatedOprojGroup:
    """The inverse exchange + output projection for the ranks of one SP group
    on one GPU.  A real group runs one launch per rank; here the ranks' kernels
    must not wait for one another, so each call runs in two phases: every
    rank's push (FU_OPROJ_GATHER_ONLY), then every rank's GEMM
    (FU_OPROJ_GEMM_ONLY)."""

    def __init__(self, *, sp_size, hidden_size, q_heads, max_local_tokens, device="cuda",
                 timeout_s=2.0):
        """``q_heads`` is the local (post base-TP) query head count."""
        self.S = sp_size
        self.H = hidden_size
        self.q_heads = q_heads
        self.max_local_tokens = max_local_tokens
        self.device = torch.device(device)
        words = _C.oproj_sync_words(max_local_tokens)
        self.gather = [torch.full((max_local_tokens, q_heads * HEAD), float("nan"),
                                  dtype=torch.bfloat16, device=self.device)
                       for _ in range(sp_size)]
        self.sync = [torch.zeros(words, dtype=torch.int32, device=self.device)
                     for _ in range(sp_size)]
        self.status = _C.StatusWord()
        self.ops = []
        for r in range(sp_size):
            t = _C.OprojTopology()
            t.device = self.device.index or 0
            t.sp_size = sp_size
            t.sp_rank = r
            t.q_heads = q_heads
            t.hidden_size = hidden_size
            t.max_local_tokens = max_local_tokens
            for d in range(sp_size):
                t.gather[d] = self.gather[d].data_ptr()
                t.sync[d] = self.sync[d].data_ptr()
            t.status = self.status.device_ptr
            t.status_host = self.status.host_ptr
            t.timeout_ns = int(timeout_s * 1e9)
            self.ops.append(_C.OprojOp(t))

    def run(self, attn_outs, weights, outs, tokens, variant=0):
        """``variant``: 0 automatic, or FU_FWD_SINGLE / FU_FWD_PAIR for the GEMM."""
        stream = _C.current_stream_handle(self.device.index or 0)
        base = _C.FU_FWD_NO_PEER_WAIT
        for r in range(self.S):
            self.ops[r].forward(attn_outs[r].data_ptr(), None, tokens, None,
                                base | _C.FU_OPROJ_GATHER_ONLY, stream)
        for r in range(self.S):
            self.ops[r].forward(attn_outs[r].data_ptr(), weights[r].data_ptr(), tokens,
                                outs[r].data_ptr(), base | _C.FU_OPROJ_GEMM_ONLY | variant,
                                stream)

    def counters_reset(self):
        """Completion, work and ready counters are back at zero after a call."""
        for block in self.sync:
            b = block.cpu()
            if int(b[_C.FU_SYNC_COUNTER]) or int(b[_C.FU_SYNC_EPOCH + 1]):
                return False
            if bool((b[_C.FU_OPROJ_READY:] != 0).any()):
                return False
        return True

    def close(self):
        for op in self.ops:
            op.destroy()
        self.status.free()


def to_device(params, device):
    out = {}
    for k, v in params.items():
        out[k] = v.to(device) if torch.is_tensor(v) else v
    return out


def isclose_stats(got, want, atol=0.01, rtol=0.01):
    """(violations, max_abs_err) of elementwise |got-want| <= atol + rtol|want|."""
    g, w = got.float().cpu(), want.float().cpu()
    bad = ~torch.isclose(g, w, atol=atol, rtol=rtol)
    diff = (g - w).abs()
    finite = torch.isfinite(diff)
    return int(bad.sum()), float(diff[finite].max()) if finite.any() else 0.0
