"""Collective receive-buffer ownership and the public QKV interface.

Drop-in for the reference's ``flash_ulysses.context.FlashUlyssesContext``
(joey-shao/flash_ulysses ``flash_ulysses/context.py:9-174``): same constructor
keywords, properties, ``ulysses_qkv_forward`` signature, output aliasing and
``close()`` semantics.  Differences, all deliberate:

* requires an sm_100 GPU (B200) instead of SM90 (context.py:59-60);
* also admits ``sp_size == world_size == 1`` (a self-exchange on one GPU);
  the reference requires ``sp_size >= 2`` (context.py:40);
* receive buffers are plain ``cudaMalloc`` allocations shared through CUDA IPC
  handles exchanged on ``control_group`` instead of ThunderKittens'
  broker-based ``TKParallelTensor``; the exit barrier is fused into the kernel
  and uses per-call epoch flags instead of a separate multicast barrier
  launch;
* a device-side wait that gives up (``timeout_s``, default 30 s) or a
  position outside the RoPE cache sets a status word; the next call (or
  ``check()``) raises ``RuntimeError`` instead of hanging, and
  ``ulysses_qkv_forward(..., check=True)`` raises for the failing call itself.
  A call that starts on the device after an earlier call gave up a wait (one
  queued behind a failed call) stores nothing into any receive buffer and
  waits for no peer.

Added (no counterpart in the reference): with ``output_projection=True``,
``ulysses_o_proj_forward`` runs the inverse exchange after attention fused with
the attention output projection.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _C


class FlashUlyssesContext:
    """Construct, call and close collectively on one B200 node.

    rank and world_size describe the participating physical GPUs on this node.
    control_group must cover those same participants for lifecycle barriers and
    the exchange of buffer handles.  Calls use the current CUDA stream.  Results
    alias Q/K/V until the next call or close.  Before reuse, every physical rank
    must finish consuming its previous output.
    """

    def __init__(
        self,
        *,
        rank,
        world_size,
        max_local_tokens,
        hidden_size=4096,
        num_heads=32,
        num_kv_heads=8,
        head_dim=128,
        sp_size=2,
        control_group=None,
        timeout_s=30.0,
        output_projection=False,
    ):
        self.rank, self.world_size = rank, world_size
        self.control_group = control_group
        self.hidden_size = hidden_size
        self.num_heads, self.num_kv_heads = num_heads, num_kv_heads
        self.head_dim, self.sp_size = head_dim, sp_size
        self.max_local_tokens = max_local_tokens
        self._op = None
        self._oproj = None
        self._status = None
        self._views = {}
        self.Q = self.K = self.V = self.barrier = None
        self.G = self.o_barrier = None

        if not 1 <= sp_size <= self.world_size <= 8 or self.world_size % sp_size:
            raise ValueError("SP must divide a single-node world of 1 to 8 GPUs")
        if hidden_size <= 0 or hidden_size % 64 or head_dim != 128:
            raise ValueError("Requires hidden_size > 0 divisible by 64 and head_dim=128")
        if (
            num_heads <= 0
            or num_kv_heads <= 0
            or num_heads % num_kv_heads
            or num_heads % self.world_size
            or num_kv_heads % self.world_size
        ):
            raise ValueError("Q heads must divide by KV heads; both must divide by world_size")
        if max_local_tokens <= 0:
            raise ValueError("max_local_tokens must be positive")
        if not 0 <= rank < world_size:
            raise ValueError("rank must be in [0, world_size)")
        self.device = torch.device("cuda", torch.cuda.current_device())
        if torch.cuda.get_device_capability(self.device) != (10, 0):
            raise ValueError("Requires SM100 (B200)")

        group_start = rank // sp_size * sp_size
        self.sp_rank = rank - group_start
        peers = list(range(group_start, group_start + sp_size))
        capacity = sp_size * max_local_tokens

        def parallel(shape, dtype):
            return _C.ParallelTensor(shape, dtype, rank, world_size, False,
                                     group=control_group, peers=peers, device=self.device)

        self.Q = parallel((capacity, self.output_q_heads * head_dim), torch.bfloat16)
        self.K = parallel((capacity, self.output_kv_heads * head_dim), torch.bfloat16)
        self.V = parallel((capacity, self.output_kv_heads * head_dim), torch.bfloat16)
        # Per-rank synchronisation block: epoch flags written by SP peers and a
        # CTA completion counter (layout in include/flash_ulysses_b200.h).
        self.barrier = parallel((_C.FU_SYNC_WORDS,), torch.int32)
        self.barrier.data_.zero_()
        self._status = _C.StatusWord()

        topo = _C.Topology()
        topo.device = self.device.index
        topo.sp_size = sp_size
        topo.sp_rank = self.sp_rank
        topo.q_heads = self.local_q_heads
        topo.kv_heads = self.local_kv_heads
        topo.hidden_size = hidden_size
        topo.capacity_rows = capacity
        for i, r in enumerate(peers):
            topo.q_recv[i] = self.Q.peer_ptr(r)
            topo.k_recv[i] = self.K.peer_ptr(r)
            topo.v_recv[i] = self.V.peer_ptr(r)
            topo.sync[i] = self.barrier.peer_ptr(r)
        topo.status = self._status.device_ptr
        topo.status_host = self._status.host_ptr
        topo.timeout_ns = int(timeout_s * 1e9)
        self._op = _C.QkvOp(topo)

        if output_projection:
            if hidden_size % 256:
                raise ValueError("output_projection requires hidden_size divisible by 256")
            # Gather buffer (peers push this rank's rows of their heads into it)
            # and a separate synchronisation block with per-m-block ready counters.
            self.G = parallel((max_local_tokens, self.local_q_heads * head_dim), torch.bfloat16)
            self.o_barrier = parallel((_C.oproj_sync_words(max_local_tokens),), torch.int32)
            self.o_barrier.data_.zero_()
            otopo = _C.OprojTopology()
            otopo.device = self.device.index
            otopo.sp_size = sp_size
            otopo.sp_rank = self.sp_rank
            otopo.q_heads = self.local_q_heads
            otopo.hidden_size = hidden_size
            otopo.max_local_tokens = max_local_tokens
            for i, r in enumerate(peers):
                otopo.gather[i] = self.G.peer_ptr(r)
                otopo.sync[i] = self.o_barrier.peer_ptr(r)
            otopo.status = self._status.device_ptr
            otopo.status_host = self._status.host_ptr
            otopo.timeout_ns = int(timeout_s * 1e9)
            self._oproj = _C.OprojOp(otopo)

        torch.cuda.current_stream(self.device).synchronize()
        if world_size > 1 or dist.is_initialized():
            dist.barrier(group=control_group)

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
    def output_q_heads(self):
        return self.num_heads // self.world_size

    @property
    def output_kv_heads(self):
        return self.num_kv_heads // self.world_size

    @property
    def packed_width(self):
        return (self.local_q_heads + 2 * self.local_kv_heads) * self.head_dim

    @property
    def epoch(self):
        """Number of calls made so far (the value published to peers)."""
        return self._op.epoch

    @torch.no_grad()
    def ulysses_qkv_forward(
        self,
        hidden_states,
        qkv_weight,
        positions,
        q_norm_weight,
        k_norm_weight,
        rope_cache,
        *,
        q_epsilon=1e-6,
        k_epsilon=1e-6,
        check=False,
        static_weights=False,
        _projection_out=None,
    ):
        """Return BF16 (q, k, v), each with L * sp_size rows.

        Inputs are contiguous CUDA tensors on the current/context device:
        hidden_states BF16 [L, H], qkv_weight BF16 [H, packed_width],
        positions int64 [L], norm weights FP32 [128], and a NeoX RoPE cache
        FP32 [max_position, 128] containing [cos(64), sin(64)]. Positions must
        index the cache. Epsilons must be positive. The caller crops padding.

        ``check=True`` waits for this call to finish on the current stream
        and raises ``RuntimeError`` if it reported a device-side error (a peer
        that never joined it, a position outside the cache), so the caller
        learns that these outputs are invalid; by default errors surface on
        the next call or ``check()``, without a synchronisation per call.

        ``static_weights=True`` is the caller's promise that no kernel that
        may still be running on the current stream writes ``qkv_weight``
        (inference, where weights do not change): the first stages of the
        weight are then read while the previous kernel finishes, which
        shortens decode-sized calls.  Results are the same; without the
        promise holding, a call may read stale weights.

        ``_projection_out`` is test instrumentation: a BF16 [L, packed_width]
        tensor that also receives this rank's BF16 projection ``x @ W``.
        """
        local_tokens = hidden_states.shape[0]
        if not 0 < local_tokens <= self.max_local_tokens:
            raise ValueError("Input length must be within [1, max_local_tokens]")
        if self._status.value:
            raise RuntimeError("an earlier call failed on the device: "
                               + _C.decode_status(self._status.value))
        _C.launch(hidden_states, qkv_weight, positions, q_norm_weight, k_norm_weight,
                  rope_cache, self._op, q_epsilon=q_epsilon, k_epsilon=k_epsilon,
                  flags=_C.FU_FWD_STATIC_WEIGHTS if static_weights else 0,
                  gemm_out=_projection_out)
        if check:
            torch.cuda.current_stream(self.device).synchronize()
            if self._status.value:
                raise RuntimeError("this call failed on the device: "
                                   + _C.decode_status(self._status.value))
        views = self._views.get(local_tokens)
        if views is None:
            output_tokens = local_tokens * self.sp_size
            views = tuple(t.data()[:output_tokens] for t in (self.Q, self.K, self.V))
            self._views = {local_tokens: views}      # row views of the receive buffers
        return views

    @torch.no_grad()
    def ulysses_o_proj_forward(self, attn_output, o_proj_weight, *, out=None):
        """Inverse Ulysses exchange fused with the attention output projection
        (no counterpart in the reference, which stops at the forward exchange).

        ``attn_output`` is this rank's attention output, BF16
        ``[L * sp_size, output_q_heads * 128]`` in the layout of the ``q``
        returned by ``ulysses_qkv_forward`` (rows ``s*L..`` belong to SP member
        ``s``); ``o_proj_weight`` is BF16 ``[hidden_size, local_q_heads * 128]``
        (nn.Linear layout).  Returns BF16 ``[L, hidden_size]`` =
        ``gathered @ o_proj_weight.T`` for this rank's L tokens, written into
        ``out`` when given.  Requires ``output_projection=True`` at
        construction; every rank of the SP group makes the same calls.
        ``attn_output`` is only read during this rank's call.
        """
        if self._oproj is None:
            raise RuntimeError("construct the context with output_projection=True")
        rows = attn_output.shape[0]
        if rows % self.sp_size:
            raise ValueError("attn_output rows must be a multiple of sp_size")
        local_tokens = rows // self.sp_size
        if not 0 < local_tokens <= self.max_local_tokens:
            raise ValueError("Input length must be within [1, max_local_tokens]")
        # The kernel's tensor maps are built from these shapes, so a tensor of
        # another shape, dtype or layout would be read or written out of bounds.
        k = self.local_q_heads * self.head_dim
        for name, t, shape in (
                ("attn_output", attn_output, (rows, self.output_q_heads * self.head_dim)),
                ("o_proj_weight", o_proj_weight, (self.hidden_size, k)),
                ("out", out, (local_tokens, self.hidden_size))):
            if t is None:
                continue
            if (tuple(t.shape) != shape or t.dtype != torch.bfloat16 or not t.is_contiguous()
                    or t.device != self.device):
                raise ValueError(f"{name} must be a contiguous BF16 tensor of shape {shape} "
                                 f"on {self.device}")
        if self._status.value:
            raise RuntimeError("an earlier call failed on the device: "
                               + _C.decode_status(self._status.value))
        if out is None:
            out = torch.empty(local_tokens, self.hidden_size, dtype=torch.bfloat16,
                              device=self.device)
        stream = _C.current_stream_handle(self.device.index)
        self._oproj.forward(attn_output.data_ptr(), o_proj_weight.data_ptr(), local_tokens,
                            out.data_ptr(), 0, stream)
        return out

    def check(self):
        """Synchronise the device and raise if any call reported a device-side error."""
        torch.cuda.synchronize(self.device)
        if self._status.value:
            raise RuntimeError("device-side error: " + _C.decode_status(self._status.value))

    def clear_error(self):
        """Reset the status word, the completion counters and the operators'
        failed marks after a reported error (call only when no launch of this
        context is in flight)."""
        torch.cuda.synchronize(self.device)
        for block in (self.barrier, self.o_barrier):
            if block is not None:
                block.data_[_C.FU_SYNC_COUNTER].zero_()
                block.data_[_C.FU_SYNC_FAILED].zero_()
        torch.cuda.synchronize(self.device)
        self._status.clear()

    def close(self):
        """Collectively release peer mappings after all output consumers finish."""
        torch.cuda.synchronize(self.device)
        if self.world_size > 1 or dist.is_initialized():
            dist.barrier(group=self.control_group)
        self._views = {}
        with torch.cuda.device(self.device):
            if self._op is not None:
                self._op.destroy()
                self._op = None
            if self._oproj is not None:
                self._oproj.destroy()
                self._oproj = None
            for name in ("Q", "K", "V", "barrier", "G", "o_barrier"):
                t = getattr(self, name)
                if t is not None:
                    t.close()
                setattr(self, name, None)
            if self._status is not None:
                self._status.free()
                self._status = None
