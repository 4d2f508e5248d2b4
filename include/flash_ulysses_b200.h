/*
 * flash_ulysses_b200 -- C ABI of the fused Ulysses QKV operator for B200
 * (sm_100a).
 *
 * The operator computes, for one rank of a single-node world of P GPUs split
 * into SP groups of S consecutive ranks (base tensor parallelism T = P / S):
 *
 *   Y = X[L, H] @ W[H, N]                      BF16 in, FP32 accumulate, BF16 out
 *   Q, K heads: RMSNorm (FP32) * gamma -> BF16 -> NeoX RoPE (FP32) -> BF16
 *   V heads:    BF16 projection as is
 *   Ulysses all-to-all: local packed head h of component c goes to SP member
 *   h / (heads_c / S), head column h % (heads_c / S), rows [sp_rank * L, +L)
 *
 * and stores every output tile directly into the destination rank's receive
 * buffer (its memory mapped into this process), then joins the SP group on
 * per-call epoch flags.  Everything happens in one kernel launch on the
 * caller's stream.
 *
 * All functions return 0 on success and a nonzero FU_ERR_* code otherwise;
 * fu_last_error() describes the most recent failure on the calling thread.
 * No function takes or returns framework (torch) types: plain pointers,
 * sizes and CUDA stream handles only.
 */
#ifndef FLASH_ULYSSES_B200_H_
#define FLASH_ULYSSES_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FU_API __attribute__((visibility("default")))
#else
#define FU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FU_MAX_SP 8          /* largest SP group: one 8-GPU node */
#define FU_HEAD_DIM 128      /* head dimension, as in the reference */
#define FU_IPC_HANDLE_BYTES 64
/* Per-rank synchronisation block (uint32 words), shared with the SP group:
 *   [0, FU_MAX_SP)            exit flags: word p holds the last epoch SP member
 *                             p finished writing into this rank
 *   [FU_SYNC_ENTRY, +FU_MAX_SP) entry flags: word p holds the last epoch SP
 *                             member p started (its stream reached the call)
 *   [FU_SYNC_COUNTER]         CTA completion counter (local use only)
 *   [FU_SYNC_EPOCH]           this rank's epoch: the number of calls made,
 *                             advanced by the kernel itself, so captured CUDA
 *                             graphs replay with fresh epochs
 *   [FU_SYNC_FAILED]          nonzero once a call of this operator gave up a
 *                             wait (sp_size > 1): later calls that start while
 *                             it is set store nothing and wait for nothing
 *                             (local use only; cleared with the counter when
 *                             the caller clears the error)
 * Calls of one SP group advance in lockstep: every rank makes the same calls.
 */
#define FU_SYNC_WORDS 64
#define FU_SYNC_ENTRY 8
#define FU_SYNC_COUNTER 32
#define FU_SYNC_EPOCH 33
#define FU_SYNC_FAILED 35

enum fu_error {
    FU_OK = 0,
    FU_ERR_INVALID = 1,      /* bad argument (shape, pointer, topology) */
    FU_ERR_CUDA = 2,         /* a CUDA runtime/driver call failed */
    FU_ERR_UNSUPPORTED = 3,  /* device is not sm_100 or lacks a feature */
    FU_ERR_DEVICE = 4        /* a previous launch reported a device-side error */
};

/* Device-side status codes (low byte of the status word; the next byte says
 * which wait gave up). */
enum fu_device_status {
    FU_STATUS_OK = 0,
    FU_STATUS_PIPELINE_TIMEOUT = 1,
    FU_STATUS_PEER_TIMEOUT = 2,
    FU_STATUS_POSITION_RANGE = 3
};

/* Default bound on a device-side wait: 30 s, long enough for ranks whose
 * calls start seconds apart (start-up, a garbage-collection pause).  A wait
 * that gives up records the failure in the status word and in the sync
 * block's FU_SYNC_FAILED word; a call that starts with that word set (queued
 * behind a failed one) stores nothing and waits for nothing, so one failure
 * costs one timeout, not one per queued call. */
#define FU_DEFAULT_TIMEOUT_NS 30000000000ull

/* Flags for fu_qkv_forward. */
#define FU_FWD_NO_PEER_WAIT 1u  /* publish entry/exit flags but wait for no peer */
/* Split-K factor 1..8 (0 = choose automatically): with n > 1 each tile is
 * reduced by a cluster of n CTAs that sum their partials over distributed
 * shared memory; 1 forces the persistent one-CTA-per-tile grid. */
#define FU_FWD_SPLITS(n) (((uint32_t)(n) & 0xFu) << 8)
/* Persistent-grid variant: 0 = automatic (CTA pairs once a call spans two
 * 128-row blocks), FU_FWD_SINGLE = one CTA per 128 x 256 tile, FU_FWD_PAIR =
 * CTA pairs (tcgen05 cta_group::2) on 256 x 256 tiles. */
#define FU_FWD_SINGLE (1u << 12)
#define FU_FWD_PAIR (2u << 12)
/* Keep whole 2-head tiles in the last round of the pair grid (by default a
 * last round that at most half fills the pairs is re-tiled into one-head
 * units). */
#define FU_FWD_NO_RETILE (1u << 14)
/* Keep Q/K in FP32 from the accumulator through RMSNorm and RoPE and round to
 * BF16 once at the end -- the numerics of the reference's Hopper kernel
 * (flash_ulysses_kernel_hopper.cu:129-152).  Default: the reference PyTorch
 * path's rounding points (BF16 projection, BF16 after the norm). */
#define FU_FWD_FP32_EPILOGUE (1u << 15)
/* Launch without programmatic dependent launch.  By default the kernel is
 * launched with cudaLaunchAttributeProgrammaticStreamSerialization: its
 * prologue (barrier set-up, TMEM allocation) may run while the previous
 * kernel of the stream finishes, and it reads or writes no global memory
 * before that kernel has completed (except qkv_weight under
 * FU_FWD_STATIC_WEIGHTS); it also lets the next such kernel of the
 * stream start its prologue early.  Results are the same either way. */
#define FU_FWD_NO_PDL (1u << 17)
/* The caller promises that no kernel that may still be running on the stream
 * when this call starts writes qkv_weight (inference: weights do not change
 * between calls).  The first operand stages of W are then requested before
 * the wait for the previous kernel, so under programmatic dependent launch
 * they stream in while it finishes (one-CTA tiles: split-K and single-CTA
 * variants; ignored by the CTA-pair variant).  Inputs written by earlier
 * kernels (hidden_states, positions, ...) are still read after that wait.
 * Without the promise holding, the call may read stale weights. */
#define FU_FWD_STATIC_WEIGHTS (1u << 18)

FU_API const char* fu_last_error(void);
FU_API int fu_version(void);

/* ------------------------------------------------------------------------
 * Receive buffers shared by the ranks of one node.  Replaces the symmetric
 * allocation of ThunderKittens' TKParallelTensor (reference
 * flash_ulysses/context.py:63-90, csrc/bindings.cu:16): every rank allocates
 * its own buffer, exports a 64-byte handle, and opens every peer's handle.
 * The handles are exchanged by the caller (e.g. torch.distributed on the
 * control group), so no fixed-name broker is involved.
 * ------------------------------------------------------------------------ */
FU_API int fu_buffer_alloc(int device, size_t bytes, void** ptr);
FU_API int fu_buffer_free(int device, void* ptr);
FU_API int fu_buffer_export(int device, void* ptr, unsigned char handle[FU_IPC_HANDLE_BYTES]);
FU_API int fu_buffer_import(int device, const unsigned char handle[FU_IPC_HANDLE_BYTES],
                     void** peer_ptr);
FU_API int fu_buffer_close(int device, void* peer_ptr);

/* Host-mapped status word the kernel writes on a device-side error.  The
 * host reads *host_ptr without synchronising. */
FU_API int fu_status_alloc(int32_t** host_ptr, int32_t** device_ptr);
FU_API int fu_status_free(int32_t* host_ptr);

/* ------------------------------------------------------------------------
 * The fused operator.
 * ------------------------------------------------------------------------ */
typedef struct fu_qkv_ctx fu_qkv_ctx;

typedef struct fu_qkv_topology {
    int32_t device;          /* CUDA device ordinal of this rank */
    int32_t sp_size;         /* S: 1..FU_MAX_SP */
    int32_t sp_rank;         /* this rank's index in its SP group */
    int32_t q_heads;         /* local (post base-TP) query heads, divisible by S */
    int32_t kv_heads;        /* local key/value heads, divisible by S */
    int32_t reserved0;
    int64_t hidden_size;     /* H, a positive multiple of 64 */
    int64_t capacity_rows;   /* rows of every receive buffer: S * max_local_tokens */
    /* Receive buffers of SP member p as mapped in this process (p == sp_rank
     * is this rank's own).  Row-major BF16 [capacity_rows, heads_c/S * 128]. */
    void* q_recv[FU_MAX_SP];
    void* k_recv[FU_MAX_SP];
    void* v_recv[FU_MAX_SP];
    /* Synchronisation block (FU_SYNC_WORDS uint32, zero-initialised) of SP
     * member p as mapped in this process. */
    uint32_t* sync[FU_MAX_SP];
    int32_t* status;         /* device pointer of a status word, may be NULL */
    int32_t* status_host;    /* host view of the same word (fu_status_alloc), may be NULL;
                                fu_qkv_forward refuses to launch while it is nonzero */
    uint64_t timeout_ns;     /* bound on every device-side wait; 0 = FU_DEFAULT_TIMEOUT_NS */
} fu_qkv_topology;

/* Create the per-rank operator state (tensor-map caches, epoch counter).
 * Replaces the descriptor set-up of the reference launcher
 * (flash_ulysses_kernel_hopper.cu:305-347).  A context is not thread-safe:
 * calls on one context (either operator) must not run concurrently on the
 * host, since each call updates the context's caches and parameter block;
 * different contexts are independent. */
FU_API int fu_qkv_create(const fu_qkv_topology* topo, fu_qkv_ctx** out);
FU_API int fu_qkv_destroy(fu_qkv_ctx* ctx);

/* One fused call: projection + Q/K RMSNorm + NeoX RoPE + Ulysses exchange +
 * exit barrier, as a single launch on `stream` (a cudaStream_t).
 * Replaces flash_ulysses::launch (reference
 * flash_ulysses/csrc/impl/flash_ulysses_kernel_hopper.cu:305-353, bound at
 * csrc/bindings.cu:17 and called from context.py:144-160).
 *
 *   x          BF16 [local_tokens, H], row-major, 16-byte aligned
 *   w          BF16 [H, (q_heads + 2 kv_heads) * 128], row-major, packed Q|K|V
 *   positions  int64 [local_tokens], indices into rope
 *   q_gamma, k_gamma  FP32 [128]
 *   rope       FP32 [rope_rows, 128] = cos(64) | sin(64)
 *   gemm_out   NULL, or BF16 [local_tokens, N]: test instrumentation that
 *              also receives the BF16-rounded projection
 *
 * 1 <= local_tokens <= capacity_rows / S.  Every rank of the SP group must
 * make the same sequence of calls; all ranks must have finished consuming
 * the previous call's outputs before any rank calls again (reference
 * README.md:67-70).  Returns FU_ERR_DEVICE without launching if an earlier
 * launch left a nonzero status word. */
FU_API int fu_qkv_forward(fu_qkv_ctx* ctx, const void* x, const void* w, const int64_t* positions,
                   const float* q_gamma, const float* k_gamma, const float* rope,
                   int64_t local_tokens, int64_t rope_rows, double q_epsilon,
                   double k_epsilon, uint32_t flags, void* stream, void* gemm_out);

/* Number of calls launched through this context (the device-side epoch of
 * the most recent call once it has run, for contexts used without graphs). */
FU_API uint32_t fu_qkv_epoch(const fu_qkv_ctx* ctx);

/* Number of CTAs the most recent call launched (persistent grid). */
FU_API int fu_qkv_last_grid(const fu_qkv_ctx* ctx);

/* ------------------------------------------------------------------------
 * Allocation-free call for a world of one GPU.  This entry point has no
 * counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they call the
 * operator -- e.g. a server that has reserved all free HBM for its own pool,
 * or a C caller that owns only the buffers it passes in.  It runs the same
 * fused kernel as fu_qkv_forward with sp_size 1 (outputs Q [L, q_heads*128],
 * K and V [L, kv_heads*128], BF16 row-major) and allocates nothing on any
 * call: its scratch (completion counter and exit flag, FU_SYNC_WORDS words =
 * 256 bytes) is a static array inside the library that every GPU loading the
 * library holds until the process exits.  The first call on a device resolves
 * that array's address and sets the kernel's shared-memory limit; make that
 * first call before any stream capture.  Calls share the scratch and each one
 * zeroes the counter before launching, so calls that overlap on the same GPU
 * race.  Rejects local_tokens outside [1, FU_NOALLOC_MAX_TOKENS].
 * `status` is an optional caller-owned device int32 that receives a device-side
 * status code (NULL: not reported).  No context object is needed. */
#define FU_NOALLOC_MAX_TOKENS (1 << 30)
FU_API int fu_qkv_forward_noalloc(int device, const void* x, const void* w,
                                  const int64_t* positions, const float* q_gamma,
                                  const float* k_gamma, const float* rope,
                                  int64_t local_tokens, int64_t hidden_size, int32_t q_heads,
                                  int32_t kv_heads, int64_t rope_rows, double q_epsilon,
                                  double k_epsilon, void* q_out, void* k_out, void* v_out,
                                  int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Inverse exchange fused with the attention output projection.  No
 * counterpart in the reference, which stops at the forward exchange; this is
 * the step its outputs feed once attention has run (reference README.md:44-46
 * describes the head <-> sequence exchange this inverts).
 *
 * SP member d holds attention output for its q_heads/S heads over the whole
 * group's sequence, attn_d BF16 [S * L, q_heads/S * 128] (rows s*L.. belong to
 * source s: the layout in which fu_qkv_forward delivers Q).  Each call returns
 * to every source s its L rows for all q_heads local heads and multiplies them
 * by the output projection:
 *     out_s = G_s . W_o^T,   G_s [L, q_heads * 128],   W_o BF16 [H, q_heads * 128]
 * (torch.nn.Linear's weight layout), FP32 accumulation, BF16 out [L, H].
 * Each rank pushes its own attention output into the owners' gather buffers
 * over NVLink while the owners' tensor cores start on the m-blocks already
 * complete.
 * ------------------------------------------------------------------------ */
typedef struct fu_oproj_ctx fu_oproj_ctx;

/* First word of the per-m-block ready counters in an o-projection sync block. */
#define FU_OPROJ_READY FU_SYNC_WORDS
/* Two-phase mode for SP ranks emulated on one GPU (whose kernels must not
 * wait for one another): one call per rank with FU_OPROJ_GATHER_ONLY, then
 * one per rank with FU_OPROJ_GEMM_ONLY.  Use with FU_FWD_NO_PEER_WAIT. */
#define FU_OPROJ_GATHER_ONLY (1u << 20)
#define FU_OPROJ_GEMM_ONLY (1u << 21)

typedef struct fu_oproj_topology {
    int32_t device;           /* CUDA device ordinal of this rank */
    int32_t sp_size;          /* S: 1..FU_MAX_SP */
    int32_t sp_rank;          /* this rank's index in its SP group */
    int32_t q_heads;          /* local (post base-TP) query heads, divisible by S */
    int32_t reserved0;
    int32_t reserved1;
    int64_t hidden_size;      /* H, a positive multiple of 256 */
    int64_t max_local_tokens; /* largest L of any call */
    /* Gather buffer of SP member p as mapped in this process: BF16
     * [max_local_tokens, q_heads * 128], 16-byte aligned; peers write their
     * columns into it (a member's own columns are read from its attn). */
    void* gather[FU_MAX_SP];
    /* O-projection sync block of SP member p (fu_oproj_sync_words words,
     * zero-initialised), separate from the forward operator's. */
    uint32_t* sync[FU_MAX_SP];
    int32_t* status;          /* device pointer of a status word, may be NULL */
    int32_t* status_host;     /* host view of the same word, may be NULL */
    uint64_t timeout_ns;      /* bound on every device-side wait; 0 = FU_DEFAULT_TIMEOUT_NS */
} fu_oproj_topology;

/* Words of an o-projection sync block for calls of up to max_local_tokens. */
FU_API int64_t fu_oproj_sync_words(int64_t max_local_tokens);
FU_API int fu_oproj_create(const fu_oproj_topology* topo, fu_oproj_ctx** out);
FU_API int fu_oproj_destroy(fu_oproj_ctx* ctx);

/* One call, one launch on `stream` (flags: FU_FWD_NO_PEER_WAIT, FU_FWD_SINGLE /
 * FU_FWD_PAIR to force the GEMM variant, FU_FWD_NO_PDL, FU_OPROJ_GATHER_ONLY /
 * FU_OPROJ_GEMM_ONLY):
 *   attn   BF16 [S * local_tokens, q_heads/S * 128], this rank's attention output
 *   w_o    BF16 [H, q_heads * 128]
 *   out    BF16 [local_tokens, H]
 * Every rank of the SP group makes the same sequence of calls.  attn is read
 * during this rank's call only, so it may be overwritten once the call has
 * completed on this rank's stream. */
FU_API int fu_oproj_forward(fu_oproj_ctx* ctx, const void* attn, const void* w_o,
                            int64_t local_tokens, void* out, uint32_t flags, void* stream);

/* Number of calls launched through this context. */
FU_API uint32_t fu_oproj_calls(const fu_oproj_ctx* ctx);
/* Number of CTAs the most recent call launched. */
FU_API int fu_oproj_last_grid(const fu_oproj_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_ULYSSES_B200_H_ */
