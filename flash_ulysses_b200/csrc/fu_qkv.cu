// Fused QKV projection + Q/K RMSNorm + NeoX RoPE + Ulysses exchange for
// B200 (sm_100a), one persistent launch per call.
//
// What it replaces: the reference's Hopper kernel and launcher
// (joey-shao/flash_ulysses flash_ulysses/csrc/impl/flash_ulysses_kernel_hopper.cu:
// kernel<N> 157-267, rmsnorm_and_rope 129-152, apply_neox_rope 86-125,
// barrier_kernel 283-288, launch 305-353).  The reference's numerics differ
// from its own PyTorch path (it keeps FP32 through the epilogue); this kernel
// follows the PyTorch path's rounding points instead (tests/torch_base.py:52-64):
// BF16 projection, FP32 norm, BF16, FP32 rotation, BF16.
//
// CTA layout (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: X tile [128 x 64] and W tile [64 x 256] per stage
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma M=128 N=256 K=16, FP32 in
//               TMEM, two accumulator buffers of 256 columns
//   warps 2..5  epilogue: one TMEM lane (= one token row) per thread; each
//               thread holds a full 128-wide head row, so the RMSNorm sum and
//               the NeoX partner (j, j+64) are thread-local; results are
//               staged in swizzled shared memory and written by TMA bulk
//               tensor stores directly into the destination rank's receive
//               buffer (a peer GPU's memory mapped into this process).
// A tile is 128 token rows x 2 heads (256 packed columns).  Each call's epoch
// lives in the rank's sync block and is advanced by the kernel itself.  At
// start the call announces the epoch to its SP peers (entry flags); before a
// CTA's first store into a peer's buffer it waits until every peer has
// started the same call (so the peer's stream has finished with the previous
// outputs).  After its last tile every CTA waits for its stores to complete
// and bumps a per-rank counter; the last CTA of the rank publishes the epoch
// into every SP member's exit flag and waits (bounded) for theirs.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "flash_ulysses_b200.h"
#include "fu_internal.h"
#include "fu_ptx.cuh"

namespace fu {

constexpr int BM = 128;                 // token rows per CTA tile = TMEM lanes
constexpr int BN = 256;                 // packed columns per tile = 2 heads
constexpr int BK = 64;                  // reduction step: one 128-byte swizzle row
constexpr int UMMA_K = 16;              // K of one tcgen05.mma kind::f16
constexpr int NUM_THREADS = 192;
constexpr int NUM_EPI_THREADS = 128;
constexpr int A_STAGE_BYTES = BM * BK * 2;                    // 16 KiB
constexpr int B_CHUNK_BYTES = BK * 64 * 2;                    // 8 KiB: 64 columns x BK rows
constexpr int BOX_BYTES = 32 * 128;                           // 32 rows x 64 BF16
constexpr int STAGING_PER_WARP = 2 * BOX_BYTES;               // lo and hi halves of one head
constexpr uint32_t TMEM_COLS = 512;

// Operand ring of a kernel variant.  One CTA per tile (kPair false): 4
// stages of X [128 x 64] + W [64 x 256].  CTA pair (kPair true): each CTA
// holds X [128 x 64] + its half of W, [64 x 128], so 6 stages fit.
template <bool kPair>
struct Ring {
    static constexpr int STAGES = kPair ? 6 : 4;
    static constexpr int B_CHUNKS = kPair ? 2 : 4;            // 64-column W boxes per CTA
    static constexpr int B_STAGE_BYTES = B_CHUNKS * B_CHUNK_BYTES;
    static constexpr uint32_t CTA_TX = A_STAGE_BYTES + B_STAGE_BYTES;
    static constexpr uint32_t STAGE_TX = kPair ? 2 * CTA_TX : CTA_TX;   // the leader counts both
    static constexpr int OFF_B = STAGES * A_STAGE_BYTES;
    static constexpr int BYTES = OFF_B + STAGES * B_STAGE_BYTES;
};
static_assert(Ring<true>::BYTES == Ring<false>::BYTES, "both variants share one layout");

constexpr int OFF_A = 0;
constexpr int OFF_STG = Ring<false>::BYTES;
constexpr int OFF_BAR = OFF_STG + 4 * STAGING_PER_WARP;
constexpr int MAX_STAGES = 6;
constexpr int NUM_BARS = 2 * MAX_STAGES + 2 + 2 + 1 + 1;
constexpr int OFF_MISC = OFF_BAR + 256;
constexpr int OFF_GAMMA = OFF_MISC + 64;
constexpr int SMEM_BYTES = OFF_GAMMA + 2 * 128 * 4;
// Split mode parks a 128 x 256 FP32 partial in the operand ring; rows are
// padded by 16 bytes so that a warp's row-per-thread stores spread over banks.
constexpr int PART_STRIDE = BN * 4 + 16;
static_assert(BM * PART_STRIDE <= OFF_STG, "split partial must fit in the operand ring");
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;                 // room to align the base to 1 KiB
static_assert(NUM_BARS * 8 <= 256, "barrier area");
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KiB per-CTA shared memory limit");

// Where a wait gave up (second byte of the status word).
enum : int { W_EMPTY = 1, W_FULL = 2, W_TEMPTY = 3, W_TFULL = 4, W_DRAIN = 5 };

struct __align__(64) QkvParams {
    CUtensorMap tm_x;                       // X [L, H]: box {64, 128}
    CUtensorMap tm_w;                       // W [H, N]: box {64, 64}
    CUtensorMap tm_out[3 * FU_MAX_SP];      // [component * FU_MAX_SP + dst]: {cols, L, S}
    const int64_t* positions;
    const float* q_gamma;
    const float* k_gamma;
    const float* rope;
    __nv_bfloat16* gemm_out;
    uint32_t* sync[FU_MAX_SP];
    int32_t* status;
    unsigned long long timeout_ns;
    int32_t L, H, N, rope_rows;
    int32_t heads, q_heads, kv_heads;
    int32_t sp_size, sp_rank, q_per_gpu, kv_per_gpu;
    int32_t num_n_blocks, num_tiles, k_blocks;
    int32_t num_m_tiles;                    // row blocks of tiles (128 rows, or 256 for a pair)
    float q_eps, k_eps;
    uint32_t wait_peers;
    uint32_t fp32_epilogue;                 // 1: no BF16 rounding before the final store
    int32_t splits;                         // >1: split-K over a cluster of this many CTAs
    int32_t split_push;                     // split mode, few rows: partials pushed to the leader
    void* out_base[3 * FU_MAX_SP];          // receive buffers (split mode stores rows directly)
    int32_t num_units;                      // work units of the persistent grid
    int32_t full_units;                     // units [0, full_units) are whole tiles; each later
                                            // pair of units is one tile's two heads
    int32_t static_weights;                 // 1: W may be read before the dependency wait
};
static_assert(sizeof(QkvParams) <= 4096, "kernel parameter block too large");

__device__ __forceinline__ float bf16_round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float round_if(float v, bool to_bf16) {
    return to_bf16 ? bf16_round(v) : v;
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(b);
}

// 1 / sqrt(mean + eps) for a sum of 128 squares, with the rounding points of
// torch's CPU operators: the mean (an exact scaling), the FP32 addition of
// eps, a correctly rounded square root and a correctly rounded reciprocal.
__device__ __forceinline__ float norm_scale(float sum_sq, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sum_sq * (1.0f / 128.0f), eps)));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&b);
}

// Bounded wait that ignores the abort flag: used only to drain in-flight
// asynchronous work before the CTA exits.
__device__ __forceinline__ bool drain_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                           int32_t* status) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > timeout_ns) {
            report_status(status, FU_DEV_PIPELINE_TIMEOUT, W_DRAIN);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------ schedule
// Which tiles and which k-blocks this CTA owns.
//   one CTA per tile, persistent (splits 1): tiles blockIdx.x, +gridDim.x, ...
//   over the full reduction; a tile is 128 rows x 256 columns;
//   split mode: the CTAs of one cluster share one tile; cluster rank s reduces
//   k-blocks [s*KB/S, (s+1)*KB/S);
//   CTA pairs, persistent: pair tiles of 256 rows x 256 columns over the
//   clusters; CTA rank r of the pair owns rows [128 r, 128 r + 128).
struct Sched {
    int first, end, stride, kb0, kb1, split, rank, rows_per_tile;
};

template <bool kPair>
__device__ __forceinline__ Sched make_sched(const QkvParams& p) {
    Sched s;
    s.rank = 0;
    s.rows_per_tile = BM;
    if (kPair) {
        s.rank = static_cast<int>(cluster_ctarank());
        s.rows_per_tile = 2 * BM;
        s.split = 0;
        s.first = static_cast<int>(blockIdx.x) / 2;
        s.end = p.num_units;
        s.stride = static_cast<int>(gridDim.x) / 2;
        s.kb0 = 0;
        s.kb1 = p.k_blocks;
    } else if (p.splits > 1) {
        s.split = static_cast<int>(blockIdx.x) % p.splits;
        s.first = static_cast<int>(blockIdx.x) / p.splits;
        s.end = s.first + 1;
        s.stride = 1;
        s.kb0 = s.split * p.k_blocks / p.splits;
        s.kb1 = (s.split + 1) * p.k_blocks / p.splits;
    } else {
        s.split = 0;
        s.first = blockIdx.x;
        s.end = p.num_tiles;
        s.stride = gridDim.x;
        s.kb0 = 0;
        s.kb1 = p.k_blocks;
    }
    return s;
}

// Tiles are numbered column-major (t -> row block t mod num_m_tiles, column
// block t / num_m_tiles), so the pairs running at the same time share W's
// column blocks and re-read X, the smaller operand, from L2: W streams from
// HBM once per call (row-major numbering re-read all of W every round, and
// the outputs written in between evicted part of it).
//
// A work unit of the persistent grid: a whole tile (both heads, half = -1),
// or one head of a tile (half = 0 or 1).  A last, partial round of a pair grid
// that at most half fills the pairs is re-tiled into one-head units, spread
// over twice as many pairs (measured on B200, c1 shape: L=1024 53.5 us against
// 57.2 us with whole tiles; neutral at L >= 4096).
struct Unit {
    int m_blk, n_blk, half;
};

__device__ __forceinline__ Unit decode_unit(const QkvParams& p, int u) {
    Unit un;
    if (u < p.full_units) {
        un.m_blk = u % p.num_m_tiles;
        un.n_blk = u / p.num_m_tiles;
        un.half = -1;
    } else {
        const int j = u - p.full_units;
        const int t = p.full_units + (j >> 1);
        un.m_blk = t % p.num_m_tiles;
        un.n_blk = t / p.num_m_tiles;
        un.half = j & 1;
    }
    return un;
}

// One work item of a CTA: a unit over k-blocks [kb0, kb1).
struct Item {
    Unit un;
    int kb0, kb1;
};

// Position of a CTA in its work list: units first, first + stride, ...
struct Walk {
    int next, end, stride;
};

__device__ __forceinline__ Walk make_walk(const QkvParams& p, const Sched& sc) {
    Walk w;
    w.next = sc.first;
    w.end = sc.end;
    w.stride = sc.stride;
    return w;
}

// Describes the next item and advances the walk; false when the CTA has no
// more work.
__device__ __forceinline__ bool next_item(const QkvParams& p, const Sched& sc, Walk& w,
                                          Item& it) {
    if (w.next >= w.end) return false;
    it.un = decode_unit(p, w.next);
    it.kb0 = sc.kb0;
    it.kb1 = sc.kb1;
    w.next += w.stride;
    return true;
}

// Shared-memory barrier layout (fixed offsets, up to MAX_STAGES stages).
struct Bars {
    uint32_t full, empty, tfull, tempty, mma_done, push;
    __device__ Bars(uint32_t base)
        : full(base), empty(base + 8 * MAX_STAGES), tfull(base + 16 * MAX_STAGES),
          tempty(base + 16 * MAX_STAGES + 16), mma_done(base + 16 * MAX_STAGES + 32),
          push(base + 16 * MAX_STAGES + 40) {}
};

// Split push mode: the staging area holds the tile's RoPE row indices
// (512 bytes), then one 1 KiB FP32 row (256 columns) per valid token row and
// cluster rank, [rank][row]: every CTA parks its rows in its own rank's slot,
// and the leader (rank 0) receives the others' slots at the same offsets.
constexpr int OFF_PUSH = OFF_STG + 512;
constexpr int PUSH_ROW_BYTES = BN * 4;
constexpr int PUSH_BYTES = 4 * STAGING_PER_WARP - 512;
// After the [rank][row] slots: the valid rows' cos|sin (512 bytes each),
// fetched by the leader while the tensor cores run.
constexpr int ROPE_ROW_BYTES = 128 * 4;
__device__ __forceinline__ int push_rope_offset(const QkvParams& p) {
    return OFF_PUSH + p.splits * p.L * PUSH_ROW_BYTES;
}

// Whether an earlier call of this operator gave up a wait: the sticky
// FU_SYNC_FAILED word of this rank's own sync block, in device memory (a read
// of the host-mapped status word from every CTA would cost a serialised
// host-memory round trip each).  Read by the thread that runs the entry
// barrier.
__device__ __forceinline__ int32_t status_at_start(const QkvParams& p) {
    if (threadIdx.x != 64 || p.sp_size == 1) return 0;
    return static_cast<int32_t>(
        *reinterpret_cast<volatile const uint32_t*>(p.sync[p.sp_rank] + FU_SYNC_FAILED));
}

// Entry barrier, run before a CTA's first store into a peer's buffer by the 4
// epilogue warps (or, in the split-K reduction, all six warps: bar_threads):
// one thread waits (bounded) until every SP member has started this call's
// epoch, then the warps meet on named barrier 1.  Returns
// false -- and the CTA stores nothing -- when an earlier call of this operator
// failed (this queued call must neither wait for peers nor write into them)
// or when the wait gives up.  Either raises the
// CTA's abort flag, so the producer and MMA issuer stop too.  In a CTA pair
// the partner's abort flag is raised as well (over distributed shared
// memory), since the pair's MMAs and accumulator hand-offs involve both.
__device__ __forceinline__ bool wait_peers_entered(const QkvParams& p, uint32_t epoch,
                                                   volatile int* abort_flag, bool pair,
                                                   int32_t status_seen,
                                                   int bar_threads = NUM_EPI_THREADS) {
    if (threadIdx.x == 64) {
        bool give_up = false;
        if (*abort_flag) {
            // Another role of this CTA (or of its cluster) already gave up.
        } else if (status_seen != 0) {
            give_up = true;
        } else if (p.sp_size > 1 && p.wait_peers) {
            const uint32_t* entry = p.sync[p.sp_rank] + FU_SYNC_ENTRY;
            const uint64_t t0 = globaltimer_ns();
            for (int s = 0; s < p.sp_size && !give_up; ++s) {
                while (static_cast<int32_t>(ld_acquire_sys_u32(entry + s) - epoch) < 0) {
                    if (globaltimer_ns() - t0 > p.timeout_ns) {
                        report_status(p.status, FU_DEV_PEER_TIMEOUT, 16 + s);
                        give_up = true;
                        break;
                    }
                }
            }
        }
        if (give_up) {
            *abort_flag = 1;
            if (pair)
                st_cluster_u32(map_cluster_smem(smem_u32(const_cast<int*>(abort_flag)),
                                                cluster_ctarank() ^ 1u), 1u);
        }
    }
    named_bar_sync(1, bar_threads);
    return *abort_flag == 0;
}

// ------------------------------------------------------------ roles
// Stages of the first work item whose W the prologue loads before the
// dependency wait (static weights, one-CTA tiles: single or split mode).
template <bool kPair>
__device__ __forceinline__ int early_w_stages(const QkvParams& p, const Sched& sc) {
    if (kPair || !p.static_weights || sc.first >= sc.end) return 0;
    return min(Ring<kPair>::STAGES, sc.kb1 - sc.kb0);
}

// The prologue's part of those stages: each stage's barrier is armed with
// the whole stage's bytes and W's four chunks are requested; the producer
// adds X after the dependency wait.
template <bool kPair>
__device__ __forceinline__ void load_early_w(const QkvParams& p, const Sched& sc, uint8_t* smem,
                                             const Bars& b) {
    using R = Ring<kPair>;
    const int n = early_w_stages<kPair>(p, sc);
    if (n == 0) return;
    const int col0 = decode_unit(p, sc.first).n_blk * BN;
    const uint32_t b0 = smem_u32(smem + R::OFF_B);
    for (int s = 0; s < n; ++s) {
        const uint32_t full = b.full + 8 * s;
        mbar_arrive_expect_tx(full, R::STAGE_TX);
        for (int c = 0; c < R::B_CHUNKS; ++c)
            tma_load_2d(b0 + s * R::B_STAGE_BYTES + c * B_CHUNK_BYTES, &p.tm_w, full,
                        col0 + c * 64, (sc.kb0 + s) * BK);
    }
}

template <bool kPair>
__device__ void run_producer(const QkvParams& p, const Sched& sc, uint8_t* smem, const Bars& b,
                             volatile int* abort_flag) {
    using R = Ring<kPair>;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0;               // stages loaded at least once
    uint32_t last_parity = 0;               // per-stage parity of the last load
    const uint32_t a0 = smem_u32(smem + OFF_A);
    const uint32_t b0 = smem_u32(smem + R::OFF_B);
    bool ok = true;
    // Stages whose W the prologue requested: their X, now that the previous
    // kernel of the stream has completed (their barriers already expect it).
    int early = early_w_stages<kPair>(p, sc);
    if (early > 0) {
        const int row0 = decode_unit(p, sc.first).m_blk * sc.rows_per_tile;
        for (int s = 0; s < early; ++s)
            tma_load_2d(a0 + s * A_STAGE_BYTES, &p.tm_x, b.full + 8 * s, (sc.kb0 + s) * BK, row0);
        issued_mask = (1u << early) - 1u;
    }
    Walk walk = make_walk(p, sc);
    Item it;
    while (ok && next_item(p, sc, walk, it)) {
        const Unit un = it.un;
        const int row0 = un.m_blk * sc.rows_per_tile + sc.rank * BM;
        // A pair's CTAs each load half of the unit's columns (64-column chunks).
        const bool one_head = un.half >= 0;
        const int chunks = kPair ? (one_head ? 1 : 2) : R::B_CHUNKS;
        const int col0 = un.n_blk * BN +
                         (kPair ? (one_head ? un.half * 128 + sc.rank * 64 : sc.rank * 128) : 0);
        const uint32_t stage_tx = kPair ? 2u * (A_STAGE_BYTES + chunks * B_CHUNK_BYTES)
                                        : R::STAGE_TX;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
            if (early > 0) {                        // loaded above (first item, first stages)
                --early;
                if (++stage == R::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
                continue;
            }
            if (*abort_flag || !fu_wait_parity(b.empty + 8 * stage, phase ^ 1u, abort_flag,
                                               p.timeout_ns, p.status, W_EMPTY)) {
                ok = false;
                break;
            }
            const uint32_t adst = a0 + stage * A_STAGE_BYTES;
            const uint32_t bdst = b0 + stage * R::B_STAGE_BYTES;
            if (kPair) {
                // Both CTAs' bytes are counted on the leader's barrier.
                const uint32_t full = map_cluster_smem(b.full + 8 * stage, 0);
                if (sc.rank == 0) mbar_arrive_expect_tx(b.full + 8 * stage, stage_tx);
                tma_load_2d_pair(adst, &p.tm_x, full, kb * BK, row0);
                for (int c = 0; c < chunks; ++c)
                    tma_load_2d_pair(bdst + c * B_CHUNK_BYTES, &p.tm_w, full, col0 + c * 64,
                                     kb * BK);
            } else {
                const uint32_t full = b.full + 8 * stage;
                mbar_arrive_expect_tx(full, stage_tx);
                tma_load_2d(adst, &p.tm_x, full, kb * BK, row0);
#pragma unroll
                for (int c = 0; c < R::B_CHUNKS; ++c)
                    tma_load_2d(bdst + c * B_CHUNK_BYTES, &p.tm_w, full, col0 + c * 64, kb * BK);
            }
            issued_mask |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == R::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    if (!ok) {
        if (kPair) {
            // This CTA's loads are counted on the leader's barriers; give any
            // still in flight time to land before shared memory is released.
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 100000) {
            }
        } else {
            // Loads already issued must land before this CTA's shared memory is released.
            for (int s = 0; s < R::STAGES; ++s)
                if (issued_mask & (1u << s))
                    drain_wait(b.full + 8 * s, (last_parity >> s) & 1u, p.timeout_ns, p.status);
        }
    }
}

template <bool kPair>
__device__ void run_mma(const QkvParams& p, const Sched& sc, uint8_t* smem, uint32_t tmem_base,
                        const Bars& b, volatile int* abort_flag) {
    using R = Ring<kPair>;
    // kPair: M = 256 over the pair, each CTA's B holds N/2 = 128 columns.
    constexpr uint32_t idesc_full = make_idesc_bf16_f32(kPair ? 2 * BM : BM, BN,
                                                        /*a_mn_major=*/false,
                                                        /*b_mn_major=*/true);
    constexpr uint32_t idesc_head = make_idesc_bf16_f32(kPair ? 2 * BM : BM, BN / 2, false, true);
    const uint32_t a0 = smem_u32(smem + OFF_A);
    const uint32_t b0 = smem_u32(smem + R::OFF_B);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    Walk walk = make_walk(p, sc);
    Item it;
    for (; ok && next_item(p, sc, walk, it); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (*abort_flag || !fu_wait_parity(b.tempty + 8 * acc, acc_phase ^ 1u, abort_flag,
                                           p.timeout_ns, p.status, W_TEMPTY)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t idesc = it.un.half >= 0 ? idesc_head : idesc_full;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
            if (!fu_wait_parity(b.full + 8 * stage, phase, abort_flag, p.timeout_ns, p.status,
                                W_FULL)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a_base = a0 + stage * A_STAGE_BYTES;
            const uint32_t b_base = b0 + stage * R::B_STAGE_BYTES;
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
                // A: K-major, 128B swizzle; K advances 32 bytes inside the swizzle row.
                const uint64_t adesc = make_smem_desc_sw128(a_base + k * UMMA_K * 2, 16, 1024);
                // B: MN-major, 128B swizzle; 64-column chunks are B_CHUNK_BYTES apart
                // (leading offset), 8-row groups 1024 bytes apart (stride offset).
                const uint64_t bdesc =
                    make_smem_desc_sw128(b_base + k * UMMA_K * 128, B_CHUNK_BYTES, 1024);
                const uint32_t accum = (kb != it.kb0 || k != 0) ? 1u : 0u;
                if (kPair)
                    tc_mma_bf16_pair(d_tmem, adesc, bdesc, idesc, accum);
                else
                    tc_mma_bf16(d_tmem, adesc, bdesc, idesc, accum);
            }
            // Frees the stage (in both CTAs of a pair) when these MMAs finish.
            if (kPair)
                tc_commit_pair_mc(b.empty + 8 * stage, 0x3);
            else
                tc_commit(b.empty + 8 * stage);
            if (++stage == R::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (ok) {                                   // accumulator ready for the epilogue
            if (kPair)
                tc_commit_pair_mc(b.tfull + 8 * acc, 0x3);
            else
                tc_commit(b.tfull + 8 * acc);
        }
    }
    // Every MMA this thread issued must finish before TMEM is released.
    if (kPair)
        tc_commit_pair_mc(b.mma_done, 0x1);
    else
        tc_commit(b.mma_done);
    drain_wait(b.mma_done, 0, p.timeout_ns, p.status);
}

// Position of token row m, clamped (and reported) when outside the cache.
__device__ __forceinline__ const float* rope_row_for(const QkvParams& p, int m, bool row_valid) {
    int64_t pos = 0;
    if (row_valid) {
        pos = __ldg(p.positions + m);
        if (pos < 0 || pos >= p.rope_rows) {
            report_status(p.status, FU_DEV_POSITION_RANGE, 0);
            pos = 0;
        }
    }
    return p.rope + pos * 128;
}

// One half (cos or sin: 64 floats) of the rope rows of a warp's 32 token
// rows, into registers of the lane that owns each row.  A row-per-lane load
// would touch 32 cache lines per instruction; instead two rows per
// instruction are copied with coalesced 16-byte cp.async into the warp's
// staging boxes (8 KiB, 16-byte chunks XOR-swizzled by row so that the
// row-per-lane reads hit distinct banks), then each lane reads its own row.
// The staging boxes must be free (no bulk store still reading them).
__device__ __forceinline__ void load_rope_half(const float* my_row, int off, uint32_t buf,
                                               int lane, float4 (&out)[16]) {
    const int c = lane & 15;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int r = 2 * k + (lane >> 4);
        const float* src = reinterpret_cast<const float*>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_row), r));
        cp_async_16(buf + r * 256 + ((c ^ (r & 7)) << 4), src + off + 4 * c);
    }
    cp_async_wait_all();
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = ld_shared_f4(buf + lane * 256 + ((i ^ (lane & 7)) << 4));
    __syncwarp();
}

// Everything after the projection for one head row, read from TMEM lane
// `taddr` (this thread's token row, the head's first column): optional
// projection dump, RMSNorm + RoPE for Q/K (V as is), swizzled staging, and
// the warp's two bulk tensor stores of its 32-row box into the destination
// rank's receive buffer.  Pass 1 (Q/K) sums the squares of the BF16-rounded
// projection; pass 2 re-reads TMEM sixteen lo/hi column pairs at a time, so
// the head row never has to be held in registers next to its cos|sin.
__device__ __forceinline__ void emit_head(const QkvParams& p, uint32_t taddr, int h, int m,
                                          bool row_valid, int box_row0,
                                          const float4 (&cosv)[16], const float4 (&sinv)[16],
                                          const float* gam, uint8_t* box_lo, uint8_t* box_hi,
                                          int lane) {
    const uint32_t swz_row = lane * 128;
    const int swz = lane & 7;
    int comp, head_id, per_gpu;
    if (h < p.q_heads) {
        comp = 0; head_id = h; per_gpu = p.q_per_gpu;
    } else if (h < p.q_heads + p.kv_heads) {
        comp = 1; head_id = h - p.q_heads; per_gpu = p.kv_per_gpu;
    } else {
        comp = 2; head_id = h - p.q_heads - p.kv_heads; per_gpu = p.kv_per_gpu;
    }
    const int dst = head_id / per_gpu;
    const int dst_col = head_id % per_gpu;

    float scale = 0.f;
    if (comp < 2) {
        // Sum of the 128 squares in the order of torch's CPU reduction, so the
        // result is bit-identical: four accumulators of eight lanes, where
        // accumulator k, lane l sums columns 32c + 8k + l over c = 0..3; the
        // accumulators are added in order k = 0..3 (into lane[l]) and then the
        // lanes l = 0..7 left to right.  One accumulator at a time keeps only
        // the eight lane sums live next to the cos|sin registers.
        float lane[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t r[4][8];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld_8cols(taddr + 32 * c + 8 * k, r[c]);
            tmem_ld_wait();
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float f = __uint_as_float(r[c][l]);
                    if (!p.fp32_epilogue) f = bf16_round(f);
                    const float sq = __fmul_rn(f, f);
                    acc = c == 0 ? sq : __fadd_rn(acc, sq);
                }
                lane[l] = k == 0 ? acc : __fadd_rn(lane[l], acc);
            }
        }
        float ss = lane[0];
#pragma unroll
        for (int l = 1; l < 8; ++l) ss = __fadd_rn(ss, lane[l]);
        const float eps = comp == 0 ? p.q_eps : p.k_eps;
        scale = norm_scale(ss, eps);
    }

    // The staging boxes must have been read by the previous store.
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();

    const float* g = gam + (comp < 2 ? comp : 0) * 128;
    const bool r16 = !p.fp32_epilogue;          // the reference path's BF16 boundaries
#pragma unroll
    for (int q = 0; q < 4; ++q) {               // columns 16q..16q+15 and 64+16q..
        uint32_t lo_raw[16], hi_raw[16];
        tmem_ld_16cols(taddr + 16 * q, lo_raw);
        tmem_ld_16cols(taddr + 64 + 16 * q, hi_raw);
        tmem_ld_wait();
        // The projection as the epilogue sees it: rounded to BF16 (reference
        // PyTorch path) or the FP32 accumulator (FP32-intermediate mode).
        float lo_v[16], hi_v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            lo_v[i] = round_if(__uint_as_float(lo_raw[i]), r16);
            hi_v[i] = round_if(__uint_as_float(hi_raw[i]), r16);
        }
        if (p.gemm_out != nullptr && row_valid) {
            __nv_bfloat16* row = p.gemm_out + static_cast<int64_t>(m) * p.N + h * 128;
            uint4* dlo = reinterpret_cast<uint4*>(row + 16 * q);
            uint4* dhi = reinterpret_cast<uint4*>(row + 64 + 16 * q);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                dlo[c] = make_uint4(pack_bf16x2(lo_v[8 * c], lo_v[8 * c + 1]),
                                    pack_bf16x2(lo_v[8 * c + 2], lo_v[8 * c + 3]),
                                    pack_bf16x2(lo_v[8 * c + 4], lo_v[8 * c + 5]),
                                    pack_bf16x2(lo_v[8 * c + 6], lo_v[8 * c + 7]));
                dhi[c] = make_uint4(pack_bf16x2(hi_v[8 * c], hi_v[8 * c + 1]),
                                    pack_bf16x2(hi_v[8 * c + 2], hi_v[8 * c + 3]),
                                    pack_bf16x2(hi_v[8 * c + 4], hi_v[8 * c + 5]),
                                    pack_bf16x2(hi_v[8 * c + 6], hi_v[8 * c + 7]));
            }
        }
        uint32_t olo[8], ohi[8];
        if (comp < 2) {
            const float cs[16] = {cosv[4 * q].x, cosv[4 * q].y, cosv[4 * q].z, cosv[4 * q].w,
                                  cosv[4 * q + 1].x, cosv[4 * q + 1].y, cosv[4 * q + 1].z,
                                  cosv[4 * q + 1].w, cosv[4 * q + 2].x, cosv[4 * q + 2].y,
                                  cosv[4 * q + 2].z, cosv[4 * q + 2].w, cosv[4 * q + 3].x,
                                  cosv[4 * q + 3].y, cosv[4 * q + 3].z, cosv[4 * q + 3].w};
            const float sn[16] = {sinv[4 * q].x, sinv[4 * q].y, sinv[4 * q].z, sinv[4 * q].w,
                                  sinv[4 * q + 1].x, sinv[4 * q + 1].y, sinv[4 * q + 1].z,
                                  sinv[4 * q + 1].w, sinv[4 * q + 2].x, sinv[4 * q + 2].y,
                                  sinv[4 * q + 2].z, sinv[4 * q + 2].w, sinv[4 * q + 3].x,
                                  sinv[4 * q + 3].y, sinv[4 * q + 3].z, sinv[4 * q + 3].w};
            // Gamma for columns 16q.. and 64+16q.. (same address in every lane: a
            // broadcast, read as 16-byte vectors).
            float gl[16], gh[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 a = reinterpret_cast<const float4*>(g + 16 * q)[i];
                const float4 b4 = reinterpret_cast<const float4*>(g + 64 + 16 * q)[i];
                gl[4 * i] = a.x; gl[4 * i + 1] = a.y; gl[4 * i + 2] = a.z; gl[4 * i + 3] = a.w;
                gh[4 * i] = b4.x; gh[4 * i + 1] = b4.y; gh[4 * i + 2] = b4.z; gh[4 * i + 3] = b4.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                // RMSNorm, * gamma, BF16 boundary (torch_base.py:56-61).
                const float nl0 =
                    round_if(__fmul_rn(__fmul_rn(lo_v[2 * i], scale), gl[2 * i]), r16);
                const float nl1 =
                    round_if(__fmul_rn(__fmul_rn(lo_v[2 * i + 1], scale), gl[2 * i + 1]), r16);
                const float nh0 =
                    round_if(__fmul_rn(__fmul_rn(hi_v[2 * i], scale), gh[2 * i]), r16);
                const float nh1 =
                    round_if(__fmul_rn(__fmul_rn(hi_v[2 * i + 1], scale), gh[2 * i + 1]), r16);
                // NeoX rotation, separately rounded products (torch_base.py:62-63).
                const float c0 = cs[2 * i], c1 = cs[2 * i + 1];
                const float s0 = sn[2 * i], s1 = sn[2 * i + 1];
                olo[i] = pack_bf16x2(__fsub_rn(__fmul_rn(nl0, c0), __fmul_rn(nh0, s0)),
                                     __fsub_rn(__fmul_rn(nl1, c1), __fmul_rn(nh1, s1)));
                ohi[i] = pack_bf16x2(__fadd_rn(__fmul_rn(nh0, c0), __fmul_rn(nl0, s0)),
                                     __fadd_rn(__fmul_rn(nh1, c1), __fmul_rn(nl1, s1)));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                olo[i] = pack_bf16x2(lo_v[2 * i], lo_v[2 * i + 1]);
                ohi[i] = pack_bf16x2(hi_v[2 * i], hi_v[2 * i + 1]);
            }
        }
        // 16-byte chunks 2q and 2q+1 of the row in each box (128-byte swizzle).
        const uint32_t off0 = swz_row + (((2 * q) ^ swz) << 4);
        const uint32_t off1 = swz_row + (((2 * q + 1) ^ swz) << 4);
        *reinterpret_cast<uint4*>(box_lo + off0) = make_uint4(olo[0], olo[1], olo[2], olo[3]);
        *reinterpret_cast<uint4*>(box_lo + off1) = make_uint4(olo[4], olo[5], olo[6], olo[7]);
        *reinterpret_cast<uint4*>(box_hi + off0) = make_uint4(ohi[0], ohi[1], ohi[2], ohi[3]);
        *reinterpret_cast<uint4*>(box_hi + off1) = make_uint4(ohi[4], ohi[5], ohi[6], ohi[7]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        // Rows past L in this source's batch are clipped by the tensor map.
        const CUtensorMap* tm = &p.tm_out[comp * FU_MAX_SP + dst];
        tma_store_3d(tm, smem_u32(box_lo), dst_col * 128, box_row0, p.sp_rank);
        tma_store_3d(tm, smem_u32(box_hi), dst_col * 128 + 64, box_row0, p.sp_rank);
        bulk_commit_group();
    }
}

template <bool kPair>
__device__ void run_epilogue(const QkvParams& p, const Sched& sc, uint8_t* smem,
                             uint32_t tmem_base, const Bars& b, const float* gam,
                             volatile int* abort_flag, uint32_t epoch) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int quarter = warp & 3;           // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* box_lo = smem + OFF_STG + (warp - 2) * STAGING_PER_WARP;
    uint8_t* box_hi = box_lo + BOX_BYTES;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // Every epilogue thread reaches this barrier; on failure nothing is stored.
    if (!wait_peers_entered(p, epoch, abort_flag, kPair, status_at_start(p))) return;

    int local = 0;
    Walk walk = make_walk(p, sc);
    Item it;
    for (; next_item(p, sc, walk, it); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const Unit un = it.un;
        const int m_blk = un.m_blk;
        const int n_blk = un.n_blk;
        const int row_base = m_blk * sc.rows_per_tile + sc.rank * BM;
        const int m = row_base + row_in_tile;
        const bool row_valid = m < p.L;
        // This row's cos|sin, fetched while the tensor cores still work on the
        // tile (shared by both heads).
        float4 cosv[16], sinv[16];
        {
            const float* rope_row = rope_row_for(p, m, row_valid);
            if (lane == 0) bulk_wait_read_all();       // staging boxes free
            __syncwarp();
            load_rope_half(rope_row, 0, smem_u32(box_lo), lane, cosv);
            load_rope_half(rope_row, 64, smem_u32(box_lo), lane, sinv);
        }
        if (!fu_wait_parity(b.tfull + 8 * acc, acc_phase, abort_flag, p.timeout_ns, p.status,
                            W_TFULL))
            break;
        tc_fence_after();
        const uint32_t acc_addr = tmem_base + lane_addr + acc * BN;
        // Heads of this unit: both of the tile (odd head count: the last tile
        // has one), or the single head of a one-head unit (accumulator column 0).
        const int h0 = n_blk * 2 + (un.half >= 0 ? un.half : 0);
        const int heads_here = un.half >= 0 ? (h0 < p.heads ? 1 : 0) : min(2, p.heads - h0);
#pragma unroll 1
        for (int hs = 0; hs < heads_here; ++hs)
            emit_head(p, acc_addr + hs * 128, h0 + hs, m, row_valid, row_base + quarter * 32,
                      cosv, sinv, gam, box_lo, box_hi, lane);
        // Both heads of this accumulator have been read: hand TMEM back (to
        // the pair leader's MMA issuer, which counts both CTAs' threads).
        tc_fence_before();
        if (kPair && sc.rank != 0)
            mbar_arrive_remote(map_cluster_smem(b.tempty + 8 * acc, 0));
        else
            mbar_arrive(b.tempty + 8 * acc);
    }
    if (lane == 0) {
        bulk_wait_all();                    // peer writes performed
        fence_proxy_async_global();
    }
    __syncwarp();
}

// Split mode, step 1 (epilogue warps): park this CTA's FP32 partial
// accumulator of the tile in its own shared memory (the operand ring, idle by
// now), rows of PART_STRIDE bytes.  Only warps holding valid rows copy.
__device__ void run_split_partial(const QkvParams& p, const Sched& sc, uint8_t* smem,
                                  uint32_t tmem_base, const Bars& b, volatile int* abort_flag) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int quarter = warp & 3;
    const int m_blk = decode_unit(p, sc.first).m_blk;
    // Read now, used by the reduction's entry barrier (after the main loop).
    if (threadIdx.x == 64) *reinterpret_cast<volatile int32_t*>(smem + OFF_MISC + 12) =
        status_at_start(p);
    // While the tensor cores work: this tile's token positions, validated, as
    // RoPE row indices in shared memory (the staging area is unused in split
    // mode), and the RoPE rows prefetched into L2, so that the reduction's
    // per-item chain is one L2 hit instead of two dependent loads.
    {
        const int row = threadIdx.x - 64;
        const int m = m_blk * BM + row;
        int32_t rope_row = 0;
        if (m < p.L) {
            const int64_t pos = __ldg(p.positions + m);
            if (pos < 0 || pos >= p.rope_rows)
                report_status(p.status, FU_DEV_POSITION_RANGE, 0);
            else
                rope_row = static_cast<int32_t>(pos);
            const int n_blk = decode_unit(p, sc.first).n_blk;
            if (n_blk * 2 < p.q_heads + p.kv_heads) {          // a Q/K head in this tile
                const float* r = p.rope + static_cast<int64_t>(rope_row) * 128;
#pragma unroll
                for (int c = 0; c < 4; ++c) prefetch_l2(r + 32 * c);
            }
        }
        reinterpret_cast<int32_t*>(smem + OFF_STG)[row] = rope_row;
    }
    if (p.split_push && cluster_ctarank() == 0) {
        // The leader reduces every item: bring the valid rows' cos|sin into
        // shared memory now, 16 bytes per thread per step.
        named_bar_sync(1, NUM_EPI_THREADS);          // the row indices above
        const int32_t* rows_idx = reinterpret_cast<const int32_t*>(smem + OFF_STG);
        const uint32_t dst = smem_u32(smem + push_rope_offset(p));
        for (int i = threadIdx.x - 64; i < p.L * 32; i += NUM_EPI_THREADS) {
            const int r = i >> 5, c = i & 31;
            cp_async_16(dst + r * ROPE_ROW_BYTES + c * 16,
                        p.rope + static_cast<int64_t>(rows_idx[r]) * 128 + c * 4);
        }
        cp_async_wait_all();
    }
    if (!fu_wait_parity(b.tfull, 0, abort_flag, p.timeout_ns, p.status, W_TFULL)) return;
    tc_fence_after();
    if (m_blk * BM + quarter * 32 >= p.L) return;          // no valid row in this warp
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    if (p.split_push) {
        // Push mode (a single block of at most a few rows): this rank's slot.
        const int r = quarter * 32 + lane;
        float* slot = reinterpret_cast<float*>(
            smem + OFF_PUSH + (static_cast<int>(cluster_ctarank()) * p.L + r) * PUSH_ROW_BYTES);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32cols(tmem_base + lane_addr + c * 32, v);
            tmem_ld_wait();
            if (r < p.L)
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    reinterpret_cast<float4*>(slot + c * 32)[i] =
                        make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                    __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        }
        fence_proxy_async_smem();          // read next by a bulk copy (async proxy)
        return;
    }
    float* row = reinterpret_cast<float*>(smem + OFF_A + (quarter * 32 + lane) * PART_STRIDE);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32cols(tmem_base + lane_addr + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
            reinterpret_cast<float4*>(row + c * 32)[i] =
                make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                            __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
    }
}

// Split mode, step 2 (every warp of every cluster CTA, after a cluster
// barrier): one item = one valid token row x one head.  A warp takes two items
// at a time; lane l owns columns 4l..4l+3 of the head, loads the partials of
// every cluster CTA at once (coalesced distributed-shared-memory reads) and
// sums them in rank order (deterministic).  The RMSNorm sum is a warp
// reduction, the NeoX partner of lane l is lane l^16, and the row leaves as
// one coalesced 256-byte store into the destination rank's receive buffer.
// cos|sin of columns 4l..4l+3 (mod 64) at token row m's position, for a Q/K
// head (V heads are not rotated); issued before the partial sums are read so
// the two latencies overlap.
struct SplitRope {
    float4 cs, sn;
};

__device__ __forceinline__ SplitRope split_item_rope(const QkvParams& p, const int32_t* rope_rows,
                                                    int row, int h, int lane) {
    SplitRope r;
    r.cs = r.sn = make_float4(0.f, 0.f, 0.f, 0.f);
    if (h < p.q_heads + p.kv_heads) {
        const float* base = p.rope + static_cast<int64_t>(rope_rows[row]) * 128 + 4 * (lane & 15);
        r.cs = __ldg(reinterpret_cast<const float4*>(base));
        r.sn = __ldg(reinterpret_cast<const float4*>(base + 64));
    }
    return r;
}

__device__ __forceinline__ void split_item_emit(const QkvParams& p, const float4& acc, int m,
                                                int h, const float* gam, int lane,
                                                const SplitRope& rope) {
    // BF16 projection of columns 4l..4l+3 of head h, token row m.
    const uint32_t u0 = pack_bf16x2(acc.x, acc.y);
    const uint32_t u1 = pack_bf16x2(acc.z, acc.w);
    const bool r16 = !p.fp32_epilogue;
    float v[4];
    if (r16) {
        const float2 a = unpack_bf16x2(u0), b = unpack_bf16x2(u1);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
        v[0] = acc.x; v[1] = acc.y; v[2] = acc.z; v[3] = acc.w;
    }
    if (p.gemm_out != nullptr)
        *reinterpret_cast<uint2*>(p.gemm_out + static_cast<int64_t>(m) * p.N + h * 128 + 4 * lane) =
            make_uint2(u0, u1);
    int comp, head_id, per_gpu;
    if (h < p.q_heads) {
        comp = 0; head_id = h; per_gpu = p.q_per_gpu;
    } else if (h < p.q_heads + p.kv_heads) {
        comp = 1; head_id = h - p.q_heads; per_gpu = p.kv_per_gpu;
    } else {
        comp = 2; head_id = h - p.q_heads - p.kv_heads; per_gpu = p.kv_per_gpu;
    }
    const int dst = head_id / per_gpu;
    const int dst_col = head_id % per_gpu;
    uint2 out = make_uint2(u0, u1);
    if (comp < 2) {
        // The sum of squares in the order of torch's CPU reduction (as in
        // emit_head): column j = 4 lane + e belongs to accumulator k =
        // (lane / 2) % 4, eight-lane slot 4 (lane % 2) + e, step lane / 8.
        // Every shuffle reads values that no earlier step of this sum changed.
        float sq[4], acc[4], a[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = sq[e] = __fmul_rn(v[e], v[e]);
#pragma unroll
        for (int step = 8; step <= 24; step += 8) {        // steps 1..3 into lanes 0..7
#pragma unroll
            for (int e = 0; e < 4; ++e)
                acc[e] = __fadd_rn(acc[e], __shfl_down_sync(0xffffffffu, sq[e], step));
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) a[e] = acc[e];
#pragma unroll
        for (int k = 2; k <= 6; k += 2) {                  // accumulators 1..3 into lanes 0, 1
#pragma unroll
            for (int e = 0; e < 4; ++e)
                a[e] = __fadd_rn(a[e], __shfl_down_sync(0xffffffffu, acc[e], k));
        }
        float hi[4];                                         // slots 4..7 (lane 1) to lane 0
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[e] = __shfl_down_sync(0xffffffffu, a[e], 1);
        float ss = a[0];
#pragma unroll
        for (int e = 1; e < 4; ++e) ss = __fadd_rn(ss, a[e]);
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, hi[e]);
        ss = __shfl_sync(0xffffffffu, ss, 0);
        const float eps = comp == 0 ? p.q_eps : p.k_eps;
        const float scale = norm_scale(ss, eps);
        const float* g = gam + comp * 128 + 4 * lane;
        float n[4], partner[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) n[i] = round_if(__fmul_rn(__fmul_rn(v[i], scale), g[i]), r16);
#pragma unroll
        for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, n[i], 16);
        const float c4[4] = {rope.cs.x, rope.cs.y, rope.cs.z, rope.cs.w};
        const float s4[4] = {rope.sn.x, rope.sn.y, rope.sn.z, rope.sn.w};
        float r[4];
        if (lane < 16) {        // lo half: lo*cos - hi*sin
#pragma unroll
            for (int i = 0; i < 4; ++i)
                r[i] = __fsub_rn(__fmul_rn(n[i], c4[i]), __fmul_rn(partner[i], s4[i]));
        } else {                // hi half: hi*cos + lo*sin
#pragma unroll
            for (int i = 0; i < 4; ++i)
                r[i] = __fadd_rn(__fmul_rn(n[i], c4[i]), __fmul_rn(partner[i], s4[i]));
        }
        out = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
    }
    const int64_t cols = static_cast<int64_t>(per_gpu) * 128;
    __nv_bfloat16* base = static_cast<__nv_bfloat16*>(p.out_base[comp * FU_MAX_SP + dst]);
    *reinterpret_cast<uint2*>(base + (static_cast<int64_t>(p.sp_rank) * p.L + m) * cols +
                              dst_col * 128 + 4 * lane) = out;
}

__device__ void run_split_reduce(const QkvParams& p, const Sched& sc, uint8_t* smem,
                                 const float* gam, volatile int* abort_flag, uint32_t epoch) {
    // The reduction reads every cluster CTA's partial: if any of them gave up
    // (its partial is incomplete), this CTA stores nothing either.  All flags
    // are requested before any is examined, so the reads overlap.
    if (threadIdx.x == 64) {
        const uint32_t flag_addr = smem_u32(const_cast<int*>(abort_flag));
        uint32_t flags[FU_MAX_SP];
#pragma unroll
        for (int r = 0; r < FU_MAX_SP; ++r)
            flags[r] = r < p.splits ? ld_cluster_u32(map_cluster_smem(flag_addr, r)) : 0u;
        uint32_t any = 0;
#pragma unroll
        for (int r = 0; r < FU_MAX_SP; ++r) any |= flags[r];
        if (any) *abort_flag = 1;
    }
    const int32_t status_seen = *reinterpret_cast<volatile int32_t*>(smem + OFF_MISC + 12);
    if (!wait_peers_entered(p, epoch, abort_flag, false, status_seen, NUM_THREADS)) return;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Unit tile = decode_unit(p, sc.first);
    const int m_blk = tile.m_blk;
    const int n_blk = tile.n_blk;
    const int rows = min(BM, p.L - m_blk * BM);
    const int heads_here = min(2, p.heads - n_blk * 2);
    const int items = rows * heads_here;
    // Every warp of every cluster CTA takes items: the producer and MMA warps
    // are idle by now, and each item's chain of shuffles and roundings is
    // latency-bound, so more warps in flight shorten the reduction.
    const int workers = NUM_THREADS / 32 * p.splits;
    const uint32_t part = smem_u32(smem + OFF_A);
    const int32_t* rope_rows = reinterpret_cast<const int32_t*>(smem + OFF_STG);
    // Item i: row i / heads_here, head slot i % heads_here.  A warp takes two
    // items per step (i0 and i0 + workers).  Each step first sums the partials
    // requested by the previous step (in rank order: deterministic), then
    // requests the next step's partials over distributed shared memory and its
    // RoPE values, and only then normalises, rotates and stores the current
    // items, so the remote reads of one step overlap the arithmetic of the
    // step before.
    struct Raw {
        float4 v[2][FU_MAX_SP];
        SplitRope rope[2];
    };
    auto request = [&](int i0, Raw& raw) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = min(i0 + k * workers, items - 1);
            raw.rope[k] = split_item_rope(p, rope_rows, i / heads_here,
                                          n_blk * 2 + i % heads_here, lane);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = min(i0 + k * workers, items - 1);
            const uint32_t local = part + (i / heads_here) * PART_STRIDE +
                                   ((i % heads_here) * 128 + 4 * lane) * 4;
#pragma unroll
            for (int r = 0; r < FU_MAX_SP; ++r)
                if (r < p.splits) raw.v[k][r] = ld_cluster_f32x4(map_cluster_smem(local, r));
        }
    };
    const int first = warp * p.splits + sc.split;
    Raw raw;
    if (first < items) request(first, raw);
    for (int i0 = first; i0 < items; i0 += 2 * workers) {
        float4 acc[2];
        SplitRope rope[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            acc[k] = raw.v[k][0];
#pragma unroll
            for (int r = 1; r < FU_MAX_SP; ++r)
                if (r < p.splits) {
                    acc[k].x += raw.v[k][r].x; acc[k].y += raw.v[k][r].y;
                    acc[k].z += raw.v[k][r].z; acc[k].w += raw.v[k][r].w;
                }
            rope[k] = raw.rope[k];
        }
        if (i0 + 2 * workers < items) request(i0 + 2 * workers, raw);
        // One copy of the item code, looped: the step's code then stays in the
        // instruction cache (two inlined copies made the warps wait on
        // instruction fetch for most of each step).
#pragma unroll 1
        for (int k = 0; k < 2; ++k) {
            const int i = i0 + k * workers;
            if (i < items)
                split_item_emit(p, acc[0], m_blk * BM + i / heads_here,
                                n_blk * 2 + i % heads_here, gam, lane, rope[0]);
            acc[0] = acc[1];                    // the second item moves up
            rope[0] = rope[1];
        }
    }
}

// Split push mode, the leader's epilogue warps: every rank's rows of the
// single row block are in this CTA's shared memory, [rank][row][256 cols].
// One item = one valid token row x one head, one warp per item, lane l owning
// columns 4l..4l+3; partials summed in rank order (deterministic), then the
// same normalisation, rotation and store as the distributed reduction.
__device__ void run_split_push_reduce(const QkvParams& p, const Sched& sc, uint8_t* smem,
                                      const float* gam, volatile int* abort_flag,
                                      uint32_t epoch) {
    const int32_t status_seen = *reinterpret_cast<volatile int32_t*>(smem + OFF_MISC + 12);
    if (!wait_peers_entered(p, epoch, abort_flag, false, status_seen)) return;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Unit tile = decode_unit(p, sc.first);
    const int rows = p.L;
    const int heads_here = min(2, p.heads - tile.n_blk * 2);
    const int items = rows * heads_here;
    const float* rope_smem = reinterpret_cast<const float*>(smem + push_rope_offset(p));
    const float* slots = reinterpret_cast<const float*>(smem + OFF_PUSH);
    for (int i = warp - 2; i < items; i += NUM_EPI_THREADS / 32) {
        const int r = i / heads_here, hs = i % heads_here;
        const int h = tile.n_blk * 2 + hs;
        SplitRope rope;
        rope.cs = rope.sn = make_float4(0.f, 0.f, 0.f, 0.f);
        if (h < p.q_heads + p.kv_heads) {
            const float* cs = rope_smem + r * 128 + 4 * (lane & 15);
            rope.cs = *reinterpret_cast<const float4*>(cs);
            rope.sn = *reinterpret_cast<const float4*>(cs + 64);
        }
        float4 acc = reinterpret_cast<const float4*>(slots + r * BN + hs * 128)[lane];
        for (int k = 1; k < p.splits; ++k) {
            const float4 v =
                reinterpret_cast<const float4*>(slots + (k * rows + r) * BN + hs * 128)[lane];
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        split_item_emit(p, acc, r, h, gam, lane, rope);
    }
}

// ------------------------------------------------------------ kernel
template <bool kPair>
__global__ void __launch_bounds__(NUM_THREADS, 1)
fused_qkv_exchange_kernel(const __grid_constant__ QkvParams p) {
    using R = Ring<kPair>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Sched sc = make_sched<kPair>(p);
    const bool split_mode = !kPair && p.splits > 1;
    const Bars b(smem_u32(smem + OFF_BAR));
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    float* gam = reinterpret_cast<float*>(smem + OFF_GAMMA);

    uint32_t* my_sync = p.sync[p.sp_rank];
    uint32_t* epoch_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC + 8);
    // Prologue: shared memory, TMEM and parameters only, so that under a
    // programmatic dependent launch it overlaps the previous kernel's tail.
    if (threadIdx.x == 0) {
        for (int s = 0; s < R::STAGES; ++s) {
            mbar_init(b.full + 8 * s, 1);
            mbar_init(b.empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(b.tfull + 8 * a, 1);
            // A pair's leader counts the epilogue threads of both CTAs.
            mbar_init(b.tempty + 8 * a, kPair ? 2 * NUM_EPI_THREADS : NUM_EPI_THREADS);
        }
        mbar_init(b.mma_done, 1);
        if (p.split_push && cluster_ctarank() == 0) {
            mbar_init(b.push, 1);
            // Every other rank's rows arrive by bulk copy.
            const int rows = p.L;
            mbar_arrive_expect_tx(b.push, static_cast<uint32_t>((p.splits - 1) * rows * PUSH_ROW_BYTES));
        }
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&p.tm_x);
        tma_prefetch_desc(&p.tm_w);
        // Static weights (the caller's promise that no kernel still running on
        // the stream writes W): the first stages' W streams in while the
        // previous kernel finishes.  X and everything else wait for it.
        load_early_w<kPair>(p, sc, smem, b);
    }
    if (warp == 1) {
        if (kPair) {
            tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
            tmem_relinquish();
        }
    }
    // Global memory from here on: the previous kernel of the stream is done.
    grid_dependency_wait();
    grid_launch_dependents();
    if (threadIdx.x == 0) {
        // This call's epoch: one past the last call's (the kernel advances it).
        const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_EPOCH) + 1;
        *epoch_slot = epoch;
        // "Entered e": this rank's stream has finished everything before this
        // call, so its earlier reads of the receive buffers are complete; the
        // flag carries no data, so posted (relaxed) stores suffice.
        if (blockIdx.x == 0 && p.sp_size > 1)
            for (int d = 0; d < p.sp_size; ++d)
                st_relaxed_sys_u32(p.sync[d] + FU_SYNC_ENTRY + p.sp_rank, epoch);
    }
    tc_fence_before();
    __syncthreads();
    // A pair's barriers and TMEM must exist in both CTAs before either uses them.
    if (kPair) cluster_sync_all();
    // Split push mode: the leader's push barrier exists before any rank copies
    // into it (this arrive, and the wait after the main loop).
    if (split_mode && p.split_push) cluster_arrive_relaxed();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const uint32_t epoch = *epoch_slot;

    if (warp == 0) {
        if (lane == 0) run_producer<kPair>(p, sc, smem, b, abort_flag);
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && (!kPair || sc.rank == 0))
            run_mma<kPair>(p, sc, smem, tmem_base, b, abort_flag);
        __syncwarp();
    } else {
        // The norm weights, staged by the epilogue warps (off the producer's
        // start-up path); the entry barrier's named barrier, or the split
        // reduction's cluster barrier, orders them before their first use.
        for (int i = threadIdx.x - 64; i < 256; i += NUM_EPI_THREADS)
            gam[i] = i < 128 ? p.q_gamma[i] : p.k_gamma[i - 128];
        if (split_mode)
            run_split_partial(p, sc, smem, tmem_base, b, abort_flag);
        else
            run_epilogue<kPair>(p, sc, smem, tmem_base, b, gam, abort_flag, epoch);
    }

    tc_fence_before();
    __syncthreads();
    // Both CTAs of a pair are done with TMEM (reads and the leader's MMAs).
    if (kPair) cluster_sync_all();
    tc_fence_after();
    if (warp == 1) {
        if (kPair)
            tmem_dealloc_pair(tmem_base, TMEM_COLS);
        else
            tmem_dealloc(tmem_base, TMEM_COLS);
    }

    if (split_mode && p.split_push) {
        // Every thread of every cluster CTA reaches both barriers on every path.
        cluster_wait();                     // the leader's push barrier exists
        const bool leader = cluster_ctarank() == 0;
        if (!leader && threadIdx.x == 64) {
            // This rank's rows (parked even after a failed wait, so the leader's
            // barrier completes; the leader checks the abort flags) to the leader.
            const uint32_t off = OFF_PUSH + cluster_ctarank() * p.L * PUSH_ROW_BYTES;
            bulk_copy_s2cluster(map_cluster_smem(smem_u32(smem + off), 0), smem_u32(smem + off),
                                static_cast<uint32_t>(p.L * PUSH_ROW_BYTES),
                                map_cluster_smem(b.push, 0));
        }
        if (leader && warp >= 2) {
            if (!drain_wait(b.push, 0, p.timeout_ns, p.status)) *abort_flag = 1;
            // A rank that gave up has pushed an incomplete partial: store nothing.
            // Its abort flag is read over distributed shared memory, so this must
            // come before the leader's arrive below: the other ranks may exit as
            // soon as every thread of the leader has arrived.
            if (threadIdx.x == 64) {
                const uint32_t flag_addr = smem_u32(const_cast<int*>(abort_flag));
                uint32_t flags[FU_MAX_SP];
#pragma unroll
                for (int r = 0; r < FU_MAX_SP; ++r)
                    flags[r] = r < p.splits ? ld_cluster_u32(map_cluster_smem(flag_addr, r)) : 0u;
                uint32_t any = 0;
#pragma unroll
                for (int r = 0; r < FU_MAX_SP; ++r) any |= flags[r];
                if (any) *abort_flag = 1;
            }
        }
        // The leader: every copy has landed (its mbarrier saw the bytes) and no
        // other rank's shared memory is read any more, so the others may exit.
        cluster_arrive_relaxed();
        if (leader && warp >= 2) {
            named_bar_sync(1, NUM_EPI_THREADS);
            if (*abort_flag == 0) run_split_push_reduce(p, sc, smem, gam, abort_flag, epoch);
        }
        cluster_wait();                     // the others keep their slots until then
    } else if (split_mode) {
        // Every CTA of the cluster reaches both barriers on every path, so a
        // CTA that gave up on a wait cannot strand its peers here.
        cluster_sync_all();                 // partials visible cluster-wide
        run_split_reduce(p, sc, smem, gam, abort_flag, epoch);   // all six warps
        cluster_sync_all();                 // peers are done reading this CTA's partial
    }

    // A world of one: no peer reads the exit flag, and the next call reads the
    // epoch only once this grid has completed, so CTA 0 alone advances it when
    // it is done (every CTA read this call's epoch at its start; one that
    // starts later -- a second wave of split clusters -- uses the epoch for
    // nothing) and no CTA counts in.
    if (p.sp_size == 1) {
        if (blockIdx.x == 0 && threadIdx.x == 64) {
            *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_EPOCH) = epoch;
            *reinterpret_cast<volatile uint32_t*>(my_sync) = epoch;
        }
        return;
    }
    // With peers: every CTA's output is complete (stores waited for, then the
    // barriers above); one system-scope fence per CTA makes its remote stores
    // visible beyond this GPU before it is counted, and the last CTA publishes
    // the epoch (cumulative over every counted CTA).
    if (threadIdx.x == 64) {
        const bool aborted = *abort_flag != 0;
        fence_acq_rel_sys();
        const uint32_t old =
            atom_add_acq_rel_gpu_u32(my_sync + FU_SYNC_COUNTER, aborted ? 0x10001u : 1u);
        if ((old & 0xFFFFu) == gridDim.x - 1) {
            // Last CTA: every CTA has read the epoch, so it can advance, and
            // the counter is ready for the next call.
            const bool any_abort = aborted || (old >> 16) != 0;
            *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_COUNTER) = 0u;
            *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_EPOCH) = epoch;
            // A failed call of a group marks the operator failed: calls queued
            // behind it skip their peer waits and stores.
            if (any_abort)
                *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_FAILED) = 1u;
            if (!any_abort) {
                // One system-scope fence orders every counted CTA's stores
                // (acquired through the counter) before all the flags; the
                // flags themselves are posted stores.
                fence_acq_rel_sys();
                for (int d = 0; d < p.sp_size; ++d)
                    st_relaxed_sys_u32(p.sync[d] + p.sp_rank, epoch);
                if (p.wait_peers) {
                    const uint64_t t0 = globaltimer_ns();
                    for (int s = 0; s < p.sp_size; ++s) {
                        while (static_cast<int32_t>(ld_acquire_sys_u32(my_sync + s) - epoch) < 0) {
                            if (globaltimer_ns() - t0 > p.timeout_ns) {
                                report_status(p.status, FU_DEV_PEER_TIMEOUT, s);
                                break;
                            }
                        }
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------ host side
static int encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                  const cuuint64_t* strides_bytes, const cuuint32_t* box, const char* what) {
    auto fn = encode_tiled_fn();
    if (fn == nullptr) return set_error(FU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint32_t elem_strides[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                    strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(FU_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what,
                         static_cast<int>(r));
    return FU_OK;
}

}  // namespace fu

struct fu_qkv_ctx {
    fu_qkv_topology topo;
    int sm_count = 0;
    int max_clusters[9] = {0};    // co-resident clusters of each size (index = CTAs per cluster)
    int max_pairs = 0;            // co-resident CTA pairs of the pair variant
    uint32_t epoch = 0;
    int last_grid = 0;
    // Tensor-map caches: encoded maps of recently seen inputs (weights are
    // typically one per layer, activations come from a few recycled buffers),
    // replaced round-robin, and the receive-buffer maps of the last length.
    struct MapEntry {
        const void* ptr = nullptr;
        int64_t rows = -1;
        CUtensorMap map;
    };
    static constexpr int kXMaps = 8, kWMaps = 16;
    MapEntry x_maps[kXMaps];
    MapEntry w_maps[kWMaps];
    int x_next = 0, w_next = 0;
    int64_t out_rows = -1;
    fu::QkvParams params;
};

using namespace fu;

// Split-K factor for `tiles` tiles of `kb` k-blocks with `rows` valid token
// rows per tile: 1 (persistent grid) unless a cluster split is estimated to be
// faster.  The estimates (microseconds) were fitted on B200 at H=4096:
//   persistent  12 + ceil(tiles / SMs) * 0.40 * kb
//   split s      8 + waves * (0.55 * ceil(kb / s) + 2.5 * ceil(2 rows / 8 s))
// (a split's CTAs share HBM bandwidth, and its reduction walks rows x 2 heads
// items two per warp over the cluster's 4 s epilogue warps).  `forced` (from
// FU_FWD_SPLITS in the call's flags) overrides the choice when the device can
// co-schedule clusters of that size.
static int choose_splits(const fu_qkv_ctx* ctx, int64_t tiles, int kb, int64_t rows, int forced) {
    if (forced >= 1 && forced <= 8)
        return forced <= kb && (forced == 1 || ctx->max_clusters[forced] > 0) ? forced : 1;
    const int64_t sms = ctx->sm_count;
    double best_cost = 12.0 + static_cast<double>((tiles + sms - 1) / sms) * 0.40 * kb;
    int best = 1;
    for (int s = 2; s <= 8 && s <= kb; ++s) {
        const int64_t cap = ctx->max_clusters[s];
        if (cap <= 0) continue;
        const int64_t waves = (tiles + cap - 1) / cap;
        const int64_t iters = (2 * rows + 8 * s - 1) / (8 * s);
        const double cost = 8.0 + static_cast<double>(waves) *
                                      (0.55 * ((kb + s - 1) / s) + 2.5 * static_cast<double>(iters));
        if (cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

extern "C" int fu_qkv_create(const fu_qkv_topology* topo, fu_qkv_ctx** out) {
    if (topo == nullptr || out == nullptr) return set_error(FU_ERR_INVALID, "null argument");
    const int S = topo->sp_size;
    if (S < 1 || S > FU_MAX_SP) return set_error(FU_ERR_INVALID, "sp_size %d not in [1, 8]", S);
    if (topo->sp_rank < 0 || topo->sp_rank >= S)
        return set_error(FU_ERR_INVALID, "sp_rank %d not in [0, %d)", topo->sp_rank, S);
    if (topo->q_heads <= 0 || topo->kv_heads <= 0 || topo->q_heads % S || topo->kv_heads % S)
        return set_error(FU_ERR_INVALID, "head counts (%d, %d) must be positive multiples of %d",
                         topo->q_heads, topo->kv_heads, S);
    if (topo->hidden_size <= 0 || topo->hidden_size % 64)
        return set_error(FU_ERR_INVALID, "hidden_size %lld must be a positive multiple of 64",
                         static_cast<long long>(topo->hidden_size));
    if (topo->capacity_rows < S || topo->capacity_rows % S)
        return set_error(FU_ERR_INVALID, "capacity_rows %lld must be a positive multiple of %d",
                         static_cast<long long>(topo->capacity_rows), S);
    for (int d = 0; d < S; ++d) {
        if (!topo->q_recv[d] || !topo->k_recv[d] || !topo->v_recv[d] || !topo->sync[d])
            return set_error(FU_ERR_INVALID, "missing buffer for SP member %d", d);
        if ((reinterpret_cast<uintptr_t>(topo->q_recv[d]) | reinterpret_cast<uintptr_t>(topo->k_recv[d]) |
             reinterpret_cast<uintptr_t>(topo->v_recv[d])) & 15)
            return set_error(FU_ERR_INVALID, "receive buffers must be 16-byte aligned");
    }
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || topo->device < 0 ||
        topo->device >= dev_count)
        return set_error(FU_ERR_INVALID, "device %d is not available", topo->device);
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, topo->device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, topo->device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, topo->device);
    if (major != 10 || minor != 0)
        return set_error(FU_ERR_UNSUPPORTED, "requires an sm_100 GPU (B200); device %d is sm_%d%d",
                         topo->device, major, minor);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(topo->device);
    cudaError_t e = cudaFuncSetAttribute(fused_qkv_exchange_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_qkv_exchange_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    cudaSetDevice(prev);
    if (e != cudaSuccess)
        return set_error(FU_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    auto* ctx = new fu_qkv_ctx();
    cudaSetDevice(topo->device);
    for (int cs = 2; cs <= 8; ++cs) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cs * 16, 1, 1);
        cfg.blockDim = dim3(NUM_THREADS, 1, 1);
        cfg.dynamicSmemBytes = SMEM_ALLOC;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = cs;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fused_qkv_exchange_kernel<false>, &cfg) !=
            cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        ctx->max_clusters[cs] = n;
        if (cs == 2) {
            n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, fused_qkv_exchange_kernel<true>, &cfg) !=
                cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
            ctx->max_pairs = n;
        }
    }
    cudaSetDevice(prev);
    ctx->topo = *topo;
    if (ctx->topo.timeout_ns == 0) ctx->topo.timeout_ns = FU_DEFAULT_TIMEOUT_NS;
    ctx->sm_count = sms;
    std::memset(&ctx->params, 0, sizeof(ctx->params));
    *out = ctx;
    return FU_OK;
}

extern "C" int fu_qkv_destroy(fu_qkv_ctx* ctx) {
    delete ctx;
    return FU_OK;
}

extern "C" uint32_t fu_qkv_epoch(const fu_qkv_ctx* ctx) { return ctx ? ctx->epoch : 0u; }
extern "C" int fu_qkv_last_grid(const fu_qkv_ctx* ctx) { return ctx ? ctx->last_grid : 0; }

extern "C" int fu_qkv_forward(fu_qkv_ctx* ctx, const void* x, const void* w,
                              const int64_t* positions, const float* q_gamma,
                              const float* k_gamma, const float* rope, int64_t local_tokens,
                              int64_t rope_rows, double q_epsilon, double k_epsilon,
                              uint32_t flags, void* stream, void* gemm_out) {
    if (ctx == nullptr) return set_error(FU_ERR_INVALID, "null context");
    const fu_qkv_topology& t = ctx->topo;
    const int S = t.sp_size;
    const int64_t L = local_tokens;
    if (L < 1 || L * S > t.capacity_rows)
        return set_error(FU_ERR_INVALID, "local_tokens %lld not in [1, %lld]",
                         static_cast<long long>(L), static_cast<long long>(t.capacity_rows / S));
    if (L > (int64_t(1) << 30)) return set_error(FU_ERR_INVALID, "local_tokens too large");
    if (!x || !w || !positions || !q_gamma || !k_gamma || !rope)
        return set_error(FU_ERR_INVALID, "null input pointer");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
         reinterpret_cast<uintptr_t>(rope) | reinterpret_cast<uintptr_t>(gemm_out)) & 15)
        return set_error(FU_ERR_INVALID, "x, w, rope and gemm_out must be 16-byte aligned");
    if (rope_rows < 1) return set_error(FU_ERR_INVALID, "rope_rows must be positive");
    if (t.status_host != nullptr && *reinterpret_cast<volatile int32_t*>(t.status_host) != 0)
        return set_error(FU_ERR_DEVICE, "an earlier launch reported device status 0x%x",
                         *t.status_host);

    QkvParams& p = ctx->params;
    const int64_t H = t.hidden_size;
    const int heads = t.q_heads + 2 * t.kv_heads;
    const int64_t N = static_cast<int64_t>(heads) * FU_HEAD_DIM;
    int rc;
    {
        fu_qkv_ctx::MapEntry* hit = nullptr;
        for (auto& e : ctx->x_maps)
            if (e.ptr == x && e.rows == L) hit = &e;
        if (hit == nullptr) {
            hit = &ctx->x_maps[ctx->x_next];
            ctx->x_next = (ctx->x_next + 1) % fu_qkv_ctx::kXMaps;
            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(L)};
            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(H * 2)};
            const cuuint32_t box[2] = {BK, BM};
            hit->ptr = nullptr;
            if ((rc = encode(&hit->map, x, 2, dims, strides, box, "hidden_states")) != FU_OK)
                return rc;
            hit->ptr = x;
            hit->rows = L;
        }
        p.tm_x = hit->map;
    }
    {
        fu_qkv_ctx::MapEntry* hit = nullptr;
        for (auto& e : ctx->w_maps)
            if (e.ptr == w) hit = &e;
        if (hit == nullptr) {
            hit = &ctx->w_maps[ctx->w_next];
            ctx->w_next = (ctx->w_next + 1) % fu_qkv_ctx::kWMaps;
            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(H)};
            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N * 2)};
            const cuuint32_t box[2] = {64, BK};
            hit->ptr = nullptr;
            if ((rc = encode(&hit->map, w, 2, dims, strides, box, "qkv_weight")) != FU_OK)
                return rc;
            hit->ptr = w;
        }
        p.tm_w = hit->map;
    }
    if (L != ctx->out_rows) {
        for (int comp = 0; comp < 3; ++comp) {
            const int per_gpu = (comp == 0 ? t.q_heads : t.kv_heads) / S;
            const int64_t cols = static_cast<int64_t>(per_gpu) * FU_HEAD_DIM;
            for (int d = 0; d < S; ++d) {
                void* base = comp == 0 ? t.q_recv[d] : (comp == 1 ? t.k_recv[d] : t.v_recv[d]);
                // Destination d's buffer seen as [S sources][L rows][cols]: a tail tile
                // is clipped at this source's L rows instead of spilling into the next.
                const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols),
                                            static_cast<cuuint64_t>(L),
                                            static_cast<cuuint64_t>(S)};
                const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2),
                                               static_cast<cuuint64_t>(L * cols * 2)};
                const cuuint32_t box[3] = {64, 32, 1};
                if ((rc = encode(&p.tm_out[comp * FU_MAX_SP + d], base, 3, dims, strides, box,
                                 "receive buffer")) != FU_OK)
                    return rc;
            }
        }
        ctx->out_rows = L;
    }

    p.positions = positions;
    p.q_gamma = q_gamma;
    p.k_gamma = k_gamma;
    p.rope = rope;
    p.gemm_out = static_cast<__nv_bfloat16*>(gemm_out);
    for (int d = 0; d < FU_MAX_SP; ++d) {
        p.sync[d] = d < S ? t.sync[d] : nullptr;
        p.out_base[0 * FU_MAX_SP + d] = d < S ? t.q_recv[d] : nullptr;
        p.out_base[1 * FU_MAX_SP + d] = d < S ? t.k_recv[d] : nullptr;
        p.out_base[2 * FU_MAX_SP + d] = d < S ? t.v_recv[d] : nullptr;
    }
    p.status = t.status;
    p.timeout_ns = t.timeout_ns;
    p.L = static_cast<int32_t>(L);
    p.H = static_cast<int32_t>(H);
    p.N = static_cast<int32_t>(N);
    p.rope_rows = rope_rows > INT32_MAX ? INT32_MAX : static_cast<int32_t>(rope_rows);
    p.heads = heads;
    p.q_heads = t.q_heads;
    p.kv_heads = t.kv_heads;
    p.sp_size = S;
    p.sp_rank = t.sp_rank;
    p.q_per_gpu = t.q_heads / S;
    p.kv_per_gpu = t.kv_heads / S;
    p.num_n_blocks = (heads + 1) / 2;
    const int64_t m_blocks = (L + BM - 1) / BM;
    const int64_t tiles = m_blocks * p.num_n_blocks;
    p.num_m_tiles = static_cast<int32_t>(m_blocks);
    if (tiles > INT32_MAX) return set_error(FU_ERR_INVALID, "too many tiles");
    p.num_tiles = static_cast<int32_t>(tiles);
    p.k_blocks = static_cast<int32_t>(H / BK);
    p.q_eps = static_cast<float>(q_epsilon);
    p.k_eps = static_cast<float>(k_epsilon);
    ++ctx->epoch;                                // calls launched (the device keeps the epoch)
    p.wait_peers = (flags & FU_FWD_NO_PEER_WAIT) ? 0u : 1u;
    p.fp32_epilogue = (flags & FU_FWD_FP32_EPILOGUE) ? 1u : 0u;
    p.static_weights = (flags & FU_FWD_STATIC_WEIGHTS) ? 1 : 0;

    p.splits = choose_splits(ctx, tiles, p.k_blocks, L < BM ? L : BM,
                             static_cast<int>((flags >> 8) & 0xFu));
    // A single row block of a few rows: the cluster's partials go to its leader
    // (every rank's rows fit the leader's staging area).
    p.split_push = p.splits > 1 && m_blocks == 1 &&
                   (static_cast<int64_t>(p.splits) * PUSH_ROW_BYTES + ROPE_ROW_BYTES) * L <=
                       PUSH_BYTES ? 1 : 0;
    // CTA pairs (256-row tiles) for the persistent grid once a call spans two
    // row blocks, unless the flags pin the variant.
    const uint32_t variant = (flags >> 12) & 0x3u;
    const bool pair = p.splits == 1 && ctx->max_pairs > 0 &&
                      (variant == 2u || (variant == 0u && m_blocks >= 2));
    int grid;
    p.num_units = p.num_tiles;
    p.full_units = p.num_tiles;
    if (pair) {
        // Whole tiles fill full rounds of the co-resident pairs; a partial last
        // round that at most half fills the pairs is re-tiled into one-head units.
        const int64_t T = (L + 2 * BM - 1) / (2 * BM) * p.num_n_blocks;
        const int64_t P = ctx->max_pairs;
        const int64_t rem = T % P;
        int64_t units = T, full = T;
        if (rem > 0 && 2 * rem <= P && (flags & FU_FWD_NO_RETILE) == 0) {
            full = T - rem;
            units = T + rem;
        }
        p.num_tiles = static_cast<int32_t>(T);
        p.num_m_tiles = static_cast<int32_t>(T / p.num_n_blocks);
        p.num_units = static_cast<int32_t>(units);
        p.full_units = static_cast<int32_t>(full);
        grid = 2 * static_cast<int>(units < P ? units : P);
    } else if (p.splits > 1) {
        grid = static_cast<int>(tiles) * p.splits;
    } else {
        grid = static_cast<int>(tiles < ctx->sm_count ? tiles : ctx->sm_count);
    }
    ctx->last_grid = grid;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != t.device) cudaSetDevice(t.device);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_ALLOC;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    int n_attrs = 0;
    if (pair || p.splits > 1) {
        attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;
        attrs[n_attrs].val.clusterDim.x = pair ? 2 : p.splits;
        attrs[n_attrs].val.clusterDim.y = 1;
        attrs[n_attrs].val.clusterDim.z = 1;
        ++n_attrs;
    }
    if ((flags & FU_FWD_NO_PDL) == 0) {
        // The prologue (barriers, TMEM, descriptor prefetch) may overlap the
        // previous kernel of the stream; the kernel waits for it before it
        // touches global memory.
        attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
        ++n_attrs;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n_attrs;
    cudaError_t e = pair ? cudaLaunchKernelEx(&cfg, fused_qkv_exchange_kernel<true>, p)
                         : cudaLaunchKernelEx(&cfg, fused_qkv_exchange_kernel<false>, p);
    if (prev != t.device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(FU_ERR_CUDA, "launch failed: %s", cudaGetErrorString(e));
    return FU_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point (one GPU).
//
// Some callers cannot allocate device memory where they call this operator:
// an inference server that reserves all free HBM for its KV cache up front and
// hands out memory only through its own pool, an embedding runtime whose
// allocator is not CUDA's, or a plain C caller that owns only the buffers it
// passes in.  For them, fu_qkv_forward_noalloc runs the same fused kernel for a
// world of one GPU (self-exchange) with every byte of its scratch -- the CTA
// completion counter and the exit flag -- in the file-scope array below, so
// the call itself allocates nothing: no cudaMalloc, cudaFree, cudaHostAlloc or
// allocating library routine, on any call.
namespace fu {
// Scratch of the allocation-free entry point: FU_SYNC_WORDS 32-bit words
// (256 bytes), laid out like a per-rank sync block.  Every GPU that loads this
// library holds it until the process exits.  Calls share it and it keeps the
// previous call's contents: each call zeroes the completion counter first, and
// calls that overlap on the same GPU (for example on two streams) race on it.
static __device__ __align__(256) uint32_t g_noalloc_scratch[FU_SYNC_WORDS];

constexpr int kNoallocMaxDevices = 64;

struct NoallocDevice {
    std::once_flag once;
    int rc = FU_OK;
    char message[256] = {0};
    uint32_t* scratch = nullptr;     // device address of g_noalloc_scratch
    int sm_count = 0;
};
static NoallocDevice g_noalloc_devices[kNoallocMaxDevices];

// Once per device, with that device current: resolve the scratch array's
// device address (host code may not use the symbol itself as an address) and
// raise the kernel's shared-memory limit.
static void noalloc_setup(int device, NoallocDevice& st) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
        st.rc = FU_ERR_CUDA;
        snprintf(st.message, sizeof(st.message), "cudaGetSymbolAddress(scratch) on device %d: %s",
                 device, cudaGetErrorString(e));
        return;
    }
    e = cudaFuncSetAttribute(fused_qkv_exchange_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount,
                                                     device);
    if (e != cudaSuccess) {
        st.rc = FU_ERR_CUDA;
        snprintf(st.message, sizeof(st.message), "set-up on device %d: %s", device,
                 cudaGetErrorString(e));
        return;
    }
    st.scratch = static_cast<uint32_t*>(ptr);
}
}  // namespace fu

extern "C" int fu_qkv_forward_noalloc(int device, const void* x, const void* w,
                                      const int64_t* positions, const float* q_gamma,
                                      const float* k_gamma, const float* rope,
                                      int64_t local_tokens, int64_t hidden_size, int32_t q_heads,
                                      int32_t kv_heads, int64_t rope_rows, double q_epsilon,
                                      double k_epsilon, void* q_out, void* k_out, void* v_out,
                                      int32_t* status, void* stream) {
    const int64_t L = local_tokens;
    if (device < 0 || device >= kNoallocMaxDevices)
        return set_error(FU_ERR_INVALID, "device %d outside [0, %d)", device, kNoallocMaxDevices);
    if (L < 1 || L > FU_NOALLOC_MAX_TOKENS)
        return set_error(FU_ERR_INVALID,
                         "local_tokens %lld outside [1, %d], the largest count the kernel's "
                         "32-bit row indices and the fixed scratch serve",
                         static_cast<long long>(L), FU_NOALLOC_MAX_TOKENS);
    if (hidden_size <= 0 || hidden_size % 64)
        return set_error(FU_ERR_INVALID, "hidden_size %lld must be a positive multiple of 64",
                         static_cast<long long>(hidden_size));
    if (hidden_size > (int64_t(1) << 30))
        return set_error(FU_ERR_INVALID, "hidden_size %lld exceeds 2^30, the kernel's 32-bit "
                         "column indices", static_cast<long long>(hidden_size));
    if (q_heads <= 0 || kv_heads <= 0 || q_heads > 4096 || kv_heads > 4096)
        return set_error(FU_ERR_INVALID, "head counts (%d, %d) out of range", q_heads, kv_heads);
    if (!x || !w || !positions || !q_gamma || !k_gamma || !rope || !q_out || !k_out || !v_out)
        return set_error(FU_ERR_INVALID, "null pointer argument");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
         reinterpret_cast<uintptr_t>(rope) | reinterpret_cast<uintptr_t>(q_out) |
         reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 15)
        return set_error(FU_ERR_INVALID, "x, w, rope and the outputs must be 16-byte aligned");
    if (rope_rows < 1) return set_error(FU_ERR_INVALID, "rope_rows must be positive");

    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return set_error(FU_ERR_CUDA, "cudaGetDevice failed");
    if (prev != device && cudaSetDevice(device) != cudaSuccess)
        return set_error(FU_ERR_INVALID, "device %d is not available", device);
    struct Restore {
        int prev, dev;
        ~Restore() { if (prev != dev) cudaSetDevice(prev); }
    } restore{prev, device};

    NoallocDevice& st = g_noalloc_devices[device];
    std::call_once(st.once, [&] {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
        if (major != 10 || minor != 0) {
            st.rc = FU_ERR_UNSUPPORTED;
            snprintf(st.message, sizeof(st.message), "requires an sm_100 GPU; device %d is sm_%d%d",
                     device, major, minor);
            return;
        }
        noalloc_setup(device, st);
    });
    if (st.rc != FU_OK) return set_error(st.rc, "%s", st.message);

    // Parameters live on the host stack; the launch copies them.
    QkvParams p;
    std::memset(&p, 0, sizeof(p));
    const int heads = q_heads + 2 * kv_heads;
    const int64_t N = static_cast<int64_t>(heads) * FU_HEAD_DIM;
    int rc;
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden_size), static_cast<cuuint64_t>(L)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden_size * 2)};
        const cuuint32_t box[2] = {BK, BM};
        if ((rc = encode(&p.tm_x, x, 2, dims, strides, box, "hidden_states")) != FU_OK) return rc;
    }
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(hidden_size)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N * 2)};
        const cuuint32_t box[2] = {64, BK};
        if ((rc = encode(&p.tm_w, w, 2, dims, strides, box, "qkv_weight")) != FU_OK) return rc;
    }
    void* outs[3] = {q_out, k_out, v_out};
    for (int comp = 0; comp < 3; ++comp) {
        const int64_t cols = static_cast<int64_t>(comp == 0 ? q_heads : kv_heads) * FU_HEAD_DIM;
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(L), 1};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2),
                                       static_cast<cuuint64_t>(L * cols * 2)};
        const cuuint32_t box[3] = {64, 32, 1};
        if ((rc = encode(&p.tm_out[comp * FU_MAX_SP], outs[comp], 3, dims, strides, box,
                         "output")) != FU_OK)
            return rc;
    }
    p.positions = positions;
    p.q_gamma = q_gamma;
    p.k_gamma = k_gamma;
    p.rope = rope;
    p.gemm_out = nullptr;
    p.sync[0] = st.scratch;
    p.status = status;
    p.timeout_ns = FU_DEFAULT_TIMEOUT_NS;
    p.L = static_cast<int32_t>(L);
    p.H = static_cast<int32_t>(hidden_size);
    p.N = static_cast<int32_t>(N);
    p.rope_rows = rope_rows > INT32_MAX ? INT32_MAX : static_cast<int32_t>(rope_rows);
    p.heads = heads;
    p.q_heads = q_heads;
    p.kv_heads = kv_heads;
    p.sp_size = 1;
    p.sp_rank = 0;
    p.q_per_gpu = q_heads;
    p.kv_per_gpu = kv_heads;
    p.num_n_blocks = (heads + 1) / 2;
    const int64_t tiles = (L + BM - 1) / BM * p.num_n_blocks;
    p.num_tiles = static_cast<int32_t>(tiles);
    p.num_m_tiles = static_cast<int32_t>((L + BM - 1) / BM);
    p.num_units = p.num_tiles;
    p.full_units = p.num_tiles;
    p.k_blocks = static_cast<int32_t>(hidden_size / BK);
    p.q_eps = static_cast<float>(q_epsilon);
    p.k_eps = static_cast<float>(k_epsilon);
    // The kernel advances the epoch word of the scratch itself; only the
    // completion counter must start at zero.
    p.wait_peers = 1u;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(st.scratch + FU_SYNC_COUNTER, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return set_error(FU_ERR_CUDA, "clearing scratch: %s", cudaGetErrorString(e));
    const int grid = static_cast<int>(tiles < st.sm_count ? tiles : st.sm_count);
    fused_qkv_exchange_kernel<false><<<grid, NUM_THREADS, SMEM_ALLOC, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(FU_ERR_CUDA, "launch failed: %s", cudaGetErrorString(e));
    return FU_OK;
}
