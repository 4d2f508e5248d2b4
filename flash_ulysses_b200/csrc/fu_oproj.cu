// Inverse Ulysses exchange fused with the attention output projection, as one
// launch per call on each SP rank (sm_100a).
//
// After attention, SP member d holds the attention output of its own heads
// for the whole group's sequence, attn_d [S*L, cpm] (cpm = q_heads/S * 128
// columns, rows s*L.. belong to source s) -- the layout in which the forward
// exchange delivered Q.  The inverse exchange returns to every source s its L
// token rows for all of its TP-local heads, G_s [L, q_heads * 128], and the
// output projection computes out_s = G_s . W_o^T with W_o [H, q_heads * 128]
// (torch.nn.Linear layout).  The reference stops at the forward exchange;
// this operator is the step its outputs feed once attention has run.
//
// Per CTA, 192 threads in six warps (single CTAs, or CTA pairs with tcgen05
// cta_group::2 once L spans two 128-row m-blocks):
//   warp 0     TMA producer: X tiles -- this rank's own heads straight from its
//              attention output, the peers' heads from its gather buffer G
//              once the m-block's ready counter is complete -- and W_o tiles
//              (half of each tile's rows per CTA of a pair)
//   warp 1     TMEM owner + tcgen05.mma issuer (M=128 or, on the pair's
//              leader, M=256; N=bn; both operands K-major)
//   warps 2-5  epilogue: TMEM -> BF16 -> swizzled staging -> TMA store of
//              out.  Before it, warps 2-3 run the push side of the exchange:
//              claim units (m-block, peer s, slice of ~32 KiB) from an atomic
//              work counter, copy the slice's rows of this rank's attention
//              output -- local reads -- into G_s with 16-byte posted stores
//              (NVLink writes), fence, and bump G_s's ready counter of that
//              m-block.
// Units are taken in m-block order by whichever warps are running, so no CTA
// depends on another being resident; every wait is bounded.
//
// Epochs: CTA 0 publishes "entered e" into every member's sync block; a
// push warp waits (bounded) until member s has entered e before its first
// store into G_s, so G_s is no longer read by s's previous call.  The ready
// counters are reset by the last CTA of their owner once every tile has been
// loaded; peers cannot count into the next call before the owner enters it.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "flash_ulysses_b200.h"
#include "fu_internal.h"
#include "fu_ptx.cuh"

namespace fu {
namespace oproj {

constexpr int BM = 128;                         // token rows per tile = TMEM lanes
constexpr int BN = 256;                         // widest tile: output columns (TMEM stride)
constexpr int BK = 64;                          // one 128-byte swizzle row of K
constexpr int UMMA_K = 16;
constexpr int MAX_STAGES = 8;                   // single CTA: 4 / 6 / 8 at bn = 256 / 128 / 64
constexpr int NUM_THREADS = 192;
constexpr int NUM_EPI_THREADS = 128;
constexpr int UNIT_BYTES = 32 * 1024;           // target bytes of one push unit
// Epilogue warps per CTA that push first.  At 2 and 4 GPUs (L = 1024..8192)
// two gave the best mean against NCCL all_to_all + cuBLAS: with one, the
// push (fenced per unit) runs below the GEMM's consumption rate; with all
// four, every m-block completes late.
constexpr int PUSH_WARPS = 2;
constexpr int A_STAGE_BYTES = BM * BK * 2;      // 16 KiB, then this CTA's rows of W_o
constexpr int RING_BYTES = 4 * (A_STAGE_BYTES + BN * BK * 2);   // 192 KiB
constexpr int OFF_RING = 0;
constexpr int OFF_STG = OFF_RING + RING_BYTES;
constexpr int BOX_BYTES = 32 * 128;             // 32 rows x 64 BF16
constexpr int STAGING_PER_WARP = 2 * BOX_BYTES;
constexpr int OFF_BAR = OFF_STG + 4 * STAGING_PER_WARP;
constexpr int OFF_MISC = OFF_BAR + 256;
constexpr int SMEM_BYTES = OFF_MISC + 64;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;   // room to align the base to 1 KiB
constexpr uint32_t TMEM_COLS = 512;
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KiB per-CTA shared memory limit");
static_assert(16 * MAX_STAGES + 40 <= 256, "barrier area");

// Sync block layout (uint32 words): entry flags [8, 16), the CTA completion
// counter, the epoch, the gather work counter; ready counters from
// OPROJ_READY on, one per m-block of this rank's gather buffer.
constexpr int SYNC_WORK = FU_SYNC_EPOCH + 1;
static_assert(SYNC_WORK < FU_SYNC_WORDS, "sync layout");

// Status "where" codes of this kernel (second byte of the status word).
enum : int {
    W_EMPTY = 33, W_FULL = 34, W_TEMPTY = 35, W_TFULL = 36, W_DRAIN = 37, W_READY = 38,
    W_ENTRY = 48,                                 // + member index
};

struct OprojParams {
    CUtensorMap tm_g;                  // this rank's gather buffer [L, K]: box {64, 128}
    CUtensorMap tm_self;               // this rank's attention output [S * L, cpm]: box {64, 128}
    const __nv_bfloat16* attn;         // this rank's attention output [S * L, cpm]
    __nv_bfloat16* gather[FU_MAX_SP];  // member d's gather buffer [>= L, K]
    CUtensorMap tm_w;                  // W_o [H, K]: box {64, bn}
    CUtensorMap tm_out;                // out [L, H]: box {64, 32}
    uint32_t* sync[FU_MAX_SP];         // member d's sync block
    int32_t* status;
    unsigned long long timeout_ns;
    int32_t L, H, K, cpm, sp_size, sp_rank;
    int32_t num_m, num_n, num_tiles, k_blocks, units;
    int32_t row_tiles;                        // tile rows (128 rows, or 256 for a pair)
    int32_t col_major;                        // 1: tiles numbered column-major (see Sched)
    int32_t bn;                        // output columns per tile: 256, 128 or 64
    int32_t stages, stage_bytes;       // operand ring: RING_BYTES / stage_bytes stages
    int32_t slice_rows, slices;        // push unit: slice_rows rows; slices = BM / slice_rows
    uint32_t wait_peers;
    uint32_t do_gather, do_gemm;       // both in one call; one each in the two-phase mode
};
static_assert(sizeof(OprojParams) <= 4096, "kernel parameter block too large");

struct Bars {
    uint32_t full, empty, tfull, tempty, mma_done;
    __device__ explicit Bars(uint32_t base)
        : full(base), empty(base + 8 * MAX_STAGES), tfull(base + 16 * MAX_STAGES),
          tempty(base + 16 * MAX_STAGES + 16), mma_done(base + 16 * MAX_STAGES + 32) {}
};

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

__device__ __forceinline__ uint32_t atom_add_relaxed_sys_u32(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.relaxed.sys.global.add.u32 %0, [%1], %2;"
                 : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ uint32_t pack_bf16x2_rn(uint32_t lo_bits, uint32_t hi_bits) {
    __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(lo_bits), __uint_as_float(hi_bits));
    return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------ gather (push)
// Run by PUSH_WARPS epilogue warps per CTA before their epilogue duty.  One unit:
// rows [row0, row0 + slice_rows) (~32 KiB) of peer s's block of this rank's
// attention output ->
// columns [me * cpm, (me + 1) * cpm) of G_s: 16-byte loads from local memory,
// 16-byte posted stores (NVLink writes for a peer), then a system-scope fence
// and one count on G_s's ready counter of the m-block.  Small units complete
// the first m-blocks early, while the rest of the transfer is still running.
__device__ void run_gather(const OprojParams& p, uint32_t epoch, volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    uint32_t* work = p.sync[p.sp_rank] + SYNC_WORK;
    const int per_m = (p.sp_size - 1) * p.slices;
    const int cpr = p.cpm / 8;                    // 16-byte chunks per row
    // i / cpr as a multiply-high: with M = floor((2^32 - 1) / cpr) + 1 the
    // quotient is exact for i < 2^32 / cpr, far above a unit's slice_rows * cpr
    // chunks.  A 32-bit integer division per chunk (a long instruction
    // sequence on the GPU) cut a warp's copy rate by 2.5x.
    const uint32_t magic = 0xFFFFFFFFu / static_cast<uint32_t>(cpr) + 1u;
    const int dst_row = p.K / 8;                  // 16-byte chunks per row of G
    uint32_t entered = 0;                         // members known to have entered this epoch
    // A call queued behind one that failed (this operator's sticky
    // FU_SYNC_FAILED word, in local device memory) pushes nothing and waits
    // for nothing; the abort flag stops this CTA's producer and MMA issuer too.
    if (p.sp_size > 1) {
        int bad = 0;
        if (lane == 0)
            bad = *reinterpret_cast<volatile const uint32_t*>(p.sync[p.sp_rank] +
                                                            FU_SYNC_FAILED) != 0u;
        if (__shfl_sync(0xffffffffu, bad, 0)) {
            *abort_flag = 1;
            return;
        }
    }
    while (true) {
        int u = 0;
        if (lane == 0) u = static_cast<int>(atomicAdd(work, 1u));
        u = __shfl_sync(0xffffffffu, u, 0);
        if (u >= p.units || *abort_flag) break;
        const int mb = u / per_m;
        const int rest = u - mb * per_m;
        const int sv = rest / p.slices;               // peers only: this rank's own
        const int s = sv + (sv >= p.sp_rank ? 1 : 0); // columns are read in place
        const int row0 = mb * BM + (rest - sv * p.slices) * p.slice_rows;
        const int rows = max(0, min(p.slice_rows, p.L - row0));
        // G_s must no longer be read by s's previous call: wait until s entered.
        if (p.wait_peers && !(entered & (1u << s))) {
            if (lane == 0) {
                const uint32_t* flag = p.sync[p.sp_rank] + FU_SYNC_ENTRY + s;
                const uint64_t t0 = globaltimer_ns();
                while (static_cast<int32_t>(ld_acquire_sys_u32(flag) - epoch) < 0) {
                    if (globaltimer_ns() - t0 > p.timeout_ns) {
                        report_status(p.status, FU_DEV_PEER_TIMEOUT, W_ENTRY + s);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            __syncwarp();
            entered |= 1u << s;
            if (*abort_flag) break;
        }
        const uint4* src = reinterpret_cast<const uint4*>(
            p.attn + (static_cast<int64_t>(s) * p.L + row0) * p.cpm);
        uint4* dst = reinterpret_cast<uint4*>(p.gather[s] + static_cast<int64_t>(row0) * p.K +
                                              static_cast<int64_t>(p.sp_rank) * p.cpm);
        const int total = rows * cpr;
        constexpr int U = 16;
        for (int i0 = 0; i0 < total; i0 += 32 * U) {
            uint4 v[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int i = i0 + j * 32 + lane;
                if (i < total) v[j] = __ldcg(src + i);
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int i = i0 + j * 32 + lane;
                if (i < total) {
                    const int r = static_cast<int>(__umulhi(static_cast<uint32_t>(i), magic));
                    dst[r * dst_row + (i - r * cpr)] = v[j];
                }
            }
        }
        // Every lane's stores are performed system-wide before the count (and
        // ordered before the owner's TMA reads of them).
        fence_proxy_async_global();
        __threadfence_system();
        __syncwarp();
        if (lane == 0) atom_add_relaxed_sys_u32(p.sync[s] + FU_OPROJ_READY + mb, 1u);
    }
}

// ------------------------------------------------------------ schedule
// Tiles of 128 (single CTA) or 256 rows (CTA pair, tcgen05 cta_group::2: each
// CTA loads its own 128 rows of X and half of the W_o tile's rows, the leader
// issues M=256 MMAs, each CTA drains its own TMEM lanes) by bn columns,
// persistent over the grid's CTAs or pairs.
template <bool kPair>
struct Sched {
    int first, stride, rank;
    __device__ Sched() {
        rank = kPair ? static_cast<int>(cluster_ctarank()) : 0;
        first = kPair ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
        stride = kPair ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
    }
    // This CTA's 128-row m-block of tile t, and the tile's column block.
    // With peers pushing rows in (S > 1) tiles go row by row, so the first
    // rounds need only the m-blocks that complete first; with nothing to wait
    // for (S = 1) they go column by column, so the CTAs running at the same
    // time share W_o's column blocks and W_o streams from HBM once.
    __device__ int m_block(const OprojParams& p, int t) const {
        const int mt = p.col_major ? t % p.row_tiles : t / p.num_n;
        return kPair ? 2 * mt + rank : mt;
    }
    __device__ int n_block(const OprojParams& p, int t) const {
        return p.col_major ? t / p.row_tiles : t % p.num_n;
    }
};

// ------------------------------------------------------------ producer
template <bool kPair>
__device__ void run_producer(const OprojParams& p, uint8_t* smem, const Bars& b,
                             volatile int* abort_flag) {
    const Sched<kPair> sc;
    const uint32_t ring = smem_u32(smem + OFF_RING);
    const uint32_t* ready = p.sync[p.sp_rank] + FU_OPROJ_READY;
    const uint32_t target = static_cast<uint32_t>((p.sp_size - 1) * p.slices);
    // K-blocks of this rank's own heads come straight from its attention output.
    const int self_kb0 = p.sp_rank * p.cpm / BK;
    const int self_kb1 = self_kb0 + p.cpm / BK;
    const int b_rows = kPair ? p.bn / 2 : p.bn;   // W_o rows this CTA loads per tile
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, last_parity = 0;
    int ready_m = -1;                             // highest m-block known complete
    bool ok = true;
    for (int t = sc.first; ok && t < p.num_tiles; t += sc.stride) {
        const int mb = sc.m_block(p, t);
        const int nb = sc.n_block(p, t);
        if (mb > ready_m && target > 0 && mb < p.num_m) {
            // Every source's slices of this m-block have landed in G.
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys_u32(ready + mb) < target) {
                if (*abort_flag) { ok = false; break; }
                if (globaltimer_ns() - t0 > p.timeout_ns) {
                    report_status(p.status, FU_DEV_PIPELINE_TIMEOUT, W_READY);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            fence_proxy_async_global();           // generic-proxy writes -> TMA reads
            ready_m = mb;
        }
        for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!fu_wait_parity(b.empty + 8 * stage, phase ^ 1u, abort_flag, p.timeout_ns,
                                p.status, W_EMPTY)) {
                ok = false;
                break;
            }
            const uint32_t adst = ring + stage * p.stage_bytes;
            const int ka = kb >= self_kb0 && kb < self_kb1;
            if (kPair) {
                // Both CTAs' bytes are counted on the leader's barrier.
                const uint32_t full = map_cluster_smem(b.full + 8 * stage, 0);
                if (sc.rank == 0) mbar_arrive_expect_tx(b.full + 8 * stage, 2 * p.stage_bytes);
                if (ka)
                    tma_load_2d_pair(adst, &p.tm_self, full, (kb - self_kb0) * BK,
                                     p.sp_rank * p.L + mb * BM);
                else
                    tma_load_2d_pair(adst, &p.tm_g, full, kb * BK, mb * BM);
                tma_load_2d_pair(adst + A_STAGE_BYTES, &p.tm_w, full, kb * BK,
                                 nb * p.bn + sc.rank * b_rows);
            } else {
                const uint32_t full = b.full + 8 * stage;
                mbar_arrive_expect_tx(full, p.stage_bytes);
                if (ka)
                    tma_load_2d(adst, &p.tm_self, full, (kb - self_kb0) * BK,
                                p.sp_rank * p.L + mb * BM);
                else
                    tma_load_2d(adst, &p.tm_g, full, kb * BK, mb * BM);
                tma_load_2d(adst + A_STAGE_BYTES, &p.tm_w, full, kb * BK, nb * p.bn);
            }
            issued_mask |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == p.stages) {
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
            // Loads already issued must land before shared memory is released.
            for (int s = 0; s < p.stages; ++s)
                if (issued_mask & (1u << s))
                    drain_wait(b.full + 8 * s, (last_parity >> s) & 1u, p.timeout_ns, p.status);
        }
    }
}

// ------------------------------------------------------------ MMA
// Single CTA, or the pair's leader only.
template <bool kPair>
__device__ void run_mma(const OprojParams& p, uint8_t* smem, uint32_t tmem_base, const Bars& b,
                        volatile int* abort_flag) {
    const Sched<kPair> sc;
    const uint32_t idesc = make_idesc_bf16_f32(kPair ? 2 * BM : BM, p.bn, /*a_mn_major=*/false,
                                               /*b_mn_major=*/false);
    const uint32_t ring = smem_u32(smem + OFF_RING);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int t = sc.first; ok && t < p.num_tiles; t += sc.stride, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!fu_wait_parity(b.tempty + 8 * acc, acc_phase ^ 1u, abort_flag, p.timeout_ns,
                            p.status, W_TEMPTY)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!fu_wait_parity(b.full + 8 * stage, phase, abort_flag, p.timeout_ns, p.status,
                                W_FULL)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a_base = ring + stage * p.stage_bytes;
            const uint32_t b_base = a_base + A_STAGE_BYTES;
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
                // Both operands K-major with 128-byte swizzle: K advances 32 bytes
                // inside the swizzle row; 8-row groups are 1024 bytes apart.  In a
                // pair each CTA holds its own A rows and half of B's rows at the
                // same offsets.
                const uint64_t adesc = make_smem_desc_sw128(a_base + k * UMMA_K * 2, 16, 1024);
                const uint64_t bdesc = make_smem_desc_sw128(b_base + k * UMMA_K * 2, 16, 1024);
                const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
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
            if (++stage == p.stages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (ok) {
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

// ------------------------------------------------------------ epilogue
template <bool kPair>
__device__ void run_epilogue(const OprojParams& p, uint8_t* smem, uint32_t tmem_base,
                             const Bars& b, volatile int* abort_flag) {
    const Sched<kPair> sc;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int quarter = warp & 3;                 // TMEM lanes this warp may access
    uint8_t* box0 = smem + OFF_STG + (warp - 2) * STAGING_PER_WARP;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t swz_row = lane * 128;
    const int swz = lane & 7;
    int local = 0;
    for (int t = sc.first; t < p.num_tiles; t += sc.stride, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        const int mb = sc.m_block(p, t);
        const int nb = sc.n_block(p, t);
        if (!fu_wait_parity(b.tfull + 8 * acc, acc_phase, abort_flag, p.timeout_ns, p.status,
                            W_TFULL))
            break;
        tc_fence_after();
        const uint32_t acc_addr = tmem_base + lane_addr + acc * BN;
        // bn / 64 boxes of 64 columns, two at a time through the warp's staging.
        const int boxes = p.bn / 64;
#pragma unroll 1
        for (int half = 0; half < (boxes + 1) / 2; ++half) {
            if (lane == 0) bulk_wait_read_all();  // the staging was read by the last store
            __syncwarp();
#pragma unroll
            for (int bx = 0; bx < 2; ++bx) {
                if (half * 2 + bx >= boxes) break;
                uint8_t* box = box0 + bx * BOX_BYTES;
                const int c0 = (half * 2 + bx) * 64;
#pragma unroll
                for (int c = 0; c < 64; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32cols(acc_addr + c0 + c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 4; ++j) {      // 16-byte chunk (c / 8 + j) of the row
                        const uint32_t w0 = pack_bf16x2_rn(r[8 * j], r[8 * j + 1]);
                        const uint32_t w1 = pack_bf16x2_rn(r[8 * j + 2], r[8 * j + 3]);
                        const uint32_t w2 = pack_bf16x2_rn(r[8 * j + 4], r[8 * j + 5]);
                        const uint32_t w3 = pack_bf16x2_rn(r[8 * j + 6], r[8 * j + 7]);
                        const int chunk = c / 8 + j;
                        *reinterpret_cast<uint4*>(box + swz_row + ((chunk ^ swz) << 4)) =
                            make_uint4(w0, w1, w2, w3);
                    }
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                // Rows past L are clipped by the tensor map.
                const int row = mb * BM + quarter * 32;
                for (int bx = 0; bx < 2 && half * 2 + bx < boxes; ++bx)
                    tma_store_2d(&p.tm_out, smem_u32(box0 + bx * BOX_BYTES),
                                 nb * p.bn + (half * 2 + bx) * 64, row);
                bulk_commit_group();
            }
        }
        // The accumulator has been read: hand TMEM back (to the pair leader's
        // MMA issuer, which counts both CTAs' threads).
        tc_fence_before();
        if (kPair && sc.rank != 0)
            mbar_arrive_remote(map_cluster_smem(b.tempty + 8 * acc, 0));
        else
            mbar_arrive(b.tempty + 8 * acc);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
}

// ------------------------------------------------------------ kernel
template <bool kPair>
__global__ void __launch_bounds__(NUM_THREADS, 1)
oproj_exchange_kernel(const __grid_constant__ OprojParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Bars b(smem_u32(smem + OFF_BAR));
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    uint32_t* epoch_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC + 8);
    uint32_t* my_sync = p.sync[p.sp_rank];
    const bool leader = !kPair || cluster_ctarank() == 0;

    // Prologue: shared memory, TMEM and parameters only (it may overlap the
    // previous kernel of the stream under a programmatic dependent launch).
    if (threadIdx.x == 0) {
        for (int s = 0; s < MAX_STAGES; ++s) {
            mbar_init(b.full + 8 * s, 1);
            mbar_init(b.empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(b.tfull + 8 * a, 1);
            // A pair's leader counts the epilogue threads of both CTAs.
            mbar_init(b.tempty + 8 * a, kPair ? 2 * NUM_EPI_THREADS : NUM_EPI_THREADS);
        }
        mbar_init(b.mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&p.tm_g);
        tma_prefetch_desc(&p.tm_self);
        tma_prefetch_desc(&p.tm_w);
        tma_prefetch_desc(&p.tm_out);
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
        const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_sync + FU_SYNC_EPOCH) + 1;
        *epoch_slot = epoch;
        // "Entered e" carries no data (this rank's earlier reads of G are
        // complete): posted stores.
        if (blockIdx.x == 0 && p.sp_size > 1 && p.do_gather)
            for (int d = 0; d < p.sp_size; ++d)
                st_relaxed_sys_u32(p.sync[d] + FU_SYNC_ENTRY + p.sp_rank, epoch);
    }
    tc_fence_before();
    __syncthreads();
    // A pair's barriers and TMEM must exist in both CTAs before either uses them.
    if (kPair) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const uint32_t epoch = *epoch_slot;

    if (warp == 0) {
        if (lane == 0 && p.do_gemm) run_producer<kPair>(p, smem, b, abort_flag);
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && p.do_gemm && leader) run_mma<kPair>(p, smem, tmem_base, b, abort_flag);
        __syncwarp();
    } else {
        // PUSH_WARPS warps per CTA push rows to their owners until the units
        // run out, then join the epilogue.  Units are small and claimed in
        // m-block order, so the first m-blocks -- the first wave of tiles --
        // complete early and the tensor cores start there.
        if (p.do_gather && warp < 2 + PUSH_WARPS) run_gather(p, epoch, abort_flag);
        if (p.do_gemm) run_epilogue<kPair>(p, smem, tmem_base, b, abort_flag);
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

    // The last CTA to finish advances the epoch and resets the work counter
    // and (once this rank's tiles are done) its ready counters.
    if (threadIdx.x == 64) {
        const bool aborted = *abort_flag != 0;
        fence_acq_rel_gpu();
        const uint32_t old =
            atom_add_acq_rel_gpu_u32(my_sync + FU_SYNC_COUNTER, aborted ? 0x10001u : 1u);
        if ((old & 0xFFFFu) == gridDim.x - 1) {
            volatile uint32_t* vs = my_sync;
            vs[FU_SYNC_COUNTER] = 0u;
            vs[FU_SYNC_EPOCH] = epoch;
            if ((old >> 16) != 0 || aborted)
                if (p.sp_size > 1) vs[FU_SYNC_FAILED] = 1u;   // later calls skip
            if (p.do_gather) vs[SYNC_WORK] = 0u;
            if (p.do_gemm)
                for (int m = 0; m < p.num_m; ++m) vs[FU_OPROJ_READY + m] = 0u;
        }
    }
}

}  // namespace oproj

// ------------------------------------------------------------ host side
// 2-D BF16 row-major [rows, cols] with a 128-byte-swizzled box {64, box_rows}.
static int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                     uint32_t box_rows, const char* what) {
    auto fn = encode_tiled_fn();
    if (fn == nullptr) return set_error(FU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                    strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(FU_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what,
                         static_cast<int>(r));
    return FU_OK;
}

}  // namespace fu

struct fu_oproj_ctx {
    fu_oproj_topology topo;
    int sm_count = 0;
    int max_pairs = 0;            // co-resident CTA pairs of the pair variant
    uint32_t calls = 0;
    int last_grid = 0;
    fu::oproj::OprojParams params;
};

using namespace fu;

extern "C" int64_t fu_oproj_sync_words(int64_t max_local_tokens) {
    if (max_local_tokens < 1) return 0;
    return FU_OPROJ_READY + (max_local_tokens + oproj::BM - 1) / oproj::BM;
}

extern "C" int fu_oproj_create(const fu_oproj_topology* topo, fu_oproj_ctx** out) {
    if (topo == nullptr || out == nullptr) return set_error(FU_ERR_INVALID, "null argument");
    const int S = topo->sp_size;
    if (S < 1 || S > FU_MAX_SP) return set_error(FU_ERR_INVALID, "sp_size %d not in [1, 8]", S);
    if (topo->sp_rank < 0 || topo->sp_rank >= S)
        return set_error(FU_ERR_INVALID, "sp_rank %d not in [0, %d)", topo->sp_rank, S);
    if (topo->q_heads <= 0 || topo->q_heads % S)
        return set_error(FU_ERR_INVALID, "q_heads %d must be a positive multiple of %d",
                         topo->q_heads, S);
    if (topo->hidden_size <= 0 || topo->hidden_size % oproj::BN)
        return set_error(FU_ERR_INVALID, "hidden_size %lld must be a positive multiple of %d",
                         static_cast<long long>(topo->hidden_size), oproj::BN);
    if (topo->max_local_tokens < 1)
        return set_error(FU_ERR_INVALID, "max_local_tokens must be positive");
    for (int d = 0; d < S; ++d) {
        if (!topo->gather[d] || !topo->sync[d])
            return set_error(FU_ERR_INVALID, "missing buffer for SP member %d", d);
        if (reinterpret_cast<uintptr_t>(topo->gather[d]) & 15)
            return set_error(FU_ERR_INVALID, "gather buffers must be 16-byte aligned");
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
    cudaError_t e = cudaFuncSetAttribute(oproj::oproj_exchange_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         oproj::SMEM_ALLOC);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(oproj::oproj_exchange_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, oproj::SMEM_ALLOC);
    int pairs = 0;
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 16, 1, 1);
        cfg.blockDim = dim3(oproj::NUM_THREADS, 1, 1);
        cfg.dynamicSmemBytes = oproj::SMEM_ALLOC;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&pairs, oproj::oproj_exchange_kernel<true>, &cfg) !=
            cudaSuccess) {
            cudaGetLastError();
            pairs = 0;
        }
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess)
        return set_error(FU_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    auto* ctx = new fu_oproj_ctx();
    ctx->max_pairs = pairs;
    ctx->topo = *topo;
    if (ctx->topo.timeout_ns == 0) ctx->topo.timeout_ns = FU_DEFAULT_TIMEOUT_NS;
    ctx->sm_count = sms;
    std::memset(&ctx->params, 0, sizeof(ctx->params));
    *out = ctx;
    return FU_OK;
}

extern "C" int fu_oproj_destroy(fu_oproj_ctx* ctx) {
    delete ctx;
    return FU_OK;
}

extern "C" uint32_t fu_oproj_calls(const fu_oproj_ctx* ctx) { return ctx ? ctx->calls : 0u; }
extern "C" int fu_oproj_last_grid(const fu_oproj_ctx* ctx) { return ctx ? ctx->last_grid : 0; }

extern "C" int fu_oproj_forward(fu_oproj_ctx* ctx, const void* attn, const void* w_o,
                                int64_t local_tokens, void* out, uint32_t flags, void* stream) {
    if (ctx == nullptr) return set_error(FU_ERR_INVALID, "null context");
    const fu_oproj_topology& t = ctx->topo;
    const int S = t.sp_size;
    const int64_t L = local_tokens;
    if (L < 1 || L > t.max_local_tokens)
        return set_error(FU_ERR_INVALID, "local_tokens %lld not in [1, %lld]",
                         static_cast<long long>(L), static_cast<long long>(t.max_local_tokens));
    const uint32_t phases = flags & (FU_OPROJ_GATHER_ONLY | FU_OPROJ_GEMM_ONLY);
    if (phases == (FU_OPROJ_GATHER_ONLY | FU_OPROJ_GEMM_ONLY))
        return set_error(FU_ERR_INVALID, "FU_OPROJ_GATHER_ONLY and FU_OPROJ_GEMM_ONLY exclude "
                                         "each other");
    const bool do_gather = (phases & FU_OPROJ_GEMM_ONLY) == 0;
    const bool do_gemm = (phases & FU_OPROJ_GATHER_ONLY) == 0;
    if (attn == nullptr || (do_gemm && (w_o == nullptr || out == nullptr)))
        return set_error(FU_ERR_INVALID, "null tensor argument");
    if ((reinterpret_cast<uintptr_t>(attn) | reinterpret_cast<uintptr_t>(w_o) |
         reinterpret_cast<uintptr_t>(out)) & 15)
        return set_error(FU_ERR_INVALID, "tensors must be 16-byte aligned");
    if (t.status_host != nullptr && *reinterpret_cast<volatile int32_t*>(t.status_host) != 0)
        return set_error(FU_ERR_DEVICE, "an earlier launch reported device status 0x%x",
                         static_cast<unsigned>(*t.status_host));
    const int64_t H = t.hidden_size;
    const int64_t K = static_cast<int64_t>(t.q_heads) * 128;
    const int cpm = t.q_heads / S * 128;

    // CTA pairs (256-row tiles) once there are two m-blocks, unless a variant
    // is forced (FU_FWD_SINGLE / FU_FWD_PAIR).  Tile width: the widest whose
    // tiles still cover half of the SMs or pairs (small L streams W_o through
    // more CTAs).
    const int64_t num_m = (L + oproj::BM - 1) / oproj::BM;
    const uint32_t variant = (flags >> 12) & 0x3u;
    const bool pair = do_gemm && ctx->max_pairs > 0 &&
                      (variant == 2u || (variant == 0u && num_m >= 2));
    const int64_t row_tiles = pair ? (L + 2 * oproj::BM - 1) / (2 * oproj::BM) : num_m;
    const int64_t slots = pair ? ctx->max_pairs : ctx->sm_count;
    int bn = 64;
    for (int c : {256, 128})
        if (row_tiles * (H / c) * 2 >= slots) {
            bn = c;
            break;
        }
    oproj::OprojParams& p = ctx->params;
    int rc = FU_OK;
    if (do_gemm) {
        rc = encode_2d(&p.tm_g, t.gather[t.sp_rank], L, K, oproj::BM, "gather");
        if (rc == FU_OK) rc = encode_2d(&p.tm_self, attn, S * L, cpm, oproj::BM, "attn");
        if (rc == FU_OK)
            rc = encode_2d(&p.tm_w, w_o, H, K, static_cast<uint32_t>(pair ? bn / 2 : bn), "w_o");
        if (rc == FU_OK) rc = encode_2d(&p.tm_out, out, L, H, 32, "out");
        if (rc != FU_OK) return rc;
    }
    p.attn = static_cast<const __nv_bfloat16*>(attn);
    for (int d = 0; d < FU_MAX_SP; ++d) {
        p.gather[d] = d < S ? static_cast<__nv_bfloat16*>(t.gather[d]) : nullptr;
        p.sync[d] = d < S ? t.sync[d] : nullptr;
    }
    p.status = t.status;
    p.timeout_ns = t.timeout_ns;
    p.L = static_cast<int32_t>(L);
    p.H = static_cast<int32_t>(H);
    p.K = static_cast<int32_t>(K);
    p.cpm = cpm;
    p.sp_size = S;
    p.sp_rank = t.sp_rank;
    p.num_m = static_cast<int32_t>(num_m);
    p.bn = bn;
    // Per CTA: 128 rows of X and bn (single) or bn / 2 (pair) rows of W_o.
    p.stage_bytes = oproj::A_STAGE_BYTES + (pair ? bn / 2 : bn) * oproj::BK * 2;
    p.stages = oproj::RING_BYTES / p.stage_bytes;
    if (p.stages > oproj::MAX_STAGES) p.stages = oproj::MAX_STAGES;
    p.num_n = static_cast<int32_t>(H / bn);
    p.row_tiles = static_cast<int32_t>(row_tiles);
    p.col_major = S == 1 ? 1 : 0;
    p.num_tiles = do_gemm ? static_cast<int32_t>(row_tiles) * p.num_n : 0;
    p.k_blocks = static_cast<int32_t>(K / oproj::BK);
    // Push units of ~32 KiB: 8 to 128 rows (a power of two) of cpm columns.
    int slice_rows = 8;
    while (slice_rows < oproj::BM && 2 * slice_rows * cpm * 2 <= oproj::UNIT_BYTES) slice_rows *= 2;
    p.slice_rows = slice_rows;
    p.slices = oproj::BM / slice_rows;
    p.units = do_gather ? p.num_m * (S - 1) * p.slices : 0;
    p.wait_peers = (flags & FU_FWD_NO_PEER_WAIT) == 0 ? 1u : 0u;
    p.do_gather = do_gather ? 1u : 0u;
    p.do_gemm = do_gemm ? 1u : 0u;
    int grid;
    if (pair) {
        // One pair per tile up to the co-resident pairs (push units ride along).
        grid = 2 * static_cast<int>(p.num_tiles < ctx->max_pairs ? p.num_tiles : ctx->max_pairs);
    } else {
        const int64_t work = p.num_tiles > p.units ? p.num_tiles : p.units;
        // At least one CTA, which advances the epoch (a push-only call of a
        // world of one has nothing else to do).
        grid = static_cast<int>(work < 1 ? 1 : work < ctx->sm_count ? work : ctx->sm_count);
    }
    ctx->last_grid = grid;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != t.device) cudaSetDevice(t.device);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(oproj::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = oproj::SMEM_ALLOC;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    int n_attrs = 0;
    if (pair) {
        attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;
        attrs[n_attrs].val.clusterDim.x = 2;
        attrs[n_attrs].val.clusterDim.y = 1;
        attrs[n_attrs].val.clusterDim.z = 1;
        ++n_attrs;
    }
    if ((flags & FU_FWD_NO_PDL) == 0) {      // as for fu_qkv_forward
        attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
        ++n_attrs;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n_attrs;
    cudaError_t e = pair ? cudaLaunchKernelEx(&cfg, oproj::oproj_exchange_kernel<true>, p)
                         : cudaLaunchKernelEx(&cfg, oproj::oproj_exchange_kernel<false>, p);
    if (prev != t.device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(FU_ERR_CUDA, "launch failed: %s", cudaGetErrorString(e));
    ++ctx->calls;
    return FU_OK;
}
