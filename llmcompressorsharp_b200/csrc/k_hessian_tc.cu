// Hessian accumulation H += X^T X on the 5th-generation tensor cores (sm_100a).
//
// Reference: HessianAccumulator.Update (src/LLMCompressorSharp.TorchExtensions/Hessian/
// HessianAccumulator.cs:47-67) — x.to(fp32).reshape(-1, d); H.add_(flat^T flat).  For bf16 /
// fp16 activations every product is exact in fp32, so an fp32-accumulating tensor-core
// GEMM gives the reference's result up to summation order.
//
// Shape of the work: C[d, d] += A[d, T] B[T, d] with A = X^T and B = X, i.e. both operands
// are the same row-major X [T, d] read "MN-major" (features contiguous, tokens = K).  Only
// tiles that touch the upper triangle are computed (the symmetric lower half is implied).
//
// Per CTA (one per SM, 128 threads):
//   * tile 128 (rows of H) x 256 (columns of H), K-block 64 tokens, 4-stage ring in shared
//     memory filled by TMA (2 + 4 boxes of 64 features x 64 tokens, 128-byte swizzle, no
//     multicast, cluster of one);
//   * one elected thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16)
//     into a 128 x 256 fp32 accumulator in TMEM and releases each stage with
//     tcgen05.commit;
//   * accuracy: the tensor core's fp32 accumulation truncates, so TMEM only ever holds the
//     sum of KF = 16 k-blocks (1,024 tokens).  Two TMEM accumulators alternate: while the MMA
//     issuer fills one, eight epilogue warps fold the other into fp32 registers with
//     round-to-nearest adds (each warp owns 32 rows x 128 columns);
//   * end of a unit: each epilogue warp writes its 32 x 128 block out in four 32 x 32 boxes
//     through its own 4 KB shared buffer (128-byte swizzle) and a tiled TMA reduce-add into
//     H, so H accumulates across calls and token splits without a read pass.  The buffers
//     are separate from the stage ring: the producer and the MMA issuer run on into the next
//     unit while the previous one drains.
// Work units are (tile, token split); units of one split run in the same wave so that the
// X rows they stream are shared through L2.
// Every wait is bounded: on expiry the kernel raises an error word, drains its own
// in-flight copies (again bounded), frees TMEM and returns.
#include "ops.h"
#include "tc_common.cuh"

#include <cuda.h>

#include <mutex>

namespace llmc {
namespace {

using namespace tc;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int EPI_WARPS = 8, NT = 32 * (2 + EPI_WARPS);  // producer, MMA issuer, 8 epilogue warps
// k-blocks (1,024 tokens) accumulated in TMEM before the epilogue folds them into fp32 registers.
// Each tensor-core MMA adds into the fp32 accumulator with truncation, so the fold cadence bounds
// the bias: 1.8e-6 relative Frobenius against fp64 at this setting (0.9e-6 at 8 k-blocks, which
// was 5-7 % slower per clock because the fold then sits on the MMA issuer's critical path).
constexpr int KF = 16;
constexpr int TMEM_COLS = 2 * BN;  // two 128 x 256 fp32 accumulators
constexpr int A_BYTES = BM * BK * 2;             // 16 KB
constexpr int B_BYTES = BN * BK * 2;             // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 48 KB
constexpr int BOX_BYTES = 64 * BK * 2;           // 8 KB: 64 features x 64 tokens
constexpr int SMEM_MAIN = STAGES * STAGE_BYTES;  // 192 KB
constexpr int OUT_BOX = 32;                      // epilogue write-out box: 32 rows x 32 fp32
constexpr int OUT_BYTES = OUT_BOX * OUT_BOX * 4; // 4 KB per epilogue warp
constexpr int SMEM_BYTES = SMEM_MAIN + EPI_WARPS * OUT_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int MAX_TJ = 160;                      // d <= 40960

static_assert(SMEM_BYTES <= 232448, "shared memory above the per-block limit");

struct SyrkArgs {
    float* H;
    int64_t ldh;
    int d;
    int nti, ntj;
    int ntiles;
    int kb_total;     // k-blocks over all rows
    int splits;       // token splits
    int kb_per_split;
    int tile_off[MAX_TJ + 1];  // first tile index of column-panel tj
    int* err;         // device error word (bit 0: a wait timed out)
    uint32_t wait_limit;
    uint32_t idesc;
};

__device__ __forceinline__ void unit_tile(const SyrkArgs& a, int tile, int* ti, int* tj) {
    int lo = 0, hi = a.ntj - 1;  // find tj with tile_off[tj] <= tile < tile_off[tj+1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.tile_off[mid] <= tile) lo = mid;
        else hi = mid - 1;
    }
    *tj = lo;
    *ti = tile - a.tile_off[lo];
}

__global__ void __launch_bounds__(NT, 1) syrk_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                       const __grid_constant__ CUtensorMap hmap, const SyrkArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* outbufs = smem + SMEM_MAIN;  // EPI_WARPS x 4 KB, 1024-byte aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(outbufs + EPI_WARPS * OUT_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2] accumulator b ready for promotion
    uint64_t* tempty = tfull + 2;       // [2] accumulator b folded, MMA may reuse it
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EPI_WARPS);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int total_units = a.ntiles * a.splits;
    uint32_t prod_it = 0, mma_it = 0, cc = 0;  // cc: chunks processed (MMA issuer / epilogue)
    int pend_par[STAGES];  // producer: parity of the latest load issued into each stage (-1: none)
#pragma unroll
    for (int s = 0; s < STAGES; s++) pend_par[s] = -1;
    int commit_par[2] = {-1, -1};  // MMA issuer: parity of its latest commit to tfull[b]

    for (int u = blockIdx.x; u < total_units && !*abort_flag; u += gridDim.x) {
        const int split = u / a.ntiles, tile = u % a.ntiles;
        int ti, tj;
        unit_tile(a, tile, &ti, &tj);
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.kb_total, kb0 + a.kb_per_split);
        const int nchunks = (kb1 - kb0 + KF - 1) / KF;
        const int i0 = ti * BM, j0 = tj * BN;

        if (warp == 0) {
            if (lane == 0) {
                // ---- TMA producer
                for (int kb = kb0; kb < kb1; kb++, prod_it++) {
                    const int s = prod_it % STAGES;
                    const uint32_t ph = (prod_it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    unsigned char* st = smem + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    const int y = kb * BK;
#pragma unroll
                    for (int b = 0; b < BM / 64; b++) tma_load_2d(st + b * BOX_BYTES, &xmap, i0 + 64 * b, y, &full[s]);
#pragma unroll
                    for (int b = 0; b < BN / 64; b++)
                        tma_load_2d(st + A_BYTES + b * BOX_BYTES, &xmap, j0 + 64 * b, y, &full[s]);
                    pend_par[s] = (int)((prod_it / STAGES) & 1u);
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0) {
                // ---- MMA issuer: chunk c accumulates into TMEM buffer (cc & 1)
                uint32_t c_it = cc;
                for (int c = 0; c < nchunks && !*abort_flag; c++, c_it++) {
                    const int b = (int)(c_it & 1u);
                    if (!mbar_wait(&tempty[b], ((c_it >> 1) & 1u) ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    tc_fence_after();
                    const uint32_t dst = tmem + (uint32_t)(b * BN);
                    const int k0 = kb0 + c * KF, k1 = min(kb1, k0 + KF);
                    bool ok = true;
                    for (int kb = k0; kb < k1; kb++, mma_it++) {
                        const int s = mma_it % STAGES;
                        const uint32_t ph = (mma_it / STAGES) & 1u;
                        if (!mbar_wait(&full[s], ph, abort_flag, a.err, a.wait_limit)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t abase = smem_u32(smem + s * STAGE_BYTES);
                        const uint32_t bbase = abase + A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            // 16 tokens = 2 swizzle atoms of 8 rows x 128 B
                            const uint64_t da = smem_desc_mn_sw128(abase + kk * 2048, BOX_BYTES);
                            const uint64_t db = smem_desc_mn_sw128(bbase + kk * 2048, BOX_BYTES);
                            umma_f16(dst, da, db, a.idesc, (kb > k0 || kk > 0) ? 1u : 0u);
                        }
                        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
                    }
                    umma_commit(&tfull[b]);  // chunk complete (fires even if the loop broke early)
                    commit_par[b] = (int)((c_it >> 1) & 1u);
                    if (!ok) break;
                }
            }
            __syncwarp();
        } else {
            // ---- epilogue warps: TMEM lane quadrant q (a warp may only touch lanes
            // [32*(warp%4), +32)), column half h.
            const int e = warp - 2, q = warp % 4, h = e / 4;
            float acc[BN / 2];
#pragma unroll
            for (int i = 0; i < BN / 2; i++) acc[i] = 0.f;
            uint32_t c_it = cc;
            for (int c = 0; c < nchunks; c++, c_it++) {
                const int b = (int)(c_it & 1u);
                const bool have = mbar_wait(&tfull[b], (c_it >> 1) & 1u, abort_flag, a.err, a.wait_limit);
                if (!__all_sync(0xffffffffu, have ? 1 : 0)) break;
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < 4; part++) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + h * 128 + part * 32), v);
#pragma unroll
                    for (int i = 0; i < 32; i++) acc[part * 32 + i] = __fadd_rn(acc[part * 32 + i], __uint_as_float(v[i]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
            }
            // Write-out: rounds of one 32 x 32 box (rows of quadrant q, columns
            // j0 + 128 h + 32 round ..) through this warp's buffer.  The buffer is reused only
            // after the previous reduce has read it; TMA clips rows / columns beyond d.
            if (!*abort_flag) {
                unsigned char* ob = outbufs + e * OUT_BYTES;
                const uint32_t ob_s = smem_u32(ob);
#pragma unroll
                for (int round = 0; round < 4; round++) {
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const int i = round * 32 + c * 4;
                        *reinterpret_cast<float4*>(ob + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                            make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        tma_reduce_add_2d(&hmap, ob_s, j0 + h * 128 + round * 32, i0 + q * 32);
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                }
            }
        }
        cc += (uint32_t)nchunks;
    }

    // Drain: every bulk reduce finishes; after an abort, also wait (bounded) for the TMA
    // loads this CTA issued and for its MMAs, so that nothing touches shared memory or
    // TMEM after they are released.
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (*abort_flag) {
        if (warp == 0 && lane == 0)
            for (int s = 0; s < STAGES; s++)
                if (pend_par[s] >= 0) mbar_wait_drain(&full[s], (uint32_t)pend_par[s]);
        if (warp == 1 && lane == 0)
            for (int b = 0; b < 2; b++)
                if (commit_par[b] >= 0) mbar_wait_drain(&tfull[b], (uint32_t)commit_par[b]);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// ---- CTA-pair variant ----------------------------------------------------------------------
// A cluster of two CTAs computes 256 x 256 tiles of the upper triangle with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r holds rows 128 r .. of the tile
// (its A panel) and columns 128 r .. of the B panel, so per 64-token k-block each SM loads
// 32 KB instead of 48 KB for the same FLOPs, and the tensor cores read each B half once for
// both SMs.  Protocol (the pair leader is CTA rank 0):
//   * full[s]  (leader): armed once per stage by the leader with both CTAs' bytes; both
//     CTAs' TMA loads complete on it;
//   * empty[s] (each CTA): one arrive from the leader's multicast commit when the MMAs that
//     read stage s have completed;
//   * tfull[b] (each CTA): one arrive from the leader's multicast commit when accumulator b
//     is complete;
//   * tempty[b] (leader): one arrive per epilogue warp of both CTAs after folding b.
// TMEM is allocated for the pair (same 512 columns in both SMs); each CTA's epilogue reads
// its own 128 rows.  Before exit each producer waits until every stage it filled has been
// released, so no arrive or load targets a CTA that has left.
//
// Work units are (token split, tile), split-major, tiles in the order of PairArgs::tiles.
// Dynamic order (DYN): the leader's producer takes the next unit from a device counter and
// hands it to every role of both CTAs through a ring of UR slots:
//   * uring[k % UR] (each CTA) holds the unit (-1 when the work is exhausted);
//   * ufull[k % UR] (each CTA): one arrive (release, cluster scope) from the leader's producer
//     after it has written the slot in both CTAs;
//   * uempty[k % UR] (leader): one arrive from each reader of the slot: the MMA issuer, the
//     other CTA's producer and the 16 epilogue warps.
// The units in flight are then always a contiguous stretch of the unit order, whose tiles
// share X panels and whose token range is one split, so their X reads meet in L2 however
// unevenly the pairs progress.  Static order: pair p runs units p, p + pairs, ...
constexpr int P_STAGES = 6;
constexpr int P_HALF_BYTES = 128 * BK * 2;         // 16 KB: 128 features x 64 tokens
constexpr int P_STAGE_BYTES = 2 * P_HALF_BYTES;    // A half + B half
constexpr int P_SMEM_MAIN = P_STAGES * P_STAGE_BYTES;  // 192 KB
constexpr int P_SMEM_BYTES = P_SMEM_MAIN + EPI_WARPS * OUT_BYTES + 1024 + 256;
static_assert(P_SMEM_BYTES <= 232448, "shared memory above the per-block limit");
constexpr int UR = 4;                             // unit ring slots
// An epilogue warp hands a folded TMEM accumulator back to the leader's MMA issuer with a
// CTA-scope release arrive: it publishes no memory, and a cluster-scope release fence after every
// fold stalled the epilogue.
#define SYRK_TEMPTY_ARRIVE mbar_arrive_cluster_cta
constexpr int UR_READERS = 2 + 2 * EPI_WARPS;     // leader's MMA issuer, rank 1's producer, 16 epilogue warps
static_assert((2 * P_STAGES + 4 + 2 * UR) * 8 + 8 + UR * 4 <= 256, "barrier area");

constexpr int P_MAX_NT = 160;                                // d <= 40960
constexpr int P_MAX_TILES = P_MAX_NT * (P_MAX_NT + 1) / 2;   // 12,880

struct PairArgs {
    float* H;
    int64_t ldh;
    int d;
    int nt;        // 256-wide blocks per side
    int ntiles;    // nt (nt + 1) / 2 upper-triangle tiles
    int kb_total;
    int splits;
    int kb_per_split;
    int* err;
    int* next_unit;  // DYN: unit counter, zero at launch
    uint32_t wait_limit;
    uint32_t idesc;
    // Tile order, (ti << 8) | tj: column strips walked row by row, so that the tiles one wave
    // of pairs works on share few X panels and those panels stay in L2.
    uint16_t tiles[P_MAX_TILES];
};
static_assert(sizeof(PairArgs) + 2 * sizeof(CUtensorMap) <= 32764, "kernel parameters above the limit");

// Unit u of PairArgs: this CTA's rows i0, the pair's columns j0 and the k-block range.
struct PairUnit {
    int i0, j0, kb0, kb1, nchunks;
};
__device__ __forceinline__ PairUnit pair_unit(const PairArgs& a, int u, uint32_t rank) {
    const int split = u / a.ntiles, tile = u % a.ntiles;
    const int ti = a.tiles[tile] >> 8, tj = a.tiles[tile] & 0xFF;
    PairUnit p;
    p.kb0 = split * a.kb_per_split;
    p.kb1 = min(a.kb_total, p.kb0 + a.kb_per_split);
    p.nchunks = (p.kb1 - p.kb0 + KF - 1) / KF;
    p.i0 = ti * 256 + (int)rank * 128;
    p.j0 = tj * 256;
    return p;
}

template <bool DYN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NT, 1)
    syrk_tc2_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap hmap, const PairArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* outbufs = smem + P_SMEM_MAIN;
    uint64_t* full = reinterpret_cast<uint64_t*>(outbufs + EPI_WARPS * OUT_BYTES);
    uint64_t* empty = full + P_STAGES;
    uint64_t* tfull = empty + P_STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* ufull = tempty + 2;
    uint64_t* uempty = ufull + UR;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(uempty + UR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* uring = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI_WARPS);
        }
        for (int k = 0; k < UR; k++) {
            mbar_init(&ufull[k], 1);
            mbar_init(&uempty[k], UR_READERS);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int total_units = a.ntiles * a.splits;
    // k-th unit of this pair, for a role that reads the ring (DYN) or walks the static order;
    // -1 when there is no further unit or the wait gave up.
    auto take = [&](uint32_t k) -> int {
        if constexpr (DYN) {
            const int slot = (int)(k % UR);
            if (!mbar_wait_cluster(&ufull[slot], (k / UR) & 1u, abort_flag, a.err, a.wait_limit)) return -1;
            const int u = uring[slot];
            mbar_arrive_cluster(mapa_shared(smem_u32(&uempty[slot]), 0));
            return u;
        } else {
            const int u = pair + (int)k * npairs;
            return u < total_units ? u : -1;
        }
    };
    // Leader producer (DYN): claim the k-th unit and publish it to both CTAs.
    auto publish = [&](uint32_t k) -> int {
        const int slot = (int)(k % UR);
        if (!mbar_wait_cluster(&uempty[slot], ((k / UR) & 1u) ^ 1u, abort_flag, a.err, a.wait_limit)) return -1;
        int u = atomicAdd(a.next_unit, 1);
        if (u >= total_units) u = -1;
        uring[slot] = u;
        st_cluster_u32(mapa_shared(smem_u32((const void*)&uring[slot]), 1), (uint32_t)u);
        mbar_arrive_cluster(mapa_shared(smem_u32(&ufull[slot]), 0));
        mbar_arrive_cluster(mapa_shared(smem_u32(&ufull[slot]), 1));
        return u;
    };

    uint32_t prod_it = 0, mma_it = 0, cc = 0;
    int pend_par[P_STAGES];
#pragma unroll
    for (int s = 0; s < P_STAGES; s++) pend_par[s] = -1;
    int commit_par[2] = {-1, -1};

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer (this CTA's halves of the A and B panels)
            for (uint32_t k = 0; !*abort_flag; k++) {
                const int u = (DYN && rank == 0) ? publish(k) : take(k);
                if (u < 0) break;
                const PairUnit pu = pair_unit(a, u, rank);
                const int jb = pu.j0 + (int)rank * 128;  // this CTA's half of the B panel
                for (int kb = pu.kb0; kb < pu.kb1; kb++, prod_it++) {
                    const int s = prod_it % P_STAGES;
                    const uint32_t ph = (prod_it / P_STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    unsigned char* st = smem + s * P_STAGE_BYTES;
                    if (rank == 0) mbar_expect_tx(&full[s], 2 * P_STAGE_BYTES);
                    const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
                    const int y = kb * BK;
                    tma_load_2d_pair(st, &xmap, pu.i0, y, fbar);
                    tma_load_2d_pair(st + BOX_BYTES, &xmap, pu.i0 + 64, y, fbar);
                    tma_load_2d_pair(st + P_HALF_BYTES, &xmap, jb, y, fbar);
                    tma_load_2d_pair(st + P_HALF_BYTES + BOX_BYTES, &xmap, jb + 64, y, fbar);
                    pend_par[s] = (int)ph;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---- MMA issuer: chunk c accumulates into TMEM buffer (cc & 1)
            for (uint32_t k = 0; !*abort_flag; k++) {
                const int u = take(k);
                if (u < 0) break;
                const PairUnit pu = pair_unit(a, u, rank);
                bool ok = true;
                for (int c = 0; c < pu.nchunks && ok; c++, cc++) {
                    const int b = (int)(cc & 1u);
                    if (!mbar_wait(&tempty[b], ((cc >> 1) & 1u) ^ 1u, abort_flag, a.err, a.wait_limit)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dst = tmem + (uint32_t)(b * BN);
                    const int k0 = pu.kb0 + c * KF, k1 = min(pu.kb1, k0 + KF);
                    for (int kb = k0; kb < k1; kb++, mma_it++) {
                        const int s = mma_it % P_STAGES;
                        const uint32_t ph = (mma_it / P_STAGES) & 1u;
                        if (!mbar_wait(&full[s], ph, abort_flag, a.err, a.wait_limit)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t abase = smem_u32(smem + s * P_STAGE_BYTES);
                        const uint32_t bbase = abase + P_HALF_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            const uint64_t da = smem_desc_mn_sw128(abase + kk * 2048, BOX_BYTES);
                            const uint64_t db = smem_desc_mn_sw128(bbase + kk * 2048, BOX_BYTES);
                            umma2_f16(dst, da, db, a.idesc, (kb > k0 || kk > 0) ? 1u : 0u);
                        }
                        umma2_commit_mc(&empty[s], 0x3);
                    }
                    umma2_commit_mc(&tfull[b], 0x3);  // chunk complete (fires even if the loop broke early)
                    commit_par[b] = (int)((cc >> 1) & 1u);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue warps: TMEM lane quadrant q, column half h
        const int e = warp - 2, q = warp % 4, h = e / 4;
        for (uint32_t k = 0; !*abort_flag; k++) {
            int u = 0;
            if (lane == 0) u = take(k);
            u = __shfl_sync(0xffffffffu, u, 0);
            if (u < 0) break;
            const PairUnit pu = pair_unit(a, u, rank);
            float acc[BN / 2];
#pragma unroll
            for (int i = 0; i < BN / 2; i++) acc[i] = 0.f;
            bool ok = true;
            for (int c = 0; c < pu.nchunks; c++, cc++) {
                const int b = (int)(cc & 1u);
                const bool have = mbar_wait(&tfull[b], (cc >> 1) & 1u, abort_flag, a.err, a.wait_limit);
                if (!__all_sync(0xffffffffu, have ? 1 : 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + h * 128);
#pragma unroll
                for (int part = 0; part < 4; part++) {
                    uint32_t v[32];
                    tmem_ld32(taddr + part * 32, v);
#pragma unroll
                    for (int i = 0; i < 32; i++) acc[part * 32 + i] = __fadd_rn(acc[part * 32 + i], __uint_as_float(v[i]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) SYRK_TEMPTY_ARRIVE(mapa_shared(smem_u32(&tempty[b]), 0));
            }
            if (!ok || *abort_flag) break;
            // Write-out: rounds of one 32 x 32 box (rows of quadrant q, columns j0 + 128 h +
            // 32 round ..) through this warp's buffer, reused only after the previous reduce has
            // read it; TMA clips rows / columns beyond d.
            unsigned char* ob = outbufs + e * OUT_BYTES;
            const uint32_t ob_s = smem_u32(ob);
#pragma unroll
            for (int round = 0; round < 4; round++) {
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const int i = round * 32 + c * 4;
                    *reinterpret_cast<float4*>(ob + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                        make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    tma_reduce_add_2d(&hmap, ob_s, pu.j0 + h * 128 + round * 32, pu.i0 + q * 32);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
        }
    }

    // Tail: the producer waits until the MMAs have released every stage it filled (so no
    // commit arrive is still on its way here), after an abort also for its loads (bounded).
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (warp == 0 && lane == 0)
        for (int s = 0; s < P_STAGES; s++)
            if (pend_par[s] >= 0) mbar_wait_drain(&empty[s], (uint32_t)pend_par[s]);
    if (*abort_flag && warp == 1 && lane == 0 && rank == 0)
        for (int b = 0; b < 2; b++)
            if (commit_par[b] >= 0) mbar_wait_drain(&tfull[b], (uint32_t)commit_par[b]);
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// ---- host side -------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

uint32_t make_idesc(int dtype, int m = BM, int n = BN) {
    const uint32_t fmt = dtype == LLMC_DTYPE_BF16 ? 1u : 0u;  // kind::f16 operand: 0 = F16, 1 = BF16
    uint32_t d = 0;
    d |= 1u << 4;                 // D format: F32
    d |= fmt << 7;                // A format
    d |= fmt << 10;               // B format
    d |= 1u << 15;                // A major: MN
    d |= 1u << 16;                // B major: MN
    d |= (uint32_t)(n >> 3) << 17;
    d |= (uint32_t)(m >> 4) << 24;
    return d;
}

// Unit order of the pair kernel: dynamic (a device counter deals units in order) or static.
constexpr bool SYRK_DYNAMIC = true;
// Dynamic order: token splits sized to about this many k-blocks per unit, so that the X rows
// of the units in flight (one split's token range) stay in L2.
constexpr int SYRK_UNIT_KB = 256;
// Index of the unit counter in the context's device flag words.
constexpr int SYRK_COUNTER_WORD = 8;

// Token splits for the dynamic order: about SYRK_UNIT_KB k-blocks per unit, at most 16 splits,
// and >= 32 k-blocks per unit when split.  From there up to half as many splits again may be
// added when that fills the last wave of `pairs` better (units are dealt one at a time, so the
// launch ends with a partly filled wave of equal units): at d = 4,096 on 58 pairs, 4 splits give
// 9.38 waves of units (0.938 of the last wave's slots used over the launch), 5 give 11.72 (0.977).
int unit_splits(int kb_total, int ntiles, int pairs) {
    int s0 = (kb_total + SYRK_UNIT_KB / 2) / SYRK_UNIT_KB;
    if (s0 > 16) s0 = 16;
    while (s0 > 1 && (kb_total + s0 - 1) / s0 < 32) s0--;
    if (s0 < 1) s0 = 1;
    if (pairs < 1) return s0;
    int best = s0;
    double best_eff = 0.0;
    for (int s = s0; s <= 16 && s <= s0 + s0 / 2; s++) {
        if (s > 1 && (kb_total + s - 1) / s < 32) break;
        const long long units = (long long)ntiles * s;
        const long long waves = (units + pairs - 1) / pairs;
        const double eff = (double)units / ((double)waves * pairs);
        if (eff > best_eff + 1e-3) {
            best_eff = eff;
            best = s;
        }
    }
    return best;
}

// Token splits: balance the last wave over `cap` workers while keeping >= 32 k-blocks (2048
// tokens) per unit.
int pick_splits(int ntiles, int kb_total, int cap) {
    int best_s = 1;
    double best_eff = 0.0;
    for (int s = 1; s <= 16; s++) {
        const int kps = (kb_total + s - 1) / s;
        if (s > 1 && kps < 32) break;
        const int units = ntiles * s;
        const int waves = (units + cap - 1) / cap;
        const double eff = (double)units / ((double)waves * cap);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best_s = s;
        }
    }
    return best_s;
}

// CTA pairs of syrk_tc2_kernel that can be resident at once on the context's device (0 when
// the pair kernel cannot be used); computed once per device.
int max_pairs(llmc_ctx* ctx) {
    static std::mutex mu;
    static int cache[64];
    static bool known[64];
    const int dev = ctx->device;
    if (dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!known[dev]) {
        known[dev] = true;
        cache[dev] = 0;
        if (cudaFuncSetAttribute(syrk_tc2_kernel<SYRK_DYNAMIC>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES) !=
            cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (unsigned)ctx->sm_count, 1, 1);
        cfg.blockDim = dim3(NT, 1, 1);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void*)syrk_tc2_kernel<SYRK_DYNAMIC>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            cfg.numAttrs = 0;
            if (cudaOccupancyMaxActiveClusters(&n, (const void*)syrk_tc2_kernel<SYRK_DYNAMIC>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
        }
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace

int syrk_tc_error_word_index() { return 2; }

llmc_status syrk_tc(llmc_ctx* ctx, const void* x, int dtype, int64_t rows, int64_t d, int64_t ld, float* H, int64_t ldh) {
    if (dtype != LLMC_DTYPE_BF16 && dtype != LLMC_DTYPE_F16) return LLMC_ERR_UNSUPPORTED;
    // Contract of the tensor map and of the bulk reduce epilogue.
    if (((uintptr_t)x % 16) != 0 || (ld % 8) != 0 || (d % 4) != 0 || (ldh % 4) != 0 || ((uintptr_t)H % 16) != 0)
        return LLMC_ERR_UNSUPPORTED;
    if (d < 64 || rows < BK || rows > (int64_t)INT32_MAX) return LLMC_ERR_UNSUPPORTED;
    const int ntj = (int)((d + BN - 1) / BN), nti = (int)((d + BM - 1) / BM);
    if (ntj > MAX_TJ) return LLMC_ERR_UNSUPPORTED;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return LLMC_ERR_UNSUPPORTED;

    SyrkArgs a{};
    a.H = H;
    a.ldh = ldh;
    a.d = (int)d;
    a.nti = nti;
    a.ntj = ntj;
    int off = 0;
    for (int tj = 0; tj < ntj; tj++) {
        a.tile_off[tj] = off;
        off += min(2 * tj + 2, nti);  // row panels ti with 128*ti <= 256*tj + 255
    }
    a.tile_off[ntj] = off;
    a.ntiles = off;
    a.kb_total = (int)((rows + BK - 1) / BK);
    const int grid_cap = persistent_sms(ctx);
    a.splits = pick_splits(a.ntiles, a.kb_total, grid_cap);
    a.kb_per_split = (a.kb_total + a.splits - 1) / a.splits;
    a.err = ctx->dflags + 2;
    a.wait_limit = ctx->wait_limit;
    a.idesc = make_idesc(dtype);

    CUtensorMap map;
    const cuuint64_t gdim[2] = {(cuuint64_t)d, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {64, BK};
    const cuuint32_t estride[2] = {1, 1};
    CUresult cr = enc(&map, dtype == LLMC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                      const_cast<void*>(x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(LLMC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);
    // H [d, d] fp32 (row stride ldh) as the target of the epilogue's 32 x 32 reduce-adds.
    CUtensorMap hmap;
    const cuuint64_t hdim[2] = {(cuuint64_t)d, (cuuint64_t)d};
    const cuuint64_t hstride[1] = {(cuuint64_t)ldh * 4};
    const cuuint32_t hbox[2] = {OUT_BOX, OUT_BOX};
    cr = enc(&hmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, H, hdim, hstride, hbox, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(LLMC_ERR_CUDA, "cuTensorMapEncodeTiled (H) failed (%d)", (int)cr);

    if (d >= 256 && d <= 256 * P_MAX_NT) {
        const int pcap = min(persistent_sms(ctx) / 2, max_pairs(ctx));
        if (pcap >= 1) {
            PairArgs p{};
            p.H = H;
            p.ldh = ldh;
            p.d = (int)d;
            p.nt = (int)((d + 255) / 256);
            p.ntiles = p.nt * (p.nt + 1) / 2;
            // Column strips GJ tiles wide (GJ ~ sqrt(2 pairs)), each walked row by row: a wave
            // of pairs covers about GJ column panels and pairs / GJ row panels of X.
            int GJ = 1;
            while ((GJ + 1) * (GJ + 1) <= 2 * pcap) GJ++;
            int n = 0;
            for (int bj = 0; bj < p.nt; bj += GJ) {
                const int ej = min(p.nt, bj + GJ);
                for (int ti = 0; ti < ej; ti++)
                    for (int tj = max(bj, ti); tj < ej; tj++) p.tiles[n++] = (uint16_t)((ti << 8) | tj);
            }
            if (n != p.ntiles) return fail(LLMC_ERR_INTERNAL, "syrk pair tile order: %d of %d tiles", n, p.ntiles);
            p.kb_total = a.kb_total;
            p.splits = SYRK_DYNAMIC ? unit_splits(p.kb_total, p.ntiles, pcap) : pick_splits(p.ntiles, p.kb_total, pcap);
            p.kb_per_split = (p.kb_total + p.splits - 1) / p.splits;
            p.err = ctx->dflags + 2;
            p.next_unit = ctx->dflags + SYRK_COUNTER_WORD;
            p.wait_limit = ctx->wait_limit;
            p.idesc = make_idesc(dtype, 256, 256);
            const int punits = p.ntiles * p.splits;
            const int pairs = punits < pcap ? punits : pcap;
            if (SYRK_DYNAMIC) LLMC_CUDA_TRY(cudaMemsetAsync(p.next_unit, 0, sizeof(int), ctx->stream));
            syrk_tc2_kernel<SYRK_DYNAMIC><<<2 * pairs, NT, P_SMEM_BYTES, ctx->stream>>>(map, hmap, p);
            return check_launch(ctx, "syrk_tc2");
        }
    }
    static bool attr[64];  // per device
    if (ctx->device < 0 || ctx->device >= 64) return LLMC_ERR_UNSUPPORTED;
    if (!attr[ctx->device]) {
        LLMC_CUDA_TRY(cudaFuncSetAttribute(syrk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr[ctx->device] = true;
    }
    const int units = a.ntiles * a.splits;
    const int grid = units < grid_cap ? units : grid_cap;
    syrk_tc_kernel<<<grid, NT, SMEM_BYTES, ctx->stream>>>(map, hmap, a);
    return check_launch(ctx, "syrk_tc");
}

}  // namespace llmc
