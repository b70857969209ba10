// fp32 GEMM on the 5th-generation tensor cores with a 3 x TF32 split (sm_100a).
//
// Serves the O(d^3) fp32 parts of the hot path: the Cholesky / triangular-inverse recursion
// (HessianInverseSolver.cs:62-90) and the GPTQ lazy tail update W[:, i2:] -= Err1 U[i1:i2, i2:]
// (GptqBlockQuantizer.cs:173-180).
//
// C[M,N] = alpha * op(A) op(B) + beta * C with fp32 operands split (by split2d_kernel) into
// x = hi + lo, hi = x rounded to TF32 (low 13 mantissa bits zero) and lo = x - hi (exact in
// fp32).  The product is hi_a hi_b + hi_a lo_b + lo_a hi_b: three tcgen05.mma kind::tf32
// per K step, error ~2^-21 relative per product (the dropped lo_a lo_b and the TF32 view of
// the lo terms), i.e. fp32-grade.
//
// Per CTA (one output tile of 128 x 128, 192 threads):
//   warp 0: TMA producer, 3-stage ring of {A hi, A lo, B hi, B lo} tiles of 32 K-elements,
//           128-byte swizzle, K-major or MN-major per operand, no multicast;
//   warp 1: one thread issues the MMAs into one of two TMEM accumulators (128 columns each);
//   warps 2-5: fold each accumulator into fp32 registers every KF k-blocks (the tensor core's
//           accumulation truncates; folding bounds that to KF*32 K-elements), then write
//           C = alpha*acc + beta*C (optionally only the lower triangle).
// Triangular operands restrict each tile's K range (the skipped region must be zero).
// Every wait is bounded (error word + drain + TMEM release, as in the Hessian kernel).
#include "ops.h"
#include "tc_common.cuh"

#include <cuda.h>

#include <mutex>

namespace llmc {
namespace {

using namespace tc;

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int EPI_WARPS = 4, NT = 32 * (2 + EPI_WARPS);
constexpr int KF = 2;                       // k-blocks (64 K-elements, 24 MMAs) per TMEM accumulation
constexpr int TILE_BYTES = BM * BK * 4;     // 16 KB per operand part
constexpr int STAGE_BYTES = 4 * TILE_BYTES; // A hi, A lo, B hi, B lo
constexpr int SMEM_MAIN = STAGES * STAGE_BYTES;
constexpr int SMEM_BYTES = SMEM_MAIN + 1024 + 256;
constexpr int TMEM_COLS = 2 * BN;

struct TcGemmArgs {
    int64_t M, N, K;
    float* C;
    int64_t ldc;
    float alpha, beta;
    int a_tri, b_tri, c_mode;
    int* err;
    uint32_t wait_limit;  // try_wait attempts per bounded wait (llmc_set_wait_limit)
    uint32_t idesc;
    int tiles_m, tiles_n, group;  // 1-D grid: tiles visited in column strips of `group` M-tiles
    int splits;                   // K splits per tile (pair kernel; > 1 needs beta == 1)
};

// Loads one operand part (128 rows of the MN dimension x 32 K-elements, K contiguous) for a
// k-block: box {32 K, 128 rows}, i.e. 128 rows of 128 B in 8-row 128-byte-swizzle atoms.
__device__ __forceinline__ void load_part(unsigned char* dst, const CUtensorMap* map, int mn0, int k0, uint64_t* bar) {
    tma_load_2d(dst, map, k0, mn0, bar);
}

// K step of 8 TF32 elements = 32 bytes inside each 128-byte K-major row.
__device__ __forceinline__ uint64_t part_desc(uint32_t base, int kk) { return smem_desc_k_sw128(base + kk * 32); }

__global__ void __launch_bounds__(NT, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap ahi,
                                                        const __grid_constant__ CUtensorMap alo,
                                                        const __grid_constant__ CUtensorMap bhi,
                                                        const __grid_constant__ CUtensorMap blo, const TcGemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SMEM_MAIN);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
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

    int pend_par[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; s++) pend_par[s] = -1;
    int commit_par[2] = {-1, -1};
    // Counters that run on across this CTA's tiles: stages filled (producer) and consumed
    // (MMA issuer); accumulation chunks (MMA issuer and epilogue: TMEM buffer cc & 1).
    uint32_t prod_it = 0, mma_it = 0, cc = 0;

    // Persistent CTAs: tile t = blockIdx.x, +gridDim.x, ...  Consecutive tiles walk a strip of
    // `group` M-tiles column by column, so the tiles in flight share few A and B panels.
    const int total_tiles = a.tiles_m * a.tiles_n;
    const int per_group = a.group * a.tiles_n;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const int gidx = t / per_group;
        const int first_m = gidx * a.group;
        const int gm = min(a.group, a.tiles_m - first_m);
        const int local = t - gidx * per_group;
        const int64_t m0 = (int64_t)(first_m + local % gm) * BM, n0 = (int64_t)(local / gm) * BN;
        if (a.c_mode == 1 && m0 + BM - 1 < n0) continue;  // tile entirely above the diagonal
        if (a.c_mode == 2 && m0 > n0 + BN - 1) continue;  // tile entirely below the diagonal

        int64_t kb_lo = 0, kb_hi = a.K;
        if (a.a_tri == TRI_KLE) kb_hi = min(kb_hi, m0 + BM);
        if (a.a_tri == TRI_KGE) kb_lo = max(kb_lo, m0);
        if (a.b_tri == TRI_KLE) kb_hi = min(kb_hi, n0 + BN);
        if (a.b_tri == TRI_KGE) kb_lo = max(kb_lo, n0);
        const int kb0 = (int)(kb_lo / BK);
        const int kb1 = kb_hi > kb_lo ? (int)((kb_hi + BK - 1) / BK) : kb0;
        const int nchunks = (kb1 - kb0 + KF - 1) / KF;

        if (warp == 0) {
            if (lane == 0) {
                for (int kb = kb0; kb < kb1; kb++, prod_it++) {
                    const int s = prod_it % STAGES;
                    const uint32_t ph = (prod_it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    unsigned char* st = smem + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    const int k0 = kb * BK;
                    load_part(st + 0 * TILE_BYTES, &ahi, (int)m0, k0, &full[s]);
                    load_part(st + 1 * TILE_BYTES, &alo, (int)m0, k0, &full[s]);
                    load_part(st + 2 * TILE_BYTES, &bhi, (int)n0, k0, &full[s]);
                    load_part(st + 3 * TILE_BYTES, &blo, (int)n0, k0, &full[s]);
                    pend_par[s] = (int)ph;
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0) {
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
                        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 8; kk++) {
                            const uint64_t dah = part_desc(base + 0 * TILE_BYTES, kk);
                            const uint64_t dal = part_desc(base + 1 * TILE_BYTES, kk);
                            const uint64_t dbh = part_desc(base + 2 * TILE_BYTES, kk);
                            const uint64_t dbl = part_desc(base + 3 * TILE_BYTES, kk);
                            const uint32_t first = (kb == k0 && kk == 0) ? 0u : 1u;
                            umma_tf32(dst, dah, dbh, a.idesc, first);
                            umma_tf32(dst, dah, dbl, a.idesc, 1u);
                            umma_tf32(dst, dal, dbh, a.idesc, 1u);
                        }
                        umma_commit(&empty[s]);
                    }
                    umma_commit(&tfull[b]);
                    commit_par[b] = (int)((c_it >> 1) & 1u);
                    if (!ok) break;
                }
            }
            __syncwarp();
        } else {
            // epilogue warps: TMEM lane quadrant q = warp % 4 = rows [32q, 32q + 32) of the tile
            const int q = warp % 4;
            float acc[BN];
#pragma unroll
            for (int i = 0; i < BN; i++) acc[i] = 0.f;
            uint32_t c_it = cc;
            bool ok = true;
            for (int c = 0; c < nchunks; c++, c_it++) {
                const int b = (int)(c_it & 1u);
                const bool have = mbar_wait(&tfull[b], (c_it >> 1) & 1u, abort_flag, a.err, a.wait_limit);
                if (!__all_sync(0xffffffffu, have ? 1 : 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < BN / 32; part++) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + part * 32), v);
#pragma unroll
                    for (int i = 0; i < 32; i++) acc[part * 32 + i] = __fadd_rn(acc[part * 32 + i], __uint_as_float(v[i]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
            }
            // Write-out of this tile; the MMA issuer meanwhile fills TMEM for the next tile.
            const int64_t r = m0 + q * 32 + lane;
            if (ok && r < a.M && !*abort_flag) {
                float* crow = a.C + r * a.ldc + n0;
                const bool vec = ((reinterpret_cast<uintptr_t>(crow) & 15u) == 0) && n0 + BN <= a.N &&
                                 !(a.c_mode == 1 && r < n0 + BN - 1);
                if (vec) {
#pragma unroll
                    for (int i = 0; i < BN; i += 4) {
                        float4 o = make_float4(a.alpha * acc[i], a.alpha * acc[i + 1], a.alpha * acc[i + 2],
                                               a.alpha * acc[i + 3]);
                        if (a.beta != 0.f) {
                            const float4 c = *reinterpret_cast<const float4*>(crow + i);
                            o.x = fmaf(a.beta, c.x, o.x);
                            o.y = fmaf(a.beta, c.y, o.y);
                            o.z = fmaf(a.beta, c.z, o.z);
                            o.w = fmaf(a.beta, c.w, o.w);
                        }
                        *reinterpret_cast<float4*>(crow + i) = o;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < BN; i++) {
                        const int64_t col = n0 + i;
                        if (col < a.N && !(a.c_mode == 1 && r < col)) {
                            const float v = a.alpha * acc[i];
                            crow[i] = (a.beta == 0.f) ? v : fmaf(a.beta, crow[i], v);
                        }
                    }
                }
            }
        }
        cc += (uint32_t)nchunks;
    }

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

// ---- CTA-pair variant (large products) -----------------------------------------------------------
// A cluster of two CTAs computes 256 x 256 output tiles with tcgen05.mma.cta_group::2.kind::tf32
// (M = 256, N = 256, K = 8): CTA r stages A hi / lo for rows 128 r .. of the tile and B hi / lo
// for columns 128 r .., so each SM moves 64 KB per 32-K step for twice the MMA work of the
// 128 x 128 kernel and the tensor cores read each B half once for both SMs.  Barrier protocol
// as in the Hessian pair kernel: the leader (rank 0) arms full[s] with both CTAs' bytes and
// issues the MMAs; its commits are multicast to both CTAs' empty / tfull barriers; epilogue
// warps of both CTAs arrive on the leader's tempty; producers wait for their last stages to be
// released before the cluster exits.
constexpr int P_EPI = 8, P_NT = 32 * (2 + P_EPI);
constexpr int P_BN = 256;                       // columns per pair tile (128 per CTA's B half)
constexpr int P_STAGE_BYTES = 4 * TILE_BYTES;   // A hi, A lo (128 rows), B hi, B lo (128 columns)
constexpr int P_SMEM_MAIN = STAGES * P_STAGE_BYTES;
constexpr int P_OUT_BYTES = 32 * 32 * 4;         // epilogue box per warp: 32 rows x 32 fp32
constexpr int P_SMEM_BYTES = P_SMEM_MAIN + P_EPI * P_OUT_BYTES + 1024 + 256;
static_assert(P_SMEM_BYTES <= 232448, "shared memory above the per-block limit");
constexpr int P_TMEM_COLS = 2 * P_BN;
// k-blocks (64 K-elements, 24 MMAs) per TMEM accumulation of the pair kernel, as in the 1-CTA
// kernel.  Folding every 4 k-blocks (128 K-elements of truncating tensor-core accumulation)
// took the fp32 Hessian of a 4,096-row, d = 576 input to 1.13e-6 relative Frobenius against the
// oracle, over the 1e-6 bar of the fp32 path.
constexpr int P_KF = 2;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_NT, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap ahi, const __grid_constant__ CUtensorMap alo,
                    const __grid_constant__ CUtensorMap bhi, const __grid_constant__ CUtensorMap blo,
                    const __grid_constant__ CUtensorMap cmap, const TcGemmArgs a, const int tma_out) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* outbufs = smem + P_SMEM_MAIN;  // P_EPI x 4 KB, 1024-byte aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(outbufs + P_EPI * P_OUT_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * P_EPI);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int pend_par[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; s++) pend_par[s] = -1;
    int commit_par[2] = {-1, -1};
    uint32_t prod_it = 0, mma_it = 0, cc = 0;

    const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
    const int total_tiles = a.tiles_m * a.tiles_n;  // 256 x 256 pair tiles
    const int per_group = a.group * a.tiles_n;
    // A unit is a tile x a K split; consecutive units are tiles of one split, which read the
    // same K range of the operands.
    const int total_units = total_tiles * a.splits;
    for (int u = pair; u < total_units && !*abort_flag; u += npairs) {
        const int t = u % total_tiles, sp = u / total_tiles;
        const int gidx = t / per_group;
        const int first_m = gidx * a.group;
        const int gm = min(a.group, a.tiles_m - first_m);
        const int local = t - gidx * per_group;
        const int64_t pm0 = (int64_t)(first_m + local % gm) * 256, n0 = (int64_t)(local / gm) * P_BN;
        if (a.c_mode == 1 && pm0 + 255 < n0) continue;
        if (a.c_mode == 2 && pm0 > n0 + P_BN - 1) continue;
        int64_t kb_lo = 0, kb_hi = a.K;
        if (a.a_tri == TRI_KLE) kb_hi = min(kb_hi, pm0 + 256);
        if (a.a_tri == TRI_KGE) kb_lo = max(kb_lo, pm0);
        if (a.b_tri == TRI_KLE) kb_hi = min(kb_hi, n0 + P_BN);
        if (a.b_tri == TRI_KGE) kb_lo = max(kb_lo, n0);
        int kb0 = (int)(kb_lo / BK);
        int kb1 = kb_hi > kb_lo ? (int)((kb_hi + BK - 1) / BK) : kb0;
        if (a.splits > 1) {
            const int per = (kb1 - kb0 + a.splits - 1) / a.splits;
            const int s0 = kb0 + sp * per, s1 = min(kb1, s0 + per);
            if (s0 >= s1) continue;  // nothing to add for this split
            kb0 = s0;
            kb1 = s1;
        }
        const int nchunks = (kb1 - kb0 + P_KF - 1) / P_KF;
        const int64_t m0 = pm0 + (int64_t)rank * 128;   // this CTA's rows
        const int64_t nb = n0 + (int64_t)rank * 128;    // this CTA's half of the B panel

        if (warp == 0) {
            if (lane == 0) {
                for (int kb = kb0; kb < kb1; kb++, prod_it++) {
                    const int s = prod_it % STAGES;
                    const uint32_t ph = (prod_it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    unsigned char* st = smem + s * P_STAGE_BYTES;
                    if (rank == 0) mbar_expect_tx(&full[s], 2 * P_STAGE_BYTES);
                    const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
                    const int k0 = kb * BK;
                    tma_load_2d_pair(st + 0 * TILE_BYTES, &ahi, k0, (int)m0, fbar);
                    tma_load_2d_pair(st + 1 * TILE_BYTES, &alo, k0, (int)m0, fbar);
                    tma_load_2d_pair(st + 2 * TILE_BYTES, &bhi, k0, (int)nb, fbar);
                    tma_load_2d_pair(st + 3 * TILE_BYTES, &blo, k0, (int)nb, fbar);
                    pend_par[s] = (int)ph;
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0 && rank == 0) {
                uint32_t c_it = cc;
                for (int c = 0; c < nchunks && !*abort_flag; c++, c_it++) {
                    const int b = (int)(c_it & 1u);
                    if (!mbar_wait(&tempty[b], ((c_it >> 1) & 1u) ^ 1u, abort_flag, a.err, a.wait_limit)) break;
                    tc_fence_after();
                    const uint32_t dst = tmem + (uint32_t)(b * P_BN);
                    const int k0 = kb0 + c * P_KF, k1 = min(kb1, k0 + P_KF);
                    bool ok = true;
                    for (int kb = k0; kb < k1; kb++, mma_it++) {
                        const int s = mma_it % STAGES;
                        const uint32_t ph = (mma_it / STAGES) & 1u;
                        if (!mbar_wait(&full[s], ph, abort_flag, a.err, a.wait_limit)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t base = smem_u32(smem + s * P_STAGE_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 8; kk++) {
                            const uint64_t dah = part_desc(base + 0 * TILE_BYTES, kk);
                            const uint64_t dal = part_desc(base + 1 * TILE_BYTES, kk);
                            const uint64_t dbh = part_desc(base + 2 * TILE_BYTES, kk);
                            const uint64_t dbl = part_desc(base + 3 * TILE_BYTES, kk);
                            const uint32_t first = (kb == k0 && kk == 0) ? 0u : 1u;
                            umma2_tf32(dst, dah, dbh, a.idesc, first);
                            umma2_tf32(dst, dah, dbl, a.idesc, 1u);
                            umma2_tf32(dst, dal, dbh, a.idesc, 1u);
                        }
                        umma2_commit_mc(&empty[s], 0x3);
                    }
                    umma2_commit_mc(&tfull[b], 0x3);
                    commit_par[b] = (int)((c_it >> 1) & 1u);
                    if (!ok) break;
                }
            }
            __syncwarp();
        } else {
            // epilogue warps: TMEM lane quadrant q (rows 32 q ..), column half h of the 256
            const int e = warp - 2, q = warp % 4, h = e / 4;
            float acc[128];
#pragma unroll
            for (int i = 0; i < 128; i++) acc[i] = 0.f;
            uint32_t c_it = cc;
            bool ok = true;
            for (int c = 0; c < nchunks; c++, c_it++) {
                const int b = (int)(c_it & 1u);
                const bool have = mbar_wait(&tfull[b], (c_it >> 1) & 1u, abort_flag, a.err, a.wait_limit);
                if (!__all_sync(0xffffffffu, have ? 1 : 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < 4; part++) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * P_BN + h * 128 + part * 32), v);
#pragma unroll
                    for (int i = 0; i < 32; i++) acc[part * 32 + i] = __fadd_rn(acc[part * 32 + i], __uint_as_float(v[i]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster_cta(mapa_shared(smem_u32(&tempty[b]), 0));
            }
            const int64_t r = m0 + q * 32 + lane;
            const int64_t c0 = n0 + h * 128;
            // TMA epilogue (tma_out: beta is 0 or 1, C 16-byte aligned with ldc % 4 == 0): the
            // warp's 32 x 128 block leaves in four 32 x 32 boxes through its shared buffer, as a
            // tensor store (beta 0) or reduce-add (beta 1), so no thread reads C.  Blocks not
            // wholly inside a triangle-only output's triangle take the register path below.
            const bool tri_cross = (a.c_mode == 1 && m0 + q * 32 < c0 + 127) ||
                                   (a.c_mode == 2 && m0 + q * 32 + 31 > c0);
            if (ok && tma_out && !tri_cross && !*abort_flag && m0 + q * 32 < a.M && c0 < a.N) {
                unsigned char* ob = outbufs + e * P_OUT_BYTES;
                const uint32_t ob_s = smem_u32(ob);
#pragma unroll
                for (int round = 0; round < 4; round++) {
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const int i = round * 32 + c * 4;
                        *reinterpret_cast<float4*>(ob + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                            make_float4(a.alpha * acc[i], a.alpha * acc[i + 1], a.alpha * acc[i + 2], a.alpha * acc[i + 3]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        if (tma_out == 2) tma_reduce_add_2d(&cmap, ob_s, (int)(c0 + round * 32), (int)(m0 + q * 32));
                        else tma_store_2d(&cmap, ob_s, (int)(c0 + round * 32), (int)(m0 + q * 32));
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                }
            } else if (ok && r < a.M && c0 < a.N && !*abort_flag && a.splits > 1) {
                // K split: other units add into the same C elements (beta is 1).
                float* crow = a.C + r * a.ldc + c0;
#pragma unroll
                for (int i = 0; i < 128; i++) {
                    const int64_t col = c0 + i;
                    if (col < a.N && !(a.c_mode == 1 && r < col) && !(a.c_mode == 2 && r > col))
                        atomicAdd(crow + i, a.alpha * acc[i]);
                }
            } else if (ok && r < a.M && c0 < a.N && !*abort_flag) {
                float* crow = a.C + r * a.ldc + c0;
                const bool vec = ((reinterpret_cast<uintptr_t>(crow) & 15u) == 0) && c0 + 128 <= a.N &&
                                 !(a.c_mode == 1 && r < c0 + 127) && !(a.c_mode == 2 && r > c0);
                if (vec) {
#pragma unroll
                    for (int i = 0; i < 128; i += 4) {
                        float4 o = make_float4(a.alpha * acc[i], a.alpha * acc[i + 1], a.alpha * acc[i + 2],
                                               a.alpha * acc[i + 3]);
                        if (a.beta != 0.f) {
                            const float4 cv = *reinterpret_cast<const float4*>(crow + i);
                            o.x = fmaf(a.beta, cv.x, o.x);
                            o.y = fmaf(a.beta, cv.y, o.y);
                            o.z = fmaf(a.beta, cv.z, o.z);
                            o.w = fmaf(a.beta, cv.w, o.w);
                        }
                        *reinterpret_cast<float4*>(crow + i) = o;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 128; i++) {
                        const int64_t col = c0 + i;
                        if (col < a.N && !(a.c_mode == 1 && r < col) && !(a.c_mode == 2 && r > col)) {
                            const float v = a.alpha * acc[i];
                            crow[i] = (a.beta == 0.f) ? v : fmaf(a.beta, crow[i], v);
                        }
                    }
                }
            }
        }
        cc += (uint32_t)nchunks;
    }

    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (warp == 0 && lane == 0)
        for (int s = 0; s < STAGES; s++)
            if (pend_par[s] >= 0) mbar_wait_drain(&empty[s], (uint32_t)pend_par[s]);
    if (*abort_flag && warp == 1 && lane == 0 && rank == 0)
        for (int b = 0; b < 2; b++)
            if (commit_par[b] >= 0) mbar_wait_drain(&tfull[b], (uint32_t)commit_par[b]);
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P_TMEM_COLS));
    }
}

// Pairs of gemm_tc2_kernel that can be resident at once on the context's device (0: unusable).
int max_pairs_gemm(llmc_ctx* ctx) {
    static std::mutex mu;
    static int cache[64];
    static bool known[64];
    const int dev = ctx->device;
    if (dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!known[dev]) {
        known[dev] = true;
        cache[dev] = 0;
        if (cudaFuncSetAttribute(gemm_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES) !=
            cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (unsigned)ctx->sm_count, 1, 1);
        cfg.blockDim = dim3(P_NT, 1, 1);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_tc2_kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            cfg.numAttrs = 0;
            if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_tc2_kernel, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
        }
        cache[dev] = n;
    }
    return cache[dev];
}

// hi = x rounded to TF32 (round to nearest, ties away), lo = x - hi (exact in fp32).
__device__ __forceinline__ void tf32_split(float x, float* h, float* l) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x1000u) & 0xFFFFE000u;  // finite: keep 10 mantissa bits
    *h = __uint_as_float(u);
    *l = __fsub_rn(x, *h);
}

// Split a K-major operand [rows, cols] (K = cols) into packed hi / lo copies (row stride ldd).
__global__ void split2d_kernel(const float* src, int64_t rows, int64_t cols, int64_t lds, float* hi, float* lo,
                               int64_t ldd) {
    const int64_t total = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t % cols;
        float h, l;
        tf32_split(src[i * lds + j], &h, &l);
        hi[i * ldd + j] = h;
        lo[i * ldd + j] = l;
    }
}

// Split an MN-major operand [K rows, MN cols] into K-major hi / lo copies [MN rows, K cols]
// (32 x 32 tiles through shared memory so both sides are coalesced).
__global__ void split2d_transpose_kernel(const float* src, int64_t rows, int64_t cols, int64_t lds, float* hi,
                                         float* lo, int64_t ldd) {
    __shared__ float th[32][33];
    __shared__ float tl[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int64_t r = r0 + y, c = c0 + threadIdx.x;
        float h = 0.f, l = 0.f;
        if (r < rows && c < cols) tf32_split(src[r * lds + c], &h, &l);
        th[y][threadIdx.x] = h;
        tl[y][threadIdx.x] = l;
    }
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int64_t orow = c0 + y, ocol = r0 + threadIdx.x;  // output [cols, rows]
        if (orow < cols && ocol < rows) {
            hi[orow * ldd + ocol] = th[threadIdx.x][y];
            lo[orow * ldd + ocol] = tl[threadIdx.x][y];
        }
    }
}

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

// Tensor map of a packed K-major fp32 operand [rows, cols = K] (row stride ld floats), box
// {32 K, 128 rows}.
llmc_status make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(LLMC_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {32, 128};
    const cuuint32_t estride[2] = {1, 1};
    CUresult cr = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim, gstride, box, estride,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(LLMC_ERR_CUDA, "cuTensorMapEncodeTiled (fp32) failed (%d)", (int)cr);
    return LLMC_OK;
}

// hi / lo K-major copies [mn, k] of an operand stored either K-major ([mn, k], ld) or
// MN-major ([k, mn], ld).
llmc_status split_operand(llmc_ctx* ctx, const float* src, int64_t mn, int64_t k, int64_t ld, int mn_major, float* hi,
                          float* lo, int64_t ldd);

int grid_for(llmc_ctx* ctx, int64_t items) {
    int64_t b = (items + 255) / 256;
    int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

llmc_status split_operand(llmc_ctx* ctx, const float* src, int64_t mn, int64_t k, int64_t ld, int mn_major, float* hi,
                          float* lo, int64_t ldd) {
    if (!mn_major) {
        split2d_kernel<<<grid_for(ctx, mn * k), 256, 0, ctx->stream>>>(src, mn, k, ld, hi, lo, ldd);
    } else {
        dim3 grid((unsigned)((mn + 31) / 32), (unsigned)((k + 31) / 32));
        if (grid.y > 65535) return fail(LLMC_ERR_UNSUPPORTED, "split: K too large");
        split2d_transpose_kernel<<<grid, dim3(32, 8), 0, ctx->stream>>>(src, k, mn, ld, hi, lo, ldd);
    }
    return check_launch(ctx, "split2d");
}

}  // namespace

// Tensor-core path of gemm_f32 (fp32 operands).  Returns LLMC_ERR_UNSUPPORTED when the shape
// is too small to pay for the split (the caller then runs the SIMT kernel).
llmc_status gemm_tc(llmc_ctx* ctx, const GemmArgs& g) {
    if (g.a_dtype != LLMC_DTYPE_F32 || g.b_dtype != LLMC_DTYPE_F32) return LLMC_ERR_UNSUPPORTED;
    if (g.M < 128 || g.N < 128 || g.K < 64) return LLMC_ERR_UNSUPPORTED;
    // K splits run on the pair kernel only (its epilogue adds atomically); beta must be 1.
    if (g.split_k > 1 && (g.M < 512 || g.N < 512 || g.beta != 1.f || max_pairs_gemm(ctx) < 1))
        return LLMC_ERR_UNSUPPORTED;
    if (g.M > (int64_t)INT32_MAX || g.N > (int64_t)INT32_MAX || g.K > (int64_t)INT32_MAX) return LLMC_ERR_UNSUPPORTED;
    if (((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN) > (int64_t)INT32_MAX) return LLMC_ERR_UNSUPPORTED;
    // Operands as stored: A is [M, K] (a_trans = 0) or [K, M] (a_trans = 1); B is [K, N]
    // (b_trans = 0) or [N, K] (b_trans = 1).  The split copies are K-major [M, K] and [N, K].
    const int64_t ldk = (g.K + 3) / 4 * 4;
    // A product of an operand with its own transpose (X^T X) splits the operand once.
    const bool same = g.A == g.B && g.M == g.N && g.lda == g.ldb && g.a_trans == !g.b_trans;
    const size_t need = (size_t)(2 * g.M * ldk + (same ? 0 : 2 * g.N * ldk)) * 4 + 4096;
    void* sp;
    LLMC_TRY(workspace2(ctx, need, &sp));
    Carver cv{(char*)sp};
    float* ah = cv.take<float>((size_t)g.M * ldk);
    float* al = cv.take<float>((size_t)g.M * ldk);
    float* bh = same ? ah : cv.take<float>((size_t)g.N * ldk);
    float* bl = same ? al : cv.take<float>((size_t)g.N * ldk);
    LLMC_TRY(split_operand(ctx, (const float*)g.A, g.M, g.K, g.lda, g.a_trans, ah, al, ldk));
    if (!same) LLMC_TRY(split_operand(ctx, (const float*)g.B, g.N, g.K, g.ldb, !g.b_trans, bh, bl, ldk));
    CUtensorMap mah, mal, mbh, mbl;
    LLMC_TRY(make_map(&mah, ah, g.M, g.K, ldk));
    LLMC_TRY(make_map(&mal, al, g.M, g.K, ldk));
    LLMC_TRY(make_map(&mbh, bh, g.N, g.K, ldk));
    LLMC_TRY(make_map(&mbl, bl, g.N, g.K, ldk));

    TcGemmArgs t{};
    t.M = g.M;
    t.N = g.N;
    t.K = g.K;
    t.C = g.C;
    t.ldc = g.ldc;
    t.alpha = g.alpha;
    t.beta = g.beta;
    t.a_tri = g.a_tri;
    t.b_tri = g.b_tri;
    t.c_mode = g.c_mode;
    t.splits = 1;
    t.err = ctx->dflags + 2;
    t.wait_limit = ctx->wait_limit;
    uint32_t d = 0;
    d |= 1u << 4;          // D: F32
    d |= 2u << 7;          // A: TF32
    d |= 2u << 10;         // B: TF32
    // A and B K-major (bits 15/16 clear)
    d |= (uint32_t)(BN >> 3) << 17;
    d |= (uint32_t)(BM >> 4) << 24;
    t.idesc = d;

    // Large products: CTA pairs on 256 x 256 tiles.
    if (g.M >= 512 && g.N >= 512) {
        const int pcap = max_pairs_gemm(ctx);
        if (pcap >= 1) {
            TcGemmArgs p = t;
            p.tiles_m = (int)((g.M + 255) / 256);
            p.tiles_n = (int)((g.N + P_BN - 1) / P_BN);
            p.group = 8;
            uint32_t d2 = 0;
            d2 |= 1u << 4;
            d2 |= 2u << 7;
            d2 |= 2u << 10;
            d2 |= (uint32_t)(P_BN >> 3) << 17;
            d2 |= (uint32_t)(256 >> 4) << 24;
            p.idesc = d2;
            p.splits = g.split_k > 1 ? g.split_k : 1;
            const int64_t units64 = (int64_t)p.tiles_m * p.tiles_n * p.splits;
            if (units64 > (int64_t)INT32_MAX / 2) return LLMC_ERR_UNSUPPORTED;
            const int units = (int)units64;
            // Persistent pairs when the context has the GPU to itself; one pair per unit when it
            // shares the SMs (its CTAs then start wherever SMs free up).
            const int pairs = (ctx->sm_limit > 0 || units < pcap) ? units : pcap;
            // C through TMA when beta is 0 (store) or 1 (reduce-add) and C's layout allows a map.
            int tma_out = 0;
            CUtensorMap mc;
            if ((g.beta == 0.f || g.beta == 1.f) && (reinterpret_cast<uintptr_t>(g.C) % 16) == 0 && g.ldc % 4 == 0) {
                EncodeTiledFn enc = encode_fn();
                const cuuint64_t cdim[2] = {(cuuint64_t)g.N, (cuuint64_t)g.M};
                const cuuint64_t cstride[1] = {(cuuint64_t)g.ldc * 4};
                const cuuint32_t cbox[2] = {32, 32};
                const cuuint32_t est[2] = {1, 1};
                if (enc && enc(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, g.C, cdim, cstride, cbox, est,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
                    tma_out = g.beta == 0.f ? 1 : 2;
            }
            if (!tma_out) mc = mah;  // unused placeholder
            gemm_tc2_kernel<<<(unsigned)(2 * pairs), P_NT, P_SMEM_BYTES, ctx->stream>>>(mah, mal, mbh, mbl, mc, p, tma_out);
            return check_launch(ctx, "gemm_tc2");
        }
    }
    static bool attr = false;
    if (!attr) {
        LLMC_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr = true;
    }
    t.tiles_m = (int)((g.M + BM - 1) / BM);
    t.tiles_n = (int)((g.N + BN - 1) / BN);
    t.group = 12;  // ~sqrt(SM count)
    const int tiles = t.tiles_m * t.tiles_n;
    // Persistent CTAs (one per SM) when the context has the GPU to itself; one CTA per tile when
    // it shares the SMs with another context (llmc_set_sm_limit), so that its CTAs start on any
    // SM the other context's kernels leave free instead of queueing behind them.
    const int grid = (ctx->sm_limit > 0 || tiles < ctx->sm_count) ? tiles : ctx->sm_count;
    gemm_tc_kernel<<<(unsigned)grid, NT, SMEM_BYTES, ctx->stream>>>(mah, mal, mbh, mbl, t);
    return check_launch(ctx, "gemm_tc");
}

}  // namespace llmc
