// proj_tc.cuh -- K4: the GaLore projection of a whole layer's gradients in one
// persistent launch.
//
// For every matrix p of the group, R_p (l x r, fp32) += contraction of its
// bf16 gradient G_p (m x n) with its projector over the smaller dimension:
//   right (m >= n): R = G Q        A = G     (K-major, box 64 x 128)
//   left  (m <  n): R^T = G^T P    A = G^T   (MN-major, two 64 x 64 boxes)
//   B = projector^T (r x s, K-major, box 64 x BN) in both cases.
// Work units are (matrix, 128-row tile of R, K split); one CTA per SM walks
// units round-robin.  Split-K partials are added into R with TMA bulk
// reduce-add (cp.reduce.async.bulk.tensor ... .add), so R accumulates across
// splits and across calls (project_and_accumulate semantics) without a
// separate reduction pass.
//
// Warps: 0 = TMEM allocation + TMA producer, 1 = UMMA issuer, 2..5 =
// epilogue.  TMEM holds two BN-column accumulators so the epilogue of unit j
// overlaps the MMAs of unit j+1.  The epilogue stages 32-column fp32 chunks in
// 128-byte-swizzled shared memory (conflict-free STS.128) for the reduce.
#pragma once
#include "umma.cuh"

namespace aeth {

constexpr int kProjMaxProblems = 8;

struct ProjProblem {
    CUtensorMap tmA;
    CUtensorMap tmB;
    CUtensorMap tmC;
    int a_mn;
    int kb_total;
    int kb_per_unit;
    int splits;
    int unit_begin;
    int pad[3];
};

struct ProjArgs {
    ProjProblem p[kProjMaxProblems];
    int nprob;
    int total_units;
    int r;
    uint32_t idesc_k;
    uint32_t idesc_mn;
};

template <int BN, int STAGES>
struct ProjLayout {
    static constexpr int kA = 128 * 64 * 2;          // 16 KB
    static constexpr int kB = BN * 64 * 2;
    static constexpr int kStage = kA + kB;
    static constexpr int kStaging = 2 * 128 * 128;  // two 128 x 32 fp32 chunks
    static constexpr int kBar = 256;
    static constexpr int kTotal = STAGES * kStage + kStaging + kBar;
};

__device__ __forceinline__ int proj_find(const ProjArgs& a, int u) {
    int p = 0;
#pragma unroll 1
    while (p + 1 < a.nprob && u >= a.p[p + 1].unit_begin) ++p;
    return p;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1) proj_grouped_kernel(const __grid_constant__ ProjArgs args, uint32_t* err) {
    using L = ProjLayout<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * L::kA;
    uint8_t* staging = base + STAGES * L::kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + L::kStaging);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 128); }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, 2 * BN); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = args.total_units;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int u = blockIdx.x; u < total && !*abort; u += gridDim.x) {
                const int p = proj_find(args, u);
                const ProjProblem& pr = args.p[p];
                const int local = u - pr.unit_begin;
                const int m0 = (local / pr.splits) * 128;
                const int kb0 = (local % pr.splits) * pr.kb_per_unit;
                const int kb1 = min(kb0 + pr.kb_per_unit, pr.kb_total);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort, err, DEVERR_TIMEOUT_TMA)) break;
                    mbar_arrive_expect_tx(&full[s], L::kStage);
                    uint8_t* a = sA + s * L::kA;
                    if (pr.a_mn) {
                        tma_load_2d_hint(a, &pr.tmA, &full[s], m0, kb * 64, l2_evict_first_policy());
                        tma_load_2d_hint(a + 8192, &pr.tmA, &full[s], m0 + 64, kb * 64, l2_evict_first_policy());
                    } else {
                        tma_load_2d_hint(a, &pr.tmA, &full[s], kb * 64, m0, l2_evict_first_policy());
                    }
                    tma_load_2d(sB + s * L::kB, &pr.tmB, &full[s], kb * 64, 0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int it = 0, j = 0;
            for (int u = blockIdx.x; u < total && !*abort; u += gridDim.x, ++j) {
                const int p = proj_find(args, u);
                const ProjProblem& pr = args.p[p];
                const int local = u - pr.unit_begin;
                const int kb0 = (local % pr.splits) * pr.kb_per_unit;
                const int kb1 = min(kb0 + pr.kb_per_unit, pr.kb_total);
                const int b = j & 1;
                if (!mbar_wait(&acc_empty[b], ((uint32_t)(j >> 1) & 1u) ^ 1u, abort, err, DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * BN);
                const uint32_t idesc = pr.a_mn ? args.idesc_mn : args.idesc_k;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&full[s], ph, abort, err, DEVERR_TIMEOUT_MMA)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * L::kA);
                    const uint32_t b_addr = smem_u32(sB + s * L::kB);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = pr.a_mn ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                                    : sdesc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b_addr + kk * 32, 16, 1024);
                        umma_f16_ss(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                umma_commit(&acc_full[b]);
            }
        }
    } else {
        // epilogue: 128 threads, thread = row of the 128-row tile
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const bool leader = threadIdx.x == 64;
        const int nchunks = (args.r + 31) / 32;
        int j = 0, cc = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x, ++j) {
            const int p = proj_find(args, u);
            const ProjProblem& pr = args.p[p];
            const int local = u - pr.unit_begin;
            const int m0 = (local / pr.splits) * 128;
            const int b = j & 1;
            if (!mbar_wait(&acc_full[b], (uint32_t)(j >> 1) & 1u, abort, err, DEVERR_TIMEOUT_EPI) || *abort) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c, ++cc) {
                float v[32];
                tmem_ld32<0>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + c * 32), v);
                tmem_wait_ld();
                uint8_t* stg = staging + (cc & 1) * (128 * 128);
                if (leader) bulk_wait_read<1>();  // the reduce that last read this buffer is done
                named_bar(1, 128);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float4 f = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                    *reinterpret_cast<float4*>(stg + row * 128 + ((k ^ (row & 7)) * 16)) = f;
                }
                fence_proxy_async();
                named_bar(1, 128);
                if (leader) {
                    tma_reduce_add_2d(&pr.tmC, stg, c * 32, m0);
                    bulk_commit();
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
        if (leader) bulk_wait<0>();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// ---------------------------------------------------------------------------
// The same projection on CTA pairs (cluster of two, tcgen05 cta_group::2),
// all of R's columns in one pass over the gradient.  Unit = (matrix, 256-row
// tile of R, k-split); each CTA of the pair holds its 128 rows of A and half
// of each 256-column block of projT per k-block, CTA 0 issues the pair's MMAs
// (M = 256; rank RT as RT / 256 MMAs of N = 256, or one of N = RT), and each
// CTA's epilogue reduce-adds its 128 rows of R.  Rank 512 (C4) reads the
// gradient once instead of once per 256-column slice; TMEM holds two
// accumulators when 2 RT <= 512, else one (a unit's k-loop is long against
// its epilogue there).
// ---------------------------------------------------------------------------
template <int RT, int STAGES>
struct ProjPairLayout {
    static constexpr int kNmma = RT < 256 ? RT : 256;   // N of one MMA
    static constexpr int kChunks = RT / kNmma;          // MMAs per k-step (1 or 2)
    static constexpr int kA = 128 * 64 * 2;             // 16 KB: this CTA's 128 rows
    static constexpr int kBc = (kNmma / 2) * 64 * 2;    // this CTA's half of one N block
    static constexpr int kB = kChunks * kBc;
    static constexpr int kStage = kA + kB;
    static constexpr int kStaging = 2 * 128 * 128;      // two 128 x 32 fp32 chunks
    static constexpr int kBar = 256;
    static constexpr int kTotal = STAGES * kStage + kStaging + kBar;
    static constexpr int kAccBufs = 2 * RT <= 512 ? 2 : 1;
    static constexpr int kTmemCols = RT * kAccBufs <= 64 ? 64 : RT * kAccBufs <= 128 ? 128 : RT * kAccBufs <= 256 ? 256 : 512;
};

template <int RT, int STAGES>
__global__ void __launch_bounds__(192, 1) proj_pair_kernel(const __grid_constant__ ProjArgs args, uint32_t* err) {
    using L = ProjPairLayout<RT, STAGES>;
    constexpr int NB = L::kAccBufs;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * L::kA;
    uint8_t* staging = base + STAGES * L::kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + L::kStaging);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    static_assert((2 * STAGES + 4) * 8 + 8 <= L::kBar, "barriers must fit the barrier area");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int crank = (int)cluster_ctarank();
    const int ustart = (int)(blockIdx.x >> 1), ustep = (int)(gridDim.x >> 1);
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        // acc_empty (CTA 0): one arrival per epilogue warp of both CTAs
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 8); }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) { tmem_alloc_pair(tmem_slot, L::kTmemCols); tmem_relinquish_pair(); }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = args.total_units;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int u = ustart; u < total && !*abort; u += ustep) {
                const int p = proj_find(args, u);
                const ProjProblem& pr = args.p[p];
                const int local = u - pr.unit_begin;
                const int m0 = (local / pr.splits) * 256 + crank * 128;  // this CTA's 128 rows of R
                const int kb0 = (local % pr.splits) * pr.kb_per_unit;
                const int kb1 = min(kb0 + pr.kb_per_unit, pr.kb_total);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort, err, DEVERR_TIMEOUT_TMA)) break;
                    if (crank == 0) mbar_arrive_expect_tx(&full[s], 2 * L::kStage);
                    uint8_t* a = sA + s * L::kA;
                    if (pr.a_mn) {
                        tma_load_2d_pair(a, &pr.tmA, &full[s], m0, kb * 64);
                        tma_load_2d_pair(a + 8192, &pr.tmA, &full[s], m0 + 64, kb * 64);
                    } else {
                        tma_load_2d_pair(a, &pr.tmA, &full[s], kb * 64, m0);
                    }
#pragma unroll
                    for (int c = 0; c < L::kChunks; ++c)
                        tma_load_2d_pair(sB + s * L::kB + c * L::kBc, &pr.tmB, &full[s], kb * 64,
                                         c * L::kNmma + crank * (L::kNmma / 2));
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && crank == 0) {
            int it = 0, j = 0;
            for (int u = ustart; u < total && !*abort; u += ustep, ++j) {
                const int p = proj_find(args, u);
                const ProjProblem& pr = args.p[p];
                const int local = u - pr.unit_begin;
                const int kb0 = (local % pr.splits) * pr.kb_per_unit;
                const int kb1 = min(kb0 + pr.kb_per_unit, pr.kb_total);
                const int b = NB == 2 ? (j & 1) : 0;
                const uint32_t use = NB == 2 ? (uint32_t)(j >> 1) : (uint32_t)j;
                if (!mbar_wait(&acc_empty[b], (use & 1u) ^ 1u, abort, err, DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * RT);
                const uint32_t idesc = pr.a_mn ? args.idesc_mn : args.idesc_k;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&full[s], ph, abort, err, DEVERR_TIMEOUT_MMA)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * L::kA);
                    const uint32_t b_addr = smem_u32(sB + s * L::kB);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = pr.a_mn ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                                    : sdesc_sw128(a_addr + kk * 32, 16, 1024);
#pragma unroll
                        for (int c = 0; c < L::kChunks; ++c) {
                            const uint64_t bd = sdesc_sw128(b_addr + c * L::kBc + kk * 32, 16, 1024);
                            umma_f16_ss_pair(d + (uint32_t)(c * L::kNmma), ad, bd, idesc,
                                             (kb > kb0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit_pair(&empty[s]);
                }
                umma_commit_pair(&acc_full[b]);
            }
        }
    } else {
        // epilogue: 128 threads, thread = row of this CTA's 128-row half
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const bool leader = threadIdx.x == 64;
        constexpr int nchunks = RT / 32;
        int j = 0, cc = 0;
        for (int u = ustart; u < total; u += ustep, ++j) {
            const int p = proj_find(args, u);
            const ProjProblem& pr = args.p[p];
            const int local = u - pr.unit_begin;
            const int m0 = (local / pr.splits) * 256 + crank * 128;
            const int b = NB == 2 ? (j & 1) : 0;
            const uint32_t use = NB == 2 ? (uint32_t)(j >> 1) : (uint32_t)j;
            if (!mbar_wait(&acc_full[b], use & 1u, abort, err, DEVERR_TIMEOUT_EPI) || *abort) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c, ++cc) {
                float v[32];
                tmem_ld32<0>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * RT + c * 32), v);
                tmem_wait_ld();
                uint8_t* stg = staging + (cc & 1) * (128 * 128);
                if (leader) bulk_wait_read<1>();  // the reduce that last read this buffer is done
                named_bar(1, 128);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float4 f = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                    *reinterpret_cast<float4*>(stg + row * 128 + ((k ^ (row & 7)) * 16)) = f;
                }
                fence_proxy_async();
                named_bar(1, 128);
                if (leader) {
                    tma_reduce_add_2d(&pr.tmC, stg, c * 32, m0);
                    bulk_commit();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(smem_leader(&acc_empty[b]));
        }
        if (leader) bulk_wait<0>();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, L::kTmemCols);
    }
}

}  // namespace aeth
