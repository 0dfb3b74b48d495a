// apply_tc.cuh -- K6: back-projection with the fused NF4 weight write, for a
// whole layer in one persistent launch.
//
// For every matrix p: dW = X Y^T (X: m x r, Y: n x r, bf16, K-major; right
// side X = N, Y = Q; left side X = P, Y = N), then for each 64-element NF4
// block of the weight: w = CODES[code] * absmax; w -= fl(lr * dW); optional
// decoupled decay; requantise bit-exactly; store.
//
// Unit = (matrix, 128-row tile, 256-column tile).  Warps: 0 = TMEM allocation
// + TMA producer, 1 = UMMA issuer, 2..17 = epilogue.  Epilogue warp e reads
// TMEM lane quarter q = warp % 4 and owns the 64-column NF4 block e / 4 of the
// tile: one row of one block per thread per unit, in two passes over 16-column
// chunks -- pass 1 dequantises the old block, applies the update, writes the
// updated values back over the accumulator columns in TMEM and reduces the new
// absmax; pass 2 reloads them and requantises.  The NF4 tile (128 rows x 128
// bytes, 128-byte swizzle) and its absmax tile (128 x 4 floats) are TMA-loaded
// into one of kApplyWSlots weight slots, rewritten in place, and written back
// with one TMA store per 32-row lane quarter as soon as that quarter's four
// warps are done; a slot returns to the producer one unit later.  Operand
// k-blocks (64 columns of r of X and Y) flow through a separate STAGES-deep
// ring.  TMEM holds two 256-column accumulators so the epilogue of one tile
// overlaps the MMAs of the next.
//
// PAIR = true runs the same unit on a cluster of two CTAs (tcgen05
// cta_group::2): the unit is 256 rows x 256 columns, each CTA holds its 128
// rows of X and 128 of the 256 rows of Y per k-block (32 KB instead of 48 KB),
// CTA 0 issues the pair's MMAs (M = 256) and its commits reach both CTAs'
// barriers, and each CTA's epilogue processes its own 128 rows as above.  At
// large ranks the single-CTA kernel is bound by the operand bytes it can keep
// in flight per SM (two 48 KB stages for 384 KB per unit at r = 512); the pair
// moves a third fewer bytes per SM through four stages of nearly the same
// memory (the NF4 byte table needs 16 copies, not 32).
#pragma once
#include "nf4.cuh"
#include "umma.cuh"

namespace aeth {

constexpr int kApplyMaxProblems = 8;
constexpr int kApplyBN = 256;
constexpr int kApplyEpiWarps = 16;
constexpr int kApplyWSlots = 3;
constexpr int kApplyThreads = 64 + 32 * kApplyEpiWarps;

struct ApplyProblem {
    CUtensorMap tmX;   // X, box 64 x 128
    CUtensorMap tmY;   // Y, box 64 x 256
    CUtensorMap tmW;   // packed NF4, box 128 B x 128 rows (load)
    CUtensorMap tmS;   // absmax, box 4 x 128 (load)
    CUtensorMap tmWq;  // packed NF4, box 128 B x 32 rows (per-quarter store)
    CUtensorMap tmSq;  // absmax, box 4 x 32 (per-quarter store)
    float* prequant_out;
    float* delta_out;
    int m, n;
    int n_tiles;
    int unit_begin;
    float lr, decay_mul;
    int has_decay;
    int pad;
};

struct ApplyArgs {
    ApplyProblem p[kApplyMaxProblems];
    int nprob;
    int total_units;
    int kb;  // k-blocks per unit = ceil(r / 64)
    uint32_t idesc;
};

template <int STAGES, bool PAIR = false>
struct ApplyLayout {
    static constexpr int kA = 128 * 64 * 2;                       // 16 KB
    static constexpr int kB = (PAIR ? kApplyBN / 2 : kApplyBN) * 64 * 2;  // 32 KB (16 KB: half of Y per CTA)
    static constexpr int kStage = kA + kB;
    static constexpr int kWPacked = 128 * 128;     // 128 rows x 128 bytes
    static constexpr int kWScale = 128 * 16;       // 128 rows x 4 floats
    static constexpr int kWSlot = (kWPacked + kWScale + 1023) / 1024 * 1024;  // slots stay 1 KB aligned
    static constexpr int kBar = 256;
    static constexpr int kTotal = STAGES * kStage + kApplyWSlots * kWSlot + kBar + (int)sizeof(Nf4Tables32);
};

__device__ __forceinline__ int apply_find(const ApplyArgs& a, int u) {
    int p = 0;
#pragma unroll 1
    while (p + 1 < a.nprob && u >= a.p[p + 1].unit_begin) ++p;
    return p;
}

// 32 lanes x 16 consecutive 32-bit TMEM columns into v[OFF .. OFF+15].
template <int OFF, int N>
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[N]) {
    static_assert(OFF + 16 <= N, "tmem_ld16 destination too small");
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[OFF + i] = __uint_as_float(r[i]);
}

// DECAY: some problem of the launch has a decoupled decay (each problem's
// has_decay still selects it); OUT: some problem writes the fp32 delta or the
// pre-quantisation weights.  Launches with neither (the usual case) carry no
// per-element test or predicated-off store for them.
template <int STAGES, bool PAIR, bool DECAY = false, bool OUT = false>
__global__ void __launch_bounds__(kApplyThreads, 1)
    apply_grouped_kernel(const __grid_constant__ ApplyArgs args, uint32_t* err) {
    using L = ApplyLayout<STAGES, PAIR>;
    constexpr int kEpiThreads = 32 * kApplyEpiWarps;
    extern __shared__ uint8_t smem_raw[];
    // an offset from the shared array (not an integer round trip), so every
    // pointer below stays known to be shared: ld/st.shared, not generic accesses
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * L::kA;
    uint8_t* wslot = base + STAGES * L::kStage;  // kApplyWSlots x (packed tile, scale tile)
    uint64_t* full = reinterpret_cast<uint64_t*>(wslot + kApplyWSlots * L::kWSlot);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* w_full = acc_empty + 2;
    uint64_t* w_empty = w_full + kApplyWSlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_empty + kApplyWSlots);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // (problem, m0, n0) of the unit in each weight slot, written by the producer
    // before the slot's full barrier is armed (its arrive releases them)
    int4* winfo = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(full) + 160);
    static_assert((2 * STAGES + 4 + 2 * kApplyWSlots) * 8 + 8 <= 160 && 160 + 16 * kApplyWSlots <= L::kBar,
                  "barriers, TMEM slot, abort flag and unit table must fit the barrier area");
    Nf4Tables32* tab = reinterpret_cast<Nf4Tables32*>(reinterpret_cast<uint8_t*>(full) + L::kBar);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // PAIR: rank in the cluster (CTA 0 issues the MMAs), units per cluster
    const int crank = PAIR ? (int)cluster_ctarank() : 0;
    const int ustart = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int rows_per_unit = PAIR ? 256 : 128;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        // acc_empty: every epilogue thread (single CTA), or one arrival per
        // epilogue warp of both CTAs on CTA 0's barrier (pair)
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], PAIR ? 2 * kApplyEpiWarps : kEpiThreads);
        }
        for (int b = 0; b < kApplyWSlots; ++b) { mbar_init(&w_full[b], 1); mbar_init(&w_empty[b], 4); }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 2 * kApplyBN);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 2 * kApplyBN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // both CTAs' barriers initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = args.total_units;
    const int kb_n = args.kb;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0, j = 0;
            for (int u = ustart; u < total && !*abort; u += ustep, ++j) {
                const int p = apply_find(args, u);
                const ApplyProblem& pr = args.p[p];
                const int local = u - pr.unit_begin;
                const int m0 = (local / pr.n_tiles) * rows_per_unit + crank * 128;  // this CTA's 128 rows
                const int n0 = (local % pr.n_tiles) * kApplyBN;
                const int wb = j % kApplyWSlots;
                if (!mbar_wait(&w_empty[wb], ((uint32_t)(j / kApplyWSlots) & 1u) ^ 1u, abort, err, DEVERR_TIMEOUT_TMA))
                    break;
                winfo[wb] = make_int4(p, m0, n0, 0);
                mbar_arrive_expect_tx(&w_full[wb], L::kWPacked + L::kWScale);
                uint8_t* ws = wslot + wb * L::kWSlot;
                tma_load_2d_hint(ws, &pr.tmW, &w_full[wb], n0 / 2, m0, l2_evict_first_policy());
                tma_load_2d_hint(ws + L::kWPacked, &pr.tmS, &w_full[wb], n0 / 64, m0, l2_evict_first_policy());
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort, err, DEVERR_TIMEOUT_TMA)) break;
                    if (PAIR) {
                        // CTA 0 expects both CTAs' bytes; each CTA loads its own halves
                        if (crank == 0) mbar_arrive_expect_tx(&full[s], 2 * L::kStage);
                        tma_load_2d_pair(sA + s * L::kA, &pr.tmX, &full[s], kb * 64, m0);
                        tma_load_2d_pair(sB + s * L::kB, &pr.tmY, &full[s], kb * 64, n0 + crank * (kApplyBN / 2));
                    } else {
                        mbar_arrive_expect_tx(&full[s], L::kStage);
                        tma_load_2d(sA + s * L::kA, &pr.tmX, &full[s], kb * 64, m0);
                        tma_load_2d(sB + s * L::kB, &pr.tmY, &full[s], kb * 64, n0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && crank == 0) {
            int it = 0, j = 0;
            for (int u = ustart; u < total && !*abort; u += ustep, ++j) {
                const int b = j & 1;
                if (!mbar_wait(&acc_empty[b], ((uint32_t)(j >> 1) & 1u) ^ 1u, abort, err, DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * kApplyBN);
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(&full[s], ph, abort, err, DEVERR_TIMEOUT_MMA)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * L::kA);
                    const uint32_t b_addr = smem_u32(sB + s * L::kB);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sdesc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b_addr + kk * 32, 16, 1024);
                        if (PAIR) umma_f16_ss_pair(d, ad, bd, args.idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                        else umma_f16_ss(d, ad, bd, args.idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    if (PAIR) umma_commit_pair(&empty[s]);
                    else umma_commit(&empty[s]);
                }
                if (PAIR) umma_commit_pair(&acc_full[b]);
                else umma_commit(&acc_full[b]);
            }
        }
    } else {
        // The epilogue warps fill the code tables while the producer's first
        // loads and MMAs are in flight, and meet at their own barrier.
        nf4_tables32_init(tab, threadIdx.x - 64, kEpiThreads);
        named_bar(5, kEpiThreads);
        const int ew = warp - 2;     // 0..15
        const int q = warp & 3;      // TMEM lane quarter this warp may access = its 32-row group
        const int blk = ew >> 2;     // 64-column NF4 block of the 256-wide tile
        const int cl = blk * 64;     // first column of the block within the tile
        const int row = q * 32 + lane;
        const bool qleader = ew < 4 && lane == 0;  // one thread per row group issues its stores
        const uint32_t tcol0 = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cl;
        const uint32_t rep_base = nf4_byte_rep_base(tab), rep_lane = nf4_byte_rep_lane(lane);
        const uint32_t bucket_bias = nf4_bucket_bias(tab), bucket_lane = tab->bucket32[lane];
        int j = 0;
        int pending = -1;  // slot of this row group's previous store, released one unit later
        for (int u = ustart; u < total; u += ustep, ++j) {
            const int b = j & 1;
            const int wb = j % kApplyWSlots;
            if (!mbar_wait(&w_full[wb], (uint32_t)(j / kApplyWSlots) & 1u, abort, err, DEVERR_TIMEOUT_EPI)) break;
            const int4 info = winfo[wb];
            const ApplyProblem& pr = args.p[info.x];
            const int m0 = info.y, n0 = info.z;
            if (!mbar_wait(&acc_full[b], (uint32_t)(j >> 1) & 1u, abort, err, DEVERR_TIMEOUT_EPI) || *abort) break;
            tc_fence_after();
            uint8_t* wp = wslot + wb * L::kWSlot;
            if (n0 + cl < pr.n) {  // warp-uniform
                const float2 nlr2 = make_float2(-pr.lr, -pr.lr);
                const float2 dmul2 = make_float2(pr.decay_mul, pr.decay_mul);
                const int ck = cl / 32;  // first 16-byte chunk of this block's 32 packed bytes
                uint8_t* rowp = wp + row * 128;
                float* sp = reinterpret_cast<float*>(wp + L::kWPacked) + row * 4 + blk;
                const float amax_old = *sp;
                const uint32_t tcol = tcol0 + (uint32_t)(b * kApplyBN);
                const int64_t grow = (int64_t)(m0 + row);
                float* dout = nullptr;
                float* pout = nullptr;
                if constexpr (OUT) {
                    if (pr.delta_out && grow < pr.m) dout = pr.delta_out + grow * pr.n + n0 + cl;
                    if (pr.prequant_out && grow < pr.m) pout = pr.prequant_out + grow * pr.n + n0 + cl;
                }
                const bool decay = DECAY && pr.has_decay;
                // pass 1: w = CODES * absmax_old - fl(lr * dW) [* decay] -> TMEM; block absmax.
                // The next chunk's TMEM load is in flight while this chunk is updated.
                float amax = 0.0f;
                float vb[2][16];
                tmem_ld16<0>(tcol, vb[0]);
                // the block's 32 packed bytes as two 16-byte chunks (whole-chunk accesses:
                // the swizzle spreads 8 consecutive rows over all 32 banks)
                const uint4 q01 = *reinterpret_cast<const uint4*>(rowp + ((ck ^ (row & 7)) * 16));
                const uint4 q23 = *reinterpret_cast<const uint4*>(rowp + (((ck + 1) ^ (row & 7)) * 16));
                tmem_wait_ld_bind(vb[0]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c < 3) tmem_ld16<0>(tcol + (uint32_t)((c + 1) * 16), vb[(c + 1) & 1]);
                    float* v = vb[c & 1];
                    float w[16];
                    // words 2c, 2c+1 of the block
                    const uint4 qa = c < 2 ? q01 : q23;
                    nf4_dequant_word_s<true>((c & 1) ? qa.z : qa.x, amax_old, rep_base, rep_lane, w);
                    nf4_dequant_word_s<true>((c & 1) ? qa.w : qa.y, amax_old, rep_base, rep_lane, w + 8);
                    // w <- fl(w - lr * dW), one fused multiply-add per element (paired),
                    // then the decoupled decay.  The reference rounds lr * dW first; the
                    // two differ by under half an ulp of the product, inside the update's
                    // tolerance, and the requantisation below is exact for whatever w is.
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        float2 ww = fma2_rn(make_float2(v[i], v[i + 1]), nlr2, make_float2(w[i], w[i + 1]));
                        if (DECAY && decay) ww = mul2_rn(ww, dmul2);
                        w[i] = ww.x;
                        w[i + 1] = ww.y;
                        amax = fmax3_nan(amax, fabsf(ww.x), fabsf(ww.y));  // NaN-propagating, as torch's max
                    }
                    tmem_st16(tcol + (uint32_t)(c * 16), w);
                    if (OUT && dout) {  // take_weight_delta: fl(lr * dW)
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *reinterpret_cast<float4*>(dout + c * 16 + i) =
                                make_float4(__fmul_rn(v[i], pr.lr), __fmul_rn(v[i + 1], pr.lr),
                                            __fmul_rn(v[i + 2], pr.lr), __fmul_rn(v[i + 3], pr.lr));
                    }
                    if (OUT && pout) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *reinterpret_cast<float4*>(pout + c * 16 + i) = make_float4(w[i], w[i + 1], w[i + 2], w[i + 3]);
                    }
                    if (c < 3) tmem_wait_ld_bind(vb[(c + 1) & 1]);
                }
                tmem_wait_st();
                // pass 2: requantise from TMEM (fast classifier; exact fix-up next to
                // boundaries), again with the next chunk's load in flight.  A block
                // holding NaN or inf (amax NaN or inf) skips the fast classifier,
                // whose table index needs a finite xn, and is requantised exactly.
                const bool bad = !(amax <= 3.402823466e38f);
                const float inv = __frcp_rn(nf4_safe(amax));
                float mw[8];  // per packed word: the smallest distance to a threshold (0: exact path)
                uint32_t pw[8];
                float wbuf[2][16];
                tmem_ld16<0>(tcol, wbuf[0]);
                tmem_wait_ld_bind(wbuf[0]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c < 3) tmem_ld16<0>(tcol + (uint32_t)((c + 1) * 16), wbuf[(c + 1) & 1]);
                    // all lanes classify (the entries come by shuffle); a non-finite
                    // block's words are rewritten on the exact path below
                    mw[2 * c] = mw[2 * c + 1] = 1.0f;
                    pw[2 * c] = nf4_fast_word8_s(wbuf[c & 1], inv, bucket_lane, mw[2 * c]);
                    pw[2 * c + 1] = nf4_fast_word8_s(wbuf[c & 1] + 8, inv, bucket_lane, mw[2 * c + 1]);
                    if (bad) mw[2 * c] = mw[2 * c + 1] = 0.0f;
                    if (c & 1)  // a whole 16-byte chunk: words 2c-2 .. 2c+1
                        *reinterpret_cast<uint4*>(rowp + (((ck + (c >> 1)) ^ (row & 7)) * 16)) =
                            make_uint4(pw[2 * c - 2], pw[2 * c - 1], pw[2 * c], pw[2 * c + 1]);
                    if (c < 3) tmem_wait_ld_bind(wbuf[(c + 1) & 1]);
                }
                const float mind = fmin3(fmin3(mw[0], mw[1], mw[2]), fmin3(mw[3], mw[4], mw[5]), fminf(mw[6], mw[7]));
                if (__any_sync(0xffffffffu, mind < kNf4NearWindow32)) {
                    // Rare: the chunks holding a near-boundary element are loaded
                    // again and their flagged words get those elements decided
                    // exactly; a non-finite block is requantised exactly
                    // throughout (a NaN scale gives code 0, as the reference's
                    // argmin does).  Warp-uniform per chunk (TMEM loads are
                    // warp-collective).
                    const float safe_x = nf4_safe(amax);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const bool n0w = mw[2 * c] < kNf4NearWindow32, n1w = mw[2 * c + 1] < kNf4NearWindow32;
                        if (!__any_sync(0xffffffffu, n0w || n1w)) continue;
                        float w[16];
                        tmem_ld16<0>(tcol + (uint32_t)(c * 16), w);
                        tmem_wait_ld();
                        uint32_t* wa = reinterpret_cast<uint32_t*>(rowp + (((ck + (c >> 1)) ^ (row & 7)) * 16) + (c & 1) * 8);
                        if (bad) {
                            wa[0] = nf4_exact_word8(w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], safe_x);
                            wa[1] = nf4_exact_word8(w[8], w[9], w[10], w[11], w[12], w[13], w[14], w[15], safe_x);
                        } else {
                            if (n0w)
                                wa[0] = nf4_fix_word8(wa[0], w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], inv, safe_x,
                                                      bucket_bias);
                            if (n1w)
                                wa[1] = nf4_fix_word8(wa[1], w[8], w[9], w[10], w[11], w[12], w[13], w[14], w[15], inv,
                                                      safe_x, bucket_bias);
                        }
                    }
                }
                *sp = nf4_store_amax(amax);
            }
            tc_fence_before();
            if (PAIR) {
                // one arrival per warp, on CTA 0's barrier (the pair's MMA issuer)
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(smem_leader(&acc_empty[b]));
            } else {
                mbar_arrive(&acc_empty[b]);
            }
            fence_proxy_async();
            named_bar(1 + q, 128);  // the four warps of this row group
            if (qleader) {
                tma_store_2d_hint(&pr.tmWq, wp + q * 32 * 128, n0 / 2, m0 + q * 32, l2_evict_first_policy());
                tma_store_2d_hint(&pr.tmSq, wp + L::kWPacked + q * 32 * 16, n0 / 64, m0 + q * 32, l2_evict_first_policy());
                bulk_commit();
                if (pending >= 0) {
                    bulk_wait_read<1>();  // this group's previous stores have read their slot
                    mbar_arrive(&w_empty[pending]);
                }
                pending = wb;
            }
        }
        if (qleader) {
            bulk_wait<0>();
            if (pending >= 0) mbar_arrive(&w_empty[pending]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // the pair's MMAs and both epilogues are done with TMEM
    if (warp == 0) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem, 2 * kApplyBN);
        else tmem_dealloc(tmem, 2 * kApplyBN);
    }
}

}  // namespace aeth
