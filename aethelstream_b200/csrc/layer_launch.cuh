// layer_launch.cuh -- host launchers for the grouped (whole-layer) kernels:
// projection (K4), squared norms, back-projection + NF4 write (K6).
#pragma once
#include <vector>

#include "adam.cuh"
#include "apply_tc.cuh"
#include "gemm_tc.cuh"
#include "proj_tc.cuh"

namespace aeth {

// ---------------------------------------------------------------------------
// K4
// ---------------------------------------------------------------------------
// Whether the projection uses CTA pairs where the rank allows (on by
// default; AETH_PROJ_PAIR=0 selects the single-CTA kernel, for comparison).
inline bool proj_use_pair() {
    static const bool on = [] {
        const char* e = getenv("AETH_PROJ_PAIR");
        return !(e && e[0] == '0');
    }();
    return on;
}

struct ProjJob {
    const void* grad;       // bf16 m x n (ksplit > 1: the stacked terms of grad_split_kernel)
    const uint16_t* projT;  // bf16 r x s (s = min(m, n)); ksplit > 1: r x projk_ld*s, the projector repeated
    float* racc;            // fp32 l x r
    int m, n;
    int ldr = 0;            // row stride of racc in floats (0: r); a column slice of a wider R
    int ksplit = 1;         // bf16 terms stacked along the contraction (1, or 2 / 3 for f16 / fp32 gradients)
    int projk_ld = 1;       // copies of the projector in each row of projT (>= ksplit)
};

template <int BN>
int proj_grouped_launch_bn(const ProjJob* jobs, int nj, int r, cudaStream_t st) {
    // As many 32-48 KB operand stages as shared memory holds: more bytes in flight per SM.
    constexpr int STAGES = BN <= 128 ? 6 : 4;
    using L = ProjLayout<BN, STAGES>;
    static_assert(1024 + L::kTotal <= 227 * 1024, "projection kernel shared memory above the per-CTA limit");
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    ProjArgs a;
    memset(&a, 0, sizeof(a));
    a.nprob = nj;
    a.r = r;
    a.idesc_k = idesc_f16(128, BN, true, false, false);
    a.idesc_mn = idesc_f16(128, BN, true, true, false);
    // Split-K depth: the persistent CTAs take units round-robin, so the launch
    // lasts about ceil(units / SMs) units of (k-blocks + epilogue) each.  Pick
    // the k-blocks per unit (at least 8) that minimises that, counting an
    // epilogue as 2 k-blocks of work.
    int kb_target = 8;
    {
        int64_t best = -1;
        for (int kt = 8; kt <= 64; ++kt) {
            int64_t units_k = 0, per_unit = 0;
            for (int i = 0; i < nj; ++i) {
                const int l = std::max(jobs[i].m, jobs[i].n), s = std::min(jobs[i].m, jobs[i].n) * jobs[i].ksplit;
                const int kbt = (s + 63) / 64;
                int sp = (kbt + kt - 1) / kt;
                const int kpu = (kbt + sp - 1) / sp;
                sp = (kbt + kpu - 1) / kpu;
                units_k += (int64_t)((l + 127) / 128) * sp;
                per_unit = std::max<int64_t>(per_unit, kpu);
            }
            const int64_t span = (units_k + num_sms() - 1) / num_sms() * (per_unit + 2);
            if (best < 0 || span < best) { best = span; kb_target = kt; }
        }
    }
    int units = 0;
    for (int i = 0; i < nj; ++i) {
        const ProjJob& j = jobs[i];
        ProjProblem& p = a.p[i];
        const bool right = j.m >= j.n;
        // contraction length s: the smaller dimension times the stacked terms
        const int l = right ? j.m : j.n, s = (right ? j.n : j.m) * j.ksplit;
        const int s1 = right ? j.n : j.m;
        if (right)
            AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)s, (uint64_t)j.m, s, 64, 128, true));
        else
            AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)j.n, (uint64_t)s, j.n, 64, 64, true));
        AETH_TRY(make_tmap_16b(&p.tmB, j.projT, (uint64_t)s, (uint64_t)r, (int64_t)s1 * j.projk_ld, 64, BN, true));
        AETH_TRY(make_tmap_2d(&p.tmC, j.racc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)r, (uint64_t)l,
                              j.ldr > 0 ? j.ldr : r, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B));
        p.a_mn = right ? 0 : 1;
        p.kb_total = (s + 63) / 64;
        p.splits = (p.kb_total + kb_target - 1) / kb_target;
        p.kb_per_unit = (p.kb_total + p.splits - 1) / p.splits;
        p.splits = (p.kb_total + p.kb_per_unit - 1) / p.kb_per_unit;
        p.unit_begin = units;
        units += ((l + 127) / 128) * p.splits;
    }
    a.total_units = units;
    const int smem = 1024 + L::kTotal;
    auto kern = proj_grouped_kernel<BN, STAGES>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (!attr_set[dev]) {
        AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[dev] = true;
    }
    const int grid = std::min(num_sms(), units);
    kern<<<grid, 192, smem, st>>>(a, rt->err_word);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// The CTA-pair projection (proj_pair_kernel) for rank RT: all of R's columns
// in one pass over each gradient.
template <int RT, int STAGES>
int proj_pair_launch(const ProjJob* jobs, int nj, cudaStream_t st) {
    using L = ProjPairLayout<RT, STAGES>;
    static_assert(1024 + L::kTotal <= 227 * 1024, "paired projection shared memory above the per-CTA limit");
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    const int clusters = num_sms() / 2;
    for (int off = 0; off < nj; off += kProjMaxProblems) {
        const int cnt = std::min(kProjMaxProblems, nj - off);
        const ProjJob* js = jobs + off;
        ProjArgs a;
        memset(&a, 0, sizeof(a));
        a.nprob = cnt;
        a.r = RT;
        a.idesc_k = idesc_f16(256, L::kNmma, true, false, false);
        a.idesc_mn = idesc_f16(256, L::kNmma, true, true, false);
        // split-K depth minimising the round-robin makespan over the clusters
        // (an epilogue counted as RT / 64 k-blocks of work)
        int kb_target = 8;
        {
            int64_t best = -1;
            for (int kt = 8; kt <= 256; kt += (kt < 64 ? 1 : 8)) {
                int64_t units_k = 0, per_unit = 0;
                for (int i = 0; i < cnt; ++i) {
                    const int l = std::max(js[i].m, js[i].n), s = std::min(js[i].m, js[i].n) * js[i].ksplit;
                    const int kbt = (s + 63) / 64;
                    int sp = (kbt + kt - 1) / kt;
                    const int kpu = (kbt + sp - 1) / sp;
                    sp = (kbt + kpu - 1) / kpu;
                    units_k += (int64_t)((l + 255) / 256) * sp;
                    per_unit = std::max<int64_t>(per_unit, kpu);
                }
                const int64_t span = (units_k + clusters - 1) / clusters * (per_unit + RT / 64);
                if (best < 0 || span < best) { best = span; kb_target = kt; }
            }
        }
        int units = 0;
        for (int i = 0; i < cnt; ++i) {
            const ProjJob& j = js[i];
            ProjProblem& p = a.p[i];
            const bool right = j.m >= j.n;
            const int l = right ? j.m : j.n, s = (right ? j.n : j.m) * j.ksplit;
            const int s1 = right ? j.n : j.m;
            if (right) AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)s, (uint64_t)j.m, s, 64, 128, true));
            else AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)j.n, (uint64_t)s, j.n, 64, 64, true));
            AETH_TRY(make_tmap_16b(&p.tmB, j.projT, (uint64_t)s, (uint64_t)RT, (int64_t)s1 * j.projk_ld, 64,
                                   L::kNmma / 2, true));
            AETH_TRY(make_tmap_2d(&p.tmC, j.racc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)RT, (uint64_t)l,
                                  j.ldr > 0 ? j.ldr : RT, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B));
            p.a_mn = right ? 0 : 1;
            p.kb_total = (s + 63) / 64;
            p.splits = (p.kb_total + kb_target - 1) / kb_target;
            p.kb_per_unit = (p.kb_total + p.splits - 1) / p.splits;
            p.splits = (p.kb_total + p.kb_per_unit - 1) / p.kb_per_unit;
            p.unit_begin = units;
            units += ((l + 255) / 256) * p.splits;
        }
        a.total_units = units;
        const int smem = 1024 + L::kTotal;
        auto kern = proj_pair_kernel<RT, STAGES>;
        static bool attr_set[kMaxDevices] = {};
        int dev = 0;
        AETH_TRY(current_device(&dev));
        if (!attr_set[dev]) {
            AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            attr_set[dev] = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * std::min(clusters, units));
        cfg.blockDim = dim3(192);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        AETH_CUDA(cudaLaunchKernelEx(&cfg, kern, a, rt->err_word));
    }
    return AETH_OK;
}

// Projects and accumulates every job; jobs must share the rank r.  Ranks 64,
// 128, 256 and 512 run on CTA pairs in one pass over each gradient
// (proj_pair_kernel).  Other ranks run on single CTAs; above 256 (one MMA's
// N) as column slices of at most 256 of R, each a launch over its rows of
// projT (R[:, c0:c1] += G Q[:, c0:c1]), reading the gradient once per slice.
inline int proj_grouped_launch(const ProjJob* jobs, int nj, int r, cudaStream_t st) {
    if (r <= 0 || r > 1024 || r % 8 != 0) return AETH_ERR_UNSUPPORTED;
    bool plain = true;  // the pair kernel writes R with its own row stride r
    for (int i = 0; i < nj; ++i) plain = plain && (jobs[i].ldr == 0 || jobs[i].ldr == r);
    if (plain && proj_use_pair()) {
        if (r == 512) return proj_pair_launch<512, 4>(jobs, nj, st);
        if (r == 256) return proj_pair_launch<256, 6>(jobs, nj, st);
        if (r == 128) return proj_pair_launch<128, 8>(jobs, nj, st);
        if (r == 64) return proj_pair_launch<64, 8>(jobs, nj, st);
    }
    if (r > 256) {
        if (r % 64 != 0) return AETH_ERR_UNSUPPORTED;
        for (int c0 = 0; c0 < r; c0 += 256) {
            const int w = std::min(256, r - c0);
            std::vector<ProjJob> slice(jobs, jobs + nj);
            for (ProjJob& j : slice) {
                const int s = std::min(j.m, j.n) * j.projk_ld;  // row stride of projT
                j.projT += (size_t)c0 * s;
                j.racc += c0;
                j.ldr = r;
            }
            AETH_TRY(proj_grouped_launch(slice.data(), nj, w, st));
        }
        return AETH_OK;
    }
    for (int off = 0; off < nj; off += kProjMaxProblems) {
        const int cnt = std::min(kProjMaxProblems, nj - off);
        if (r <= 64) AETH_TRY(proj_grouped_launch_bn<64>(jobs + off, cnt, r, st));
        else if (r <= 128) AETH_TRY(proj_grouped_launch_bn<128>(jobs + off, cnt, r, st));
        else AETH_TRY(proj_grouped_launch_bn<256>(jobs + off, cnt, r, st));
    }
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// Squared norms of several accumulators in one launch, deterministic: the
// accumulators are cut into chunks of chunk_elems elements (a chunk never
// spans two accumulators), one CTA per chunk, about four per SM; each CTA
// writes the f64 partial sum of its chunk into a fixed slot; the CTA that
// takes the last ticket sums each accumulator's slots in chunk order into
// out[p] and, when asked, also computes the global clip coefficient of
// clip_coeff_kernel (hook.rs:184-187) from out[0..np), then resets the ticket
// for the next launch.  One launch takes up to kSqGroupMax accumulators (a
// whole model's parameters on one GPU: 560 for the 80-layer 70B sweep); the
// per-accumulator tables travel in the kernel parameters, sized by the
// template capacity so a single layer's launch stays small.
// ---------------------------------------------------------------------------
constexpr int kSqGroupSmall = 16;     // capacity of the launch of one layer's step
constexpr int kSqGroupMax = 1024;     // capacity of a whole-model launch (20 KB of kernel parameters)
constexpr int kSqPartialSlots = 4096; // chunk partials per launch
constexpr int kClipGroupMax = 16;     // GPUs in a clip group

struct PeerSlot {
    double sum;
    uint64_t epoch;
};

// A group of GPUs that share one global clip through peer memory.
struct ClipGroup {
    int rank = 0, world = 1;
    PeerSlot* slots[kClipGroupMax] = {};
    uint64_t* epoch = nullptr;  // device counter of exchanges, advanced by the kernel (graph-replay safe)
    uint64_t timeout_ns = kWaitLimitNs;
};

// Scalars and pointers shared by every capacity.
struct SqGroupCommon {
    int64_t chunk_elems;   // a multiple of 1024
    int np;
    float max_norm;
    float* clip_out;       // null: norms only
    double* gnorm_out;     // optional, with clip_out
    double* out;           // np sums
    double* partials;      // kSqPartialSlots
    unsigned int* ticket;  // zero between launches
    // Exchange of the local sum with the other GPUs of a clip group (world > 1):
    // slots[p] is rank p's slot buffer (peer memory for p != rank), laid out as
    // [parity][world] entries of {double sum, uint64 epoch}.
    PeerSlot* slots[kClipGroupMax];
    int rank, world;
    uint64_t* epoch;  // advanced by one per launch by the last CTA
    uint64_t timeout_ns;
    uint32_t* err;
};

template <int CAP>
struct SqGroupArgs {
    const float* x[CAP];
    int64_t n[CAP];
    int chunk_begin[CAP + 1];  // first chunk of each accumulator; chunk_begin[np] = chunks
    SqGroupCommon c;
};

// Peer exchange primitives: a release store of the epoch after the value, an
// acquire load on the reader's side, both at system scope (NVLink peers).
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Writes this rank's sum into every group member's slot for this epoch, waits
// (bounded) for every member's sum, and returns the total in rank order, so
// every rank gets the same bits.  On timeout: flags the error and returns NaN.
__device__ inline double clip_group_total(const SqGroupCommon& a, double local) {
    const uint64_t epoch = *a.epoch + 1;
    *a.epoch = epoch;
    const int par = (int)(epoch & 1u);
    for (int p = 0; p < a.world; ++p) {
        PeerSlot* s = a.slots[p] + par * a.world + a.rank;
        s->sum = local;
        st_release_sys_u64(&s->epoch, epoch);
    }
    double total = 0.0;
    const uint64_t t0 = global_ns();
    for (int p = 0; p < a.world; ++p) {
        PeerSlot* s = a.slots[a.rank] + par * a.world + p;
        while (ld_acquire_sys_u64(&s->epoch) != epoch) {
            if (global_ns() - t0 > a.timeout_ns) {
                report_dev_error(a.err, DEVERR_TIMEOUT_PEER);
                return __longlong_as_double(0x7ff8000000000000ll);
            }
        }
        total += *reinterpret_cast<volatile double*>(&s->sum);
    }
    return total;
}

template <int CAP>
__global__ void __launch_bounds__(256) sqnorm_group_kernel(const __grid_constant__ SqGroupArgs<CAP> a) {
    __shared__ double red[8];
    __shared__ double sums[CAP];
    __shared__ unsigned int taken;
    const SqGroupCommon& cm = a.c;
    const int chunk = blockIdx.x;
    // the accumulator of this chunk: the last p with chunk_begin[p] <= chunk
    int lo = 0, hi = cm.np - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.chunk_begin[mid] <= chunk) lo = mid;
        else hi = mid - 1;
    }
    const int p = lo;
    const int64_t c0 = (int64_t)(chunk - a.chunk_begin[p]) * cm.chunk_elems;
    const int64_t c1 = c0 + cm.chunk_elems < a.n[p] ? c0 + cm.chunk_elems : a.n[p];
    const float4* x4 = reinterpret_cast<const float4*>(a.x[p] + c0);  // c0 % 4 == 0: still 16-byte aligned
    const int n4 = (int)((c1 - c0) / 4);
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    int i = threadIdx.x;
    for (; i + 3 * 256 < n4; i += 4 * 256) {  // four independent 16-byte loads in flight
        float4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = __ldcg(x4 + i + k * 256);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            s[k] += (double)u[k].x * u[k].x + (double)u[k].y * u[k].y + (double)u[k].z * u[k].z +
                    (double)u[k].w * u[k].w;
    }
    for (; i < n4; i += 256) {
        const float4 u = __ldcg(x4 + i);
        s[0] += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
    }
    for (int64_t k = c0 + 4 * (int64_t)n4 + threadIdx.x; k < c1; k += 256) {
        const double v = (double)a.x[p][k];
        s[0] += v * v;
    }
    const double sum = warp_sum_d((s[0] + s[1]) + (s[2] + s[3]));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; ++w) t += red[w];
        cm.partials[chunk] = t;
        __threadfence();
        taken = atomicAdd(cm.ticket, 1u);
    }
    __syncthreads();
    if (taken != gridDim.x - 1) return;
    __threadfence();
    // Last CTA: warp w sums accumulators w, w + 8, ... (lane L: chunks L,
    // L + 32, ... of the accumulator in order; then a fixed shuffle tree).
    const int lane = threadIdx.x & 31;
    for (int q = threadIdx.x >> 5; q < cm.np; q += 8) {
        double t = 0.0;
        for (int c = a.chunk_begin[q] + lane; c < a.chunk_begin[q + 1]; c += 32) t += __ldcg(cm.partials + c);
        t = warp_sum_d(t);
        if (lane == 0) {
            cm.out[q] = t;
            sums[q] = t;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (cm.clip_out) {
            double t = 0.0;
            for (int k = 0; k < cm.np; ++k) t += sums[k];
            if (cm.world > 1) t = clip_group_total(cm, t);
            const double gnorm = sqrt(t);
            const float c = (float)((double)cm.max_norm / (gnorm + 1e-6));
            // a missing peer: this step's gradients are dropped (clip 0); the
            // error word tells the host, which restores the saved state
            *cm.clip_out = t != t ? 0.0f : (c < 1.0f ? c : 1.0f);
            if (cm.gnorm_out) *cm.gnorm_out = gnorm;
        }
        *cm.ticket = 0u;
    }
}

template <int CAP>
int sqnorm_group_launch(const float* const* xs, const int64_t* ns, int cnt, const SqGroupCommon& common,
                        cudaStream_t st) {
    SqGroupArgs<CAP> a;
    memset(&a, 0, sizeof(a));
    a.c = common;
    a.c.np = cnt;
    for (int i = 0; i < cnt; ++i) {
        a.x[i] = xs[i];
        a.n[i] = ns[i];
        if ((reinterpret_cast<uintptr_t>(a.x[i]) & 15) != 0) return AETH_ERR_UNSUPPORTED;
    }
    // Chunks of at least 4096 elements, about four CTAs per SM, within the
    // kSqPartialSlots partial slots (a chunk per accumulator more than
    // total / chunk_elems at most).
    int64_t total = 0;
    for (int i = 0; i < cnt; ++i) total += a.n[i];
    const int64_t slots = (int64_t)kSqPartialSlots - cnt;
    int64_t ce = std::max<int64_t>(total / (4 * (int64_t)num_sms()), (total + slots - 1) / slots);
    ce = std::max<int64_t>(4096, (ce + 1023) / 1024 * 1024);
    a.c.chunk_elems = ce;
    int chunks = 0;
    for (int i = 0; i < cnt; ++i) {
        a.chunk_begin[i] = chunks;
        chunks += (int)std::max<int64_t>(1, (a.n[i] + ce - 1) / ce);
    }
    a.chunk_begin[cnt] = chunks;
    if (chunks > kSqPartialSlots) return AETH_ERR_UNSUPPORTED;
    sqnorm_group_kernel<CAP><<<chunks, 256, 0, st>>>(a);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// out[i] = sum of squares of xs[i] (f64).  With clip_out (np <= kSqGroupMax)
// the same launch also writes the global clip coefficient for max_norm.
// With a clip group of several GPUs the clip is computed from the sum over
// the whole group (clip_group_total); the device epoch advances once per launch.
inline int sqnorm_group(const float* const* xs, const int64_t* ns, int np, double* out, double* partials,
                        unsigned int* ticket, float max_norm, float* clip_out, double* gnorm_out, cudaStream_t st,
                        ClipGroup* group = nullptr) {
    if (np <= 0) return AETH_ERR_ARG;
    if (clip_out && np > kSqGroupMax) return AETH_ERR_UNSUPPORTED;
    if (group && group->world > 1 && !clip_out) return AETH_ERR_ARG;
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    SqGroupCommon c;
    memset(&c, 0, sizeof(c));
    c.max_norm = max_norm;
    c.clip_out = clip_out;
    c.gnorm_out = gnorm_out;
    c.partials = partials;
    c.ticket = ticket;
    c.world = 1;
    c.err = rt->err_word;
    if (group && group->world > 1) {
        c.rank = group->rank;
        c.world = group->world;
        for (int p = 0; p < group->world; ++p) c.slots[p] = group->slots[p];
        c.epoch = group->epoch;
        c.timeout_ns = group->timeout_ns;
    }
    for (int off = 0; off < np; off += kSqGroupMax) {
        const int cnt = std::min(kSqGroupMax, np - off);
        c.out = out + off;
        if (cnt <= kSqGroupSmall) AETH_TRY(sqnorm_group_launch<kSqGroupSmall>(xs + off, ns + off, cnt, c, st));
        else AETH_TRY(sqnorm_group_launch<kSqGroupMax>(xs + off, ns + off, cnt, c, st));
    }
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// K6
// ---------------------------------------------------------------------------
struct ApplyJob {
    const uint16_t* X;  // m x r bf16
    const uint16_t* Y;  // n x r bf16
    uint8_t* wp;        // m x n/2
    float* wa;          // m x n/64
    int m, n;
    float lr, decay_mul;
    int has_decay;
    float* prequant;
    float* delta;
};

// The grouped kernel needs n % 256 == 0 (absmax rows a multiple of 16 bytes)
// and r % 8 == 0; the rank is the MMAs' K, taken 64 at a time.
inline bool apply_grouped_supported(int m, int n, int r) {
    return m > 0 && n > 0 && n % 256 == 0 && r > 0 && r % 8 == 0 && r <= 1024;
}

// Whether the apply launches use CTA pairs (cluster of two, cta_group::2).
// On by default; AETH_APPLY_PAIR=0 in the environment selects the single-CTA
// kernel (for comparison).
inline bool apply_use_pair() {
    static const bool on = [] {
        const char* e = getenv("AETH_APPLY_PAIR");
        return !(e && e[0] == '0');
    }();
    return on;
}

// One launch of the specialisation for the group's decay and output flags.
template <int STAGES, bool PAIR, bool DECAY, bool OUT>
int apply_kernel_launch(const ApplyArgs& a, int units, uint32_t* err_word, cudaStream_t st) {
    using L = ApplyLayout<STAGES, PAIR>;
    const int smem = 1024 + L::kTotal;
    auto kern = apply_grouped_kernel<STAGES, PAIR, DECAY, OUT>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (!attr_set[dev]) {
        AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[dev] = true;
    }
    if (PAIR) {
        // one cluster of two CTAs per pair unit, at most a CTA per SM
        const int grid = 2 * std::min(num_sms() / 2, units);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kApplyThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        AETH_CUDA(cudaLaunchKernelEx(&cfg, kern, a, err_word));
    } else {
        const int grid = std::min(num_sms(), units);
        kern<<<grid, kApplyThreads, smem, st>>>(a, err_word);
        AETH_LAUNCH_CHECK();
    }
    return AETH_OK;
}

template <int STAGES, bool PAIR>
int apply_grouped_launch_t(const ApplyJob* jobs, int nj, int r, cudaStream_t st) {
    using L = ApplyLayout<STAGES, PAIR>;
    static_assert(1024 + L::kTotal <= 227 * 1024, "apply kernel shared memory above the per-CTA limit");
    constexpr int rows_per_unit = PAIR ? 256 : 128;
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    for (int off = 0; off < nj; off += kApplyMaxProblems) {
        const int cnt = std::min(kApplyMaxProblems, nj - off);
        ApplyArgs a;
        memset(&a, 0, sizeof(a));
        a.nprob = cnt;
        a.kb = (r + 63) / 64;
        a.idesc = idesc_f16(rows_per_unit, kApplyBN, true, false, false);
        int units = 0;
        for (int i = 0; i < cnt; ++i) {
            const ApplyJob& j = jobs[off + i];
            if (!apply_grouped_supported(j.m, j.n, r)) return AETH_ERR_UNSUPPORTED;
            ApplyProblem& p = a.p[i];
            AETH_TRY(make_tmap_16b(&p.tmX, j.X, (uint64_t)r, (uint64_t)j.m, r, 64, 128, true));
            AETH_TRY(make_tmap_16b(&p.tmY, j.Y, (uint64_t)r, (uint64_t)j.n, r, 64, PAIR ? kApplyBN / 2 : kApplyBN,
                                   true));
            AETH_TRY(make_tmap_2d(&p.tmW, j.wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(j.n / 2), (uint64_t)j.m,
                                  j.n / 2, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B));
            AETH_TRY(make_tmap_2d(&p.tmS, j.wa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(j.n / 64), (uint64_t)j.m,
                                  j.n / 64, 4, 128, CU_TENSOR_MAP_SWIZZLE_NONE));
            AETH_TRY(make_tmap_2d(&p.tmWq, j.wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(j.n / 2), (uint64_t)j.m,
                                  j.n / 2, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B));
            AETH_TRY(make_tmap_2d(&p.tmSq, j.wa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(j.n / 64), (uint64_t)j.m,
                                  j.n / 64, 4, 32, CU_TENSOR_MAP_SWIZZLE_NONE));
            p.prequant_out = j.prequant;
            p.delta_out = j.delta;
            p.m = j.m;
            p.n = j.n;
            p.n_tiles = (j.n + kApplyBN - 1) / kApplyBN;
            p.unit_begin = units;
            p.lr = j.lr;
            p.decay_mul = j.decay_mul;
            p.has_decay = j.has_decay;
            units += ((j.m + rows_per_unit - 1) / rows_per_unit) * p.n_tiles;
        }
        a.total_units = units;
        bool decay = false, out = false;
        for (int i = 0; i < cnt; ++i) {
            decay = decay || a.p[i].has_decay;
            out = out || a.p[i].prequant_out || a.p[i].delta_out;
        }
        int st_launch;
        if (decay) st_launch = out ? apply_kernel_launch<STAGES, PAIR, true, true>(a, units, rt->err_word, st)
                                   : apply_kernel_launch<STAGES, PAIR, true, false>(a, units, rt->err_word, st);
        else st_launch = out ? apply_kernel_launch<STAGES, PAIR, false, true>(a, units, rt->err_word, st)
                             : apply_kernel_launch<STAGES, PAIR, false, false>(a, units, rt->err_word, st);
        AETH_TRY(st_launch);
    }
    return AETH_OK;
}

inline int apply_grouped_launch(const ApplyJob* jobs, int nj, int r, cudaStream_t st) {
    // Two operand stages of 48 KB (single CTA) or four of 32 KB (pair): up to
    // r = 256 a unit's MMAs take a fraction of its epilogue; larger ranks
    // stream more k-blocks through the same ring, where the pair's smaller
    // per-SM operand bytes matter.
    if (apply_use_pair()) return apply_grouped_launch_t<4, true>(jobs, nj, r, st);
    return apply_grouped_launch_t<2, false>(jobs, nj, r, st);
}

}  // namespace aeth
