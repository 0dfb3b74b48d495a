// sqnorm.cuh -- squared norms of a step's accumulators (f64, deterministic)
// and the global clip (hook.rs:139-203), in one launch or as the first phase
// of the Adam launch, with the optional exchange of the local sum with the
// other GPUs of a clip group through peer memory.
#pragma once
#include <algorithm>

#include "common.cuh"

namespace aeth {

// ---------------------------------------------------------------------------
// Squared norms of several accumulators in one launch, deterministic: CTA
// (c, p) writes the f64 partial sum of chunk c of accumulator p into a fixed
// slot; the CTA that takes the last ticket sums each accumulator's slots in
// chunk order into out[p] and, when asked, also computes the global clip
// coefficient of clip_coeff_kernel (hook.rs:184-187) from out[0..np), then
// resets the ticket for the next launch.
// ---------------------------------------------------------------------------
constexpr int kSqGroupMax = 16;
constexpr int kSqChunks = 128;
constexpr int kClipGroupMax = 16;  // GPUs in a clip group

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

struct SqGroupArgs {
    const float* x[kSqGroupMax];
    int64_t n[kSqGroupMax];
    int np;
    float max_norm;
    float* clip_out;       // null: norms only
    double* gnorm_out;     // optional, with clip_out
    double* out;           // np sums
    double* partials;      // kSqGroupMax * kSqChunks
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

// Peer exchange primitives: a release store of the epoch after the value, an
// acquire load on the reader's side, both at system scope (NVLink peers).
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_gpu_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Writes this rank's sum into every group member's slot for this epoch, waits
// (bounded) for every member's sum, and returns the total in rank order, so
// every rank gets the same bits.  On timeout: flags the error and returns NaN.
__device__ inline double clip_group_total(const SqGroupArgs& a, double local) {
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

// Chunk c (of `chunks`) of accumulator p, as one 256-thread CTA computes it:
// thread t sums elements t, t + stride, ... (stride = chunks * 256 floats as
// float4 groups) in four interleaved f64 sums, then a fixed warp and CTA
// reduction; thread 0 stores the partial.  All threads of the CTA must call
// it (it synchronises).  The same arithmetic serves the stand-alone kernel and
// the norm phase fused into Adam, so both give the same bits.
__device__ inline void sq_chunk(const SqGroupArgs& a, int c, int p, int chunks, double* red) {
    const float4* x4 = reinterpret_cast<const float4*>(a.x[p]);
    const int64_t n = a.n[p], n4 = n / 4;
    const int64_t stride = (int64_t)chunks * 256;
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    int64_t i = c * (int64_t)256 + threadIdx.x;
    for (; i + 3 * stride < n4; i += 4 * stride) {  // four independent 16-byte loads in flight
        float4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = __ldcg(x4 + i + k * stride);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            s[k] += (double)u[k].x * u[k].x + (double)u[k].y * u[k].y + (double)u[k].z * u[k].z +
                    (double)u[k].w * u[k].w;
    }
    for (; i < n4; i += stride) {
        const float4 u = __ldcg(x4 + i);
        s[0] += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
    }
    for (int64_t k = n4 * 4 + c * (int64_t)256 + threadIdx.x; k < n; k += stride) {
        const double v = (double)a.x[p][k];
        s[0] += v * v;
    }
    const double sum = warp_sum_d((s[0] + s[1]) + (s[2] + s[3]));
    __syncthreads();  // red is free (a previous call of this CTA has read it)
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; ++w) t += red[w];
        a.partials[p * kSqChunks + c] = t;
    }
}

// The last CTA's work: warp w reduces accumulators w, w + 8, ... in a fixed
// order (lane L: chunks L, L + 32, ...; then a fixed shuffle tree) into
// out[], then thread 0 forms the clip (with the clip group's exchange) and
// resets the ticket.  All threads of the CTA must call it.
__device__ inline void sq_finish(const SqGroupArgs& a, int chunks) {
    const int lane = threadIdx.x & 31;
    for (int q = threadIdx.x >> 5; q < a.np; q += (int)(blockDim.x >> 5)) {
        double t = 0.0;
        for (int c = lane; c < chunks; c += 32) t += __ldcg(a.partials + q * kSqChunks + c);
        t = warp_sum_d(t);
        if (lane == 0) a.out[q] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (a.clip_out) {
            double t = 0.0;
            for (int k = 0; k < a.np; ++k) t += a.out[k];
            if (a.world > 1) t = clip_group_total(a, t);
            const double gnorm = sqrt(t);
            const float c = (float)((double)a.max_norm / (gnorm + 1e-6));
            // a missing peer: this step's gradients are dropped (clip 0); the
            // error word tells the host, which restores the saved state
            *a.clip_out = t != t ? 0.0f : (c < 1.0f ? c : 1.0f);
            if (a.gnorm_out) *a.gnorm_out = gnorm;
        }
        *a.ticket = 0u;
    }
}

// Number of chunks per accumulator: about 8K elements each, at most kSqChunks.
inline int sq_chunks_for(int64_t largest) {
    return (int)std::min<int64_t>(kSqChunks, std::max<int64_t>(1, (largest + 8191) / 8192));
}

__global__ void __launch_bounds__(256) sqnorm_group_kernel(const __grid_constant__ SqGroupArgs a) {
    __shared__ double red[8];
    __shared__ unsigned int taken;
    sq_chunk(a, blockIdx.x, blockIdx.y, gridDim.x, red);
    if (threadIdx.x == 0) {
        __threadfence();
        taken = atomicAdd(a.ticket, 1u);
    }
    __syncthreads();
    if (taken != gridDim.x * gridDim.y - 1) return;
    __threadfence();
    sq_finish(a, gridDim.x);
}

}  // namespace aeth
