// common.cuh -- status codes, per-thread last error, bounded device waits and
// small numeric helpers shared by every kernel of libaeth_galore.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/aeth_galore.h"

namespace aeth {

// Last status recorded on the calling host thread (read by aeth_last_error()).
inline thread_local int tl_last_error = AETH_OK;

inline int set_err(int st) {
    if (st != AETH_OK) tl_last_error = st;
    return st;
}

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? AETH_OK : set_err((int)e); }

#define AETH_TRY(expr)                                 \
    do {                                               \
        int _st = (expr);                              \
        if (_st != AETH_OK) return ::aeth::set_err(_st); \
    } while (0)

#define AETH_CUDA(expr)                                         \
    do {                                                        \
        cudaError_t _e = (expr);                                \
        if (_e != cudaSuccess) return ::aeth::set_err((int)_e); \
    } while (0)

// Kernel-launch check: configuration errors surface here, asynchronous
// errors on the next synchronising call.
#define AETH_LAUNCH_CHECK() AETH_CUDA(cudaGetLastError())

inline cudaStream_t to_stream(aeth_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// Device-side error word.  Kernels with spin waits give up after a time limit
// and OR a code into this word instead of hanging; the host reads it with
// aeth_device_error().  One word per device, allocated on first use.
// ---------------------------------------------------------------------------
enum : uint32_t {
    DEVERR_TIMEOUT_TMA = 1u,
    DEVERR_TIMEOUT_MMA = 2u,
    DEVERR_TIMEOUT_EPI = 4u,
    DEVERR_BAD_ARG = 8u,
    DEVERR_TIMEOUT_PEER = 16u,  // a peer GPU's squared-norm sum did not arrive in time
};

struct DeviceRuntime {
    uint32_t* err_word = nullptr;   // device
    std::atomic<bool> init{false};  // published (release) after err_word is stored
};

constexpr int kMaxDevices = 64;
inline DeviceRuntime g_rt[kMaxDevices];
// Serialises the first-use set-up of g_rt (and of any other per-device state
// that shares its error word), so two host threads that touch a device for
// the first time together neither allocate two words nor read a half-set one.
inline std::mutex g_rt_mu;

inline int current_device(int* dev) { return cuda_status(cudaGetDevice(dev)); }

inline int runtime_for_current(DeviceRuntime** out) {
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_err(AETH_ERR_UNSUPPORTED);
    DeviceRuntime& rt = g_rt[dev];
    if (!rt.init.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_rt_mu);
        if (!rt.init.load(std::memory_order_relaxed)) {
            uint32_t* w = nullptr;
            AETH_CUDA(cudaMalloc(&w, sizeof(uint32_t)));
            cudaError_t e = cudaMemset(w, 0, sizeof(uint32_t));
            if (e != cudaSuccess) {
                cudaFree(w);
                return set_err((int)e);
            }
            rt.err_word = w;
            rt.init.store(true, std::memory_order_release);
        }
    }
    *out = &rt;
    return AETH_OK;
}

// Nanosecond global timer (PTX %globaltimer).
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bound for every device-side wait: long enough for any legitimate stall of
// these kernels (they never wait on another rank), short enough that a bug
// ends the kernel within seconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ void report_dev_error(uint32_t* err, uint32_t code) {
    if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------------------
// Numeric helpers.  IEEE-rounded intrinsics are used wherever the CPU oracle
// must be reproduced bit for bit (no FMA contraction, correctly rounded
// division and square root).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
    if (dtype == AETH_DTYPE_F32) return static_cast<const float*>(p)[i];
    if (dtype == AETH_DTYPE_BF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Warp maximum of values that are >= 0 and not NaN (+inf allowed): their bit
// patterns order like unsigned integers, so one redux.sync does it.
__device__ __forceinline__ float warp_max_nonneg(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t smem_u32_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Loads from read-only shared tables at a 32-bit shared address (no memory
// clobber: use only for tables written before a __syncthreads and never after).
__device__ __forceinline__ uint32_t lds_u32(uint32_t saddr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr));
    return v;
}
__device__ __forceinline__ float2 lds_f2(uint32_t saddr) {
    float2 v;
    asm("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(saddr));
    return v;
}

// prmt.b32 in its default mode: a selector nibble with bit 3 set fills the
// output byte with the sign of the selected byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Three-input min / max of sm_100 (one instruction each).  fmax3 ignores a
// NaN operand; fmax3_nan returns NaN when any operand is NaN.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Packed f32x2 arithmetic of sm_100 (two lanes per instruction); each lane
// rounds exactly as the scalar __fmul_rn / __fadd_rn / __fmaf_rn does.
// Caution, measured on sm_100a with this toolchain: ptxas contracts a packed
// multiply whose only use is a packed add into one fused multiply-add, even
// with the explicit .rn and -fmad=false.  A sum of products that must round
// twice therefore adds with scalar __fadd_rn (add2_sep), which ptxas keeps
// separate; add2_rn is only for sums whose operands are not fresh products or
// where the fused rounding cannot change the result.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2_sep(float2 a, float2 b) {
    return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// atomicMax on a non-negative float stored as its bit pattern.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
    atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

inline int grid_for(int64_t work, int threads, int cap = 148 * 16) {
    int64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (int)g;
}

}  // namespace aeth
