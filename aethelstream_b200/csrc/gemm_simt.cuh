// gemm_simt.cuh -- fp32 CUDA-core GEMM that reproduces the reference's CPU
// loops bit for bit (galore/src/project.rs:6-16, 36-46).
//
// Each output element is owned by one thread and accumulated as
//     sum = 0; for k in 0..K: sum = sum + a(i,k) * b(k,j)
// with separately rounded multiply and add, in increasing k -- exactly the
// Rust `sum += a * b` loop.  This is the REF-mode projection engine (the
// parity target); the B200-mode projections run on tcgen05 tensor cores.
#pragma once
#include "common.cuh"

namespace aeth {

enum SimtEpilogue : int {
    SIMT_STORE = 0,        // C = sum
    SIMT_SCALE = 1,        // C = sum * alpha            (weight_delta *= lr, optimizer.rs:337-340)
    SIMT_ACCUM = 2,        // C = C + sum                (accumulate_grad, adamw.rs:91-96)
    SIMT_SUB_SCALED = 3,   // C = C - sum * alpha        (w -= lr * dW on an fp32 weight)
};

constexpr int kSimtTile = 64, kSimtK = 16;

// A(i,k) = A[i*sai + k*sak], B(k,j) = B[k*sbk + j*sbj], C(i,j) = C[i*ldc + j].
__global__ void __launch_bounds__(256) simt_gemm_exact_kernel(const float* __restrict__ A, int64_t sai, int64_t sak,
                                                              const float* __restrict__ B, int64_t sbk, int64_t sbj,
                                                              float* __restrict__ Cm, int64_t ldc, int M, int N,
                                                              int K, int epi, float alpha,
                                                              float* __restrict__ Cdelta) {
    __shared__ float As[kSimtK][kSimtTile + 1];
    __shared__ float Bs[kSimtK][kSimtTile + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.y * kSimtTile, j0 = blockIdx.x * kSimtTile;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += kSimtK) {
        for (int t = threadIdx.x; t < kSimtK * kSimtTile; t += 256) {
            int kk = t / kSimtTile, ii = t % kSimtTile;
            int gi = i0 + ii, gk = k0 + kk;
            As[kk][ii] = (gi < M && gk < K) ? A[gi * sai + gk * sak] : 0.0f;
            int gj = j0 + ii;
            Bs[kk][ii] = (gj < N && gk < K) ? B[gk * sbk + gj * sbj] : 0.0f;
        }
        __syncthreads();
        const int kmax = K - k0 < kSimtK ? K - k0 : kSimtK;
        for (int kk = 0; kk < kmax; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) av[a] = As[kk][ty + 16 * a];
#pragma unroll
            for (int b = 0; b < 4; ++b) bv[b] = Bs[kk][tx + 16 * b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(av[a], bv[b]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            int gi = i0 + ty + 16 * a, gj = j0 + tx + 16 * b;
            if (gi >= M || gj >= N) continue;
            float* c = Cm + (int64_t)gi * ldc + gj;
            float s = acc[a][b];
            if (epi == SIMT_STORE) *c = s;
            else if (epi == SIMT_SCALE) *c = __fmul_rn(s, alpha);
            else if (epi == SIMT_ACCUM) *c = __fadd_rn(*c, s);
            else {
                float d = __fmul_rn(s, alpha);
                if (Cdelta) Cdelta[(int64_t)gi * ldc + gj] = d;
                *c = __fsub_rn(*c, d);
            }
        }
}

inline int simt_gemm_exact(const float* A, int64_t sai, int64_t sak, const float* B, int64_t sbk, int64_t sbj,
                           float* C, int64_t ldc, int M, int N, int K, int epi, float alpha, float* Cdelta,
                           cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return AETH_ERR_ARG;
    dim3 grid((N + kSimtTile - 1) / kSimtTile, (M + kSimtTile - 1) / kSimtTile);
    simt_gemm_exact_kernel<<<grid, 256, 0, st>>>(A, sai, sak, B, sbk, sbj, C, ldc, M, N, K, epi, alpha, Cdelta);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// Elementwise helpers used by the REF path.
__global__ void to_f32_kernel(const void* __restrict__ x, int dtype, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = load_as_f32(x, i, dtype);
}

}  // namespace aeth
