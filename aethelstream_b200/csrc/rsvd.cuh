// rsvd.cuh -- K8: randomized-SVD projector refresh on the device
// (galore/src/randomized_svd.rs:38-271, called from optimizer.rs:208-246).
//
//   Omega (n x l, l = r + p) ~ N(0,1) by Box-Muller over xorshift64 from
//   max(seed, 1), drawn in row-major order (randomized_svd.rs:38-66, 93-97);
//   Y = G Omega; Q^ = orthonormal basis of Y; B = Q^T G; U = the reference's
//   50-rotation Jacobi on B B^T; P = Q^ U[:, :r]; Q = orthonormalised B^T U[:, :r].
//
// Device mapping:
//   * Omega: one thread per kOmegaChunk consecutive Gaussians; the xorshift64
//     state at the start of chunk t is M^(2 kOmegaChunk t) applied to the
//     seed, with M the generator's 64 x 64 matrix over GF(2) (the generator is
//     linear), so every thread starts exactly where the sequential draw would
//     be.  The host passes M^(2 kOmegaChunk 2^k) for every bit k of t.
//   * G Omega, Q^T G, B B^T, Q^ U, B^T U: the exact-order SIMT GEMM
//     (gemm_simt.cuh), the reference's f32 loops bit for bit on equal inputs.
//   * The orthonormal bases, exact path: the reference's modified
//     Gram-Schmidt in its own operation order (mgs_exact_kernel), so with the
//     same sketch the exact path gives the reference's P and Q bit for bit.
//   * The orthonormal bases, tensor-core path: Cholesky QR with an f64 Gram
//     matrix (two GEMMs and one small factorisation instead of l^2 / 2
//     sequential Gram-Schmidt dot products).  It equals modified Gram-Schmidt
//     in exact arithmetic (both give the Q factor with a positive R
//     diagonal); in f32 the two differ by rounding.  A Gram matrix that is not
//     positive definite is the rank-deficiency error of qr_columns.  The final
//     orthonormalisation of Q (orthonormalize_columns, which clamps tiny
//     norms instead of failing) falls back to a one-CTA modified Gram-Schmidt
//     when its Gram matrix is not positive definite.
//   * Jacobi: one CTA; every rotation reproduces the reference's in-place
//     update loop, including the values it reads back for k = p and k = q.
//   * Optional power iterations (a B200 extension; the reference never runs
//     them): Y <- G (G^T Q^) re-orthonormalised, power_iters times.
#pragma once
#include "common.cuh"
#include "gemm_simt.cuh"
#include "split_gemm.cuh"

namespace aeth {

// ---------------------------------------------------------------------------
// xorshift64 over GF(2): 64 x 64 bit matrices stored by column.
// ---------------------------------------------------------------------------
struct Gf2Mat64 {
    uint64_t col[64];
};

inline uint64_t xorshift64_step(uint64_t x) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
}

inline uint64_t gf2_apply(const Gf2Mat64& m, uint64_t x) {
    uint64_t y = 0;
    for (int j = 0; j < 64; ++j)
        if ((x >> j) & 1u) y ^= m.col[j];
    return y;
}

inline Gf2Mat64 gf2_mul(const Gf2Mat64& a, const Gf2Mat64& b) {
    Gf2Mat64 c;
    for (int j = 0; j < 64; ++j) c.col[j] = gf2_apply(a, b.col[j]);
    return c;
}

inline Gf2Mat64 gf2_xorshift_matrix() {
    Gf2Mat64 m;
    for (int j = 0; j < 64; ++j) m.col[j] = xorshift64_step(1ull << j);
    return m;
}

constexpr int kOmegaChunk = 128;  // Gaussians (256 draws) per thread
constexpr int kOmegaLevels = 40;  // chunk indices below 2^40

// jump[k] = M^(2 kOmegaChunk 2^k), k < kOmegaLevels.
inline void omega_jump_tables(Gf2Mat64* jump) {
    Gf2Mat64 step = gf2_xorshift_matrix();
    for (int i = 0; i < 8; ++i) step = gf2_mul(step, step);  // M^256 = M^(2 kOmegaChunk)
    static_assert(2 * kOmegaChunk == 256, "jump base assumes 256 draws per chunk");
    jump[0] = step;
    for (int k = 1; k < kOmegaLevels; ++k) jump[k] = gf2_mul(jump[k - 1], jump[k - 1]);
}

// The tables, built once per process (thread-safe static initialisation).
inline const Gf2Mat64* omega_jump_host() {
    static const std::vector<Gf2Mat64> tables = [] {
        std::vector<Gf2Mat64> t(kOmegaLevels);
        omega_jump_tables(t.data());
        return t;
    }();
    return tables.data();
}

__device__ __forceinline__ uint64_t gf2_apply_dev(const uint64_t* __restrict__ col, uint64_t x) {
    uint64_t y = 0;
#pragma unroll 8
    for (int j = 0; j < 64; ++j) y ^= ((x >> j) & 1u) ? col[j] : 0ull;
    return y;
}

__device__ __forceinline__ uint64_t xorshift64_dev(uint64_t x) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
}

// Rng::next_gaussian (randomized_svd.rs:61-65).
__device__ __forceinline__ float rsvd_gaussian(uint64_t& s) {
    s = xorshift64_dev(s);
    const float u1 = fmaxf(__fmul_rn((float)(s >> 40), 0x1p-24f), 1e-7f);
    s = xorshift64_dev(s);
    const float u2 = __fmul_rn((float)(s >> 40), 0x1p-24f);
    const float two_pi = 2.0f * 3.14159265358979323846f;
    // ln and cos of the f32 arguments in f64, rounded once to f32: the
    // correctly rounded values except where the f64 result lies within its
    // own error of an f32 rounding boundary.  A host libm that is not
    // correctly rounded differs from them by one ulp on a few inputs.
    const float ln_u1 = (float)log((double)u1);
    const float cos_a = (float)cos((double)__fmul_rn(two_pi, u2));
    return __fmul_rn(__fsqrt_rn(__fmul_rn(-2.0f, ln_u1)), cos_a);
}

__global__ void rsvd_omega_kernel(const uint64_t* __restrict__ jump, uint64_t s0, int64_t count,
                                  float* __restrict__ out) {
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t first = t * kOmegaChunk;
    if (first >= count) return;
    uint64_t s = s0;
    for (int k = 0; k < kOmegaLevels && (t >> k) != 0; ++k)
        if ((t >> k) & 1) s = gf2_apply_dev(jump + 64 * k, s);
    const int64_t last = first + kOmegaChunk < count ? first + kOmegaChunk : count;
    for (int64_t i = first; i < last; ++i) out[i] = rsvd_gaussian(s);
}

// ---------------------------------------------------------------------------
// C(i,j) = sum_k A(i,k) B(k,j), f64 accumulation in increasing k, strided
// operands (A(i,k) = A[i*sai + k*sak], B(k,j) = B[k*sbk + j*sbj]).
// ---------------------------------------------------------------------------
template <typename TA, typename TB, typename TC>
__global__ void __launch_bounds__(256) gemm_f64acc_kernel(const TA* __restrict__ A, int64_t sai, int64_t sak,
                                                          const TB* __restrict__ B, int64_t sbk, int64_t sbj,
                                                          TC* __restrict__ C, int64_t ldc, int M, int N, int K) {
    __shared__ double As[16][65];
    __shared__ double Bs[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
    double acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int t = threadIdx.x; t < 16 * 64; t += 256) {
            const int kk = t / 64, ii = t % 64;
            const int gi = i0 + ii, gj = j0 + ii, gk = k0 + kk;
            As[kk][ii] = (gi < M && gk < K) ? (double)A[gi * sai + gk * sak] : 0.0;
            Bs[kk][ii] = (gj < N && gk < K) ? (double)B[gk * sbk + gj * sbj] : 0.0;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < 16; ++kk) {
            double av[4], bv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) av[a] = As[kk][ty + 16 * a];
#pragma unroll
            for (int b = 0; b < 4; ++b) bv[b] = Bs[kk][tx + 16 * b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fma(av[a], bv[b], acc[a][b]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int gi = i0 + ty + 16 * a, gj = j0 + tx + 16 * b;
            if (gi < M && gj < N) C[gi * ldc + gj] = (TC)acc[a][b];
        }
}

template <typename TA, typename TB, typename TC>
inline int gemm_f64acc(const TA* A, int64_t sai, int64_t sak, const TB* B, int64_t sbk, int64_t sbj, TC* C,
                       int64_t ldc, int M, int N, int K, cudaStream_t st) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    gemm_f64acc_kernel<TA, TB, TC><<<grid, 256, 0, st>>>(A, sai, sak, B, sbk, sbj, C, ldc, M, N, K);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// Gram matrix G = X^T X (cols x cols, f64) of an f32 rows x cols matrix:
// only the lower-triangle 64 x 64 tiles, each over `chunks` slices of the
// rows (gridDim.y), the slice sums written to part[slice] and added in slice
// order by gram_reduce_kernel (deterministic); far more CTAs than one per
// output tile for the tall operands of the refresh (rows up to 28672).
// ---------------------------------------------------------------------------
constexpr int kGramMaxChunks = 8;

__global__ void __launch_bounds__(256) gram_f64_kernel(const float* __restrict__ x, int rows, int cols,
                                                       int rows_per_chunk, double* __restrict__ part) {
    __shared__ double As[16][65];
    __shared__ double Bs[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    int bi = (int)((sqrt(8.0 * blockIdx.x + 1.0) - 1.0) * 0.5);
    while ((bi + 1) * (bi + 2) / 2 <= (int)blockIdx.x) ++bi;
    while (bi * (bi + 1) / 2 > (int)blockIdx.x) --bi;
    const int bj = blockIdx.x - bi * (bi + 1) / 2;
    const int i0 = bi * 64, j0 = bj * 64;
    const int r0 = blockIdx.y * rows_per_chunk, r1 = min(rows, r0 + rows_per_chunk);
    double acc[4][4] = {};
    for (int k0 = r0; k0 < r1; k0 += 16) {
        for (int t = threadIdx.x; t < 16 * 64; t += 256) {
            const int kk = t / 64, ii = t % 64;
            const int gk = k0 + kk;
            const bool kin = gk < r1;
            As[kk][ii] = (kin && i0 + ii < cols) ? (double)x[(int64_t)gk * cols + i0 + ii] : 0.0;
            Bs[kk][ii] = (kin && j0 + ii < cols) ? (double)x[(int64_t)gk * cols + j0 + ii] : 0.0;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < 16; ++kk) {
            double av[4], bv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) av[a] = As[kk][ty + 16 * a];
#pragma unroll
            for (int b = 0; b < 4; ++b) bv[b] = Bs[kk][tx + 16 * b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fma(av[a], bv[b], acc[a][b]);
        }
        __syncthreads();
    }
    double* out = part + (int64_t)blockIdx.y * cols * cols;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int gi = i0 + ty + 16 * a, gj = j0 + tx + 16 * b;
            if (gi < cols && gj < cols) out[(int64_t)gi * cols + gj] = acc[a][b];
        }
}

__global__ void gram_reduce_kernel(const double* __restrict__ part, int chunks, int cols, double* __restrict__ g) {
    const int64_t n = (int64_t)cols * cols;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(t / cols), j = (int)(t % cols);
        if (j > i) continue;  // the lower triangle is all the factorisation reads
        double s = 0.0;
        for (int z = 0; z < chunks; ++z) s += part[z * n + t];
        g[t] = s;
    }
}

inline int gram_f64(const float* x, int rows, int cols, double* part, double* g, cudaStream_t st) {
    const int tiles_1d = (cols + 63) / 64;
    const int tiles = tiles_1d * (tiles_1d + 1) / 2;
    int chunks = (2 * num_sms() + tiles - 1) / tiles;
    chunks = std::max(1, std::min(chunks, std::min(kGramMaxChunks, (rows + 255) / 256)));
    const int per = ((rows + chunks - 1) / chunks + 15) / 16 * 16;
    chunks = (rows + per - 1) / per;
    gram_f64_kernel<<<dim3(tiles, chunks), 256, 0, st>>>(x, rows, cols, per, part);
    gram_reduce_kernel<<<grid_for((int64_t)cols * cols, 256), 256, 0, st>>>(part, chunks, cols, g);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// One CTA: Cholesky of the l x l f64 Gram matrix in place (lower triangle),
// then the inverse of the factor into Linv (lower; column c by thread c).
// *fail = 1 when a pivot is not positive.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) chol_inverse_kernel(double* __restrict__ a, int l, double* __restrict__ linv,
                                                            int* __restrict__ fail) {
    __shared__ int bad;
    __shared__ double piv;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    for (int k = 0; k < l; ++k) {
        if (threadIdx.x == 0) {
            const double d = a[(int64_t)k * l + k];
            if (!(d > 0.0)) bad = 1;
            piv = d > 0.0 ? sqrt(d) : 1.0;
            a[(int64_t)k * l + k] = piv;
        }
        __syncthreads();
        if (bad) break;
        for (int i = k + 1 + threadIdx.x; i < l; i += blockDim.x) a[(int64_t)i * l + k] /= piv;
        __syncthreads();
        const int rem = l - k - 1;
        const int64_t pairs = (int64_t)rem * (rem + 1) / 2;
        for (int64_t t = threadIdx.x; t < pairs; t += blockDim.x) {
            // (i, j) with k < j <= i < l, enumerated row by row
            int i = (int)((sqrt(8.0 * (double)t + 1.0) - 1.0) * 0.5);
            while ((int64_t)(i + 1) * (i + 2) / 2 <= t) ++i;
            while ((int64_t)i * (i + 1) / 2 > t) --i;
            const int j = (int)(t - (int64_t)i * (i + 1) / 2);
            const int gi = k + 1 + i, gj = k + 1 + j;
            a[(int64_t)gi * l + gj] -= a[(int64_t)gi * l + k] * a[(int64_t)gj * l + k];
        }
        __syncthreads();
    }
    if (bad) {
        if (threadIdx.x == 0) *fail = 1;
        return;
    }
    for (int c = threadIdx.x; c < l; c += blockDim.x) {
        for (int i = 0; i < c; ++i) linv[(int64_t)i * l + c] = 0.0;
        for (int i = c; i < l; ++i) {
            double s = i == c ? 1.0 : 0.0;
            for (int k = c; k < i; ++k) s -= a[(int64_t)i * l + k] * linv[(int64_t)k * l + c];
            linv[(int64_t)i * l + c] = s / a[(int64_t)i * l + i];
        }
    }
}

// ---------------------------------------------------------------------------
// A cluster of kCholCtas CTAs, blocked by 32 columns: the same factorisation
// and inverse as chol_inverse_kernel for l <= kCholMaxL.  The matrix stays in
// global memory (L2-resident); the CTAs meet at hardware cluster barriers,
// whose release / acquire order their global writes for each other.
//   Cholesky (right-looking), per 32-column step: every CTA loads the panel
//   below the diagonal into shared memory (pitch 33 doubles) and factors it
//   redundantly -- warp 0 the diagonal block in registers (lane = row, the
//   pivots and scaled columns by shuffle), one thread per row the solve
//   against it -- so all CTAs hold the same panel without an exchange; the
//   32 x 32 blocks of the trailing lower triangle are then shared out over
//   the cluster's warps (lane = row, 32 accumulators; the panel rows of the
//   column block are broadcast reads).  CTA 0 writes each factored panel
//   back after the step's closing barrier, when no CTA still reads it.
//   Inverse: each diagonal block's inverse by one warp (lane = column,
//   forward substitution); then block rows ib in order,
//   X_ij = -inv(L_ii) sum_{k = j}^{i-1} L_ik X_kj, with the (jb, 4-column
//   group) pieces of block row ib shared out over the cluster's warps.
// *fail = 1 when a pivot is not positive (or NaN); every CTA reaches the same
// decision at the same step (identical redundant arithmetic), so all leave
// together.
// ---------------------------------------------------------------------------
constexpr int kCholMaxL = 640;
constexpr int kCholThreads = 512;
constexpr int kCholCtas = 8;
constexpr size_t kCholSmem = sizeof(double) * kCholMaxL * 33;  // also a 32-row block of L in the inverse
static_assert(32 * (kCholMaxL + 1) <= kCholMaxL * 33, "the inverse's block row of L must fit the panel buffer");

__device__ __forceinline__ void chol_store_panel(double* __restrict__ a, const double* __restrict__ pan, int l, int k0,
                                                 int kw) {
    const int prow = l - k0;
    for (int t = threadIdx.x; t < prow * 32; t += blockDim.x) {
        const int i = t >> 5, c = t & 31;
        if (c < kw && c <= i) a[(int64_t)(k0 + i) * l + k0 + c] = pan[i * 33 + c];
    }
}

// The panel rows k0 .. l-1, columns k0 .. k0+kw-1 (lower triangle of the
// diagonal block, zeros elsewhere) into shared memory, as asynchronous 8-byte
// copies (zero-filled outside the triangle): a thread's copies are all in
// flight at once instead of one L2 round trip per element, and they hold no
// registers.  The caller waits with cp_async_wait_all() and a barrier.
__device__ __forceinline__ void chol_load_panel(double* __restrict__ pan, const double* __restrict__ a, int l, int k0,
                                                int kw, int prow) {
    const int n = prow * 32;
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int i = t >> 5, c = t & 31;
        const bool in = c < kw && c <= i;
        const double* src = a + (int64_t)(k0 + (in ? i : 0)) * l + k0 + (in ? c : 0);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32_addr(pan + i * 33 + c)), "l"(src),
                     "r"(in ? 8 : 0)
                     : "memory");
    }
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kCholThreads) chol_cluster_kernel(double* __restrict__ a, int l,
                                                                    double* __restrict__ linv, int* __restrict__ fail) {
    extern __shared__ double pan[];  // (l - k0) x 33
    __shared__ double rdiag[32];
    __shared__ int bad;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int crank = (int)cluster_ctarank();
    const int gw = crank * nwarps + warp, gwarps = kCholCtas * nwarps;  // warp index over the cluster
    const int nb = (l + 31) / 32;
    if (tid == 0) bad = 0;
    __syncthreads();
    int kb = 0;
    for (; kb < nb; ++kb) {
        const int k0 = kb * 32, kw = min(32, l - k0), prow = l - k0;
        if (kb > 0 && crank == 0) {  // the previous panel, which no CTA reads any more
            chol_store_panel(a, pan, l, k0 - 32, 32);
            __syncthreads();
        }
        chol_load_panel(pan, a, l, k0, kw, prow);
        cp_async_wait_all();
        __syncthreads();
        if (warp == 0) {
            // the diagonal block in registers, lane = row: column c's pivot comes
            // by shuffle, the lanes below scale their entry, and every lane
            // updates its row's later columns with the scaled column (shuffled)
            double r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = (lane < kw && j <= lane) ? pan[lane * 33 + j] : 0.0;
            bool okall = true;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                if (c < kw) {  // warp-uniform
                    const double d = __shfl_sync(0xffffffffu, r[c], c);
                    const bool ok = d > 0.0;
                    okall = okall && ok;
                    // 1 / pivot from rsqrt (no square root and no division on the
                    // chain from one pivot to the next); the solve below reuses it
                    const double ip = ok ? rsqrt(d) : 1.0;
                    if (lane == c) {
                        r[c] = ok ? d * ip : 1.0;
                        rdiag[c] = ip;
                    } else if (lane > c) {
                        r[c] = r[c] * ip;
                    }
#pragma unroll
                    for (int j = c + 1; j < 32; ++j) {
                        const double ljc = __shfl_sync(0xffffffffu, r[c], j);
                        if (lane >= j) r[j] -= r[c] * ljc;
                    }
                }
            }
            if (!okall && lane == 0) bad = 1;
            if (lane < kw)
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j <= lane) pan[lane * 33 + j] = r[j];
        }
        __syncthreads();
        if (bad) break;  // the same step in every CTA
        // the panel below the diagonal block: row i solves x L_kk^T = a_i
        // (the pivots' reciprocals from the factorisation above instead of a
        // division per element)
        for (int i = kw + tid; i < prow; i += blockDim.x) {
            double x[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                if (c < kw) {
                    double v = pan[i * 33 + c];
#pragma unroll
                    for (int t = 0; t < c; ++t) v -= x[t] * pan[c * 33 + t];
                    x[c] = v * rdiag[c];
                } else {
                    x[c] = 0.0;
                }
            }
#pragma unroll
            for (int c = 0; c < 32; ++c)
                if (c < kw) pan[i * 33 + c] = x[c];
        }
        __syncthreads();
        // trailing update of the lower triangle: blocks (ib, jb), kb < jb <= ib,
        // shared out over the cluster's warps
        const int q = nb - kb - 1;
        const int pairs = q * (q + 1) / 2;
        for (int p = gw; p < pairs; p += gwarps) {
            int bi = (int)((sqrt(8.0 * p + 1.0) - 1.0) * 0.5);
            while ((bi + 1) * (bi + 2) / 2 <= p) ++bi;
            while (bi * (bi + 1) / 2 > p) --bi;
            const int bj = p - bi * (bi + 1) / 2;
            // lane = column gj of the block, acc[i] = row gi0 + i: the global
            // read-modify-write of each row is one coalesced 256-byte access
            const int gi0 = (kb + 1 + bi) * 32, gj = (kb + 1 + bj) * 32 + lane;
            double acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.0;
            const int ni = min(32, l - gi0);  // rows of the block inside the matrix (warp-uniform)
            if (gj < l) {
                const double* prow = pan + (gi0 - k0) * 33;
                for (int t = 0; t < kw; ++t) {
                    const double lj = pan[(gj - k0) * 33 + t];
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (i < ni) acc[i] += prow[i * 33 + t] * lj;
                }
                double* arow = a + (int64_t)gi0 * l + gj;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (i < ni && gj <= gi0 + i) arow[i * l] -= acc[i];
            }
        }
        cluster_sync();  // the trailing updates of every CTA before the next panel load
    }
    if (bad) {
        if (crank == 0 && tid == 0) *fail = 1;
        return;  // every CTA of the cluster leaves here, with no barrier outstanding
    }
    if (crank == 0) chol_store_panel(a, pan, l, (nb - 1) * 32, l - (nb - 1) * 32);
    cluster_sync();
    // L^-1: diagonal blocks first, on the first four warps of each CTA (lane =
    // column c of the block's inverse, forward substitution); each such warp
    // stages its 32 x 32 block of L and keeps the inverse's columns in its own
    // part of the panel buffer (pitch 33: lane-private columns, broadcast rows)
    if (warp < 4) {
        for (int db = warp * kCholCtas + crank; db < nb; db += 4 * kCholCtas) {
            const int d0 = db * 32, dw = min(32, l - d0);
            double* ld = pan + warp * (2 * 32 * 33);
            double* xc = ld + 32 * 33;
            // asynchronous copies, zero-filled outside the block's lower
            // triangle; rows past the matrix get a unit diagonal afterwards
            for (int i = 0; i < 32; ++i) {
                const bool in = i < dw && lane <= i;
                const double* src = a + (int64_t)(d0 + (in ? i : 0)) * l + d0 + (in ? lane : 0);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32_addr(ld + i * 33 + lane)),
                             "l"(src), "r"(in ? 8 : 0)
                             : "memory");
            }
            cp_async_wait_all();
            if (lane >= dw) ld[lane * 33 + lane] = 1.0;
            __syncwarp();
            for (int i = 0; i < 32; ++i) {
                double v = (i == lane) ? 1.0 : 0.0;
#pragma unroll 8
                for (int t = 0; t < i; ++t) v -= ld[i * 33 + t] * xc[t * 33 + lane];
                xc[i * 33 + lane] = v / ld[i * 33 + i];
            }
            if (lane < dw)
                for (int i = 0; i < dw; ++i) linv[(int64_t)(d0 + i) * l + d0 + lane] = xc[i * 33 + lane];
            __syncwarp();
        }
    }
    cluster_sync();
    // off-diagonal blocks by block rows: X_ij = -inv(L_ii) sum_{k = j}^{i-1}
    // L_ik X_kj needs only earlier block rows of L^-1.  For block row ib every
    // CTA stages L's rows i0 .. i0 + 31 (columns < i0) and inv(L_ii) in shared
    // memory; the pieces (jb < ib, 4-column group g) go to the cluster's warps:
    // lane = row, 4 accumulators.  X_kj comes 32 rows at a time: each lane
    // loads one row's 4 values into the warp's staging tile, the next batch's
    // loads in flight while the lanes read the tile as broadcasts; then
    // -inv(L_ii) S from S's rows staged the same way.
    __shared__ double xs[kCholThreads / 32][32 * 4];
    __shared__ double dinv_s[32 * 33];
    const int pitch = l + 1;  // odd pitch: the lanes' rows fall in different banks
    double* xw = xs[warp];
    for (int ib = 1; ib < nb; ++ib) {
        const int i0 = ib * 32, iw = min(32, l - i0);
        // columns 0 .. i0 - 1 of the block row (i0 < l < pitch)
        // (a warp per row; asynchronous copies, zero rows past the matrix)
        for (int r = warp; r < 32; r += nwarps) {
            const double* src = a + (int64_t)(i0 + (r < iw ? r : 0)) * l;
            for (int k = lane; k < i0; k += 32)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32_addr(pan + r * pitch + k)),
                             "l"(src + k), "r"(r < iw ? 8 : 0)
                             : "memory");
        }
        for (int t = tid; t < 32 * 32; t += blockDim.x) {
            const int r = t >> 5, c = t & 31;
            dinv_s[r * 33 + c] = (r < iw && c < iw) ? linv[(int64_t)(i0 + r) * l + i0 + c] : 0.0;
        }
        cp_async_wait_all();
        __syncthreads();
        const double* lrow = pan + lane * pitch;
        for (int piece = gw; piece < ib * 8; piece += gwarps) {
            const int jb = piece >> 3, c0 = jb * 32 + (piece & 7) * 4;  // jb < ib: a full block column
            double acc[4] = {0.0, 0.0, 0.0, 0.0};
            double nx[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) nx[c] = linv[(int64_t)(jb * 32 + lane) * l + c0 + c];
            for (int kb2 = jb; kb2 < ib; ++kb2) {
                __syncwarp();  // the previous batch's tile is read
#pragma unroll
                for (int c = 0; c < 4; ++c) xw[lane * 4 + c] = nx[c];
                __syncwarp();
                if (kb2 + 1 < ib)
#pragma unroll
                    for (int c = 0; c < 4; ++c) nx[c] = linv[(int64_t)((kb2 + 1) * 32 + lane) * l + c0 + c];
                const double* lk = lrow + kb2 * 32;
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const double lik = lk[t];
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[c] += lik * xw[t * 4 + c];
                }
            }
            // X_ij (4 columns) = -inv(L_ii) S: S's rows through the staging tile
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 4; ++c) xw[lane * 4 + c] = acc[c];
            __syncwarp();
            double out[4] = {0.0, 0.0, 0.0, 0.0};
            const double* drow = dinv_s + lane * 33;
#pragma unroll
            for (int t = 0; t < 32; ++t) {
                const double dv = drow[t];
#pragma unroll
                for (int c = 0; c < 4; ++c) out[c] -= dv * xw[t * 4 + c];
            }
            if (lane < iw)
#pragma unroll
                for (int c = 0; c < 4; ++c) linv[(int64_t)(i0 + lane) * l + c0 + c] = out[c];
            __syncwarp();
        }
        cluster_sync();  // block row ib of L^-1 for every CTA; the staging buffers are free again
    }
    // zero the strict upper triangle of L^-1 (callers read all of it)
    for (int64_t t = (int64_t)crank * blockDim.x + tid; t < (int64_t)l * l; t += (int64_t)kCholCtas * blockDim.x) {
        const int i = (int)(t / l), j = (int)(t % l);
        if (j > i) linv[t] = 0.0;
    }
}

// Cholesky and inverse of the l x l Gram matrix: the cluster kernel when its
// panel fits shared memory, else the per-element one.
inline int chol_inverse(double* gram, int l, double* linv, int* fail, cudaStream_t st) {
    if (l <= kCholMaxL) {
        static bool attr_set[kMaxDevices] = {};
        int dev = 0;
        AETH_TRY(current_device(&dev));
        if (!attr_set[dev]) {
            AETH_CUDA(cudaFuncSetAttribute(chol_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kCholSmem));
            attr_set[dev] = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kCholCtas);
        cfg.blockDim = dim3(kCholThreads);
        cfg.dynamicSmemBytes = kCholSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = kCholCtas;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        AETH_CUDA(cudaLaunchKernelEx(&cfg, chol_cluster_kernel, gram, l, linv, fail));
        return AETH_OK;
    } else {
        chol_inverse_kernel<<<1, 1024, 0, st>>>(gram, l, linv, fail);
    }
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// dst = src where *flag is set (the fallback's starting point), else nothing.
__global__ void copy_if_flag_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t n,
                                    const int* __restrict__ flag) {
    if (!*flag) return;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// ---------------------------------------------------------------------------
// One CTA: modified Gram-Schmidt with the norm clamp of
// orthonormalize_columns (randomized_svd.rs:187-207); the rare fallback.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) mgs_clamped_kernel(float* __restrict__ q, int rows, int cols,
                                                           const int* __restrict__ only_if = nullptr) {
    if (only_if && !*only_if) return;
    __shared__ float red[32];
    __shared__ float bcast;
    auto block_sum = [&](float v) -> float {
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.0f;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
            bcast = t;
        }
        __syncthreads();
        const float r = bcast;
        __syncthreads();
        return r;
    };
    for (int j = 0; j < cols; ++j) {
        for (int i = 0; i < j; ++i) {
            float d = 0.0f;
            for (int r = threadIdx.x; r < rows; r += blockDim.x)
                d = __fadd_rn(d, __fmul_rn(q[(int64_t)r * cols + i], q[(int64_t)r * cols + j]));
            d = block_sum(d);
            for (int r = threadIdx.x; r < rows; r += blockDim.x)
                q[(int64_t)r * cols + j] = __fsub_rn(q[(int64_t)r * cols + j], __fmul_rn(d, q[(int64_t)r * cols + i]));
            __syncthreads();
        }
        float nn = 0.0f;
        for (int r = threadIdx.x; r < rows; r += blockDim.x)
            nn = __fadd_rn(nn, __fmul_rn(q[(int64_t)r * cols + j], q[(int64_t)r * cols + j]));
        nn = __fsqrt_rn(fmaxf(block_sum(nn), 1e-12f));
        for (int r = threadIdx.x; r < rows; r += blockDim.x)
            q[(int64_t)r * cols + j] = __fdiv_rn(q[(int64_t)r * cols + j], nn);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// One CTA: modified Gram-Schmidt in the reference's exact order, bit for bit:
// qr_columns (randomized_svd.rs:160-185; fail_on_small: a column norm below
// 1e-12 sets *status to 1 and ends the kernel) or orthonormalize_columns
// (:187-207, the norm clamped to 1e-12).  q is rows x cols, row-major.
//
// The reference runs left-looking: for column j, the dots with columns
// 0 .. j-1 in turn, each followed by its subtraction, then the norm.  This
// kernel runs the same operations right-looking: once column i is final
// (normalised), every column j > i takes its dot with column i and its
// subtraction.  Column j sees exactly the same values in the same order
// (the subtractions of columns 0 .. i-1 before the dot with column i), so
// every rounding is the reference's; only the dots of different columns now
// run side by side, one thread per column, each summing its rows in
// increasing order with separately rounded products and sums.  Column i's
// values are staged in shared memory kMgsChunk rows at a time and read as
// broadcasts.  The thread that updates column i + 1 sums that column's
// squares in row order as it writes them: the next step's norm.
// ---------------------------------------------------------------------------
constexpr int kMgsThreads = 1024;
constexpr int kMgsChunk = 4096;
constexpr int kMgsMaxCols = 2 * kMgsThreads;

__global__ void __launch_bounds__(kMgsThreads) mgs_exact_kernel(float* __restrict__ q, int rows, int cols,
                                                                int fail_on_small, int* __restrict__ status) {
    __shared__ float ci[kMgsChunk];
    __shared__ float s_sumsq;
    const int tid = threadIdx.x;
    auto norm_of = [&](float s) -> float {
        return fail_on_small ? __fsqrt_rn(s) : __fsqrt_rn(fmaxf(s, 1e-12f));
    };
    if (tid == 0) {
        float s = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const float x = q[(int64_t)r * cols];
            s = __fadd_rn(s, __fmul_rn(x, x));
        }
        s_sumsq = s;
    }
    for (int i = 0; i < cols; ++i) {
        __syncthreads();  // s_sumsq of column i; column i's subtractions done
        const float nrm = norm_of(s_sumsq);
        if (fail_on_small && nrm < 1e-12f) {
            if (tid == 0 && status) *status = 1;
            return;
        }
        for (int r = tid; r < rows; r += kMgsThreads)
            q[(int64_t)r * cols + i] = __fdiv_rn(q[(int64_t)r * cols + i], nrm);
        if (i + 1 == cols) break;
        // this thread's columns of the trailing block: j0 = i + 1 + tid and j0 + kMgsThreads
        const int j0 = i + 1 + tid, j1 = j0 + kMgsThreads;
        const bool h0 = j0 < cols, h1 = j1 < cols;
        float d0 = 0.0f, d1 = 0.0f;
        for (int c0 = 0; c0 < rows; c0 += kMgsChunk) {
            const int cn = min(kMgsChunk, rows - c0);
            __syncthreads();  // the previous chunk is read; column i is normalised
            for (int r = tid; r < cn; r += kMgsThreads) ci[r] = q[(int64_t)(c0 + r) * cols + i];
            __syncthreads();
            const float* p0 = q + (int64_t)c0 * cols + j0;
            if (h1) {
                const float* p1 = p0 + kMgsThreads;
#pragma unroll 8
                for (int r = 0; r < cn; ++r) {
                    d0 = __fadd_rn(d0, __fmul_rn(ci[r], p0[(int64_t)r * cols]));
                    d1 = __fadd_rn(d1, __fmul_rn(ci[r], p1[(int64_t)r * cols]));
                }
            } else if (h0) {
#pragma unroll 8
                for (int r = 0; r < cn; ++r) d0 = __fadd_rn(d0, __fmul_rn(ci[r], p0[(int64_t)r * cols]));
            }
        }
        float s = 0.0f;  // column i + 1's squared norm (thread 0 owns j0 = i + 1)
        for (int c0 = 0; c0 < rows; c0 += kMgsChunk) {
            const int cn = min(kMgsChunk, rows - c0);
            __syncthreads();
            for (int r = tid; r < cn; r += kMgsThreads) ci[r] = q[(int64_t)(c0 + r) * cols + i];
            __syncthreads();
            float* p0 = q + (int64_t)c0 * cols + j0;
            if (h0) {
#pragma unroll 8
                for (int r = 0; r < cn; ++r) {
                    const float x = __fsub_rn(p0[(int64_t)r * cols], __fmul_rn(d0, ci[r]));
                    p0[(int64_t)r * cols] = x;
                    s = __fadd_rn(s, __fmul_rn(x, x));
                }
            }
            if (h1) {
                float* p1 = p0 + kMgsThreads;
#pragma unroll 8
                for (int r = 0; r < cn; ++r) p1[(int64_t)r * cols] = __fsub_rn(p1[(int64_t)r * cols], __fmul_rn(d1, ci[r]));
            }
        }
        if (tid == 0) s_sumsq = s;
    }
}

// ---------------------------------------------------------------------------
// One CTA: jacobi_eigenvectors (randomized_svd.rs:210-271) on the f32 n x n
// matrix `mat` (destroyed), eigenvector estimate into u.  Bit-exact with the
// reference's loop: each rotation zeroes the largest |a_ij|, i < j, the first
// in row-major order winning ties (a strict > scan, so NaN and zero entries
// are never picked), with the reference's arithmetic.
//
// The pick keeps a running maximum per row in shared memory (value and first
// column of the row's upper part) instead of rescanning the matrix: the
// global pick is the largest row maximum, the first row winning ties, which
// is the first maximal element in row-major order.  A rotation of (p, q)
// rewrites rows p and q (rescanned by one warp each) and, in every other row
// k < q, the upper entries (k, p) and (k, q): a row whose maximum sat in one
// of those columns is rescanned, any other takes the new entries into its
// maximum by the same comparison rules.
// ---------------------------------------------------------------------------
constexpr int kJacobiMaxN = 2048;

// First maximum of |mat[i][j]|, j > i, over the warp's lanes (strict >; the
// smaller column on equal values).
__device__ __forceinline__ void jacobi_row_scan(const float* __restrict__ mat, int n, int i, int lane, float& v,
                                                int& idx) {
    float bv = 0.0f;
    int bi = -1;
    for (int j = i + 1 + lane; j < n; j += 32) {
        const float x = fabsf(mat[(int64_t)i * n + j]);
        if (x > bv) { bv = x; bi = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi >= 0 && (bi < 0 || oi < bi))) { bv = ov; bi = oi; }
    }
    v = bv;
    idx = bi;
}

__global__ void __launch_bounds__(1024) jacobi50_kernel(float* __restrict__ mat, int n, float* __restrict__ u) {
    __shared__ float rmax[kJacobiMaxN];
    __shared__ int ridx[kJacobiMaxN];
    __shared__ int rescan[kJacobiMaxN];
    __shared__ float red_v[32];
    __shared__ int red_i[32];
    __shared__ int s_p, s_q, s_stop, s_nres;
    __shared__ float s_c, s_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    for (int64_t t = tid; t < (int64_t)n * n; t += blockDim.x) u[t] = (t / n == t % n) ? 1.0f : 0.0f;
    for (int i = warp; i < n; i += nwarps) {
        float v;
        int idx;
        jacobi_row_scan(mat, n, i, lane, v, idx);
        if (lane == 0) { rmax[i] = v; ridx[i] = idx; }
    }
    __syncthreads();
    for (int it = 0; it < 50; ++it) {
        // the largest row maximum, the first row on ties
        float bv = 0.0f;
        int bi = -1;
        for (int i = tid; i < n; i += blockDim.x)
            if (ridx[i] >= 0 && rmax[i] > bv) { bv = rmax[i]; bi = i; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi >= 0 && (bi < 0 || oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            float v = 0.0f;
            int row = -1;
            for (int w = 0; w < nwarps; ++w)
                if (red_v[w] > v || (red_v[w] == v && red_i[w] >= 0 && (row < 0 || red_i[w] < row))) {
                    v = red_v[w];
                    row = red_i[w];
                }
            // reference defaults p = 0, q = 1 and stops when max_off < 1e-10
            s_stop = v < 1e-10f;
            const int p = row >= 0 ? row : 0, q = row >= 0 ? ridx[row] : 1;
            s_p = p;
            s_q = q;
            s_nres = 0;
            if (!s_stop) {
                const float app = mat[(int64_t)p * n + p], aqq = mat[(int64_t)q * n + q], apq = mat[(int64_t)p * n + q];
                const float tau = __fdiv_rn(__fsub_rn(aqq, app), __fmul_rn(2.0f, apq));
                const float root = __fsqrt_rn(__fadd_rn(1.0f, __fmul_rn(tau, tau)));
                const float t = tau >= 0.0f ? __fdiv_rn(1.0f, __fadd_rn(tau, root))
                                            : __fdiv_rn(-1.0f, __fadd_rn(-tau, root));
                const float c = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(1.0f, __fmul_rn(t, t))));
                s_c = c;
                s_s = __fmul_rn(t, c);
            }
        }
        __syncthreads();
        if (s_stop) break;
        const int p = s_p, q = s_q;
        const float c = s_c, s = s_s;
        // rows k other than p, q read only their own (unchanged) entries
        for (int k = tid; k < n; k += blockDim.x) {
            if (k != p && k != q) {
                const float mkp = mat[(int64_t)k * n + p], mkq = mat[(int64_t)k * n + q];
                const float np_ = __fsub_rn(__fmul_rn(c, mkp), __fmul_rn(s, mkq));
                const float nq_ = __fadd_rn(__fmul_rn(s, mkp), __fmul_rn(c, mkq));
                mat[(int64_t)k * n + p] = np_;
                mat[(int64_t)p * n + k] = np_;
                mat[(int64_t)k * n + q] = nq_;
                mat[(int64_t)q * n + k] = nq_;
                // row k's maximum over its upper part (k < p: column p; k < q: column q)
                if (k < q) {
                    if (ridx[k] == p || ridx[k] == q) {
                        rescan[atomicAdd(&s_nres, 1)] = k;
                    } else {
                        float v = rmax[k];
                        int idx = ridx[k];
                        if (k < p) {
                            const float x = fabsf(np_);
                            if (x > v || (x == v && idx >= 0 && p < idx)) { v = x; idx = p; }
                        }
                        const float x = fabsf(nq_);
                        if (x > v || (x == v && idx >= 0 && q < idx)) { v = x; idx = q; }
                        rmax[k] = v;
                        ridx[k] = idx;
                    }
                }
            }
            const float ukp = u[(int64_t)k * n + p], ukq = u[(int64_t)k * n + q];
            u[(int64_t)k * n + p] = __fsub_rn(__fmul_rn(c, ukp), __fmul_rn(s, ukq));
            u[(int64_t)k * n + q] = __fadd_rn(__fmul_rn(s, ukp), __fmul_rn(c, ukq));
        }
        if (tid == 0) {
            // k = p (p < q) runs first and rewrites a_pq, which k = q then reads
            const float app = mat[(int64_t)p * n + p], aqq = mat[(int64_t)q * n + q], apq = mat[(int64_t)p * n + q];
            const float npp = __fsub_rn(__fmul_rn(c, app), __fmul_rn(s, apq));
            const float tpq = __fadd_rn(__fmul_rn(s, app), __fmul_rn(c, apq));
            const float nqq = __fadd_rn(__fmul_rn(s, tpq), __fmul_rn(c, aqq));
            mat[(int64_t)p * n + p] = npp;
            mat[(int64_t)q * n + q] = nqq;
            mat[(int64_t)p * n + q] = 0.0f;
            mat[(int64_t)q * n + p] = 0.0f;
            rescan[atomicAdd(&s_nres, 1)] = p;
            rescan[atomicAdd(&s_nres, 1)] = q;
        }
        __syncthreads();
        // rows p, q and the rows whose maximum was rewritten: one warp each
        const int nres = s_nres;
        for (int w = warp; w < nres; w += nwarps) {
            const int i = rescan[w];
            float v;
            int idx;
            jacobi_row_scan(mat, n, i, lane, v, idx);
            if (lane == 0) { rmax[i] = v; ridx[i] = idx; }
        }
        __syncthreads();
    }
}

__global__ void bf16_to_f32_rsvd_kernel(const uint16_t* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = bf16_bits_to_f32(x[i]);
}

// ---------------------------------------------------------------------------
// Host orchestration.
// ---------------------------------------------------------------------------
struct RsvdWork {
    float* omega = nullptr;  // n x l
    float* y = nullptr;      // m x l (sketch, then Q^)
    float* y2 = nullptr;     // max(m, n) x l scratch
    float* b = nullptr;      // l x n
    float* bbt = nullptr;    // l x l
    float* u = nullptr;      // l x l
    float* ur = nullptr;     // l x r: the first r columns of u
    double* gpart = nullptr; // kGramMaxChunks x l x l: slice sums of the Gram matrix
    uint16_t* xt = nullptr;  // fast path: bf16 terms of the matrix being orthonormalised (3 x rows x l)
    uint16_t* lt = nullptr;  // fast path: bf16 terms of Linv (3 x l x l)
    float* linv32 = nullptr; // fast path: Linv in f32
    double* gram = nullptr;  // l x l
    double* linv = nullptr;  // l x l
    uint64_t* jump = nullptr;
    int* fail = nullptr;
};

// Orthonormal basis of the columns of x (rows x cols) by Cholesky QR, in
// place; `tmp` holds rows x cols floats.  Two passes.  Returns 1 in *fail_dev
// when the Gram matrix is not positive definite.
__global__ void f64_to_f32_kernel(const double* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = (float)x[i];
}

inline int cholqr2(float* x, float* tmp, int rows, int cols, RsvdWork& w, cudaStream_t st, int* fail = nullptr,
                   int passes = 2) {
    // with the tensor-core workspace (fast path) the product x Linv^T runs
    // on tcgen05 over exact bf16 terms of x and of Linv rounded to f32
    const bool tc = w.xt && w.lt && cols % 8 == 0;
    for (int pass = 0; pass < passes; ++pass) {
        AETH_TRY(gram_f64(x, rows, cols, w.gpart, w.gram, st));
        AETH_TRY(chol_inverse(w.gram, cols, w.linv, fail ? fail : w.fail, st));
        // tmp = x Linv^T
        if (tc) {
            const int64_t xc = (int64_t)rows * cols, lc = (int64_t)cols * cols;
            f64_to_f32_kernel<<<grid_for(lc, 256), 256, 0, st>>>(w.linv, lc, w.linv32);
            AETH_TRY(split3_terms(w.linv32, lc, w.lt, st));
            AETH_TRY(split3_terms(x, xc, w.xt, st));
            // A = x K-major (rows x cols), B(k, j) = Linv[j][k]: K-major (cols x cols)
            AETH_TRY(terms_gemm(TermOp{w.xt, 3, xc, cols, false}, TermOp{w.lt, 3, lc, cols, false}, tmp, cols, rows,
                                cols, cols, false, st));
        } else {
            AETH_TRY((gemm_f64acc<float, double, float>(x, cols, 1, w.linv, 1, cols, tmp, cols, rows, cols, cols, st)));
        }
        AETH_CUDA(cudaMemcpyAsync(x, tmp, sizeof(float) * (size_t)rows * cols, cudaMemcpyDeviceToDevice, st));
    }
    return AETH_OK;
}

// The tensor-core refresh: every product of randomized_svd_projections on
// tcgen05 GEMMs over exact bf16 terms (split_gemm.cuh; G is its own single
// term when it is bf16), the orthonormal bases by Cholesky QR with f64 Gram
// matrices, the reference's Jacobi.  fp32-accurate products, not the
// reference's summation order.  Needs every pitch a multiple of 8 elements.
inline bool rsvd_fast_shape(int m, int n, int r, int l) { return m % 8 == 0 && n % 8 == 0 && r % 8 == 0 && l % 8 == 0; }

inline int rsvd_fast(const void* g, bool g_bf16, int m, int n, int r, int l, int power_iters, RsvdWork& w,
                     uint16_t* gt, uint16_t* at, uint16_t* bt, uint16_t* ut, float* p_out, float* q_out,
                     cudaStream_t st) {
    const int64_t mn = (int64_t)m * n;
    if (!g_bf16) AETH_TRY(split3_terms(static_cast<const float*>(g), mn, gt, st));
    const uint16_t* gterms = g_bf16 ? static_cast<const uint16_t*>(g) : gt;
    const int gk = g_bf16 ? 1 : 3;
    const TermOp G_k{gterms, gk, mn, n, false};   // G read K-major (A = G, K = n)
    const TermOp G_mn{gterms, gk, mn, n, true};   // G read MN-major (A = G^T or B = G, K = m)
    // 2. Y = G Omega (m x l)
    AETH_TRY(split3_terms(w.omega, (int64_t)n * l, at, st));
    AETH_TRY(terms_gemm(G_k, TermOp{at, 3, (int64_t)n * l, l, true}, w.y, l, m, l, n, false, st));
    // 3. Q^ = orthonormal basis of Y, optional power iterations.  The bases
    // between the power iterations only keep the iterates well conditioned:
    // one Cholesky QR pass each; the final Q^ gets the second pass.
    AETH_TRY(cholqr2(w.y, w.y2, m, l, w, st, nullptr, power_iters > 0 ? 1 : 2));
    for (int it = 0; it < power_iters; ++it) {
        // Z = G^T Q^ (n x l), orthonormalised; Y = G Z, orthonormalised
        AETH_TRY(split3_terms(w.y, (int64_t)m * l, at, st));
        AETH_TRY(terms_gemm(G_mn, TermOp{at, 3, (int64_t)m * l, l, true}, w.y2, l, n, l, m, false, st));
        AETH_TRY(cholqr2(w.y2, w.omega, n, l, w, st, nullptr, 1));
        AETH_TRY(split3_terms(w.y2, (int64_t)n * l, at, st));
        AETH_TRY(terms_gemm(G_k, TermOp{at, 3, (int64_t)n * l, l, true}, w.y, l, m, l, n, false, st));
        AETH_TRY(cholqr2(w.y, w.y2, m, l, w, st, nullptr, it + 1 == power_iters ? 2 : 1));
    }
    // 4. B = Q^T G (l x n): A = Q^T (Q^ read MN-major), B = G (MN-major), K = m
    AETH_TRY(split3_terms(w.y, (int64_t)m * l, at, st));
    AETH_TRY(terms_gemm(TermOp{at, 3, (int64_t)m * l, l, true}, G_mn, w.b, n, l, n, m, false, st));
    // 5. B B^T (l x l), K = n: both operands B read K-major; 6. Jacobi
    AETH_TRY(split3_terms(w.b, (int64_t)l * n, bt, st));
    const TermOp B_k{bt, 3, (int64_t)l * n, n, false};
    AETH_TRY(terms_gemm(B_k, B_k, w.bbt, l, l, l, n, false, st));
    jacobi50_kernel<<<1, 1024, 0, st>>>(w.bbt, l, w.u);
    AETH_LAUNCH_CHECK();
    // U[:, :r] compact (l x r), as terms
    AETH_CUDA(cudaMemcpy2DAsync(w.ur, sizeof(float) * r, w.u, sizeof(float) * l, sizeof(float) * r, l,
                                cudaMemcpyDeviceToDevice, st));
    AETH_TRY(split3_terms(w.ur, (int64_t)l * r, ut, st));
    const TermOp U_mn{ut, 3, (int64_t)l * r, r, true};
    // 7. P = Q^ U[:, :r] (A = Q^ K-major, K = l)
    if (p_out) AETH_TRY(terms_gemm(TermOp{at, 3, (int64_t)m * l, l, false}, U_mn, p_out, r, m, r, l, false, st));
    // 8. Q = B^T U[:, :r] (A = B^T: B read MN-major, K = l)
    if (q_out) AETH_TRY(terms_gemm(TermOp{bt, 3, (int64_t)l * n, n, true}, U_mn, q_out, r, n, r, l, false, st));
    return AETH_OK;
}

// randomized_svd_projections on the device, enqueued on `st` without waiting:
// g m x n, f32 or (g_bf16) bf16; p_out (m x r) and q_out (n x r) f32, either
// may be null.  fast selects the tensor-core products (rsvd_fast) when the
// shape allows; otherwise the exact-order CUDA-core GEMM reproduces the
// reference's f32 loops on equal inputs (a bf16 g is widened exactly first).
// *status_dev becomes 1 when the sketch is rank-deficient (the reference's
// GaLoreError::Linalg from qr_columns); the outputs are then meaningless.
// Q's orthonormalisation falls back to the reference's clamped Gram-Schmidt
// on the device when its Cholesky factorisation fails.  Workspace comes from
// the stream-ordered pool.  Returns AETH_ERR_CONFIG for an invalid rank or
// oversampling.
inline int rsvd_launch(const void* gin, bool g_bf16, int m, int n, int r, int oversampling, int power_iters,
                       uint64_t seed, bool fast, float* p_out, float* q_out, int* status_dev, cudaStream_t st,
                       const float* omega_in = nullptr) {
    const int l = r + oversampling;
    if (r <= 0 || oversampling < 0 || power_iters < 0 || l > (m < n ? m : n) || l > kJacobiMaxN) return AETH_ERR_CONFIG;
    fast = fast && rsvd_fast_shape(m, n, r, l);
    RsvdWork w;
    w.fail = status_dev;
    const size_t big = (size_t)(m > n ? m : n) * l;
    const int64_t mn = (int64_t)m * n;
    std::vector<void*> allocs;
    auto alloc = [&](void** p, size_t bytes) -> int {
        cudaError_t e = cudaMallocAsync(p, bytes, st);
        if (e != cudaSuccess) return set_err((int)e);
        allocs.push_back(*p);
        return AETH_OK;
    };
    int status = AETH_OK;
    uint16_t *gt = nullptr, *at = nullptr, *bt = nullptr, *ut = nullptr;
    float* qraw = nullptr;
    int* fail_q = nullptr;
    const float* g = static_cast<const float*>(gin);
    do {
        if ((status = alloc((void**)&w.omega, sizeof(float) * big)) ||
            (status = alloc((void**)&w.y, sizeof(float) * (size_t)m * l)) ||
            (status = alloc((void**)&w.y2, sizeof(float) * big)) ||
            (status = alloc((void**)&w.b, sizeof(float) * (size_t)l * n)) ||
            (status = alloc((void**)&w.bbt, sizeof(float) * (size_t)l * l)) ||
            (status = alloc((void**)&w.u, sizeof(float) * (size_t)l * l)) ||
            (status = alloc((void**)&w.ur, sizeof(float) * (size_t)l * r)) ||
            (status = alloc((void**)&w.gram, sizeof(double) * (size_t)l * l)) ||
            (status = alloc((void**)&w.gpart, sizeof(double) * kGramMaxChunks * (size_t)l * l)) ||
            (status = alloc((void**)&w.linv, sizeof(double) * (size_t)l * l)) ||
            (status = alloc((void**)&w.jump, sizeof(uint64_t) * 64 * kOmegaLevels)) ||
            (status = alloc((void**)&fail_q, sizeof(int))))
            break;
        if (q_out && (status = alloc((void**)&qraw, sizeof(float) * (size_t)n * r))) break;
        if (fast) {
            if ((!g_bf16 && (status = alloc((void**)&gt, sizeof(uint16_t) * 3 * (size_t)mn))) ||
                (status = alloc((void**)&at, sizeof(uint16_t) * 3 * big)) ||
                (status = alloc((void**)&bt, sizeof(uint16_t) * 3 * (size_t)l * n)) ||
                (status = alloc((void**)&ut, sizeof(uint16_t) * 3 * (size_t)l * r)) ||
                (status = alloc((void**)&w.xt, sizeof(uint16_t) * 3 * big)) ||
                (status = alloc((void**)&w.lt, sizeof(uint16_t) * 3 * (size_t)l * l)) ||
                (status = alloc((void**)&w.linv32, sizeof(float) * (size_t)l * l)))
                break;
        } else if (g_bf16) {
            // the exact path reads fp32: widen the bf16 gradient exactly
            float* gf = nullptr;
            if ((status = alloc((void**)&gf, sizeof(float) * (size_t)mn))) break;
            bf16_to_f32_rsvd_kernel<<<grid_for(mn, 256), 256, 0, st>>>(static_cast<const uint16_t*>(gin), mn, gf);
            g = gf;
        }
        cudaError_t e =
            cudaMemcpyAsync(w.jump, omega_jump_host(), sizeof(Gf2Mat64) * kOmegaLevels, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(fail_q, 0, sizeof(int), st);
        if (e != cudaSuccess) { status = set_err((int)e); break; }
        // 1. Omega (n x l), drawn here or the caller's
        const int64_t count = (int64_t)n * l;
        if (omega_in) {
            e = cudaMemcpyAsync(w.omega, omega_in, sizeof(float) * (size_t)count, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) { status = set_err((int)e); break; }
        } else {
            const int64_t chunks = (count + kOmegaChunk - 1) / kOmegaChunk;
            rsvd_omega_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(w.jump, seed > 1 ? seed : 1, count,
                                                                               w.omega);
        }
        if (fast) {
            if ((status = rsvd_fast(gin, g_bf16, m, n, r, l, power_iters, w, gt, at, bt, ut, p_out, q_out, st)))
                break;
        } else {
            // 2. Y = G Omega
            if ((status = simt_gemm_exact(g, n, 1, w.omega, l, 1, w.y, l, m, l, n, SIMT_STORE, 1.0f, nullptr, st)))
                break;
            // 3. Q^ = qr_columns(Y), the reference's Gram-Schmidt in its own order
            // (+ optional power iterations, each basis by the same Gram-Schmidt)
            mgs_exact_kernel<<<1, kMgsThreads, 0, st>>>(w.y, m, l, 1, w.fail);
            if ((status = cuda_status(cudaGetLastError()))) break;
            for (int it = 0; it < power_iters && status == AETH_OK; ++it) {
                // Z = G^T Q^ (n x l) into y2, orthonormalise, Y = G Z, orthonormalise
                if ((status = simt_gemm_exact(g, 1, n, w.y, l, 1, w.y2, l, n, l, m, SIMT_STORE, 1.0f, nullptr, st)))
                    break;
                mgs_exact_kernel<<<1, kMgsThreads, 0, st>>>(w.y2, n, l, 1, w.fail);
                if ((status = cuda_status(cudaGetLastError()))) break;
                if ((status = simt_gemm_exact(g, n, 1, w.y2, l, 1, w.y, l, m, l, n, SIMT_STORE, 1.0f, nullptr, st)))
                    break;
                mgs_exact_kernel<<<1, kMgsThreads, 0, st>>>(w.y, m, l, 1, w.fail);
                if ((status = cuda_status(cudaGetLastError()))) break;
            }
            if (status) break;
            // 4. B = Q^T G (l x n), 5. B B^T (l x l), 6. Jacobi
            if ((status = simt_gemm_exact(w.y, 1, l, g, n, 1, w.b, n, l, n, m, SIMT_STORE, 1.0f, nullptr, st))) break;
            if ((status = simt_gemm_exact(w.b, n, 1, w.b, 1, n, w.bbt, l, l, l, n, SIMT_STORE, 1.0f, nullptr, st)))
                break;
            jacobi50_kernel<<<1, 1024, 0, st>>>(w.bbt, l, w.u);
            AETH_LAUNCH_CHECK();
            // 7. P = Q^ U[:, :r]
            if (p_out &&
                (status = simt_gemm_exact(w.y, l, 1, w.u, l, 1, p_out, r, m, r, l, SIMT_STORE, 1.0f, nullptr, st)))
                break;
            // 8. Q = B^T U[:, :r]
            if (q_out &&
                (status = simt_gemm_exact(w.b, 1, n, w.u, l, 1, q_out, r, n, r, l, SIMT_STORE, 1.0f, nullptr, st)))
                break;
        }
        // 9. Q orthonormalised (orthonormalize_columns).  Exact path: the
        // reference's clamped Gram-Schmidt in its own order.  Tensor-core path:
        // Cholesky QR, or, where its Gram matrix is not positive definite, the
        // clamped Gram-Schmidt from B^T U again -- chosen on the device.
        if (q_out && !fast) {
            mgs_exact_kernel<<<1, kMgsThreads, 0, st>>>(q_out, n, r, 0, nullptr);
            if ((status = cuda_status(cudaGetLastError()))) break;
        } else if (q_out) {
            e = cudaMemcpyAsync(qraw, q_out, sizeof(float) * (size_t)n * r, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) { status = set_err((int)e); break; }
            if ((status = cholqr2(q_out, w.y2, n, r, w, st, fail_q))) break;
            copy_if_flag_kernel<<<grid_for((int64_t)n * r, 256), 256, 0, st>>>(qraw, q_out, (int64_t)n * r, fail_q);
            mgs_clamped_kernel<<<1, 1024, 0, st>>>(q_out, n, r, fail_q);
            AETH_LAUNCH_CHECK();
        }
    } while (false);
    for (void* p : allocs) cudaFreeAsync(p, st);
    return status;
}

// rsvd_launch, then waits on `st` for the factorisation status: returns
// AETH_ERR_LINALG for a rank-deficient sketch.
inline int rsvd_device(const void* gin, bool g_bf16, int m, int n, int r, int oversampling, int power_iters,
                       uint64_t seed, bool fast, float* p_out, float* q_out, cudaStream_t st,
                       const float* omega_in = nullptr) {
    int* flag = nullptr;
    AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&flag), sizeof(int), st));
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), st);
    int status = e == cudaSuccess ? AETH_OK : (int)e;
    if (status == AETH_OK)
        status = rsvd_launch(gin, g_bf16, m, n, r, oversampling, power_iters, seed, fast, p_out, q_out, flag, st,
                             omega_in);
    int h = 0;
    if (status == AETH_OK) {
        e = cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) status = (int)e;
    }
    cudaFreeAsync(flag, st);
    if (status == AETH_OK && h) status = AETH_ERR_LINALG;
    return status == AETH_OK ? AETH_OK : set_err(status);
}

}  // namespace aeth
