// Decima Weights mode (W8A32: int8 weights in blocks, f32 activations), Matrix::apply_with_rows
// with mode == Weights (decima/int8.rs:166-283).  The reference's arithmetic is a sequential f32
// chain per output, so the kernel keeps each output's accumulator in one thread and walks k in
// ascending order; the work is spread over outputs (64 x 64 tiles, 4 x 4 outputs per thread,
// k staged through shared memory 32 at a time).  CUDA cores, not tensor cores: no tensor-core
// reduction reproduces a single fma chain over k.
//   fused (the AVX2 kernel, decima/int8/weights_x86.rs:51-113): every weight decoded to the f32
//     product code * scale (:63-76), then sum = fma(x_k, w_k, sum) for k = 0..K-1 from 0 (:86-100);
//   portable (decima/int8.rs:384-407): per block dot += x_k * code_k (a multiply and an add), then
//     sum += dot * scale.
// Then y = sum + bias[n] (bias null: + 0).  A non-finite x raises *nonfinite; the host call then
// fills y with NaN (int8.rs:183-187).
#include "common.cuh"
#include "kernels.h"

namespace db {
namespace {

constexpr int W32_BM = 64, W32_BN = 64, W32_BK = 32, W32_THREADS = 256;

template <bool FUSED>
__global__ void __launch_bounds__(W32_THREADS)
    decima_w8a32_kernel(const float* __restrict__ x, int64_t ldx, int M, int K, const int8_t* __restrict__ wc,
                        int64_t ldw, const float* __restrict__ sw, int64_t ldsw, int N, int block,
                        const float* __restrict__ bias, float* __restrict__ y, int64_t ldy,
                        int* __restrict__ nonfinite) {
    __shared__ __align__(16) float xs[W32_BK][W32_BM + 4];  // k-major activation tile
    __shared__ __align__(16) float ws[W32_BK][W32_BN + 4];  // decoded weights (fused) or codes
    __shared__ float ss[W32_BN];                             // portable: the step's block scales
    pdl_wait();
    const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
    const int m0 = blockIdx.y * W32_BM, n0 = blockIdx.x * W32_BN;
    float acc[4][4], dot[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = dot[i][j] = 0.f;
    bool bad = false;
    for (int k0 = 0; k0 < K; k0 += W32_BK) {
        for (int i = tid; i < W32_BM * W32_BK; i += W32_THREADS) {
            const int r = i / W32_BK, kk = i % W32_BK, m = m0 + r, k = k0 + kk;
            const float v = (m < M && k < K) ? x[(size_t)m * ldx + k] : 0.f;
            bad |= !isfinite(v);
            xs[kk][r] = v;
        }
        for (int i = tid; i < W32_BN * W32_BK; i += W32_THREADS) {
            const int c = i / W32_BK, kk = i % W32_BK, n = n0 + c, k = k0 + kk;
            float v = 0.f;
            if (n < N && k < K) {
                v = (float)wc[(size_t)n * ldw + k];
                if (FUSED) v = __fmul_rn(v, sw[(size_t)(k / block) * ldsw + n]);
            }
            ws[kk][c] = v;
        }
        if (!FUSED)
            for (int i = tid; i < W32_BN; i += W32_THREADS)
                ss[i] = n0 + i < N ? sw[(size_t)(k0 / block) * ldsw + n0 + i] : 0.f;
        __syncthreads();
        const int kmax = min(W32_BK, K - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            const float4 a4 = *reinterpret_cast<const float4*>(&xs[kk][tm * 4]);
            const float4 w4 = *reinterpret_cast<const float4*>(&ws[kk][tn * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w}, w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (FUSED) acc[i][j] = __fmaf_rn(a[i], w[j], acc[i][j]);
                    else dot[i][j] = __fadd_rn(dot[i][j], __fmul_rn(a[i], w[j]));
                }
        }
        // portable: a block ends with this step (blocks are multiples of the 32-wide step) or at K
        if (!FUSED && ((k0 + W32_BK) % block == 0 || k0 + W32_BK >= K)) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(dot[i][j], ss[tn * 4 + j]));
                    dot[i][j] = 0.f;
                }
        }
        __syncthreads();
    }
    if (bad && nonfinite) atomicOr(nonfinite, 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tn * 4 + j;
            if (n < N) y[(size_t)m * ldy + n] = __fadd_rn(acc[i][j], bias ? bias[n] : 0.f);
        }
    }
}

}  // namespace
}  // namespace db

using namespace db;

// x f32 [M, ldx]; w codes int8 [N, ldw] (ldw >= K, the Q8 device layout of Matrix::new) with
// group-major scales [ceil(K / block), ldsw]; y f32 [M, ldy].  block 32, 64 or 128.
int db_launch_decima_w8a32(const float* x, int64_t ldx, int M, int K, const uint8_t* w_codes, int64_t ldw,
                           const float* sw, int64_t ldsw, int N, int block, int fused, const float* bias, float* y,
                           int64_t ldy, int* nonfinite, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return 0;
    if (K <= 0 || (block != 32 && block != 64 && block != 128) || ldx < K || ldw < K || ldy < N || ldsw < N)
        return (int)cudaErrorInvalidValue;
    const dim3 grid((unsigned)((N + W32_BN - 1) / W32_BN), (unsigned)((M + W32_BM - 1) / W32_BM));
    const int8_t* wc = reinterpret_cast<const int8_t*>(w_codes);
    const cudaError_t e =
        fused ? db_launch_pdl(decima_w8a32_kernel<true>, grid, dim3(W32_THREADS), 0, stream, x, ldx, M, K, wc, ldw, sw,
                              ldsw, N, block, bias, y, ldy, nonfinite)
              : db_launch_pdl(decima_w8a32_kernel<false>, grid, dim3(W32_THREADS), 0, stream, x, ldx, M, K, wc, ldw,
                              sw, ldsw, N, block, bias, y, ldy, nonfinite);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}
