// Small-M grouped GEMV (decode / scoring steps): weight bytes stream from HBM once.
//
// Numerics are those of the tensor-core path and of int8.rs:526-585: exact integer dots per
// 64-group (here dp4a), then acc = fma(float(dot_g), sw*sa, acc) in ascending g (or the
// portable sum += dot*(sa*sw) of int8.rs:276-278 / packed.rs:111 when fused == 0).
//
// Layout: one warp per output row n; lanes take 16-byte chunks of the row's codes (Q4: half a
// group, Q8: a quarter), compute integer partial dots for every activation row, reduce them
// across the lanes of a group, park them in shared memory, and then lanes 0..M-1 run the
// sequential per-group fold for their activation row.
#include "common.cuh"
#include "kernels.h"

namespace db {

constexpr int GEMV_MAX_ROWS = 8;
constexpr int GEMV_WARPS = 8;
constexpr int GEMV_MAX_GROUPS = 160;  // K <= 10240 (static smem: 8 warps x 8 rows x 160 x 4 B)

__device__ __forceinline__ int dp4a_su(int a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int BITS, int MR, bool FUSED, bool RESIDUAL>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
    gemv_kernel(const int8_t* __restrict__ a, int64_t lda, const float* __restrict__ sa,
                const int32_t* __restrict__ asum, int64_t ldsa, const uint8_t* __restrict__ w,
                const float* __restrict__ sw, int M, int N, int G, float* __restrict__ y, int64_t ldy,
                const int* __restrict__ nonfinite) {
    __shared__ int dots[GEMV_WARPS][MR][GEMV_MAX_GROUPS];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int n = blockIdx.x * GEMV_WARPS + warp;
    if (n >= N) return;
    constexpr int CHUNKS_PER_GROUP = BITS == 4 ? 2 : 4;  // 16-byte chunks per 64-code group
    const int chunks = G * CHUNKS_PER_GROUP;
    const int Kp = G * DB_GROUP;
    const uint4* wrow = reinterpret_cast<const uint4*>(w + (size_t)n * Kp * BITS / 8);
    for (int c0 = 0; c0 < chunks; c0 += 32) {
        const int c = c0 + lane;
        int part[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) part[r] = 0;
        const bool valid = c < chunks;
        if (valid) {
            const uint4 wv = __ldg(wrow + c);
            const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
            // this chunk covers codes k = c * (128 / BITS) .. +(128/BITS)-1 of the row
            const int k0 = c * (128 / BITS);
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                if (r < M) {
                    const int8_t* arow = a + (size_t)r * lda + k0;
                    if (BITS == 4) {
                        // 32 codes = 4 blocks of 8; A stored as (k0,k2,k4,k6),(k1,k3,k5,k7) per block
                        const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(arow));
                        const uint4 a1 = __ldg(reinterpret_cast<const uint4*>(arow + 16));
                        const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                        int s = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint32_t lo = words[b] & 0x0F0F0F0Fu;         // u(k0),u(k2),u(k4),u(k6)
                            const uint32_t hi = (words[b] >> 4) & 0x0F0F0F0Fu;  // u(k1),u(k3),u(k5),u(k7)
                            s = dp4a_su((int)av[2 * b], lo, s);
                            s = dp4a_su((int)av[2 * b + 1], hi, s);
                        }
                        part[r] = s;
                    } else {
                        // 16 codes = 2 blocks of 8, weights natural order
                        const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(arow));
                        const uint32_t av[4] = {a0.x, a0.y, a0.z, a0.w};
                        int s = 0;
#pragma unroll
                        for (int b = 0; b < 2; ++b) {
                            const uint32_t we = __byte_perm(words[2 * b], words[2 * b + 1], 0x6420);
                            const uint32_t wo = __byte_perm(words[2 * b], words[2 * b + 1], 0x7531);
                            s = dp4a_ss((int)av[2 * b], (int)we, s);
                            s = dp4a_ss((int)av[2 * b + 1], (int)wo, s);
                        }
                        part[r] = s;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            int v = part[r];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            if (CHUNKS_PER_GROUP == 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
            part[r] = v;
        }
        if (valid && (lane % CHUNKS_PER_GROUP) == 0) {
            const int g = c / CHUNKS_PER_GROUP;
#pragma unroll
            for (int r = 0; r < MR; ++r)
                if (r < M) {
                    int d = part[r];
                    if (BITS == 4) d -= 8 * __ldg(asum + (size_t)g * ldsa + r);  // codes were u = code + 8
                    dots[warp][r][g] = d;
                }
        }
    }
    __syncwarp();
    if (lane < M && lane < MR) {
        const int r = lane;
        float acc = 0.f;
        for (int g = 0; g < G; ++g) {
            const float d = (float)dots[warp][r][g];
            const float s_a = __ldg(sa + (size_t)g * ldsa + r);
            const float s_w = __ldg(sw + (size_t)g * db_scale_stride(N) + n);
            if (FUSED) acc = __fmaf_rn(d, __fmul_rn(s_w, s_a), acc);
            else acc = __fadd_rn(acc, __fmul_rn(d, __fmul_rn(s_a, s_w)));
        }
        float* dst = y + (size_t)r * ldy + n;
        if (RESIDUAL) acc = __fadd_rn(*dst, acc);
        if (nonfinite && *nonfinite) acc = __int_as_float(0x7fc00000);
        *dst = acc;
    }
}

template <int BITS, bool FUSED, bool RESIDUAL>
static void launch_rows(const DbGemvArgs& a, int G, cudaStream_t s) {
    dim3 grid((a.N + GEMV_WARPS - 1) / GEMV_WARPS);
    if (a.M <= 1)
        gemv_kernel<BITS, 1, FUSED, RESIDUAL><<<grid, GEMV_WARPS * 32, 0, s>>>(
            a.a_codes, a.lda, a.sa, a.a_sums, a.ldsa, a.w_codes, a.sw, a.M, a.N, G, a.y, a.ldy, a.nonfinite);
    else if (a.M <= 4)
        gemv_kernel<BITS, 4, FUSED, RESIDUAL><<<grid, GEMV_WARPS * 32, 0, s>>>(
            a.a_codes, a.lda, a.sa, a.a_sums, a.ldsa, a.w_codes, a.sw, a.M, a.N, G, a.y, a.ldy, a.nonfinite);
    else
        gemv_kernel<BITS, 8, FUSED, RESIDUAL><<<grid, GEMV_WARPS * 32, 0, s>>>(
            a.a_codes, a.lda, a.sa, a.a_sums, a.ldsa, a.w_codes, a.sw, a.M, a.N, G, a.y, a.ldy, a.nonfinite);
}

}  // namespace db

using namespace db;

int db_gemv_rows_limit() { return GEMV_MAX_ROWS; }

int db_launch_gemv(const DbGemvArgs& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.M > GEMV_MAX_ROWS || (a.bits != 4 && a.bits != 8)) return (int)cudaErrorInvalidValue;
    const int G = (a.K + DB_GROUP - 1) / DB_GROUP;
    if (G > GEMV_MAX_GROUPS) return (int)cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.a_codes) & 15) || (a.lda & 15) || (reinterpret_cast<uintptr_t>(a.w_codes) & 15))
        return (int)cudaErrorMisalignedAddress;
    if (a.bits == 4) {
        if (a.fused) a.residual ? launch_rows<4, true, true>(a, G, stream) : launch_rows<4, true, false>(a, G, stream);
        else a.residual ? launch_rows<4, false, true>(a, G, stream) : launch_rows<4, false, false>(a, G, stream);
    } else {
        if (a.fused) a.residual ? launch_rows<8, true, true>(a, G, stream) : launch_rows<8, true, false>(a, G, stream);
        else a.residual ? launch_rows<8, false, true>(a, G, stream) : launch_rows<8, false, false>(a, G, stream);
    }
    return (int)cudaGetLastError();
}
