// Elementwise / row kernels around the projections of one encoder layer:
//   rms_quantize   RMSNorm (cpu.rs:310-333) fused with the group-64 activation quantiser
//                  (int8.rs:178-202), writing tensor-core or GEMV code layouts
//   qk_norm_rope   per-head RMSNorm of q and k (backbone.rs:519-520) + rotate-half RoPE
//                  (backbone.rs:471-483) from a host-computed cos/sin table, f16 outputs
//   mean_pool      sequential mean over tokens of the final hidden rows
#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"

namespace db {

__device__ __forceinline__ int tc_pos(int k) {
    const int b = k & ~7, j = k & 7;
    return b + ((j & 3) << 1) + (j >> 2);  // stored order 0,4,1,5,2,6,3,7
}
__device__ __forceinline__ int gemv_pos(int k) {
    const int b = k & ~7, j = k & 7;
    return b + ((j & 1) << 2) + (j >> 1);  // stored order 0,2,4,6,1,3,5,7
}

// One warp per row; D % 128 == 0 and D <= 4096.  Each lane owns float4 columns 4l + 128j.
template <int VEC>
__global__ void rms_quantize_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w, int T,
                                    int D, float eps, int zero_centered, float* __restrict__ normed,
                                    int64_t ldn, void* __restrict__ codes, int layout, int64_t ldc,
                                    float* __restrict__ scales, int32_t* __restrict__ sums, int64_t lds,
                                    int* __restrict__ nonfinite) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const int t = warp;
    const int J = D / 128;
    float4 v[VEC];
    float ss = 0.f;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
        if (j < J) {
            v[j] = *reinterpret_cast<const float4*>(x + (size_t)t * ldx + 4 * lane + 128 * j);
            bad |= !(isfinite(v[j].x) && isfinite(v[j].y) && isfinite(v[j].z) && isfinite(v[j].w));
            ss = __fadd_rn(ss, __fmul_rn(v[j].x, v[j].x));
            ss = __fadd_rn(ss, __fmul_rn(v[j].y, v[j].y));
            ss = __fadd_rn(ss, __fmul_rn(v[j].z, v[j].z));
            ss = __fadd_rn(ss, __fmul_rn(v[j].w, v[j].w));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (__any_sync(0xffffffffu, bad) && lane == 0 && nonfinite) atomicOr(nonfinite, 1);
    const float scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
        if (j >= J) continue;
        const int c = 4 * lane + 128 * j;
        const float4 wv = *reinterpret_cast<const float4*>(w + c);
        float o[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        const float ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            o[i] = __fmul_rn(__fmul_rn(o[i], scale), zero_centered ? __fadd_rn(1.f, ww[i]) : ww[i]);
        if (normed) *reinterpret_cast<float4*>(normed + (size_t)t * ldn + c) = make_float4(o[0], o[1], o[2], o[3]);
        if (codes) {
            // group 2j (lanes 0-15) or 2j+1 (lanes 16-31): absmax over 16 lanes
            float amax = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
            for (int s = 8; s; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
            const float gs = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
            const float inv = __fdiv_rn(1.f, gs);
            int qs = 0;
            int qv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                qv[i] = (int)fminf(fmaxf(rintf(__fmul_rn(o[i], inv)), -127.f), 127.f);
                qs += qv[i];
            }
            const int g = c / DB_GROUP;
            if (layout == DB_CODES_TC_F16) {
                __half* dst = static_cast<__half*>(codes) + (size_t)t * ldc;
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[tc_pos(c + i)] = __int2half_rn(qv[i]);
            } else {
                int8_t* dst = static_cast<int8_t*>(codes) + (size_t)t * ldc;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    dst[layout == DB_CODES_GEMV_I8 ? gemv_pos(c + i) : c + i] = (int8_t)qv[i];
            }
#pragma unroll
            for (int s = 8; s; s >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, s);
            if ((lane & 15) == 0) {
                scales[(size_t)g * lds + t] = gs;
                if (sums) sums[(size_t)g * lds + t] = qs;
            }
        }
    }
}

// One warp per (token, head) of q or k; head_dim 128.  qkv row: [q heads | k heads | v heads].
// RoPE pairs (i, i+64); lane l holds dims 4l..4l+3, lanes 0-15 the first half.
__global__ void qk_norm_rope_kernel(const float* __restrict__ qkv, int64_t ld, int T, int Hq, int Hk,
                                    const float* __restrict__ qw, const float* __restrict__ kw, float eps,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                    __half* __restrict__ q16, __half* __restrict__ k16, __half* __restrict__ v16) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int heads = Hq + 2 * Hk;
    if (warp >= T * heads) return;
    const int t = warp / heads, h = warp % heads;
    const float* src = qkv + (size_t)t * ld + h * 128;
    float4 v = *reinterpret_cast<const float4*>(src + 4 * lane);
    if (h >= Hq + Hk) {  // value head: convert only
        __half* dst = v16 + ((size_t)t * Hk + (h - Hq - Hk)) * 128 + 4 * lane;
        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(v.x, v.y);
        *reinterpret_cast<__half2*>(dst + 2) = __floats2half2_rn(v.z, v.w);
        return;
    }
    const bool is_q = h < Hq;
    const float* w = is_q ? qw : kw;
    float ss = __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                         __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w)));
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.f), eps)));
    const float4 wv = *reinterpret_cast<const float4*>(w + 4 * lane);
    float o[4] = {__fmul_rn(__fmul_rn(v.x, scale), wv.x), __fmul_rn(__fmul_rn(v.y, scale), wv.y),
                  __fmul_rn(__fmul_rn(v.z, scale), wv.z), __fmul_rn(__fmul_rn(v.w, scale), wv.w)};
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, o[i], 16);  // partner dims +-64
    const int i0 = (4 * lane) & 63;
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float c = cos_t[(size_t)t * 64 + i0 + i], s = sin_t[(size_t)t * 64 + i0 + i];
        if (lane < 16) r[i] = __fsub_rn(__fmul_rn(o[i], c), __fmul_rn(p[i], s));  // a*c - b*s
        else r[i] = __fadd_rn(__fmul_rn(o[i], c), __fmul_rn(p[i], s));           // b*c + a*s
    }
    __half* dst = is_q ? q16 + ((size_t)t * Hq + h) * 128 : k16 + ((size_t)t * Hk + (h - Hq)) * 128;
    *reinterpret_cast<__half2*>(dst + 4 * lane) = __floats2half2_rn(r[0], r[1]);
    *reinterpret_cast<__half2*>(dst + 4 * lane + 2) = __floats2half2_rn(r[2], r[3]);
}

// pooled[d] = (sum over t, in order, of x[t, d]) / T
__global__ void mean_pool_kernel(const float* __restrict__ x, int64_t ldx, int T, int D, float* __restrict__ out) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    float s = 0.f;
    for (int t = 0; t < T; ++t) s = __fadd_rn(s, x[(size_t)t * ldx + d]);
    out[d] = __fdiv_rn(s, (float)T);
}

__global__ void fill_nan_if_kernel(float* __restrict__ y, int64_t n, const int* __restrict__ flag) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && *flag) y[i] = __int_as_float(0x7fc00000);
}

}  // namespace db

using namespace db;

int db_launch_rms_quantize(const float* x, int64_t ldx, const float* w, int T, int D, float eps, int zero_centered,
                           float* normed, int64_t ldn, void* codes, int layout, int64_t ldc, float* scales,
                           int32_t* sums, int64_t lds, int* nonfinite, cudaStream_t stream) {
    if (T <= 0) return 0;
    if (D % 128 || D > 4096) return (int)cudaErrorInvalidValue;
    const unsigned blocks = (unsigned)((T + 7) / 8);
    const int J = D / 128;
    if (J <= 8)
        rms_quantize_kernel<8><<<blocks, 256, 0, stream>>>(x, ldx, w, T, D, eps, zero_centered, normed, ldn, codes,
                                                           layout, ldc, scales, sums, lds, nonfinite);
    else
        rms_quantize_kernel<32><<<blocks, 256, 0, stream>>>(x, ldx, w, T, D, eps, zero_centered, normed, ldn, codes,
                                                            layout, ldc, scales, sums, lds, nonfinite);
    return (int)cudaGetLastError();
}

int db_launch_qk_norm_rope(const float* qkv, int64_t ld, int T, int Hq, int Hk, const float* qw, const float* kw,
                           float eps, const float* cos_t, const float* sin_t, __half* q16, __half* k16, __half* v16,
                           cudaStream_t stream) {
    if (T <= 0) return 0;
    const int64_t warps = (int64_t)T * (Hq + 2 * Hk);
    qk_norm_rope_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(qkv, ld, T, Hq, Hk, qw, kw, eps, cos_t,
                                                                          sin_t, q16, k16, v16);
    return (int)cudaGetLastError();
}

int db_launch_mean_pool(const float* x, int64_t ldx, int T, int D, float* out, cudaStream_t stream) {
    mean_pool_kernel<<<(D + 127) / 128, 128, 0, stream>>>(x, ldx, T, D, out);
    return (int)cudaGetLastError();
}

int db_launch_fill_nan_if(float* y, int64_t n, const int* flag, cudaStream_t stream) {
    if (n <= 0) return 0;
    fill_nan_if_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(y, n, flag);
    return (int)cudaGetLastError();
}
