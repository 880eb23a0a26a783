// Elementwise / row kernels around the projections of one encoder layer:
//   rms_quantize   RMSNorm (cpu.rs:310-333) fused with the group-64 activation quantiser
//                  (int8.rs:178-202), writing tensor-core, GEMV, natural or dequantised layouts
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

// One CTA per row, one float4 per thread (blockDim = D/4, D % 128 == 0, D <= 4096): short
// per-thread dependency chains and enough CTAs in flight to cover memory latency.
// normalize = 0 skips the RMSNorm (plain group-64 activation quantiser of int8.rs:178-202).
// Each warp covers 128 columns = two 64-groups (lanes 0-15, 16-31).  Code stores: lanes 2b and
// 2b+1 hold the two halves (k0..k3, k4..k7) of one 8-code block; they swap halves with one
// shuffle so each lane writes its part of the block's stored order with a single 8-byte
// (tensor-core f16 order) or 4-byte (GEMV int8 order) store.
// add0 / add1 (optional, [T, D] with row stride D): the two K-half partial sums of the projection
// that feeds the residual stream (dequantised mode); x = (x + add0) + add1 is written back to x
// first, then normalised as usual.
__global__ void rms_quantize_kernel(float* __restrict__ x, int64_t ldx, const float* __restrict__ w, int T,
                                    int D, float eps, int zero_centered, int normalize, float* __restrict__ normed,
                                    int64_t ldn, void* __restrict__ codes, int layout, int64_t ldc,
                                    float* __restrict__ scales, int32_t* __restrict__ sums, int64_t lds,
                                    int* __restrict__ nonfinite, const float* __restrict__ add0,
                                    const float* __restrict__ add1) {
    __shared__ float partial[32];
    pdl_wait();
    // dequantised layout: the next kernel is the projection's weight unpack, which reads nothing
    // this kernel writes; let it start while this one runs
    if (layout == DB_CODES_DQ_F16) pdl_trigger();
    const int t = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int c = 4 * threadIdx.x;
    float4 v = *reinterpret_cast<const float4*>(x + (size_t)t * ldx + c);
    if (add0) {
        const float4 p = *reinterpret_cast<const float4*>(add0 + (size_t)t * D + c);
        const float4 q = *reinterpret_cast<const float4*>(add1 + (size_t)t * D + c);
        v = make_float4(__fadd_rn(__fadd_rn(v.x, p.x), q.x), __fadd_rn(__fadd_rn(v.y, p.y), q.y),
                        __fadd_rn(__fadd_rn(v.z, p.z), q.z), __fadd_rn(__fadd_rn(v.w, p.w), q.w));
        *reinterpret_cast<float4*>(x + (size_t)t * ldx + c) = v;
    }
    const bool bad = !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
    if (__any_sync(0xffffffffu, bad) && lane == 0 && nonfinite) atomicOr(nonfinite, 1);
    float scale = 1.f;
    if (normalize) {
        float ss = __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                             __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w)));
#pragma unroll
        for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if (lane == 0) partial[wid] = ss;
        __syncthreads();
        if (wid == 0) {
            float tot = lane < (int)(blockDim.x >> 5) ? partial[lane] : 0.f;
#pragma unroll
            for (int o = 16; o; o >>= 1) tot = __fadd_rn(tot, __shfl_xor_sync(0xffffffffu, tot, o));
            if (lane == 0) partial[0] = tot;
        }
        __syncthreads();
        scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(partial[0], (float)D), eps)));
    }
    float o[4] = {v.x, v.y, v.z, v.w};
    if (normalize) {
        const float4 wv = *reinterpret_cast<const float4*>(w + c);
        const float ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            o[i] = __fmul_rn(__fmul_rn(o[i], scale), zero_centered ? __fadd_rn(1.f, ww[i]) : ww[i]);
    }
    if (normed) *reinterpret_cast<float4*>(normed + (size_t)t * ldn + c) = make_float4(o[0], o[1], o[2], o[3]);
    if (!codes) return;
    float amax = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
    for (int s2 = 8; s2; s2 >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s2));
    const float gs = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
    const float inv = __fdiv_rn(1.f, gs);
    int q[4], p[4];
    int qs = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q[i] = (int)fminf(fmaxf(rintf(__fmul_rn(o[i], inv)), -127.f), 127.f);
        qs += q[i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, q[i], 1);
    const bool odd = lane & 1;
    const int* lo = odd ? p : q;  // codes k0..k3 of the 8-code block
    const int* hi = odd ? q : p;  // codes k4..k7
    const int b8 = c & ~7;
    if (layout == DB_CODES_TC_F16) {
        // stored order k0,k4,k1,k5 | k2,k6,k3,k7
        const int e0 = odd ? 2 : 0;
        __half2 h0 = __halves2half2(__int2half_rn(lo[e0]), __int2half_rn(hi[e0]));
        __half2 h1 = __halves2half2(__int2half_rn(lo[e0 + 1]), __int2half_rn(hi[e0 + 1]));
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(static_cast<__half*>(codes) + (size_t)t * ldc + b8 + (odd ? 4 : 0)) = pk;
    } else if (layout == DB_CODES_DQ_F16) {
        // dequantised, natural order: f16(code * group scale) of k = c..c+3
        const __half2 h0 = __halves2half2(__float2half_rn(__fmul_rn((float)q[0], gs)), __float2half_rn(__fmul_rn((float)q[1], gs)));
        const __half2 h1 = __halves2half2(__float2half_rn(__fmul_rn((float)q[2], gs)), __float2half_rn(__fmul_rn((float)q[3], gs)));
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&h0);
        pk.y = *reinterpret_cast<const uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(static_cast<__half*>(codes) + (size_t)t * ldc + c) = pk;
    } else if (layout == DB_CODES_GEMV_I8) {
        // stored order k0,k2,k4,k6 | k1,k3,k5,k7
        const int e = odd ? 1 : 0;
        const uint32_t word = (uint32_t)(lo[e] & 255) | ((uint32_t)(lo[e + 2] & 255) << 8) |
                              ((uint32_t)(hi[e] & 255) << 16) | ((uint32_t)(hi[e + 2] & 255) << 24);
        *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(codes) + (size_t)t * ldc + b8 + (odd ? 4 : 0)) = word;
    } else {
        const uint32_t word = (uint32_t)(q[0] & 255) | ((uint32_t)(q[1] & 255) << 8) |
                              ((uint32_t)(q[2] & 255) << 16) | ((uint32_t)(q[3] & 255) << 24);
        *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(codes) + (size_t)t * ldc + c) = word;
    }
#pragma unroll
    for (int s2 = 8; s2; s2 >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, s2);
    if ((lane & 15) == 0) {
        const int g = c / DB_GROUP;
        scales[(size_t)g * lds + t] = gs;
        if (sums) sums[(size_t)g * lds + t] = qs;
    }
}

// One warp per (token, 4 consecutive heads); head_dim 128.  qkv row: [q heads | k heads | v heads].
// RoPE pairs (i, i+64); lane l holds dims 4l..4l+3 of a head, lanes 0-15 the first half.
constexpr int QK_HEADS_PER_WARP = 4;
__global__ void qk_norm_rope_kernel(const float* __restrict__ qkv, int64_t ld, int T, int Hq, int Hk,
                                    const float* __restrict__ qw, const float* __restrict__ kw, float eps,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                    __half* __restrict__ q16, __half* __restrict__ k16, __half* __restrict__ v16,
                                    int pos0, int seq_len, const int* __restrict__ positions) {
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int heads = Hq + 2 * Hk;
    const int units = (heads + QK_HEADS_PER_WARP - 1) / QK_HEADS_PER_WARP;
    if (warp >= T * units) return;
    const int t = warp / units, h0 = (warp % units) * QK_HEADS_PER_WARP;
    float4 v[QK_HEADS_PER_WARP];
#pragma unroll
    for (int u = 0; u < QK_HEADS_PER_WARP; ++u)
        if (h0 + u < heads) v[u] = *reinterpret_cast<const float4*>(qkv + (size_t)t * ld + (h0 + u) * 128 + 4 * lane);
    const int i0 = (4 * lane) & 63;
    // rows are seq_len-token items placed one after another, each starting at position pos0, or
    // carry their own positions (ragged sequences packed together)
    const size_t pos = positions ? (size_t)positions[t] : (size_t)(pos0 + t % seq_len);
    const float4 cs = *reinterpret_cast<const float4*>(cos_t + pos * 64 + i0);
    const float4 sn = *reinterpret_cast<const float4*>(sin_t + pos * 64 + i0);
    const float cc[4] = {cs.x, cs.y, cs.z, cs.w}, ssn[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
    for (int u = 0; u < QK_HEADS_PER_WARP; ++u) {
        const int h = h0 + u;
        if (h >= heads) break;
        if (h >= Hq + Hk) {  // value head: convert only
            __half* dst = v16 + ((size_t)t * Hk + (h - Hq - Hk)) * 128 + 4 * lane;
            __half2 a = __floats2half2_rn(v[u].x, v[u].y), b2 = __floats2half2_rn(v[u].z, v[u].w);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&a);
            pk.y = *reinterpret_cast<uint32_t*>(&b2);
            *reinterpret_cast<uint2*>(dst) = pk;
            continue;
        }
        const bool is_q = h < Hq;
        const float* w = is_q ? qw : kw;
        float ss = __fadd_rn(__fadd_rn(__fmul_rn(v[u].x, v[u].x), __fmul_rn(v[u].y, v[u].y)),
                             __fadd_rn(__fmul_rn(v[u].z, v[u].z), __fmul_rn(v[u].w, v[u].w)));
#pragma unroll
        for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        const float scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.f), eps)));
        const float4 wv = *reinterpret_cast<const float4*>(w + 4 * lane);
        float o[4] = {__fmul_rn(__fmul_rn(v[u].x, scale), wv.x), __fmul_rn(__fmul_rn(v[u].y, scale), wv.y),
                      __fmul_rn(__fmul_rn(v[u].z, scale), wv.z), __fmul_rn(__fmul_rn(v[u].w, scale), wv.w)};
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, o[i], 16);  // partner dims +-64
            if (lane < 16) r[i] = __fsub_rn(__fmul_rn(o[i], cc[i]), __fmul_rn(p, ssn[i]));  // a*c - b*s
            else r[i] = __fadd_rn(__fmul_rn(o[i], cc[i]), __fmul_rn(p, ssn[i]));           // b*c + a*s
        }
        __half* dst = is_q ? q16 + ((size_t)t * Hq + h) * 128 : k16 + ((size_t)t * Hk + (h - Hq)) * 128;
        __half2 a = __floats2half2_rn(r[0], r[1]), b2 = __floats2half2_rn(r[2], r[3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&a);
        pk.y = *reinterpret_cast<uint32_t*>(&b2);
        *reinterpret_cast<uint2*>(dst + 4 * lane) = pk;
    }
}

// pooled[d] = (sum over t, in order, of x[t, d]) / T
__global__ void mean_pool_kernel(const float* __restrict__ x, int64_t ldx, int T, int D, float* __restrict__ out) {
    pdl_wait();
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    float s = 0.f;
#pragma unroll 16
    for (int t = 0; t < T; ++t) s = __fadd_rn(s, x[(size_t)t * ldx + d]);
    out[d] = __fdiv_rn(s, (float)T);
}

// Mean over each ragged sequence's rows (rows cu[i]..cu[i+1]-1 -> out[i]), in row order as
// mean_pool_kernel sums a single sequence.
__global__ void mean_pool_varlen_kernel(const float* __restrict__ x, int64_t ldx, const int* __restrict__ cu, int D,
                                        float* __restrict__ out) {
    pdl_wait();
    const int d = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (d >= D) return;
    const int t0 = cu[i], t1 = cu[i + 1];
    float s = 0.f;
#pragma unroll 16
    for (int t = t0; t < t1; ++t) s = __fadd_rn(s, x[(size_t)t * ldx + d]);
    out[(size_t)i * D + d] = __fdiv_rn(s, (float)(t1 - t0));
}

__global__ void fill_nan_if_kernel(float* __restrict__ y, int64_t n, const int* __restrict__ flag) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && *flag) y[i] = __int_as_float(0x7fc00000);
}

}  // namespace db

using namespace db;

int db_launch_rms_quantize(const float* x, int64_t ldx, const float* w, int T, int D, float eps, int zero_centered,
                           float* normed, int64_t ldn, void* codes, int layout, int64_t ldc, float* scales,
                           int32_t* sums, int64_t lds, int* nonfinite, cudaStream_t stream, int normalize,
                           const float* add0, const float* add1) {
    if (T <= 0) return 0;
    if (D % 128 || D > 4096 || (add0 == nullptr) != (add1 == nullptr)) return (int)cudaErrorInvalidValue;
    // with add0 / add1 the kernel updates x in place (x is the caller's writable residual stream)
    const cudaError_t e = db_launch_pdl(rms_quantize_kernel, dim3(T), dim3(D / 4), 0, stream, const_cast<float*>(x), ldx,
                                        w, T, D, eps, zero_centered, normalize, normed, ldn, codes, layout, ldc, scales,
                                        sums, lds, nonfinite, add0, add1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int db_launch_mean_pool_varlen(const float* x, int64_t ldx, const int* cu_seqlens, int nseq, int D, float* out,
                               cudaStream_t stream) {
    if (nseq <= 0) return 0;
    const cudaError_t e = db_launch_pdl(mean_pool_varlen_kernel, dim3((D + 127) / 128, nseq), dim3(128), 0, stream, x,
                                        ldx, cu_seqlens, D, out);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int db_launch_qk_norm_rope(const float* qkv, int64_t ld, int T, int Hq, int Hk, const float* qw, const float* kw,
                           float eps, const float* cos_t, const float* sin_t, __half* q16, __half* k16, __half* v16,
                           cudaStream_t stream, int pos0, int seq_len, const int* positions) {
    if (T <= 0) return 0;
    const int64_t warps = (int64_t)T * ((Hq + 2 * Hk + QK_HEADS_PER_WARP - 1) / QK_HEADS_PER_WARP);
    const cudaError_t e = db_launch_pdl(qk_norm_rope_kernel, dim3((unsigned)((warps + 3) / 4)), dim3(128), 0, stream,
                                        qkv, ld, T, Hq, Hk, qw, kw, eps, cos_t, sin_t, q16, k16, v16, pos0,
                                        seq_len > 0 ? seq_len : T, positions);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int db_launch_mean_pool(const float* x, int64_t ldx, int T, int D, float* out, cudaStream_t stream) {
    const cudaError_t e = db_launch_pdl(mean_pool_kernel, dim3((D + 127) / 128), dim3(128), 0, stream, x, ldx, T, D, out);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int db_launch_fill_nan_if(float* y, int64_t n, const int* flag, cudaStream_t stream) {
    if (n <= 0) return 0;
    fill_nan_if_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(y, n, flag);
    return (int)cudaGetLastError();
}
