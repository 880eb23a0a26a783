// Group-64 quantisers, the device weight layout, and dequantisation.
//
// Device layout (this library's own, chosen for TMA and coalescing):
//   weight codes  Q4: [N, Kp/2] bytes, row n holds k = 0..Kp-1, low nibble = even k, nibble = code+8
//                      (the code bytes of reference packed.rs:22-28, without the interleaved scale)
//                 Q8: [N, Kp] int8
//   weight scales f32 [G, Ns], Ns = db_scale_stride(N) = roundup(N, 128), padding zero (group-major so
//                 that one group's scales for a tile of columns are one aligned bulk copy)
//   activation codes, tensor-core order: f16 integer values [M, Kp]; inside every 8 consecutive k
//                 the stored order is k = 0,4,1,5,2,6,3,7 (matches the nibble extraction of the GEMM)
//   activation codes, GEMV order: int8 [M, Kp]; inside every 8 consecutive k: 0,2,4,6,1,3,5,7
//   activation codes, natural order: int8 [M, Kp] (reference Scratch::values, int8.rs:7-11)
//   dequantised activations: f16 [M, Kp], natural order, f16(code * group scale)
//   activation scales f32 [G, lds] and code sums int32 [G, lds]; the tensor-core GEMM needs
//                 lds >= roundup(M, 128) and lds % 4 == 0 (bulk-copied per 128-row tile)
// Kp = ceil(K/64)*64; padding codes are 0 (nibble 8).
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace db {

__device__ __forceinline__ float load_as_f32(const void* x, int dtype, size_t i) {
    if (dtype == DB_F32) return static_cast<const float*>(x)[i];
    if (dtype == DB_F16) return __half2float(static_cast<const __half*>(x)[i]);
    return __uint_as_float((uint32_t) static_cast<const uint16_t*>(x)[i] << 16);  // bf16
}

__device__ __forceinline__ int code_position(int layout, int k) {
    int b = k & ~7, j = k & 7;
    if (layout == DB_CODES_TC_F16) {  // stored order 0,4,1,5,2,6,3,7 -> position of k
        const int pos[8] = {0, 2, 4, 6, 1, 3, 5, 7};
        return b + pos[j];
    }
    if (layout == DB_CODES_GEMV_I8) {  // stored order 0,2,4,6,1,3,5,7
        const int pos[8] = {0, 4, 1, 5, 2, 6, 3, 7};
        return b + pos[j];
    }
    return k;
}

// One warp per (row, group): int8.rs:178-202 (activation quantiser) for one 64-value group.
// scale = max(max|x| / limit, MIN_POSITIVE); code = clamp(rint(x * (1/scale)), +-limit).
__global__ void quantize_rows_kernel(const void* __restrict__ x, int dtype, int64_t ldx, int M, int K, int bits,
                                     void* __restrict__ codes, int layout, int64_t ldc, float* __restrict__ scales,
                                     int32_t* __restrict__ sums, int64_t lds, int* __restrict__ nonfinite) {
    int G = (K + DB_GROUP - 1) / DB_GROUP;
    int64_t warp = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (warp >= (int64_t)M * G) return;
    int m = (int)(warp / G), g = (int)(warp % G);
    int k0 = g * DB_GROUP + 2 * lane;
    float v0 = 0.f, v1 = 0.f;
    if (k0 < K) v0 = load_as_f32(x, dtype, (size_t)m * ldx + k0);
    if (k0 + 1 < K) v1 = load_as_f32(x, dtype, (size_t)m * ldx + k0 + 1);
    bool bad = !(isfinite(v0) && isfinite(v1));
    if (__any_sync(0xffffffffu, bad) && lane == 0 && nonfinite) atomicOr(nonfinite, 1);
    float limit = bits == 4 ? 7.f : 127.f;
    float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
    float scale = fmaxf(__fdiv_rn(amax, limit), FLT_MIN);
    float inv = __fdiv_rn(1.f, scale);
    float c0 = fminf(fmaxf(rintf(__fmul_rn(v0, inv)), -limit), limit);
    float c1 = fminf(fmaxf(rintf(__fmul_rn(v1, inv)), -limit), limit);
    if (k0 >= K) c0 = 0.f;
    if (k0 + 1 >= K) c1 = 0.f;
    if (layout == DB_CODES_TC_F16) {
        __half* out = static_cast<__half*>(codes) + (size_t)m * ldc;
        out[code_position(layout, k0)] = __float2half_rn(c0);
        out[code_position(layout, k0 + 1)] = __float2half_rn(c1);
    } else if (layout == DB_CODES_DQ_F16) {
        // dequantised: each code times its group scale, rounded to f16 (natural order)
        __half* out = static_cast<__half*>(codes) + (size_t)m * ldc;
        out[k0] = __float2half_rn(__fmul_rn((float)(int)c0, scale));  // a zero code is +0
        out[k0 + 1] = __float2half_rn(__fmul_rn((float)(int)c1, scale));
    } else {
        int8_t* out = static_cast<int8_t*>(codes) + (size_t)m * ldc;
        out[code_position(layout, k0)] = (int8_t)(int)c0;
        out[code_position(layout, k0 + 1)] = (int8_t)(int)c1;
    }
    if (lane == 0) scales[(size_t)g * lds + m] = scale;
    if (sums) {
        int s = warp_sum_i((int)c0 + (int)c1);
        if (lane == 0) sums[(size_t)g * lds + m] = s;
    }
}

// Weight quantiser, absmax (int8.rs:89-132 absmax branch; packed.rs:31-56): bf16 [N, K] -> device layout.
__global__ void pack_weights_kernel(const uint16_t* __restrict__ w, int N, int K, int bits,
                                    uint8_t* __restrict__ codes, float* __restrict__ scales,
                                    int* __restrict__ bad) {
    int G = (K + DB_GROUP - 1) / DB_GROUP, Kp = G * DB_GROUP;
    int64_t warp = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (warp >= (int64_t)N * G) return;
    int n = (int)(warp / G), g = (int)(warp % G);
    int k0 = g * DB_GROUP + 2 * lane;
    float v0 = k0 < K ? __uint_as_float((uint32_t)w[(size_t)n * K + k0] << 16) : 0.f;
    float v1 = k0 + 1 < K ? __uint_as_float((uint32_t)w[(size_t)n * K + k0 + 1] << 16) : 0.f;
    if (__any_sync(0xffffffffu, !(isfinite(v0) && isfinite(v1))) && lane == 0) atomicOr(bad, 1);
    float limit = bits == 4 ? 7.f : 127.f;
    float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
    float scale = fmaxf(__fdiv_rn(amax, limit), FLT_MIN);
    float inv = __fdiv_rn(1.f, scale);
    int c0 = (int)fminf(fmaxf(rintf(__fmul_rn(v0, inv)), -limit), limit);
    int c1 = (int)fminf(fmaxf(rintf(__fmul_rn(v1, inv)), -limit), limit);
    if (bits == 4) {
        codes[(size_t)n * (Kp / 2) + k0 / 2] = (uint8_t)((c0 + 8) | ((c1 + 8) << 4));
    } else {
        codes[(size_t)n * Kp + k0] = (uint8_t)(int8_t)c0;
        codes[(size_t)n * Kp + k0 + 1] = (uint8_t)(int8_t)c1;
    }
    if (lane == 0) scales[(size_t)g * db_scale_stride(N) + n] = scale;
}

// packed.rs:59-73 / quantized_rows.rs:89-110: out[t, k] = code(ids[t], k) * scale(ids[t], g).
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales, int N,
                                    int K, int bits, const int32_t* __restrict__ ids, int T,
                                    float* __restrict__ out, int64_t ldo, int* __restrict__ bad) {
    int Kp = (K + DB_GROUP - 1) / DB_GROUP * DB_GROUP;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * K) return;
    int t = (int)(i / K), k = (int)(i % K);
    int row = ids ? ids[t] : t;
    if (row < 0 || row >= N) {
        if (k == 0) atomicOr(bad, 1);
        out[(size_t)t * ldo + k] = __int_as_float(0x7fc00000);
        return;
    }
    int code;
    if (bits == 4) code = (int)((codes[(size_t)row * (Kp / 2) + k / 2] >> ((k & 1) * 4)) & 15) - 8;
    else code = (int)(int8_t)codes[(size_t)row * Kp + k];
    out[(size_t)t * ldo + k] = __fmul_rn((float)code, scales[(size_t)(k / DB_GROUP) * db_scale_stride(N) + row]);
}

// Reference packed rows (packed.rs:10-28: per (row, group) 32|64 code bytes then f32 scale) <-> device layout.
__global__ void packed_convert_kernel(uint8_t* __restrict__ packed, uint8_t* __restrict__ codes,
                                      float* __restrict__ scales, int N, int K, int bits, int to_device) {
    int G = K / DB_GROUP;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)N * G) return;
    int n = (int)(i / G), g = (int)(i % G);
    int cb = DB_GROUP * bits / 8;
    uint8_t* p = packed + ((size_t)n * G + g) * (cb + 4);
    uint8_t* c = codes + (size_t)n * G * cb + (size_t)g * cb;
    if (to_device) {
        for (int j = 0; j < cb; ++j) c[j] = p[j];
        float s;
        memcpy(&s, p + cb, 4);
        scales[(size_t)g * db_scale_stride(N) + n] = s;
    } else {
        for (int j = 0; j < cb; ++j) p[j] = c[j];
        float s = scales[(size_t)g * db_scale_stride(N) + n];
        memcpy(p + cb, &s, 4);
    }
}

// int8 natural / GEMV / tensor-core code layouts back to natural int8 (tests and export).
__global__ void codes_to_natural_kernel(const void* __restrict__ codes, int layout, int64_t ldc, int M, int Kp,
                                        int8_t* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)M * Kp) return;
    int m = (int)(i / Kp), k = (int)(i % Kp);
    int p = code_position(layout, k);
    if (layout == DB_CODES_TC_F16)
        out[i] = (int8_t)(int)__half2float(static_cast<const __half*>(codes)[(size_t)m * ldc + p]);
    else
        out[i] = static_cast<const int8_t*>(codes)[(size_t)m * ldc + p];
}

// Decima int8 quantiser (decima/int8.rs:413-418, used for weights by Matrix::new :106-151 and for
// activations by the per-row fill :239-253): blocks of `block` values (16/32/64/128, the last one
// partial), scale = max(max|x| / 127, MIN_POSITIVE), code = round-half-away-from-zero(x / scale)
// with a correctly rounded division, clamped to +-127.  One warp per (row, block).  Codes of the
// row's padding up to Kp = ceil(K/64)*64 are written as 0 by the warp of the last block.
// out_layout: DB_CODES_TC_F16 (f16 codes, tensor-core order) or DB_CODES_NATURAL_I8 (int8).
__global__ void decima_quantize_rows_kernel(const float* __restrict__ x, int64_t ldx, int M, int K, int block,
                                            void* __restrict__ codes, int layout, int64_t ldc,
                                            float* __restrict__ scales, int64_t lds, bool row_major_scales,
                                            int* __restrict__ nonfinite) {
    const int G = (K + block - 1) / block, Kp = (K + DB_GROUP - 1) / DB_GROUP * DB_GROUP;
    const int64_t warp = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (warp >= (int64_t)M * G) return;
    const int m = (int)(warp / G), g = (int)(warp % G);
    const int k0 = g * block, per = (block + 31) / 32;  // values per lane (1..4)
    float v[4];
    float amax = 0.f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int k = k0 + lane + 32 * i;
        v[i] = (i < per && lane + 32 * i < block && k < K) ? x[(size_t)m * ldx + k] : 0.f;
        bad |= !isfinite(v[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0 && nonfinite) atomicOr(nonfinite, 1);
    amax = warp_max(amax);
    const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
    auto put = [&](int k, float c) {
        if (layout == DB_CODES_TC_F16)
            static_cast<__half*>(codes)[(size_t)m * ldc + code_position(layout, k)] = __float2half_rn(c);
        else
            static_cast<int8_t*>(codes)[(size_t)m * ldc + k] = (int8_t)(int)c;
    };
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int k = k0 + lane + 32 * i;
        if (i < per && lane + 32 * i < block && k < Kp) {
            const float c = k < K ? fminf(fmaxf(roundf(__fdiv_rn(v[i], scale)), -127.f), 127.f) : 0.f;
            put(k, c);
        }
    }
    if (g == G - 1)
        for (int k = G * block + lane; k < Kp; k += 32) put(k, 0.f);
    if (lane == 0) {
        if (row_major_scales) scales[(size_t)m * lds + g] = scale;
        else scales[(size_t)g * lds + m] = scale;
    }
}

}  // namespace db

using namespace db;

static inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

int db_launch_decima_quantize(const float* x, int64_t ldx, int M, int K, int block, void* codes, int layout,
                              int64_t ldc, float* scales, int64_t lds, int row_major_scales, int* nonfinite,
                              cudaStream_t stream) {
    if (M <= 0 || K <= 0) return 0;
    if (block != 16 && block != 32 && block != 64 && block != 128) return (int)cudaErrorInvalidValue;
    const int64_t warps = (int64_t)M * ((K + block - 1) / block);
    decima_quantize_rows_kernel<<<blocks_for(warps, 8), 256, 0, stream>>>(x, ldx, M, K, block, codes, layout, ldc,
                                                                            scales, lds, row_major_scales != 0,
                                                                            nonfinite);
    return (int)cudaGetLastError();
}

int db_launch_quantize_rows(const void* x, int dtype, int64_t ldx, int M, int K, int bits, void* codes, int layout,
                            int64_t ldc, float* scales, int32_t* sums, int64_t lds, int* nonfinite,
                            cudaStream_t stream) {
    if (M <= 0 || K <= 0) return 0;
    int G = (K + DB_GROUP - 1) / DB_GROUP;
    int64_t warps = (int64_t)M * G;
    quantize_rows_kernel<<<blocks_for(warps, 8), 256, 0, stream>>>(x, dtype, ldx, M, K, bits, codes, layout, ldc,
                                                                     scales, sums, lds, nonfinite);
    return (int)cudaGetLastError();
}

int db_launch_pack_weights(const uint16_t* w, int N, int K, int bits, uint8_t* codes, float* scales, int* bad,
                           cudaStream_t stream) {
    int G = (K + DB_GROUP - 1) / DB_GROUP;
    int Kp = G * DB_GROUP;
    size_t code_bytes = (size_t)N * Kp * bits / 8;
    cudaMemsetAsync(codes, bits == 4 ? 0x88 : 0, code_bytes, stream);  // padding codes = 0
    cudaMemsetAsync(scales, 0, (size_t)G * db_scale_stride(N) * sizeof(float), stream);  // padding scales = 0
    int64_t warps = (int64_t)N * G;
    pack_weights_kernel<<<blocks_for(warps, 8), 256, 0, stream>>>(w, N, K, bits, codes, scales, bad);
    return (int)cudaGetLastError();
}

int db_launch_dequant_rows(const uint8_t* codes, const float* scales, int N, int K, int bits, const int32_t* ids,
                           int T, float* out, int64_t ldo, int* bad, cudaStream_t stream) {
    int64_t n = (int64_t)T * K;
    if (n == 0) return 0;
    dequant_rows_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(codes, scales, N, K, bits, ids, T, out, ldo, bad);
    return (int)cudaGetLastError();
}

int db_launch_packed_convert(uint8_t* packed, uint8_t* codes, float* scales, int N, int K, int bits, int to_device,
                             cudaStream_t stream) {
    int64_t n = (int64_t)N * (K / DB_GROUP);
    if (to_device) cudaMemsetAsync(scales, 0, (size_t)(K / DB_GROUP) * db_scale_stride(N) * sizeof(float), stream);
    packed_convert_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(packed, codes, scales, N, K, bits, to_device);
    return (int)cudaGetLastError();
}

int db_launch_codes_to_natural(const void* codes, int layout, int64_t ldc, int M, int Kp, int8_t* out,
                               cudaStream_t stream) {
    int64_t n = (int64_t)M * Kp;
    codes_to_natural_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(codes, layout, ldc, M, Kp, out);
    return (int)cudaGetLastError();
}
