// GQA attention with cached prefix keys and/or causal own keys (the decoder forms), head_dim 128,
// f16 operands with f32 accumulation and an online softmax (the reference computes scale * q.k,
// softmax, then P.v per head in f32: backbone.rs:560-600).  One CTA = 64 queries of one head,
// 4 warps x 16 query rows on mma.sync; K/V tiles of 64 keys double-buffered in 128B-swizzled
// shared memory via cp.async.  The plain non-causal calls run on the tcgen05 kernel of
// attention_tc.cu.
#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"

namespace db {

constexpr int ATT_BQ = 64, ATT_BKV = 64, ATT_D = 128;
constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE_BYTES = ATT_BKV * ATT_D * 2;  // 16 KB

// byte offset of (row, 16-byte chunk) in a [64][128] f16 tile, chunk XOR-swizzled by row
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
    return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

// 16-byte cp.async that zero-fills the bytes past src_bytes (rows past the sequence end).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// rows [t0, t0+64) of head h of a [T, H, 128] f16 tensor -> swizzled tile (rows >= T zero-filled)
__device__ __forceinline__ void load_tile(uint32_t dst, const __half* base, int T, int H, int h, int t0, int tid) {
#pragma unroll
    for (int i = 0; i < (ATT_BKV * 16) / ATT_THREADS; ++i) {
        const int idx = tid + i * ATT_THREADS;
        const int row = idx >> 4, chunk = idx & 15;
        const int t = t0 + row;
        const __half* src = base + ((size_t)(t < T ? t : T - 1) * H + h) * ATT_D + chunk * 8;
        cp_async16(dst + tile_off(row, chunk), src, t < T ? 16 : 0);
    }
}

// The context leaves as what the output projection consumes: quantised per 64-wide group with the activation quantiser (int8.rs:178-202, 305-391): f16 codes
// in tensor-core order [T, ldc] and scales [groups, lds] -- and raise *nonfinite on a non-finite
// value (the NaN guard of Matrix::apply, int8.rs:170-173).
__global__ void __launch_bounds__(ATT_THREADS)
    attention_kernel(const __half* __restrict__ q16, const __half* __restrict__ k16, const __half* __restrict__ v16,
                     int T, int Hq, int Hk, float scale_log2, void* __restrict__ codes, int64_t ldc,
                     float* __restrict__ scales, int64_t lds, int* __restrict__ nonfinite, const __half* __restrict__ kp,
                     const __half* __restrict__ vp, int P, int causal, int codes_i8) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sQ = smem_u32(smem);
    const uint32_t sK[2] = {sQ + ATT_TILE_BYTES, sQ + 2 * ATT_TILE_BYTES};
    const uint32_t sV[2] = {sQ + 3 * ATT_TILE_BYTES, sQ + 4 * ATT_TILE_BYTES};
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, kh = h / (Hq / Hk);
    const int q0 = blockIdx.x * ATT_BQ;
    // item blockIdx.z of a batch: its rows follow the previous items' in every row-indexed tensor
    const int64_t rb = (int64_t)blockIdx.z * T;
    q16 += rb * Hq * ATT_D;
    k16 += rb * Hk * ATT_D;
    v16 += rb * Hk * ATT_D;
    // key tiles: the P cached prefix keys first, then the item's own T keys (causal: only the
    // tiles that reach this query tile)
    const int tiles_p = (P + ATT_BKV - 1) / ATT_BKV, tiles_own_all = (T + ATT_BKV - 1) / ATT_BKV;
    const int tiles_own = causal ? min(tiles_own_all, (q0 + ATT_BQ + ATT_BKV - 1) / ATT_BKV) : tiles_own_all;
    const int tiles = tiles_p + tiles_own;
    auto load_kv = [&](int buf, int j) {
        if (j < tiles_p) {
            load_tile(sK[buf], kp, P, Hk, kh, j * ATT_BKV, tid);
            load_tile(sV[buf], vp, P, Hk, kh, j * ATT_BKV, tid);
        } else {
            load_tile(sK[buf], k16, T, Hk, kh, (j - tiles_p) * ATT_BKV, tid);
            load_tile(sV[buf], v16, T, Hk, kh, (j - tiles_p) * ATT_BKV, tid);
        }
    };

    load_tile(sQ, q16, T, Hq, h, q0, tid);
    load_kv(0, 0);
    cp_async_commit();

    uint32_t qf[8][4];
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

    for (int j = 0; j < tiles; ++j) {
        if (j + 1 < tiles) load_kv((j + 1) & 1, j + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (j == 0) {
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const int row = warp * 16 + (lane & 15), chunk = 2 * s + (lane >> 4);
                ldsm_x4(sQ + tile_off(row, chunk), qf[s][0], qf[s][1], qf[s][2], qf[s][3]);
            }
        }
        const uint32_t kb = sK[j & 1], vb = sV[j & 1];
        // S = Q K^T : 16 x 64 per warp
        float sc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                const int row = n * 8 + (lane & 7) + ((lane >> 4) << 3);
                const int chunk = 2 * s + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + tile_off(row, chunk), b0, b1, b2, b3);
                mma16816(sc[n], qf[s], b0, b1);
                mma16816(sc[n + 1], qf[s], b2, b3);
            }
        }
        // mask keys past the segment's end (and, causal, past the query), scale into the log2 domain
        const bool seg_p = j < tiles_p;
        const int kv0 = (seg_p ? j : j - tiles_p) * ATT_BKV, kend = seg_p ? P : T;
        const int qrow = q0 + warp * 16 + (lane >> 2);
        float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kv0 + n * 8 + 2 * (lane & 3) + (e & 1);
                const bool ok = key < kend && (seg_p || !causal || key <= qrow + ((e >> 1) << 3));
                float v = ok ? sc[n][e] * scale_log2 : -INFINITY;
                sc[n][e] = v;
                mx[e >> 1] = fmaxf(mx[e >> 1], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            corr[r] = mrow[r] == -INFINITY ? 0.f : exp2f(mrow[r] - mx[r]);
            mrow[r] = mx[r];
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = exp2f(sc[n][e] - mrow[e >> 1]);
                sc[n][e] = p;
                rs[e >> 1] += p;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            lrow[r] = lrow[r] * corr[r] + rs[r];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            o[i][0] *= corr[0]; o[i][1] *= corr[0];
            o[i][2] *= corr[1]; o[i][3] *= corr[1];
        }
        // O += P V
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t pa[4];
            pa[0] = pack_h2(sc[2 * s][0], sc[2 * s][1]);
            pa[1] = pack_h2(sc[2 * s][2], sc[2 * s][3]);
            pa[2] = pack_h2(sc[2 * s + 1][0], sc[2 * s + 1][1]);
            pa[3] = pack_h2(sc[2 * s + 1][2], sc[2 * s + 1][3]);
#pragma unroll
            for (int n = 0; n < 16; n += 2) {
                const int row = s * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int chunk = n + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + tile_off(row, chunk), b0, b1, b2, b3);
                mma16816(o[n], pa, b0, b1);
                mma16816(o[n + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }
    // normalise and store
    const float inv0 = 1.f / lrow[0], inv1 = 1.f / lrow[1];
    {
        // Rows r0 and r0 + 8 of this warp: 16 values per 64-wide group per thread, the rest of the
        // group on the other three lanes of the quad.  Codes go through shared memory (the Q tile,
        // free after the last iteration's barrier) -- f16 codes in the tensor-core order
        // k0,k4,k1,k5,k2,k6,k3,k7 of every 8 consecutive features, or int8 codes in natural order
        // (codes_i8) -- then out as 16-byte rows.
        const int q = lane & 3;
        // stored position of feature 2q in its 8-block, and the step to feature 2q + 1
        const int pos0 = codes_i8 ? 2 * q : (q < 2) ? 4 * q : 4 * (q - 2) + 1;
        const int pos1 = codes_i8 ? 1 : 2;
        bool bad = false;
#pragma unroll
        for (int grp = 0; grp < 2; ++grp) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const float inv = rr ? inv1 : inv0;
                float v[16];
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[2 * i] = o[grp * 8 + i][2 * rr] * inv;
                    v[2 * i + 1] = o[grp * 8 + i][2 * rr + 1] * inv;
                    amax = fmaxf(amax, fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1])));
                    bad |= !isfinite(v[2 * i]) || !isfinite(v[2 * i + 1]);
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                // group_scale (int8.rs:305-313) and pack_bits (int8.rs:347-360)
                const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                const float rinv = __fdiv_rn(1.f, scale);
                const int row = warp * 16 + (lane >> 2) + 8 * rr;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int col = grp * 64 + i * 8 + pos0;  // feature grp*64 + 8i + 2q and its neighbour
                    const float c0 = fminf(fmaxf(rintf(__fmul_rn(v[2 * i], rinv)), -127.f), 127.f);
                    const float c1 = fminf(fmaxf(rintf(__fmul_rn(v[2 * i + 1], rinv)), -127.f), 127.f);
                    if (codes_i8) {
                        reinterpret_cast<int8_t*>(smem)[row * ATT_D + col] = (int8_t)(int)c0;
                        reinterpret_cast<int8_t*>(smem)[row * ATT_D + col + pos1] = (int8_t)(int)c1;
                    } else {
                        reinterpret_cast<__half*>(smem)[row * ATT_D + col] = __float2half_rn(c0);
                        reinterpret_cast<__half*>(smem)[row * ATT_D + col + pos1] = __float2half_rn(c1);
                    }
                }
                const int t = q0 + row;
                if (q == 0 && t < T) scales[(size_t)(h * 2 + grp) * lds + rb + t] = scale;
            }
        }
        if (bad) atomicOr(nonfinite, 1);
        __syncthreads();
        // 64 rows x 256 bytes (f16) or 128 bytes (int8): 16-byte chunks, 16 or 8 per row
        if (codes_i8) {
#pragma unroll
            for (int i = 0; i < (ATT_BQ * 8) / ATT_THREADS; ++i) {
                const int idx = tid + i * ATT_THREADS;
                const int row = idx >> 3, chunk = idx & 7;
                const int t = q0 + row;
                if (t < T)
                    *reinterpret_cast<uint4*>(static_cast<int8_t*>(codes) + (size_t)(rb + t) * ldc + h * ATT_D +
                                              chunk * 16) = reinterpret_cast<const uint4*>(smem)[row * 8 + chunk];
            }
        } else {
#pragma unroll
            for (int i = 0; i < (ATT_BQ * 16) / ATT_THREADS; ++i) {
                const int idx = tid + i * ATT_THREADS;
                const int row = idx >> 4, chunk = idx & 15;
                const int t = q0 + row;
                if (t < T)
                    *reinterpret_cast<uint4*>(static_cast<__half*>(codes) + (size_t)(rb + t) * ldc + h * ATT_D +
                                              chunk * 8) = reinterpret_cast<const uint4*>(smem)[row * 16 + chunk];
            }
        }
    }
}

}  // namespace db

using namespace db;

int db_launch_attention(const __half* q16, const __half* k16, const __half* v16, int T, int Hq, int Hk, float scale,
                        float* out, int64_t ldo, cudaStream_t stream) {
    return db_launch_attention_tc(q16, k16, v16, 1, T, Hq, Hk, scale, out, ldo, nullptr, 0, nullptr, 0, nullptr,
                                  stream);
}

int db_launch_attention_quant(const __half* q16, const __half* k16, const __half* v16, int T, int Hq, int Hk,
                              float scale, void* codes, int64_t ldc, float* scales, int64_t lds, int* nonfinite,
                              cudaStream_t stream, int codes_i8) {
    if (!codes) return (int)cudaErrorInvalidValue;
    return db_launch_attention_tc(q16, k16, v16, 1, T, Hq, Hk, scale, nullptr, 0, codes, ldc, scales, lds, nonfinite,
                                  stream, codes_i8);
}

int db_launch_attention_prefix_quant(const __half* q16, const __half* k16, const __half* v16, int B, int T,
                                     const __half* kp, const __half* vp, int P, int causal, int Hq, int Hk,
                                     float scale, void* codes, int64_t ldc, float* scales, int64_t lds,
                                     int* nonfinite, cudaStream_t stream, int codes_i8) {
    if (T <= 0 || B <= 0) return 0;
    if (Hk <= 0 || Hq % Hk || !codes || !scales || !nonfinite || (ldc & (codes_i8 ? 15 : 7)) || P < 0 ||
        (P > 0 && (!kp || !vp)) || B > 65535)
        return (int)cudaErrorInvalidValue;
    const int smem = 5 * ATT_TILE_BYTES;
    {
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(attention_kernel), smem);
        if (e != cudaSuccess) return (int)e;
    }
    dim3 grid((T + ATT_BQ - 1) / ATT_BQ, Hq, B);
    attention_kernel<<<grid, ATT_THREADS, smem, stream>>>(q16, k16, v16, T, Hq, Hk, scale * 1.4426950408889634f,
                                                          codes, ldc, scales, lds, nonfinite, kp, vp, P, causal,
                                                          codes_i8);
    return (int)cudaGetLastError();
}
