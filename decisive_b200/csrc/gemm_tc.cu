// Tensor-core grouped W4A8 / W8A8 GEMM with fused group dequantisation (sm_100a, tcgen05).
//
// Computes, for every output (m, n), the reference's grouped sum (int8.rs:526-585):
//     acc = 0; for g ascending: acc = fma(float(dot_g), sw[n,g] * sa[m,g], acc)
// where dot_g is the exact integer dot of 64 activation codes with 64 weight codes.
//
// The integer dots come from tcgen05.mma kind::f16 on integer-valued f16 operands: every code
// is exact in f16, every product and every partial sum of one group (|sum| <= 64*127*127 < 2^24)
// is an exact f32 integer, so the tensor core returns dot_g exactly.  Each 64-wide group is one
// K-block; its dot lands in its own TMEM buffer (double buffered) and the epilogue warps fold it
// into their register accumulators with the reference's rounding, in group order.
//
// Roles (448 threads, one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: activation-code tiles (128 x 64 f16, 128B swizzle) and raw weight
//               code tiles (BN rows x 32|64 bytes) into smem rings
//   warp 1      TMEM owner + MMA issuer (one elected lane): 4 x (128 x BN x 16) MMAs per group
//   warps 2-5   converters: weight nibbles/bytes -> f16 codes in the UMMA K-major SW128 layout
//   warps 6-13  epilogue: TMEM -> registers, per-group scale fold, final store / fused SwiGLU
//               re-quantisation (grouped_q4_mlp.wgsl:83-105 semantics)
// Every mbarrier wait is bounded (DB_WAIT_LIMIT_NS); on expiry the CTA records an error in the
// device error word, stops issuing work, and releases its tensor memory.
#include <float.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace db {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int B_STAGES = 3;   // converted f16 weight tiles (converter -> MMA)
constexpr int NUM_ACC = 4;    // TMEM accumulator buffers (NUM_ACC x BN columns <= 512)
// Warp roles: 0 = TMA producer, 1 = MMA issuer, then the converters, then 8 epilogue warps.
#ifndef DB_GEMM_CONVERTER_WARPS
#define DB_GEMM_CONVERTER_WARPS 2
#endif
constexpr int CONVERTER_WARP0 = 2;
constexpr int CONVERTER_WARPS = DB_GEMM_CONVERTER_WARPS;
constexpr int EPILOGUE_WARP0 = CONVERTER_WARP0 + CONVERTER_WARPS;
constexpr int EPILOGUE_WARPS = 8;
constexpr int NUM_THREADS = 32 * (EPILOGUE_WARP0 + EPILOGUE_WARPS);
constexpr int XCH_STRIDE = 65;  // floats per row of the SwiGLU exchange buffer (bank-conflict free)

// One pipeline stage per 64-wide K group holds everything the group needs: the activation-code
// tile, the raw weight-code tile and the group's scale vectors.  The epilogue is the last
// consumer of every part, so it alone releases the stage; the producer issues one wait, one
// expect-tx and four copies per group.
template <int BN, int BITS, int EPI>
struct GemmSmem {
    static constexpr int STAGES = BITS == 4 ? 6 : 5;
    static constexpr int A_BYTES = BM * BK * 2;          // 16 KB
    static constexpr int W_ROW = BK * BITS / 8;          // 32 or 64 bytes of raw codes per row
    static constexpr int W_BYTES = BN * W_ROW;
    static constexpr int SC_BYTES = (BM + BN) * 4;       // sa then sw of the group
    static constexpr int ST_A = 0, ST_W = A_BYTES, ST_S = A_BYTES + W_BYTES;
    static constexpr int STAGE_BYTES = (ST_S + SC_BYTES + 1023) / 1024 * 1024;
    static constexpr int TX_BYTES = A_BYTES + W_BYTES + SC_BYTES;
    static constexpr int B_BYTES = BN * BK * 2;          // f16 codes
    static constexpr int XCH_BYTES = EPI == DB_EPI_SWIGLU_QUANT ? BM * XCH_STRIDE * 4 : 0;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_B = OFF_STAGE + STAGES * STAGE_BYTES;
    static constexpr int OFF_X = OFF_B + B_STAGES * B_BYTES;
    static constexpr int OFF_BAR = (OFF_X + XCH_BYTES + 15) / 16 * 16;
    static constexpr int NUM_BARS = 2 * STAGES + 2 * B_STAGES + 2 * NUM_ACC + 2;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
    static_assert(BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
    bool ok = mbar_wait(bar, parity, abort_flag, err, code);
    return __all_sync(0xffffffffu, ok);
}

// 8 weight nibbles (bytes of one row, k = 8c..8c+7) -> 8 f16 codes in the order 0,4,1,5,2,6,3,7.
__device__ __forceinline__ uint4 nibbles_to_f16(uint32_t w) {
    const uint32_t magic = 0x64006400u;
    uint32_t t0 = (w & 0x000F000Fu) | magic;         // 1024+u(k0), 1024+u(k4)
    uint32_t t1 = (w & 0x00F000F0u) | magic;         // 1024+16u(k1), 1024+16u(k5)
    uint32_t w8 = w >> 8;
    uint32_t t2 = (w8 & 0x000F000Fu) | magic;        // k2, k6
    uint32_t t3 = (w8 & 0x00F000F0u) | magic;        // k3, k7
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));   // 1032
    const __half2 sixteenth = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
    const __half2 m72 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));        // -72
    __half2 o0 = __hsub2(*reinterpret_cast<__half2*>(&t0), bias);
    __half2 o1 = __hfma2(*reinterpret_cast<__half2*>(&t1), sixteenth, m72);
    __half2 o2 = __hsub2(*reinterpret_cast<__half2*>(&t2), bias);
    __half2 o3 = __hfma2(*reinterpret_cast<__half2*>(&t3), sixteenth, m72);
    uint4 r;
    r.x = *reinterpret_cast<uint32_t*>(&o0);
    r.y = *reinterpret_cast<uint32_t*>(&o1);
    r.z = *reinterpret_cast<uint32_t*>(&o2);
    r.w = *reinterpret_cast<uint32_t*>(&o3);
    return r;
}

// 8 int8 weight codes (k = 8c..8c+3 in w0, 8c+4..8c+7 in w1) -> f16 codes in order 0,4,1,5,2,6,3,7.
__device__ __forceinline__ uint4 bytes_to_f16(uint32_t w0, uint32_t w1) {
    uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;  // code + 128, unsigned
    uint32_t p = __byte_perm(x0, x1, 0x5140);              // k0 k4 k1 k5
    uint32_t q = __byte_perm(x0, x1, 0x7362);              // k2 k6 k3 k7
    const uint32_t hi = 0x64646464u;
    uint32_t t0 = __byte_perm(p, hi, 0x4140), t1 = __byte_perm(p, hi, 0x4342);
    uint32_t t2 = __byte_perm(q, hi, 0x4140), t3 = __byte_perm(q, hi, 0x4342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    __half2 o0 = __hsub2(*reinterpret_cast<__half2*>(&t0), bias);
    __half2 o1 = __hsub2(*reinterpret_cast<__half2*>(&t1), bias);
    __half2 o2 = __hsub2(*reinterpret_cast<__half2*>(&t2), bias);
    __half2 o3 = __hsub2(*reinterpret_cast<__half2*>(&t3), bias);
    uint4 r;
    r.x = *reinterpret_cast<uint32_t*>(&o0);
    r.y = *reinterpret_cast<uint32_t*>(&o1);
    r.z = *reinterpret_cast<uint32_t*>(&o2);
    r.w = *reinterpret_cast<uint32_t*>(&o3);
    return r;
}

__device__ __forceinline__ float silu_ref(float x) {
    // cpu.rs:513-518: x * (1 / (1 + exp(-x)))
    return __fmul_rn(x, __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x))));
}

// Epilogue helpers: one warp owns 32 rows (its TMEM lane quadrant) x COLS columns of the tile.
template <int COLS>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, uint32_t (&v)[COLS]) {
#pragma unroll
    for (int c = 0; c < COLS / 32; ++c)
        tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
}
template <int COLS>
__device__ __forceinline__ void tmem_wait_cols(uint32_t (&v)[COLS]) {
    tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(&v[0]));
#pragma unroll
    for (int c = 1; c < COLS / 32; ++c) {
        uint32_t(&w)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]);
        asm volatile(""
                     : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3]), "+r"(w[4]), "+r"(w[5]), "+r"(w[6]),
                       "+r"(w[7]), "+r"(w[8]), "+r"(w[9]), "+r"(w[10]), "+r"(w[11]), "+r"(w[12]), "+r"(w[13]),
                       "+r"(w[14]), "+r"(w[15]), "+r"(w[16]), "+r"(w[17]), "+r"(w[18]), "+r"(w[19]), "+r"(w[20]),
                       "+r"(w[21]), "+r"(w[22]), "+r"(w[23]), "+r"(w[24]), "+r"(w[25]), "+r"(w[26]), "+r"(w[27]),
                       "+r"(w[28]), "+r"(w[29]), "+r"(w[30]), "+r"(w[31]));
    }
}
// acc[j] = fma(d[j], sw[j]*sa, acc[j]) (fused) or acc[j] + d[j]*(sa*sw[j]) (portable).  Scalar
// FMUL/FFMA: on this part the packed f32x2 forms run at a lower element rate than scalar FFMA.
template <int COLS, bool FUSED>
__device__ __forceinline__ void fold_group(float2 (&acc)[COLS / 2], const uint32_t (&v)[COLS], const float* swp,
                                           float s_a) {
#pragma unroll
    for (int j = 0; j < COLS; j += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(swp + j);
        const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float& a = (e & 1) ? acc[(j + e) / 2].y : acc[(j + e) / 2].x;
            const float d = __uint_as_float(v[j + e]);
            if (FUSED) a = __fmaf_rn(d, __fmul_rn(w[e], s_a), a);
            else a = __fadd_rn(a, __fmul_rn(d, __fmul_rn(s_a, w[e])));
        }
    }
}

template <int BN, int BITS, int EPI, bool FUSED>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const float* __restrict__ sa, int64_t ldsa, const float* __restrict__ sw, int64_t ldsw, int M,
                   int N, int G, float* __restrict__ y, int64_t ldy, __half* __restrict__ out_codes, int64_t ldoc,
                   float* __restrict__ out_scales, int64_t ldos, const int* __restrict__ nonfinite,
                   int* __restrict__ dev_error) {
    using S = GemmSmem<BN, BITS, EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* full = bars;                   // stage loaded (TMA tx)
    uint64_t* empty = full + S::STAGES;      // stage released by the epilogue warps
    uint64_t* b_full = empty + S::STAGES;    // converted weight tile ready
    uint64_t* b_empty = b_full + B_STAGES;   // converted tile consumed by the MMA
    uint64_t* acc_full = b_empty + B_STAGES;
    uint64_t* acc_empty = acc_full + NUM_ACC;
    uint64_t* xch_full = acc_empty + NUM_ACC;  // SwiGLU exchange: up half -> gate half
    uint64_t* xch_empty = xch_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S::STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], EPILOGUE_WARPS); }
        for (int i = 0; i < B_STAGES; ++i) { mbar_init(&b_full[i], CONVERTER_WARPS); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < NUM_ACC; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPILOGUE_WARPS); }
        mbar_init(xch_full, 4);
        mbar_init(xch_empty, 4);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, NUM_ACC * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int is = 0;
            uint32_t ps = 0;
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
                for (int g = 0; g < G; ++g) {
                    if (!mbar_wait(&empty[is], ps ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_TMA)) goto done;
                    uint8_t* st = smem + S::OFF_STAGE + is * S::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[is], S::TX_BYTES);
                    tma_load_2d(st + S::ST_A, &tmA, &full[is], g * BK, m0);
                    tma_load_2d(st + S::ST_W, &tmW, &full[is], g * S::W_ROW, n0);
                    bulk_load(st + S::ST_S, sa + (size_t)g * ldsa + m0, BM * 4, &full[is]);
                    bulk_load(st + S::ST_S + BM * 4, sw + (size_t)g * ldsw + n0, BN * 4, &full[is]);
                    if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_f16_f32(BM, BN);
            int is = 0, ib = 0, ic = 0;
            uint32_t ps = 0, pb = 0, pc = 0;
            const uint32_t st_base = smem_u32(smem + S::OFF_STAGE), b_base = smem_u32(smem + S::OFF_B);
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                for (int g = 0; g < G; ++g) {
                    if (!mbar_wait(&full[is], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA)) goto done;
                    if (!mbar_wait(&b_full[ib], pb, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA)) goto done;
                    if (!mbar_wait(&acc_empty[ic], pc ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA)) goto done;
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(ic * BN);
                    const uint32_t a_addr = st_base + is * S::STAGE_BYTES + S::ST_A, b_addr = b_base + ib * S::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_f16(d, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC, kk > 0);
                    umma_commit(&b_empty[ib]);
                    umma_commit(&acc_full[ic]);
                    if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                    if (++ib == B_STAGES) { ib = 0; pb ^= 1u; }
                    if (++ic == NUM_ACC) { ic = 0; pc ^= 1u; }
                }
            }
        }
    } else if (warp < EPILOGUE_WARP0) {
        // ---------------------------------------------------------------- converters
        const int ct = threadIdx.x - CONVERTER_WARP0 * 32;
        int is = 0, ib = 0;
        uint32_t ps = 0, pb = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            for (int g = 0; g < G; ++g) {
                if (!warp_wait(&full[is], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_CVT)) goto done;
                if (!warp_wait(&b_empty[ib], pb ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_CVT)) goto done;
                const uint8_t* wsrc = smem + S::OFF_STAGE + is * S::STAGE_BYTES + S::ST_W;
                uint8_t* bdst = smem + S::OFF_B + ib * S::B_BYTES;
#pragma unroll
                for (int r = ct; r < BN; r += CONVERTER_WARPS * 32) {
                    const uint4* src = reinterpret_cast<const uint4*>(wsrc + r * S::W_ROW);
                    uint8_t* row = bdst + r * 128;
                    const int swz = r & 7;
                    if (BITS == 4) {
                        const uint4 v0 = src[0], v1 = src[1];
                        const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4*>(row + ((c ^ swz) << 4)) = nibbles_to_f16(words[c]);
                    } else {
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            const uint4 v = src[h];
                            *reinterpret_cast<uint4*>(row + (((2 * h) ^ swz) << 4)) = bytes_to_f16(v.x, v.y);
                            *reinterpret_cast<uint4*>(row + (((2 * h + 1) ^ swz) << 4)) = bytes_to_f16(v.z, v.w);
                        }
                    }
                }
                // generic writes of the B tile become MMA (async proxy) reads
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[ib]);
                if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                if (++ib == B_STAGES) { ib = 0; pb ^= 1u; }
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        // Software pipeline over 32-column chunks: the TMEM load of the next chunk (of this group
        // or of the next group) is in flight while the current chunk is folded; a TMEM buffer is
        // released as soon as all of its chunks sit in registers.
        constexpr int COLS = BN / 2;  // columns per thread
        constexpr int CHUNKS = COLS / 32;
        const int q = warp & 3;                         // TMEM lane quadrant this warp may access
        const int half = (warp - EPILOGUE_WARP0) >> 2;  // which half of the tile's columns
        const int r = q * 32 + lane;                    // row inside the tile
        const int col0 = half * COLS;
        const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
        const bool any_nonfinite = nonfinite != nullptr && *nonfinite != 0;
        float* xch = reinterpret_cast<float*>(smem + S::OFF_X);
        int ic = 0, is = 0;
        uint32_t pc = 0, ps = 0, px = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
            const int m = m0 + r;
            const bool full_cols = n0 + BN <= N;
            float2 acc[COLS / 2];
#pragma unroll
            for (int j = 0; j < COLS / 2; ++j) acc[j] = make_float2(0.f, 0.f);
            uint32_t va[32], vb[32];
            // prologue: chunk 0 of group 0
            if (!warp_wait(&acc_full[ic], pc, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) goto done;
            tc_fence_after();
            tmem_ld_32x32b_x32(tlane + (uint32_t)(ic * BN), va);
            tmem_wait_ld(va);
            for (int g = 0; g < G; ++g) {
                if (!warp_wait(&full[is], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) goto done;
                const float* slot = reinterpret_cast<const float*>(smem + S::OFF_STAGE + is * S::STAGE_BYTES + S::ST_S);
                const float s_a = slot[r];
                const float* swp = slot + BM + col0;
                if (CHUNKS == 2) {
                    tmem_ld_32x32b_x32(tlane + (uint32_t)(ic * BN + 32), vb);  // chunk 1 of g
                    fold_group<32, FUSED>(*reinterpret_cast<float2(*)[16]>(&acc[0]), va, swp, s_a);
                    tmem_wait_ld(vb);
                } else {
                    vb[0] = vb[0];
                }
                // every chunk of group g is in registers: release its TMEM buffer
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ic]);
                if (++ic == NUM_ACC) { ic = 0; pc ^= 1u; }
                const bool next = g + 1 < G;
                if (next) {
                    if (!warp_wait(&acc_full[ic], pc, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) goto done;
                    tc_fence_after();
                    if (CHUNKS == 2) tmem_ld_32x32b_x32(tlane + (uint32_t)(ic * BN), va);  // chunk 0 of g+1
                }
                if (CHUNKS == 2) {
                    fold_group<32, FUSED>(*reinterpret_cast<float2(*)[16]>(&acc[16]), vb, swp + 32, s_a);
                } else {
                    fold_group<32, FUSED>(*reinterpret_cast<float2(*)[16]>(&acc[0]), va, swp, s_a);
                    if (next) tmem_ld_32x32b_x32(tlane + (uint32_t)(ic * BN), va);
                }
                // the stage's next fill is an async-proxy (TMA / bulk copy) write: order this warp's
                // generic-proxy reads of it before releasing the stage
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[is]);
                if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                if (next) tmem_wait_ld(va);
            }
            float* accf = reinterpret_cast<float*>(acc);
            if (EPI == DB_EPI_SWIGLU_QUANT) {
                // half 1 holds the up projection of the same 64 features: hand it to half 0.
                if (half == 1) {
                    if (!warp_wait(xch_empty, px ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) goto done;
#pragma unroll
                    for (int j = 0; j < COLS; ++j) xch[r * XCH_STRIDE + j] = accf[j];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_full);
                } else {
                    if (!warp_wait(xch_full, px, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) goto done;
                    if (m < M) {
                        float h[COLS];
                        float amax = 0.f;
#pragma unroll
                        for (int j = 0; j < COLS; ++j) {
                            h[j] = __fmul_rn(silu_ref(accf[j]), xch[r * XCH_STRIDE + j]);
                            amax = fmaxf(amax, fabsf(h[j]));
                        }
                        const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                        const float inv = __fdiv_rn(1.f, scale);
                        const int f0 = (n0 / BN) * 64;  // first output feature of this tile
                        __half* dst = out_codes + (size_t)m * ldoc + f0;
#pragma unroll
                        for (int b = 0; b < COLS; b += 8) {
                            const int order[8] = {0, 4, 1, 5, 2, 6, 3, 7};
                            __half hv[8];
#pragma unroll
                            for (int p = 0; p < 8; ++p)
                                hv[p] = __float2half_rn(
                                    fminf(fmaxf(rintf(__fmul_rn(h[b + order[p]], inv)), -127.f), 127.f));
                            *reinterpret_cast<uint4*>(dst + b) = *reinterpret_cast<uint4*>(hv);
                        }
                        out_scales[(size_t)(n0 / BN) * ldos + m] = scale;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_empty);
                }
                px ^= 1u;
            } else if (m < M) {
                float* dst = y + (size_t)m * ldy + n0 + col0;
                const float nanv = __int_as_float(0x7fc00000);
                if (full_cols && (ldy & 3) == 0 && (N & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < COLS; j += 4) {
                        float4 o = make_float4(accf[j], accf[j + 1], accf[j + 2], accf[j + 3]);
                        if (EPI == DB_EPI_RESIDUAL) {
                            const float4 rr = *reinterpret_cast<const float4*>(dst + j);
                            o.x = __fadd_rn(rr.x, o.x); o.y = __fadd_rn(rr.y, o.y);
                            o.z = __fadd_rn(rr.z, o.z); o.w = __fadd_rn(rr.w, o.w);
                        }
                        if (any_nonfinite) o = make_float4(nanv, nanv, nanv, nanv);
                        *reinterpret_cast<float4*>(dst + j) = o;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < COLS; ++j) {
                        if (n0 + col0 + j < N) {
                            float o = accf[j];
                            if (EPI == DB_EPI_RESIDUAL) o = __fadd_rn(dst[j], o);
                            dst[j] = any_nonfinite ? nanv : o;
                        }
                    }
                }
            }
        }
    }
done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, NUM_ACC * BN);
    }
}

}  // namespace db

using namespace db;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int db_num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <int BN, int BITS, int EPI, bool FUSED>
static int launch_variant(const DbGemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmW, int G,
                          cudaStream_t stream) {
    using S = GemmSmem<BN, BITS, EPI>;
    auto kernel = gemm_tc_kernel<BN, BITS, EPI, FUSED>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES);
        if (e != cudaSuccess) return (int)e;
        configured = true;
    }
    const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    int ctas = a.max_ctas > 0 ? a.max_ctas : db_num_sms();
    if (ctas > tiles) ctas = tiles;
    kernel<<<ctas, NUM_THREADS, S::BYTES, stream>>>(tmA, tmW, a.sa, a.ldsa, a.sw, db_scale_stride(a.N), a.M, a.N, G,
                                                    a.y, a.ldy,
                                                    static_cast<__half*>(a.out_codes), a.ldoc, a.out_scales, a.ldos,
                                                    a.nonfinite, a.dev_error);
    return (int)cudaGetLastError();
}

template <int BN, int BITS>
static int dispatch_epi(const DbGemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmW, int G,
                        cudaStream_t s) {
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) {
        if (BN != 128) return (int)cudaErrorInvalidValue;
        return a.fused ? launch_variant<BN, BITS, DB_EPI_SWIGLU_QUANT, true>(a, tmA, tmW, G, s)
                       : launch_variant<BN, BITS, DB_EPI_SWIGLU_QUANT, false>(a, tmA, tmW, G, s);
    }
    if (a.epilogue == DB_EPI_RESIDUAL)
        return a.fused ? launch_variant<BN, BITS, DB_EPI_RESIDUAL, true>(a, tmA, tmW, G, s)
                       : launch_variant<BN, BITS, DB_EPI_RESIDUAL, false>(a, tmA, tmW, G, s);
    return a.fused ? launch_variant<BN, BITS, DB_EPI_STORE, true>(a, tmA, tmW, G, s)
                   : launch_variant<BN, BITS, DB_EPI_STORE, false>(a, tmA, tmW, G, s);
}

int db_launch_gemm_tc(const DbGemmArgs& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.K <= 0 || (a.bits != 4 && a.bits != 8)) return (int)cudaErrorInvalidValue;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    const int G = (a.K + BK - 1) / BK, Kp = G * BK;
    int bn = a.block_n ? a.block_n : 128;
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) bn = 128;
    if (bn != 64 && bn != 128) return (int)cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.a_codes) & 15) || (a.lda * 2) % 16 || a.lda < Kp ||
        (reinterpret_cast<uintptr_t>(a.w_codes) & 15) || (reinterpret_cast<uintptr_t>(a.sa) & 15) ||
        (reinterpret_cast<uintptr_t>(a.sw) & 15) || a.ldsa < db_scale_stride(a.M) || (a.ldsa & 3))
        return (int)cudaErrorMisalignedAddress;
    CUtensorMap tmA, tmW;
    {
        cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.lda * 2};
        cuuint32_t box[2] = {BK, BM};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.a_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    {
        const cuuint64_t row_bytes = (cuuint64_t)Kp * a.bits / 8;
        cuuint64_t dims[2] = {row_bytes, (cuuint64_t)a.N};
        cuuint64_t strides[1] = {row_bytes};
        cuuint32_t box[2] = {(cuuint32_t)(BK * a.bits / 8), (cuuint32_t)bn};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.w_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    if (bn == 64) return a.bits == 4 ? dispatch_epi<64, 4>(a, tmA, tmW, G, stream) : dispatch_epi<64, 8>(a, tmA, tmW, G, stream);
    return a.bits == 4 ? dispatch_epi<128, 4>(a, tmA, tmW, G, stream) : dispatch_epi<128, 8>(a, tmA, tmW, G, stream);
}
