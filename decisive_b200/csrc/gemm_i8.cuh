// Tensor-core grouped W4A8 / W8A8 GEMM on int8 activation codes (sm_100a, tcgen05 kind::i8).
//
// Computes, for every output (m, n), the reference's grouped sum (int8.rs:526-585):
//     acc = 0; for g ascending: acc = fma(float(dot_g), sw[n,g] * sa[m,g], acc)
// (or the portable acc = acc + dot_g * (sa * sw), int8.rs:259-287), where dot_g is the exact
// integer dot of one scale block (64 values; 32 for Decima's blocks of 32) of activation codes
// with weight codes.
//
// The dots come from tcgen05.mma kind::i8 (signed 8-bit A and B, s32 accumulators in tensor
// memory, K = 32 per instruction): each scale block is one job with its own TMEM accumulator
// buffer.  The epilogue converts a dot exactly without an integer-to-float conversion: adding
// DOT_BIAS = 0x4B400000 (the bits of 1.5 * 2^23) to the s32 dot gives the bits of the float
// 12582912 + dot (|dot| <= 64 * 127 * 127 < 2^22), and subtracting 12582912 is exact.
//
// Layout.  A: int8 codes [M, lda] in natural k order.  W: the device layout (Q4 [N, Kp/2] bytes,
// low nibble = even k, nibble = code + 8; Q8 [N, Kp] int8), scales f32 [GS, ldsw].  A pipeline
// stage holds 128 k: the activation tile (128 rows x 128 bytes, 128B swizzle) and the weight
// tile, loaded by TMA as-is for Q8 (128B swizzle) or as raw nibbles for Q4, which two converter
// warps turn into the swizzled int8 tile.
//
// Tiles are 128 x BN with BN = 32, 64, 128 or 256 (32: single CTAs, store / residual epilogues; it
// serves small M, where wider tiles leave most SMs without a tile).
// Roles (384 threads, one CTA per SM, persistent over MT x BN output tiles):
//   warp 0      TMA producer
//   warp 1      TMEM owner + MMA issuer (lane 0; in pair mode the even CTA issues M = 256 MMAs
//               for both CTAs of the cluster, each CTA holding 128 rows of A and BN/2 rows of W)
//   warps 2-3   Q4 weight converters (idle for Q8)
//   warps 4-11  epilogue (216 registers each through setmaxnreg): warp w reads TMEM lanes
//               32 (w % 4).. and half of the tile's columns; per job: dot conversion and scale
//               fold in f32 (packed f32x2 operations, each an IEEE operation); per tile: TMA
//               store / reduce-add of the outputs, or SwiGLU + re-quantisation
// Every mbarrier wait is bounded (DB_WAIT_LIMIT_NS); on expiry the CTA records an error in the
// device error word, stops issuing work, lets its own copies and MMAs land and frees its tensor
// memory.  No TMA multicast.
#pragma once
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace db {
namespace gi8 {

constexpr int BM = 128;    // tile rows held by one CTA
constexpr int KS = 128;    // k (bytes of int8 codes) per pipeline stage: two groups of 64
constexpr int CONV_WARP0 = 2;
constexpr int CONV_WARPS = 2;
constexpr int EPI_WARP0 = 4;
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_WARPS);  // 384
// Register split (setmaxnreg): __launch_bounds__(384, 1) gives every thread 168 registers at
// launch (65536 / 384, rounded down to a multiple of 8); warpgroup 0 (producer, MMA, converters)
// drops to 64 and warpgroups 1-2 (epilogue) rise to 216: 128 * 64 + 256 * 216 <= 168 * 384.
constexpr int REGS_LAUNCH = 65536 / NUM_THREADS / 8 * 8;
#ifndef GI8_REGS_CONTROL
#define GI8_REGS_CONTROL 64
#endif
constexpr int REGS_CONTROL = GI8_REGS_CONTROL;
constexpr int REGS_EPI = (REGS_LAUNCH * NUM_THREADS - 128 * REGS_CONTROL) / 256 / 8 * 8;
static_assert(128 * REGS_CONTROL + 256 * REGS_EPI <= REGS_LAUNCH * NUM_THREADS, "register split");
// How the epilogue waits for a finished job and the producer for free ring slots.
#ifndef GI8_EPI_WAIT
#define GI8_EPI_WAIT mbar_spin_polite
#endif
#ifndef GI8_PROD_WAIT
#define GI8_PROD_WAIT mbar_spin_polite
#endif
constexpr uint32_t DOT_BIAS = 0x4B400000u;  // bits of 12582912.0f
constexpr float DOT_BIAS_F = 12582912.0f;
constexpr uint64_t DRAIN_NS = 100000000ull;

template <int BN, int BITS, int EPI, bool PAIR>
struct Smem {
    static constexpr int WR = PAIR ? BN / 2 : BN;               // weight rows held by this CTA
    static constexpr int NBUF = 512 / BN > 16 ? 16 : 512 / BN;  // TMEM accumulator buffers
    static constexpr int A_BYTES = BM * KS;                     // 16 KB
    static constexpr int B_BYTES = WR * KS;                     // int8 weight tile of a stage
    static constexpr int RAW_BYTES = BITS == 4 ? WR * KS / 2 : 0;
    static constexpr int STAGE_BYTES = A_BYTES + (BITS == 8 ? B_BYTES : RAW_BYTES);
    static constexpr int CB_BYTES = BITS == 4 ? B_BYTES : 0;    // converted Q4 tile of a stage
    static constexpr int COLS = BN / 2;                         // accumulator columns per epilogue thread
    static constexpr int SCJ = BN <= 32 ? 32 : 16;              // scale ring: jobs loaded ahead of the epilogue
    static constexpr int SC_SLOT = (BM + BN) * 4;               // sa of this CTA's 128 rows + sw of the tile's columns
    static constexpr int SC_BYTES = SCJ * SC_SLOT;
    static constexpr int Y_CHUNK = 32 * 16 * 4;                 // 32 rows x 16 f32 columns
    static constexpr int Y_BUFS = 2;
    static constexpr int Y_BYTES = EPI == DB_EPI_SWIGLU_QUANT ? 0 : EPI_WARPS * Y_BUFS * Y_CHUNK;
    // SwiGLU on 128-wide tiles: 32 exchanged columns per row from each half, plus row maxima
    static constexpr int X_BYTES = (EPI == DB_EPI_SWIGLU_QUANT && BN == 128) ? (2 * BM * 33 + 2 * BM) * 4 : 0;
    static constexpr int BUDGET = 232448 - 1024 - 1024;         // opt-in limit - alignment - barriers
    static constexpr int PER_STAGE = STAGE_BYTES + CB_BYTES;
    static constexpr int FIT = (BUDGET - SC_BYTES - Y_BYTES - X_BYTES) / PER_STAGE;
    static constexpr int STAGES = FIT > 6 ? 6 : FIT;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_CB = OFF_STAGE + STAGES * STAGE_BYTES;
    static constexpr int OFF_SC = OFF_CB + STAGES * CB_BYTES;
    static constexpr int OFF_Y = OFF_SC + SC_BYTES;
    static constexpr int OFF_X = OFF_Y + Y_BYTES;
    static constexpr int OFF_BAR = (OFF_X + X_BYTES + 15) / 16 * 16;
    // full, empty, wfull, cbf per stage; done, acc_empty per buffer; sc_full, sc_empty per scale
    // slot; mma_done; 2 x 4 SwiGLU exchange barriers; two teardown barriers
    static constexpr int NUM_BARS = 4 * STAGES + 2 * NBUF + 2 * SCJ + 1 + 8 + 2;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;
    static_assert(STAGES >= 2, "at least two pipeline stages");
    static_assert(BYTES <= 232448, "shared memory budget");
    static_assert(STAGE_BYTES % 1024 == 0 && CB_BYTES % 1024 == 0 && A_BYTES % 1024 == 0,
                  "128B-swizzled tiles need 1024-byte alignment");
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}
// Warp-wide wait for the producer and the converters: one lane polls with mbarrier.test_wait and a
// short sleep between polls.  (A thread suspended in mbarrier.try_wait was measured to resume up to
// microseconds after the phase completed, which paced the whole pipeline at one stage per ~1 us.)
__device__ __forceinline__ bool warp_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_spin_polite(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// 8 weight nibbles (one 32-bit word of a Q4 row: k = 8c..8c+7, even k in the low nibbles,
// nibble = code + 8) -> 8 int8 codes in natural order, as two words (k0..k3, k4..k7).
__device__ __forceinline__ uint2 nibbles_to_s8(uint32_t w) {
    // nibble + 0x78 stays inside its byte; xor 0x80 then gives nibble - 8 as a two's complement byte
    const uint32_t lo = ((w & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;         // k0 k2 k4 k6
    const uint32_t hi = (((w >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;  // k1 k3 k5 k7
    return make_uint2(__byte_perm(lo, hi, 0x5140), __byte_perm(lo, hi, 0x7362));
}

// Orders later uses of r after the preceding tcgen05.wait::ld (the registers are written
// asynchronously by tcgen05.ld).
__device__ __forceinline__ void tie32(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

__device__ __forceinline__ void tie16(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]));
}
// One job's HC columns of this warp's lanes: 32-column loads, or one 16-column load at 32-wide tiles.
template <int HC>
__device__ __forceinline__ void load_cols(uint32_t taddr, uint32_t* v) {
    if constexpr (HC == 16) {
        tmem_ld_32x32b_x16(taddr, *reinterpret_cast<uint32_t(*)[16]>(v));
    } else {
#pragma unroll
        for (int c = 0; c < HC / 32; ++c) tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
    }
}
template <int HC>
__device__ __forceinline__ void tie_cols(uint32_t* v) {
    if constexpr (HC == 16) {
        tie16(*reinterpret_cast<uint32_t(*)[16]>(v));
    } else {
#pragma unroll
        for (int c = 0; c < HC / 32; ++c) tie32(*reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
    }
}

// 16 * Q16 values h (pairs in v) -> int8 codes clamp(rint(h * inv), +-127), natural order, as
// Q16 16-byte stores to dst (16-byte aligned): pack_bits of int8.rs:347-360.
template <int Q16, int NV>
__device__ __forceinline__ void store_codes(int8_t* dst, const uint64_t (&v)[NV], float inv) {
#pragma unroll
    for (int q16 = 0; q16 < Q16; ++q16) {
        uint32_t wds[4];
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int f = q16 * 16 + wq * 4 + e;
                const float h = (f & 1) ? f2_hi(v[f / 2]) : f2_lo(v[f / 2]);
                const int code = (int)fminf(fmaxf(rintf(__fmul_rn(h, inv)), -127.f), 127.f);
                word |= ((uint32_t)code & 0xFFu) << (8 * e);
            }
            wds[wq] = word;
        }
        *reinterpret_cast<uint4*>(dst + q16 * 16) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
    }
}

__device__ __forceinline__ float silu_ref(float x) {
    // cpu.rs:513-518: x * (1 / (1 + exp(-x))); the correctly rounded reciprocal is exactly the
    // correctly rounded quotient 1 / y
    return __fmul_rn(x, __frcp_rn(__fadd_rn(1.f, expf(-x))));
}

// Folds 16 columns of one job: v holds the biased dots (float bits), w_addr the 16 weight scales
// in shared memory.  fused: acc = fma(d, sw * sa, acc); portable: acc = acc + d * (sa * sw).
template <bool FUSED>
__device__ __forceinline__ void fold16(uint64_t* acc, const uint32_t (&v)[16], uint32_t w_addr, float s_a) {
    const uint64_t sa2 = f2_pack(__float_as_uint(s_a), __float_as_uint(s_a));
    const uint64_t nb2 = f2_pack(__float_as_uint(-DOT_BIAS_F), __float_as_uint(-DOT_BIAS_F));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 w = lds128(w_addr + i * 16);
        // the s32 dot plus the bias bits, read as a float, is 12582912 + dot exactly; subtracting
        // 12582912 is exact too: float(dot) without an integer-to-float conversion
        const uint64_t d0 = f2_add(f2_pack(v[4 * i] + DOT_BIAS, v[4 * i + 1] + DOT_BIAS), nb2);
        const uint64_t d1 = f2_add(f2_pack(v[4 * i + 2] + DOT_BIAS, v[4 * i + 3] + DOT_BIAS), nb2);
#ifdef GI8_SCALAR_FOLD
        if (FUSED) {
            const float dd[4] = {f2_lo(d0), f2_hi(d0), f2_lo(d1), f2_hi(d1)};
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint64_t a = acc[2 * i + e / 2];
                const float prev = (e & 1) ? f2_hi(a) : f2_lo(a);
                o[e] = __fmaf_rn(dd[e], __fmul_rn(__uint_as_float(ww[e]), s_a), prev);
            }
            acc[2 * i] = f2_pack(__float_as_uint(o[0]), __float_as_uint(o[1]));
            acc[2 * i + 1] = f2_pack(__float_as_uint(o[2]), __float_as_uint(o[3]));
        } else
#endif
        if (FUSED) {
            acc[2 * i] = f2_fma(d0, f2_mul(f2_pack(w.x, w.y), sa2), acc[2 * i]);
            acc[2 * i + 1] = f2_fma(d1, f2_mul(f2_pack(w.z, w.w), sa2), acc[2 * i + 1]);
        } else {
            const float dd[4] = {f2_lo(d0), f2_hi(d0), f2_lo(d1), f2_hi(d1)};
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint64_t a = acc[2 * i + e / 2];
                const float prev = (e & 1) ? f2_hi(a) : f2_lo(a);
                o[e] = __fadd_rn(prev, __fmul_rn(dd[e], __fmul_rn(s_a, __uint_as_float(ww[e]))));
            }
            acc[2 * i] = f2_pack(__float_as_uint(o[0]), __float_as_uint(o[1]));
            acc[2 * i + 1] = f2_pack(__float_as_uint(o[2]), __float_as_uint(o[3]));
        }
    }
}

template <int BN, int BITS, int EPI, bool FUSED, bool PAIR, int SUB>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmY, int y_tma, const float* __restrict__ sa, int64_t ldsa,
                   const float* __restrict__ sw, int64_t ldsw, int M, int N, int G, int GS, float* __restrict__ y,
                   int64_t ldy, int8_t* __restrict__ out_codes, int64_t ldoc, float* __restrict__ out_scales,
                   int64_t ldos, const int* __restrict__ nonfinite, const float* __restrict__ bias, int add_bias,
                   int* __restrict__ dev_error) {
    using S = Smem<BN, BITS, EPI, PAIR>;
    static_assert(EPI != DB_EPI_SWIGLU_QUANT || BN == 256 || BN == 128, "SwiGLU needs whole 64 + 64 blocks per tile");
    static_assert(SUB == 1 || (SUB == 2 && BITS == 8 && EPI != DB_EPI_SWIGLU_QUANT), "blocks of 32: Q8 only");
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* full = bars;                     // stage: activation (+ Q8 weight) tiles landed; leader counts both CTAs
    uint64_t* empty = full + S::STAGES;        // stage: the MMAs are done with it (committed to both CTAs)
    uint64_t* wfull = empty + S::STAGES;       // stage (Q4): this CTA's raw weight codes landed
    uint64_t* cbf = wfull + S::STAGES;         // stage (Q4): both CTAs' converted weight tiles ready (leader)
    uint64_t* done = cbf + S::STAGES;          // buffer: the job's MMAs completed (both CTAs)
    uint64_t* acc_empty = done + S::NBUF;      // buffer: both CTAs' epilogues read it and wrote the bias back
    uint64_t* sc_full = acc_empty + S::NBUF;   // scale slot: the job's sa / sw landed (this CTA)
    uint64_t* sc_empty = sc_full + S::SCJ;     // scale slot: every epilogue warp of this CTA read it
    uint64_t* mma_done = sc_empty + S::SCJ;    // final commit of the MMA issuer
    auto end_bar = [&](int i) { return reinterpret_cast<uint64_t*>(smem + S::OFF_BAR) + (S::NUM_BARS - 2 + i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    constexpr int MT = PAIR ? 2 * BM : BM;  // tile rows
    const int m_tiles = (M + MT - 1) / MT, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int row_off = (int)rank * BM, wrow_off = (int)rank * S::WR;
    const int NS = (G + 1) / 2;  // stages per tile
    auto at_leader = [&](uint64_t* b) { return PAIR ? mapa_shared(smem_u32(b), 0) : smem_u32(b); };
    auto at_peer = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 1); };

    if (threadIdx.x == 0) {
        constexpr int NC = PAIR ? 2 : 1;
        for (int i = 0; i < S::STAGES; ++i) {
            mbar_init(&full[i], 1);  // the leader's arrive (pair: armed with both CTAs' bytes)
            mbar_init(&empty[i], 1);
            mbar_init(&wfull[i], 1);
            mbar_init(&cbf[i], NC * CONV_WARPS);
        }
        for (int i = 0; i < S::NBUF; ++i) {
            mbar_init(&done[i], 1);
            mbar_init(&acc_empty[i], NC * EPI_WARPS);
        }
        for (int i = 0; i < S::SCJ; ++i) {
            mbar_init(&sc_full[i], 1);
            mbar_init(&sc_empty[i], EPI_WARPS);
        }
        mbar_init(mma_done, 1);
        for (int i = 0; i < 8; ++i) mbar_init(mma_done + 1 + i, 2);  // SwiGLU exchange (two warps each)
        mbar_init(end_bar(0), NUM_THREADS / 32);
        mbar_init(end_bar(1), 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (warp < EPI_WARP0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CONTROL));
        if (warp == 0) {
            // ------------------------------------------------------------ TMA producer
            // Two independent issue chains: lane 0 loads the stages (activation and weight tiles),
            // lane 1 the scale ring (per job: this CTA's 128 activation scales and the tile's BN
            // weight scales, clipped to the padded scale rows ldsa, ldsw; 16-byte multiples).  An
            // mbarrier test costs ~200-300 cycles before its result can be used and a copy issue
            // ~100-150, so one chain of ~14 operations per stage took ~1,900 cycles and paced the
            // pipeline; the two diverged lanes interleave and hide each other's latency.  No
            // warp-wide handshake inside the loops.
            if (lane == 0) {
                int st = 0, issued = 0;
                uint32_t ps = 0;
                for (int tile = tile0; tile < tiles; tile += tstride) {
                    const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN + wrow_off;
                    for (int s = 0; s < NS; ++s) {
                        if (!GI8_PROD_WAIT(&empty[st], ps ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_TMA)) goto stage_drain;
                        uint8_t* sp = smem + S::OFF_STAGE + st * S::STAGE_BYTES;
                        // full boxes are counted, also where they reach past K or M (zero fill)
                        constexpr uint32_t TX = S::A_BYTES + (BITS == 8 ? S::B_BYTES : 0);
                        if (PAIR) {
                            // both CTAs' loads complete on the leader's barrier, which the leader
                            // alone arms with both CTAs' bytes by a local arrive (in the dequantised
                            // GEMM's pairs a cluster-scope arrive from each CTA measured ~1,000
                            // cycles per stage); a peer's bytes may land first, but the phase waits
                            // for the leader's arrive and a stage is reloaded only after its
                            // previous MMAs completed
                            if (leader) mbar_arrive_expect_tx(&full[st], 2 * TX);
                            tma_load_2d_pair(sp, &tmA, at_leader(&full[st]), s * KS, m0);
                            if (BITS == 8) tma_load_2d_pair(sp + S::A_BYTES, &tmW, at_leader(&full[st]), s * KS, n0);
                        } else {
                            mbar_arrive_expect_tx(&full[st], TX);
                            tma_load_2d(sp, &tmA, &full[st], s * KS, m0);
                            if (BITS == 8) tma_load_2d(sp + S::A_BYTES, &tmW, &full[st], s * KS, n0);
                        }
                        if (BITS == 4) {
                            mbar_arrive_expect_tx(&wfull[st], S::RAW_BYTES);
                            tma_load_2d(sp + S::A_BYTES, &tmW, &wfull[st], s * (KS / 2), n0);
                        }
                        ++issued;
                        if (++st == S::STAGES) { st = 0; ps ^= 1u; }
                    }
                }
                goto stage_done;
            stage_drain:
                // after an abort: let the stages this lane issued land before the CTA winds down
                for (int k = 0; k < issued && k < S::STAGES; ++k) {
                    if (st == 0) { st = S::STAGES - 1; ps ^= 1u; } else --st;
                    if (BITS == 4) mbar_wait_drain(&wfull[st], ps, DRAIN_NS);
                    if (leader) mbar_wait_drain(&full[st], ps, DRAIN_NS);
                }
            stage_done:;
            } else if (lane == 1) {
                int jn = 0, sc_issued = 0;
                for (int tile = tile0; tile < tiles; tile += tstride) {
                    const int m0 = (tile % m_tiles) * MT + row_off, ncol0 = (tile / m_tiles) * BN;
                    const int sa_rows = (int)min((int64_t)BM, ldsa - m0), sw_cols = (int)min((int64_t)BN, ldsw - ncol0);
                    const uint32_t sc_bytes = (uint32_t)(max(sa_rows, 0) + max(sw_cols, 0)) * 4u;
                    for (int j = 0; j < GS; ++j, ++jn) {
                        const int slot = jn % S::SCJ;
                        if (!GI8_PROD_WAIT(&sc_empty[slot], ((uint32_t)(jn / S::SCJ) & 1u) ^ 1u, abort_flag, dev_error,
                                           DB_DEV_ERR_TIMEOUT_TMA))
                            goto scale_drain;
                        uint8_t* dst = smem + S::OFF_SC + slot * S::SC_SLOT;
                        mbar_arrive_expect_tx(&sc_full[slot], sc_bytes);
                        if (sa_rows > 0) bulk_load(dst, sa + (int64_t)j * ldsa + m0, (uint32_t)sa_rows * 4u, &sc_full[slot]);
                        if (sw_cols > 0)
                            bulk_load(dst + BM * 4, sw + (int64_t)j * ldsw + ncol0, (uint32_t)sw_cols * 4u, &sc_full[slot]);
                        ++sc_issued;
                    }
                }
                goto scale_done;
            scale_drain:
                // after an abort: let the scale slots this lane issued land before the CTA winds down
                for (int k = 0; k < sc_issued && k < S::SCJ; ++k) {
                    const int jj = jn - 1 - k;
                    mbar_wait_drain(&sc_full[jj % S::SCJ], (uint32_t)(jj / S::SCJ) & 1u, DRAIN_NS);
                }
            scale_done:;
            }
            __syncwarp();
        } else if (warp == 1) {
            // ------------------------------------------------------------ MMA issuer
            // Lane 0 alone runs the issue loop (no warp-wide handshakes per job); descriptors are
            // built once and advanced by the stage / k offsets (start address field, in 16-byte
            // units: shared memory is below 256 KB, so the 14-bit field never carries).
            constexpr uint32_t IDESC = idesc_s8_s32(MT, BN);
            // the epilogue's steps (jobs per completion wait); with GS a multiple of JPS_E (and
            // NBUF a multiple of JPS_E) every buffer is always either the last of a step or never
            // waited on, so only the last jobs of steps need a completion commit
            constexpr int JPS_E = S::COLS >= 128 ? 1 : 128 / S::COLS;
            static_assert(S::NBUF % JPS_E == 0, "steps of jobs fall on whole buffer groups");
            const bool SPARSE_DONE = JPS_E > 1 && GS % JPS_E == 0;
            constexpr int KPJ = 2 / SUB;  // K = 32 MMAs per job
            constexpr int JB = 64 / SUB;  // k bytes per job
            if (leader && lane == 0) {
                const uint32_t st_base = smem_u32(smem + S::OFF_STAGE), cb_base = smem_u32(smem + S::OFF_CB);
                const uint64_t a_desc0 = sw128_desc(st_base);
                const uint64_t b_desc0 = sw128_desc(BITS == 8 ? st_base + S::A_BYTES : cb_base);
                constexpr int B_STRIDE = BITS == 8 ? S::STAGE_BYTES : S::CB_BYTES;
                int st = 0, jn = 0;
                uint32_t ps = 0;
                for (int tile = tile0; tile < tiles; tile += tstride) {
                    for (int s = 0; s < NS; ++s) {
                        // the stage's tiles (and, Q4, its converted weights): both tests in flight
                        if (BITS == 4 ? !mbar_spin2(&full[st], ps, &cbf[st], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA)
                                      : !mbar_spin(&full[st], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA))
                            goto mma_end;
                        const uint64_t ad = a_desc0 + (uint64_t)((st * S::STAGE_BYTES) >> 4);
                        const uint64_t bd = b_desc0 + (uint64_t)((st * B_STRIDE) >> 4);
                        const int j0 = s * 2 * SUB, j1 = min(j0 + 2 * SUB, GS);
                        // Each job's buffer must be free and its scale vectors landed (the epilogue
                        // then needs to wait for the job's completion only).  With four or more
                        // buffers the stage's jobs are checked together (two jobs' four barriers per
                        // test); with two (256-wide tiles) the next job's buffer is the one the
                        // epilogue is reading, so each job waits for its own just before its MMAs.
                        if (S::NBUF >= 4) {
                            for (int q = 0; q < j1 - j0; q += 2) {
                                const int ja = jn + q, jb = ja + 1;
                                const bool ok =
                                    q + 1 < j1 - j0
                                        ? mbar_spin4(&acc_empty[ja % S::NBUF], (uint32_t)(ja / S::NBUF) & 1u,
                                                     &sc_full[ja % S::SCJ], (uint32_t)(ja / S::SCJ) & 1u,
                                                     &acc_empty[jb % S::NBUF], (uint32_t)(jb / S::NBUF) & 1u,
                                                     &sc_full[jb % S::SCJ], (uint32_t)(jb / S::SCJ) & 1u, abort_flag,
                                                     dev_error, DB_DEV_ERR_TIMEOUT_MMA)
                                        : mbar_spin2(&acc_empty[ja % S::NBUF], (uint32_t)(ja / S::NBUF) & 1u,
                                                     &sc_full[ja % S::SCJ], (uint32_t)(ja / S::SCJ) & 1u, abort_flag,
                                                     dev_error, DB_DEV_ERR_TIMEOUT_MMA);
                                if (!ok) goto mma_end;
                            }
                            tc_fence_after();
                        }
                        for (int j = j0; j < j1; ++j, ++jn) {
                            const int b = jn % S::NBUF;
                            if (S::NBUF < 4) {
                                if (!mbar_spin2(&acc_empty[b], (uint32_t)(jn / S::NBUF) & 1u, &sc_full[jn % S::SCJ],
                                                (uint32_t)(jn / S::SCJ) & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA))
                                    goto mma_end;
                                tc_fence_after();
                            }
                            const uint32_t d = tmem_base + (uint32_t)(b * BN);
#pragma unroll
                            for (int kk = 0; kk < KPJ; ++kk) {
                                const uint64_t off = (uint64_t)(((j - j0) * JB + kk * 32) >> 4);
                                const uint32_t acc_in = kk > 0 ? 1u : 0u;  // a job starts from zero
                                if (PAIR) umma_i8_pair(d, ad + off, bd + off, IDESC, acc_in);
                                else umma_i8(d, ad + off, bd + off, IDESC, acc_in);
                            }
                            // completion is signalled where the epilogue waits: every job, or (steps
                            // of JPS_E jobs dividing the tile) the last job of each step
                            if (!SPARSE_DONE || jn % JPS_E == JPS_E - 1) {
                                if (PAIR) {
                                    umma_commit_pair(smem_u32(&done[b]));
                                    umma_commit_pair(at_peer(&done[b]));
                                } else {
                                    umma_commit(&done[b]);
                                }
                            }
                        }
                        if (PAIR) {
                            umma_commit_pair(smem_u32(&empty[st]));
                            umma_commit_pair(at_peer(&empty[st]));
                        } else {
                            umma_commit(&empty[st]);
                        }
                        if (++st == S::STAGES) { st = 0; ps ^= 1u; }
                    }
                }
            mma_end:
                // every MMA this thread issued has completed before the CTA releases tensor memory
                if (PAIR) {
                    umma_commit_pair(smem_u32(mma_done));
                    umma_commit_pair(at_peer(mma_done));
                } else {
                    umma_commit(mma_done);
                }
                mbar_wait_drain(mma_done, 0, DRAIN_NS);
            } else if (!leader && lane == 0) {
                // the peer CTA's tensor memory is written by the leader's MMAs: wait for their last
                // commit (a wait as long as the whole launch, so bounded by the launch-wide limit)
                mbar_wait_drain(mma_done, 0, DB_WAIT_LIMIT_NS);
            }
            __syncwarp();
        } else if (BITS == 4 && warp < CONV_WARP0 + CONV_WARPS) {
            // ------------------------------------------------------------ Q4 converters
            const int ct = threadIdx.x - CONV_WARP0 * 32;
            const uint32_t st_base = smem_u32(smem + S::OFF_STAGE), cb_base = smem_u32(smem + S::OFF_CB);
            int st = 0;
            uint32_t ps = 0;
            for (int tile = tile0; tile < tiles; tile += tstride) {
                for (int s = 0; s < NS; ++s) {
                    if (!warp_wait_backoff(&wfull[st], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_CVT)) goto ctl_done;
                    const uint32_t raw = st_base + st * S::STAGE_BYTES + S::A_BYTES;
                    const uint32_t cb = cb_base + st * S::CB_BYTES;
                    for (int row = ct; row < S::WR; row += 32 * CONV_WARPS) {
                        const int swz = row & 7;
#pragma unroll
                        for (int i0 = 0; i0 < 4; ++i0) {
                            // rotate the 16-byte column by the row so that eight lanes read eight
                            // different bank groups of their 64-byte rows
                            const int i = (i0 + (row >> 1)) & 3;
                            const uint4 v = lds128(raw + row * (KS / 2) + i * 16);
                            const uint2 a = nibbles_to_s8(v.x), b = nibbles_to_s8(v.y);
                            const uint2 c = nibbles_to_s8(v.z), d = nibbles_to_s8(v.w);
                            sts128(cb + row * KS + (((2 * i) ^ swz) << 4), make_uint4(a.x, a.y, b.x, b.y));
                            sts128(cb + row * KS + (((2 * i + 1) ^ swz) << 4), make_uint4(c.x, c.y, d.x, d.y));
                        }
                    }
                    // generic writes of the tile become MMA (async proxy) reads
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (PAIR) mbar_arrive_cluster(at_leader(&cbf[st]));
                        else mbar_arrive(&cbf[st]);
                    }
                    if (++st == S::STAGES) { st = 0; ps ^= 1u; }
                }
            }
        }
    ctl_done:;
    } else {
        // ---------------------------------------------------------------- epilogue
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPI));
        constexpr int COLS = S::COLS;
        const int ew = warp - EPI_WARP0;
        const int q = warp & 3;       // TMEM lane quadrant this warp may access
        const int half = ew >> 2;     // which half of the tile's columns
        const int r = q * 32 + lane;  // row inside this CTA's 128 rows
        const int col0 = half * COLS;
        const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
        const uint32_t sc_base = smem_u32(smem + S::OFF_SC);
        const bool any_nonfinite = nonfinite != nullptr && *nonfinite != 0;
        // every accumulator buffer starts free
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < S::NBUF; ++b) {
                if (PAIR) mbar_arrive_cluster(at_leader(&acc_empty[b]));
                else mbar_arrive(&acc_empty[b]);
            }
        // job jn's accumulators are ready (its MMAs completed; the MMA issuer waited for the job's
        // scale vectors before issuing them, so those have landed too); false: aborted
        auto wait_job = [&](int jn) -> bool {
            int ok = 1;
            if (lane == 0)
                ok = GI8_EPI_WAIT(&done[jn % S::NBUF], (uint32_t)(jn / S::NBUF) & 1u, abort_flag, dev_error,
                                  DB_DEV_ERR_TIMEOUT_EPI);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            __syncwarp();
            return ok != 0;
        };
        int ybuf = 0;
        // Output of a finished tile: the fused SwiGLU + re-quantisation, a TMA store / reduce-add
        // through shared memory, or plain stores.  jt counts this CTA's tiles (exchange phases).
        auto finish_tile = [&](uint64_t (&acc)[COLS / 2], int m0, int n0, int jt) -> bool {
            const int m = m0 + r;
            if constexpr (EPI == DB_EPI_SWIGLU_QUANT) {
                // the columns are blocks of 64 gate rows followed by the 64 matching up rows
                // (db_interleave_gate_up): h = silu(gate) * up for 64 features of a block, then the
                // group-64 re-quantisation of grouped_q4_mlp.wgsl:83-105 (= int8.rs:178-202)
                if constexpr (COLS == 128) {
                    // a thread holds a whole block: gate in columns 0-63, up in 64-127
                    const int blk = (n0 + col0) / 128;
                    if (blk * 128 < N && m < M) {
                        float amax = 0.f;
#pragma unroll
                        for (int f = 0; f < 32; ++f) {
                            const uint64_t g2 = acc[f], u2 = acc[32 + f];
                            const float h0 = __fmul_rn(silu_ref(f2_lo(g2)), f2_lo(u2));
                            const float h1 = __fmul_rn(silu_ref(f2_hi(g2)), f2_hi(u2));
                            acc[f] = f2_pack(__float_as_uint(h0), __float_as_uint(h1));
                            amax = fmaxf(amax, fmaxf(fabsf(h0), fabsf(h1)));
                        }
                        const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                        const float inv = __fdiv_rn(1.f, scale);
                        store_codes<4>(out_codes + (size_t)m * ldoc + (size_t)blk * 64, acc, inv);
                        out_scales[(size_t)blk * ldos + m] = scale;
                    }
                } else {
                    // 128-wide tile = one block: half 0 holds the gate rows, half 1 the up rows of the
                    // same 64 features.  Half 0 finishes features 0-31, half 1 features 32-63; the two
                    // warps of a lane quadrant trade 32 columns and then their row maxima through
                    // shared memory (bounded mbarrier waits, phase = tile count).
                    float* xg = reinterpret_cast<float*>(smem + S::OFF_X);  // gate 32-63, by half 0
                    float* xu = xg + BM * 33;                                 // up 0-31, by half 1
                    float* xm = xu + BM * 33;                                 // [2][BM] row maxima
                    uint64_t* xf = bars + S::NUM_BARS - 2 - 8;                // [4] columns published
                    uint64_t* xa = xf + 4;                                    // [4] maxima published
                    float* mine = (half == 0 ? xg : xu) + r * 33;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint64_t v = acc[(half == 0 ? 16 : 0) + i];
                        mine[2 * i] = f2_lo(v);
                        mine[2 * i + 1] = f2_hi(v);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xf[q]);
                    if (!warp_wait(&xf[q], (uint32_t)jt & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) return false;
                    const float* other = (half == 0 ? xu : xg) + r * 33;
                    float amax = 0.f;
                    uint64_t hv[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        // half 0: own gate f (acc[i]) with up f from the exchange; half 1: gate from the
                        // exchange with own up (acc[16 + i]), features 32 + 2i, 33 + 2i
                        const uint64_t own = acc[(half == 0 ? 0 : 16) + i];
                        const float g0 = half == 0 ? f2_lo(own) : other[2 * i], g1 = half == 0 ? f2_hi(own) : other[2 * i + 1];
                        const float u0 = half == 0 ? other[2 * i] : f2_lo(own), u1 = half == 0 ? other[2 * i + 1] : f2_hi(own);
                        const float h0 = __fmul_rn(silu_ref(g0), u0), h1 = __fmul_rn(silu_ref(g1), u1);
                        hv[i] = f2_pack(__float_as_uint(h0), __float_as_uint(h1));
                        amax = fmaxf(amax, fmaxf(fabsf(h0), fabsf(h1)));
                    }
                    xm[half * BM + r] = amax;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xa[q]);
                    if (!warp_wait(&xa[q], (uint32_t)jt & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) return false;
                    const float scale = fmaxf(__fdiv_rn(fmaxf(xm[r], xm[BM + r]), 127.f), FLT_MIN);
                    const float inv = __fdiv_rn(1.f, scale);
                    const int blk = n0 / 128;
                    if (m < M) {
                        store_codes<2>(out_codes + (size_t)m * ldoc + (size_t)blk * 64 + half * 32, hv, inv);
                        if (half == 0) out_scales[(size_t)blk * ldos + m] = scale;
                    }
                }
                return true;
            } else {
                if (y_tma) {
                    // Stage 32 rows x 16 columns per chunk in shared memory and hand them to the TMA:
                    // a coalesced store (y = acc) or an in-L2 reduce-add (y = y + acc, round to
                    // nearest, y never read here).  Rows/columns past M/N are clipped by the TMA.
                    const float nanv = __int_as_float(0x7fc00000);
                    const uint32_t ystage = smem_u32(smem + S::OFF_Y) + ew * S::Y_BUFS * S::Y_CHUNK;
#pragma unroll
                    for (int c = 0; c < COLS / 16; ++c) {
                        const uint32_t buf = ystage + ybuf * S::Y_CHUNK;
                        if (lane == 0) bulk_wait_group_read<S::Y_BUFS - 1>();  // this buffer's last store read it
                        __syncwarp();
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint64_t p0 = acc[c * 8 + 2 * i], p1 = acc[c * 8 + 2 * i + 1];
                            uint4 o = make_uint4((uint32_t)p0, (uint32_t)(p0 >> 32), (uint32_t)p1, (uint32_t)(p1 >> 32));
                            if (add_bias) {
                                // y = sum + bias[n] (or + 0), decima/int8.rs:492-496
                                const int nb = n0 + col0 + c * 16 + 4 * i;
                                o.x = __float_as_uint(__fadd_rn(__uint_as_float(o.x), bias && nb < N ? __ldg(bias + nb) : 0.f));
                                o.y = __float_as_uint(__fadd_rn(__uint_as_float(o.y), bias && nb + 1 < N ? __ldg(bias + nb + 1) : 0.f));
                                o.z = __float_as_uint(__fadd_rn(__uint_as_float(o.z), bias && nb + 2 < N ? __ldg(bias + nb + 2) : 0.f));
                                o.w = __float_as_uint(__fadd_rn(__uint_as_float(o.w), bias && nb + 3 < N ? __ldg(bias + nb + 3) : 0.f));
                            }
                            if (any_nonfinite) o = make_uint4(__float_as_uint(nanv), __float_as_uint(nanv),
                                                              __float_as_uint(nanv), __float_as_uint(nanv));
                            sts128(buf + lane * 64 + i * 16, o);
                        }
                        fence_proxy_async_smem();  // generic writes of the staging buffer -> TMA reads
                        __syncwarp();
                        if (lane == 0) {
                            if (EPI == DB_EPI_RESIDUAL) tma_reduce_add_2d(&tmY, buf, n0 + col0 + c * 16, m0 + q * 32);
                            else tma_store_2d(&tmY, buf, n0 + col0 + c * 16, m0 + q * 32);
                            bulk_commit_group();
                        }
                        if (++ybuf == S::Y_BUFS) ybuf = 0;
                    }
                } else if (m < M) {
                    float* dst = y + (size_t)m * ldy + n0 + col0;
                    const float nanv = __int_as_float(0x7fc00000);
#pragma unroll
                    for (int j = 0; j < COLS; ++j) {
                        if (n0 + col0 + j < N) {
                            float o = (j & 1) ? f2_hi(acc[j / 2]) : f2_lo(acc[j / 2]);
                            if (add_bias) o = __fadd_rn(o, bias ? __ldg(bias + n0 + col0 + j) : 0.f);
                            if (EPI == DB_EPI_RESIDUAL) o = __fadd_rn(dst[j], o);
                            dst[j] = any_nonfinite ? nanv : o;
                        }
                    }
                }
                return true;
            }
        };
        // Jobs are handled in steps of JPS = 128 / COLS (4 at 64-wide tiles, 2 at 128-wide, 1 at
        // 256-wide): one wait for the step's last job (commits complete in issue order, so the
        // earlier ones are done too), all of the step's accumulators loaded under one wait (128
        // registers; 256-wide tiles in two halves of 64 columns), the buffers handed back to the MMA
        // issuer as soon as their values are in registers, then the folds in job order and the
        // scale slots returned.  Steps never cross a tile.
        constexpr int JPS = COLS >= 128 ? 1 : 128 / COLS;  // jobs per step
        constexpr int NH = COLS > 64 ? COLS / 64 : 1;       // loads per job (256-wide tiles: 2)
        constexpr int HC = COLS / NH;                       // columns per load (32 or 64)
        auto release_buf = [&](int jn) {
            if (PAIR) mbar_arrive_cluster(at_leader(&acc_empty[jn % S::NBUF]));
            else mbar_arrive(&acc_empty[jn % S::NBUF]);
        };
        for (int tile = tile0, jn = 0, jt = 0; tile < tiles; tile += tstride, ++jt) {
            const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN;
            uint64_t acc[COLS / 2];
#pragma unroll
            for (int j = 0; j < COLS / 2; ++j) acc[j] = 0ull;
            for (int j = 0; j < GS;) {
                // a whole step, or the tile's last jobs one at a time
                const int nj = (JPS > 1 && GS - j >= JPS) ? JPS : 1;
                if (!wait_job(jn + nj - 1)) goto done;
                tc_fence_after();
                if (JPS > 1 && nj == JPS) {
                    uint32_t v[JPS][COLS];
#pragma unroll
                    for (int q = 0; q < JPS; ++q)
                        load_cols<COLS>(tlane + (uint32_t)(((jn + q) % S::NBUF) * BN), v[q]);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < JPS; ++q) tie_cols<COLS>(v[q]);
                    // every column of the step's jobs is in registers: their buffers are free
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        for (int q = 0; q < JPS; ++q) release_buf(jn + q);
#pragma unroll
                    for (int q = 0; q < JPS; ++q) {
                        const uint32_t slot = sc_base + ((jn + q) % S::SCJ) * S::SC_SLOT;
                        const float s_a = lds_f32(slot + r * 4);
                        const uint32_t wsc = slot + BM * 4 + col0 * 4;
#pragma unroll
                        for (int c = 0; c < COLS / 16; ++c)
                            fold16<FUSED>(&acc[c * 8], *reinterpret_cast<const uint32_t(*)[16]>(&v[q][16 * c]),
                                          wsc + 64 * c, s_a);
                    }
                } else {
                    const uint32_t tb = tlane + (uint32_t)((jn % S::NBUF) * BN);
                    const uint32_t slot = sc_base + (jn % S::SCJ) * S::SC_SLOT;
                    const float s_a = lds_f32(slot + r * 4);
                    const uint32_t wsc = slot + BM * 4 + col0 * 4;
#pragma unroll
                    for (int h = 0; h < NH; ++h) {
                        uint32_t v[HC];
                        load_cols<HC>(tb + (uint32_t)(h * HC), v);
                        tmem_wait_ld();
                        tie_cols<HC>(v);
                        if (h == NH - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) release_buf(jn);
                        }
#pragma unroll
                        for (int c = 0; c < HC / 16; ++c)
                            fold16<FUSED>(&acc[(h * HC) / 2 + c * 8], *reinterpret_cast<const uint32_t(*)[16]>(&v[16 * c]),
                                          wsc + (h * HC + 16 * c) * 4, s_a);
                    }
                }
                __syncwarp();  // every lane has read the step's scale slots
                if (lane == 0)
                    for (int q = 0; q < nj; ++q) mbar_arrive(&sc_empty[(jn + q) % S::SCJ]);
                jn += nj;
                j += nj;
            }
            if (!finish_tile(acc, m0, n0, jt)) goto done;
        }
    }
done:
    if (warp >= EPI_WARP0) tmem_wait_ld();  // tensor-memory loads this warp issued have completed
    bulk_wait_all();  // output stores issued by this thread have completed
    // Teardown through mbarriers (a hardware CTA barrier reached from the different role branches
    // was measured to release some warps before the others arrived): warp 1 frees tensor memory
    // once every warp has arrived; in pair mode it first trades a signal with the other CTA's
    // warp 1, so neither CTA leaves while the other may still arrive on its barriers or have its
    // shared memory read by the pair's MMAs.  Every wait above is bounded, so all warps get here.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(end_bar(0));
    if (warp == 1) {
        if (lane == 0) {
            // the other warps may still be finishing their last tile
            mbar_wait_drain(end_bar(0), 0, DB_WAIT_LIMIT_NS);
            if (PAIR) {
                mbar_arrive_cluster(mapa_shared(smem_u32(end_bar(1)), cluster_ctarank() ^ 1u));
                mbar_wait_drain(end_bar(1), 0, DB_WAIT_LIMIT_NS);
            }
        }
        __syncwarp();
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, 512);
        else tmem_dealloc(tmem_base, 512);
    }
}

// Host side: launch one instantiation (tensor maps built by the caller).
template <int BN, int BITS, int EPI, bool FUSED, bool PAIR, int SUB>
int launch(const DbGemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmY, int y_tma,
           int G, cudaStream_t stream) {
    using S = Smem<BN, BITS, EPI, PAIR>;
    auto kernel = gemm_i8_kernel<BN, BITS, EPI, FUSED, PAIR, SUB>;
    {
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), S::BYTES);
        if (e != cudaSuccess) return (int)e;
    }
    constexpr int MT = PAIR ? 2 * BM : BM;
    const int tiles = ((a.M + MT - 1) / MT) * ((a.N + BN - 1) / BN);
    int units = a.max_ctas > 0 ? a.max_ctas : db_num_sms();
    if (PAIR) units /= 2;
    if (units < 1) units = 1;
    if (units > tiles) units = tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(PAIR ? 2 * units : units));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = S::BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = PAIR ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int GS = (a.K + 64 / SUB - 1) / (64 / SUB);
    const cudaError_t e = cudaLaunchKernelEx(
        &cfg, kernel, tmA, tmW, tmY, y_tma, a.sa, a.ldsa, a.sw, (int64_t)db_scale_stride(a.N), a.M, a.N, G, GS, a.y,
        a.ldy, static_cast<int8_t*>(a.out_codes), a.ldoc, a.out_scales, a.ldos, a.nonfinite, a.bias, a.add_bias,
        a.dev_error);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// Dispatch over tile width, pairing, epilogue and numerics for one weight width (one translation
// unit per width, so the instantiations compile in parallel).
struct Maps {
    CUtensorMap a, w, y;
    int y_tma;
    int G;
};
template <int BITS, int EPI, bool FUSED, int SUB>
int launch_bn(const DbGemmArgs& a, int bn, bool pair, const Maps& mp, cudaStream_t s) {
    if constexpr (EPI == DB_EPI_SWIGLU_QUANT) {
        if (bn == 128)
            return pair ? launch<128, BITS, EPI, FUSED, true, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s)
                        : launch<128, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
        return pair ? launch<256, BITS, EPI, FUSED, true, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s)
                    : launch<256, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
    } else {
        if (bn == 32) return launch<32, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
        if (bn == 64)
            return pair ? launch<64, BITS, EPI, FUSED, true, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s)
                        : launch<64, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
        if (bn == 256)
            return pair ? launch<256, BITS, EPI, FUSED, true, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s)
                        : launch<256, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
        return pair ? launch<128, BITS, EPI, FUSED, true, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s)
                    : launch<128, BITS, EPI, FUSED, false, SUB>(a, mp.a, mp.w, mp.y, mp.y_tma, mp.G, s);
    }
}

}  // namespace gi8
}  // namespace db
