// Tensor-core grouped W4A8 / W8A8 GEMM with fused group dequantisation (sm_100a, tcgen05).
//
// Computes, for every output (m, n), the reference's grouped sum (int8.rs:526-585):
//     acc = 0; for g ascending: acc = fma(float(dot_g), sw[n,g] * sa[m,g], acc)
// where dot_g is the exact integer dot of 64 activation codes with 64 weight codes.
//
// The integer dots come from tcgen05.mma kind::f16 on integer-valued f16 operands: every code
// is exact in f16, every product and every partial sum of one group (|sum| <= 64*127*127 < 2^24)
// is an exact f32 integer, so the tensor core returns dot_g exactly.  Each 64-wide group is one
// K-block; its dot lands in its own TMEM buffer (512 / BN buffers, at most eight) and the epilogue
// warps fold it into their register accumulators with the reference's rounding, in group order.
//
// Roles (512 threads, one CTA per SM, persistent over 128 x BN output tiles, BN = 64, 128 or 256;
// the pipeline hands work over in jobs of two K groups, one for BN = 256):
//   warp 0      TMA producer: one stage per pair of K groups, loaded by a single three-lane TMA
//               instruction (activation tiles of both groups, 128 x 64 f16 with 128B swizzle, and
//               the raw weight codes of both groups, BN rows)
//   warp 1      TMEM owner + MMA issuer (one elected lane): 4 x (128 x BN x 16) MMAs per group,
//               one combined wait (three polling lanes) and one commit per job plus the stage's
//   warps 2-5   converters (one per SM sub-partition): weight nibbles/bytes -> f16 codes in the
//               UMMA K-major SW128 layout, one B tile per group (warps 6-7 idle)
//   warps 8-15  epilogue (192 registers each through setmaxnreg): one warp polls the job barrier
//               while the others sleep in a hardware barrier; per-group scale vectors prefetched
//               with cp.async a few groups ahead, a group's TMEM columns loaded under one wait,
//               f32x2 scale fold, final store / fused SwiGLU re-quantisation
//               (grouped_q4_mlp.wgsl:83-105 semantics)
// Every mbarrier wait is bounded (DB_WAIT_LIMIT_NS); on expiry the CTA records an error in the
// device error word, stops issuing work, lets its own copies and MMAs land, and releases its
// tensor memory.
#include <float.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace db {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int CONVERTER_WARP0 = 2;
constexpr int CONVERTER_WARPS = 4;  // warps 2-5; warps 6-7 only fill their warpgroup
constexpr int EPILOGUE_WARP0 = 8;   // warps 8-15: warpgroups 2 and 3
constexpr int EPILOGUE_WARPS = 8;
constexpr int NUM_THREADS = 32 * (EPILOGUE_WARP0 + EPILOGUE_WARPS);  // 512
// Register split (setmaxnreg, per warpgroup): the launch gives every thread 65536 / 512 = 128;
// warpgroups 0-1 (producer, MMA, converters) drop to 64 and warpgroups 2-3 (epilogue) rise to
// 192, so 2 * 128 * 64 + 2 * 128 * 192 = 65536 stays within the launch's allocation.
constexpr int REGS_CONTROL = 64;
constexpr int REGS_EPILOGUE = 192;
static_assert(2 * 128 * REGS_CONTROL + 2 * 128 * REGS_EPILOGUE == 65536, "register split");
constexpr int XCH_STRIDE = 33;     // floats per row of the SwiGLU exchange buffers (bank-conflict free)
constexpr uint64_t DRAIN_NS = 100000000ull;  // wind-down wait for in-flight copies / MMAs

// The pipeline moves in jobs of GPJ K-groups (two for tiles up to 128 wide, one for 256): one
// combined wait and one or two tcgen05.commits per job in the MMA issuer, whose instruction stream
// (an MMA issue costs ~60 cycles, a commit ~100-170, a satisfied wait ~165) otherwise sets the pace.
// JS job slots hold the converted weight tiles and the TMEM accumulators of a job; one MMA commit
// per job ("done") tells both the converters (weight slot free) and the epilogue (accumulators
// ready).  A phase of done[js] cannot be skipped by any waiter: the job JS later needs the same
// weight slot and accumulator buffers, which those waiters release first.
template <int BN, int BITS, int EPI, bool PAIR, int SUB = 1>
struct GemmSmem {
    static constexpr int GPJ = BN <= 128 ? 2 : 1;          // 64-wide K slabs per job
    static constexpr int BUFS = 512 / BN > 8 ? 8 : 512 / BN;  // TMEM accumulator buffers (BUFS x BN <= 512 columns)
    static constexpr int JS = BUFS / (GPJ * SUB);           // job slots: 4 (BN 64), 2 (BN 128, 256; BN 64 with SUB 2)
    static constexpr int SC_DEPTH = BN >= 256 ? 3 : 6;      // groups of scale vectors each epilogue warp keeps in flight
    static constexpr int WR = PAIR ? BN / 2 : BN;          // weight rows held by this CTA
    static constexpr int A_BYTES = BM * BK * 2;            // one group of activation codes, 16 KB
    static constexpr int W_ROW = BK * BITS / 8;            // raw weight-code bytes per row and group
    static constexpr int WP_BYTES = WR * 2 * W_ROW;        // raw weight codes of a group pair
    static constexpr int STAGE_BYTES = (2 * A_BYTES + WP_BYTES + 1023) / 1024 * 1024;
    static constexpr int TX_BYTES = 2 * A_BYTES + WP_BYTES;  // full boxes, also for a lone tail group
    static constexpr int BG_BYTES = WR * BK * 2;           // converted f16 weight tile of one group
    static constexpr int B_SLOT = GPJ * BG_BYTES;          // converted weight tiles of one job
    static constexpr int COLS = BN / 2;                    // accumulator columns per epilogue thread
    static constexpr int SC_SLOT = (32 + COLS) * 4;        // sa of a warp's 32 rows + sw of its columns
    static constexpr int SC_BYTES = EPILOGUE_WARPS * SC_DEPTH * SC_SLOT;
    // SwiGLU exchange: 32 gate and 32 up columns per row, plus each half's row maxima
    static constexpr int XCH_BYTES = EPI == DB_EPI_SWIGLU_QUANT ? 2 * BM * XCH_STRIDE * 4 + 2 * BM * 4 : 0;
    // output staging for the TMA store: per epilogue warp one or two buffers of 32 rows x 16 f32 columns
    static constexpr int Y_CHUNK = 32 * 16 * 4;
    static constexpr int BUDGET = 232448 - 1024 - 512;     // opt-in limit - alignment slack - barriers
    static constexpr bool fits(int st, int ybufs) {
        return SC_BYTES + XCH_BYTES + (EPI == DB_EPI_SWIGLU_QUANT ? 0 : EPILOGUE_WARPS * ybufs * Y_CHUNK) +
                   st * STAGE_BYTES + JS * B_SLOT <= BUDGET;
    }
    // preference: stages (TMA lookahead) first, then double-buffered output staging
    static constexpr int STAGES = fits(4, 2) ? 4 : fits(3, 1) ? 3 : 2;
    static constexpr int Y_BUFS = fits(STAGES, 2) ? 2 : 1;
    static constexpr int Y_BYTES = EPI == DB_EPI_SWIGLU_QUANT ? 0 : EPILOGUE_WARPS * Y_BUFS * Y_CHUNK;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_B = OFF_STAGE + STAGES * STAGE_BYTES;
    static constexpr int OFF_SC = OFF_B + JS * B_SLOT;
    static constexpr int OFF_X = OFF_SC + SC_BYTES;
    static constexpr int OFF_Y = OFF_X + XCH_BYTES;
    static constexpr int OFF_BAR = (OFF_Y + Y_BYTES + 15) / 16 * 16;
    static constexpr int NUM_BARS = 3 * STAGES + 3 * JS + 6;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;     // + alignment slack
    static_assert(fits(STAGES, Y_BUFS) && BYTES <= 232448, "shared memory budget");
    static_assert(STAGE_BYTES % 1024 == 0 && BG_BYTES % 1024 == 0, "SW128 tiles need 1024-byte alignment");
    static_assert(JS >= 2, "job slots must double-buffer");
};

// Warp-wide bounded wait.  Only lane 0 polls the barrier (32 pollers per warp would flood the
// shared-memory barrier unit that every role's waits go through); the other lanes are released by
// the __syncwarp, which also orders their later accesses after lane 0's acquire.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}
__device__ __forceinline__ bool warp_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_backoff(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
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
    // cpu.rs:513-518: x * (1 / (1 + exp(-x))); the correctly rounded reciprocal is exactly the
    // correctly rounded quotient 1 / y
    return __fmul_rn(x, __frcp_rn(__fadd_rn(1.f, expf(-x))));
}

// Folds NC columns of one group into NC / 2 packed accumulator pairs:
//   fused:    acc = fma(d, sw * sa, acc)     (AVX2 path, int8.rs:566-572)
//   portable: acc = acc + d * (sa * sw)      (int8.rs:259-287)
// w holds the 16 weight scales of these columns (the same for every lane).
template <bool FUSED, int NC>
__device__ __forceinline__ void fold_cols(uint64_t* acc, const uint32_t (&v)[NC], const uint4 (&w)[NC / 4], float s_a) {
    const uint64_t sa2 = f2_pack(__float_as_uint(s_a), __float_as_uint(s_a));
#pragma unroll
    for (int i = 0; i < NC / 4; ++i) {
        const int j = 4 * i;
        if (FUSED) {
            acc[j / 2] = f2_fma(f2_pack(v[j], v[j + 1]), f2_mul(f2_pack(w[i].x, w[i].y), sa2), acc[j / 2]);
            acc[j / 2 + 1] = f2_fma(f2_pack(v[j + 2], v[j + 3]), f2_mul(f2_pack(w[i].z, w[i].w), sa2), acc[j / 2 + 1]);
        } else {
            // scalar: the packed add/mul pair does not reproduce the reference's rounding here
            const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                uint64_t& a = acc[(j + e) / 2];
                const float lo = __fadd_rn(f2_lo(a), __fmul_rn(__uint_as_float(v[j + e]),
                                                               __fmul_rn(s_a, __uint_as_float(ww[e]))));
                const float hi = __fadd_rn(f2_hi(a), __fmul_rn(__uint_as_float(v[j + e + 1]),
                                                               __fmul_rn(s_a, __uint_as_float(ww[e + 1]))));
                a = f2_pack(__float_as_uint(lo), __float_as_uint(hi));
            }
        }
    }
}

// SwiGLU finish, in slices.  pend holds a thread's 32 own values of a tile (gate for half 0, up
// for half 1) and receives h = silu(gate) * up in place; other_row holds the other half's values.
template <int B>
__device__ __forceinline__ void swiglu_silu4(uint64_t (&pend)[16], const float* other_row, int half, float& amax) {
#pragma unroll
    for (int j = B; j < B + 4; ++j) {
        uint64_t& p = pend[j / 2];
        const float own = (j & 1) ? f2_hi(p) : f2_lo(p);
        const float oth = other_row[j];
        const float h = __fmul_rn(silu_ref(half == 0 ? own : oth), half == 0 ? oth : own);
        p = (j & 1) ? f2_pack(__float_as_uint(f2_lo(p)), __float_as_uint(h))
                    : f2_pack(__float_as_uint(h), __float_as_uint(f2_hi(p)));
        amax = fmaxf(amax, fabsf(h));
    }
}
// int8 codes (as f16, TC order 0,4,1,5,2,6,3,7) of features B..B+7.
template <int B>
__device__ __forceinline__ void swiglu_store8(const uint64_t (&pend)[16], float inv, __half* dst) {
    const int order[8] = {0, 4, 1, 5, 2, 6, 3, 7};
    __half hv[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const int j = B + order[p];
        const float h = (j & 1) ? f2_hi(pend[j / 2]) : f2_lo(pend[j / 2]);
        hv[p] = __float2half_rn(fminf(fmaxf(rintf(__fmul_rn(h, inv)), -127.f), 127.f));
    }
    *reinterpret_cast<uint4*>(dst + B) = *reinterpret_cast<uint4*>(hv);
}

template <int BN, int BITS, int EPI, bool FUSED, bool PAIR, int SUB>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmY, int y_tma,
                   const float* __restrict__ sa, int64_t ldsa, const float* __restrict__ sw, int64_t ldsw, int M,
                   int N, int G, int GS, float* __restrict__ y, int64_t ldy, __half* __restrict__ out_codes, int64_t ldoc,
                   float* __restrict__ out_scales, int64_t ldos, const int* __restrict__ nonfinite,
                   const float* __restrict__ bias, int add_bias, int* __restrict__ dev_error) {
    using S = GemmSmem<BN, BITS, EPI, PAIR, SUB>;
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* full = bars;                   // stage loaded (TMA tx)
    uint64_t* empty = full + S::STAGES;      // stage released by the MMA commit
    uint64_t* wfull = empty + S::STAGES;     // pair mode: this CTA's raw weight codes loaded
    uint64_t* b_full = wfull + S::STAGES;    // job slot: converted weight tiles ready (4 converter warps)
    uint64_t* done = b_full + S::JS;         // job slot: the job's MMAs completed (weights free, accumulators ready)
    uint64_t* acc_empty = done + S::JS;      // job slot: the epilogue has read the accumulators
    uint64_t* xch_full = acc_empty + S::JS;  // SwiGLU exchange: both halves' columns published
    uint64_t* xch_empty = xch_full + 1;      // every epilogue warp is done with this tile's exchange
    uint64_t* xch_amax = xch_empty + 1;      // both halves' row maxima published
    uint64_t* mma_done = xch_amax + 1;       // final commit of the MMA issuer
    // the last two barriers (teardown): every warp of this CTA is done with tensor memory and its
    // copies; pair mode: the other CTA of the pair is done.  Addressed from the shared-memory base
    // where used, so no register holds them through the main loops.
    auto end_bar = [&](int i) { return reinterpret_cast<uint64_t*>(smem + S::OFF_BAR) + (S::NUM_BARS - 2 + i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    // Pair mode: a cluster of two CTAs computes 256 x BN tiles; CTA `rank` owns rows 128*rank.. of
    // the tile and weight rows (BN/2)*rank.. of it, the even CTA issues the M = 256 MMAs.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    constexpr int MT = PAIR ? 2 * BM : BM;    // tile rows
    const int m_tiles = (M + MT - 1) / MT, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int row_off = (int)rank * BM, wrow_off = (int)rank * S::WR;
    // barrier addresses as the pair sees them (rank-0 copies for the leader-counted barriers)
    auto at_leader = [&](uint64_t* b) { return PAIR ? mapa_shared(smem_u32(b), 0) : smem_u32(b); };
    auto at_peer = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 1); };

    if (threadIdx.x == 0) {
        constexpr int NC = PAIR ? 2 : 1;  // leader-counted barriers hear from both CTAs
        for (int i = 0; i < S::STAGES; ++i) {
            mbar_init(&full[i], NC);
            mbar_init(&empty[i], 1);
            mbar_init(&wfull[i], 1);
        }
        for (int i = 0; i < S::JS; ++i) {
            mbar_init(&b_full[i], NC * CONVERTER_WARPS);
            mbar_init(&done[i], 1);
            mbar_init(&acc_empty[i], NC * EPILOGUE_WARPS);
        }
        mbar_init(xch_full, EPILOGUE_WARPS);
        mbar_init(xch_empty, EPILOGUE_WARPS);
        mbar_init(xch_amax, EPILOGUE_WARPS);
        mbar_init(mma_done, 1);
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
            tmem_alloc_pair(tmem_slot, S::BUFS * BN);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, S::BUFS * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (warp < EPILOGUE_WARP0) {
    // warpgroups 0-1 give registers back; one instruction, executed by all eight warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CONTROL));
    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        int is = 0, issued = 0;
        uint32_t ps = 0;
        for (int tile = tile0; tile < tiles; tile += tstride) {
            const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN + wrow_off;
            for (int g = 0; g < G; g += 2) {
                if (!warp_wait_backoff(&empty[is], ps ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_TMA)) goto drain;
                uint8_t* st = smem + S::OFF_STAGE + is * S::STAGE_BYTES;
                if (PAIR) {
                    // activation tiles count on the leader's barrier (both CTAs' bytes); this CTA's
                    // weight codes on its own barrier, read by its converters
                    if (lane == 0) {
                        mbar_arrive_expect_tx_cluster(at_leader(&full[is]), 2 * S::A_BYTES);
                        mbar_arrive_expect_tx(&wfull[is], S::WP_BYTES);
                    }
                    __syncwarp();
                    if (lane < 2) tma_load_2d_pair(st + lane * S::A_BYTES, &tmA, at_leader(&full[is]), (g + lane) * BK, m0);
                    else if (lane == 2) tma_load_2d(st + 2 * S::A_BYTES, &tmW, &wfull[is], g * S::W_ROW, n0);
                } else {
                    if (lane == 0) mbar_arrive_expect_tx(&full[is], S::TX_BYTES);
                    __syncwarp();
                    // lanes 0, 1: activation tiles of groups g, g+1 (past K the box reads zeros);
                    // lane 2: raw weight codes of both groups.  One instruction, three copies.
                    if (lane < 3) {
                        const bool is_a = lane < 2;
                        tma_load_2d(st + (is_a ? lane * S::A_BYTES : 2 * S::A_BYTES), is_a ? &tmA : &tmW,
                                    &full[is], is_a ? (g + lane) * BK : g * S::W_ROW, is_a ? m0 : n0);
                    }
                }
                ++issued;
                if (++is == S::STAGES) { is = 0; ps ^= 1u; }
            }
        }
        goto done;
    drain:
        // after an abort: let the stages this warp issued land before the CTA winds down
        if (lane == 0) {
            for (int k = 0; k < issued && k < S::STAGES; ++k) {
                if (is == 0) { is = S::STAGES - 1; ps ^= 1u; } else --is;
                if (PAIR) mbar_wait_drain(&wfull[is], ps, DRAIN_NS);
                if (leader) mbar_wait_drain(&full[is], ps, DRAIN_NS);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        // The whole warp runs the loop (lane 0 polls the barriers and issues), so the warp stays
        // converged instead of idling 31 lanes at the CTA barrier.
        constexpr uint32_t IDESC = idesc_f16_f32(MT, BN);
        constexpr int GPJ = S::GPJ;
        int is = 0, js = 0;
        uint32_t ps = 0, pj = 0;
        const uint32_t st_base = smem_u32(smem + S::OFF_STAGE), b_base = smem_u32(smem + S::OFF_B);
        if (!leader) goto mma_peer;  // the even CTA issues the pair's MMAs
        for (int tile = tile0; tile < tiles; tile += tstride) {
            for (int g = 0; g < G; g += GPJ) {
                const int ng = (GPJ == 2 && g + 1 < G) ? 2 : 1;  // a lone last group past an odd G
                const bool ends_stage = ((g + ng - 1) & 1) || g + ng - 1 == G - 1;
                {
                    // lanes 0-2 poll the stage, the job slot's weight tiles and its accumulator
                    // buffers at the same time
                    const bool need = (lane == 0 && !(g & 1)) || lane == 1 || lane == 2;
                    uint64_t* bar = lane == 0 ? &full[is] : lane == 1 ? &b_full[js] : &acc_empty[js];
                    const uint32_t par = lane == 0 ? ps : lane == 1 ? pj : (pj ^ 1u);
                    const int ok = need ? (int)mbar_wait(bar, par, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA) : 1;
                    const bool all_ok = __all_sync(0xffffffffu, ok) != 0;
                    __syncwarp();  // orders the pollers' acquires before lane 0's MMAs
                    if (!all_ok) goto mma_end;
                }
                tc_fence_after();
                if (lane == 0) {
                    // MMAs that accumulate into the same TMEM buffer run one after another (~160
                    // cycles each, whatever N); the job's groups use separate buffers, so their
                    // K steps are interleaved and the two accumulation chains overlap
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
                        for (int h = 0; h < GPJ; ++h) {
                            if (h < ng) {
                                // K steps 0..4/SUB-1 of a slab go to its first scale group's buffer
                                constexpr int KPS = (BK / 16) / SUB;  // K steps per scale group
                                const uint32_t d = tmem_base + (uint32_t)((((js * GPJ + h) * SUB) + kk / KPS) * BN);
                                const uint32_t a_addr = st_base + is * S::STAGE_BYTES + ((g + h) & 1) * S::A_BYTES;
                                const uint32_t b_addr = b_base + js * S::B_SLOT + h * S::BG_BYTES;
                                const uint32_t acc_in = (kk % KPS) > 0;
                                if (PAIR) umma_f16_pair(d, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC, acc_in);
                                else umma_f16(d, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC, acc_in);
                            }
                        }
                    }
                    // one completion signal per job (both CTAs of a pair hear it), plus the stage's
                    if (PAIR) {
                        umma_commit_pair(smem_u32(&done[js]));
                        umma_commit_pair(at_peer(&done[js]));
                        if (ends_stage) {
                            umma_commit_pair(smem_u32(&empty[is]));
                            umma_commit_pair(at_peer(&empty[is]));
                        }
                    } else {
                        umma_commit(&done[js]);
                        if (ends_stage) umma_commit(&empty[is]);
                    }
                }
                __syncwarp();
                if (ends_stage) {
                    if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                }
                if (++js == S::JS) { js = 0; pj ^= 1u; }
            }
        }
    mma_end:
        // every MMA this warp issued has completed before the CTA releases tensor memory
        if (lane == 0) {
            if (PAIR) {
                umma_commit_pair(smem_u32(mma_done));
                umma_commit_pair(at_peer(mma_done));
            } else {
                umma_commit(mma_done);
            }
            mbar_wait_drain(mma_done, 0, DRAIN_NS);
        }
        __syncwarp();
        goto done;
    mma_peer:
        // the peer CTA's tensor memory is written by the leader's MMAs: wait for their last commit
        if (lane == 0) mbar_wait_drain(mma_done, 0, DRAIN_NS);
        __syncwarp();
    } else if (warp < CONVERTER_WARP0 + CONVERTER_WARPS) {
        // ---------------------------------------------------------------- converters
        constexpr int TPR = S::WR >= 128 ? 1 : 128 / S::WR;  // threads per weight row (1 or 2)
        constexpr int RPT = S::WR > 128 ? S::WR / 128 : 1;   // weight rows per thread (1 or 2)
        constexpr int WORDS = S::W_ROW / 4;        // raw 32-bit words per row and group (8 or 16)
        constexpr int WPT = WORDS / TPR;           // words per thread and row
        constexpr int CPT = 8 / TPR;               // 16-byte f16 chunks written per thread and row
        const int ct = threadIdx.x - CONVERTER_WARP0 * 32;
        const int row0 = ct / TPR, part = ct % TPR, swz = row0 & 7;  // rows row0 + 128 i share the swizzle
        const uint32_t st_base = smem_u32(smem + S::OFF_STAGE), b_base = smem_u32(smem + S::OFF_B);
        int is = 0, js = 0;
        uint32_t ps = 0, pj = 0;
        for (int tile = tile0; tile < tiles; tile += tstride) {
            for (int g = 0; g < G; g += S::GPJ) {
                const int ng = (S::GPJ == 2 && g + 1 < G) ? 2 : 1;
                if (!(g & 1) &&
                    !warp_wait_backoff(PAIR ? &wfull[is] : &full[is], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_CVT))
                    goto done;
                // the job slot's previous job (JS jobs back) has been multiplied
                if (!warp_wait_backoff(&done[js], pj ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_CVT)) goto done;
#pragma unroll
                for (int h = 0; h < S::GPJ; ++h) {
                    if (h < ng) {
#pragma unroll
                        for (int rr = 0; rr < RPT; ++rr) {
                            const int row = row0 + rr * 128;
                            const uint32_t src = st_base + is * S::STAGE_BYTES + 2 * S::A_BYTES + row * (2 * S::W_ROW) +
                                                 ((g + h) & 1) * S::W_ROW + part * WPT * 4;
                            const uint32_t dst = b_base + js * S::B_SLOT + h * S::BG_BYTES + row * 128;
                            uint32_t words[WPT];
#pragma unroll
                            for (int i = 0; i < WPT / 4; ++i) {
                                const uint4 v = lds128(src + i * 16);
                                words[4 * i] = v.x; words[4 * i + 1] = v.y; words[4 * i + 2] = v.z; words[4 * i + 3] = v.w;
                            }
#pragma unroll
                            for (int c = 0; c < CPT; ++c) {
                                const int chunk = part * CPT + c;
                                const uint4 hv =
                                    BITS == 4 ? nibbles_to_f16(words[c]) : bytes_to_f16(words[2 * c], words[2 * c + 1]);
                                sts128(dst + ((chunk ^ swz) << 4), hv);
                            }
                        }
                    }
                }
                // generic writes of the B tiles become MMA (async proxy) reads; the generic reads of
                // the raw codes are ordered before the stage's next TMA fill as well
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR) mbar_arrive_cluster(at_leader(&b_full[js]));
                    else mbar_arrive(&b_full[js]);
                }
                if (((g + ng - 1) & 1) || g + ng - 1 == G - 1) {
                    if (++is == S::STAGES) { is = 0; ps ^= 1u; }
                }
                if (++js == S::JS) { js = 0; pj ^= 1u; }
            }
        }
    }
    } else {
        // ---------------------------------------------------------------- epilogue
        // warpgroups 2-3 take the registers the control warpgroups released
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPILOGUE));
        constexpr int COLS = S::COLS;  // columns per thread: 128 (BN 256), 64 (BN 128) or 32 (BN 64)
        constexpr int LDC = BN >= 256 ? 8 : 16;  // columns per TMEM load (fewer live registers at BN 256)
        // TMEM loads per wait: a whole group's columns where the registers allow (not beside 128
        // accumulators or the SwiGLU epilogue's pending values)
        constexpr int LDN = (BN >= 256 || EPI == DB_EPI_SWIGLU_QUANT) ? 1 : COLS / LDC;
        const int ew = warp - EPILOGUE_WARP0;
        const int q = warp & 3;          // TMEM lane quadrant this warp may access
        const int half = ew >> 2;        // which half of the tile's columns
        const int r = q * 32 + lane;     // row inside the tile
        const int col0 = half * COLS;
        const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
        const uint32_t sc_base = smem_u32(smem + S::OFF_SC) + ew * S::SC_DEPTH * S::SC_SLOT;
        const bool any_nonfinite = nonfinite != nullptr && *nonfinite != 0;
        float* xch = reinterpret_cast<float*>(smem + S::OFF_X);
        // The SwiGLU epilogue has further bounded waits inside the job loop, after which a warp may
        // leave on its own; a hardware barrier there could then wait for a warp that has left.
        constexpr bool ONE_POLLER = EPI != DB_EPI_SWIGLU_QUANT;
        volatile int* epi_go = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 8);
        int jn = 0;
        // Scale vectors of one job (one group of one tile) go to the next ring slot: lanes 0-7
        // fetch the sa of this warp's 32 rows, lanes 8.. the sw of its COLS columns (16 bytes
        // each).  The prefetch cursor walks this CTA's jobs in order, SC_DEPTH jobs ahead.
        // Chunk ch = lane (and lane + 32 where 8 + COLS / 4 > 32): 0-7 sa, 8.. sw.  Weight-scale
        // chunks at or past the padded row length ldsw (columns past N in a 256-wide tile) are
        // not fetched; their columns are never stored.
        constexpr int PF_CHUNKS = 8 + COLS / 4;
        int pf_tile = tile0, pf_g = 0, pf_slot = 0;
        const float* pf_src[2] = {nullptr, nullptr};
        bool pf_on[2] = {false, false};
        auto pf_tile_start = [&]() {
            if (pf_tile < tiles) {
                const int m0 = (pf_tile % m_tiles) * MT + row_off, n0 = (pf_tile / m_tiles) * BN;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int ch = lane + 32 * h;
                    const int n = n0 + col0 + (ch - 8) * 4;
                    pf_src[h] = ch < 8 ? sa + m0 + q * 32 + ch * 4 : sw + n;
                    pf_on[h] = ch < PF_CHUNKS && (ch < 8 || n < ldsw);
                }
            }
        };
        const int64_t pf_ld[2] = {lane < 8 ? ldsa : ldsw, ldsw};
        const uint32_t pf_dst[2] = {lane < 8 ? (uint32_t)lane * 16u : 128u + (uint32_t)(lane - 8) * 16u,
                                    128u + (uint32_t)(lane + 24) * 16u};
        auto prefetch = [&]() {
            if (pf_tile < tiles) {
#pragma unroll
                for (int h = 0; h < (PF_CHUNKS > 32 ? 2 : 1); ++h) {
                    if (pf_on[h]) cp_async16(sc_base + pf_slot * S::SC_SLOT + pf_dst[h], pf_src[h]);
                    pf_src[h] += pf_ld[h];
                }
                if (++pf_g == GS) {
                    pf_g = 0;
                    pf_tile += tstride;
                    pf_tile_start();
                }
            }
            cp_async_commit();
            if (++pf_slot == S::SC_DEPTH) pf_slot = 0;
        };
        pf_tile_start();
        for (int j = 0; j < S::SC_DEPTH; ++j) prefetch();
        int js = 0, slot_i = 0, ybuf = 0;
        uint32_t pj = 0;
        bool refill = false;  // the scale slot consumed by the previous group is free to refill
        cp_async_wait<S::SC_DEPTH - 1>();
        __syncwarp();
        float s_a_next = lds_f32(sc_base + lane * 4);
        // ---- SwiGLU: a tile's finish (exchange, silu * up, row absmax, re-quantisation) is spread
        // over the groups of the next tile, where the fold leaves the epilogue warps idle time.
        // Half 0 holds the gate projection of the tile's 64 features, half 1 the up projection;
        // half 0 finishes features 0-31, half 1 features 32-63 (grouped_q4_mlp.wgsl:83-105).
        float* xg = xch;                        // gate columns 32..63, written by half 0
        float* xu = xch + BM * XCH_STRIDE;      // up columns 0..31, written by half 1
        float* xm = xch + 2 * BM * XCH_STRIDE;  // [2][BM] row maxima of each half
        uint64_t pend[16];                      // own 32 values of the pending tile, then h
        int pstep = -1, p_m = 0, p_n0 = 0, xc = 0;
        uint32_t p_par = 0;
        float p_amax = 0.f, p_scale = 0.f, p_inv = 0.f;
        auto swiglu_step = [&]() -> bool {
            const float* other_row = (half == 0 ? xu : xg) + r * XCH_STRIDE;
            switch (pstep) {
                case 0:
                    if (!warp_wait(xch_full, p_par, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) return false;
                    swiglu_silu4<0>(pend, other_row, half, p_amax);
                    break;
                case 1: swiglu_silu4<4>(pend, other_row, half, p_amax); break;
                case 2: swiglu_silu4<8>(pend, other_row, half, p_amax); break;
                case 3: swiglu_silu4<12>(pend, other_row, half, p_amax); break;
                case 4: swiglu_silu4<16>(pend, other_row, half, p_amax); break;
                case 5: swiglu_silu4<20>(pend, other_row, half, p_amax); break;
                case 6: swiglu_silu4<24>(pend, other_row, half, p_amax); break;
                case 7:
                    swiglu_silu4<28>(pend, other_row, half, p_amax);
                    xm[half * BM + r] = p_amax;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_amax);
                    break;
                case 8: {
                    if (!warp_wait(xch_amax, p_par, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) return false;
                    const float amax = fmaxf(xm[r], xm[BM + r]);
                    p_scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                    p_inv = __fdiv_rn(1.f, p_scale);
                    if (p_m < M) {
                        __half* dst = out_codes + (size_t)p_m * ldoc + (p_n0 / BN) * 64 + half * 32;
                        swiglu_store8<0>(pend, p_inv, dst);
                        swiglu_store8<8>(pend, p_inv, dst);
                    }
                    break;
                }
                default: {
                    if (p_m < M) {
                        __half* dst = out_codes + (size_t)p_m * ldoc + (p_n0 / BN) * 64 + half * 32;
                        swiglu_store8<16>(pend, p_inv, dst);
                        swiglu_store8<24>(pend, p_inv, dst);
                        if (half == 0) out_scales[(size_t)(p_n0 / BN) * ldos + p_m] = p_scale;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xch_empty);  // this warp is done reading the exchange
                    pstep = -2;
                    break;
                }
            }
            ++pstep;
            return true;
        };
        for (int tile = tile0; tile < tiles; tile += tstride) {
            const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN;
            const int m = m0 + r;
            const bool full_cols = n0 + BN <= N;
            uint64_t acc[COLS / 2];
#pragma unroll
            for (int j = 0; j < COLS / 2; ++j) acc[j] = 0ull;
            for (int g = 0; g < G; g += S::GPJ) {
                const int ng = (S::GPJ == 2 && g + 1 < G) ? 2 : 1;
                if (ONE_POLLER) {
                    // one warp polls the job's barrier; the other seven sleep in a hardware
                    // barrier.  The decision goes through shared memory (two slots, alternating by
                    // job) so that every epilogue warp leaves on the same job.
                    if (ew == 0) {
                        const bool ok = warp_wait(&done[js], pj, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI);
                        if (lane == 0) epi_go[jn & 1] = ok && !*abort_flag;
                    }
                    named_barrier_sync(1, 32 * EPILOGUE_WARPS);
                    if (!epi_go[jn & 1]) goto done;
                    ++jn;
                } else if (!warp_wait(&done[js], pj, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)) {
                    goto done;
                }
                tc_fence_after();
#pragma unroll
                for (int hs = 0; hs < S::GPJ * SUB; ++hs) {
                    const int h = hs / SUB, gi = (g + h) * SUB + hs % SUB;  // slab, scale group
                    if (h < ng && gi < GS) {
                        // the job's last scale group (past K, the last slab may hold only one)
                        const bool last = h == ng - 1 && (hs % SUB == SUB - 1 || gi + 1 == GS);
                        // This group's scale vectors landed before its s_a was read (end of the
                        // previous group).  Refill the slot the previous group used: every lane has
                        // finished reading it (the __syncwarp that ended the previous group).
                        if (refill) prefetch();
                        refill = true;
                        const uint32_t slot = sc_base + slot_i * S::SC_SLOT;
                        const float s_a = s_a_next;
                        const uint32_t tbuf = tlane + (uint32_t)((js * S::GPJ * SUB + hs) * BN);
                        // LDN TMEM loads in flight per wait; each chunk's weight scales are read
                        // from shared memory just before its fold
#pragma unroll
                        for (int c = 0; c < COLS / LDC; c += LDN) {
                            uint32_t v[LDN][LDC];
#pragma unroll
                            for (int u = 0; u < LDN; ++u) tmem_ld_32x32b(tbuf + (uint32_t)((c + u) * LDC), v[u]);
#pragma unroll
                            for (int u = 0; u < LDN; ++u) tmem_wait_ld(v[u]);
                            if (last && c + LDN == COLS / LDC) {
                                // every accumulator of this job is in registers: release its buffers
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0) {
                                    if (PAIR) mbar_arrive_cluster(at_leader(&acc_empty[js]));
                                    else mbar_arrive(&acc_empty[js]);
                                }
                            }
#pragma unroll
                            for (int u = 0; u < LDN; ++u) {
                                uint4 w[LDC / 4];
#pragma unroll
                                for (int i = 0; i < LDC / 4; ++i) w[i] = lds128(slot + 128 + (c + u) * LDC * 4 + i * 16);
                                fold_cols<FUSED, LDC>(&acc[(c + u) * LDC / 2], v[u], w, s_a);
                            }
                        }
                        if (++slot_i == S::SC_DEPTH) slot_i = 0;
                        // the next group's scale vectors: its commit group is the oldest but SC_DEPTH - 2
                        cp_async_wait<S::SC_DEPTH - 2>();
                        __syncwarp();
                        s_a_next = lds_f32(sc_base + slot_i * S::SC_SLOT + lane * 4);
                        if (EPI == DB_EPI_SWIGLU_QUANT && pstep >= 0 && !swiglu_step()) goto done;
                    }
                }
                if (++js == S::JS) { js = 0; pj ^= 1u; }
            }
            if (EPI == DB_EPI_SWIGLU_QUANT) {
                // finish the previous tile if this one was too short to absorb it
                while (pstep >= 0)
                    if (!swiglu_step()) goto done;
                // publish the columns the other half needs, once every warp is done with the
                // previous tile's exchange; keep this thread's own 32 values pending
                if (!warp_wait(xch_empty, (uint32_t)(xc & 1) ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI))
                    goto done;
                // (separate branches keep every accumulator index a compile-time constant)
                if (half == 0) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        xg[r * XCH_STRIDE + 2 * j] = f2_lo(acc[16 + j]);
                        xg[r * XCH_STRIDE + 2 * j + 1] = f2_hi(acc[16 + j]);
                        pend[j] = acc[j];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        xu[r * XCH_STRIDE + 2 * j] = f2_lo(acc[j]);
                        xu[r * XCH_STRIDE + 2 * j + 1] = f2_hi(acc[j]);
                        pend[j] = acc[16 + j];
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(xch_full);
                p_m = m;
                p_n0 = n0;
                p_par = (uint32_t)(xc & 1);
                p_amax = 0.f;
                pstep = 0;
                ++xc;
            } else if (y_tma) {
                // Stage 32 rows x 16 columns per chunk in shared memory and hand them to the TMA:
                // a coalesced store (y = acc) or an in-L2 reduce-add (y = y + acc, round to nearest,
                // so y is never read here).  Rows/columns past M/N are clipped by the TMA.
                const float nanv = __int_as_float(0x7fc00000);
                const uint32_t ystage = smem_u32(smem + S::OFF_Y) + ew * S::Y_BUFS * S::Y_CHUNK;
#pragma unroll
                for (int c = 0; c < COLS / 16; ++c) {
                    const uint32_t buf = ystage + ybuf * S::Y_CHUNK;
                    if (lane == 0) bulk_wait_group_read<S::Y_BUFS - 1>();  // this buffer's previous store has read it
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
                if (full_cols && (ldy & 3) == 0 && (N & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < COLS; j += 4) {
                        float4 o = make_float4(f2_lo(acc[j / 2]), f2_hi(acc[j / 2]), f2_lo(acc[j / 2 + 1]),
                                               f2_hi(acc[j / 2 + 1]));
                        if (add_bias) {
                            const int nb = n0 + col0 + j;
                            o.x = __fadd_rn(o.x, bias ? __ldg(bias + nb) : 0.f);
                            o.y = __fadd_rn(o.y, bias ? __ldg(bias + nb + 1) : 0.f);
                            o.z = __fadd_rn(o.z, bias ? __ldg(bias + nb + 2) : 0.f);
                            o.w = __fadd_rn(o.w, bias ? __ldg(bias + nb + 3) : 0.f);
                        }
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
                            float o = (j & 1) ? f2_hi(acc[j / 2]) : f2_lo(acc[j / 2]);
                            if (add_bias) o = __fadd_rn(o, bias ? __ldg(bias + n0 + col0 + j) : 0.f);
                            if (EPI == DB_EPI_RESIDUAL) o = __fadd_rn(dst[j], o);
                            dst[j] = any_nonfinite ? nanv : o;
                        }
                    }
                }
            }
        }
        // the last tile's pending SwiGLU finish
        if (EPI == DB_EPI_SWIGLU_QUANT)
            while (pstep >= 0)
                if (!swiglu_step()) goto done;
    }
done:
    cp_async_wait_all();
    bulk_wait_all();  // output stores issued by this thread have completed
    // Teardown through mbarriers, not __syncthreads / barrier.cluster: a hardware barrier reached
    // from the different role branches was measured (clock64 per warp) to release some warps long
    // before the others arrived.  Warp 1 frees tensor memory once every warp has arrived; in pair
    // mode it first trades a signal with the other CTA's warp 1, so neither CTA leaves while the
    // other may still arrive on its barriers or have its shared memory read by the pair's MMAs.
    // Every wait above is bounded, so all warps get here.
    tc_fence_before();
    // Not relied on for ordering (see above); kept because without it the compiler lays the role
    // branches out differently and the 256-wide epilogue spills three times as much.
    __syncthreads();
    __syncwarp();
    if (lane == 0) mbar_arrive(end_bar(0));
    if (warp == 1) {
        if (lane == 0) {
            mbar_wait_drain(end_bar(0), 0, DRAIN_NS);
            if (PAIR) {
                mbar_arrive_cluster(mapa_shared(smem_u32(end_bar(1)), cluster_ctarank() ^ 1u));
                mbar_wait_drain(end_bar(1), 0, DRAIN_NS);
            }
        }
        __syncwarp();
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, S::BUFS * BN);
        else tmem_dealloc(tmem_base, S::BUFS * BN);
    }
}

}  // namespace db

using namespace db;

DbEncodeTiledFn db_encode_tiled() {
    static DbEncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<DbEncodeTiledFn>(p);
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

template <int BN, int BITS, int EPI, bool FUSED, bool PAIR, int SUB>
static int launch_variant(const DbGemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmW,
                          const CUtensorMap& tmY, int y_tma, int G, cudaStream_t stream) {
    using S = GemmSmem<BN, BITS, EPI, PAIR, SUB>;
    auto kernel = gemm_tc_kernel<BN, BITS, EPI, FUSED, PAIR, SUB>;
    {
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), S::BYTES);
        if (e != cudaSuccess) return (int)e;
    }
    constexpr int MT = PAIR ? 2 * BM : BM;
    const int tiles = ((a.M + MT - 1) / MT) * ((a.N + BN - 1) / BN);
    int units = a.max_ctas > 0 ? a.max_ctas : db_num_sms();  // CTAs available
    if (PAIR) units /= 2;                                      // pairs available
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
    // CTAs may start on SMs the previous kernel has released; the kernel waits (pdl_wait) first
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int GS = (a.K + 64 / SUB - 1) / (64 / SUB);  // scale groups (blocks of 64 / SUB)
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmA, tmW, tmY, y_tma, a.sa, a.ldsa, a.sw,
                                             (int64_t)db_scale_stride(a.N), a.M, a.N, G, GS, a.y, a.ldy,
                                             static_cast<__half*>(a.out_codes), a.ldoc, a.out_scales, a.ldos,
                                             a.nonfinite, a.bias, a.add_bias, a.dev_error);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int BN, int BITS, int EPI, bool FUSED>
static int launch_pairing(const DbGemmArgs& a, bool pair, const CUtensorMap& tmA, const CUtensorMap& tmW,
                          const CUtensorMap& tmY, int y_tma, int G, cudaStream_t s) {
    if constexpr (BN == 128) {
        if (pair) return launch_variant<BN, BITS, EPI, FUSED, true, 1>(a, tmA, tmW, tmY, y_tma, G, s);
    }
    if constexpr (BN == 64 && BITS == 8 && EPI != DB_EPI_SWIGLU_QUANT) {
        // scale blocks of 32 (Decima int8): two scale groups per 64-wide K slab, 64-wide tiles only
        if (a.block == 32) return launch_variant<BN, BITS, EPI, FUSED, false, 2>(a, tmA, tmW, tmY, y_tma, G, s);
    }
    if (a.block == 32) return (int)cudaErrorInvalidValue;
    return launch_variant<BN, BITS, EPI, FUSED, false, 1>(a, tmA, tmW, tmY, y_tma, G, s);
}

template <int BN, int BITS>
static int dispatch_epi(const DbGemmArgs& a, bool pair, const CUtensorMap& tmA, const CUtensorMap& tmW,
                        const CUtensorMap& tmY, int y_tma, int G, cudaStream_t s) {
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) {
        // the SwiGLU epilogue pairs the 64 gate and 64 up rows of a 128-wide tile
        if constexpr (BN != 128) {
            return (int)cudaErrorInvalidValue;
        } else {
            return a.fused ? launch_pairing<BN, BITS, DB_EPI_SWIGLU_QUANT, true>(a, pair, tmA, tmW, tmY, y_tma, G, s)
                           : launch_pairing<BN, BITS, DB_EPI_SWIGLU_QUANT, false>(a, pair, tmA, tmW, tmY, y_tma, G, s);
        }
    }
    if (a.epilogue == DB_EPI_RESIDUAL)
        return a.fused ? launch_pairing<BN, BITS, DB_EPI_RESIDUAL, true>(a, pair, tmA, tmW, tmY, y_tma, G, s)
                       : launch_pairing<BN, BITS, DB_EPI_RESIDUAL, false>(a, pair, tmA, tmW, tmY, y_tma, G, s);
    return a.fused ? launch_pairing<BN, BITS, DB_EPI_STORE, true>(a, pair, tmA, tmW, tmY, y_tma, G, s)
                   : launch_pairing<BN, BITS, DB_EPI_STORE, false>(a, pair, tmA, tmW, tmY, y_tma, G, s);
}

int db_launch_gemm_tc(const DbGemmArgs& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.K <= 0 || (a.bits != 4 && a.bits != 8)) return (int)cudaErrorInvalidValue;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    const int G = (a.K + BK - 1) / BK, Kp = G * BK;
    int bn = a.block_n ? a.block_n : 128;
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) bn = 128;
    if (a.block != 0 && a.block != 64 && a.block != 32) return (int)cudaErrorInvalidValue;
    if (a.block == 32) bn = 64;  // scale blocks of 32 need eight TMEM buffers of 64 columns
    if (bn != 64 && bn != 128 && bn != 256) return (int)cudaErrorInvalidValue;
    // CTA pairs (M = 256 MMAs) for 128-wide tiles when asked for and there are rows for both CTAs
    const bool pair = bn == 128 && a.M > BM && a.pair_ctas;
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
        // a pair of K groups; in pair mode each CTA loads half of the tile's weight rows
        cuuint32_t box[2] = {(cuuint32_t)(2 * BK * a.bits / 8), (cuuint32_t)(pair ? bn / 2 : bn)};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.w_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    // output tensor map for the TMA store / reduce-add (fallback: plain per-thread stores)
    CUtensorMap tmY;
    memset(&tmY, 0, sizeof(tmY));
    int y_tma = 0;
    if (a.epilogue != DB_EPI_SWIGLU_QUANT && a.y && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ldy % 4 == 0 &&
        a.ldy >= a.N) {
        cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.ldy * 4};
        cuuint32_t box[2] = {16, 32};
        cuuint32_t estr[2] = {1, 1};
        y_tma = enc(&tmY, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.y, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (bn == 64) return a.bits == 4 ? dispatch_epi<64, 4>(a, pair, tmA, tmW, tmY, y_tma, G, stream) : dispatch_epi<64, 8>(a, pair, tmA, tmW, tmY, y_tma, G, stream);
    if (bn == 256) return a.bits == 4 ? dispatch_epi<256, 4>(a, pair, tmA, tmW, tmY, y_tma, G, stream) : dispatch_epi<256, 8>(a, pair, tmA, tmW, tmY, y_tma, G, stream);
    return a.bits == 4 ? dispatch_epi<128, 4>(a, pair, tmA, tmW, tmY, y_tma, G, stream) : dispatch_epi<128, 8>(a, pair, tmA, tmW, tmY, y_tma, G, stream);
}
