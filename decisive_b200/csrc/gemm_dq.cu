// Tensor-core W4A16 / W8A16 GEMM on dequantised operands (sm_100a, tcgen05 kind::f16, f32
// accumulation over the whole K in tensor memory).
//
// Numerics ("dequantised" mode, the one the reference's GPU kernels use: its WGSL GEMMs dequantise
// each weight and accumulate in f32 over K, grouped_q4_tuned.wgsl): for every output (m, n)
//     y = sum over k of a'[m, k] * w'[n, k],   a' = f16(code_a * sa),  w' = f16(code_w * sw)
// summed by the tensor core in f32.  a' comes from the activation quantiser's DB_CODES_DQ_F16
// layout (the reference's group quantisation, then each code times its group scale, rounded to
// f16); w' from the unpack pass below.  The result differs from the reference CPU path's exact
// grouped fold (int8.rs:526-585) by the two f16 roundings per product and the summation order:
// ~1.5e-3 of the output RMS at most over the tested shapes (the contract is 2e-3).  Every tile
// configuration issues the same MMAs over the same K steps in the same order, so all
// configurations are bitwise equal to each other.
//
// Two kernels per call:
//   unpack   Q4 / Q8 device codes + f32 group scales -> w' f16 [N, Kp] (natural k order), with
//            coalesced loads and 16-byte stores; the weights stay 4 / 8 bits in HBM and
//            w' (at most tens of MB) is written to, and re-read from, the 126 MB L2.  Each weight
//            is unpacked once per call: a converter inside the GEMM would redo it for every row
//            tile (8 times at M = 1024), and clock64 traces of such a kernel (converter warps
//            writing the swizzled tile in shared memory) showed the conversion and its per-stage
//            hand-over pacing the tensor core at ~2,400 cycles per 64-k stage (MMA: 512).
//   GEMM     one CTA per SM, persistent over 128 x BN output tiles (BN = 64, 128, 256), or over
//            256 x BN tiles with CTA pairs (cta_group::2: each CTA holds 128 rows of A and BN/2
//            rows of w', the even CTA issues M = 256 MMAs; no multicast), 320 threads:
//     warp 0      TMA producer (lane 0): per stage (64 k) the A box (128 x 64 f16) and the w' box
//                 (BN x 64 f16), both with the 128-byte swizzle (UMMA K-major operands as-is)
//     warp 1      TMEM owner + MMA issuer (lane 0): four K = 16 MMAs per stage into the tile's
//                 accumulator (two buffers of BN columns, alternating by tile, so a tile's epilogue
//                 overlaps the next tile's MMAs), issued in one asm block with the stage's commit and
//                 the next stage's barrier test; one commit per tile hands the accumulator to the
//                 epilogue
//     warps 2-9   epilogue, two warps per TMEM lane quadrant: warp w reads lanes 32 (w % 4).. and
//                 half of the tile's columns, 32 at a time, and hands them to the TMA through shared
//                 memory (store, or reduce-add into y), or stores them itself where y's rows are not
//                 16-byte aligned; or (gate/up) the SwiGLU + re-quantisation of whole 64 + 64 column
//                 blocks into f16(code * scale), one block per warp
// Work units are tiles, or with k_splits = 2 (store epilogue) the two halves of each tile's K range,
// each storing its partial sum to its own [M, N] buffer; the model's RMSNorm adds them to the
// residual stream in a fixed order (deterministic, independent of the tiling).
// Every mbarrier wait is bounded (DB_WAIT_LIMIT_NS); on expiry the CTA records an error in the
// device error word, stops issuing work, lets its own copies and MMAs land and frees its tensor
// memory.  No TMA multicast.
#include <float.h>
#include <string.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace db {
namespace gdq {

constexpr int BM = 128;  // tile rows
constexpr int KS = 64;   // k per pipeline stage (one scale group): four K = 16 MMAs
constexpr int EPI_WARP0 = 2;
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_WARPS);  // 320
constexpr uint64_t DRAIN_NS = 100000000ull;
constexpr int UNPACK_CHUNKS = 4;  // 8-k chunks per thread of the unpack pass

template <int BN, bool PAIR>
struct Smem {
    static constexpr int WR = PAIR ? BN / 2 : BN;           // weight rows held by this CTA
    static constexpr int A_BYTES = BM * KS * 2;             // 16 KB f16 activation box
    static constexpr int B_BYTES = WR * KS * 2;             // f16 weight box (this CTA's rows)
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int Y_CHUNK = 32 * 16 * 4;             // 32 rows x 16 f32 columns
    static constexpr int Y_BUFS = 2;
    static constexpr int Y_BYTES = EPI_WARPS * Y_BUFS * Y_CHUNK;
    static constexpr int BUDGET = 232448 - 1024 - 1024;     // opt-in limit - alignment - barriers
    static constexpr int FIT = (BUDGET - Y_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = FIT > 8 ? 8 : FIT;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_Y = STAGES * STAGE_BYTES;
    static constexpr int OFF_BAR = (OFF_Y + Y_BYTES + 15) / 16 * 16;
    // full, empty per stage; done, acc_empty per accumulator buffer; mma_done; two teardown
    static constexpr int NUM_BARS = 2 * STAGES + 4 + 1 + 2;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;
    static_assert(STAGES >= 3, "at least three pipeline stages");
    static_assert(BYTES <= 232448, "shared memory budget");
    static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "128B-swizzled tiles need 1024-byte alignment");
};

// The f32 group scale s is carried as two f16 parts, s_hi = f16(s) and s_lo = f16(s - s_hi), and a
// code c (exact in f16) becomes fma(c, s_hi, c * s_lo): c * s_lo is ~2^-11 of the result, so the
// fma's rounding is the only one that matters -- f16(c * s) rounded once from the f32 scale, not
// from an f16 copy of it (which would add a second rounding, correlated across the group).
struct Scale2 {
    __half2 hi, lo;
};
__device__ __forceinline__ Scale2 split_scale(float s) {
    const __half h = __float2half_rn(s);
    return Scale2{__half2half2(h), __half2half2(__float2half_rn(s - __half2float(h)))};
}
__device__ __forceinline__ uint32_t scale_codes(__half2 c, Scale2 s) {
    const __half2 v = __hfma2(c, s.hi, __hmul2(c, s.lo));
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Q4: one 32-bit word of a weight row (k = 8c..8c+7, byte j = code(2j) + 8 | (code(2j+1) + 8) << 4)
// -> the eight f16 values code * s in natural k order (16 bytes).  Per pair of k: the byte is
// copied into both halves, masked to (low nibble, 16 x high nibble) under the f16 exponent bits of
// 1024, and one f16x2 fma maps (1024 + u, 1024 + 16 v) to (u - 8, v - 8) exactly.
__device__ __forceinline__ uint4 q4_word_to_f16(uint32_t w, Scale2 s) {
    const __half2 mul = __halves2half2(__ushort_as_half(0x3C00), __ushort_as_half(0x2C00));  // 1, 1/16
    const __half2 add = __halves2half2(__ushort_as_half(0xE408), __ushort_as_half(0xD480));  // -1032, -72
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = (__byte_perm(w, 0u, 0x4040u + 0x0101u * (uint32_t)j) & 0x00F0000Fu) | 0x64006400u;
        o[j] = scale_codes(__hfma2(*reinterpret_cast<const __half2*>(&u), mul, add), s);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Q8: two words of int8 codes (k = 8c..8c+3, 8c+4..8c+7) -> eight f16 values code * s, natural
// order.  code + 128 under the exponent bits of 1024 is the f16 1152 + code; subtracting 1152 is
// exact.
__device__ __forceinline__ uint4 q8_words_to_f16(uint32_t w0, uint32_t w1, Scale2 s) {
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;
    const uint32_t t[4] = {__byte_perm(x0, 0x64646464u, 0x4140u), __byte_perm(x0, 0x64646464u, 0x4342u),
                           __byte_perm(x1, 0x64646464u, 0x4140u), __byte_perm(x1, 0x64646464u, 0x4342u)};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = scale_codes(__hsub2(*reinterpret_cast<const __half2*>(&t[j]), bias), s);
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Unpack pass: a thread converts UNPACK_CHUNKS 8-k chunks of weights (16 bytes of w' each), the
// chunks UNPACK_CHUNKS x the grid's threads apart, consecutive threads consecutive chunks, so each
// round of a warp reads 128 (Q4) or 256 (Q8) contiguous bytes of codes and writes 512 contiguous
// bytes of w' [N, Kp] f16; all of a thread's loads are issued before its first conversion.  overlap = 1 (the caller guarantees that
// no kernel still running reads `out`, e.g. by alternating two buffers): the pass reads only the
// weights, so it runs while the previous kernel in the stream finishes and waits for that kernel
// only before it exits (its completion still implies the previous kernel's, so the kernels after
// it keep their ordering).
template <int BITS>
__global__ void __launch_bounds__(256) unpack_weights_kernel(const uint8_t* __restrict__ codes,
                                                             const float* __restrict__ sw, int64_t ldsw, int N,
                                                             int Kp, __half* __restrict__ out, int overlap) {
    if (!overlap) pdl_wait();
    const int per_row = Kp / 8;
    const int64_t total = (int64_t)N * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint2 v[UNPACK_CHUNKS];
    float sc[UNPACK_CHUNKS];
#pragma unroll
    for (int u = 0; u < UNPACK_CHUNKS; ++u) {
        const int64_t i = i0 + u * stride;
        v[u] = make_uint2(0u, 0u);
        sc[u] = 0.f;
        if (i < total) {
            const int n = (int)(i / per_row), c = (int)(i % per_row);
            sc[u] = __ldg(sw + (int64_t)(c / 8) * ldsw + n);
            if (BITS == 4) v[u].x = __ldg(reinterpret_cast<const uint32_t*>(codes + (size_t)n * (Kp / 2)) + c);
            else v[u] = __ldg(reinterpret_cast<const uint2*>(codes + (size_t)n * Kp) + c);
        }
    }
#pragma unroll
    for (int u = 0; u < UNPACK_CHUNKS; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < total) {
            const Scale2 s = split_scale(sc[u]);
            reinterpret_cast<uint4*>(out)[i] = BITS == 4 ? q4_word_to_f16(v[u].x, s) : q8_words_to_f16(v[u].x, v[u].y, s);
        }
    }
    if (overlap) pdl_wait();
    pdl_trigger();
}

__device__ __forceinline__ void tie32(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// One stage of the MMA issuer in one asm block: the test of the NEXT stage's full barrier goes out
// first, then the stage's four K = 16 MMAs (the first with accumulate = acc_first) and its commit,
// and only then is the test's result read, so the ~250-cycle mbarrier round trip overlaps the
// issue of the MMAs instead of preceding it (warps issue in order: a read of the result right
// after the test would stall the MMAs behind it).  Returns the next stage's test result.
__device__ __forceinline__ uint32_t umma4_f16_commit_test(uint32_t d, uint64_t a0, uint64_t a1, uint64_t a2,
                                                         uint64_t a3, uint64_t b0, uint64_t b1, uint64_t b2,
                                                         uint64_t b3, uint32_t idesc, uint32_t acc_first,
                                                         uint32_t commit_bar, uint32_t test_bar, uint32_t test_parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, t, q;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%13], %14;\n\t"
        "setp.ne.b32 p, %11, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %2, %6, %10, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %3, %7, %10, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %4, %8, %10, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %5, %9, %10, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%12];\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(ok)
        : "r"(d), "l"(a0), "l"(a1), "l"(a2), "l"(a3), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(acc_first),
          "r"(commit_bar), "r"(test_bar), "r"(test_parity)
        : "memory");
    return ok;
}

// The same for a CTA pair: four M = 256 MMAs, then a commit to this CTA's barrier and one to the
// peer CTA's barrier at the same offset (cluster address).
__device__ __forceinline__ uint32_t umma4_f16_pair_commit_test(uint32_t d, uint64_t a0, uint64_t a1, uint64_t a2,
                                                              uint64_t a3, uint64_t b0, uint64_t b1, uint64_t b2,
                                                              uint64_t b3, uint32_t idesc, uint32_t acc_first,
                                                              uint32_t commit_bar, uint32_t test_bar,
                                                              uint32_t test_parity, uint32_t peer_commit_bar) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, t, q;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%13], %14;\n\t"
        "setp.ne.b32 p, %11, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%1], %2, %6, %10, p;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%1], %3, %7, %10, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%1], %4, %8, %10, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%1], %5, %9, %10, t;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%12];\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%15];\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(ok)
        : "r"(d), "l"(a0), "l"(a1), "l"(a2), "l"(a3), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(acc_first),
          "r"(commit_bar), "r"(test_bar), "r"(test_parity), "r"(peer_commit_bar)
        : "memory");
    return ok;
}

__device__ __forceinline__ bool warp_wait_polite(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                                 int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_spin_polite(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_dq_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmY, int y_tma, float* __restrict__ y, int64_t ldy, int M,
                   int N, int G, int ksplit, __half* __restrict__ out_codes, int64_t ldoc,
                   const int* __restrict__ nonfinite, int* __restrict__ dev_error) {
    using S = Smem<BN, PAIR>;
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
    static_assert(EPI == DB_EPI_STORE || EPI == DB_EPI_RESIDUAL || (EPI == DB_EPI_SWIGLU_QUANT && BN >= 128),
                  "store, residual, or SwiGLU on whole 64 + 64 blocks");
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* full = bars;                   // stage: activation and weight boxes landed
    uint64_t* empty = full + S::STAGES;      // stage: its MMAs completed
    uint64_t* done = empty + S::STAGES;      // accumulator buffer: the tile's MMAs completed
    uint64_t* acc_empty = done + 2;          // accumulator buffer: the epilogue has read it
    uint64_t* mma_done = acc_empty + 2;      // final commit of the MMA issuer
    auto end_bar = [&](int i) { return reinterpret_cast<uint64_t*>(smem + S::OFF_BAR) + (S::NUM_BARS - 2 + i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    // Pair mode: a cluster of two CTAs computes 256 x BN tiles; CTA `rank` holds rows 128*rank.. of
    // the tile (its A box, its TMEM lanes) and weight rows (BN/2)*rank.. of it, and the even CTA
    // issues the M = 256 MMAs for both (B is read from both CTAs' shared memory; no multicast).
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    constexpr int MT = PAIR ? 2 * BM : BM;  // tile rows
    const int m_tiles = (M + MT - 1) / MT, n_tiles = (N + BN - 1) / BN;
    // Work units: a tile, or with ksplit = 2 one half of a tile's K range (its partial sum goes to
    // its own output buffer, rows s*M.., and the consumer adds the halves in a fixed order)
    const int units = m_tiles * n_tiles * ksplit;
    const int gsplit = (G + ksplit - 1) / ksplit;
    const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int row_off = (int)rank * BM, wrow_off = (int)rank * S::WR;
    // barrier addresses as the pair sees them (the leader's copies count both CTAs)
    auto at_leader = [&](uint64_t* b) { return PAIR ? mapa_shared(smem_u32(b), 0) : smem_u32(b); };
    auto at_peer = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 1); };

    if (threadIdx.x == 0) {
        constexpr int NC = PAIR ? 2 : 1;
        for (int i = 0; i < S::STAGES; ++i) {
            mbar_init(&full[i], 1);  // the leader's arrive (pair: armed with both CTAs' bytes)
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&done[i], 1);
            mbar_init(&acc_empty[i], NC * EPI_WARPS);
        }
        mbar_init(mma_done, 1);
        mbar_init(end_bar(0), NUM_THREADS / 32);
        mbar_init(end_bar(1), 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        if (y_tma) tma_prefetch_desc(&tmY);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 2 * BN);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 2 * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t st_base = smem_u32(smem + S::OFF_STAGE);
    // the next kernel may be scheduled now: it waits for this grid's completion before it reads
    // anything this kernel writes (an overlapped unpack pass writes a buffer no running GEMM reads)
    pdl_trigger();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (lane 0)
        if (lane == 0) {
            int st = 0, issued = 0;
            uint32_t ps = 0;
            for (int unit = tile0; unit < units; unit += tstride) {
                const int tile = unit / ksplit, gb = (unit % ksplit) * gsplit, ge = min(G, gb + gsplit);
                const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN + wrow_off;
                for (int g = gb; g < ge; ++g) {
                    if (!mbar_spin_polite(&empty[st], ps ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_TMA)) goto drain;
                    uint8_t* sp = smem + S::OFF_STAGE + st * S::STAGE_BYTES;
                    // full boxes are counted, also where they reach past M or N (zero fill).  Pair mode:
                    // both CTAs' loads complete on the leader's barrier, which the leader alone arms
                    // with both CTAs' bytes by a local arrive (an arrive of each CTA at cluster scope
                    // cost ~1,000 cycles per stage in clock64 traces and paced the pair).  A peer's
                    // bytes may land before the leader arms the phase: the phase still waits for the
                    // leader's arrive, and the peer loads a stage only after the MMAs of its previous
                    // use completed, so the bytes always belong to the current phase.
                    if (PAIR) {
                        if (leader) mbar_arrive_expect_tx(&full[st], 2 * S::STAGE_BYTES);
                        tma_load_2d_pair(sp, &tmA, at_leader(&full[st]), g * KS, m0);
                        tma_load_2d_pair(sp + S::A_BYTES, &tmW, at_leader(&full[st]), g * KS, n0);
                    } else {
                        mbar_arrive_expect_tx(&full[st], S::STAGE_BYTES);
                        tma_load_2d(sp, &tmA, &full[st], g * KS, m0);
                        tma_load_2d(sp + S::A_BYTES, &tmW, &full[st], g * KS, n0);
                    }
                    ++issued;
                    if (++st == S::STAGES) { st = 0; ps ^= 1u; }
                }
            }
            goto prod_done;
        drain:
            // after an abort: let the stages this lane issued land before the CTA winds down
            for (int k = 0; k < issued && k < S::STAGES; ++k) {
                if (st == 0) { st = S::STAGES - 1; ps ^= 1u; } else --st;
                if (leader) mbar_wait_drain(&full[st], ps, DRAIN_NS);
            }
        prod_done:;
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (lane 0)
        // Descriptors are built once and advanced by the stage / k offsets (start address field in
        // 16-byte units; shared memory is below 256 KB, so the 14-bit field never carries).
        constexpr uint32_t IDESC = idesc_f16_f32(MT, BN);
        if (leader && lane == 0) {
            const uint64_t a_desc0 = sw128_desc(st_base), b_desc0 = sw128_desc(st_base + S::A_BYTES);
            int st = 0, t = 0;
            uint32_t ps = 0, ready = 0;  // ready: the result of the current stage's early test
            for (int unit = tile0; unit < units; unit += tstride, ++t) {
                const int b = t & 1;
                const int gb = (unit % ksplit) * gsplit, ge = min(G, gb + gsplit);
                if (!mbar_spin(&acc_empty[b], (uint32_t)(t >> 1) & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA))
                    goto mma_end;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(b * BN);
                for (int g = gb; g < ge; ++g) {
                    if (!ready && !mbar_spin(&full[st], ps, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA)) goto mma_end;
                    tc_fence_after();
                    const uint64_t off = (uint64_t)((st * S::STAGE_BYTES) >> 4);
                    // the stage's four K = 16 MMAs (32 bytes along the row each; a unit's first MMA
                    // starts from zero) and the commit that frees the stage (pair: in both CTAs),
                    // with the next stage's test issued ahead of them
                    const int st2 = st + 1 == S::STAGES ? 0 : st + 1;
                    const uint32_t ps2 = st + 1 == S::STAGES ? ps ^ 1u : ps;
                    const uint64_t ad = a_desc0 + off, bd = b_desc0 + off;
                    if constexpr (PAIR)
                        ready = umma4_f16_pair_commit_test(d, ad, ad + 2, ad + 4, ad + 6, bd, bd + 2, bd + 4, bd + 6,
                                                           IDESC, g != gb ? 1u : 0u, smem_u32(&empty[st]),
                                                           smem_u32(&full[st2]), ps2, at_peer(&empty[st]));
                    else
                        ready = umma4_f16_commit_test(d, ad, ad + 2, ad + 4, ad + 6, bd, bd + 2, bd + 4, bd + 6, IDESC,
                                                      g != gb ? 1u : 0u, smem_u32(&empty[st]), smem_u32(&full[st2]),
                                                      ps2);
                    st = st2;
                    ps = ps2;
                }
                if (PAIR) {
                    umma_commit_pair(smem_u32(&done[b]));
                    umma_commit_pair(at_peer(&done[b]));
                } else {
                    umma_commit(&done[b]);
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
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may access: rows 32q..
        const int half = (warp - EPI_WARP0) >> 2;  // which half of the tile's columns (or blocks)
        const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16);
        const bool any_nonfinite = nonfinite != nullptr && *nonfinite != 0;
        const uint32_t ystage = smem_u32(smem + S::OFF_Y) + (warp - EPI_WARP0) * S::Y_BUFS * S::Y_CHUNK;
        const uint32_t nanv = 0x7fc00000u;
        int ybuf = 0, t = 0;
        // both accumulator buffers start free (the leader's barriers count both CTAs' warps)
        auto release = [&](int b) {
            if (PAIR) mbar_arrive_cluster(at_leader(&acc_empty[b]));
            else mbar_arrive(&acc_empty[b]);
        };
        if (lane == 0) {
            release(0);
            release(1);
        }
        for (int unit = tile0; unit < units; unit += tstride, ++t) {
            const int b = t & 1;
            const int tile = unit / ksplit, split = unit % ksplit;
            const int m0 = (tile % m_tiles) * MT + row_off, n0 = (tile / m_tiles) * BN;
            if (!warp_wait_polite(&done[b], (uint32_t)(t >> 1) & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI))
                goto epi_done;
            tc_fence_after();
            if constexpr (EPI == DB_EPI_SWIGLU_QUANT) {
                // The columns are blocks of 64 gate rows followed by the 64 matching up rows
                // (db_interleave_gate_up), so a thread holds whole blocks of its row: h = silu(gate) *
                // up for the block's 64 features (cpu.rs:513-518, the correctly rounded quotient),
                // the group scale max(max|h| / 127, MIN_POSITIVE), codes clamp(rint(h / scale))
                // (int8.rs:178-202, the operations of the int8 GEMM's SwiGLU epilogue), and the
                // dequantised f16(code * scale) stored for the down projection.
                const int m = m0 + q * 32 + lane;
#pragma unroll 1
                for (int blk = half; blk < BN / 128; blk += 2) {
                    uint32_t gv[2][32], uv[2][32];
                    const uint32_t base = tlane + (uint32_t)(b * BN + blk * 128);
                    tmem_ld_32x32b_x32(base, gv[0]);
                    tmem_ld_32x32b_x32(base + 32, gv[1]);
                    tmem_ld_32x32b_x32(base + 64, uv[0]);
                    tmem_ld_32x32b_x32(base + 96, uv[1]);
                    tmem_wait_ld();
                    tie32(gv[0]);
                    tie32(gv[1]);
                    tie32(uv[0]);
                    tie32(uv[1]);
                    float amax = 0.f;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const float g = __uint_as_float(gv[h][i]);
                            const float s = __fmul_rn(g, __frcp_rn(__fadd_rn(1.f, expf(-g))));
                            const float hv = __fmul_rn(s, __uint_as_float(uv[h][i]));
                            gv[h][i] = __float_as_uint(hv);
                            amax = fmaxf(amax, fabsf(hv));
                        }
                    const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                    const float inv = __fdiv_rn(1.f, scale);
                    const int fblk = (n0 + blk * 128) / 128;  // 64-feature block of the output
                    if (m < M && fblk * 128 < N) {
                        uint4* dst = reinterpret_cast<uint4*>(out_codes + (size_t)m * ldoc + (size_t)fblk * 64);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int f = 8 * j + 2 * e;
                                const float c0 = fminf(fmaxf(rintf(__fmul_rn(__uint_as_float(gv[f >> 5][f & 31]), inv)), -127.f), 127.f);
                                const float c1 = fminf(fmaxf(rintf(__fmul_rn(__uint_as_float(gv[(f + 1) >> 5][(f + 1) & 31]), inv)), -127.f), 127.f);
                                const __half2 o = __floats2half2_rn(__fmul_rn((float)(int)c0, scale), __fmul_rn((float)(int)c1, scale));
                                w[e] = *reinterpret_cast<const uint32_t*>(&o);
                            }
                            dst[j] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
                }
                // this warp's columns are in registers (at BN = 128 the second warp of the quadrant
                // has none): hand the buffer back
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release(b);
                continue;
            }
            constexpr int CPW = BN / 64;  // 32-column chunks per warp (half of the tile's columns)
#pragma unroll 1
            for (int c = half * CPW; c < (half + 1) * CPW; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tlane + (uint32_t)(b * BN + c * 32), v);
                tmem_wait_ld();
                tie32(v);
                if (c == (half + 1) * CPW - 1) {
                    // every column of the buffer is in registers: hand it back to the MMA issuer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) release(b);
                }
                if (!y_tma) {
                    // plain stores of this thread's row: rows whose stride is not a 16-byte multiple,
                    // or the partial sums of split units (split s writes rows s*M..)
                    const int m = m0 + q * 32 + lane;
                    if (m < M) {
                        float* dst = y + ((size_t)split * M + m) * ldy;
                        const int nb = n0 + c * 32;
                        if (EPI == DB_EPI_STORE && nb + 32 <= N && ((reinterpret_cast<uintptr_t>(dst + nb) & 15) == 0)) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                uint4 o = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                                if (any_nonfinite) o = make_uint4(nanv, nanv, nanv, nanv);
                                reinterpret_cast<uint4*>(dst + nb)[j] = o;
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const int n = nb + j;
                                if (n < N) {
                                    const float o = any_nonfinite ? __uint_as_float(nanv) : __uint_as_float(v[j]);
                                    dst[n] = EPI == DB_EPI_RESIDUAL ? __fadd_rn(dst[n], o) : o;
                                }
                            }
                        }
                    }
                    continue;
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t buf = ystage + ybuf * S::Y_CHUNK;
                    if (lane == 0) bulk_wait_group_read<S::Y_BUFS - 1>();  // this buffer's last store read it
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint4 o = make_uint4(v[16 * h + 4 * i], v[16 * h + 4 * i + 1], v[16 * h + 4 * i + 2],
                                             v[16 * h + 4 * i + 3]);
                        if (any_nonfinite) o = make_uint4(nanv, nanv, nanv, nanv);
                        sts128(buf + lane * 64 + i * 16, o);
                    }
                    fence_proxy_async_smem();  // generic writes of the staging buffer -> TMA reads
                    __syncwarp();
                    const int x = n0 + c * 32 + h * 16, yrow = m0 + q * 32;
                    if (lane == 0 && x < N && yrow < M) {
                        if (EPI == DB_EPI_RESIDUAL) tma_reduce_add_2d(&tmY, buf, x, yrow);
                        else tma_store_2d(&tmY, buf, x, yrow);
                        bulk_commit_group();
                    }
                    ybuf ^= 1;
                }
            }
        }
    epi_done:
        tmem_wait_ld();
    }
    bulk_wait_all();  // output stores issued by this thread have completed
    // Teardown through mbarriers: warp 1 frees tensor memory once every warp has arrived.  Every
    // wait above is bounded, so all warps get here.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(end_bar(0));
    if (warp == 1) {
        if (lane == 0) {
            mbar_wait_drain(end_bar(0), 0, DB_WAIT_LIMIT_NS);
            if (PAIR) {
                // neither CTA leaves while the other may still arrive on its barriers or have its
                // shared memory read by the pair's MMAs
                mbar_arrive_cluster(mapa_shared(smem_u32(end_bar(1)), rank ^ 1u));
                mbar_wait_drain(end_bar(1), 0, DB_WAIT_LIMIT_NS);
            }
        }
        __syncwarp();
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, 2 * BN);
        else tmem_dealloc(tmem_base, 2 * BN);
    }
}

template <int BN, int EPI, bool PAIR>
int launch(const DbGemmArgs& a, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmY, int y_tma,
           int G, cudaStream_t stream) {
    using S = Smem<BN, PAIR>;
    auto kernel = gemm_dq_kernel<BN, EPI, PAIR>;
    {
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), S::BYTES);
        if (e != cudaSuccess) return (int)e;
    }
    constexpr int MT = PAIR ? 2 * BM : BM;
    const int ksplit = a.k_splits > 1 ? a.k_splits : 1;
    const int tiles = ((a.M + MT - 1) / MT) * ((a.N + BN - 1) / BN) * ksplit;
    int units = a.max_ctas > 0 ? a.max_ctas : db_num_sms();
    if (PAIR) units /= 2;
    if (units > tiles) units = tiles;
    if (units < 1) units = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(PAIR ? 2 * units : units));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = S::BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = PAIR ? 2 : 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmA, tmW, tmY, y_tma, a.y, a.ldy, a.M, a.N, G, ksplit,
                                             static_cast<__half*>(a.out_codes), a.ldoc, a.nonfinite, a.dev_error);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int EPI, bool PAIR>
int launch_bn(const DbGemmArgs& a, int bn, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmY,
              int y_tma, int G, cudaStream_t s) {
    if constexpr (EPI == DB_EPI_SWIGLU_QUANT) {
        if (bn == 128) return launch<128, EPI, PAIR>(a, tmA, tmW, tmY, y_tma, G, s);
        return launch<256, EPI, PAIR>(a, tmA, tmW, tmY, y_tma, G, s);
    } else {
        if (bn == 64) return launch<64, EPI, PAIR>(a, tmA, tmW, tmY, y_tma, G, s);
        if (bn == 128) return launch<128, EPI, PAIR>(a, tmA, tmW, tmY, y_tma, G, s);
        return launch<256, EPI, PAIR>(a, tmA, tmW, tmY, y_tma, G, s);
    }
}
template <int EPI>
int launch_pair(const DbGemmArgs& a, int bn, bool pair, const CUtensorMap& tmA, const CUtensorMap& tmW,
                const CUtensorMap& tmY, int y_tma, int G, cudaStream_t s) {
    return pair ? launch_bn<EPI, true>(a, bn, tmA, tmW, tmY, y_tma, G, s)
                : launch_bn<EPI, false>(a, bn, tmA, tmW, tmY, y_tma, G, s);
}

}  // namespace gdq
}  // namespace db

// Tile width of the dequantised GEMM when none is given: the widest tile that still gives at
// least 96 tiles (two thirds of the SMs); persistent CTAs overlap a tile's epilogue with the next
// tile's MMAs, so a partial last wave costs less than narrower tiles do (measured on the C2
// projections: 256 for N = 3072, 4096, 6144 at M = 1024, 64 for N = 1024).
int db_gemm_dq_default_block_n(int64_t M, int64_t N, int k_splits) {
    const int64_t mt = (M + 127) / 128, ks = k_splits > 1 ? k_splits : 1;
    for (int bn : {256, 128}) {
        if (mt * ((N + bn - 1) / bn) * ks >= 96) return bn;
    }
    return 64;
}

size_t db_gemm_dq_scratch_bytes(int64_t N, int64_t K) { return (size_t)N * ((K + 63) / 64 * 64) * 2; }

// Unpacked-weight scratch for callers that pass none: one buffer per (device, stream), kept for
// the life of the process and grown in stream order (the old buffer is freed on the same stream
// after its last use).  A stream that is being captured into a graph only reuses a buffer that is
// already large enough.
static int dq_cached_scratch(cudaStream_t stream, size_t bytes, void** out) {
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> cache;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    std::lock_guard<std::mutex> lock(mu);
    auto& slot = cache[{dev, stream}];
    if (slot.second < bytes) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &cap);
        if (e != cudaSuccess) return (int)e;
        if (cap != cudaStreamCaptureStatusNone) return (int)cudaErrorStreamCaptureUnsupported;
        if (slot.first) cudaFreeAsync(slot.first, stream);
        slot = {nullptr, 0};
        e = cudaMallocAsync(&slot.first, bytes, stream);
        if (e != cudaSuccess) return (int)e;
        slot.second = bytes;
    }
    *out = slot.first;
    return 0;
}

int db_launch_gemm_dq(const DbGemmArgs& a, cudaStream_t stream) {
    using namespace db::gdq;
    if (a.M <= 0 || a.N <= 0) return 0;
    const bool swiglu = a.epilogue == DB_EPI_SWIGLU_QUANT;
    if (a.K <= 0 || (a.bits != 4 && a.bits != 8) || (a.block != 0 && a.block != 64) ||
        (a.epilogue != DB_EPI_STORE && a.epilogue != DB_EPI_RESIDUAL && !swiglu))
        return (int)cudaErrorInvalidValue;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    const int G = (a.K + 63) / 64, Kp = G * 64;
    int bn = a.block_n ? a.block_n : db_gemm_dq_default_block_n(a.M, a.N, a.k_splits);
    if (bn != 64 && bn != 128 && bn != 256) return (int)cudaErrorInvalidValue;
    // CTA pairs (M = 256 MMAs) when asked for and there are rows for both CTAs
    const bool pair = a.pair_ctas && a.M > BM;
    // split K: two halves of every tile's K range, their partial sums stored to y rows 0..M-1 and
    // M..2M-1 (store epilogue only; y holds 2M rows)
    const bool split = a.k_splits > 1;
    if (a.k_splits < 0 || a.k_splits > 2 || (split && (a.epilogue != DB_EPI_STORE || pair || G < 2)))
        return (int)cudaErrorInvalidValue;
    if (swiglu) {
        // SwiGLU: whole blocks of 64 gate + 64 up columns per tile; out_codes f16 [M, ldoc]
        if (bn == 64) bn = 128;
        if (a.N % 128 || !a.out_codes || (reinterpret_cast<uintptr_t>(a.out_codes) & 15) || (a.ldoc & 7) ||
            a.ldoc < a.N / 2)
            return (int)cudaErrorInvalidValue;
    }
    // A rows are TMA boxes of f16 (16-byte aligned rows); codes rows are read 16 bytes at a time
    if ((reinterpret_cast<uintptr_t>(a.a_codes) & 15) || (a.lda & 7) || a.lda < Kp ||
        (reinterpret_cast<uintptr_t>(a.w_codes) & 15) || (reinterpret_cast<uintptr_t>(a.sw) & 3) ||
        (!swiglu && (!a.y || a.ldy < a.N)) || (reinterpret_cast<uintptr_t>(a.w_scratch) & 15))
        return (int)cudaErrorMisalignedAddress;
    // w' [N, Kp] f16: the caller's scratch, or the cached buffer of this device and stream
    void* scratch = a.w_scratch;
    if (!scratch && a.overlap_unpack) return (int)cudaErrorInvalidValue;  // overlap needs the caller's buffers
    if (!scratch) {
        const int e = dq_cached_scratch(stream, db_gemm_dq_scratch_bytes(a.N, a.K), &scratch);
        if (e) return e;
    }
    __half* wq = static_cast<__half*>(scratch);
    int rc = 0;
    {
        const int64_t threads = ((int64_t)a.N * (Kp / 8) + UNPACK_CHUNKS - 1) / UNPACK_CHUNKS;
        const dim3 grid((unsigned)((threads + 255) / 256));
        const cudaError_t e = a.bits == 4
                                  ? db_launch_pdl(unpack_weights_kernel<4>, grid, dim3(256), 0, stream, a.w_codes, a.sw,
                                                  (int64_t)db_scale_stride(a.N), a.N, Kp, wq, a.overlap_unpack)
                                  : db_launch_pdl(unpack_weights_kernel<8>, grid, dim3(256), 0, stream, a.w_codes, a.sw,
                                                  (int64_t)db_scale_stride(a.N), a.N, Kp, wq, a.overlap_unpack);
        rc = e != cudaSuccess ? (int)e : (int)cudaGetLastError();
    }
    CUtensorMap tmA, tmW, tmY;
    memset(&tmY, 0, sizeof(tmY));
    int y_tma = 0;
    if (!rc) {
        cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.lda * 2};
        cuuint32_t box[2] = {KS, BM};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.a_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            rc = (int)cudaErrorInvalidValue;
    }
    if (!rc) {
        cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)a.N};
        cuuint64_t strides[1] = {(cuuint64_t)Kp * 2};
        cuuint32_t box[2] = {KS, (cuuint32_t)(pair ? bn / 2 : bn)};  // this CTA's weight rows
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wq, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            rc = (int)cudaErrorInvalidValue;
    }
    // output tensor map for the TMA store / reduce-add (16-byte aligned rows; else plain stores)
    // output tensor map for the TMA store / reduce-add (16-byte aligned rows; else plain stores;
    // direct 16-byte stores from registers were measured slower for the store epilogue, 0.66 against
    // 0.60 ms of qkv per C2 step)
    if (!rc && !swiglu && !split && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && (a.ldy & 3) == 0) {
        cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.ldy * 4};
        cuuint32_t box[2] = {16, 32};
        cuuint32_t estr[2] = {1, 1};
        y_tma = enc(&tmY, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.y, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (!rc)
        rc = swiglu ? launch_pair<DB_EPI_SWIGLU_QUANT>(a, bn, pair, tmA, tmW, tmY, y_tma, G, stream)
             : a.epilogue == DB_EPI_RESIDUAL ? launch_pair<DB_EPI_RESIDUAL>(a, bn, pair, tmA, tmW, tmY, y_tma, G, stream)
                                             : launch_pair<DB_EPI_STORE>(a, bn, pair, tmA, tmW, tmY, y_tma, G, stream);
    return rc;
}
