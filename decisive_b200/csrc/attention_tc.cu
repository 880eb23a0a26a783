// Non-causal GQA attention on the 5th-generation tensor cores (tcgen05 MMAs into tensor memory,
// TMA tile loads), head_dim 128, f16 operands with f32 accumulation.  Same mathematics as the
// reference's attention core (scale * q.k, a softmax over the keys, then P.v per head in f32:
// backbone.rs:560-600).  It serves every attention call: the encoder's (items of T rows, or ragged
// sequences packed one after another, each attending to its own keys) and the decoder's (causal
// own keys after P cached prefix keys, kev/mod.rs:163-300).
//
// Decoder mode: a CTA's keys are the P prefix keys (shared by every item; their own tensor maps)
// followed by its item's own keys, causal ones only up to its query tile's diagonal; keys past the
// prefix, past the item or (causal) past the query row score -inf.  Every CTA computes one item's
// query tile against that item's keys alone, so a result does not depend on the other items of
// the batch.
//
// One CTA = 128 queries of one query head (one query per TMEM lane); keys in tiles of 128, one
// pass.  Key tiles alternate between two S buffers, two O accumulators and two softmax warpgroups
// (even / odd tiles), so the tensor pipe always holds two independent accumulation chains and each
// warpgroup runs its own online softmax over its tiles: running maximum m (scaled, log2 domain),
// P = 2^(S*c - m) rounded to f16 (c = scale * log2 e), row sum l, O += P V.  The maximum is moved
// (and O, l rescaled in place) only when a tile raises it by more than 8, so P stays below 2^8 and
// rescales are rare.  The epilogue combines the two halves: with m = max(m_even, m_odd),
// O = (O_even 2^(m_even - m) + O_odd 2^(m_odd - m)) / (l_even 2^(m_even - m) + l_odd 2^(m_odd - m)).
// The context leaves either as f32 or quantised per 64-wide group for the output projection.
//
// Warps: 0 TMA producer; 1 TMEM owner + MMA issuer (lane 0 issues); 2-3 idle; 4-7 softmax of the
// even tiles (warpgroup A); 8-11 softmax of the odd tiles (warpgroup B).  Thread (warp w, lane i)
// of a softmax warpgroup owns query row 32*(w%4)+i, its TMEM lane.  In the epilogue warpgroup A
// writes features 0-63 of the head, B features 64-127: one quantisation group each.
//
// Tensor memory (512 columns): S_even 0-127, S_odd 128-255, O_even 256-383, O_odd 384-511.
// Shared memory: the Q tile, two P tiles and a ring of four K/V tiles, 32 KB each, every tile two
// 128-byte-swizzled columns of 64 features x 128 rows.  Q, K and P are K-major UMMA operands; V is
// read as an MN-major operand straight from its natural [keys][features] layout.
#include <float.h>

#include "capi_internal.h"
#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"

namespace db {
namespace {

constexpr int AT_Q = 128;                  // queries per CTA
constexpr int AT_KT = 128;                 // keys per tile
constexpr int AT_D = 128;                  // head dimension
constexpr int AT_TILE = AT_KT * AT_D * 2;  // one f16 tile (Q, K, V or P): 32 KB
constexpr int AT_HALF = AT_TILE / 2;       // 64 features x 128 rows: one swizzle column
constexpr int AT_STAGES = 4;               // K/V ring
constexpr int AT_THREADS = 384;
constexpr int AT_SOFTMAX_WARP0 = 4;

constexpr int OFF_Q = 0;
constexpr int OFF_P = OFF_Q + AT_TILE;
constexpr int OFF_KV = OFF_P + 2 * AT_TILE;
constexpr int OFF_BAR = OFF_KV + AT_STAGES * AT_TILE;
constexpr int BAR_Q = 0;
constexpr int BAR_KV_FULL = BAR_Q + 1;                  // ring stage loaded (TMA bytes)
constexpr int BAR_KV_EMPTY = BAR_KV_FULL + AT_STAGES;   // ring stage read by its MMAs
constexpr int BAR_S_FULL = BAR_KV_EMPTY + AT_STAGES;    // S buffer b computed
constexpr int BAR_S_EMPTY = BAR_S_FULL + 2;             // S buffer b loaded into registers (4 warps)
constexpr int BAR_P_FULL = BAR_S_EMPTY + 2;             // P tile b written (4 warps)
constexpr int BAR_P_EMPTY = BAR_P_FULL + 2;             // P tile b read by its MMAs
constexpr int BAR_XCH = BAR_P_EMPTY + 2;                // (m, l) exchange between the warpgroups (8 warps)
constexpr int BAR_O_FULL = BAR_XCH + 1;                 // last P.V accumulated
constexpr int BAR_MMA_DONE = BAR_O_FULL + 1;            // every MMA issued has completed
constexpr int BAR_END = BAR_MMA_DONE + 1;               // every warp is done with tensor memory
constexpr int NUM_BARS = BAR_END + 1;
constexpr int OFF_MISC = OFF_BAR + ((NUM_BARS * 8 + 15) / 16) * 16;  // TMEM address, abort flag
constexpr int AT_SMEM = OFF_MISC + 16 + 1024;                         // + 1024-byte alignment slack
static_assert(AT_SMEM <= 232448, "shared memory budget");

constexpr uint32_t TM_S = 0, TM_O = 256;  // TMEM columns of S_even and O_even (odd: +128)
constexpr uint64_t DRAIN_NS = 100000000ull;

// K-major operand (Q, K, P): K step kk (16 features or keys) of a tile.
__device__ __forceinline__ uint32_t kmajor_step(uint32_t tile, int kk) {
    return tile + (uint32_t)((kk >> 2) * AT_HALF + (kk & 3) * 32);
}

// MN-major operand, 128-byte swizzle: rows of 128 bytes hold 64 consecutive N elements for one
// K index; 8-row atoms are 1024 bytes apart along K (stride byte offset); the next 64 N elements
// start AT_HALF bytes further (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((AT_HALF >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
        "%6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

// 2^x on the special-function unit (PTX ex2.approx, flushes subnormal results to zero).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Makes every later use of r depend on this point (placed after tcgen05.wait::ld, so the compiler
// cannot hoist a use of registers loaded by tcgen05.ld above the wait).
__device__ __forceinline__ void tie32(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Bounded wait that polls with the non-suspending test_wait: a thread suspended in try_wait was
// observed to resume 0.3-1.4 us after the phase completed, which this kernel's chain of hand-offs
// (scores -> softmax -> P -> MMA) cannot absorb.  Only one lane per warp polls.
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// 32 lanes x 32 consecutive 32-bit columns from registers into tensor memory.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Warp-wide bounded wait: lane 0 polls, the warp leaves together.
__device__ __forceinline__ bool warp_wait_at(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                             int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_spin(bar, parity, abort_flag, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// Decoder-mode parameters: P prefix keys (maps tmKp/tmVp) before the item's own keys, causal.
struct DecoderArgs {
    int dec, P, causal;
};

template <bool QUANT>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKp,
                        const __grid_constant__ CUtensorMap tmVp, int T, int Hq, int Hk, float scale_log2,
                        float* __restrict__ out, int64_t ldo, void* __restrict__ codes, int64_t ldc,
                        float* __restrict__ scales, int64_t lds, int* __restrict__ nonfinite,
                        int* __restrict__ dev_error, int codes_i8, const int* __restrict__ cu_seqlens,
                        const DecoderArgs da) {
    pdl_wait();
    // dequantised output: the next kernel is the output projection's weight unpack, which reads
    // nothing this kernel writes; let it start while this one runs
    if (codes_i8 == 2) pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, kh = h / (Hq / Hk);
    const int q0 = blockIdx.x * AT_Q;
    // Equal items: item blockIdx.z of T rows (4-D maps [B][T][H][D]).  Ragged items (cu_seqlens):
    // sequence blockIdx.z holds rows cu[z]..cu[z+1]-1 of the packed rows (maps [1][R][H][D]); its
    // keys are its own rows only.  A CTA whose query tile lies past its sequence has no work.
    int item = blockIdx.z, row0 = 0;
    int64_t obase = (int64_t)blockIdx.z * T;
    if (cu_seqlens) {
        row0 = cu_seqlens[blockIdx.z];
        T = cu_seqlens[blockIdx.z + 1] - row0;
        obase = row0;
        item = 0;
        if (q0 >= T) return;
    }
    // key tiles: npre prefix tiles (decoder mode), then nown tiles of the item's own keys (causal:
    // up to the tile holding this query tile's diagonal; AT_Q == AT_KT)
    int npre = 0, nown = (T + AT_KT - 1) / AT_KT;
    if (da.dec) {
        npre = (da.P + AT_KT - 1) / AT_KT;
        if (da.causal) nown = min(nown, q0 / AT_KT + 1);
    }
    const int nt = npre + nown;  // key tiles
    const int np = (nt + 1) / 2; // pairs of tiles (even, odd)
    const uint32_t sQ = smem_u32(smem + OFF_Q), sP = smem_u32(smem + OFF_P), sKV = smem_u32(smem + OFF_KV);

    if (threadIdx.x == 0) {
        mbar_init(&bars[BAR_Q], 1);
        for (int i = 0; i < AT_STAGES; ++i) {
            mbar_init(&bars[BAR_KV_FULL + i], 1);
            mbar_init(&bars[BAR_KV_EMPTY + i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[BAR_S_FULL + b], 1);
            mbar_init(&bars[BAR_S_EMPTY + b], 4);
            mbar_init(&bars[BAR_P_FULL + b], 4);
            mbar_init(&bars[BAR_P_EMPTY + b], 1);
        }
        mbar_init(&bars[BAR_XCH], 8);
        mbar_init(&bars[BAR_O_FULL], 1);
        mbar_init(&bars[BAR_MMA_DONE], 1);
        mbar_init(&bars[BAR_END], AT_THREADS / 32);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (npre) {
            tma_prefetch_desc(&tmKp);
            tma_prefetch_desc(&tmVp);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp < AT_SOFTMAX_WARP0) {
        if (warp == 0) {
            // ---------------------------------------------------------------- TMA producer
            // Load order = consumption order: the K tiles of pair p, then the V tiles of pair p-1, ...,
            // and last the V tiles of the last pair.
            int st = 0, issued = 0;
            uint32_t ph = 0;
            bool ok = true;
            auto load = [&](bool is_v, int tile) -> bool {
                if (!warp_wait_at(&bars[BAR_KV_EMPTY + st], ph ^ 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_TMA))
                    return false;
                if (lane == 0) {
                    const bool pre = tile < npre;
                    const CUtensorMap* map = pre ? (is_v ? &tmVp : &tmKp) : (is_v ? &tmV : &tmK);
                    const int y = pre ? tile * AT_KT : row0 + (tile - npre) * AT_KT, z = pre ? 0 : item;
                    const uint32_t dst = sKV + (uint32_t)(st * AT_TILE);
                    mbar_arrive_expect_tx(&bars[BAR_KV_FULL + st], AT_TILE);
                    tma_load_4d(dst, map, &bars[BAR_KV_FULL + st], 0, kh, y, z);
                    tma_load_4d(dst + AT_HALF, map, &bars[BAR_KV_FULL + st], 64, kh, y, z);
                }
                __syncwarp();
                ++issued;
                if (++st == AT_STAGES) {
                    st = 0;
                    ph ^= 1u;
                }
                return true;
            };
            if (lane == 0) {
                mbar_arrive_expect_tx(&bars[BAR_Q], AT_TILE);
                tma_load_4d(sQ, &tmQ, &bars[BAR_Q], 0, h, row0 + q0, item);
                tma_load_4d(sQ + AT_HALF, &tmQ, &bars[BAR_Q], 64, h, row0 + q0, item);
            }
            __syncwarp();
            for (int p = 0; p <= np && ok; ++p) {
                if (p < np)
                    for (int j = 2 * p; j < min(2 * p + 2, nt) && ok; ++j) ok = load(false, j);
                if (p > 0)
                    for (int j = 2 * p - 2; j < min(2 * p, nt) && ok; ++j) ok = load(true, j);
            }
            if (!ok && lane == 0) {
                // after an abort: let the copies this warp issued land before the CTA winds down
                mbar_wait_drain(&bars[BAR_Q], 0, DRAIN_NS);
                for (int k = 0; k < issued && k < AT_STAGES; ++k) {
                    if (st == 0) {
                        st = AT_STAGES - 1;
                        ph ^= 1u;
                    } else {
                        --st;
                    }
                    mbar_wait_drain(&bars[BAR_KV_FULL + st], ph, DRAIN_NS);
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            // ---------------------------------------------------------------- MMA issuer
            constexpr uint32_t IDESC_S = idesc_f16_f32(128, 128);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(128, 128) | (1u << 16);  // B (= V) MN-major
            int st = 0;
            uint32_t ph = 0;
            uint32_t su[2] = {0u, 0u}, pu[2] = {0u, 0u};  // uses of S buffer / P tile b so far
            // descriptors of the tiles' first K step; a K step adds a constant (addresses < 256 KB,
            // so the 14-bit start field never carries)
            const uint64_t dQ = sw128_desc(sQ), dP = sw128_desc(sP), dKV = sw128_desc(sKV),
                           dV = sw128_mn_desc(sKV);
            auto kstep = [](int kk) -> uint64_t { return (uint64_t)(((kk >> 2) * AT_HALF + (kk & 3) * 32) >> 4); };
            // The pair's n tiles take the next n ring stages.  Lanes 2t and 2t+1 poll tile t's stage
            // and its S buffer (or P tile) at the same time; the warp proceeds when all have passed.
            auto wait_pair = [&](int n, int (&slot)[2], int second, const uint32_t (&par)[2]) -> bool {
                uint64_t* bar = nullptr;
                uint32_t parity = 0;
                for (int t = 0; t < n; ++t) {
                    slot[t] = st;
                    if (lane == 2 * t) {
                        bar = &bars[BAR_KV_FULL + st];
                        parity = ph;
                    } else if (lane == 2 * t + 1) {
                        bar = &bars[second + t];
                        parity = par[t];
                    }
                    if (++st == AT_STAGES) {
                        st = 0;
                        ph ^= 1u;
                    }
                }
                const int ok = bar ? (int)mbar_spin(bar, parity, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA) : 1;
                const bool all = __all_sync(0xffffffffu, ok) != 0;
                __syncwarp();  // orders the pollers' acquires before lane 0's MMAs
                return all;
            };
            // S_t = Q K_{2p+t}^T for the pair's tiles, K steps of the two chains interleaved
            auto s_pair = [&](int p) -> bool {
                const int n = min(2, nt - 2 * p);
                int slot[2] = {0, 0};
                const uint32_t par[2] = {(su[0] & 1u) ^ 1u, (su[1] & 1u) ^ 1u};  // S buffer free
                if (!wait_pair(n, slot, BAR_S_EMPTY, par)) return false;
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t dK[2] = {dKV + (uint64_t)((slot[0] * AT_TILE) >> 4),
                                            dKV + (uint64_t)((slot[1] * AT_TILE) >> 4)};
#pragma unroll
                    for (int kk = 0; kk < AT_D / 16; ++kk)
                        for (int t = 0; t < n; ++t)
                            umma_f16(tmem + TM_S + 128u * t, dQ + kstep(kk), dK[t] + kstep(kk), IDESC_S, kk > 0);
                    for (int t = 0; t < n; ++t) {
                        umma_commit(&bars[BAR_KV_EMPTY + slot[t]]);
                        umma_commit(&bars[BAR_S_FULL + t]);
                    }
                }
                __syncwarp();
                for (int t = 0; t < n; ++t) ++su[t];
                return true;
            };
            // O_t += P_t V_{2p+t}
            auto pv_pair = [&](int p) -> bool {
                const int n = min(2, nt - 2 * p);
                int slot[2] = {0, 0};
                const uint32_t par[2] = {pu[0] & 1u, pu[1] & 1u};  // P tile written
                if (!wait_pair(n, slot, BAR_P_FULL, par)) return false;
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t dVt[2] = {dV + (uint64_t)((slot[0] * AT_TILE) >> 4),
                                             dV + (uint64_t)((slot[1] * AT_TILE) >> 4)};
#pragma unroll
                    for (int kk = 0; kk < AT_KT / 16; ++kk)
                        for (int t = 0; t < n; ++t)
                            umma_f16(tmem + TM_O + 128u * t, dP + (uint64_t)((t * AT_TILE) >> 4) + kstep(kk),
                                     dVt[t] + (uint64_t)(kk * (2048 >> 4)), IDESC_PV, p > 0 || kk > 0);
                    for (int t = 0; t < n; ++t) {
                        umma_commit(&bars[BAR_KV_EMPTY + slot[t]]);
                        umma_commit(&bars[BAR_P_EMPTY + t]);
                    }
                    if (p == np - 1) umma_commit(&bars[BAR_O_FULL]);
                }
                __syncwarp();
                for (int t = 0; t < n; ++t) ++pu[t];
                return true;
            };
            bool ok = warp_wait_at(&bars[BAR_Q], 0, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_MMA);
            // the next pair's scores are issued before this pair's P.V, so the softmax of one pair
            // overlaps the P.V of the previous
            for (int p = 0; p <= np && ok; ++p) {
                if (p < np) ok = s_pair(p);
                if (ok && p > 0) ok = pv_pair(p - 1);
            }
            // every MMA this warp issued has completed before the CTA releases tensor memory
            if (lane == 0) {
                umma_commit(&bars[BAR_MMA_DONE]);
                mbar_wait_drain(&bars[BAR_MMA_DONE], 0, DRAIN_NS);
            }
            __syncwarp();
        }
    } else {
        // ---------------------------------------------------------------- softmax + epilogue
        const int b = (warp - AT_SOFTMAX_WARP0) >> 2;  // 0: even tiles, 1: odd tiles
        const int qw = warp & 3;                       // TMEM lane quarter this warp may access
        const int row = qw * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(qw * 32) << 16;
        const uint32_t s_tm = tmem + lane_addr + TM_S + 128u * b;
        const uint32_t o_own = tmem + lane_addr + TM_O + 128u * b;
        const uint32_t p_tile = sP + (uint32_t)(b * AT_TILE);
        uint32_t su = 0, pu = 0;
        float m = -INFINITY, l = 0.f;  // running maximum (scaled, log2 domain) and row sum
        bool ok = true;
        uint32_t r[4][32];
        // own keys this row may see: [0, own_end) of the item
        const int own_end = da.dec && da.causal ? min(T, q0 + row + 1) : T;
        for (int p = 0; p < np && ok; ++p) {
            const int j = 2 * p + b;
            if (j >= nt) break;
            if (!(ok = warp_wait_at(&bars[BAR_S_FULL + b], su & 1u, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI)))
                break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(s_tm + 32u * c, r[c]);
            tmem_wait_ld(r[0]);
            tie32(r[1]);
            tie32(r[2]);
            tie32(r[3]);
            // the S buffer may be overwritten from here on
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[BAR_S_EMPTY + b]);
            ++su;
            // keys past the prefix, past the sequence end or (causal) past the query row score
            // -inf: 2^(-inf) = 0.  Every tile keeps at least its first key for every row.
            const int hi_c = j < npre ? da.P - j * AT_KT : own_end - (j - npre) * AT_KT;
            if (__any_sync(0xffffffffu, hi_c < AT_KT)) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (32 * c + i >= hi_c) r[c][i] = __float_as_uint(-INFINITY);
            }
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(r[c][i]));
            const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;  // a key is kept
            float factor = 1.f;
            if (p == 0) {
                m = mt;
            } else if (mt > m + 8.f) {
                factor = ex2(m - mt);
                m = mt;
                l *= factor;
            }
            const bool rescale = __any_sync(0xffffffffu, factor != 1.f);
            uint32_t pk[64];
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = ex2(fmaf(__uint_as_float(r[c][2 * i]), scale_log2, -m));
                    const float p1 = ex2(fmaf(__uint_as_float(r[c][2 * i + 1]), scale_log2, -m));
                    ls[2 * (i & 1)] += p0;
                    ls[2 * (i & 1) + 1] += p1;
                    pk[16 * c + i] = pack_f16x2(p0, p1);
                }
            l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
            // the previous P.V into this warpgroup's accumulator has completed: the P tile is free
            // and O is stable
            if (!(ok = warp_wait_at(&bars[BAR_P_EMPTY + b], (pu & 1u) ^ 1u, abort_flag, dev_error,
                                    DB_DEV_ERR_TIMEOUT_EPI)))
                break;
            if (rescale) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    tmem_ld_32x32b_x32(o_own + 32u * c, r[c]);
                    tmem_wait_ld(r[c]);
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[c][i] = __float_as_uint(__uint_as_float(r[c][i]) * factor);
                    tmem_st_32x32b_x32(o_own + 32u * c, r[c]);
                }
                tmem_wait_st();
            }
            // 128 keys = sixteen 16-byte chunks of 8 keys per row, 128-byte swizzle
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) {
                const uint32_t addr =
                    p_tile + (uint32_t)((cc >> 3) * AT_HALF + row * 128 + (((cc & 7) ^ (row & 7)) << 4));
                sts128(addr, make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]));
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
            tc_fence_before();         // orders the rescale's tensor-memory stores before the MMA
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[BAR_P_FULL + b]);
            ++pu;
        }
        // epilogue: the accumulators are final once the last P.V committed; every MMA has read its
        // operands by then, so the Q tile holds the (m, l) exchange
        float* xm = reinterpret_cast<float*>(smem + OFF_Q);
        if (ok) ok = warp_wait_at(&bars[BAR_O_FULL], 0, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI);
        if (ok) {
            tc_fence_after();
            xm[b * AT_Q + row] = m;
            xm[2 * AT_Q + b * AT_Q + row] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[BAR_XCH]);
            ok = warp_wait_at(&bars[BAR_XCH], 0, abort_flag, dev_error, DB_DEV_ERR_TIMEOUT_EPI);
        }
        if (ok) {
            const float m_even = xm[row], m_odd = xm[AT_Q + row];
            const float mm = fmaxf(m_even, m_odd);  // finite: every tile keeps a key
            const float f_even = ex2(m_even - mm);
            const float f_odd = nt > 1 ? ex2(m_odd - mm) : 0.f;
            const float inv = 1.f / (xm[2 * AT_Q + row] * f_even + xm[3 * AT_Q + row] * f_odd);
            const uint32_t o_tm = tmem + lane_addr + TM_O + 64u * b;  // this warpgroup's 64 features
            float v[64];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                tmem_ld_32x32b_x32(o_tm + 32u * c, r[0]);
                if (nt > 1) tmem_ld_32x32b_x32(o_tm + 128u + 32u * c, r[1]);
                tmem_wait_ld(r[0]);
                tie32(r[1]);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    v[32 * c + i] =
                        (__uint_as_float(r[0][i]) * f_even + (nt > 1 ? __uint_as_float(r[1][i]) * f_odd : 0.f)) * inv;
            }
            tc_fence_before();
            const int t = q0 + row;
            const int64_t orow = obase + t;
            if (t < T) {
                if constexpr (QUANT) {
                    // group_scale (int8.rs:305-313) and pack_bits (int8.rs:347-360) over this row's
                    // 64-wide group; codes in tensor-core order k0,k4,k1,k5,k2,k6,k3,k7 per 8 features
                    float amax = 0.f;
                    bool bad = false;
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        amax = fmaxf(amax, fabsf(v[i]));
                        bad |= !isfinite(v[i]);
                    }
                    const float scale = fmaxf(__fdiv_rn(amax, 127.f), FLT_MIN);
                    const float rinv = __fdiv_rn(1.f, scale);
                    if (codes_i8 == 2) {
                        // dequantised: f16(code * scale) in natural order (a zero code is +0)
                        __half* dst = static_cast<__half*>(codes) + orow * ldc + h * AT_D + 64 * b;
#pragma unroll
                        for (int g8 = 0; g8 < 8; ++g8) {
                            uint32_t hw[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float c0 = fminf(fmaxf(rintf(__fmul_rn(v[8 * g8 + 2 * e], rinv)), -127.f), 127.f);
                                const float c1 = fminf(fmaxf(rintf(__fmul_rn(v[8 * g8 + 2 * e + 1], rinv)), -127.f), 127.f);
                                hw[e] = pack_f16x2(__fmul_rn((float)(int)c0, scale), __fmul_rn((float)(int)c1, scale));
                            }
                            *reinterpret_cast<uint4*>(dst + 8 * g8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                        }
                    } else if (codes_i8) {
                        // int8 codes in natural order
                        int8_t* dst = static_cast<int8_t*>(codes) + orow * ldc + h * AT_D + 64 * b;
#pragma unroll
                        for (int g16 = 0; g16 < 4; ++g16) {
                            uint32_t wd[4];
#pragma unroll
                            for (int wq = 0; wq < 4; ++wq) {
                                uint32_t word = 0;
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float c = fminf(fmaxf(rintf(__fmul_rn(v[16 * g16 + 4 * wq + e], rinv)), -127.f), 127.f);
                                    word |= ((uint32_t)(int)c & 0xFFu) << (8 * e);
                                }
                                wd[wq] = word;
                            }
                            *reinterpret_cast<uint4*>(dst + 16 * g16) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                        }
                    } else {
                        __half* dst = static_cast<__half*>(codes) + orow * ldc + h * AT_D + 64 * b;
#pragma unroll
                        for (int g8 = 0; g8 < 8; ++g8) {
                            float c8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                c8[e] = fminf(fmaxf(rintf(__fmul_rn(v[8 * g8 + e], rinv)), -127.f), 127.f);
                            const uint4 w = make_uint4(pack_f16x2(c8[0], c8[4]), pack_f16x2(c8[1], c8[5]),
                                                       pack_f16x2(c8[2], c8[6]), pack_f16x2(c8[3], c8[7]));
                            *reinterpret_cast<uint4*>(dst + 8 * g8) = w;
                        }
                    }
                    scales[(size_t)(h * 2 + b) * lds + orow] = scale;
                    if (bad) atomicOr(nonfinite, 1);
                } else {
                    float* dst = out + orow * ldo + h * AT_D + 64 * b;
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        *reinterpret_cast<float4*>(dst + 4 * i) =
                            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                }
            }
        }
    }
    // Teardown through an mbarrier, not __syncthreads: a hardware CTA barrier reached from the
    // different role branches was measured (clock64 per warp) to release warps 0-3 long before the
    // softmax warps arrived, which would free tensor memory under their last reads.
    tc_fence_before();
    // Not relied on for ordering; kept because without it the compiler lays the role branches out
    // differently and the kernel runs ~40 % slower.
    __syncthreads();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[BAR_END]);
    if (warp == 1) {
        if (lane == 0) mbar_wait_drain(&bars[BAR_END], 0, DRAIN_NS);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

int make_head_map(DbEncodeTiledFn enc, CUtensorMap* map, const __half* base, int H, int T, int B) {
    cuuint64_t dims[4] = {(cuuint64_t)AT_D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)AT_D * 2, (cuuint64_t)H * AT_D * 2, (cuuint64_t)T * H * AT_D * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)AT_KT, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? 0
               : -1;
}

}  // namespace
}  // namespace db

using namespace db;

namespace {

// Output checks shared by the launchers: either out (f32, row stride ldo) or codes/scales/nonfinite
// (the context quantised for the output projection).
int check_io(const __half* q16, const __half* k16, const __half* v16, int Hq, int Hk, float* out, int64_t ldo,
             void* codes, int64_t ldc, float* scales, int* nonfinite, int codes_i8) {
    const bool quant = codes != nullptr;
    if (Hk <= 0 || Hq % Hk || Hq > 65535 || codes_i8 < 0 || codes_i8 > 2 ||
        (quant && (!scales || !nonfinite || (ldc & (codes_i8 == 1 ? 15 : 7)))) ||
        (!quant && (!out || (ldo & 3))))
        return (int)cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(q16) | reinterpret_cast<uintptr_t>(k16) | reinterpret_cast<uintptr_t>(v16)) & 15)
        return (int)cudaErrorMisalignedAddress;
    if (!quant && (reinterpret_cast<uintptr_t>(out) & 15)) return (int)cudaErrorMisalignedAddress;
    if (quant && (reinterpret_cast<uintptr_t>(codes) & 15)) return (int)cudaErrorMisalignedAddress;
    return 0;
}

int launch(const dim3& grid, const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
           const CUtensorMap& tmKp, const CUtensorMap& tmVp, int T, int Hq, int Hk, float scale, float* out,
           int64_t ldo, void* codes, int64_t ldc, float* scales, int64_t lds, int* nonfinite, int codes_i8,
           const int* cu_seqlens, const DecoderArgs& da, cudaStream_t stream) {
    int* err = db_device_error_ptr();
    if (!err) return (int)cudaErrorMemoryAllocation;
    auto kernel = codes ? attention_tc_kernel<true> : attention_tc_kernel<false>;
    {
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), AT_SMEM);
        if (e != cudaSuccess) return (int)e;
    }
    const cudaError_t e = db_launch_pdl(kernel, grid, dim3(AT_THREADS), AT_SMEM, stream, tmQ, tmK, tmV, tmKp, tmVp, T,
                                        Hq, Hk, scale * 1.4426950408889634f, out, ldo, codes, ldc, scales, lds,
                                        nonfinite, err, codes_i8, cu_seqlens, da);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace

// q16 [B*T, Hq, 128], k16/v16 [B*T, Hk, 128] (f16, 16-byte aligned); either out (f32, row stride
// ldo) or codes/scales/nonfinite (quantised for the output projection) receives the context.
int db_launch_attention_tc(const __half* q16, const __half* k16, const __half* v16, int B, int T, int Hq, int Hk,
                           float scale, float* out, int64_t ldo, void* codes, int64_t ldc, float* scales,
                           int64_t lds, int* nonfinite, cudaStream_t stream, int codes_i8) {
    if (T <= 0 || B <= 0) return 0;
    if (B > 65535) return (int)cudaErrorInvalidValue;
    if (const int rc = check_io(q16, k16, v16, Hq, Hk, out, ldo, codes, ldc, scales, nonfinite, codes_i8)) return rc;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    CUtensorMap tmQ, tmK, tmV;
    if (make_head_map(enc, &tmQ, q16, Hq, T, B) || make_head_map(enc, &tmK, k16, Hk, T, B) ||
        make_head_map(enc, &tmV, v16, Hk, T, B))
        return (int)cudaErrorInvalidValue;
    const dim3 grid((unsigned)((T + AT_Q - 1) / AT_Q), (unsigned)Hq, (unsigned)B);
    return launch(grid, tmQ, tmK, tmV, tmK, tmV, T, Hq, Hk, scale, out, ldo, codes, ldc, scales, lds, nonfinite,
                  codes_i8, nullptr, DecoderArgs{0, 0, 0}, stream);
}

// Ragged items packed one after another: R rows in total, sequence i holds rows
// cu_seqlens[i]..cu_seqlens[i+1]-1 (device array of nseq + 1 ints, cu_seqlens[nseq] = R) and attends
// to its own rows only; max_len bounds the longest sequence (sizes the grid).  Outputs as
// db_launch_attention_tc, row-indexed by the packed row.
int db_launch_attention_varlen(const __half* q16, const __half* k16, const __half* v16, const int* cu_seqlens,
                               int nseq, int max_len, int R, int Hq, int Hk, float scale, float* out, int64_t ldo,
                               void* codes, int64_t ldc, float* scales, int64_t lds, int* nonfinite,
                               cudaStream_t stream, int codes_i8) {
    if (nseq <= 0 || R <= 0 || max_len <= 0) return 0;
    if (!cu_seqlens || nseq > 65535) return (int)cudaErrorInvalidValue;
    if (const int rc = check_io(q16, k16, v16, Hq, Hk, out, ldo, codes, ldc, scales, nonfinite, codes_i8)) return rc;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    CUtensorMap tmQ, tmK, tmV;
    if (make_head_map(enc, &tmQ, q16, Hq, R, 1) || make_head_map(enc, &tmK, k16, Hk, R, 1) ||
        make_head_map(enc, &tmV, v16, Hk, R, 1))
        return (int)cudaErrorInvalidValue;
    const dim3 grid((unsigned)((max_len + AT_Q - 1) / AT_Q), (unsigned)Hq, (unsigned)nseq);
    return launch(grid, tmQ, tmK, tmV, tmK, tmV, max_len, Hq, Hk, scale, out, ldo, codes, ldc, scales, lds, nonfinite,
                  codes_i8, cu_seqlens, DecoderArgs{0, 0, 0}, stream);
}

// The decoder form: B items of T rows each (q16/k16/v16 and the outputs hold the items one after
// another); every item's keys are the P cached prefix keys kp/vp [P, Hk, 128] (shared by the items;
// P = 0: none) followed by its own T keys, which are causal (row i sees own keys 0..i) when
// causal != 0.
int db_launch_attention_decoder(const __half* q16, const __half* k16, const __half* v16, int B, int T,
                                const __half* kp, const __half* vp, int P, int causal, int Hq, int Hk, float scale,
                                float* out, int64_t ldo, void* codes, int64_t ldc, float* scales, int64_t lds,
                                int* nonfinite, cudaStream_t stream, int codes_i8) {
    if (T <= 0 || B <= 0) return 0;
    if (P < 0 || (P > 0 && (!kp || !vp)) || B > 65535) return (int)cudaErrorInvalidValue;
    if (const int rc = check_io(q16, k16, v16, Hq, Hk, out, ldo, codes, ldc, scales, nonfinite, codes_i8)) return rc;
    if (P > 0 && ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) & 15))
        return (int)cudaErrorMisalignedAddress;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    CUtensorMap tmQ, tmK, tmV, tmKp, tmVp;
    if (make_head_map(enc, &tmQ, q16, Hq, T, B) || make_head_map(enc, &tmK, k16, Hk, T, B) ||
        make_head_map(enc, &tmV, v16, Hk, T, B))
        return (int)cudaErrorInvalidValue;
    tmKp = tmK;  // no prefix: the maps are never read
    tmVp = tmV;
    if (P > 0 && (make_head_map(enc, &tmKp, kp, Hk, P, 1) || make_head_map(enc, &tmVp, vp, Hk, P, 1)))
        return (int)cudaErrorInvalidValue;
    const dim3 grid((unsigned)((T + AT_Q - 1) / AT_Q), (unsigned)Hq, (unsigned)B);
    return launch(grid, tmQ, tmK, tmV, tmKp, tmVp, T, Hq, Hk, scale, out, ldo, codes, ldc, scales, lds, nonfinite,
                  codes_i8, nullptr, DecoderArgs{1, P, causal ? 1 : 0}, stream);
}

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
    if (!codes) return (int)cudaErrorInvalidValue;
    return db_launch_attention_decoder(q16, k16, v16, B, T, kp, vp, P, causal, Hq, Hk, scale, nullptr, 0, codes, ldc,
                                       scales, lds, nonfinite, stream, codes_i8);
}
