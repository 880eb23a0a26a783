// Small-M grouped GEMV (decode / scoring steps): HBM-bound, weight bytes stream from HBM once.
//
// Numerics are those of the tensor-core path and of int8.rs:526-585: exact integer dots per
// 64-group (dp4a), then acc = fma(float(dot_g), sw*sa, acc) in ascending g (or the portable
// sum += dot*(sa*sw) of int8.rs:276-278 / packed.rs:111 when fused == 0).  Because every dot is an
// exact integer, who computes it does not matter: the K range is split freely across threads and
// only the final per-(row, activation row) fold runs in group order.
//
// Layout: thread t of a CTA owns the 16-byte chunk column t of every weight row (Q4: 32 codes,
// Q8: 16), so a CTA has one thread per chunk of a row (rounded up to whole warps).  The thread
// loads the matching activation codes of all MR activation rows into registers once per launch and
// reuses them for every weight row it sees.  CTAs are persistent and walk blocks of R weight rows:
// per block a thread loads its R weight chunks (R 16-byte streaming loads in flight), forms the R x
// MR chunk dots, the CPG chunks of a group are summed across neighbouring lanes and parked in
// shared memory with the block's weight scales, and after a CTA barrier one thread per (row,
// activation row) runs the sequential fold out of shared memory (the activation scales are staged
// there once per launch).  The next block's weights and weight scales are loaded before that
// barrier, so they are in flight during the fold; the parking space is double-buffered, so the
// fold of one block runs while the other warps form the next block's dots (the barrier of the
// next block orders a buffer's fold before its reuse two blocks later).
//
// The kernel is launched with programmatic dependent launch: its first weight loads (weights are
// never written by the kernel before it) go out before it waits for the previous kernel, and it
// lets the next kernel start right after them, so in a decode chain the weight streams of
// consecutive projections overlap.  Activations, activation scales and code sums are read only
// after the wait.
#include "common.cuh"
#include "kernels.h"

namespace db {

constexpr int GEMV_MAX_ROWS = 8;       // activation rows (M) handled by this path
constexpr int GEMV_MAX_GROUPS = 160;   // K <= 10240
// one thread per 16-byte chunk of a row: at K = 10240, 320 (Q4) or 640 (Q8) threads
__host__ __device__ constexpr int gemv_max_threads(int bits) { return bits == 4 ? 320 : 640; }

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
// Streaming 16-byte weight load (read once: do not keep it in L1).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Activation codes of one chunk column for one activation row, in registers.
//   Q4: 32 codes = 4 blocks of 8 in GEMV order (k0,k2,k4,k6),(k1,k3,k5,k7): 8 words.
//   Q8: 16 codes in natural order: 4 words (the upper 4 unused).
struct ActChunk {
    uint32_t w[8];
};

// Integer dot of one 16-byte weight chunk with one row's activation chunk.
//   Q4: weight bytes hold (code+8) nibbles, low = even k; the +8 offset is removed later with the
//       activation code sums.  lo / hi are the chunk's low and high nibbles (shared by every row).
//   Q8: natural order on both sides.
template <int BITS>
__device__ __forceinline__ int chunk_dot(const uint4& wv, const uint32_t (&lo)[4], const uint32_t (&hi)[4],
                                         const ActChunk& a) {
    int s = 0;
    if (BITS == 4) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            s = dp4a_su((int)a.w[2 * b], lo[b], s);
            s = dp4a_su((int)a.w[2 * b + 1], hi[b], s);
        }
    } else {
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            s = dp4a_ss((int)a.w[2 * b], (int)__byte_perm(words[2 * b], words[2 * b + 1], 0x6420), s);
            s = dp4a_ss((int)a.w[2 * b + 1], (int)__byte_perm(words[2 * b], words[2 * b + 1], 0x7531), s);
        }
    }
    return s;
}

// R weight rows per block, MR activation rows (M <= MR; rows past M are zero and not stored).
template <int BITS, int MR, int R, bool FUSED, bool RESIDUAL>
__global__ void __launch_bounds__(gemv_max_threads(BITS))
    gemv_kernel(const int8_t* __restrict__ a, int64_t lda, const float* __restrict__ sa,
                const int32_t* __restrict__ asum, int64_t ldsa, const uint8_t* __restrict__ w,
                const float* __restrict__ sw, int M, int N, int G, float* __restrict__ y, int64_t ldy,
                const int* __restrict__ nonfinite) {
    // shared memory: two buffers of (dots [R][MR][G] | sw_s [G][R]), then sa_s [G][MR]
    extern __shared__ int gemv_smem[];
    const int buf_words = (R * MR + R) * G;
    float* sa_s = reinterpret_cast<float*>(gemv_smem + 2 * buf_words);
    constexpr int CPG = BITS == 4 ? 2 : 4;            // 16-byte chunks per 64-code group
    // weight scales of a block per thread: R * G over >= CPG * G threads
    constexpr int SWPT = (R + CPG - 1) / CPG;
    constexpr int CODES = 128 / BITS;                 // codes per chunk
    const int C = G * CPG;                            // chunks per weight row
    const int c = threadIdx.x;                        // this thread's chunk column
    const bool has_chunk = c < C;
    const int64_t row_bytes = (int64_t)G * DB_GROUP * BITS / 8;
    const int64_t lds_w = db_scale_stride(N);
    const int nblocks = (N + R - 1) / R;
    auto load_block = [&](int blk, uint4 (&wv)[R], float (&swv)[SWPT]) {
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int n = blk * R + j;
            wv[j] = (has_chunk && blk < nblocks && n < N)
                        ? ld_stream(reinterpret_cast<const uint4*>(w + (size_t)n * row_bytes) + c)
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < SWPT; ++k) {
            const int i = threadIdx.x + k * (int)blockDim.x;  // (g, j) = (i / R, i % R)
            const int n = blk * R + i % R;
            swv[k] = (i < R * G && blk < nblocks && n < N) ? __ldg(sw + (size_t)(i / R) * lds_w + n) : 0.f;
        }
    };
    // the first weight loads go out before the wait for the previous kernel (the weights are not
    // among its outputs), and the next kernel may start once every CTA has issued them
    uint4 wv[R];
    float swv[SWPT];
    int blk = blockIdx.x;
    load_block(blk, wv, swv);
    pdl_trigger();
    pdl_wait();
    for (int i = threadIdx.x; i < G * MR; i += blockDim.x) {
        const int g = i / MR, r = i % MR;
        sa_s[i] = r < M ? __ldg(sa + (size_t)g * ldsa + r) : 0.f;
    }
    // this chunk column's activation codes for every activation row, and (Q4) the group's
    // code-sum correction: the weight codes were read as u = code + 8
    ActChunk act[MR];
    int corr[MR];
    const int g_own = c / CPG;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        const bool live = has_chunk && r < M;
        const int8_t* arow = a + (size_t)r * lda + (size_t)c * CODES;
        if (BITS == 4) {
            const uint4 a0 = live ? __ldg(reinterpret_cast<const uint4*>(arow)) : make_uint4(0u, 0u, 0u, 0u);
            const uint4 a1 = live ? __ldg(reinterpret_cast<const uint4*>(arow + 16)) : make_uint4(0u, 0u, 0u, 0u);
            act[r] = ActChunk{{a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w}};
        } else {
            const uint4 a0 = live ? __ldg(reinterpret_cast<const uint4*>(arow)) : make_uint4(0u, 0u, 0u, 0u);
            act[r] = ActChunk{{a0.x, a0.y, a0.z, a0.w, 0u, 0u, 0u, 0u}};
        }
        corr[r] = (BITS == 4 && live && (c % CPG) == 0) ? 8 * __ldg(asum + (size_t)g_own * ldsa + r) : 0;
    }
    const bool poisoned = nonfinite && *nonfinite;
    for (int it = 0; blk < nblocks; blk += gridDim.x, ++it) {
        int* dots = gemv_smem + (it & 1) * buf_words;
        float* sw_s = reinterpret_cast<float*>(dots + R * MR * G);
        // chunk dots of the block's R rows, summed over the CPG chunks of a group (neighbouring
        // lanes), parked for the fold
        int part[R][MR];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            uint32_t lo[4] = {0u, 0u, 0u, 0u}, hi[4] = {0u, 0u, 0u, 0u};
            if (BITS == 4) {
                const uint32_t words[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    lo[b] = words[b] & 0x0F0F0F0Fu;
                    hi[b] = (words[b] >> 4) & 0x0F0F0F0Fu;
                }
            }
#pragma unroll
            for (int r = 0; r < MR; ++r) part[j][r] = chunk_dot<BITS>(wv[j], lo, hi, act[r]);
        }
#pragma unroll
        for (int k = 0; k < SWPT; ++k) {
            const int i = threadIdx.x + k * (int)blockDim.x;
            if (i < R * G) sw_s[i] = swv[k];
        }
        // the registers are free: the next block's weights are in flight during the fold
        load_block(blk + (int)gridDim.x, wv, swv);
#pragma unroll
        for (int j = 0; j < R; ++j)
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                int v = part[j][r];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                if (CPG == 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
                part[j][r] = v;
            }
        if (has_chunk && (c % CPG) == 0) {
#pragma unroll
            for (int j = 0; j < R; ++j)
#pragma unroll
                for (int r = 0; r < MR; ++r) dots[(j * MR + r) * G + g_own] = part[j][r] - corr[r];
        }
        __syncthreads();
        // sequential fold, one thread per (output row, activation row)
        const int q = threadIdx.x;
        if (q < R * MR) {
            const int j = q / MR, r = q % MR;
            const int n = blk * R + j;
            if (r < M && n < N) {
                const int* drow = dots + (j * MR + r) * G;
                float acc = 0.f;
#pragma unroll 8
                for (int g = 0; g < G; ++g) {
                    const float d = (float)drow[g];
                    const float s_a = sa_s[g * MR + r], s_w = sw_s[g * R + j];
                    if (FUSED) acc = __fmaf_rn(d, __fmul_rn(s_w, s_a), acc);
                    else acc = __fadd_rn(acc, __fmul_rn(d, __fmul_rn(s_a, s_w)));
                }
                float* dst = y + (size_t)r * ldy + n;
                if (RESIDUAL) acc = __fadd_rn(*dst, acc);
                if (poisoned) acc = __int_as_float(0x7fc00000);
                *dst = acc;
            }
        }
    }
}

static size_t gemv_smem_bytes(int R, int MR, int G) { return (size_t)(2 * (R * MR + R) + MR) * G * 4; }

// Persistent grid: as many CTAs as fit on the SMs (at most one per block).  R = 8 rows per block
// when that still gives every resident CTA a block, else 4 (more blocks for short N); MR = 8
// always takes 4 (its R x MR partial dots and activation codes fill the registers).
template <int BITS, int MR, int R, bool FUSED, bool RESIDUAL>
static int launch_r(const DbGemvArgs& a, int G, int threads, cudaStream_t s) {
    auto kernel = gemv_kernel<BITS, MR, R, FUSED, RESIDUAL>;
    const size_t smem = gemv_smem_bytes(R, MR, G);
    cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), (int)gemv_smem_bytes(R, MR, GEMV_MAX_GROUPS));
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return (int)e;
    // every CTA walks the same number of blocks
    const int nblocks = (a.N + R - 1) / R, resident = std::max(per_sm, 1) * db_num_sms();
    const int grid = std::max(1, std::min(nblocks, resident));
    e = db_launch_pdl(kernel, dim3(grid), dim3(threads), smem, s, a.a_codes, a.lda, a.sa, a.a_sums, a.ldsa,
                      a.w_codes, a.sw, a.M, a.N, G, a.y, a.ldy, a.nonfinite);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// Whether blocks of R rows give every CTA that fits on the SMs at least one block.
template <int BITS, int MR, int R, bool FUSED, bool RESIDUAL>
static bool fills(const DbGemvArgs& a, int G, int threads) {
    if (db_set_max_smem(reinterpret_cast<const void*>(gemv_kernel<BITS, MR, R, FUSED, RESIDUAL>),
                        (int)gemv_smem_bytes(R, MR, GEMV_MAX_GROUPS)) != cudaSuccess)
        return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel<BITS, MR, R, FUSED, RESIDUAL>, threads,
                                                      gemv_smem_bytes(R, MR, G)) != cudaSuccess)
        return false;
    return (a.N + R - 1) / R >= std::max(per_sm, 1) * db_num_sms();
}

template <int BITS, int MR, bool FUSED, bool RESIDUAL>
static int launch_mr(const DbGemvArgs& a, int G, cudaStream_t s) {
    const int C = G * (BITS == 4 ? 2 : 4);
    const int threads = (C + 31) / 32 * 32;
    if constexpr (MR < 8) {
        if (fills<BITS, MR, 8, FUSED, RESIDUAL>(a, G, threads))
            return launch_r<BITS, MR, 8, FUSED, RESIDUAL>(a, G, threads, s);
    }
    return launch_r<BITS, MR, 4, FUSED, RESIDUAL>(a, G, threads, s);
}

template <int BITS, bool FUSED, bool RESIDUAL>
static int launch_rows(const DbGemvArgs& a, int G, cudaStream_t s) {
    if (a.M <= 1) return launch_mr<BITS, 1, FUSED, RESIDUAL>(a, G, s);
    if (a.M <= 2) return launch_mr<BITS, 2, FUSED, RESIDUAL>(a, G, s);
    if (a.M <= 4) return launch_mr<BITS, 4, FUSED, RESIDUAL>(a, G, s);
    return launch_mr<BITS, 8, FUSED, RESIDUAL>(a, G, s);
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
        if (a.fused) return a.residual ? launch_rows<4, true, true>(a, G, stream) : launch_rows<4, true, false>(a, G, stream);
        return a.residual ? launch_rows<4, false, true>(a, G, stream) : launch_rows<4, false, false>(a, G, stream);
    }
    if (a.fused) return a.residual ? launch_rows<8, true, true>(a, G, stream) : launch_rows<8, true, false>(a, G, stream);
    return a.residual ? launch_rows<8, false, true>(a, G, stream) : launch_rows<8, false, false>(a, G, stream);
}
