// Small-M grouped GEMV (decode / scoring steps): HBM-bound, weight bytes stream from HBM once.
//
// Numerics are those of the tensor-core path and of int8.rs:526-585: exact integer dots per
// 64-group (dp4a), then acc = fma(float(dot_g), sw*sa, acc) in ascending g (or the portable
// sum += dot*(sa*sw) of int8.rs:276-278 / packed.rs:111 when fused == 0).  Because every dot is an
// exact integer, who computes it does not matter: the K range is split freely across threads and
// only the final per-(row, activation row) fold runs in group order.
//
// Layout: a CTA owns ROWS output rows (32 at M = 1, 16 at M <= 4, 8 at M <= 8: the parked dots
// [ROWS][M][G] stay within shared memory).  Work items are (16-byte chunk of K, block of GEMV_RB
// rows): a thread loads the chunk's activation codes once (L1-resident, shared by every CTA) and
// reuses them for GEMV_RB weight rows, so activation traffic per weight byte stays low even at
// M = 8.  Partial dots of the chunks of one group are reduced across neighbouring lanes and parked
// in shared memory; after one CTA barrier, one thread per (row, activation row) runs the sequential
// fold from shared memory (weight and activation scales staged there first).
//
// The kernel is launched with programmatic dependent launch: its first weight loads (weights are
// never written by the kernel before it) go out before it waits for the previous kernel, so in a
// decode chain the weight stream of one projection overlaps the tail of the one before.
#include "common.cuh"
#include "kernels.h"

namespace db {

constexpr int GEMV_MAX_ROWS = 8;      // activation rows (M) handled by this path
constexpr int GEMV_RB = 4;            // output rows sharing one activation load
// output rows per CTA for MR activation rows
__host__ __device__ constexpr int gemv_rows(int mr) { return mr == 1 ? 32 : mr <= 4 ? 16 : 8; }
constexpr int GEMV_MAX_THREADS = 512;  // block size grows with K: items per CTA = 2 * chunks per row
constexpr int GEMV_MAX_GROUPS = 160;  // K <= 10240
constexpr int GEMV_BATCH = 2;         // items whose weight loads are in flight together

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

// Integer dot of one 16-byte weight chunk with the matching activation codes of one row.
//   Q4: 32 codes = 4 blocks of 8; weight bytes hold (code+8) nibbles, low = even k; activations
//       in GEMV order (k0,k2,k4,k6),(k1,k3,k5,k7) per block.  The +8 offset is removed later with
//       the activation code sums.
//   Q8: 16 codes = 2 blocks of 8, natural order on both sides.
template <int BITS>
__device__ __forceinline__ int chunk_dot(const uint4& wv, const int8_t* arow) {
    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
    int s = 0;
    if (BITS == 4) {
        const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(arow));
        const uint4 a1 = __ldg(reinterpret_cast<const uint4*>(arow + 16));
        const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            s = dp4a_su((int)av[2 * b], words[b] & 0x0F0F0F0Fu, s);
            s = dp4a_su((int)av[2 * b + 1], (words[b] >> 4) & 0x0F0F0F0Fu, s);
        }
    } else {
        const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(arow));
        const uint32_t av[4] = {a0.x, a0.y, a0.z, a0.w};
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            s = dp4a_ss((int)av[2 * b], (int)__byte_perm(words[2 * b], words[2 * b + 1], 0x6420), s);
            s = dp4a_ss((int)av[2 * b + 1], (int)__byte_perm(words[2 * b], words[2 * b + 1], 0x7531), s);
        }
    }
    return s;
}

template <int BITS, int MR, bool FUSED, bool RESIDUAL>
__global__ void __launch_bounds__(GEMV_MAX_THREADS)
    gemv_kernel(const int8_t* __restrict__ a, int64_t lda, const float* __restrict__ sa,
                const int32_t* __restrict__ asum, int64_t ldsa, const uint8_t* __restrict__ w,
                const float* __restrict__ sw, int M, int N, int G, float* __restrict__ y, int64_t ldy,
                const int* __restrict__ nonfinite) {
    // dynamic shared memory, sized by G:
    //   dots [GEMV_ROWS][MR][G] | sw_s [G][GEMV_ROWS] | sa_s [G][MR] | corr_s [G][MR]
    constexpr int GEMV_ROWS = gemv_rows(MR);
    extern __shared__ int gemv_smem[];
    int* dots = gemv_smem;
    float* sw_s = reinterpret_cast<float*>(gemv_smem + GEMV_ROWS * MR * G);
    float* sa_s = sw_s + G * GEMV_ROWS;
    int* corr_s = reinterpret_cast<int*>(sa_s + G * MR);
    constexpr int CPG = BITS == 4 ? 2 : 4;            // 16-byte chunks per 64-code group
    constexpr int CODES = 128 / BITS;                 // codes per chunk
    constexpr int RBLKS = GEMV_ROWS / GEMV_RB;
    const int n0 = blockIdx.x * GEMV_ROWS;
    const int C = G * CPG;                            // chunks per weight row (even)
    const int64_t row_bytes = (int64_t)G * DB_GROUP * BITS / 8;
    const int64_t lds_w = db_scale_stride(N);
    const int items = RBLKS * C;
    // item = rb * C + c; consecutive threads take consecutive chunks, so the CPG chunks of one
    // group sit on neighbouring lanes of one warp (C and the warp size are multiples of CPG)
    auto load_batch = [&](int base, uint4 (&wv)[GEMV_BATCH][GEMV_RB]) {
#pragma unroll
        for (int b = 0; b < GEMV_BATCH; ++b) {
            const int it = base + b * (int)blockDim.x + threadIdx.x;
            const int rb = it / C, c = it % C;
#pragma unroll
            for (int j = 0; j < GEMV_RB; ++j) {
                const int n = n0 + rb * GEMV_RB + j;
                wv[b][j] = (it < items && n < N)
                               ? ld_stream(reinterpret_cast<const uint4*>(w + (size_t)n * row_bytes) + c)
                               : make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    // the first weight loads go out before anything else -- before the wait for the previous kernel
    // (the weights are not among its outputs) -- so their HBM latency overlaps that kernel's tail
    // and the staging of the scales and code sums below
    uint4 wv[GEMV_BATCH][GEMV_RB];
    load_batch(0, wv);
    pdl_wait();
    for (int i = threadIdx.x; i < G * GEMV_ROWS; i += blockDim.x) {
        const int g = i / GEMV_ROWS, j = i % GEMV_ROWS;
        sw_s[i] = n0 + j < N ? __ldg(sw + (size_t)g * lds_w + n0 + j) : 0.f;
    }
    for (int i = threadIdx.x; i < G * MR; i += blockDim.x) {
        const int g = i / MR, r = i % MR;
        sa_s[i] = r < M ? __ldg(sa + (size_t)g * ldsa + r) : 0.f;
        corr_s[i] = (BITS == 4 && r < M) ? 8 * __ldg(asum + (size_t)g * ldsa + r) : 0;  // codes were u = code + 8
    }
    __syncthreads();
    for (int base = 0; base < items; base += (int)blockDim.x * GEMV_BATCH) {
        if (base > 0) load_batch(base, wv);
#pragma unroll
        for (int b = 0; b < GEMV_BATCH; ++b) {
            const int it = base + b * (int)blockDim.x + threadIdx.x;
            const int rb = it / C, c = it % C;
            const bool valid = it < items;
            int part[GEMV_RB][MR];
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                const bool act = valid && r < M;
                const int8_t* arow = a + (size_t)r * lda + (size_t)c * CODES;
#pragma unroll
                for (int j = 0; j < GEMV_RB; ++j) part[j][r] = act ? chunk_dot<BITS>(wv[b][j], arow) : 0;
            }
            // reduce the CPG chunks of one group (neighbouring lanes); all lanes take part
#pragma unroll
            for (int j = 0; j < GEMV_RB; ++j)
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    int v = part[j][r];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    if (CPG == 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
                    part[j][r] = v;
                }
            if (valid && (c % CPG) == 0) {
                const int g = c / CPG;
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    if (r >= M) continue;
                    const int corr = corr_s[g * MR + r];
#pragma unroll
                    for (int j = 0; j < GEMV_RB; ++j) dots[((rb * GEMV_RB + j) * MR + r) * G + g] = part[j][r] - corr;
                }
            }
        }
    }
    __syncthreads();
    // sequential fold, one thread per (output row, activation row)
    if (threadIdx.x < GEMV_ROWS * MR) {
        const int j = threadIdx.x / MR, r = threadIdx.x % MR;
        const int n = n0 + j;
        if (r < M && n < N) {
            float acc = 0.f;
#pragma unroll 8
            for (int g = 0; g < G; ++g) {
                const float d = (float)dots[(j * MR + r) * G + g];
                const float s_a = sa_s[g * MR + r], s_w = sw_s[g * GEMV_ROWS + j];
                if (FUSED) acc = __fmaf_rn(d, __fmul_rn(s_w, s_a), acc);
                else acc = __fadd_rn(acc, __fmul_rn(d, __fmul_rn(s_a, s_w)));
            }
            float* dst = y + (size_t)r * ldy + n;
            if (RESIDUAL) acc = __fadd_rn(*dst, acc);
            if (nonfinite && *nonfinite) acc = __int_as_float(0x7fc00000);
            *dst = acc;
        }
    }
}

template <int BITS, int MR, bool FUSED, bool RESIDUAL>
static int launch_mr(const DbGemvArgs& a, int G, cudaStream_t s) {
    constexpr int GEMV_ROWS = gemv_rows(MR);
    auto kernel = gemv_kernel<BITS, MR, FUSED, RESIDUAL>;
    {
        const int max_bytes = (GEMV_ROWS * MR + GEMV_ROWS + 2 * MR) * GEMV_MAX_GROUPS * 4;
        const cudaError_t e = db_set_max_smem(reinterpret_cast<const void*>(kernel), max_bytes);
        if (e != cudaSuccess) return (int)e;
    }
    const size_t bytes = (size_t)(GEMV_ROWS * MR + GEMV_ROWS + 2 * MR) * G * 4;
    dim3 grid((a.N + GEMV_ROWS - 1) / GEMV_ROWS);
    // enough threads for about two items each (long rows get wider CTAs), at least one per fold chain
    const int items = (GEMV_ROWS / GEMV_RB) * G * (BITS == 4 ? 2 : 4);
    int threads = 128;
    while (threads < GEMV_MAX_THREADS && threads * GEMV_BATCH < items) threads *= 2;
    const cudaError_t e = db_launch_pdl(kernel, grid, dim3(threads), bytes, s, a.a_codes, a.lda, a.sa, a.a_sums,
                                        a.ldsa, a.w_codes, a.sw, a.M, a.N, G, a.y, a.ldy, a.nonfinite);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int BITS, bool FUSED, bool RESIDUAL>
static int launch_rows(const DbGemvArgs& a, int G, cudaStream_t s) {
    if (a.M <= 1) return launch_mr<BITS, 1, FUSED, RESIDUAL>(a, G, s);
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
