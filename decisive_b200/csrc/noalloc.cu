// Allocation-free variant of the full projection (db_linear_g64_noalloc).
//
// Some hosts hand this library device pointers but do not let it allocate device memory on its
// own: an engine that owns a fixed device-memory budget and accounts for every byte, or a caller
// on a latency-critical path that must never hit cudaMalloc (it can synchronise the device and
// its cost is unbounded).  Such callers cannot provide the workspace db_linear_g64 asks for
// either, when they cannot size it up front.  This entry point instead uses one scratch array
// compiled into the library: a file-scope __device__ array of DB_NOALLOC_SCRATCH_BYTES that
// every GPU which loads the library holds until the process exits.
//
// Rules of use:
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress with
//     that device current) and caches it; make that first call before any stream capture.
//   * The array is shared by every call on the device and keeps the last call's contents; the
//     entry point clears what must start at zero (the non-finite flag) itself.  Calls whose work
//     overlaps on the GPU (different streams, no ordering between them) race on the array and
//     must be serialised by the caller.
//   * Shapes whose scratch does not fit are rejected (status DB_ERR_INVALID_ARGUMENT, code
//     SCRATCH_LIMIT); nothing is allocated, ever: no cudaMalloc, cudaFree or allocating library
//     routine is called.
//   * The GEMM's bounded waits report an expiry in a second compiled-in word (g_noalloc_error),
//     not in the allocated word behind db_device_error_word(); db_linear_noalloc_error_word()
//     reads and clears it.  Calls never clear it themselves, so an expiry stays visible until read.
#include <mutex>
#include <string>
#include <vector>

#include "../../include/decisive_b200.h"
#include "capi_internal.h"
#include "common.cuh"
#include "kernels.h"

namespace {

// 8 MiB; the carve is noalloc_need() below (e.g. M = 1024 rows fit up to K = 3840, M = 4096 up
// to K = 960: the f16 codes dominate).
constexpr size_t kScratchBytes = DB_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) uint8_t g_scratch[kScratchBytes];
// device error word of the GEMM launched from this entry point (bounded-wait expiries)
__device__ int g_noalloc_error;

std::mutex g_mu;
struct Symbols {
    uint8_t* scratch = nullptr;  // device address of g_scratch (nullptr = not looked up)
    int* error = nullptr;        // device address of g_noalloc_error
};
std::vector<Symbols> g_addr;  // per device

// Device addresses of g_scratch and g_noalloc_error for the current device.  In host code these
// names are only host-side stand-ins for the symbols, never device addresses.
const Symbols* symbols_for_current_device(int* status) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *status = db_fail(DB_ERR_CUDA, "CUDA_ERROR", "no current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if ((int)g_addr.size() <= dev) g_addr.resize(dev + 1);
    Symbols& s = g_addr[dev];
    if (!s.scratch) {
        void *p = nullptr, *q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_noalloc_error);
        if (e != cudaSuccess || !p || !q) {
            *status = db_cuda_status(e != cudaSuccess ? (int)e : (int)cudaErrorInvalidSymbol,
                                     "scratch symbol address");
            return nullptr;
        }
        s.error = static_cast<int*>(q);
        s.scratch = static_cast<uint8_t*>(p);
    }
    *status = DB_OK;
    return &s;
}

inline size_t up256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

extern "C" {

size_t db_linear_noalloc_scratch_bytes(void) { return kScratchBytes; }

int db_linear_noalloc_error_word(void) {
    int status = DB_OK;
    const Symbols* sym = symbols_for_current_device(&status);
    if (!sym) return -1;
    int v = 0;
    // synchronous copies of one word each way; neither allocates
    if (cudaMemcpy(&v, sym->error, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    const int zero = 0;
    if (cudaMemcpy(sym->error, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    return v;
}

int db_linear_g64_noalloc(const float* x, int64_t M, int64_t K, const uint8_t* w_codes, const float* sw, int64_t N,
                          int weight_bits, int activation_bits, int fused, float* y, void* stream) {
    if (M < 0 || K <= 0 || N <= 0 || (weight_bits != 4 && weight_bits != 8) ||
        (activation_bits != 4 && activation_bits != 8) || !x || !w_codes || !sw || !y)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "linear_noalloc: bad shape or pointer");
    if (M == 0) return DB_OK;
    const int64_t G = (K + DB_GROUP - 1) / DB_GROUP, Kp = G * DB_GROUP, lds = db_scale_stride(M);
    // carving: codes | activation scales | code sums | non-finite flag
    const size_t codes_b = up256((size_t)M * Kp * 2), scales_b = up256((size_t)G * lds * 4);
    const size_t need = codes_b + 2 * scales_b + 256;
    if (need > kScratchBytes)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "SCRATCH_LIMIT",
                       "linear_noalloc: " + std::to_string(M) + "x" + std::to_string(K) + " needs " +
                           std::to_string(need) + " scratch bytes, the fixed array holds " +
                           std::to_string(kScratchBytes));
    int status = DB_OK;
    const Symbols* sym = symbols_for_current_device(&status);
    if (!sym) return status;
    uint8_t* base = sym->scratch;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* codes = base;
    float* sa = reinterpret_cast<float*>(base + codes_b);
    int32_t* sums = reinterpret_cast<int32_t*>(base + codes_b + scales_b);
    int* flag = reinterpret_cast<int*>(base + codes_b + 2 * scales_b);
    // the array keeps the previous call's contents: the non-finite flag must start at zero
    if (cudaMemsetAsync(flag, 0, sizeof(int), s) != cudaSuccess) return db_cuda_status(1, "linear_noalloc clear");
    const bool gemv = M <= db_gemv_rows_limit();
    int rc = db_launch_quantize_rows(x, DB_F32, K, (int)M, (int)K, activation_bits, codes,
                                     gemv ? DB_CODES_GEMV_I8 : DB_CODES_TC_F16, Kp, sa, gemv ? sums : nullptr, lds,
                                     flag, s);
    if (rc) return db_cuda_status(rc, "linear_noalloc quantize");
    if (gemv) {
        DbGemvArgs g{static_cast<const int8_t*>(codes), Kp, sa, sums, lds, w_codes, sw, (int)M, (int)N, (int)K,
                     weight_bits, fused, 0, y, N, flag};
        return db_cuda_status(db_launch_gemv(g, s), "linear_noalloc gemv");
    }
    DbGemmArgs a{};
    a.a_codes = codes;
    a.lda = Kp;
    a.sa = sa;
    a.ldsa = lds;
    a.w_codes = w_codes;
    a.sw = sw;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.bits = weight_bits;
    a.fused = fused;
    a.epilogue = DB_EPI_STORE;
    a.y = y;
    a.ldy = N;
    a.nonfinite = flag;
    a.dev_error = sym->error;
    return db_cuda_status(db_launch_gemm_tc(a, s), "linear_noalloc gemm");
}

}  // extern "C"
