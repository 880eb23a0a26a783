// Kernel-level C ABI (include/decisive_b200.h): argument checks, workspace carving, launches.
#include <cuda_bf16.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/decisive_b200.h"
#include "capi_internal.h"
#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"

namespace {
thread_local std::string g_code = "OK", g_message;
}

void db_set_error(const char* code, const std::string& message) {
    g_code = code;
    g_message = message;
}
int db_fail(int status, const char* code, const std::string& message) {
    db_set_error(code, message);
    return status;
}
int db_cuda_status(int e, const char* what) {
    if (e == 0) return DB_OK;
    return db_fail(DB_ERR_CUDA, "CUDA_ERROR", std::string(what) + ": " + cudaGetErrorString((cudaError_t)e));
}

cudaError_t db_set_max_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == kernel && d.second == dev) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.emplace_back(kernel, dev);
    return e;
}

int* db_device_error_ptr() {
    static std::mutex mu;
    static std::vector<int*> words;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if ((int)words.size() <= dev) words.resize(dev + 1, nullptr);
    if (!words[dev]) {
        if (cudaMalloc(&words[dev], sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(words[dev], 0, sizeof(int));
    }
    return words[dev];
}

extern "C" {

int db_abi_version(void) { return DB_ABI_VERSION; }
const char* db_last_error_code(void) { return g_code.c_str(); }
const char* db_last_error_message(void) { return g_message.c_str(); }
int db_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}
int db_device_error_word(void) {
    int* p = db_device_error_ptr();
    if (!p) return -1;
    int v = 0;
    cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
    cudaMemset(p, 0, sizeof(int));
    return v;
}

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }
static inline int64_t groups_of(int64_t K) { return (K + DB_GROUP - 1) / DB_GROUP; }

int db_quantize_activations_g64(const void* x, int dtype, int64_t ldx, int64_t M, int64_t K, int bits, void* codes,
                                int layout, int64_t ldc, float* scales, int32_t* sums, int64_t lds, int* nonfinite,
                                void* stream) {
    if (M < 0 || K <= 0 || (bits != 4 && bits != 8) || dtype < 0 || dtype > 2 || layout < 0 || layout > DB_CODES_DQ)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "quantize: bad shape, bits, dtype or layout");
    if (ldx < K || ldc < groups_of(K) * DB_GROUP || lds < M || !x || !codes || !scales)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "quantize: bad strides or null pointer");
    return db_cuda_status(db_launch_quantize_rows(x, dtype, ldx, (int)M, (int)K, bits, codes, layout, ldc, scales,
                                                  sums, lds, nonfinite, S(stream)),
                          "quantize");
}

int db_pack_weights_g64(const uint16_t* bf16, int64_t N, int64_t K, int bits, uint8_t* codes, float* scales,
                        void* stream) {
    if (N <= 0 || K <= 0 || (bits != 4 && bits != 8) || !bf16 || !codes || !scales)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "invalid INT8 matrix shape");
    int* bad = nullptr;
    if (cudaMallocAsync(&bad, sizeof(int), S(stream)) != cudaSuccess) return db_cuda_status(1, "pack alloc");
    cudaMemsetAsync(bad, 0, sizeof(int), S(stream));
    int rc = db_launch_pack_weights(bf16, (int)N, (int)K, bits, codes, scales, bad, S(stream));
    int h = 0;
    cudaMemcpyAsync(&h, bad, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
    cudaFreeAsync(bad, S(stream));
    int e = (int)cudaStreamSynchronize(S(stream));
    if (rc) return db_cuda_status(rc, "pack weights");
    if (e) return db_cuda_status(e, "pack weights");
    if (h) return db_fail(DB_ERR_NONFINITE, "INVALID_WEIGHTS", "non-finite INT8 weight");
    return DB_OK;
}

int db_import_packed(const uint8_t* packed, int64_t N, int64_t K, int bits, uint8_t* codes, float* scales,
                     void* stream) {
    if (N <= 0 || K <= 0 || K % DB_GROUP || (bits != 4 && bits != 8))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "invalid group-64 matrix shape");
    return db_cuda_status(db_launch_packed_convert(const_cast<uint8_t*>(packed), codes, scales, (int)N, (int)K, bits,
                                                   1, S(stream)),
                          "import packed");
}

int db_export_packed(const uint8_t* codes, const float* scales, int64_t N, int64_t K, int bits, uint8_t* packed,
                     void* stream) {
    if (N <= 0 || K <= 0 || K % DB_GROUP || (bits != 4 && bits != 8))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "invalid group-64 matrix shape");
    return db_cuda_status(db_launch_packed_convert(packed, const_cast<uint8_t*>(codes), const_cast<float*>(scales),
                                                   (int)N, (int)K, bits, 0, S(stream)),
                          "export packed");
}

int db_dequant_rows_g64(const uint8_t* codes, const float* scales, int64_t N, int64_t K, int bits, const int32_t* ids,
                        int64_t T, float* out, int64_t ldo, void* stream) {
    if (N <= 0 || K <= 0 || T < 0 || ldo < K || (bits != 4 && bits != 8))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "dequant: bad shape");
    int* bad = nullptr;
    if (cudaMallocAsync(&bad, sizeof(int), S(stream)) != cudaSuccess) return db_cuda_status(1, "dequant alloc");
    cudaMemsetAsync(bad, 0, sizeof(int), S(stream));
    int rc = db_launch_dequant_rows(codes, scales, (int)N, (int)K, bits, ids, (int)T, out, ldo, bad, S(stream));
    int h = 0;
    cudaMemcpyAsync(&h, bad, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
    cudaFreeAsync(bad, S(stream));
    int e = (int)cudaStreamSynchronize(S(stream));
    if (rc) return db_cuda_status(rc, "dequant");
    if (e) return db_cuda_status(e, "dequant");
    if (h) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_REQUEST", "row id out of range");
    return DB_OK;
}

int db_gemv_max_rows(void) { return db_gemv_rows_limit(); }

int db_gemm_g64(const void* a_codes, int layout, int64_t lda, const float* sa, const int32_t* a_sums, int64_t ldsa,
                const uint8_t* w_codes, const float* sw, int64_t M, int64_t N, int64_t K, int bits, int fused,
                int residual, float* y, int64_t ldy, const int* nonfinite, void* stream) {
    return db_gemm_g64_config(a_codes, layout, lda, sa, a_sums, ldsa, w_codes, sw, M, N, K, bits, fused, residual, y,
                              ldy, nonfinite, nullptr, stream);
}

int db_gemm_g64_config(const void* a_codes, int layout, int64_t lda, const float* sa, const int32_t* a_sums,
                       int64_t ldsa, const uint8_t* w_codes, const float* sw, int64_t M, int64_t N, int64_t K,
                       int bits, int fused, int residual, float* y, int64_t ldy, const int* nonfinite,
                       const db_gemm_config* config, void* stream) {
    if (config && ((config->block_n != 0 && config->block_n != 64 && config->block_n != 128 && config->block_n != 256 &&
                    !(config->block_n == 32 && layout == DB_CODES_NATURAL)) ||
                   config->max_ctas < 0 ||
                   (config->pair_ctas != 0 && config->pair_ctas != 1)))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "gemm: bad tile configuration");
    if (M < 0 || N <= 0 || K <= 0 || (bits != 4 && bits != 8) || ldy < N || (layout != DB_CODES_DQ && ldsa < M))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "gemm: bad shape");
    if (M == 0) return DB_OK;
    if (layout == DB_CODES_GEMV) {
        if (M > db_gemv_rows_limit() || (bits == 4 && !a_sums))
            return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "gemv: too many rows or missing sums");
        DbGemvArgs g{static_cast<const int8_t*>(a_codes), lda, sa, a_sums, ldsa, w_codes, sw, (int)M, (int)N, (int)K,
                     bits, fused, residual, y, ldy, nonfinite};
        return db_cuda_status(db_launch_gemv(g, S(stream)), "gemv");
    }
    if (layout != DB_CODES_TC && layout != DB_CODES_NATURAL && layout != DB_CODES_DQ)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "gemm: unknown code layout");
    DbGemmArgs a{};
    a.a_codes = a_codes;
    a.lda = lda;
    a.sa = sa;
    a.ldsa = ldsa;
    a.w_codes = w_codes;
    a.sw = sw;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.bits = bits;
    a.fused = fused;
    a.epilogue = residual ? DB_EPI_RESIDUAL : DB_EPI_STORE;
    a.y = y;
    a.ldy = ldy;
    a.nonfinite = nonfinite;
    a.dev_error = db_device_error_ptr();
    if (config) {
        a.block_n = config->block_n;
        a.max_ctas = config->max_ctas;
        a.pair_ctas = config->pair_ctas;
    }
    if (layout == DB_CODES_DQ) return db_cuda_status(db_launch_gemm_dq(a, S(stream)), "gemm");
    if (layout == DB_CODES_NATURAL) {
        if (!config) {
            const db_gemm_config d = db_gemm_i8_default_config(M, N, a.epilogue);
            a.block_n = d.block_n;
            a.pair_ctas = d.pair_ctas;
        }
        return db_cuda_status(db_launch_gemm_i8(a, S(stream)), "gemm");
    }
    return db_cuda_status(db_launch_gemm_tc(a, S(stream)), "gemm");
}

}  // extern "C"

// Tile configuration of the int8 tensor-core GEMM when none is given: the widest tile that still
// occupies the SMs -- each candidate is scored by the fraction of the last wave of CTAs that has
// work, with a small preference for wide tiles (fewer re-reads of A per output).  CTA pairs
// measured slower than single CTAs on the C1/C2 shapes (the pair's MMA waits for both CTAs), so
// they are scored down; the tuner still tries them.
db_gemm_config db_gemm_i8_default_config(int64_t M, int64_t N, int epilogue) {
    const int sms = db_num_sms();
    const int cands[6][2] = {{256, 1}, {128, 1}, {64, 1}, {256, 0}, {128, 0}, {64, 0}};
    double best = -1.0;
    db_gemm_config out{256, 0, 0};
    for (const auto& c : cands) {
        const int bn = c[0], pair = c[1];
        if (pair && M <= 128) continue;
        if (epilogue == DB_EPI_SWIGLU_QUANT && bn == 64) continue;
        const int64_t mt = pair ? 256 : 128;
        const int64_t ctas = ((M + mt - 1) / mt) * ((N + bn - 1) / bn) * (pair ? 2 : 1);
        const int64_t waves = (ctas + sms - 1) / sms;
        const double fill = (double)ctas / (double)(waves * sms);
        const double score = fill * (bn == 256 ? 1.0 : bn == 128 ? 0.97 : 0.88) * (pair ? 0.85 : 1.0);
        if (score > best + 1e-9) {
            best = score;
            out = db_gemm_config{bn, 0, pair};
        }
    }
    return out;
}

extern "C" {

size_t db_linear_workspace_bytes(int64_t M, int64_t K) {
    const int64_t G = groups_of(K), Kp = G * DB_GROUP;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    return up((size_t)M * Kp * 2) + 2 * up((size_t)G * db_scale_stride(M) * 4) + 256;
}

int64_t db_scale_row_stride(int64_t n) { return db_scale_stride(n); }

int db_linear_g64(const float* x, int64_t M, int64_t K, const uint8_t* w_codes, const float* sw, int64_t N,
                  int weight_bits, int activation_bits, int fused, float* y, void* workspace, void* stream) {
    if (M < 0 || K <= 0 || N <= 0 || (weight_bits != 4 && weight_bits != 8) ||
        (activation_bits != 4 && activation_bits != 8) || !workspace)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "linear: bad shape");
    if (M == 0) return DB_OK;
    const int64_t G = groups_of(K), Kp = G * DB_GROUP;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    void* codes = ws;
    const int64_t lds = db_scale_stride(M);
    float* sa = reinterpret_cast<float*>(ws + up((size_t)M * Kp * 2));
    int32_t* sums = reinterpret_cast<int32_t*>(ws + up((size_t)M * Kp * 2) + up((size_t)G * lds * 4));
    int* flag = reinterpret_cast<int*>(ws + up((size_t)M * Kp * 2) + 2 * up((size_t)G * lds * 4));
    cudaMemsetAsync(flag, 0, sizeof(int), S(stream));
    const bool gemv = M <= db_gemv_rows_limit();
    const int layout = gemv ? DB_CODES_GEMV : DB_CODES_TC;
    int rc = db_quantize_activations_g64(x, DB_DTYPE_F32, K, M, K, activation_bits, codes, layout, Kp, sa,
                                         gemv ? sums : nullptr, lds, flag, stream);
    if (rc) return rc;
    return db_gemm_g64(codes, layout, Kp, sa, sums, lds, w_codes, sw, M, N, K, weight_bits, fused, 0, y, N, flag,
                       stream);
}

// ---- Decima int8 (decima/int8.rs): blocks of 32 or 64, round half away from zero of x / scale
static inline bool decima_block_ok(int block) { return block == 16 || block == 32 || block == 64 || block == 128; }

int db_decima_quantize_weights(const float* w, int64_t N, int64_t K, int block, uint8_t* codes, float* scales,
                               void* stream) {
    if (N <= 0 || K <= 0 || !decima_block_ok(block) || !w || !codes || !scales)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT",
                       "INT8 block must be 16, 32, 64 or 128 and the shape positive");
    const int64_t Kp = groups_of(K) * DB_GROUP, GS = (K + block - 1) / block, ldw = db_scale_stride(N);
    int* bad = nullptr;
    if (cudaMallocAsync(&bad, sizeof(int), S(stream)) != cudaSuccess) return db_cuda_status(1, "quantize alloc");
    cudaMemsetAsync(bad, 0, sizeof(int), S(stream));
    cudaMemsetAsync(scales, 0, (size_t)GS * ldw * sizeof(float), S(stream));  // padding columns: scale 0
    int rc = db_launch_decima_quantize(w, K, (int)N, (int)K, block, codes, DB_CODES_NATURAL_I8, Kp, scales, ldw, 0,
                                       bad, S(stream));
    int h = 0;
    cudaMemcpyAsync(&h, bad, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
    cudaFreeAsync(bad, S(stream));
    int e = (int)cudaStreamSynchronize(S(stream));
    if (rc) return db_cuda_status(rc, "decima quantize weights");
    if (e) return db_cuda_status(e, "decima quantize weights");
    if (h) return db_fail(DB_ERR_NONFINITE, "INVALID_WEIGHTS", "non-finite INT8 weights");
    return DB_OK;
}

int db_decima_quantize_activations(const float* x, int64_t M, int64_t K, int block, void* codes, int layout,
                                   int64_t ldc, float* scales, int64_t lds, int* nonfinite, void* stream) {
    const int64_t Kp = groups_of(K) * DB_GROUP;
    if (M < 0 || K <= 0 || !decima_block_ok(block) || ldc < Kp ||
        (layout != DB_CODES_TC && layout != DB_CODES_NATURAL) || lds < M)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "decima quantize: bad shape or layout");
    if (M == 0) return DB_OK;
    return db_cuda_status(db_launch_decima_quantize(x, K, (int)M, (int)K, block, codes,
                                                    layout == DB_CODES_TC ? DB_CODES_TC_F16 : DB_CODES_NATURAL_I8,
                                                    ldc, scales, lds, 0, nonfinite, S(stream)),
                          "decima quantize activations");
}

size_t db_decima_workspace_bytes(int64_t M, int64_t K, int block) {
    if (M < 0 || K <= 0 || !decima_block_ok(block)) return 0;
    const int64_t Kp = groups_of(K) * DB_GROUP, GS = (K + block - 1) / block;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    return up((size_t)M * Kp * 2) + up((size_t)GS * db_scale_stride(M) * 4) + 256;
}

int db_decima_linear(const float* x, int64_t M, int64_t K, const uint8_t* w_codes, const float* sw, int64_t N,
                     int block, int fused, const float* bias, float* y, void* workspace, void* stream) {
    if (M < 0 || K <= 0 || N <= 0 || !decima_block_ok(block) || !workspace || !w_codes || !sw || !y)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "decima linear: bad shape");
    if (block != 32 && block != 64)
        return db_fail(DB_ERR_UNSUPPORTED, "UNSUPPORTED", "decima linear: the GPU GEMM takes blocks of 32 or 64");
    if (M == 0) return DB_OK;
    const int64_t Kp = groups_of(K) * DB_GROUP, GS = (K + block - 1) / block, lds = db_scale_stride(M);
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    void* codes = ws;
    float* sa = reinterpret_cast<float*>(ws + up((size_t)M * Kp * 2));
    int* flag = reinterpret_cast<int*>(ws + up((size_t)M * Kp * 2) + up((size_t)GS * lds * 4));
    cudaMemsetAsync(flag, 0, sizeof(int), S(stream));
    int rc = db_launch_decima_quantize(x, K, (int)M, (int)K, block, codes, DB_CODES_TC_F16, Kp, sa, lds, 0, flag,
                                       S(stream));
    if (rc) return db_cuda_status(rc, "decima quantize activations");
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
    a.bits = 8;
    a.fused = fused;
    a.epilogue = DB_EPI_STORE;
    a.y = y;
    a.ldy = N;
    a.nonfinite = flag;  // a non-finite x gives all-NaN y (decima/int8.rs:186-190)
    a.dev_error = db_device_error_ptr();
    a.block = block;
    a.bias = bias;
    a.add_bias = 1;
    return db_cuda_status(db_launch_gemm_tc(a, S(stream)), "decima gemm");
}

int db_decima_linear_w8a32(const float* x, int64_t M, int64_t K, const uint8_t* w_codes, const float* sw, int64_t N,
                           int block, int fused, const float* bias, float* y, int* nonfinite, void* stream) {
    if (M < 0 || K <= 0 || N <= 0 || !decima_block_ok(block) || !w_codes || !sw || !y || !nonfinite ||
        (M > 0 && !x))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "decima linear: bad shape");
    if (block == 16)
        return db_fail(DB_ERR_UNSUPPORTED, "UNSUPPORTED", "decima W8A32: the GPU kernel takes blocks of 32, 64 or 128");
    if (M == 0) return DB_OK;
    cudaMemsetAsync(nonfinite, 0, sizeof(int), S(stream));
    int rc = db_launch_decima_w8a32(x, K, (int)M, (int)K, w_codes, groups_of(K) * DB_GROUP, sw, db_scale_stride(N),
                                    (int)N, block, fused, bias, y, N, nonfinite, S(stream));
    if (rc) return db_cuda_status(rc, "decima w8a32");
    // a non-finite x gives all-NaN y (decima/int8.rs:183-187)
    return db_cuda_status(db_launch_fill_nan_if(y, M * N, nonfinite, S(stream)), "decima w8a32");
}

int db_project_packed(const float* x, int64_t K, const uint8_t* w_codes, const float* sw, int64_t outputs, int bits,
                      float* y, void* workspace, void* stream) {
    if (K <= 0 || K % DB_GROUP || outputs <= 0 || !workspace)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "invalid packed readout shape");
    int rc = db_linear_g64(x, 1, K, w_codes, sw, outputs, bits, 8, 0, y, workspace, stream);
    if (rc) return rc;
    const int64_t G = K / DB_GROUP, Kp = K;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    const int* flag = reinterpret_cast<const int*>(static_cast<uint8_t*>(workspace) + up((size_t)Kp * 2) +
                                                   2 * up((size_t)G * db_scale_stride(1) * 4));
    int h = 0;
    cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, S(stream));
    int e = (int)cudaStreamSynchronize(S(stream));
    if (e) return db_cuda_status(e, "project");
    if (h) return db_fail(DB_ERR_NONFINITE, "INVALID_REQUEST", "nonfinite readout activation");
    return DB_OK;
}

int db_mlp_g64(const void* a_codes, int64_t lda, const float* sa, int64_t ldsa, const uint8_t* w_gu_codes,
               const float* w_gu_scales, int64_t M, int64_t F, int64_t K, int bits, int fused, void* out_codes,
               int64_t ldoc, float* out_scales, int64_t ldos, const int* nonfinite, void* stream) {
    if (M < 0 || F <= 0 || F % DB_GROUP || K <= 0 || (bits != 4 && bits != 8) || ldoc < F ||
        ldos < db_scale_stride(M) || (ldos & 3))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "mlp: bad shape");
    if (M == 0) return DB_OK;
    DbGemmArgs a{};
    a.a_codes = a_codes;
    a.lda = lda;
    a.sa = sa;
    a.ldsa = ldsa;
    a.w_codes = w_gu_codes;
    a.sw = w_gu_scales;
    a.M = (int)M;
    a.N = (int)(2 * F);
    a.K = (int)K;
    a.bits = bits;
    a.fused = fused;
    a.epilogue = DB_EPI_SWIGLU_QUANT;
    a.out_codes = out_codes;
    a.ldoc = ldoc;
    a.out_scales = out_scales;
    a.ldos = ldos;
    a.nonfinite = nonfinite;
    a.dev_error = db_device_error_ptr();
    return db_cuda_status(db_launch_gemm_tc(a, S(stream)), "mlp");
}

int db_mlp_g64_natural(const void* a_codes, int64_t lda, const float* sa, int64_t ldsa, const uint8_t* w_gu_codes,
                       const float* w_gu_scales, int64_t M, int64_t F, int64_t K, int bits, int fused, void* out_codes,
                       int64_t ldoc, float* out_scales, int64_t ldos, const int* nonfinite, void* stream) {
    if (M < 0 || F <= 0 || F % DB_GROUP || K <= 0 || (bits != 4 && bits != 8) || ldoc < F || (ldoc & 15) ||
        ldos < db_scale_stride(M) || (ldos & 3))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "mlp: bad shape");
    if (M == 0) return DB_OK;
    DbGemmArgs a{};
    a.a_codes = a_codes;
    a.lda = lda;
    a.sa = sa;
    a.ldsa = ldsa;
    a.w_codes = w_gu_codes;
    a.sw = w_gu_scales;
    a.M = (int)M;
    a.N = (int)(2 * F);
    a.K = (int)K;
    a.bits = bits;
    a.fused = fused;
    a.epilogue = DB_EPI_SWIGLU_QUANT;
    a.out_codes = out_codes;
    a.ldoc = ldoc;
    a.out_scales = out_scales;
    a.ldos = ldos;
    a.nonfinite = nonfinite;
    a.dev_error = db_device_error_ptr();
    const db_gemm_config d = db_gemm_i8_default_config(M, 2 * F, DB_EPI_SWIGLU_QUANT);
    a.block_n = d.block_n;
    a.pair_ctas = d.pair_ctas;
    return db_cuda_status(db_launch_gemm_i8(a, S(stream)), "mlp");
}

}  // extern "C"

namespace {
__global__ void interleave_kernel(const uint8_t* __restrict__ gc, const float* __restrict__ gs,
                                  const uint8_t* __restrict__ uc, const float* __restrict__ us, int F, int G,
                                  int row_bytes, uint8_t* __restrict__ oc, float* __restrict__ os) {
    const int row = blockIdx.x;  // output row in [0, 2F)
    const int b = row / 128, j = row % 128;
    const bool is_up = j >= 64;
    const int src = b * 64 + (j & 63);
    const uint8_t* s = (is_up ? uc : gc) + (size_t)src * row_bytes;
    for (int i = threadIdx.x; i < row_bytes; i += blockDim.x) oc[(size_t)row * row_bytes + i] = s[i];
    for (int g = threadIdx.x; g < G; g += blockDim.x)
        os[(size_t)g * db_scale_stride(2 * F) + row] = (is_up ? us : gs)[(size_t)g * db_scale_stride(F) + src];
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
// Box-Muller on two 24-bit uniforms of one 64-bit hash per pair of outputs.
__global__ void synthetic_kernel(uint64_t seed, uint64_t tensor, int64_t n, float stdv, uint16_t* __restrict__ out) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (2 * p >= n) return;
    const uint64_t h = mix64(mix64(seed * 0x100000001B3ull ^ (tensor + 1) * 0xC2B2AE3D27D4EB4Full) ^ (uint64_t)p);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.f / 16777216.f);
    const float u2 = ((float)((h >> 8) & 0xFFFFFFu) + 0.5f) * (1.f / 16777216.f);
    const float r = sqrtf(-2.f * logf(u1));
    float s, c;
    sincospif(2.f * u2, &s, &c);
    out[2 * p] = __bfloat16_as_ushort(__float2bfloat16_rn(stdv * r * c));
    if (2 * p + 1 < n) out[2 * p + 1] = __bfloat16_as_ushort(__float2bfloat16_rn(stdv * r * s));
}
}  // namespace

extern "C" {

int db_interleave_gate_up(const uint8_t* gate_codes, const float* gate_scales, const uint8_t* up_codes,
                          const float* up_scales, int64_t F, int64_t K, int bits, uint8_t* out_codes,
                          float* out_scales, void* stream) {
    if (F <= 0 || F % DB_GROUP || K <= 0 || (bits != 4 && bits != 8))
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "interleave: F must be a multiple of 64");
    const int G = (int)groups_of(K), row_bytes = G * DB_GROUP * bits / 8;
    cudaMemsetAsync(out_scales, 0, (size_t)G * db_scale_stride(2 * F) * sizeof(float), S(stream));
    interleave_kernel<<<(unsigned)(2 * F), 128, 0, S(stream)>>>(gate_codes, gate_scales, up_codes, up_scales, (int)F,
                                                                  G, row_bytes, out_codes, out_scales);
    return db_cuda_status((int)cudaGetLastError(), "interleave");
}

int db_attention(const void* q16, const void* k16, const void* v16, int64_t T, int64_t q_heads, int64_t kv_heads,
                 int64_t head_dim, float scale, float* out, int64_t ldo, void* stream) {
    if (head_dim != 128 || T < 0 || kv_heads <= 0 || q_heads % kv_heads || ldo < q_heads * head_dim)
        return db_fail(DB_ERR_UNSUPPORTED, "UNSUPPORTED", "attention: head_dim 128 and Hq % Hk == 0 required");
    return db_cuda_status(db_launch_attention(static_cast<const __half*>(q16), static_cast<const __half*>(k16),
                                              static_cast<const __half*>(v16), (int)T, (int)q_heads, (int)kv_heads,
                                              scale, out, ldo, S(stream)),
                          "attention");
}

int db_attention_decoder(const void* q16, const void* k16, const void* v16, int64_t B, int64_t T, const void* kp,
                         const void* vp, int64_t P, int causal, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                         float scale, float* out, int64_t ldo, void* stream) {
    if (head_dim != 128 || B < 0 || T < 0 || P < 0 || B > 65535 || T > (1 << 30) || P > (1 << 30) || kv_heads <= 0 ||
        q_heads % kv_heads || ldo < q_heads * head_dim || (P > 0 && (!kp || !vp)))
        return db_fail(DB_ERR_UNSUPPORTED, "UNSUPPORTED",
                       "attention: head_dim 128, Hq % Hk == 0 and prefix keys for P > 0 required");
    return db_cuda_status(db_launch_attention_decoder(static_cast<const __half*>(q16), static_cast<const __half*>(k16),
                                                      static_cast<const __half*>(v16), (int)B, (int)T,
                                                      static_cast<const __half*>(kp), static_cast<const __half*>(vp),
                                                      (int)P, causal, (int)q_heads, (int)kv_heads, scale, out, ldo,
                                                      nullptr, 0, nullptr, 0, nullptr, S(stream)),
                          "attention");
}

int db_synthetic_bf16(uint64_t seed, uint64_t tensor, int64_t n, float stdv, uint16_t* out, void* stream) {
    if (n < 0 || !out) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "synthetic: bad size");
    if (n == 0) return DB_OK;
    const int64_t pairs = (n + 1) / 2;
    synthetic_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, S(stream)>>>(seed, tensor, n, stdv, out);
    return db_cuda_status((int)cudaGetLastError(), "synthetic");
}

}  // extern "C"
