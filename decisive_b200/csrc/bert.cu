// C4: the Decima-shaped (BERT) encoder on the Decima int8 kernels (decima/mod.rs:492-556):
//   x = LN(word[id] + type[0] + pos[p])
//   per layer: qkv = W8A8(x) + b; ctx = attn(q, k, v); x = LN(x + Wo ctx + bo);
//              h = gelu(W1 x + b1); x = LN(x + W2 h + b2)
//   pooled = mean_t x
// Every projection quantises its input with the Decima block quantiser (round half away from zero
// of x / scale, blocks of cfg.block) and runs the block grouped GEMM with the bias epilogue.
// Attention reuses the head-dim-128 kernel with heads zero-padded to 128 (zero q/k dims add
// nothing to the dot products; the zero v dims are dropped when the heads are merged).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/decisive_b200.h"
#include "capi_internal.h"
#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"

namespace {

__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ in, int64_t n, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __uint_as_float((uint32_t)in[i] << 16);
}

// x[t] = (word[id] + type[0]) + pos[p]   (decima/mod.rs:503-508); p = t, or positions[t] for
// sequences packed one after another
__global__ void embed_kernel(const int32_t* __restrict__ ids, const float* __restrict__ word,
                             const float* __restrict__ type, const float* __restrict__ pos,
                             const int32_t* __restrict__ positions, int D, float* __restrict__ x) {
    const int t = blockIdx.x;
    const float* w = word + (size_t)ids[t] * D;
    const size_t p = positions ? (size_t)positions[t] : (size_t)t;
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        x[(size_t)t * D + i] = __fadd_rn(__fadd_rn(w[i], type[i]), pos[p * D + i]);
}

// Scorer head (f32 linear, sequential sums as the reference's portable f32 kernel): logits[s, o] =
// sum_k pooled[s, k] * w[o, k] + b[o] for NO outputs; one warp per (sequence, output), lane 0
// accumulates in index order.
__global__ void head_kernel(const float* __restrict__ pooled, const float* __restrict__ w, const float* __restrict__ b,
                            int nseq, int D, int NO, float* __restrict__ out) {
    const int s = blockIdx.x, o = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (s >= nseq || o >= NO || lane != 0) return;
    float acc = 0.f;
    for (int k = 0; k < D; ++k) acc = __fadd_rn(acc, __fmul_rn(pooled[(size_t)s * D + k], w[(size_t)o * D + k]));
    out[(size_t)s * NO + o] = __fadd_rn(acc, b[o]);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
    return t;
}

// x = LN(x + r) (r may be null), decima/cpu.rs:529-539: mean, variance, (v - mean) * inv * w + b.
// One CTA per row, up to 8 values per thread.
__global__ void layer_norm_kernel(float* __restrict__ x, const float* __restrict__ r, const float* __restrict__ w,
                                  const float* __restrict__ b, int D, float eps) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    float v[8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        v[j] = 0.f;
        if (i < D) {
            v[j] = x[(size_t)t * D + i];
            if (r) v[j] = __fadd_rn(v[j], r[(size_t)t * D + i]);
            s = __fadd_rn(s, v[j]);
        }
    }
    const float mean = __fdiv_rn(block_sum(s, red), (float)D);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < D) {
            const float c = __fsub_rn(v[j], mean);
            q = __fadd_rn(q, __fmul_rn(c, c));
        }
    }
    const float var = __fdiv_rn(block_sum(q, red), (float)D);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < D) x[(size_t)t * D + i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j], mean), inv), w[i]), b[i]);
    }
}

// decima/cpu.rs:542-556: 0.5 x (1 + erf(x / sqrt 2))
__global__ void gelu_kernel(float* __restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.f, erff(__fmul_rn(v, 0.70710678118654752440f))));
    }
}

// qkv f32 [T, 3D] (q | k | v, head h at h*hd) -> f16 [T, H, 128] each, dims past hd zero
__global__ void split_heads_kernel(const float* __restrict__ qkv, int T, int H, int hd, __half* __restrict__ q,
                                   __half* __restrict__ k, __half* __restrict__ v) {
    const int t = blockIdx.x, D = H * hd;
    for (int i = threadIdx.x; i < 3 * H * 128; i += blockDim.x) {
        const int which = i / (H * 128), h = (i / 128) % H, d = i % 128;
        const float val = d < hd ? qkv[(size_t)t * 3 * D + which * D + h * hd + d] : 0.f;
        __half* dst = which == 0 ? q : which == 1 ? k : v;
        dst[((size_t)t * H + h) * 128 + d] = __float2half_rn(val);
    }
}

// ctx f32 [T, H*128] -> [T, H*hd]
__global__ void merge_heads_kernel(const float* __restrict__ in, int H, int hd, float* __restrict__ out) {
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < H * hd; i += blockDim.x)
        out[(size_t)t * H * hd + i] = in[((size_t)t * H + i / hd) * 128 + i % hd];
}

inline unsigned grid_for(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 4096); }

void fill_error(db_error* err, const char* code, const std::string& msg) {
    if (!err) return;
    std::snprintf(err->code, sizeof err->code, "%s", code);
    std::snprintf(err->message, sizeof err->message, "%s", msg.c_str());
}

}  // namespace

struct db_bert {
    int device = 0;
    db_bert_config cfg{};
    cudaStream_t stream = nullptr;
    std::vector<void*> allocations;
    float *word = nullptr, *pos = nullptr, *type = nullptr, *emb_ln_w = nullptr, *emb_ln_b = nullptr;
    struct Layer {
        uint8_t *qkv_c, *o_c, *f1_c, *f2_c;
        float *qkv_s, *o_s, *f1_s, *f2_s;
        float *bqkv, *bo, *b1, *b2, *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    };
    std::vector<Layer> layers;
    float *head_w = nullptr, *head_b = nullptr;  // scorer head [DB_BERT_HEAD_OUTPUTS, hidden] + bias
    // workspace for cap rows (one sequence of cfg.max_positions tokens, or a request's packed
    // sequences: kBatchSeqs of them)
    int cap = 0;
    float *x = nullptr, *tmp = nullptr, *qkv = nullptr, *h = nullptr, *ctx128 = nullptr, *ctx = nullptr,
          *scales = nullptr, *pooled = nullptr, *logits = nullptr;
    int8_t* codes = nullptr;
    __half *q16 = nullptr, *k16 = nullptr, *v16 = nullptr;
    int32_t *ids = nullptr, *positions = nullptr, *cu = nullptr;
    int* flag = nullptr;
    template <class T>
    bool alloc(T** p, size_t count) {
        if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 256) != cudaSuccess) return false;
        allocations.push_back(*p);
        return true;
    }
};

namespace {

// synthetic tensor ids (db_synthetic_bf16 keys): word 0, pos 1, type 2; layer l: 16 + 16 l + kind
enum { K_Q = 0, K_K, K_V, K_O, K_FF1, K_FF2, K_BQ, K_BK, K_BV, K_BO, K_B1, K_B2 };
constexpr uint64_t K_HEAD_W = 3, K_HEAD_B = 4;  // scorer head (model-level ids, below the layers')
constexpr int kBatchSeqs = 16;                  // sequences one packed pass holds (a request has 8)
inline uint64_t tid(int l, int kind) { return 16 + 16ull * l + kind; }

int build_synthetic(db_bert* m, uint64_t seed, float stdv) {
    const auto& c = m->cfg;
    const int D = c.hidden, F = c.ffn, L = c.layers, P = c.max_positions;
    cudaStream_t st = m->stream;
    const size_t big = std::max({(size_t)c.vocab * D, (size_t)3 * D * D, (size_t)F * D});
    // staging (freed at the end of the build)
    uint16_t* stage16 = nullptr;
    float* stage32 = nullptr;
    int* bad = nullptr;
    struct Free {
        void* p[3];
        ~Free() {
            for (void* q : p) cudaFree(q);
        }
    } staging{{nullptr, nullptr, nullptr}};
    if (cudaMalloc(&stage16, big * 2) != cudaSuccess || (staging.p[0] = stage16, false) ||
        cudaMalloc(&stage32, big * 4) != cudaSuccess || (staging.p[1] = stage32, false) ||
        cudaMalloc(&bad, 4) != cudaSuccess || (staging.p[2] = bad, false))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "staging exceeds device limits");
    cudaMemsetAsync(bad, 0, 4, st);
    auto gen = [&](uint64_t id, int64_t n, float* out) -> int {
        int rc = db_synthetic_bf16(seed, id, n, stdv, stage16, st);
        bf16_to_f32_kernel<<<grid_for(n), 256, 0, st>>>(stage16, n, out);
        return rc ? rc : db_cuda_status((int)cudaGetLastError(), "synthetic");
    };
    auto ones = [&](int n, float v, float** out) -> int {
        if (!m->alloc(out, n)) return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "allocation");
        std::vector<float> h(n, v);
        return db_cuda_status((int)cudaMemcpy(*out, h.data(), n * 4, cudaMemcpyHostToDevice), "upload");
    };
    // rows [N, K] of synthetic tensors (several tensors stacked) -> Decima int8 codes + scales
    auto quantize = [&](const std::vector<uint64_t>& ids, int rows_each, int K, uint8_t** codes, float** scales) {
        const int N = rows_each * (int)ids.size();
        const int64_t Kp = (K + 63) / 64 * 64, GS = (K + c.block - 1) / c.block;
        if (!m->alloc(codes, (size_t)N * Kp) || !m->alloc(scales, (size_t)GS * db_scale_stride(N)))
            return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight allocation");
        for (size_t i = 0; i < ids.size(); ++i) {
            const int rc = gen(ids[i], (int64_t)rows_each * K, stage32 + i * (size_t)rows_each * K);
            if (rc) return rc;
        }
        cudaMemsetAsync(*scales, 0, (size_t)GS * db_scale_stride(N) * 4, st);
        return db_cuda_status(db_launch_decima_quantize(stage32, K, N, K, c.block, *codes, DB_CODES_NATURAL_I8, Kp,
                                                        *scales, db_scale_stride(N), 0, bad, st),
                              "quantize weights");
    };
    auto bias = [&](const std::vector<uint64_t>& ids, int n_each, float** out) -> int {
        if (!m->alloc(out, (size_t)n_each * ids.size())) return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "allocation");
        for (size_t i = 0; i < ids.size(); ++i) {
            const int rc = gen(ids[i], n_each, *out + i * n_each);
            if (rc) return rc;
        }
        return 0;
    };
    int rc = 0;
    if (!m->alloc(&m->word, (size_t)c.vocab * D) || !m->alloc(&m->pos, (size_t)P * D) || !m->alloc(&m->type, 2 * D))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "embedding allocation");
    rc = gen(0, (int64_t)c.vocab * D, m->word);
    if (!rc) rc = gen(1, (int64_t)P * D, m->pos);
    if (!rc) rc = gen(2, 2 * D, m->type);
    if (!rc) rc = ones(D, 1.f, &m->emb_ln_w);
    if (!rc) rc = ones(D, 0.f, &m->emb_ln_b);
    m->layers.resize(L);
    for (int l = 0; l < L && !rc; ++l) {
        auto& w = m->layers[l];
        rc = quantize({tid(l, K_Q), tid(l, K_K), tid(l, K_V)}, D, D, &w.qkv_c, &w.qkv_s);
        if (!rc) rc = quantize({tid(l, K_O)}, D, D, &w.o_c, &w.o_s);
        if (!rc) rc = quantize({tid(l, K_FF1)}, F, D, &w.f1_c, &w.f1_s);
        if (!rc) rc = quantize({tid(l, K_FF2)}, D, F, &w.f2_c, &w.f2_s);
        if (!rc) rc = bias({tid(l, K_BQ), tid(l, K_BK), tid(l, K_BV)}, D, &w.bqkv);
        if (!rc) rc = bias({tid(l, K_BO)}, D, &w.bo);
        if (!rc) rc = bias({tid(l, K_B1)}, F, &w.b1);
        if (!rc) rc = bias({tid(l, K_B2)}, D, &w.b2);
        if (!rc) rc = ones(D, 1.f, &w.ln1_w);
        if (!rc) rc = ones(D, 0.f, &w.ln1_b);
        if (!rc) rc = ones(D, 1.f, &w.ln2_w);
        if (!rc) rc = ones(D, 0.f, &w.ln2_b);
        cudaStreamSynchronize(st);  // the staging buffers are reused by the next layer
    }
    int h = 0;
    cudaMemcpy(&h, bad, 4, cudaMemcpyDeviceToHost);  // synchronises: the staging is free to go
    if (!rc && h) rc = db_fail(DB_ERR_NONFINITE, "INVALID_WEIGHTS", "non-finite synthetic weight");
    // scorer head (f32, like the reference's Precision::F32 score linear)
    if (!rc && (!m->alloc(&m->head_w, (size_t)DB_BERT_HEAD_OUTPUTS * D) || !m->alloc(&m->head_b, DB_BERT_HEAD_OUTPUTS)))
        rc = db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "head allocation");
    if (!rc) rc = gen(K_HEAD_W, (int64_t)DB_BERT_HEAD_OUTPUTS * D, m->head_w);
    if (!rc) rc = gen(K_HEAD_B, DB_BERT_HEAD_OUTPUTS, m->head_b);
    cudaStreamSynchronize(st);
    // workspace
    const int H = c.heads, Kmax = std::max(D, F), R = kBatchSeqs * P;
    m->cap = R;
    const int64_t lds = db_scale_stride(R), GSmax = (Kmax + c.block - 1) / c.block;
    if (!rc && (!m->alloc(&m->x, (size_t)R * D) || !m->alloc(&m->tmp, (size_t)R * D) ||
                !m->alloc(&m->qkv, (size_t)R * 3 * D) || !m->alloc(&m->h, (size_t)R * F) ||
                !m->alloc(&m->ctx128, (size_t)R * H * 128) || !m->alloc(&m->ctx, (size_t)R * D) ||
                !m->alloc(&m->scales, (size_t)GSmax * lds) || !m->alloc(&m->pooled, (size_t)kBatchSeqs * D) ||
                !m->alloc(&m->logits, (size_t)kBatchSeqs * DB_BERT_HEAD_OUTPUTS) ||
                !m->alloc(&m->codes, (size_t)R * ((Kmax + 63) / 64 * 64)) || !m->alloc(&m->q16, (size_t)R * H * 128) ||
                !m->alloc(&m->k16, (size_t)R * H * 128) || !m->alloc(&m->v16, (size_t)R * H * 128) ||
                !m->alloc(&m->ids, R) || !m->alloc(&m->positions, R) || !m->alloc(&m->cu, kBatchSeqs + 1) ||
                !m->alloc(&m->flag, 4)))
        rc = db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "workspace exceeds device limits");
    return rc;
}

// y [T, N] = W8A8(x [T, K]) + bias (codes of x are quantised first), or W8A32 (x as f32)
int linear(db_bert* m, const float* x, int T, int K, const uint8_t* wc, const float* ws, int N, const float* b,
           float* y) {
    const auto& c = m->cfg;
    if (c.mode == 1)
        return db_launch_decima_w8a32(x, K, T, K, wc, (K + 63) / 64 * 64, ws, db_scale_stride(N), N, c.block, c.fused,
                                      b, y, N, m->flag, m->stream);
    const int64_t Kp = (K + 63) / 64 * 64, lds = db_scale_stride(m->cap);
    int rc = db_launch_decima_quantize(x, K, T, K, c.block, m->codes, DB_CODES_NATURAL_I8, Kp, m->scales, lds, 0,
                                       m->flag, m->stream);
    if (rc) return rc;
    DbGemmArgs a{};
    a.a_codes = m->codes;
    a.lda = Kp;
    a.sa = m->scales;
    a.ldsa = lds;
    a.w_codes = wc;
    a.sw = ws;
    a.M = T;
    a.N = N;
    a.K = K;
    a.bits = 8;
    a.fused = c.fused;
    a.epilogue = DB_EPI_STORE;
    a.y = y;
    a.ldy = N;
    a.nonfinite = m->flag;
    a.dev_error = db_device_error_ptr();
    a.block = c.block;
    a.bias = b;
    a.add_bias = 1;
    const db_gemm_config d = db_gemm_i8_default_config(T, N, DB_EPI_STORE);
    a.block_n = d.block_n;
    a.pair_ctas = d.pair_ctas;
    return db_launch_gemm_i8(a, m->stream);
}

// T rows: one sequence (nseq == 0), or nseq sequences packed one after another (m->cu holds
// their row boundaries, m->positions each row's position; attention per sequence, pooled into
// m->pooled [nseq, D]).
int forward(db_bert* m, int T, int nseq = 0, int max_len = 0) {
    const auto& c = m->cfg;
    const int D = c.hidden, F = c.ffn, H = c.heads, hd = D / H;
    cudaStream_t st = m->stream;
    cudaMemsetAsync(m->flag, 0, 4, st);
    embed_kernel<<<T, 256, 0, st>>>(m->ids, m->word, m->type, m->pos, nseq ? m->positions : nullptr, D, m->x);
    layer_norm_kernel<<<T, 128, 0, st>>>(m->x, nullptr, m->emb_ln_w, m->emb_ln_b, D, c.eps);
    int rc = (int)cudaGetLastError();
    for (int l = 0; l < c.layers && !rc; ++l) {
        const auto& w = m->layers[l];
        rc = linear(m, m->x, T, D, w.qkv_c, w.qkv_s, 3 * D, w.bqkv, m->qkv);
        if (rc) break;
        split_heads_kernel<<<T, 256, 0, st>>>(m->qkv, T, H, hd, m->q16, m->k16, m->v16);
        rc = nseq ? db_launch_attention_varlen(m->q16, m->k16, m->v16, m->cu, nseq, max_len, T, H, H,
                                               1.f / sqrtf((float)hd), m->ctx128, (int64_t)H * 128, nullptr, 0,
                                               nullptr, 0, nullptr, st)
                  : db_launch_attention(m->q16, m->k16, m->v16, T, H, H, 1.f / sqrtf((float)hd), m->ctx128,
                                        (int64_t)H * 128, st);
        if (rc) break;
        merge_heads_kernel<<<T, 256, 0, st>>>(m->ctx128, H, hd, m->ctx);
        rc = linear(m, m->ctx, T, D, w.o_c, w.o_s, D, w.bo, m->tmp);
        if (rc) break;
        layer_norm_kernel<<<T, 128, 0, st>>>(m->x, m->tmp, w.ln1_w, w.ln1_b, D, c.eps);
        rc = linear(m, m->x, T, D, w.f1_c, w.f1_s, F, w.b1, m->h);
        if (rc) break;
        gelu_kernel<<<grid_for((int64_t)T * F), 256, 0, st>>>(m->h, (int64_t)T * F);
        rc = linear(m, m->h, T, F, w.f2_c, w.f2_s, D, w.b2, m->tmp);
        if (rc) break;
        layer_norm_kernel<<<T, 128, 0, st>>>(m->x, m->tmp, w.ln2_w, w.ln2_b, D, c.eps);
        rc = (int)cudaGetLastError();
    }
    if (!rc) rc = nseq ? db_launch_mean_pool_varlen(m->x, D, m->cu, nseq, D, m->pooled, st)
                       : db_launch_mean_pool(m->x, D, T, D, m->pooled, st);
    return rc;
}

}  // namespace

extern "C" {

db_bert* db_bert_create_synthetic(int device, const db_bert_config* cfg, uint64_t seed, float stdv, db_error* err) {
    if (!cfg || cfg->layers <= 0 || cfg->hidden <= 0 || cfg->heads <= 0 || cfg->hidden % cfg->heads ||
        cfg->hidden / cfg->heads > 128 || cfg->hidden > 1024 || cfg->ffn <= 0 || cfg->vocab <= 0 ||
        cfg->max_positions <= 0 || cfg->max_positions > 4096 || (cfg->block != 32 && cfg->block != 64) ||
        !(cfg->eps > 0.f) || (cfg->mode != 0 && cfg->mode != 1)) {
        fill_error(err, "INVALID_PARAMETERS", "unsupported Decima encoder configuration");
        return nullptr;
    }
    if (device < 0 || device >= db_device_count() || cudaSetDevice(device) != cudaSuccess) {
        fill_error(err, "GPU_UNAVAILABLE", "no CUDA device " + std::to_string(device));
        return nullptr;
    }
    auto* m = new db_bert();
    m->device = device;
    m->cfg = *cfg;
    cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (build_synthetic(m, seed, stdv)) {
        fill_error(err, db_last_error_code(), db_last_error_message());
        db_bert_destroy(m);
        return nullptr;
    }
    return m;
}

void db_bert_destroy(db_bert* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (void* p : m->allocations) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int db_bert_predict(db_bert* m, const int32_t* ids, size_t n, float* pooled, float* hidden, db_error* err) {
    if (!m || !ids || !pooled) {
        fill_error(err, "INVALID_PARAMETERS", "null model, ids or output");
        return -1;
    }
    if (n == 0 || n > (size_t)m->cfg.max_positions) {
        fill_error(err, n == 0 ? "INVALID_REQUEST" : "INPUT_TOO_LONG",
                   "the encoder takes 1.." + std::to_string(m->cfg.max_positions) + " tokens");
        return -1;
    }
    for (size_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab) {
            fill_error(err, "INVALID_REQUEST", "token id " + std::to_string(ids[i]) + " outside the vocabulary");
            return -1;
        }
    cudaSetDevice(m->device);
    cudaMemcpyAsync(m->ids, ids, n * 4, cudaMemcpyHostToDevice, m->stream);
    const int rc = forward(m, (int)n);
    int flag = 0;
    cudaMemcpyAsync(&flag, m->flag, 4, cudaMemcpyDeviceToHost, m->stream);
    cudaMemcpyAsync(pooled, m->pooled, (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost, m->stream);
    if (hidden) cudaMemcpyAsync(hidden, m->x, n * m->cfg.hidden * 4, cudaMemcpyDeviceToHost, m->stream);
    const cudaError_t e = cudaStreamSynchronize(m->stream);
    if (rc || e != cudaSuccess) {
        fill_error(err, "INFERENCE_FAILED", rc ? cudaGetErrorString((cudaError_t)rc) : cudaGetErrorString(e));
        return -1;
    }
    if (flag) {
        fill_error(err, "INFERENCE_FAILED", "non-finite hidden state");
        return -1;
    }
    return 0;
}

// One request of the cross-encoder: sequence i = state ++ choices[i] (positions restart at 0 for
// every sequence), all count sequences packed into one pass; logits [count, DB_BERT_HEAD_OUTPUTS]
// = head(mean-pooled final state) per sequence, pooled [count, hidden] when non-null.
int db_bert_score(db_bert* m, const int32_t* state, size_t n_state, const int32_t* const* choices,
                  const size_t* choice_lens, size_t count, float* logits, float* pooled, db_error* err) {
    if (!m || (!state && n_state) || !choices || !choice_lens || !logits) {
        fill_error(err, "INVALID_PARAMETERS", "null model, state, choices or output");
        return -1;
    }
    if (count == 0 || count > (size_t)kBatchSeqs) {
        fill_error(err, "INVALID_REQUEST", "a request scores 1.." + std::to_string(kBatchSeqs) + " choices");
        return -1;
    }
    const auto& c = m->cfg;
    std::vector<int32_t> ids, pos;
    std::vector<int> cu(count + 1, 0);
    int max_len = 0;
    for (size_t i = 0; i < count; ++i) {
        const size_t L = n_state + choice_lens[i];
        if (L == 0 || L > (size_t)c.max_positions || (choice_lens[i] && !choices[i])) {
            fill_error(err, L == 0 || L <= (size_t)c.max_positions ? "INVALID_REQUEST" : "INPUT_TOO_LONG",
                       "each state + choice sequence takes 1.." + std::to_string(c.max_positions) + " tokens");
            return -1;
        }
        for (size_t t = 0; t < L; ++t) {
            const int32_t id = t < n_state ? state[t] : choices[i][t - n_state];
            if (id < 0 || id >= c.vocab) {
                fill_error(err, "INVALID_REQUEST", "token id " + std::to_string(id) + " outside the vocabulary");
                return -1;
            }
            ids.push_back(id);
            pos.push_back((int32_t)t);
        }
        cu[i + 1] = cu[i] + (int)L;
        max_len = std::max(max_len, (int)L);
    }
    const int T = cu[count], D = c.hidden, NO = DB_BERT_HEAD_OUTPUTS;
    cudaSetDevice(m->device);
    cudaStream_t st = m->stream;
    cudaMemcpyAsync(m->ids, ids.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->positions, pos.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->cu, cu.data(), (count + 1) * 4, cudaMemcpyHostToDevice, st);
    int rc = forward(m, T, (int)count, max_len);
    if (!rc) {
        head_kernel<<<(unsigned)count, 32 * NO, 0, st>>>(m->pooled, m->head_w, m->head_b, (int)count, D, NO, m->logits);
        rc = (int)cudaGetLastError();
    }
    int flag = 0;
    cudaMemcpyAsync(&flag, m->flag, 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(logits, m->logits, count * NO * 4, cudaMemcpyDeviceToHost, st);
    if (pooled) cudaMemcpyAsync(pooled, m->pooled, count * D * 4, cudaMemcpyDeviceToHost, st);
    const cudaError_t e = cudaStreamSynchronize(st);
    if (rc || e != cudaSuccess) {
        fill_error(err, "INFERENCE_FAILED", rc ? cudaGetErrorString((cudaError_t)rc) : cudaGetErrorString(e));
        return -1;
    }
    if (flag) {
        fill_error(err, "INFERENCE_FAILED", "non-finite hidden state");
        return -1;
    }
    return 0;
}

}  // extern "C"
