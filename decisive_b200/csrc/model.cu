// Model-level C ABI: the Pplx-shaped Q4/Q8 encoder on one device, behind a mirror of the
// reference's inference API (src/inference/mod.rs:140-273):
//   Model::create_cache / clear_cache / predict / predict_batch with cache ownership
//   (CACHE_OWNER), cancellation (CANCELLED), parameter validation (INVALID_PARAMETERS),
//   request validation (INVALID_REQUEST), the "never truncate" rule (INPUT_TOO_LONG,
//   input.rs:261-269) and the finiteness check of the hidden state (backbone.rs:243-247).
//
// Forward of one sequence (pre-norm residual block, backbone.rs:197-249, Qwen3 attention mixer):
//   x = embedding rows (quantized_rows.rs:89-110)
//   per layer: n = rms(x); qkv = Wqkv n; q,k = rope(qknorm(q,k)); ctx = attn(q,k,v);
//              x += Wo ctx; n = rms(x); h = silu(Wg n) * (Wu n); x += Wd h
//   pooled = mean_t rms(x)
// Every projection is the group-64 quantised GEMM; activations are quantised by the kernel
// that produces them (rms_quantize, the SwiGLU epilogue) except the attention context.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/decisive_b200.h"
#include "capi_internal.h"
#include "common.cuh"
#include "kernels.h"
#include "layer_ops.h"
#include "packed_io.h"

namespace {

struct LayerW {
    uint8_t *qkv_c = nullptr, *o_c = nullptr, *gu_c = nullptr, *dn_c = nullptr;
    float *qkv_s = nullptr, *o_s = nullptr, *gu_s = nullptr, *dn_s = nullptr;
    float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

void fill_error(db_error* err, const char* code, const std::string& msg) {
    if (!err) return;
    std::snprintf(err->code, sizeof err->code, "%s", code);
    std::snprintf(err->message, sizeof err->message, "%s", msg.c_str());
}

}  // namespace

static const char* kProfNames[DB_PROF_KINDS] = {"dequant_rows", "rms_quantize", "gemm_qkv", "qk_norm_rope",
                                                "attention", "quantize_rows", "gemm_o", "gemm_mlp_swiglu",
                                                "gemm_down", "final_norm", "mean_pool"};

struct db_model {
    int device = 0;
    db_encoder_config cfg{};
    cudaStream_t stream = nullptr;
    std::shared_ptr<char> identity = std::make_shared<char>(0);
    bool synthetic = false;
    uint64_t seed = 0;
    float std = 0.f;
    uint8_t* emb_c = nullptr;
    float* emb_s = nullptr;
    std::vector<LayerW> layers;
    float* final_norm = nullptr;
    std::vector<void*> allocations;
    // workspace for up to cap_T tokens
    int cap_T = 0;
    std::vector<void*> ws_allocations;
    int rope_T = 0;  // positions covered by the RoPE tables
    std::vector<void*> rope_allocations;
    // layer streaming (the reference's two-bank scheme, webgpu/streaming.rs): the projection weights
    // of every layer live in pinned host memory and are copied into one of two device banks on a
    // copy stream while the other bank's layer computes
    bool streaming = false;
    struct Span { size_t off, bytes; };
    std::vector<uint8_t*> host_layers;   // pinned, one block per layer
    std::vector<Span> spans;              // qkv_c, qkv_s, o_c, o_s, gu_c, gu_s, dn_c, dn_s inside a block
    size_t layer_bytes = 0;
    uint8_t* banks[2] = {nullptr, nullptr};
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t uploaded[2] = {nullptr, nullptr}, consumed[2] = {nullptr, nullptr};
    // per-layer prefix keys/values of a continuation call whose cache cannot keep them
    std::vector<__half*> tmp_k, tmp_v;
    int tmp_cap = 0;
    // continuation scoring: the prefix's last final-normed state [D] (when no cache keeps it), the
    // LM head's input rows [1 + continuation rows, D] and a logits chunk [kLmRows, vocab]
    float *prefix_last = nullptr, *lm_x = nullptr, *logits = nullptr;
    int lm_x_rows = 0;
    float *x = nullptr, *qkv = nullptr, *ctx = nullptr, *normed = nullptr, *pooled = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr, *sa = nullptr, *sh = nullptr;
    __half *acodes = nullptr, *hcodes = nullptr, *q16 = nullptr, *k16 = nullptr, *v16 = nullptr;
    int32_t* ids = nullptr;
    int32_t *cu = nullptr, *pos = nullptr;  // ragged batch: sequence boundaries, row positions
    int* flag = nullptr;
    int* dev_err = nullptr;
    // one CUDA graph per token count for the plain forward (captured on the second call for a T)
    bool use_graphs = true;
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int> graph_calls;
    void drop_graphs() {
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);
        graphs.clear();
        graph_calls.clear();
    }
    // tile configurations chosen by db_model_tune for qkv, o, gate/up, down (zero = defaults)
    db_gemm_config tuned[4] = {};
    // activation codes of the projections: int8 natural order through the kind::i8 GEMM (default),
    // or f16 codes through the kind::f16 GEMM (db_model_set_code_layout)
    bool i8 = true;
    // dequantised mode (DB_CODES_DQ): the layers' projections take f16(code * scale) activations
    // through the full-K kind::f16 GEMM (gemm_dq.cu); dq_w[2] hold the unpacked weights of
    // consecutive projections (alternating, so one projection's unpack overlaps the kernel before it
    // while the previous GEMM may still read the other buffer)
    bool dq = false;
    void* dq_w[2] = {nullptr, nullptr};
    // dequantised mode: the o and down projections split K in two; their partial sums ([2, T, D])
    // are added to the residual stream by the next RMSNorm kernel
    float* dq_part = nullptr;
    // per-launch CUDA-event profiling (mirror of the reference's projection_ms accounting,
    // cpu.rs:8-16 / native.rs:229-258), enabled by db_model_profile
    bool profile = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_next = 0;
    struct Rec { int kind; cudaEvent_t a, b; };
    std::vector<Rec> recs;
    double prof_ms[DB_PROF_KINDS] = {};
    int64_t prof_n[DB_PROF_KINDS] = {};
    cudaEvent_t next_event() {
        if (ev_next == ev_pool.size()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            ev_pool.push_back(e);
        }
        return ev_pool[ev_next++];
    }

    int D() const { return cfg.hidden; }
    int Nq() const { return cfg.q_heads * cfg.head_dim; }
    int Nk() const { return cfg.kv_heads * cfg.head_dim; }
    int Nqkv() const { return Nq() + 2 * Nk(); }
    int F() const { return cfg.ffn; }
    int Kmax() const { return std::max(std::max(D(), Nq()), F()); }

    template <class T>
    cudaError_t alloc(T** p, size_t count, std::vector<void*>& into) {
        cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 256);
        if (e == cudaSuccess) into.push_back(*p);
        return e;
    }
    void free_all(std::vector<void*>& v) {
        for (void* p : v) cudaFree(p);
        v.clear();
    }
};

struct db_cache {
    std::shared_ptr<char> identity;
    size_t max_bytes = 0;
    bool prefix_cache = false;
    // the kept prefix: its ids and, per layer, keys and values [cap_P, Hk, 128] f16
    int device = 0;
    std::vector<int32_t> ids;
    int cap_P = 0;
    std::vector<__half*> k, v;
    float* last = nullptr;  // the prefix's last final-normed state [hidden] (predicts the first continuation token)
    int64_t hits = 0, reused = 0, computed = 0;
    void release() {
        if (!k.empty() || last) cudaSetDevice(device);
        for (__half* p : k) cudaFree(p);
        for (__half* p : v) cudaFree(p);
        if (last) cudaFree(last);
        last = nullptr;
        k.clear();
        v.clear();
        ids.clear();
        cap_P = 0;
    }
    ~db_cache() { release(); }
};

namespace {

enum { T_EMB = 0, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN };
uint64_t tensor_id(int kind, int layer) { return kind == T_EMB ? 0 : 1 + 8ull * layer + (kind - 1); }

int check_config(const db_encoder_config* c, db_error* err) {
    if (!c || c->layers <= 0 || c->hidden <= 0 || c->hidden % 128 || c->hidden > 4096 || c->head_dim != 128 ||
        c->q_heads <= 0 || c->kv_heads <= 0 || c->q_heads % c->kv_heads || c->ffn <= 0 || c->ffn % 64 ||
        c->vocab <= 0 || (c->weight_bits != 4 && c->weight_bits != 8) || c->max_sequence_tokens <= 0) {
        fill_error(err, "INVALID_PARAMETERS", "unsupported encoder configuration");
        return -1;
    }
    return 0;
}

// Quantises a bf16 device tensor [N, K] into freshly allocated codes/scales.
int pack(db_model* m, const uint16_t* bf16, int N, int K, uint8_t** codes, float** scales) {
    const int G = (K + 63) / 64;
    if (m->alloc(codes, (size_t)N * G * 64 * m->cfg.weight_bits / 8, m->allocations) ||
        m->alloc(scales, (size_t)G * db_scale_stride(N), m->allocations))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight allocation exceeds device limits");
    return db_pack_weights_g64(bf16, N, K, m->cfg.weight_bits, *codes, *scales, m->stream);
}

int upload_norm(db_model* m, const float* host, int n, float** out) {
    if (m->alloc(out, n, m->allocations)) return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "norm allocation");
    if (host) return db_cuda_status(cudaMemcpy(*out, host, n * sizeof(float), cudaMemcpyHostToDevice), "norm upload");
    std::vector<float> ones(n, 1.f);
    return db_cuda_status(cudaMemcpy(*out, ones.data(), n * sizeof(float), cudaMemcpyHostToDevice), "norm upload");
}

// rotate-half RoPE table for positions 0..n-1 (backbone.rs:214-216, :471-483):
// angle = t * theta^(-2i/head_dim)
int ensure_rope(db_model* m, int n) {
    if (n <= m->rope_T) return 0;
    cudaStreamSynchronize(m->stream);
    m->drop_graphs();
    m->free_all(m->rope_allocations);
    m->rope_T = 0;
    if (m->alloc(&m->cos_t, (size_t)n * 64, m->rope_allocations) ||
        m->alloc(&m->sin_t, (size_t)n * 64, m->rope_allocations))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "RoPE table exceeds device limits");
    const int half = m->cfg.head_dim / 2;
    std::vector<float> freq(half), c((size_t)n * 64), s((size_t)n * 64);
    for (int i = 0; i < half; ++i) freq[i] = 1.f / powf(m->cfg.rope_theta, (float)(2 * i) / (float)m->cfg.head_dim);
    for (int t = 0; t < n; ++t)
        for (int i = 0; i < half; ++i) {
            const float angle = (float)t * freq[i];
            c[(size_t)t * 64 + i] = cosf(angle);
            s[(size_t)t * 64 + i] = sinf(angle);
        }
    cudaMemcpy(m->cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(m->sin_t, s.data(), s.size() * 4, cudaMemcpyHostToDevice);
    m->rope_T = n;
    return 0;
}

int ensure_workspace(db_model* m, int T) {
    if (T <= m->cap_T) return 0;
    cudaStreamSynchronize(m->stream);
    m->drop_graphs();  // captured graphs hold the old buffers
    m->free_all(m->ws_allocations);
    m->cap_T = 0;
    const int D = m->D(), F = m->F(), Kmax = m->Kmax();
    const int Gmax = (Kmax + 63) / 64;
    auto& v = m->ws_allocations;
    if (m->alloc(&m->x, (size_t)T * D, v) || m->alloc(&m->qkv, (size_t)T * m->Nqkv(), v) ||
        m->alloc(&m->ctx, (size_t)T * m->Nq(), v) || m->alloc(&m->normed, (size_t)T * D, v) ||
        m->alloc(&m->pooled, (size_t)T * D, v) || m->alloc(&m->cu, (size_t)T + 1, v) ||
        m->alloc(&m->pos, (size_t)T, v) ||
        m->alloc(&m->sa, (size_t)Gmax * db_scale_stride(T), v) || m->alloc(&m->sh, (size_t)(F / 64) * db_scale_stride(T), v) ||
        m->alloc(&m->acodes, (size_t)T * Kmax, v) || m->alloc(&m->hcodes, (size_t)T * F, v) ||
        m->alloc(&m->q16, (size_t)T * m->Nq(), v) || m->alloc(&m->k16, (size_t)T * m->Nk(), v) ||
        m->alloc(&m->v16, (size_t)T * m->Nk(), v) || m->alloc(&m->ids, T, v) || m->alloc(&m->flag, 4, v) ||
        (m->dq && m->alloc(&m->dq_part, (size_t)2 * T * D, v)))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "workspace exceeds device limits");
    m->cap_T = T;
    return ensure_rope(m, T);
}

int build(db_model* m, const db_encoder_weights* w) {
    const int D = m->D(), L = m->cfg.layers, F = m->F(), Nq = m->Nq(), Nk = m->Nk();
    cudaStream_t st = m->stream;
    // scratch bf16 buffer big enough for any one projection block
    const size_t big = std::max({(size_t)m->cfg.vocab * D, (size_t)m->Nqkv() * D, (size_t)F * D, (size_t)D * Nq});
    uint16_t* scratch = nullptr;
    if (cudaMalloc(&scratch, big * 2 + 256) != cudaSuccess)
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight staging exceeds device limits");
    auto fill = [&](int kind, int layer, const uint16_t* host, size_t n, uint16_t* dst) -> int {
        if (m->synthetic) return db_synthetic_bf16(m->seed, tensor_id(kind, layer), (int64_t)n, m->std, dst, st);
        return db_cuda_status(cudaMemcpyAsync(dst, host, n * 2, cudaMemcpyHostToDevice, st), "weight upload");
    };
    int rc = 0;
    rc = fill(T_EMB, 0, w ? w->embedding : nullptr, (size_t)m->cfg.vocab * D, scratch);
    if (!rc) rc = pack(m, scratch, m->cfg.vocab, D, &m->emb_c, &m->emb_s);
    m->layers.resize(L);
    for (int l = 0; l < L && !rc; ++l) {
        LayerW& lw = m->layers[l];
        rc = fill(T_Q, l, w ? w->q[l] : nullptr, (size_t)Nq * D, scratch);
        if (!rc) rc = fill(T_K, l, w ? w->k[l] : nullptr, (size_t)Nk * D, scratch + (size_t)Nq * D);
        if (!rc) rc = fill(T_V, l, w ? w->v[l] : nullptr, (size_t)Nk * D, scratch + (size_t)(Nq + Nk) * D);
        if (!rc) rc = pack(m, scratch, m->Nqkv(), D, &lw.qkv_c, &lw.qkv_s);
        if (!rc) rc = fill(T_O, l, w ? w->o[l] : nullptr, (size_t)D * Nq, scratch);
        if (!rc) rc = pack(m, scratch, D, Nq, &lw.o_c, &lw.o_s);
        uint8_t *gc = nullptr, *uc = nullptr;
        float *gs = nullptr, *us = nullptr;
        if (!rc) rc = fill(T_GATE, l, w ? w->gate[l] : nullptr, (size_t)F * D, scratch);
        if (!rc) rc = pack(m, scratch, F, D, &gc, &gs);
        if (!rc) rc = fill(T_UP, l, w ? w->up[l] : nullptr, (size_t)F * D, scratch);
        if (!rc) rc = pack(m, scratch, F, D, &uc, &us);
        if (!rc) {
            const int G = (D + 63) / 64;
            if (m->alloc(&lw.gu_c, (size_t)2 * F * G * 64 * m->cfg.weight_bits / 8, m->allocations) ||
                m->alloc(&lw.gu_s, (size_t)G * db_scale_stride(2 * F), m->allocations))
                rc = db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight allocation exceeds device limits");
            if (!rc) rc = db_interleave_gate_up(gc, gs, uc, us, F, D, m->cfg.weight_bits, lw.gu_c, lw.gu_s, st);
            cudaStreamSynchronize(st);
        }
        if (!rc) rc = fill(T_DOWN, l, w ? w->down[l] : nullptr, (size_t)D * F, scratch);
        if (!rc) rc = pack(m, scratch, D, F, &lw.dn_c, &lw.dn_s);
        if (!rc) rc = upload_norm(m, w ? w->input_norm[l] : nullptr, D, &lw.in_norm);
        if (!rc) rc = upload_norm(m, w ? w->post_norm[l] : nullptr, D, &lw.post_norm);
        if (!rc) rc = upload_norm(m, w ? w->q_norm[l] : nullptr, m->cfg.head_dim, &lw.q_norm);
        if (!rc) rc = upload_norm(m, w ? w->k_norm[l] : nullptr, m->cfg.head_dim, &lw.k_norm);
    }
    if (!rc) rc = upload_norm(m, w ? w->final_norm : nullptr, D, &m->final_norm);
    cudaStreamSynchronize(st);
    cudaFree(scratch);
    if (!rc) rc = ensure_workspace(m, m->cfg.max_sequence_tokens);
    return rc;
}

db_model* create(int device, const db_encoder_config* cfg, const db_encoder_weights* w, bool synthetic,
                 uint64_t seed, float stdv, db_error* err) {
    if (check_config(cfg, err)) return nullptr;
    if (device < 0 || device >= db_device_count() || cudaSetDevice(device) != cudaSuccess) {
        fill_error(err, "GPU_UNAVAILABLE", "no CUDA device " + std::to_string(device));
        return nullptr;
    }
    auto* m = new db_model();
    m->device = device;
    m->cfg = *cfg;
    m->synthetic = synthetic;
    m->seed = seed;
    m->std = stdv;
    m->dev_err = db_device_error_ptr();
    cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (build(m, w)) {
        fill_error(err, db_last_error_code(), db_last_error_message());
        db_model_destroy(m);
        return nullptr;
    }
    return m;
}

// A decoder pass over `items` sequences of T tokens each: RoPE positions start at `prefix`, the
// attention of every item also sees the cached prefix keys/values pk[l], pv[l] (P = prefix rows);
// sk/sv (a prefix pass) receive each layer's own keys and values; pool: mean-pool into m->pooled.
struct Pass {
    int items = 1;
    int prefix = 0;
    __half* const* pk = nullptr;
    __half* const* pv = nullptr;
    __half* const* sk = nullptr;
    __half* const* sv = nullptr;
    bool pool = true;
    // ragged encoder batch: nseq sequences packed into T rows, sequence i = rows cu[i]..cu[i+1]-1
    // (device arrays; pos = each row's position in its sequence), pooled into m->pooled [nseq, D]
    const int* cu = nullptr;
    const int* pos = nullptr;
    int nseq = 0;
    int max_len = 0;
};

// Enqueues the forward of ids (device, T tokens) -> m->pooled.  Host-side cancellation is polled
// between layers.  Returns 0, 1 when cancelled, or a negative status.
int enqueue_forward(db_model* m, int T, const volatile uint8_t* cancel, const Pass* pass = nullptr) {
    // rows: `items` token sequences of T tokens one after another
    const int items = pass ? pass->items : 1, R = items * T, P = pass ? pass->prefix : 0;
    const auto& c = m->cfg;
    const int D = c.hidden, Nq = m->Nq(), F = m->F(), Nqkv = m->Nqkv();
    const int bits = c.weight_bits, fused = c.fused;
    cudaStream_t st = m->stream;
    const int64_t ld_codes = m->Kmax(), lds = db_scale_stride(m->cap_T);
    int rc = 0;
    auto timed = [&](int kind, auto&& launch) -> int {
        if (!m->profile) return launch();
        cudaEvent_t a = m->next_event(), b = m->next_event();
        cudaEventRecord(a, st);
        const int r = launch();
        cudaEventRecord(b, st);
        m->recs.push_back({kind, a, b});
        return r;
    };
    cudaMemsetAsync(m->flag, 0, sizeof(int), st);
    rc = timed(0, [&] {
        return db_launch_dequant_rows(m->emb_c, m->emb_s, c.vocab, D, bits, m->ids, R, m->x, D, m->flag, st);
    });
    const int code_layout = m->dq ? DB_CODES_DQ_F16 : m->i8 ? DB_CODES_NATURAL_I8 : DB_CODES_TC_F16;
    const int attn_codes = m->dq ? 2 : m->i8 ? 1 : 0;  // the attention's quantised output layout
    // one projection; the tuned tile configuration, else the i8 path's default for the shape
    auto launch = [&](int proj, DbGemmArgs& g) {
        if (m->dq) {
            g.w_scratch = m->dq_w[proj & 1];  // qkv, gate/up: 0; o, down: 1
            g.overlap_unpack = 1;
            return db_launch_gemm_dq(g, st);
        }
        g.block_n = m->tuned[proj].block_n;
        g.max_ctas = m->tuned[proj].max_ctas;
        g.pair_ctas = m->tuned[proj].pair_ctas;
        if (!m->i8) return db_launch_gemm_tc(g, st);
        if (g.block_n == 0) {
            const db_gemm_config d = db_gemm_i8_default_config(g.M, g.N, g.epilogue);
            g.block_n = d.block_n;
            g.pair_ctas = d.pair_ctas;
        }
        return db_launch_gemm_i8(g, st);
    };
    auto gemm = [&](int proj, const void* a, const uint8_t* wc, const float* ws, const float* sa, int N, int K, int epi,
                    float* y, int64_t ldy, int ksplit = 0) {
        DbGemmArgs g{};
        g.k_splits = ksplit;
        g.a_codes = a;
        g.lda = ld_codes;
        g.sa = sa;
        g.ldsa = lds;
        g.w_codes = wc;
        g.sw = ws;
        g.M = R;
        g.N = N;
        g.K = K;
        g.bits = bits;
        g.fused = fused;
        g.epilogue = epi;
        g.y = y;
        g.ldy = ldy;
        g.out_codes = m->hcodes;
        g.ldoc = F;
        g.out_scales = m->sh;
        g.ldos = lds;
        g.nonfinite = m->flag;
        g.dev_error = m->dev_err;
        return launch(proj, g);
    };
    const float attn_scale = 1.f / sqrtf((float)c.head_dim);
    auto own_k = [&](int l) { return pass && pass->sk ? pass->sk[l] : m->k16; };
    auto own_v = [&](int l) { return pass && pass->sv ? pass->sv[l] : m->v16; };
    // streaming: layer l computes from bank l % 2; the upload of layer l + 2 into that bank waits
    // for layer l's last kernel (the copy stream and the compute stream meet only at events)
    auto upload = [&](int l) {
        const int b = l & 1;
        cudaStreamWaitEvent(m->copy_stream, m->consumed[b], 0);
        cudaMemcpyAsync(m->banks[b], m->host_layers[l], m->layer_bytes, cudaMemcpyHostToDevice, m->copy_stream);
        cudaEventRecord(m->uploaded[b], m->copy_stream);
    };
    auto bank_layer = [&](int l) {
        LayerW w = m->layers[l];  // norms stay resident
        uint8_t* base = m->banks[l & 1];
        auto at = [&](int i) { return base + m->spans[i].off; };
        w.qkv_c = at(0);
        w.qkv_s = reinterpret_cast<float*>(at(1));
        w.o_c = at(2);
        w.o_s = reinterpret_cast<float*>(at(3));
        w.gu_c = at(4);
        w.gu_s = reinterpret_cast<float*>(at(5));
        w.dn_c = at(6);
        w.dn_s = reinterpret_cast<float*>(at(7));
        return w;
    };
    if (m->streaming) {
        upload(0);
        if (c.layers > 1) upload(1);
    }
    // dequantised mode: the o and down projections store two K-half partial sums (dq_part); the next
    // RMSNorm kernel adds them to the residual stream, (x + p0) + p1, in that order
    const float* pend = nullptr;
    auto take = [&](int i) -> const float* {
        if (!pend) return nullptr;
        return i == 0 ? pend : pend + (size_t)R * D;
    };
    for (int l = 0; l < c.layers && !rc; ++l) {
        if (cancel && *cancel) return 1;
        if (m->streaming) cudaStreamWaitEvent(st, m->uploaded[l & 1], 0);
        const LayerW w = m->streaming ? bank_layer(l) : m->layers[l];
        rc = timed(1, [&] {
            return db_launch_rms_quantize(m->x, D, w.in_norm, R, D, c.eps, 0, nullptr, 0, m->acodes, code_layout,
                                          ld_codes, m->sa, nullptr, lds, m->flag, st, 1, take(0), take(1));
        });
        pend = nullptr;
        if (!rc) rc = timed(2, [&] { return gemm(0, m->acodes, w.qkv_c, w.qkv_s, m->sa, Nqkv, D, DB_EPI_STORE, m->qkv, Nqkv); });
        if (!rc)
            rc = timed(3, [&] {
                // a prefix pass stores this layer's keys and values straight into the cache
                return db_launch_qk_norm_rope(m->qkv, Nqkv, R, c.q_heads, c.kv_heads, w.q_norm, w.k_norm, c.eps,
                                              m->cos_t, m->sin_t, m->q16, own_k(l), own_v(l), st, P, T,
                                              pass ? pass->pos : nullptr);
            });
        // attention writes the context already quantised for the output projection
        if (!rc)
            rc = timed(4, [&] {
                if (!c.causal && pass && pass->cu)
                    return db_launch_attention_varlen(m->q16, m->k16, m->v16, pass->cu, pass->nseq, pass->max_len, R,
                                                      c.q_heads, c.kv_heads, attn_scale, nullptr, 0, m->acodes,
                                                      ld_codes, m->sa, lds, m->flag, st, attn_codes);
                if (!c.causal && !pass)
                    return db_launch_attention_quant(m->q16, m->k16, m->v16, T, c.q_heads, c.kv_heads, attn_scale,
                                                     m->acodes, ld_codes, m->sa, lds, m->flag, st, attn_codes);
                return db_launch_attention_prefix_quant(m->q16, own_k(l), own_v(l), items, T,
                                                        pass && pass->pk ? pass->pk[l] : nullptr,
                                                        pass && pass->pv ? pass->pv[l] : nullptr, P, c.causal,
                                                        c.q_heads, c.kv_heads, attn_scale,
                                                        m->acodes, ld_codes, m->sa, lds, m->flag, st, attn_codes);
            });
        // (a split needs at least two 64-groups of K)
        if (!rc && m->dq && Nq >= 128) {
            rc = timed(6, [&] { return gemm(1, m->acodes, w.o_c, w.o_s, m->sa, D, Nq, DB_EPI_STORE, m->dq_part, D, 2); });
            pend = m->dq_part;
        } else if (!rc) {
            rc = timed(6, [&] { return gemm(1, m->acodes, w.o_c, w.o_s, m->sa, D, Nq, DB_EPI_RESIDUAL, m->x, D); });
        }
        if (!rc)
            rc = timed(1, [&] {
                return db_launch_rms_quantize(m->x, D, w.post_norm, R, D, c.eps, 0, nullptr, 0, m->acodes, code_layout,
                                              ld_codes, m->sa, nullptr, lds, m->flag, st, 1, take(0), take(1));
            });
        pend = nullptr;
        if (!rc)
            rc = timed(7, [&] { return gemm(2, m->acodes, w.gu_c, w.gu_s, m->sa, 2 * F, D, DB_EPI_SWIGLU_QUANT, nullptr, 0); });
        if (!rc) rc = timed(8, [&] {
            DbGemmArgs g{};
            g.a_codes = m->hcodes;
            g.lda = F;
            g.sa = m->sh;
            g.ldsa = lds;
            g.w_codes = w.dn_c;
            g.sw = w.dn_s;
            g.M = R;
            g.N = D;
            g.K = F;
            g.bits = bits;
            g.fused = fused;
            g.epilogue = DB_EPI_RESIDUAL;
            g.y = m->x;
            g.ldy = D;
            if (m->dq && F >= 128) {
                g.epilogue = DB_EPI_STORE;  // two K-half partial sums, added by the next RMSNorm
                g.y = m->dq_part;
                g.k_splits = 2;
            }
            g.nonfinite = m->flag;
            g.dev_error = m->dev_err;
            return launch(3, g);
        });
        if (!rc && m->dq && F >= 128) pend = m->dq_part;
        if (m->streaming) {
            cudaEventRecord(m->consumed[l & 1], st);
            if (l + 2 < c.layers) upload(l + 2);
        }
    }
    if (!rc)
        rc = timed(9, [&] {
            return db_launch_rms_quantize(m->x, D, m->final_norm, R, D, c.eps, 0, m->normed, D, nullptr, DB_CODES_TC, 0,
                                          nullptr, nullptr, 0, m->flag, st, 1, take(0), take(1));
        });
    if (!rc && pass && pass->cu)
        rc = timed(10, [&] { return db_launch_mean_pool_varlen(m->normed, D, pass->cu, pass->nseq, D, m->pooled, st); });
    else if (!rc && (!pass || pass->pool))
        rc = timed(10, [&] { return db_launch_mean_pool(m->normed, D, T, D, m->pooled, st); });
    return rc ? db_cuda_status(rc, "forward") : 0;
}

// Runs the plain forward of T tokens.  From the second call for a T on, it runs as one CUDA graph
// (captured then), which removes the per-launch gaps of ~230 kernels; the layer-by-layer path is
// kept when a cancellation flag must be polled between layers (as the reference does), when
// per-kernel profiling is on, while weights stream, or when graphs are switched off.
int run_forward(db_model* m, int T, const volatile uint8_t* cancel) {
    if (cancel || m->profile || m->streaming || !m->use_graphs) return enqueue_forward(m, T, cancel);
    auto it = m->graphs.find(T);
    if (it == m->graphs.end()) {
        if (m->graph_calls[T]++ == 0) return enqueue_forward(m, T, nullptr);  // first call: eager
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            return enqueue_forward(m, T, nullptr);
        }
        const int rc = enqueue_forward(m, T, nullptr);
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rc || e != cudaSuccess || !g) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            m->use_graphs = false;  // capture failed: stay eager
            return enqueue_forward(m, T, nullptr);
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            cudaGetLastError();
            m->use_graphs = false;
            return enqueue_forward(m, T, nullptr);
        }
        it = m->graphs.emplace(T, exec).first;
    }
    return db_cuda_status((int)cudaGraphLaunch(it->second, m->stream), "graph launch");
}

// Backend::predict for one request; errors use the reference's codes.
int predict_one(db_model* m, const int32_t* ids, size_t n, const db_parameters* params, const volatile uint8_t* cancel,
                float* out, db_error* err) {
    if (cancel && *cancel) {
        fill_error(err, "CANCELLED", "Inference was cancelled");
        return -1;
    }
    if (!ids || n == 0) {
        fill_error(err, "INVALID_REQUEST", "a nonempty token sequence is required");
        return -1;
    }
    const int limit = params ? params->max_sequence_tokens : m->cfg.max_sequence_tokens;
    if (limit <= 0) {
        fill_error(err, "INVALID_PARAMETERS", "maxSequenceTokens must be positive");
        return -1;
    }
    if (n > (size_t)limit) {
        fill_error(err, "INPUT_TOO_LONG", "single question exceeds token limit: " + std::to_string(n) + " > " +
                                              std::to_string(limit) + "; inputs are never truncated");
        return -1;
    }
    for (size_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab) {
            fill_error(err, "INVALID_REQUEST", "token id " + std::to_string(ids[i]) + " outside the vocabulary");
            return -1;
        }
    cudaSetDevice(m->device);
    if (ensure_workspace(m, (int)n)) {
        fill_error(err, "RESOURCE_LIMIT", db_last_error_message());
        return -1;
    }
    cudaMemcpyAsync(m->ids, ids, n * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream);
    int rc = run_forward(m, (int)n, cancel);
    if (rc == 1) {
        cudaStreamSynchronize(m->stream);
        fill_error(err, "CANCELLED", "Inference was cancelled");
        return -1;
    }
    int flag = 0;
    cudaMemcpyAsync(&flag, m->flag, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    cudaMemcpyAsync(out, m->pooled, m->cfg.hidden * sizeof(float), cudaMemcpyDeviceToHost, m->stream);
    const cudaError_t e = cudaStreamSynchronize(m->stream);
    if (rc || e != cudaSuccess) {
        fill_error(err, "INFERENCE_FAILED", rc ? db_last_error_message() : cudaGetErrorString(e));
        return -1;
    }
    int word = 0;
    cudaMemcpy(&word, m->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (word) {
        cudaMemset(m->dev_err, 0, sizeof(int));
        fill_error(err, "INFERENCE_FAILED", "device wait expired (error word " + std::to_string(word) + ")");
        return -1;
    }
    if (flag) {
        fill_error(err, "INFERENCE_FAILED", "non-finite hidden state");
        return -1;
    }
    if (cancel && *cancel) {
        fill_error(err, "CANCELLED", "Inference was cancelled");
        return -1;
    }
    return 0;
}

// Request checks of predict_one (the reference's codes); returns 0 or fills err.
int validate_request(const db_model* m, const int32_t* ids, size_t n, int limit, db_error* err) {
    if (!ids || n == 0) {
        fill_error(err, "INVALID_REQUEST", "a nonempty token sequence is required");
        return -1;
    }
    if (n > (size_t)limit) {
        fill_error(err, "INPUT_TOO_LONG", "single question exceeds token limit: " + std::to_string(n) + " > " +
                                              std::to_string(limit) + "; inputs are never truncated");
        return -1;
    }
    for (size_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab) {
            fill_error(err, "INVALID_REQUEST", "token id " + std::to_string(ids[i]) + " outside the vocabulary");
            return -1;
        }
    return 0;
}

// Model::predict_batch for an encoder (mod.rs:250-273: ordered outcomes, one per request) as packed
// ragged passes: the valid requests' tokens are concatenated (up to kPackRows rows per pass), every
// row-wise kernel and GEMM runs once over all rows, attention runs per sequence over its own keys
// (cu_seqlens), and each sequence is mean-pooled.  Every kernel computes a row (or a sequence's
// attention) exactly as the one-request forward does, so outcomes are bit-identical to predict.
// A pass whose hidden state turns non-finite is re-run request by request, so that the failure is
// reported for the request it belongs to.
constexpr size_t kPackRows = 65536;
int predict_packed(db_model* m, const int32_t* const* ids, const size_t* lens, size_t count,
                   const db_parameters* params, const volatile uint8_t* cancel, float* outs, int32_t* status,
                   db_error* errs) {
    const int D = m->cfg.hidden;
    const int limit = params ? params->max_sequence_tokens : m->cfg.max_sequence_tokens;
    std::vector<size_t> valid;
    for (size_t i = 0; i < count; ++i) {
        db_error* e = errs ? &errs[i] : nullptr;
        status[i] = -1;
        if (cancel && *cancel) {
            fill_error(e, "CANCELLED", "Inference was cancelled");
        } else if (limit <= 0) {
            fill_error(e, "INVALID_PARAMETERS", "maxSequenceTokens must be positive");
        } else if (validate_request(m, ids[i], lens[i], limit, e) == 0) {
            valid.push_back(i);
        }
    }
    cudaSetDevice(m->device);
    size_t next = 0;
    while (next < valid.size()) {
        // one pass: as many whole requests as fit kPackRows rows (and the grid's 65535 sequences)
        size_t end = next, rows = 0;
        while (end < valid.size() && end - next < 65535 && (end == next || rows + lens[valid[end]] <= kPackRows))
            rows += lens[valid[end++]];
        const int nseq = (int)(end - next), R = (int)rows;
        auto fail_all = [&](const char* code, const std::string& msg) {
            for (size_t k = next; k < end; ++k) fill_error(errs ? &errs[valid[k]] : nullptr, code, msg);
        };
        if (cancel && *cancel) {
            fail_all("CANCELLED", "Inference was cancelled");
            next = end;
            continue;
        }
        if (ensure_workspace(m, R)) {
            fail_all("RESOURCE_LIMIT", db_last_error_message());
            next = end;
            continue;
        }
        std::vector<int32_t> h_ids(R), h_pos(R), h_cu(nseq + 1);
        int max_len = 0, r0 = 0;
        for (int k = 0; k < nseq; ++k) {
            const size_t i = valid[next + k];
            const int n = (int)lens[i];
            h_cu[k] = r0;
            std::memcpy(h_ids.data() + r0, ids[i], (size_t)n * sizeof(int32_t));
            for (int t = 0; t < n; ++t) h_pos[r0 + t] = t;
            r0 += n;
            max_len = std::max(max_len, n);
        }
        h_cu[nseq] = R;
        cudaMemcpyAsync(m->ids, h_ids.data(), (size_t)R * 4, cudaMemcpyHostToDevice, m->stream);
        cudaMemcpyAsync(m->pos, h_pos.data(), (size_t)R * 4, cudaMemcpyHostToDevice, m->stream);
        cudaMemcpyAsync(m->cu, h_cu.data(), (size_t)(nseq + 1) * 4, cudaMemcpyHostToDevice, m->stream);
        Pass pass;
        pass.cu = m->cu;
        pass.pos = m->pos;
        pass.nseq = nseq;
        pass.max_len = max_len;
        const int rc = enqueue_forward(m, R, cancel, &pass);
        std::vector<float> pooled((size_t)nseq * D);
        int flag = 0;
        if (rc == 0) {
            cudaMemcpyAsync(&flag, m->flag, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
            cudaMemcpyAsync(pooled.data(), m->pooled, pooled.size() * 4, cudaMemcpyDeviceToHost, m->stream);
        }
        const cudaError_t e = cudaStreamSynchronize(m->stream);
        if (rc == 1 || (cancel && *cancel)) {
            fail_all("CANCELLED", "Inference was cancelled");
        } else if (rc || e != cudaSuccess) {
            fail_all("INFERENCE_FAILED", rc ? db_last_error_message() : cudaGetErrorString(e));
        } else {
            int word = 0;
            cudaMemcpy(&word, m->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
            if (word) {
                cudaMemset(m->dev_err, 0, sizeof(int));
                fail_all("INFERENCE_FAILED", "device wait expired (error word " + std::to_string(word) + ")");
            } else if (flag) {
                for (size_t k = next; k < end; ++k) {
                    const size_t i = valid[k];
                    status[i] = predict_one(m, ids[i], lens[i], params, cancel, outs + i * (size_t)D,
                                            errs ? &errs[i] : nullptr);
                }
            } else {
                for (int k = 0; k < nseq; ++k) {
                    const size_t i = valid[next + k];
                    std::memcpy(outs + i * (size_t)D, pooled.data() + (size_t)k * D, (size_t)D * sizeof(float));
                    status[i] = 0;
                }
            }
        }
        next = end;
    }
    return 0;
}

}  // namespace

namespace {

// ---- packed checkpoints (the reference's export_packed.rs:13-103 manifest and file layout)
const char* kLayerTensors[11] = {"self_attn.q_proj.weight",  "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                 "self_attn.o_proj.weight",  "mlp.gate_proj.weight",    "mlp.up_proj.weight",
                                 "mlp.down_proj.weight",     "input_layernorm.weight",  "post_attention_layernorm.weight",
                                 "self_attn.q_norm.weight",  "self_attn.k_norm.weight"};

inline size_t group_bytes(int bits) { return bits == 4 ? 36 : 68; }  // packed.rs:10-20
inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
inline float bf16_to_f32(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// device layout [N, K] -> packed row-group bytes on the host
int export_matrix(db_model* m, const uint8_t* codes, const float* scales, int N, int K, uint8_t* dev_stage,
                  std::vector<uint8_t>* out) {
    const size_t bytes = (size_t)N * (K / 64) * group_bytes(m->cfg.weight_bits);
    int rc = db_export_packed(codes, scales, N, K, m->cfg.weight_bits, dev_stage, m->stream);
    out->resize(bytes);
    if (!rc) rc = db_cuda_status(cudaMemcpyAsync(out->data(), dev_stage, bytes, cudaMemcpyDeviceToHost, m->stream),
                                 "export copy");
    if (!rc) rc = db_cuda_status(cudaStreamSynchronize(m->stream), "export");
    return rc;
}
std::vector<uint8_t> norm_bytes(const float* dev, int n) {
    std::vector<float> h(n);
    cudaMemcpy(h.data(), dev, n * 4, cudaMemcpyDeviceToHost);
    std::vector<uint8_t> b(2 * n);
    for (int i = 0; i < n; ++i) {
        const uint16_t v = f32_to_bf16_rne(h[i]);
        b[2 * i] = (uint8_t)v;
        b[2 * i + 1] = (uint8_t)(v >> 8);
    }
    return b;
}

// packed row-group bytes (host) -> freshly allocated device codes/scales
int import_matrix(db_model* m, const uint8_t* packed, int N, int K, uint8_t* dev_stage, uint8_t** codes,
                  float** scales) {
    const int G = K / 64, bits = m->cfg.weight_bits;
    if (m->alloc(codes, (size_t)N * G * 64 * bits / 8, m->allocations) ||
        m->alloc(scales, (size_t)G * db_scale_stride(N), m->allocations))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight allocation exceeds device limits");
    cudaMemsetAsync(*scales, 0, (size_t)G * db_scale_stride(N) * 4, m->stream);
    const size_t bytes = (size_t)N * G * group_bytes(bits);
    int rc = db_cuda_status(cudaMemcpyAsync(dev_stage, packed, bytes, cudaMemcpyHostToDevice, m->stream), "upload");
    if (!rc) rc = db_import_packed(dev_stage, N, K, bits, *codes, *scales, m->stream);
    if (!rc) rc = db_cuda_status(cudaStreamSynchronize(m->stream), "import");
    return rc;
}

int norm_from_bytes(db_model* m, const uint8_t* p, int n, float** out) {
    std::vector<float> h(n);
    for (int i = 0; i < n; ++i) h[i] = bf16_to_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
    return upload_norm(m, h.data(), n, out);
}

int build_packed(db_model* m, const dbio::Manifest& man, const std::string& dir, bool verify) {
    const int D = m->D(), L = m->cfg.layers, F = m->F(), Nq = m->Nq(), Nk = m->Nk(), bits = m->cfg.weight_bits;
    const size_t gb = group_bytes(bits);
    std::string err;
    if (man.bits != bits) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_WEIGHTS", "manifest scheme is not Q" + std::to_string(bits));
    if ((int)man.layers.size() < L) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_WEIGHTS", "manifest has too few layers");
    const size_t big = std::max({(size_t)m->cfg.vocab * D, (size_t)m->Nqkv() * D, (size_t)F * D, (size_t)D * Nq}) / 64 * gb;
    uint8_t* stage = nullptr;
    if (cudaMalloc(&stage, big + 256) != cudaSuccess)
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight staging exceeds device limits");
    auto bad = [&](const std::string& what) { return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_WEIGHTS", what); };
    int rc = 0;
    std::vector<uint8_t> bytes;
    if (!dbio::read_checked(dir, man.embedding, man, verify, &bytes, &err)) rc = bad(err);
    else if (bytes.size() != (size_t)m->cfg.vocab * (D / 64) * gb) rc = bad("embedding size does not match the configuration");
    if (!rc) rc = import_matrix(m, bytes.data(), m->cfg.vocab, D, stage, &m->emb_c, &m->emb_s);
    m->layers.resize(L);
    for (int l = 0; l < L && !rc; ++l) {
        const dbio::LayerEntry& le = man.layers[l];
        if (!dbio::read_checked(dir, le.file, man, verify, &bytes, &err)) { rc = bad(err); break; }
        const dbio::TensorEntry* t[11];
        const int64_t rows[11] = {Nq, Nk, Nk, D, F, F, D, D, D, m->cfg.head_dim, m->cfg.head_dim};
        const int64_t cols[11] = {D, D, D, Nq, D, D, F, 0, 0, 0, 0};
        for (int i = 0; i < 11 && !rc; ++i) {
            t[i] = le.find_suffix(std::string("layers.") + std::to_string(l) + "." + kLayerTensors[i]);
            if (!t[i]) { rc = bad(le.file + ": missing " + kLayerTensors[i]); break; }
            const bool mat = cols[i] > 0;
            const size_t want = mat ? (size_t)rows[i] * (cols[i] / 64) * gb : (size_t)rows[i] * 2;
            const bool shape_ok = mat ? (t[i]->shape.size() == 2 && t[i]->shape[0] == rows[i] && t[i]->shape[1] == cols[i])
                                      : (t[i]->shape.size() == 1 && t[i]->shape[0] == rows[i]);
            if (!shape_ok || t[i]->end - t[i]->start != want || t[i]->end > bytes.size())
                rc = bad(t[i]->name + ": shape or byte range does not match the configuration");
        }
        if (rc) break;
        LayerW& lw = m->layers[l];
        // q, k and v rows one after another are the packed form of the concatenated projection
        std::vector<uint8_t> qkv;
        for (int i = 0; i < 3; ++i) qkv.insert(qkv.end(), bytes.begin() + t[i]->start, bytes.begin() + t[i]->end);
        rc = import_matrix(m, qkv.data(), m->Nqkv(), D, stage, &lw.qkv_c, &lw.qkv_s);
        if (!rc) rc = import_matrix(m, bytes.data() + t[3]->start, D, Nq, stage, &lw.o_c, &lw.o_s);
        uint8_t *gc = nullptr, *uc = nullptr;
        float *gs = nullptr, *us = nullptr;
        if (!rc) rc = import_matrix(m, bytes.data() + t[4]->start, F, D, stage, &gc, &gs);
        if (!rc) rc = import_matrix(m, bytes.data() + t[5]->start, F, D, stage, &uc, &us);
        if (!rc) {
            const int G = D / 64;
            if (m->alloc(&lw.gu_c, (size_t)2 * F * G * 64 * bits / 8, m->allocations) ||
                m->alloc(&lw.gu_s, (size_t)G * db_scale_stride(2 * F), m->allocations))
                rc = db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "weight allocation exceeds device limits");
            if (!rc) rc = db_interleave_gate_up(gc, gs, uc, us, F, D, bits, lw.gu_c, lw.gu_s, m->stream);
            cudaStreamSynchronize(m->stream);
        }
        if (!rc) rc = import_matrix(m, bytes.data() + t[6]->start, D, F, stage, &lw.dn_c, &lw.dn_s);
        if (!rc) rc = norm_from_bytes(m, bytes.data() + t[7]->start, D, &lw.in_norm);
        if (!rc) rc = norm_from_bytes(m, bytes.data() + t[8]->start, D, &lw.post_norm);
        if (!rc) rc = norm_from_bytes(m, bytes.data() + t[9]->start, m->cfg.head_dim, &lw.q_norm);
        if (!rc) rc = norm_from_bytes(m, bytes.data() + t[10]->start, m->cfg.head_dim, &lw.k_norm);
    }
    if (!rc) {
        if (!dbio::read_checked(dir, man.norm, man, verify, &bytes, &err)) rc = bad(err);
        else if (bytes.size() != (size_t)D * 2) rc = bad("final norm size does not match the configuration");
        else rc = norm_from_bytes(m, bytes.data(), D, &m->final_norm);
    }
    cudaStreamSynchronize(m->stream);
    cudaFree(stage);
    if (!rc) rc = ensure_workspace(m, m->cfg.max_sequence_tokens);
    return rc;
}

}  // namespace

extern "C" {

db_model* db_model_create(int device, const db_encoder_config* cfg, const db_encoder_weights* w, db_error* err) {
    if (!w || !w->embedding || !w->q || !w->k || !w->v || !w->o || !w->gate || !w->up || !w->down || !w->final_norm) {
        fill_error(err, "INVALID_PARAMETERS", "missing weights");
        return nullptr;
    }
    return create(device, cfg, w, false, 0, 0.f, err);
}

db_model* db_model_create_synthetic(int device, const db_encoder_config* cfg, uint64_t seed, float stdv,
                                    db_error* err) {
    return create(device, cfg, nullptr, true, seed, stdv, err);
}

int64_t db_model_synthetic_weight(const db_model* m, const char* name, int layer, uint16_t* host_out, int64_t cap) {
    if (!m || !m->synthetic || !name) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "not synthetic");
    const int D = m->D(), F = m->F(), Nq = m->Nq(), Nk = m->Nk();
    static const char* names[] = {"embedding", "q", "k", "v", "o", "gate", "up", "down"};
    int kind = -1;
    for (int i = 0; i < 8; ++i)
        if (!std::strcmp(name, names[i])) kind = i;
    if (kind < 0 || layer < 0 || layer >= m->cfg.layers)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "unknown weight");
    const int64_t sizes[8] = {(int64_t)m->cfg.vocab * D, (int64_t)Nq * D, (int64_t)Nk * D, (int64_t)Nk * D,
                              (int64_t)D * Nq,          (int64_t)F * D,  (int64_t)F * D,  (int64_t)D * F};
    const int64_t n = sizes[kind];
    if (!host_out) return n;
    if (cap < n) return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "buffer too small");
    cudaSetDevice(m->device);
    uint16_t* d = nullptr;
    if (cudaMalloc(&d, n * 2) != cudaSuccess) return db_cuda_status(1, "weight export");
    int rc = db_synthetic_bf16(m->seed, tensor_id(kind, layer), n, m->std, d, m->stream);
    if (!rc) rc = db_cuda_status(cudaMemcpyAsync(host_out, d, n * 2, cudaMemcpyDeviceToHost, m->stream), "copy");
    cudaStreamSynchronize(m->stream);
    cudaFree(d);
    return rc ? rc : n;
}

void db_model_destroy(db_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    m->drop_graphs();
    m->free_all(m->ws_allocations);
    m->free_all(m->rope_allocations);
    m->free_all(m->allocations);
    if (m->lm_x) cudaFree(m->lm_x);
    for (uint8_t* h : m->host_layers) cudaFreeHost(h);
    for (uint8_t* b : m->banks) cudaFree(b);
    for (int i = 0; i < 2; ++i) {
        if (m->uploaded[i]) cudaEventDestroy(m->uploaded[i]);
        if (m->consumed[i]) cudaEventDestroy(m->consumed[i]);
    }
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    for (__half* p : m->tmp_k) cudaFree(p);
    for (__half* p : m->tmp_v) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
    delete m;
}

int db_model_capabilities(const db_model* m, char* json, size_t cap) {
    if (!m || !json) return DB_ERR_INVALID_ARGUMENT;
    // adapters.rs:167-176 (Pplx: no caches); backend is this library
    int n = std::snprintf(json, cap,
                          "{\"model\":\"%s\",\"backend\":\"cuda\",\"caches\":[%s],\"tuning\":\"tiles\","
                          "\"weightBits\":%d,\"layers\":%d,\"hidden\":%d}",
                          m->cfg.causal ? "decoder" : "pplx-flash", m->cfg.causal ? "\"prefix\"" : "",
                          m->cfg.weight_bits, m->cfg.layers, m->cfg.hidden);
    return n < 0 || (size_t)n >= cap ? DB_ERR_INVALID_ARGUMENT : DB_OK;
}

db_cache* db_cache_create(db_model* m, size_t max_bytes, int require_prefix, db_error* err) {
    if (!m) {
        fill_error(err, "INVALID_PARAMETERS", "no model");
        return nullptr;
    }
    if (require_prefix && !m->cfg.causal) {  // mod.rs:177-182: the encoder has no prefix cache
        fill_error(err, "UNSUPPORTED_CACHE", "This model/backend does not support prefix caching");
        return nullptr;
    }
    auto* c = new db_cache();
    c->identity = m->identity;
    c->max_bytes = max_bytes;
    c->prefix_cache = m->cfg.causal != 0;
    c->device = m->device;
    return c;
}

int db_cache_clear(db_model* m, db_cache* c, db_error* err) {
    if (!m || !c || c->identity != m->identity) {
        fill_error(err, "CACHE_OWNER", "Cache belongs to another model instance");
        return -1;
    }
    c->release();  // encoders keep no state (adapters.rs:180-181); decoders drop the prefix
    return 0;
}

void db_cache_destroy(db_cache* c) { delete c; }

int db_predict(db_model* m, const int32_t* ids, size_t n, const db_parameters* params, db_cache* cache,
               const volatile uint8_t* cancel, float* out, db_error* err) {
    if (!m || !out) {
        fill_error(err, "INVALID_PARAMETERS", "null model or output");
        return -1;
    }
    if (cache && cache->identity != m->identity) {
        fill_error(err, "CACHE_OWNER", "Cache belongs to another model instance");
        return -1;
    }
    return predict_one(m, ids, n, params, cancel, out, err);  // errors clear the (stateless) cache
}

int db_predict_batch(db_model* m, const int32_t* const* ids, const size_t* lens, size_t count,
                     const db_parameters* params, db_cache* cache, const volatile uint8_t* cancel, float* outs,
                     int32_t* status, db_error* errs, db_error* err) {
    if (!m || (count && (!ids || !lens || !outs || !status))) {
        fill_error(err, "INVALID_PARAMETERS", "null batch arguments");
        return -1;
    }
    if (cache && cache->identity != m->identity) {
        fill_error(err, "CACHE_OWNER", "Cache belongs to another model instance");
        return -1;
    }
    if (m->cfg.causal || count <= 1 || m->streaming) {
        for (size_t i = 0; i < count; ++i)
            status[i] = predict_one(m, ids[i], lens[i], params, cancel, outs + i * (size_t)m->cfg.hidden,
                                    errs ? &errs[i] : nullptr);
        return 0;
    }
    return predict_packed(m, ids, lens, count, params, cancel, outs, status, errs);
}

int db_model_set_code_layout(db_model* m, int layout) {
    if (!m || (layout != DB_CODES_NATURAL && layout != DB_CODES_TC && layout != DB_CODES_DQ))
        return DB_ERR_INVALID_ARGUMENT;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    m->drop_graphs();
    for (auto& t : m->tuned) t = db_gemm_config{0, 0, 0};  // tile choices belong to one kernel
    const bool dq = layout == DB_CODES_DQ;
    if (dq && !m->dq_w[0]) {
        // the unpacked weights of the largest projection of a layer, twice
        const int D = m->D(), F = m->F();
        const size_t bytes = std::max({db_gemm_dq_scratch_bytes(m->Nqkv(), D), db_gemm_dq_scratch_bytes(D, m->Nq()),
                                       db_gemm_dq_scratch_bytes(2 * F, D), db_gemm_dq_scratch_bytes(D, F)});
        for (int i = 0; i < 2; ++i) {
            if (cudaMalloc(&m->dq_w[i], bytes) != cudaSuccess) {
                m->dq_w[i] = nullptr;
                return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "dequantised weight scratch exceeds device limits");
            }
            m->allocations.push_back(m->dq_w[i]);
        }
    }
    if (dq != m->dq) {
        // the workspace holds the split-K partial sums in dequantised mode only
        m->free_all(m->ws_allocations);
        m->cap_T = 0;
        m->dq_part = nullptr;
    }
    m->dq = dq;
    // the LM head and the int8 paths outside the layers keep int8 codes in dequantised mode
    m->i8 = layout != DB_CODES_TC;
    return DB_OK;
}

int db_model_use_graphs(db_model* m, int enable) {
    if (!m) return DB_ERR_INVALID_ARGUMENT;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    m->drop_graphs();
    m->use_graphs = enable != 0;
    return DB_OK;
}

int db_model_profile(db_model* m, int enable) {
    if (!m) return DB_ERR_INVALID_ARGUMENT;
    m->profile = enable != 0;
    return DB_OK;
}

int db_model_profile_read(db_model* m, double* ms, int64_t* counts, int n, int reset) {
    if (!m || n < DB_PROF_KINDS) return DB_ERR_INVALID_ARGUMENT;
    cudaSetDevice(m->device);
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return db_cuda_status(1, "profile sync");
    for (auto& r : m->recs) {
        float t = 0.f;
        cudaEventElapsedTime(&t, r.a, r.b);
        m->prof_ms[r.kind] += t;
        m->prof_n[r.kind] += 1;
    }
    m->recs.clear();
    m->ev_next = 0;
    for (int k = 0; k < DB_PROF_KINDS; ++k) {
        if (ms) ms[k] = m->prof_ms[k];
        if (counts) counts[k] = m->prof_n[k];
        if (reset) {
            m->prof_ms[k] = 0;
            m->prof_n[k] = 0;
        }
    }
    return DB_OK;
}

const char* db_model_profile_name(int kind) { return kind >= 0 && kind < DB_PROF_KINDS ? kProfNames[kind] : ""; }

int db_model_tune(db_model* m, int64_t tokens, const char* cache_path, char* report_json, size_t cap, db_error* err) {
    if (!m || tokens <= 0 || tokens > m->cfg.max_sequence_tokens) {
        fill_error(err, "INVALID_PARAMETERS", "tune: tokens must be in [1, max_sequence_tokens]");
        return DB_ERR_INVALID_ARGUMENT;
    }
    cudaSetDevice(m->device);
    if (m->dq) {
        // the dequantised GEMM has one configuration per shape (no candidates to select among)
        if (report_json && cap) std::snprintf(report_json, cap, "{\"dequantised\": true}");
        return DB_OK;
    }
    const int D = m->D(), F = m->F();
    // the four projections of a layer: {N, K, epilogue}
    const int64_t shapes[4][3] = {{m->Nqkv(), D, DB_EPI_STORE},
                                  {D, m->Nq(), DB_EPI_RESIDUAL},
                                  {2 * F, D, DB_EPI_SWIGLU_QUANT},
                                  {D, F, DB_EPI_RESIDUAL}};
    static const char* names[4] = {"qkv", "o", "gate_up", "down"};
    db_gemm_config chosen[4] = {};
    std::string all = "{";
    for (int p = 0; p < 4; ++p) {
        std::string rep;
        const int rc = db_tune_gemm_shape(tokens, shapes[p][0], shapes[p][1], m->cfg.weight_bits, (int)shapes[p][2],
                                          cache_path, &chosen[p], &rep, m->stream, m->i8);
        if (rc) {
            fill_error(err, db_last_error_code(), db_last_error_message());
            return rc;
        }
        all += std::string(p ? "," : "") + "\"" + names[p] + "\":" + rep;
    }
    all += "}";
    for (int p = 0; p < 4; ++p) m->tuned[p] = chosen[p];
    m->drop_graphs();  // captured graphs hold the previous tile choices
    if (report_json && cap) std::snprintf(report_json, cap, "%s", all.c_str());
    return DB_OK;
}

int db_forward_device(db_model* m, const int32_t* ids_dev, int64_t n, float* out_dev, void* stream) {
    if (!m || !ids_dev || n <= 0 || !out_dev)
        return db_fail(DB_ERR_INVALID_ARGUMENT, "INVALID_ARGUMENT", "forward: bad arguments");
    cudaSetDevice(m->device);
    if (ensure_workspace(m, (int)n)) return DB_ERR_CUDA;
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    cudaEvent_t ev;
    cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    cudaEventRecord(ev, caller);
    cudaStreamWaitEvent(m->stream, ev, 0);
    cudaMemcpyAsync(m->ids, ids_dev, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, m->stream);
    int rc = run_forward(m, (int)n, nullptr);
    cudaMemcpyAsync(out_dev, m->pooled, m->cfg.hidden * sizeof(float), cudaMemcpyDeviceToDevice, m->stream);
    cudaEventRecord(ev, m->stream);
    cudaStreamWaitEvent(caller, ev, 0);
    cudaEventDestroy(ev);
    return rc;
}

int db_model_export_packed(db_model* m, const char* directory, db_error* err) {
    if (!m || !directory) {
        fill_error(err, "INVALID_PARAMETERS", "null model or directory");
        return DB_ERR_INVALID_ARGUMENT;
    }
    if (m->streaming) {
        fill_error(err, "INVALID_PARAMETERS", "export needs resident weights (streaming is on)");
        return DB_ERR_INVALID_ARGUMENT;
    }
    cudaSetDevice(m->device);
    const int D = m->D(), L = m->cfg.layers, F = m->F(), Nq = m->Nq(), Nk = m->Nk(), bits = m->cfg.weight_bits;
    const size_t gb = group_bytes(bits);
    const std::string dir = directory, prefix = bits == 4 ? "q4-e4" : "q8-e8";
    const size_t big = std::max({(size_t)m->cfg.vocab * D, (size_t)m->Nqkv() * D, (size_t)2 * F * D, (size_t)D * Nq}) / 64 * gb;
    uint8_t* stage = nullptr;
    if (cudaMalloc(&stage, big + 256) != cudaSuccess) {
        fill_error(err, "RESOURCE_LIMIT", "export staging exceeds device limits");
        return DB_ERR_CUDA;
    }
    std::string e, files = "{", layers = "[";
    int rc = 0;
    uint64_t decoder_bytes = 0;
    auto put = [&](const std::string& name, const std::vector<uint8_t>& b) {
        if (!dbio::write_file(dir + "/" + name, b.data(), b.size(), &e)) return false;
        files += std::string(files.size() > 1 ? "," : "") + dbio::json_quote(name) + ":{\"bytes\":" +
                 std::to_string(b.size()) + ",\"sha256\":" + dbio::json_quote(dbio::sha256_hex(b.data(), b.size())) + "}";
        return true;
    };
    for (int l = 0; l < L && !rc; ++l) {
        const LayerW& lw = m->layers[l];
        std::vector<uint8_t> qkv, o, gu, dn;
        rc = export_matrix(m, lw.qkv_c, lw.qkv_s, m->Nqkv(), D, stage, &qkv);
        if (!rc) rc = export_matrix(m, lw.o_c, lw.o_s, D, Nq, stage, &o);
        if (!rc) rc = export_matrix(m, lw.gu_c, lw.gu_s, 2 * F, D, stage, &gu);
        if (!rc) rc = export_matrix(m, lw.dn_c, lw.dn_s, D, F, stage, &dn);
        if (rc) break;
        const size_t row_q = (size_t)(D / 64) * gb, row_o = (size_t)(Nq / 64) * gb, row_d = (size_t)(F / 64) * gb;
        // gate and up rows come interleaved in blocks of 64 in the device layout
        std::vector<uint8_t> gate, up;
        for (int b = 0; b < 2 * F / 64; ++b)
            (b % 2 ? up : gate).insert((b % 2 ? up : gate).end(), gu.begin() + (size_t)b * 64 * row_q,
                                       gu.begin() + (size_t)(b + 1) * 64 * row_q);
        std::vector<std::vector<uint8_t>> parts = {
            std::vector<uint8_t>(qkv.begin(), qkv.begin() + (size_t)Nq * row_q),
            std::vector<uint8_t>(qkv.begin() + (size_t)Nq * row_q, qkv.begin() + (size_t)(Nq + Nk) * row_q),
            std::vector<uint8_t>(qkv.begin() + (size_t)(Nq + Nk) * row_q, qkv.end()),
            o, gate, up, dn, norm_bytes(lw.in_norm, D), norm_bytes(lw.post_norm, D),
            norm_bytes(lw.q_norm, m->cfg.head_dim), norm_bytes(lw.k_norm, m->cfg.head_dim)};
        (void)row_o;
        (void)row_d;
        const std::vector<std::vector<int64_t>> shapes = {{Nq, D}, {Nk, D}, {Nk, D}, {D, Nq}, {F, D}, {F, D}, {D, F},
                                                          {D}, {D}, {m->cfg.head_dim}, {m->cfg.head_dim}};
        std::vector<uint8_t> file;
        std::string tensors = "[";
        for (int i = 0; i < 11; ++i) {
            std::string shape = "[";
            for (size_t d = 0; d < shapes[i].size(); ++d) shape += (d ? "," : "") + std::to_string(shapes[i][d]);
            tensors += std::string(i ? "," : "") + "{\"name\":" +
                       dbio::json_quote("language_model.layers." + std::to_string(l) + "." + kLayerTensors[i]) +
                       ",\"shape\":" + shape + "],\"start\":" + std::to_string(file.size()) +
                       ",\"end\":" + std::to_string(file.size() + parts[i].size()) + "}";
            file.insert(file.end(), parts[i].begin(), parts[i].end());
        }
        char name[64];
        std::snprintf(name, sizeof name, "%s-layer-%02d.bin", prefix.c_str(), l);
        if (!put(name, file)) { rc = DB_ERR_INVALID_ARGUMENT; break; }
        layers += std::string(l ? "," : "") + "{\"file\":" + dbio::json_quote(name) + ",\"bytes\":" +
                  std::to_string(file.size()) + ",\"tensors\":" + tensors + "]}";
        decoder_bytes += file.size();
    }
    std::vector<uint8_t> emb;
    if (!rc) rc = export_matrix(m, m->emb_c, m->emb_s, m->cfg.vocab, D, stage, &emb);
    if (!rc && !put(prefix + "-embedding.bin", emb)) rc = DB_ERR_INVALID_ARGUMENT;
    if (!rc && !put(prefix + "-norm.bin", norm_bytes(m->final_norm, D))) rc = DB_ERR_INVALID_ARGUMENT;
    cudaFree(stage);
    if (!rc) {
        const std::string manifest =
            "{\"schema_version\":1,\"revision\":\"decisive-b200\",\"scheme\":\"q" + std::to_string(bits) + "-w" +
            std::to_string(bits) + "a8-e" + std::to_string(bits) + "-r" + std::to_string(bits) +
            "-g64\",\"group_size\":64,\"group_bytes\":" + std::to_string(gb) + ",\"embedding_row_bytes\":" +
            std::to_string((size_t)(D / 64) * gb) + ",\"layers\":" + layers + "],\"headers\":[],\"embedding\":" +
            dbio::json_quote(prefix + "-embedding.bin") + ",\"readout\":null,\"norm\":" +
            dbio::json_quote(prefix + "-norm.bin") + ",\"decoder_bytes\":" + std::to_string(decoder_bytes) +
            ",\"files\":" + files + "}}";
        if (!dbio::write_file(dir + "/packed-" + prefix + ".json", manifest.data(), manifest.size(), &e))
            rc = DB_ERR_INVALID_ARGUMENT;
    }
    if (rc) {
        fill_error(err, rc == DB_ERR_INVALID_ARGUMENT ? "IO_ERROR" : db_last_error_code(),
                   rc == DB_ERR_INVALID_ARGUMENT ? e : std::string(db_last_error_message()));
        return rc;
    }
    return DB_OK;
}

db_model* db_model_create_packed(int device, const db_encoder_config* cfg, const char* manifest_path, int verify,
                                 db_error* err) {
    if (!manifest_path) {
        fill_error(err, "INVALID_PARAMETERS", "null manifest path");
        return nullptr;
    }
    if (check_config(cfg, err)) return nullptr;
    dbio::Manifest man;
    std::string e;
    if (!dbio::read_manifest(manifest_path, &man, &e)) {
        fill_error(err, "INVALID_WEIGHTS", e);
        return nullptr;
    }
    if (device < 0 || device >= db_device_count() || cudaSetDevice(device) != cudaSuccess) {
        fill_error(err, "GPU_UNAVAILABLE", "no CUDA device " + std::to_string(device));
        return nullptr;
    }
    std::string path = manifest_path, dir = ".";
    const size_t slash = path.find_last_of('/');
    if (slash != std::string::npos) dir = path.substr(0, slash);
    auto* m = new db_model();
    m->device = device;
    m->cfg = *cfg;
    m->dev_err = db_device_error_ptr();
    cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (build_packed(m, man, dir, verify != 0)) {
        fill_error(err, db_last_error_code(), db_last_error_message());
        db_model_destroy(m);
        return nullptr;
    }
    return m;
}

int db_model_set_streaming(db_model* m, int enable, db_error* err) {
    if (!m) {
        fill_error(err, "INVALID_PARAMETERS", "null model");
        return DB_ERR_INVALID_ARGUMENT;
    }
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    if ((enable != 0) == m->streaming) return DB_OK;
    m->drop_graphs();  // the weight buffers move
    const int L = m->cfg.layers, D = m->D(), F = m->F(), Nq = m->Nq(), bits = m->cfg.weight_bits;
    const size_t G = (size_t)D / 64;
    // the eight projection buffers of a layer, in bank order
    const size_t sizes[8] = {(size_t)m->Nqkv() * D * bits / 8, G * db_scale_stride(m->Nqkv()) * 4,
                             (size_t)D * Nq * bits / 8,           (size_t)(Nq / 64) * db_scale_stride(D) * 4,
                             (size_t)2 * F * D * bits / 8,        G * db_scale_stride(2 * F) * 4,
                             (size_t)D * F * bits / 8,            (size_t)(F / 64) * db_scale_stride(D) * 4};
    auto fail = [&](const char* what) {
        fill_error(err, "RESOURCE_LIMIT", what);
        return DB_ERR_CUDA;
    };
    if (enable) {
        m->spans.clear();
        size_t off = 0;
        for (size_t b : sizes) {
            m->spans.push_back({off, b});
            off += (b + 1023) / 1024 * 1024;
        }
        m->layer_bytes = off;
        if (cudaMalloc(&m->banks[0], off) != cudaSuccess || cudaMalloc(&m->banks[1], off) != cudaSuccess)
            return fail("streaming banks exceed device limits");
        if (!m->copy_stream && cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking) != cudaSuccess)
            return fail("copy stream");
        for (int i = 0; i < 2; ++i) {
            if (!m->uploaded[i]) cudaEventCreateWithFlags(&m->uploaded[i], cudaEventDisableTiming);
            if (!m->consumed[i]) cudaEventCreateWithFlags(&m->consumed[i], cudaEventDisableTiming);
            cudaEventRecord(m->consumed[i], m->stream);  // the banks start free
        }
        m->host_layers.assign(L, nullptr);
        for (int l = 0; l < L; ++l) {
            if (cudaMallocHost(&m->host_layers[l], off) != cudaSuccess) return fail("pinned host memory");
            LayerW& w = m->layers[l];
            const void* src[8] = {w.qkv_c, w.qkv_s, w.o_c, w.o_s, w.gu_c, w.gu_s, w.dn_c, w.dn_s};
            for (int i = 0; i < 8; ++i)
                cudaMemcpy(m->host_layers[l] + m->spans[i].off, src[i], sizes[i], cudaMemcpyDeviceToHost);
        }
        // release the resident copies: only the two banks stay on the device
        for (int l = 0; l < L; ++l) {
            LayerW& w = m->layers[l];
            void* ptrs[8] = {w.qkv_c, w.qkv_s, w.o_c, w.o_s, w.gu_c, w.gu_s, w.dn_c, w.dn_s};
            for (void* p : ptrs) {
                auto it = std::find(m->allocations.begin(), m->allocations.end(), p);
                if (it != m->allocations.end()) {
                    cudaFree(p);
                    m->allocations.erase(it);
                }
            }
            w.qkv_c = w.o_c = w.gu_c = w.dn_c = nullptr;
            w.qkv_s = w.o_s = w.gu_s = w.dn_s = nullptr;
        }
        m->streaming = true;
        return DB_OK;
    }
    // back to resident weights
    for (int l = 0; l < L; ++l) {
        LayerW& w = m->layers[l];
        uint8_t* dst[8];
        for (int i = 0; i < 8; ++i) {
            if (m->alloc(&dst[i], sizes[i], m->allocations)) return fail("weight allocation exceeds device limits");
            cudaMemcpy(dst[i], m->host_layers[l] + m->spans[i].off, sizes[i], cudaMemcpyHostToDevice);
        }
        w.qkv_c = dst[0]; w.qkv_s = reinterpret_cast<float*>(dst[1]);
        w.o_c = dst[2];   w.o_s = reinterpret_cast<float*>(dst[3]);
        w.gu_c = dst[4];  w.gu_s = reinterpret_cast<float*>(dst[5]);
        w.dn_c = dst[6];  w.dn_s = reinterpret_cast<float*>(dst[7]);
    }
    cudaStreamSynchronize(m->copy_stream);
    for (uint8_t* h : m->host_layers) cudaFreeHost(h);
    m->host_layers.clear();
    for (uint8_t*& b : m->banks) {
        cudaFree(b);
        b = nullptr;
    }
    m->streaming = false;
    return DB_OK;
}

}  // extern "C"

namespace {
// (re)allocates per-layer key/value buffers for cap rows of Hk heads
int ensure_kv(std::vector<__half*>& k, std::vector<__half*>& v, int& cap, int rows, int layers, int Hk) {
    if (rows <= cap && (int)k.size() == layers) return 0;
    for (__half* p : k) cudaFree(p);
    for (__half* p : v) cudaFree(p);
    k.assign(layers, nullptr);
    v.assign(layers, nullptr);
    cap = 0;
    for (int l = 0; l < layers; ++l)
        if (cudaMalloc(&k[l], (size_t)rows * Hk * 128 * 2) != cudaSuccess ||
            cudaMalloc(&v[l], (size_t)rows * Hk * 128 * 2) != cudaSuccess)
            return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "prefix state exceeds device limits");
    cap = rows;
    return 0;
}
}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Log-probabilities of continuation tokens from LM-head logits.  Logits rows (global index gr =
// r0 + blockIdx.x): row 0 is the prefix's last state and predicts token 0 of every continuation;
// row 1 + b*T + j is continuation b's token j and predicts its token j + 1 (the last token of a
// continuation predicts nothing).  out[b*T + t] = logits[row, ids[b*T + t]] - logsumexp(row), the
// log-sum-exp kept as a running (max, scaled sum) per thread and merged across the CTA.
__global__ void __launch_bounds__(512) lm_logprob_kernel(const float* __restrict__ logits, int V, int r0,
                                                         const int32_t* __restrict__ ids, int B, int T,
                                                         float* __restrict__ out) {
    const int gr = r0 + blockIdx.x;
    if (gr > 0 && (gr - 1) % T == T - 1) return;
    const float* x = logits + (size_t)blockIdx.x * V;
    float mx = -INFINITY, sum = 0.f;
    auto add = [&](float v) {
        if (v > mx) {
            sum = sum * expf(mx - v) + 1.f;
            mx = v;
        } else {
            sum += expf(v - mx);
        }
    };
    if ((V & 3) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int i = threadIdx.x; i < V / 4; i += blockDim.x) {
            const float4 v = x4[i];
            add(v.x);
            add(v.y);
            add(v.z);
            add(v.w);
        }
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) add(x[i]);
    }
    auto merge = [](float& m1, float& s1, float m2, float s2) {
        const float m = fmaxf(m1, m2);
        if (m == -INFINITY) return;
        s1 = (m1 == -INFINITY ? 0.f : s1 * expf(m1 - m)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - m));
        m1 = m;
    };
#pragma unroll
    for (int o = 16; o; o >>= 1) merge(mx, sum, __shfl_xor_sync(0xffffffffu, mx, o), __shfl_xor_sync(0xffffffffu, sum, o));
    __shared__ float sm[16], ss[16];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) {
        sm[wid] = mx;
        ss[wid] = sum;
    }
    __syncthreads();
    if (wid == 0) {
        const int nw = blockDim.x >> 5;
        mx = lane < nw ? sm[lane] : -INFINITY;
        sum = lane < nw ? ss[lane] : 0.f;
#pragma unroll
        for (int o = 16; o; o >>= 1)
            merge(mx, sum, __shfl_xor_sync(0xffffffffu, mx, o), __shfl_xor_sync(0xffffffffu, sum, o));
        const float lse = mx + logf(sum);
        if (gr == 0) {
            for (int b = lane; b < B; b += 32) out[(size_t)b * T] = x[ids[(size_t)b * T]] - lse;
        } else if (lane == 0) {
            const int b = (gr - 1) / T, j = (gr - 1) % T;
            out[(size_t)b * T + j + 1] = x[ids[(size_t)b * T + j + 1]] - lse;
        }
    }
}

constexpr int kLmRows = 256;  // logits rows per LM-head chunk

int finish_call(db_model* m, db_error* err) {
    int flag = 0;
    cudaMemcpyAsync(&flag, m->flag, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    const cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
        fill_error(err, "INFERENCE_FAILED", cudaGetErrorString(e));
        return -1;
    }
    int word = 0;
    cudaMemcpy(&word, m->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (word) {
        cudaMemset(m->dev_err, 0, sizeof(int));
        fill_error(err, "INFERENCE_FAILED", "device wait expired (error word " + std::to_string(word) + ")");
        return -1;
    }
    if (flag) {
        fill_error(err, "INFERENCE_FAILED", "non-finite hidden state");
        return -1;
    }
    return 0;
}

// The shared part of predict and score: checks the request (the reference's codes), runs or reuses
// the prefix (kev/mod.rs:186-236: its per-layer keys and values go into the cache when its byte
// budget holds them) and then all continuations in one batched pass after it.  On success m->normed
// holds the count*tokens final-normed continuation states and *last the prefix's last one.
int run_continuations(db_model* m, db_cache* cache, const int32_t* prefix, size_t prefix_len,
                      const int32_t* continuations, size_t count, size_t tokens, int extra_rows,
                      const volatile uint8_t* cancel, const float** last, db_error* err) {
    if (!m->cfg.causal) {
        fill_error(err, "UNSUPPORTED_CACHE", "continuations need a causal (decoder) model");
        return -1;
    }
    if (cache && cache->identity != m->identity) {
        fill_error(err, "CACHE_OWNER", "Cache belongs to another model instance");
        return -1;
    }
    if (cancel && *cancel) {
        fill_error(err, "CANCELLED", "Inference was cancelled");
        return -1;
    }
    if (prefix_len == 0 || count == 0 || tokens == 0) {
        fill_error(err, "INVALID_REQUEST", "a nonempty prefix and nonempty continuations are required");
        return -1;
    }
    if (prefix_len + tokens > (size_t)m->cfg.max_sequence_tokens || count > 65535) {
        fill_error(err, "INPUT_TOO_LONG", "prefix + continuation exceeds token limit: " +
                                              std::to_string(prefix_len + tokens) + " > " +
                                              std::to_string(m->cfg.max_sequence_tokens) + "; inputs are never truncated");
        return -1;
    }
    for (size_t i = 0; i < prefix_len + count * tokens; ++i) {
        const int32_t id = i < prefix_len ? prefix[i] : continuations[i - prefix_len];
        if (id < 0 || id >= m->cfg.vocab) {
            fill_error(err, "INVALID_REQUEST", "token id " + std::to_string(id) + " outside the vocabulary");
            return -1;
        }
    }
    cudaSetDevice(m->device);
    const int P = (int)prefix_len, T = (int)tokens, B = (int)count, L = m->cfg.layers, Hk = m->cfg.kv_heads;
    const int D = m->cfg.hidden;
    if (ensure_workspace(m, std::max(P, B * T + extra_rows)) || ensure_rope(m, P + T) ||
        (!m->prefix_last && m->alloc(&m->prefix_last, D, m->allocations) &&
         db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "prefix state exceeds device limits"))) {
        fill_error(err, "RESOURCE_LIMIT", db_last_error_message());
        return -1;
    }
    auto failed = [&](int rc) {
        cudaStreamSynchronize(m->stream);
        if (rc == 1) fill_error(err, "CANCELLED", "Inference was cancelled");
        else fill_error(err, "INFERENCE_FAILED", db_last_error_message());
        return -1;
    };
    const bool reuse = cache && cache->prefix_cache && (int)cache->ids.size() == P &&
                       std::equal(prefix, prefix + P, cache->ids.begin()) && (int)cache->k.size() == L &&
                       cache->last;
    std::vector<__half*>* pk = &m->tmp_k;
    std::vector<__half*>* pv = &m->tmp_v;
    if (reuse) {
        pk = &cache->k;
        pv = &cache->v;
        *last = cache->last;
        cache->hits += 1;
        cache->reused += P;
    } else {
        const size_t state_bytes = (size_t)L * P * Hk * 128 * 2 * 2 + (size_t)D * 4;
        const bool keep = cache && cache->prefix_cache && state_bytes <= cache->max_bytes;
        int rc = 0;
        float* keep_last = m->prefix_last;
        if (keep) {
            cache->ids.clear();
            rc = ensure_kv(cache->k, cache->v, cache->cap_P, P, L, Hk);
            if (!rc && !cache->last && cudaMalloc(&cache->last, (size_t)D * 4) != cudaSuccess) {
                cache->last = nullptr;
                rc = db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "prefix state exceeds device limits");
            }
            pk = &cache->k;
            pv = &cache->v;
            keep_last = cache->last;
        } else {
            rc = ensure_kv(m->tmp_k, m->tmp_v, m->tmp_cap, P, L, Hk);
        }
        if (rc) {
            fill_error(err, "RESOURCE_LIMIT", db_last_error_message());
            return -1;
        }
        cudaMemcpyAsync(m->ids, prefix, (size_t)P * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream);
        Pass pass;
        pass.sk = pk->data();
        pass.sv = pv->data();
        pass.pool = false;
        rc = enqueue_forward(m, P, cancel, &pass);
        if (rc) return failed(rc);
        cudaMemcpyAsync(keep_last, m->normed + (size_t)(P - 1) * D, (size_t)D * 4, cudaMemcpyDeviceToDevice, m->stream);
        *last = keep_last;
        if (cache && cache->prefix_cache) cache->computed += P;
        if (keep) cache->ids.assign(prefix, prefix + P);
    }
    cudaMemcpyAsync(m->ids, continuations, (size_t)B * T * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream);
    Pass pass;
    pass.items = B;
    pass.prefix = P;
    pass.pk = pk->data();
    pass.pv = pv->data();
    pass.pool = false;
    const int rc = enqueue_forward(m, T, cancel, &pass);
    if (rc) return failed(rc);
    return 0;
}

// The LM head over the rows [last; the B*T continuation states] (the tied embedding matrix, the
// model's own quantised weights) and the log-probability of every continuation token
// (logprobs [B*T], device), in chunks of kLmRows logits rows.  Rows are quantised like every
// projection's input (g64, 8-bit codes).
int enqueue_lm_logprobs(db_model* m, const float* last, int B, int T, float* logprobs) {
    const auto& c = m->cfg;
    const int D = c.hidden, V = c.vocab, R = 1 + B * T;
    cudaStream_t st = m->stream;
    if (R > m->lm_x_rows) {
        m->lm_x_rows = 0;
        if (m->lm_x) cudaFree(m->lm_x);
        m->lm_x = nullptr;
        if (cudaMalloc(&m->lm_x, (size_t)R * D * 4) != cudaSuccess) {
            m->lm_x = nullptr;
            return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "LM-head rows exceed device limits");
        }
        m->lm_x_rows = R;
    }
    if (!m->logits && m->alloc(&m->logits, (size_t)kLmRows * V, m->allocations))
        return db_fail(DB_ERR_CUDA, "RESOURCE_LIMIT", "LM-head logits exceed device limits");
    cudaMemcpyAsync(m->lm_x, last, (size_t)D * 4, cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(m->lm_x + D, m->normed, (size_t)B * T * D * 4, cudaMemcpyDeviceToDevice, st);
    const int64_t ld_codes = m->Kmax(), lds = db_scale_stride(m->cap_T);
    const int layout = m->i8 ? DB_CODES_NATURAL_I8 : DB_CODES_TC_F16;
    int rc = db_launch_quantize_rows(m->lm_x, DB_F32, D, R, D, 8, m->acodes, layout, ld_codes, m->sa, nullptr, lds,
                                     m->flag, st);
    const uint8_t* a8 = reinterpret_cast<const uint8_t*>(m->acodes);
    const size_t code_bytes = m->i8 ? 1 : 2;
    for (int r0 = 0; r0 < R && !rc; r0 += kLmRows) {
        const int rows = std::min(kLmRows, R - r0);
        DbGemmArgs g{};
        g.a_codes = a8 + (size_t)r0 * ld_codes * code_bytes;
        g.lda = ld_codes;
        g.sa = m->sa + r0;
        g.ldsa = lds;
        g.w_codes = m->emb_c;
        g.sw = m->emb_s;
        g.M = rows;
        g.N = V;
        g.K = D;
        g.bits = c.weight_bits;
        g.fused = c.fused;
        g.epilogue = DB_EPI_STORE;
        g.y = m->logits;
        g.ldy = V;
        g.nonfinite = m->flag;
        g.dev_error = m->dev_err;
        if (m->i8) {
            const db_gemm_config d = db_gemm_i8_default_config(rows, V, DB_EPI_STORE);
            g.block_n = d.block_n;
            g.pair_ctas = d.pair_ctas;
            rc = db_launch_gemm_i8(g, st);
        } else {
            rc = db_launch_gemm_tc(g, st);
        }
        if (rc) break;
        lm_logprob_kernel<<<rows, 512, 0, st>>>(m->logits, V, r0, m->ids, B, T, logprobs);
        rc = (int)cudaGetLastError();
    }
    return rc ? db_cuda_status(rc, "LM head") : 0;
}

}  // namespace

extern "C" {

int db_predict_continuations(db_model* m, db_cache* cache, const int32_t* prefix, size_t prefix_len,
                             const int32_t* continuations, size_t count, size_t tokens,
                             const volatile uint8_t* cancel, float* hidden, db_error* err) {
    if (!m || !hidden || !prefix || !continuations) {
        fill_error(err, "INVALID_PARAMETERS", "null model, ids or output");
        return -1;
    }
    const float* last = nullptr;
    if (run_continuations(m, cache, prefix, prefix_len, continuations, count, tokens, 0, cancel, &last, err))
        return -1;
    cudaMemcpyAsync(hidden, m->normed, count * tokens * m->cfg.hidden * sizeof(float), cudaMemcpyDeviceToHost,
                    m->stream);
    return finish_call(m, err);
}

int db_score_continuations(db_model* m, db_cache* cache, const int32_t* prefix, size_t prefix_len,
                           const int32_t* continuations, size_t count, size_t tokens,
                           const volatile uint8_t* cancel, float* logprobs, float* hidden, db_error* err) {
    if (!m || !logprobs || !prefix || !continuations) {
        fill_error(err, "INVALID_PARAMETERS", "null model, ids or output");
        return -1;
    }
    const float* last = nullptr;
    if (run_continuations(m, cache, prefix, prefix_len, continuations, count, tokens, 1, cancel, &last, err))
        return -1;
    const int D = m->cfg.hidden, BT = (int)(count * tokens);
    // the log-probabilities land in the spare pooled buffer (cap_T * D floats >= B*T)
    int rc = enqueue_lm_logprobs(m, last, (int)count, (int)tokens, m->pooled);
    if (rc) {
        cudaStreamSynchronize(m->stream);
        fill_error(err, "INFERENCE_FAILED", db_last_error_message());
        return -1;
    }
    cudaMemcpyAsync(logprobs, m->pooled, (size_t)BT * 4, cudaMemcpyDeviceToHost, m->stream);
    if (hidden) cudaMemcpyAsync(hidden, m->lm_x, (size_t)(1 + BT) * D * 4, cudaMemcpyDeviceToHost, m->stream);
    return finish_call(m, err);
}

int db_cache_stats(const db_cache* c, int64_t* hits, int64_t* reused_tokens, int64_t* computed_tokens) {
    if (!c) return DB_ERR_INVALID_ARGUMENT;
    if (hits) *hits = c->hits;
    if (reused_tokens) *reused_tokens = c->reused;
    if (computed_tokens) *computed_tokens = c->computed;
    return DB_OK;
}

}  // extern "C"
