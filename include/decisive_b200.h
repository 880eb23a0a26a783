/*
 * decisive_b200 -- C ABI of the B200 (sm_100a) backend for decisive's quantised projection path.
 *
 * Two layers of entry points:
 *   1. kernel level: device pointers + sizes + an optional cudaStream_t (passed as void*; NULL =
 *      the calling thread's current-device default stream).  Each replaces one reference
 *      function of src/models/pplx_flash/ (cited per entry).  Return 0 or a negative DB_ERR_*;
 *      db_last_error_code()/db_last_error_message() describe the failure (thread-local).
 *   2. model level: an opaque model handle mirroring `inference::Model<B: Backend>`
 *      (src/inference/mod.rs:140-273) for the Pplx-shaped encoder, with per-request
 *      {code, message} errors using the reference's error codes.
 *
 * Numerics: group-64 symmetric quantisation with f32 scales; activation codes in [-127, 127]
 * (int8.rs:178-202); weight codes Q4 in [-7, 7] (or [-8, 7] when fitted) or Q8 in [-127, 127];
 * per output sum = fma(float(dot_g), sw*sa, sum) over ascending groups (int8.rs:562-565) or the
 * portable sum += dot*(sa*sw) (int8.rs:276-278) -- both bit-exact against the reference's CPU
 * arithmetic.
 *
 * Device weight layout (see DB_LAYOUT comment below) differs from the reference's packed row
 * format (packed.rs) only in where the scales live; db_import_packed/db_export_packed convert
 * losslessly.
 */
#ifndef DECISIVE_B200_H
#define DECISIVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DB_ABI_VERSION 1

/* ---- status codes ---- */
#define DB_OK 0
#define DB_ERR_INVALID_ARGUMENT (-1) /* bad shape / pointer / alignment */
#define DB_ERR_CUDA (-2)             /* a CUDA runtime call failed */
#define DB_ERR_DEVICE_TIMEOUT (-3)   /* a kernel's bounded wait expired (device error word set) */
#define DB_ERR_NONFINITE (-4)        /* non-finite input where the reference rejects it */
#define DB_ERR_UNSUPPORTED (-5)

/* ---- element types and code layouts ---- */
#define DB_DTYPE_F32 0
#define DB_DTYPE_F16 1
#define DB_DTYPE_BF16 2
/* activation code layouts (int8 values in [-127,127]):
 *   DB_CODES_NATURAL  int8 [M, Kp], k in order (reference Scratch::values, int8.rs:7-11)
 *   DB_CODES_GEMV     int8 [M, Kp], inside each 8 consecutive k stored as k0,k2,k4,k6,k1,k3,k5,k7
 *   DB_CODES_TC       f16  [M, Kp] integer-valued, inside each 8 stored as k0,k4,k1,k5,k2,k6,k3,k7
 *   DB_CODES_DQ       f16  [M, Kp] dequantised values f16(code * group scale), k in order: the
 *                     operand of the dequantised-operand GEMM (no grouped fold; see db_gemm_g64)
 * Kp = ceil(K/64)*64; activation scales f32 [G, lds], sums int32 [G, lds], G = Kp/64.
 * DB_LAYOUT: weight codes Q4 [N, Kp/2] bytes (low nibble = even k, nibble = code+8, i.e. the
 * code bytes of packed.rs:22-28), Q8 [N, Kp] int8; weight scales f32 [G, Ns] with
 * Ns = db_scale_row_stride(N) = roundup(N, 128), entries n >= N zero.  Activation scales passed
 * to the tensor-core path need lds >= db_scale_row_stride(M) (and lds % 4 == 0). */
#define DB_CODES_NATURAL 0
#define DB_CODES_GEMV 1
#define DB_CODES_TC 2
#define DB_CODES_DQ 3

int db_abi_version(void);
/* row stride (elements) of a scale array with n columns: roundup(n, 128) */
int64_t db_scale_row_stride(int64_t n);
const char *db_last_error_code(void);
const char *db_last_error_message(void);
int db_device_count(void);
/* reads and clears the calling device's kernel error word (bounded-wait expiries) */
int db_device_error_word(void);

/* ---- kernel level ---- */

/* Activation quantiser.  Replaces int8::Matrix::prepare (int8.rs:178-202) and the grouped
 * WGSL quantiser `int8_input` (webgpu/grouped_q4.rs:3-25).  x [M, K] (row stride ldx elements)
 * of dtype -> codes (layout, row stride ldc elements), scales [G, lds], sums [G, lds] (optional).
 * bits 8 (limit 127) or 4 (limit 7).  *nonfinite (optional, device int) is OR-ed with 1 when any
 * input is NaN/Inf. */
int db_quantize_activations_g64(const void *x, int dtype, int64_t ldx, int64_t M, int64_t K, int bits,
                                void *codes, int layout, int64_t ldc, float *scales, int32_t *sums, int64_t lds,
                                int *nonfinite, void *stream);

/* Weight quantiser, absmax.  Replaces int8::Matrix::from_bf16_optimized's absmax branch
 * (int8.rs:51-152) and packed::pack (packed.rs:31-56): bf16 [N, K] ([output, input], the
 * reference's weight order) -> codes/scales in DB_LAYOUT.  Returns DB_ERR_NONFINITE for a
 * non-finite weight ("non-finite INT8 weight", int8.rs:99-102). */
int db_pack_weights_g64(const uint16_t *bf16, int64_t N, int64_t K, int bits, uint8_t *codes, float *scales,
                        void *stream);

/* Reference packed rows (packed.rs:10-56: per (row, group) 32|64 code bytes then the f32
 * scale; K % 64 == 0) <-> DB_LAYOUT, lossless. */
int db_import_packed(const uint8_t *packed, int64_t N, int64_t K, int bits, uint8_t *codes, float *scales,
                     void *stream);
int db_export_packed(const uint8_t *codes, const float *scales, int64_t N, int64_t K, int bits, uint8_t *packed,
                     void *stream);

/* Row dequantisation: out[t, k] = code(row ids[t], k) * scale.  Replaces packed::unpack
 * (packed.rs:59-73) and Embedding::append (quantized_rows.rs:89-110); ids may be NULL
 * (rows 0..T-1).  An id outside [0, N) yields DB_ERR_INVALID_ARGUMENT. */
int db_dequant_rows_g64(const uint8_t *codes, const float *scales, int64_t N, int64_t K, int bits,
                        const int32_t *ids, int64_t T, float *out, int64_t ldo, void *stream);

/* Grouped GEMM on prepared activations.  Replaces Matrix::apply_prepared (int8.rs:229-288)
 * and the WGSL int8_gemm family (grouped_q4_tuned.wgsl): y[m, n] (+)= sum over groups.
 * a_codes in DB_CODES_NATURAL layout (int8, lda % 16 == 0; the kind::i8 tensor-core kernel) or
 * DB_CODES_TC layout (f16 codes; the kind::f16 kernel), M >= 1, or DB_CODES_GEMV when
 * M <= db_gemv_max_rows();
 * a_sums is required by the GEMV layout with Q4 weights.  fused: 1 = AVX2 numerics (fma),
 * 0 = portable numerics.  residual: 1 adds into y.  nonfinite (optional): when *nonfinite != 0
 * every output is NaN (int8.rs:170-173).
 * DB_CODES_DQ (dequantised mode, the numerics of the reference's WGSL GEMMs, which dequantise the
 * weights and accumulate in f32): a_codes f16 [M, lda] from the quantiser's DB_CODES_DQ layout
 * (lda % 8 == 0; sa, ldsa and fused unused); the weights are unpacked to f16(code * scale) into
 * a library scratch buffer (N x Kp f16, kept per device and stream and grown when a call needs
 * more; growing is refused while the stream is being captured) and y = the tcgen05 kind::f16 sum
 * over all K in f32.  Not bit-exact against the grouped fold: within ~1.5e-3 of the output RMS
 * (the contract is 2e-3); every tile configuration gives the same bits. */
int db_gemm_g64(const void *a_codes, int layout, int64_t lda, const float *sa, const int32_t *a_sums, int64_t ldsa,
                const uint8_t *w_codes, const float *sw, int64_t M, int64_t N, int64_t K, int bits, int fused,
                int residual, float *y, int64_t ldy, const int *nonfinite, void *stream);

/* Tile configuration of the tensor-core GEMM: the candidate space of the kernel-selection tuner
 * (checkpoint.rs:279-294, 428-563 select among kernel variants; a candidate is accepted only when
 * its output is bitwise equal to the baseline's).  Every configuration computes the same
 * per-group fold in the same order (DB_CODES_DQ: the same MMAs over the same K steps), so all are
 * bitwise equal by construction.
 *   block_n    output columns per tile: 0 (default: 128 for DB_CODES_TC, 256 for DB_CODES_NATURAL,
 *              for DB_CODES_DQ the widest tile giving >= 96 tiles), 64, 128 or 256, or 32 on
 *              DB_CODES_NATURAL (single CTAs; store and residual epilogues: small M) (the SwiGLU
 *              epilogue takes 128 or 256)
 *   max_ctas   persistent grid cap: 0 = one CTA per SM
 *   pair_ctas  1 = clusters of two CTAs issue M = 256 MMAs (M > 128; DB_CODES_TC: 128-wide tiles
 *              only); 0 = off
 * A NULL configuration on DB_CODES_NATURAL inputs picks the widest tile that still fills the SMs.
 * No counterpart in the reference's CPU path (its tuner picks WGSL variants). */
typedef struct db_gemm_config {
    int block_n;
    int max_ctas;
    int pair_ctas;
} db_gemm_config;
/* db_gemm_g64 with an explicit tile configuration (NULL = defaults).  GEMV-layout inputs ignore it. */
int db_gemm_g64_config(const void *a_codes, int layout, int64_t lda, const float *sa, const int32_t *a_sums,
                       int64_t ldsa, const uint8_t *w_codes, const float *sw, int64_t M, int64_t N, int64_t K,
                       int bits, int fused, int residual, float *y, int64_t ldy, const int *nonfinite,
                       const db_gemm_config *config, void *stream);
int db_gemv_max_rows(void);

/* Kernel-selection tuner for one tensor-core GEMM shape, with the reference's rule
 * (webgpu/checkpoint.rs:420-565, the int8_gemm candidate selection): each candidate tile
 * configuration runs on synthetic inputs; the fastest candidate whose output is bitwise equal to
 * the default configuration's and that is at least 1 % faster (best of 10 timed launches) is
 * chosen, else the default.  cache_path (NULL = no cache): a text file of tuned choices keyed by
 * a hash of the device name, SM count, compute capability, driver version, library build and
 * shape (the reference keys by adapter, user agent, weight bits and kernel sources,
 * checkpoint.rs:279-294); a cached choice is only checked for equality again.  epilogue:
 * 0 store, 1 residual add, 2 SwiGLU re-quantisation (N = 2F, N % 128 == 0).  report_json
 * (optional): the candidates, their equality and best times, and the choice. */
int db_gemm_tune(int64_t M, int64_t N, int64_t K, int bits, int epilogue, const char *cache_path,
                 db_gemm_config *choice, char *report_json, size_t cap);

/* Full projection: quantise x (f32 [M, K]) then GEMM, choosing the GEMV path for
 * M <= db_gemv_max_rows() and the tensor-core path otherwise.  Replaces Matrix::apply
 * (int8.rs:166-176) including its non-finite guard.  workspace: device bytes from
 * db_linear_workspace_bytes(M, K). */
size_t db_linear_workspace_bytes(int64_t M, int64_t K);
int db_linear_g64(const float *x, int64_t M, int64_t K, const uint8_t *w_codes, const float *sw, int64_t N,
                  int weight_bits, int activation_bits, int fused, float *y, void *workspace, void *stream);

/* Allocation-free variant of db_linear_g64 -- this entry point has no counterpart in the
 * reference.  For hosts that pass device pointers but do not let the library allocate device
 * memory (a fixed device-memory budget owned by the host, or a latency-critical caller that must
 * never reach cudaMalloc and its implicit synchronisation) and that cannot size a workspace up
 * front.  Its scratch is one array of DB_NOALLOC_SCRATCH_BYTES compiled into the library, held
 * by every GPU that loads it until the process exits.  A call needs up256(M*Kp*2) +
 * 2*up256(G*roundup(M,128)*4) + 256 bytes of it (up256 rounds up to 256; e.g. M = 1024 fits up
 * to K = 3840, M = 4096 up to K = 960); larger shapes are rejected with code SCRATCH_LIMIT.
 * The first call on a device looks up the array's device address, so make it before any stream
 * capture.  All calls on a device share the array (the entry point clears what
 * must start at zero); calls that overlap on the GPU race on it and must be serialised by the
 * caller.  No cudaMalloc, cudaFree or allocating library routine is called. */
#define DB_NOALLOC_SCRATCH_BYTES (8u << 20)
size_t db_linear_noalloc_scratch_bytes(void);
int db_linear_g64_noalloc(const float *x, int64_t M, int64_t K, const uint8_t *w_codes, const float *sw, int64_t N,
                          int weight_bits, int activation_bits, int fused, float *y, void *stream);
/* The allocation-free entry point's own device error word (its GEMM's bounded-wait expiries; the
 * word behind db_device_error_word() is allocated, so this path cannot use it): reads and clears
 * it for the calling device, synchronously.  0 = no expiry since the last read; -1 = CUDA error.
 * Like db_device_error_word(), read it after synchronising the stream of the calls it covers. */
int db_linear_noalloc_error_word(void);

/* Readout GEMV on one activation row.  Replaces packed::project (packed.rs:75-119; portable
 * numerics, activation 8-bit).  Returns DB_ERR_NONFINITE for a non-finite x. */
int db_project_packed(const float *x, int64_t K, const uint8_t *w_codes, const float *sw, int64_t outputs,
                      int bits, float *y, void *workspace, void *stream);

/* ---- Decima int8 (C4 scheme, src/models/decima/int8.rs): weights and activations quantised in
 * blocks of 16/32/64/128 values, scale = max(max|x| / 127, FLT_MIN), code = round-half-away-from-
 * zero(x / scale) with a correctly rounded division, clamped to +-127 (int8.rs:413-418).
 *
 * Weights: Matrix::new (int8.rs:106-151) from f32 [N, K] (row-major, [output, input]) into the Q8
 * device layout codes [N, Kp] and group-major scales [ceil(K/block), db_scale_row_stride(N)];
 * DB_ERR_NONFINITE for a non-finite weight (the reference rejects them). */
int db_decima_quantize_weights(const float *w, int64_t N, int64_t K, int block, uint8_t *codes, float *scales,
                               void *stream);
/* The activation fill of Matrix::apply_with_rows (int8.rs:239-253, pack_x86.rs:4-56): f32 [M, K]
 * -> codes (DB_CODES_TC f16 or DB_CODES_NATURAL int8, [M, ldc], ldc >= Kp) and scales
 * [ceil(K/block), lds]; *nonfinite is set for a non-finite x. */
int db_decima_quantize_activations(const float *x, int64_t M, int64_t K, int block, void *codes, int layout,
                                   int64_t ldc, float *scales, int64_t lds, int *nonfinite, void *stream);
/* Matrix::apply_with_rows in WeightsActivations mode (W8A8): quantise x, grouped GEMM in blocks of
 * 32 or 64 (16 and 128 give DB_ERR_UNSUPPORTED), y [M, N] = sum + bias[n] (bias NULL: + 0).
 * fused = 1 follows the AVX2 order sums = fma(float(dot), sw*sa, sums) (int8.rs:459-498), 0 the
 * portable sum += float(dot) * (sw*sa) (int8.rs:380-420).  A non-finite x gives all-NaN y.
 * workspace: device bytes from db_decima_workspace_bytes(M, K, block). */
size_t db_decima_workspace_bytes(int64_t M, int64_t K, int block);
/* Matrix::apply_with_rows in Weights mode (W8A32: the same int8 weight codes and scales, f32
 * activations), blocks of 32, 64 or 128 (16 gives DB_ERR_UNSUPPORTED).  fused = 1 follows the AVX2
 * kernel (decima/int8/weights_x86.rs:51-113): weights decoded to the f32 product code * scale, one
 * fma chain over k per output; 0 the portable kernel (int8.rs:384-407): per block dot += x * code,
 * sum += dot * scale.  y [M, N] = sum + bias[n] (bias NULL: + 0); a non-finite x gives all-NaN y.
 * nonfinite: one device int the call uses as its flag (no allocation). */
int db_decima_linear_w8a32(const float *x, int64_t M, int64_t K, const uint8_t *w_codes, const float *sw, int64_t N,
                           int block, int fused, const float *bias, float *y, int *nonfinite, void *stream);
int db_decima_linear(const float *x, int64_t M, int64_t K, const uint8_t *w_codes, const float *sw, int64_t N,
                     int block, int fused, const float *bias, float *y, void *workspace, void *stream);

/* Fused gate/up projection + SiLU(gate)*up + group-64 re-quantisation, the semantics of the
 * reference's fused q4_mlp (grouped_q4_mlp.wgsl:1-105) == apply_pair + silu_mul + prepare
 * (backbone.rs:229-236, cpu.rs:348-371, int8.rs:178-202).  w_gu: 2*F rows in blocks of
 * 64 gate rows followed by the 64 matching up rows (db_interleave_gate_up builds it).
 * Output: codes DB_CODES_TC [M, ldoc] and scales [F/64, ldos] (ldos >= db_scale_row_stride(M)
 * so they can feed the down projection directly).  F % 64 == 0. */
int db_mlp_g64(const void *a_codes, int64_t lda, const float *sa, int64_t ldsa, const uint8_t *w_gu_codes,
               const float *w_gu_scales, int64_t M, int64_t F, int64_t K, int bits, int fused, void *out_codes,
               int64_t ldoc, float *out_scales, int64_t ldos, const int *nonfinite, void *stream);
/* db_mlp_g64 on int8 activation codes in DB_CODES_NATURAL layout (the kind::i8 tensor-core path,
 * half the operand bytes of DB_CODES_TC): a_codes int8 [M, lda] (lda % 16 == 0), out_codes int8
 * natural [M, ldoc] (ldoc % 16 == 0), out_scales as db_mlp_g64.  Same numerics. */
int db_mlp_g64_natural(const void *a_codes, int64_t lda, const float *sa, int64_t ldsa, const uint8_t *w_gu_codes,
                       const float *w_gu_scales, int64_t M, int64_t F, int64_t K, int bits, int fused,
                       void *out_codes, int64_t ldoc, float *out_scales, int64_t ldos, const int *nonfinite,
                       void *stream);
/* gate/up [F, K] each (DB_LAYOUT) -> interleaved [2F, K] (DB_LAYOUT) for db_mlp_g64 */
int db_interleave_gate_up(const uint8_t *gate_codes, const float *gate_scales, const uint8_t *up_codes,
                          const float *up_scales, int64_t F, int64_t K, int bits, uint8_t *out_codes,
                          float *out_scales, void *stream);

/* Non-causal GQA attention (backbone.rs:485-615 without the output gate): q f16 [T, Hq, 128],
 * k/v f16 [T, Hk, 128], out f32 [T, Hq*128] (row stride ldo); scale multiplies q.k. */
int db_attention(const void *q16, const void *k16, const void *v16, int64_t T, int64_t q_heads, int64_t kv_heads,
                 int64_t head_dim, float scale, float *out, int64_t ldo, void *stream);
/* The decoder form (kev/mod.rs:163-300 continuation from a cached prefix): B items of T rows one
 * after another (q f16 [B*T, Hq, 128], k/v f16 [B*T, Hk, 128]); each item attends to the P cached
 * prefix keys kp/vp f16 [P, Hk, 128] (shared; P = 0: none, kp/vp may be NULL) and then to its own
 * keys, causally (row i of an item sees its own keys 0..i) when causal != 0.  out f32
 * [B*T, Hq*128] (row stride ldo). */
int db_attention_decoder(const void *q16, const void *k16, const void *v16, int64_t B, int64_t T, const void *kp,
                         const void *vp, int64_t P, int causal, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                         float scale, float *out, int64_t ldo, void *stream);

/* Deterministic synthetic bf16 tensor on the device: value_i = std * N(0,1) from a
 * counter-based generator keyed by (seed, tensor). */
int db_synthetic_bf16(uint64_t seed, uint64_t tensor, int64_t n, float std, uint16_t *out, void *stream);

/* ---- model level: mirror of inference::Model / Backend (src/inference/mod.rs) ---- */

typedef struct db_model db_model;
typedef struct db_cache db_cache;

/* {code, message} of inference::Error (mod.rs:44-85). */
typedef struct {
    char code[32];
    char message[224];
} db_error;

/* Qwen3-shaped bidirectional encoder, Q4/Q8 group-64 projections. */
typedef struct {
    int32_t layers, hidden, q_heads, kv_heads, head_dim, ffn, vocab;
    int32_t weight_bits;         /* 4 or 8 */
    float rope_theta, eps;
    int32_t max_sequence_tokens; /* PplxParameters default (parameters.rs:81-92) */
    int32_t fused;               /* 1 = AVX2 numerics (default), 0 = portable */
    int32_t causal;              /* 1 = decoder (causal attention; prefix caches, C5), 0 = encoder */
} db_encoder_config;

/* PplxParameters (parameters.rs:81-103): max_sequence_tokens must be positive. */
typedef struct {
    int32_t max_sequence_tokens;
} db_parameters;

/* Host weights: bf16 [out, in] per projection per layer (q, k, v, o, gate, up, down),
 * f32 norms, bf16 embedding [vocab, hidden]. */
typedef struct {
    const uint16_t *embedding;
    const uint16_t *const *q, *const *k, *const *v, *const *o, *const *gate, *const *up, *const *down;
    const float *const *input_norm, *const *post_norm, *const *q_norm, *const *k_norm;
    const float *final_norm;
} db_encoder_weights;

db_model *db_model_create(int device, const db_encoder_config *cfg, const db_encoder_weights *w, db_error *err);
/* random-init weights (N(0, std) via db_synthetic_bf16, norms = 1) generated on the device */
db_model *db_model_create_synthetic(int device, const db_encoder_config *cfg, uint64_t seed, float std,
                                    db_error *err);
/* copies the bf16 weight `name` ("embedding", "q", ..., "down") of `layer` of a synthetic model
 * into host memory (for the CPU oracle); returns elements copied or a negative status */
int64_t db_model_synthetic_weight(const db_model *m, const char *name, int layer, uint16_t *host_out, int64_t cap);
void db_model_destroy(db_model *m);
/* Capabilities (mod.rs:118-125) as JSON: {"model":..., "backend":"cuda", "caches":[...], "tuning":...} */
int db_model_capabilities(const db_model *m, char *json, size_t cap);

/* Model::create_cache (mod.rs:176-189): require_prefix on a model without prefix caching ->
 * NULL with code UNSUPPORTED_CACHE.  max_bytes excludes weights and scratch. */
db_cache *db_cache_create(db_model *m, size_t max_bytes, int require_prefix, db_error *err);
/* Model::clear_cache (mod.rs:190-194): a cache of another model -> CACHE_OWNER */
int db_cache_clear(db_model *m, db_cache *c, db_error *err);
void db_cache_destroy(db_cache *c);

/* Model::predict (mod.rs:206-249): ids [n] -> pooled f32 [hidden].  params NULL = the model's
 * defaults; cache NULL = an ephemeral cache; *cancel != 0 -> CANCELLED (checked before and
 * after the forward, and between layers).  cancel is one byte so that the reference's
 * Cancellation(Arc<AtomicBool>) (mod.rs:87-100) can be passed as-is.  Returns 0, or -1 with
 * *err filled. */
int db_predict(db_model *m, const int32_t *ids, size_t n, const db_parameters *params, db_cache *cache,
               const volatile uint8_t *cancel, float *out, db_error *err);

/* Model::predict_batch (mod.rs:250-273): ordered per-request outcomes; status[i] = 0 success
 * (outs + i*hidden filled) or -1 (errs[i] filled).  A foreign cache fails the whole call. */
int db_predict_batch(db_model *m, const int32_t *const *ids, const size_t *lens, size_t count,
                     const db_parameters *params, db_cache *cache, const volatile uint8_t *cancel, float *outs,
                     int32_t *status, db_error *errs, db_error *err);

/* ---- C4: the Decima-shaped (BERT) encoder on the Decima int8 kernels (decima/mod.rs:492-556):
 * x = LN(word[id] + type[0] + pos[p]); per layer x = LN(x + Wo attn(qkv) + bo),
 * x = LN(x + W2 gelu(W1 x + b1) + b2); every projection W8A8 in blocks of `block` (32 or 64) with
 * the Decima quantiser, or W8A32 with mode = 1; heads of hidden/heads <= 128 dims, non-causal attention scaled by
 * 1/sqrt(head dim); erf GELU; LayerNorm eps `eps`.  Synthetic weights (db_synthetic_bf16 keys:
 * word 0, pos 1, type 2; layer l: 16 + 16 l + {q 0, k 1, v 2, o 3, ff1 4, ff2 5, bq 6, bk 7, bv 8,
 * bo 9, b1 10, b2 11}; LayerNorm weights 1, biases 0).  db_bert_predict writes the mean-pooled
 * state [hidden] and, when hidden != NULL, the final states [n, hidden]. */
typedef struct {
    int32_t layers, hidden, heads, ffn, vocab, max_positions, block;
    float eps;
    int32_t fused; /* 1 = AVX2 accumulation order (default), 0 = portable */
    int32_t mode;  /* 0 = W8A8 (WeightsActivations, the int8 tensor-core GEMM), 1 = W8A32 (Weights:
                      f32 activations, db_decima_linear_w8a32's kernel) */
} db_bert_config;
typedef struct db_bert db_bert;
db_bert *db_bert_create_synthetic(int device, const db_bert_config *cfg, uint64_t seed, float std, db_error *err);
void db_bert_destroy(db_bert *m);
int db_bert_predict(db_bert *m, const int32_t *ids, size_t n, float *pooled, float *hidden, db_error *err);
/* The cross-encoder request (one state paired with `count` choices, 1..16): sequence i is
 * state ++ choices[i] with positions restarting at 0, every sequence of 1..max_positions tokens;
 * the sequences run packed in one pass (per-sequence attention, segmented mean pool) and each
 * yields DB_BERT_HEAD_OUTPUTS f32 logits from the scorer head, an f32 linear over the pooled state
 * with sequential sums in index order (decima/mod.rs:482, 701: the `score` linear, Precision::F32,
 * portable kernel; synthetic weights: key 3 [outputs, hidden], bias key 4).  logits
 * [count, DB_BERT_HEAD_OUTPUTS]; pooled [count, hidden] when non-null. */
#define DB_BERT_HEAD_OUTPUTS 3
int db_bert_score(db_bert *m, const int32_t *state, size_t n_state, const int32_t *const *choices,
                  const size_t *choice_lens, size_t count, float *logits, float *pooled, db_error *err);

/* Prefix-state cache and continuation batching for causal models (C5; the reference's Kev prefix
 * reuse, kev/mod.rs:163-240, and per-question continuation from a clone of the prefix state,
 * :245-300).  A cache made with require_prefix = 1 (causal models only; encoders answer
 * UNSUPPORTED_CACHE) keeps the per-layer keys and values of the last prefix whose state fits in
 * max_bytes.  db_predict_continuations runs `count` continuations of `tokens` tokens each after
 * the prefix, batched in one pass (every continuation sees the prefix and, causally, its own
 * tokens; the prefix is computed once, or reused when the cache holds the same ids), and writes
 * the final-normed hidden states [count, tokens, hidden].  prefix_len + tokens must not exceed
 * max_sequence_tokens (INPUT_TOO_LONG).  cache may be NULL (nothing is kept); a kept prefix also
 * keeps its last final-normed state. */
int db_predict_continuations(db_model *m, db_cache *cache, const int32_t *prefix, size_t prefix_len,
                             const int32_t *continuations, size_t count, size_t tokens,
                             const volatile uint8_t *cancel, float *hidden, db_error *err);
/* Scores the continuations by log-probability: the same pass as db_predict_continuations, then an
 * LM head tied to the embedding matrix (logits = the model's quantised embedding rows times the
 * final-normed state, quantised to 8-bit g64 codes like every projection input) and a log-softmax
 * over the vocabulary.  logprobs [count, tokens]: log p(token t of continuation b | prefix and
 * tokens 0..t-1 of b); token 0 is predicted from the prefix's last state.  hidden, when non-null,
 * receives the LM head's input rows [1 + count*tokens, hidden] (the prefix's last state, then the
 * continuations' states).  Errors as db_predict_continuations. */
int db_score_continuations(db_model *m, db_cache *cache, const int32_t *prefix, size_t prefix_len,
                           const int32_t *continuations, size_t count, size_t tokens,
                           const volatile uint8_t *cancel, float *logprobs, float *hidden, db_error *err);
/* hits / prefix tokens reused / prefix tokens computed (kev/mod.rs Stats) */
int db_cache_stats(const db_cache *c, int64_t *hits, int64_t *reused_tokens, int64_t *computed_tokens);

/* Per-launch CUDA-event timing of the forward's kernels (the reference's projection_ms
 * accounting, cpu.rs:8-16).  Kinds 0..DB_PROF_KINDS-1, named by db_model_profile_name.
 * db_model_profile_read synchronises the model's stream and returns accumulated ms and
 * launch counts per kind. */
/* The plain forward of a token count runs as one captured CUDA graph from its second call on
 * (1 = on, the default); a cancellation flag, per-kernel profiling or streaming keeps the
 * layer-by-layer path.  0 switches graphs off (results are bit-identical either way). */
int db_model_use_graphs(db_model *m, int enable);

/* Activation codes of the model's projections: DB_CODES_NATURAL (int8 codes, the kind::i8
 * tensor-core GEMM; the default) or DB_CODES_TC (f16 codes, the kind::f16 GEMM).  Both compute
 * the same per-group integer dots and fold them in the same order, so outputs are bit-identical;
 * only speed differs.  DB_CODES_DQ switches the layers' projections to the dequantised numerics
 * (f16(code * scale) operands, f32 accumulation over the whole K: the reference's WGSL GEMM
 * numerics, within the contract's tolerance of the grouped fold, not bit-identical), and the
 * model keeps an unpacked-weight scratch of its largest projection.  Resets tuned tile choices (they
 * belong to one kernel); db_model_tune has nothing to select in dequantised mode. */
int db_model_set_code_layout(db_model *m, int layout);

#define DB_PROF_KINDS 11
int db_model_profile(db_model *m, int enable);
int db_model_profile_read(db_model *m, double *ms, int64_t *counts, int n, int reset);
const char *db_model_profile_name(int kind);

/* Tunes the model's four projection GEMMs (qkv, o, gate/up + SwiGLU, down) at `tokens` rows with
 * db_gemm_tune's rule and uses the choices in every later forward.  Every configuration is
 * bitwise equal, so only speed changes.  report_json: one object per projection. */
int db_model_tune(db_model *m, int64_t tokens, const char *cache_path, char *report_json, size_t cap,
                  db_error *err);

/* Packed checkpoints in the reference's export format (export_packed.rs:13-103): a directory
 * holding packed-q4-e4.json (or packed-q8-e8.json) -- schema_version 1, scheme, group_size 64,
 * layers[{file, bytes, tensors[{name, shape, start, end}]}], embedding, norm, files{name: {bytes,
 * sha256}} -- and one file per layer (Qwen3 tensor names, 2-D tensors in the packed row-group
 * format of packed.rs:10-56, 1-D tensors raw bf16), the embedding and the final norm.  The encoder
 * has no readout ("readout": null).  db_model_export_packed writes one from a model's weights;
 * db_model_create_packed loads one (verify = 1 checks every file's SHA-256), failing with
 * INVALID_WEIGHTS on a missing tensor, a shape or size that does not match cfg, or a digest
 * mismatch. */
int db_model_export_packed(db_model *m, const char *directory, db_error *err);
db_model *db_model_create_packed(int device, const db_encoder_config *cfg, const char *manifest_path, int verify,
                                 db_error *err);

/* Layer streaming (the reference's two-bank scheme, webgpu/streaming.rs): with enable = 1 every
 * layer's projection weights move to pinned host memory and only two device banks remain; each
 * forward copies layer l + 2 into the bank of layer l on a copy stream as soon as layer l's last
 * kernel has run, so uploads overlap compute and at most two layers are on the device.  Results
 * are bit-identical to resident weights.  enable = 0 makes the weights resident again.  Export
 * needs resident weights. */
int db_model_set_streaming(db_model *m, int enable, db_error *err);

/* Device-resident variant for throughput measurement: ids already on the device, output left on
 * the device; no host synchronisation.  Used by bench.py's device-timed leg. */
int db_forward_device(db_model *m, const int32_t *ids_dev, int64_t n, float *out_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
