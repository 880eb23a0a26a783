/*
 * CPU oracle for the decisive-b200 quantised-GEMM path.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load
 * this library; the product (libdecisive_b200.so) never links or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference Rust crate (decisive,
 * src/models/pplx_flash/...).  Every function cites the reference file:line it follows.
 * Parity of this restatement is pinned against the reference's own unit tests
 * (int8.rs:590-962, packed.rs:124-208, quantized_rows.rs:117-208, quantization.rs:304-370,
 * cpu.rs:632-677), re-expressed in tests/test_oracle_*.py; the reference itself (Rust)
 * cannot be compiled in this image.
 */
#ifndef DECISIVE_ORACLE_H
#define DECISIVE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_GROUP 64

/* ---- bf16 (half 2.7.1 bf16::from_f32 / to_f32) ---- */
uint16_t oracle_f32_to_bf16(float x);
float oracle_bf16_to_f32(uint16_t b);
void oracle_f32_to_bf16_array(const float *x, size_t n, uint16_t *out);

/* ---- group quantiser primitives (int8.rs:305-360) ---- */
float oracle_group_scale(const float *x, size_t n, int bits);
void oracle_pack_codes(const float *x, size_t n, float scale, int bits, int8_t *out);

/* ---- packed row-group format (packed.rs:10-119) ---- */
/* returns bytes, or 0 on an invalid shape (packed.rs:10-19) */
size_t oracle_packed_size(size_t rows, size_t columns, int bits);
/* returns 0 on success, -1 invalid shape, -2 non-finite weight */
int oracle_packed_pack(const uint16_t *bf16, size_t rows, size_t columns, int bits, uint8_t *out);
/* returns 0, or -1 when the bytes or a scale are invalid */
int oracle_packed_unpack(const uint8_t *packed, size_t bytes, int bits, float *out);
/* readout GEMV; returns 0, -1 invalid shape, -2 non-finite activation */
int oracle_packed_project(const uint8_t *packed, size_t bytes, int bits, size_t columns,
                          const float *x, size_t outputs, float *y);

/* ---- int8::Matrix panel layout (int8.rs:51-152) ---- */
size_t oracle_matrix_data_bytes(size_t input, size_t output, int weight_bits);
size_t oracle_matrix_scale_count(size_t input, size_t output);
/* fit: 0 absmax, 1 mse (quantization.rs:25-71), 2 affine (quantization.rs:147-200).
 * simd: 1 follows the AVX2 lane order of the fitters' statistics (quantization.rs:84-121,
 * 203-244); absmax is identical for both.  offsets may be NULL unless fit == 2.
 * returns 0, -1 invalid, -2 non-finite weight */
int oracle_matrix_from_bf16(const uint16_t *bf16, size_t input, size_t output, int weight_bits,
                            int fit, int simd, int8_t *data, float *scales, float *offsets);
/* activation quantiser (int8.rs:178-202): values [tokens, groups*64], scales/sums [tokens, groups] */
void oracle_matrix_prepare(const float *x, size_t tokens, size_t input, int activation_bits,
                           int8_t *values, float *scales, int32_t *sums);
/* mode 0: AVX2 rows<R,Q4> numerics, sum = fma(dot, sw*sa, sum) (int8.rs:526-585)
 * mode 1: portable apply_prepared, sum += dot*(sa*sw) (int8.rs:259-287)
 * mode 2: mode 0 computed with the AVX2 instruction mix (maddubs/madd/fmadd), 32-column
 *         parallel tiles and the unpack-once Q4 panel for tokens >= 16 (int8.rs:229-258,
 *         448-480); bit-identical to mode 0, used as the timed CPU baseline.
 * offsets may be NULL (no affine term). */
void oracle_matrix_apply_prepared(const int8_t *data, const float *scales, const float *offsets,
                                  size_t input, size_t output, int weight_bits,
                                  const int8_t *values, const float *act_scales,
                                  const int32_t *sums, size_t tokens, int mode, float *y);
/* full apply with the non-finite guard (int8.rs:166-176); threads <= 0 means all cores */
void oracle_matrix_apply(const int8_t *data, const float *scales, const float *offsets,
                         size_t input, size_t output, int weight_bits, int activation_bits,
                         const float *x, size_t tokens, int mode, float *y);

/* ---- fitted Q4 scales (quantization.rs) ---- */
float oracle_fit_mse(const float *x, size_t n, int simd, int8_t *codes);
void oracle_fit_affine(const float *x, size_t n, int simd, int8_t *codes, float *scale, float *offset);
float oracle_fit_nf4(const float *x, size_t n, int8_t *codes);
extern const float ORACLE_NF4[16];

/* ---- embedding rows (quantized_rows.rs:21-110) ---- */
/* fit: 0 absmax, 1 mse, 2 affine, 3 nf4.  data: rows*columns*bits/8, scales/offsets: rows*columns/64 */
int oracle_embedding_from_bf16(const uint16_t *bf16, size_t rows, size_t columns, int bits,
                               int fit, int simd, uint8_t *data, float *scales, float *offsets);
void oracle_embedding_append(const uint8_t *data, const float *scales, const float *offsets,
                             size_t columns, int bits, int nf4, size_t id, float *out);

/* ---- layer math (cpu.rs:293-371, 513-529; backbone.rs:471-615) ---- */
void oracle_rms(const float *x, float *y, size_t rows, size_t width, const float *weight,
                float eps, int zero_centered);
void oracle_silu_mul(float *gate, const float *up, size_t n);
void oracle_softmax(float *x, size_t n);
void oracle_rope(float *x, size_t tokens, size_t heads, size_t head_dim, size_t rotary,
                 size_t offset, float theta);
/* non-causal GQA attention: q [T, Hq*D], k/v [T, Hkv*D] -> out [T, Hq*D] */
void oracle_attention(const float *q, const float *k, const float *v, size_t tokens,
                      size_t q_heads, size_t kv_heads, size_t head_dim, float scale, float *out);
/* the same with causal = 1: token i attends keys 0..i (a decoder's prefill; the continuation
 * of a cached prefix is the tail of a causal pass over prefix + continuation) */
void oracle_attention_masked(const float *q, const float *k, const float *v, size_t tokens, size_t q_heads,
                             size_t kv_heads, size_t head_dim, float scale, int causal, float *out);

/* ---- composed Qwen3-shaped Q4 encoder (composition of the above) ---- */
typedef struct {
    int layers, hidden, q_heads, kv_heads, head_dim, ffn, vocab;
    int weight_bits, activation_bits;
    float rope_theta, eps;
    int causal; /* 1: decoder (causal attention) */
} oracle_encoder_config;

/* Weights as bf16 [out,in] per projection (reference "[output,input]" order).  Per layer:
 * q, k, v, o, gate, up, down.  Norm weights are f32.  Embedding bf16 [vocab, hidden].
 * Quantised internally with the absmax quantiser; returns 0 or <0 on error. */
typedef struct {
    const uint16_t *embedding;
    const uint16_t **q, **k, **v, **o, **gate, **up, **down;
    const float **input_norm, **post_norm, **q_norm, **k_norm;
    const float *final_norm;
} oracle_encoder_weights;

void *oracle_encoder_create(const oracle_encoder_config *cfg, const oracle_encoder_weights *w);
void oracle_encoder_destroy(void *enc);
/* ids [tokens] -> pooled [hidden]; layers_limit < 0 runs all layers.  hidden_out optional
 * [tokens, hidden] final-norm output.  mode as in oracle_matrix_apply_prepared. */
int oracle_encoder_forward(void *enc, const int32_t *ids, size_t tokens, int layers_limit,
                           int mode, float *pooled, float *hidden_out);

/* ---- Decima int8 (src/models/decima/int8.rs): blocks of 16/32/64/128, scale = max|x|/127
 * (min f32::MIN_POSITIVE), code = round-half-away(x / scale) clamped to +-127 (true division).
 * Codes are row-major [rows, groups*block] with zeros past cols; scales [rows, groups]. */
float oracle_decima_scale(const float *x, size_t n);
int8_t oracle_decima_quantize(float x, float scale);
/* Matrix::new quantiser for weights and the per-row activation packer (int8.rs:106-151, 239-253). */
void oracle_decima_quantize_rows(const float *x, size_t rows, size_t cols, size_t block, int8_t *codes,
                                 float *scales);
/* Matrix::apply_with_rows in WeightsActivations mode: quantise x, then per output
 * mode 0 (AVX2, int8.rs:459-498): sums = fma(float(dot_g), sw*sa, sums) over ascending g;
 * mode 1 (portable, int8.rs:380-420): sum += float(dot_g) * (sw*sa);
 * then y = sum + (bias ? bias[n] : 0).  A non-finite x gives all-NaN y (int8.rs:186-190). */
void oracle_decima_apply_w8a8(const int8_t *w_codes, const float *w_scales, size_t rows, size_t cols,
                              size_t block, const float *x, size_t m, const float *bias, int mode, float *y);
void oracle_decima_apply_w8a32(const int8_t *w_codes, const float *w_scales, size_t rows, size_t cols,
                               size_t block, const float *x, size_t m, const float *bias, int mode, float *y);

/* Decima encoder pieces (decima/cpu.rs): LayerNorm with sequential f32 sums (:529-539) and the
 * erf GELU (:542-556); the composed C4 forward lives in oracle.py (bert_forward). */
void oracle_layer_norm(float *x, size_t rows, size_t d, const float *w, const float *b, float eps);
void oracle_gelu(float *x, size_t n);

int oracle_num_threads(void);
void oracle_set_threads(int n);
int oracle_has_avx2(void);

#ifdef __cplusplus
}
#endif
#endif
