// Launchers of the layer kernels (internal to libdecisive_b200.so).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

int db_launch_rms_quantize(const float* x, int64_t ldx, const float* w, int T, int D, float eps, int zero_centered,
                           float* normed, int64_t ldn, void* codes, int layout, int64_t ldc, float* scales,
                           int32_t* sums, int64_t lds, int* nonfinite, cudaStream_t stream, int normalize = 1,
                           const float* add0 = nullptr, const float* add1 = nullptr);
// Rows are items of seq_len tokens (0 = T) one after another; row t gets RoPE position
// pos0 + t % seq_len (a continuation after a cached prefix of pos0 tokens), or positions[t] when
// positions (device, T ints) is given (ragged sequences packed together).
int db_launch_qk_norm_rope(const float* qkv, int64_t ld, int T, int Hq, int Hk, const float* qw, const float* kw,
                           float eps, const float* cos_t, const float* sin_t, __half* q16, __half* k16, __half* v16,
                           cudaStream_t stream, int pos0 = 0, int seq_len = 0, const int* positions = nullptr);
int db_launch_mean_pool(const float* x, int64_t ldx, int T, int D, float* out, cudaStream_t stream);
// Mean of each ragged sequence's rows: out [nseq, D], sequence i = rows cu_seqlens[i]..cu_seqlens[i+1]-1.
int db_launch_mean_pool_varlen(const float* x, int64_t ldx, const int* cu_seqlens, int nseq, int D, float* out,
                               cudaStream_t stream);
int db_launch_fill_nan_if(float* y, int64_t n, const int* flag, cudaStream_t stream);

// Non-causal GQA attention over head_dim 128: q16 [T, Hq, 128], k16/v16 [T, Hk, 128] (f16),
// out f32 [T, Hq*128] with row stride ldo.  scale multiplies q.k before the softmax.
int db_launch_attention(const __half* q16, const __half* k16, const __half* v16, int T, int Hq, int Hk, float scale,
                        float* out, int64_t ldo, cudaStream_t stream);
// Same attention, writing the context already quantised for the output projection: f16 codes in
// tensor-core order [T, ldc], or with codes_i8 = 1 int8 codes in natural order [T, ldc] (ldc % 16 == 0),
// or with codes_i8 = 2 dequantised f16 values f16(code * scale) in natural order (DB_CODES_DQ_F16)
// (head h occupies features 128h..128h+127), per-64 scales [2*Hq, lds]; *nonfinite is raised
// when a context value is not finite.
int db_launch_attention_quant(const __half* q16, const __half* k16, const __half* v16, int T, int Hq, int Hk,
                              float scale, void* codes, int64_t ldc, float* scales, int64_t lds, int* nonfinite,
                              cudaStream_t stream, int codes_i8 = 0);
// The tensor-core (tcgen05) attention behind the two calls above: B items of T rows each
// (q16/k16/v16 and the outputs hold the items one after another, 16-byte aligned), non-causal;
// the context goes to out (f32) when codes is null, else quantised as above.
int db_launch_attention_tc(const __half* q16, const __half* k16, const __half* v16, int B, int T, int Hq, int Hk,
                           float scale, float* out, int64_t ldo, void* codes, int64_t ldc, float* scales,
                           int64_t lds, int* nonfinite, cudaStream_t stream, int codes_i8 = 0);
// Ragged sequences packed one after another (R rows; sequence i = rows cu_seqlens[i] ..
// cu_seqlens[i+1]-1, a device array; max_len >= every length): non-causal attention of each
// sequence over its own rows, outputs as db_launch_attention_tc.
int db_launch_attention_varlen(const __half* q16, const __half* k16, const __half* v16, const int* cu_seqlens,
                               int nseq, int max_len, int R, int Hq, int Hk, float scale, float* out, int64_t ldo,
                               void* codes, int64_t ldc, float* scales, int64_t lds, int* nonfinite,
                               cudaStream_t stream, int codes_i8 = 0);
// Decoder form of the attention (tcgen05, one item's query tile per CTA): B items of T
// rows each (q16/k16/v16 and the outputs hold the items one after another); every item's keys are
// the P cached prefix keys kp/vp [P, Hk, 128] (shared by the items; P = 0: none) followed by its
// own T keys, which are causal (row i sees own keys 0..i) when causal != 0.  Outputs as
// db_launch_attention_tc; db_launch_attention_prefix_quant is its quantising form.
int db_launch_attention_decoder(const __half* q16, const __half* k16, const __half* v16, int B, int T,
                                const __half* kp, const __half* vp, int P, int causal, int Hq, int Hk, float scale,
                                float* out, int64_t ldo, void* codes, int64_t ldc, float* scales, int64_t lds,
                                int* nonfinite, cudaStream_t stream, int codes_i8 = 0);
int db_launch_attention_prefix_quant(const __half* q16, const __half* k16, const __half* v16, int B, int T,
                                     const __half* kp, const __half* vp, int P, int causal, int Hq, int Hk,
                                     float scale, void* codes, int64_t ldc, float* scales, int64_t lds,
                                     int* nonfinite, cudaStream_t stream, int codes_i8 = 0);
