// Host-side launchers of the device kernels (internal to libdecisive_b200.so).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Scale vectors are stored with a row stride padded to 128 entries ([G, db_scale_stride(N)]) so
// that every 128-wide tile of one group is a 16-byte aligned, in-bounds bulk copy.
__host__ __device__ inline int64_t db_scale_stride(int64_t n) { return (n + 127) / 128 * 128; }

// element types of activation inputs
enum { DB_F32 = 0, DB_F16 = 1, DB_BF16 = 2 };
// activation code layouts
// DB_CODES_DQ_F16: f16 [M, Kp], natural k order, each value f16(code * group scale) (the
// dequantised activations of the kind::f16 full-K GEMM, gemm_dq.cu)
enum { DB_CODES_NATURAL_I8 = 0, DB_CODES_GEMV_I8 = 1, DB_CODES_TC_F16 = 2, DB_CODES_DQ_F16 = 3 };
// GEMM epilogues
enum { DB_EPI_STORE = 0, DB_EPI_RESIDUAL = 1, DB_EPI_SWIGLU_QUANT = 2 };

int db_launch_quantize_rows(const void* x, int dtype, int64_t ldx, int M, int K, int bits, void* codes, int layout,
                            int64_t ldc, float* scales, int32_t* sums, int64_t lds, int* nonfinite,
                            cudaStream_t stream);
// Decima int8 quantiser (blocks of 16/32/64/128, round half away from zero of x / scale).  Weights
// use it with layout DB_CODES_NATURAL_I8 into the Q8 device layout and group-major scales
// [G, lds]; activations with DB_CODES_TC_F16.  row_major_scales = 1 writes scales [M, lds].
// Decima Weights mode (W8A32): y [M, ldy] = x [M, ldx] (f32) times int8 weight codes [N, ldw] in
// blocks of 32/64/128 with group-major scales [ceil(K/block), ldsw], + bias; fused = the AVX2 order.
int db_launch_decima_w8a32(const float* x, int64_t ldx, int M, int K, const uint8_t* w_codes, int64_t ldw,
                           const float* sw, int64_t ldsw, int N, int block, int fused, const float* bias, float* y,
                           int64_t ldy, int* nonfinite, cudaStream_t stream);
int db_launch_decima_quantize(const float* x, int64_t ldx, int M, int K, int block, void* codes, int layout,
                              int64_t ldc, float* scales, int64_t lds, int row_major_scales, int* nonfinite,
                              cudaStream_t stream);
int db_launch_pack_weights(const uint16_t* w, int N, int K, int bits, uint8_t* codes, float* scales, int* bad,
                           cudaStream_t stream);
int db_launch_dequant_rows(const uint8_t* codes, const float* scales, int N, int K, int bits, const int32_t* ids,
                           int T, float* out, int64_t ldo, int* bad, cudaStream_t stream);
int db_launch_packed_convert(uint8_t* packed, uint8_t* codes, float* scales, int N, int K, int bits, int to_device,
                             cudaStream_t stream);
int db_launch_codes_to_natural(const void* codes, int layout, int64_t ldc, int M, int Kp, int8_t* out,
                               cudaStream_t stream);

// Tensor-core grouped GEMM.  A: f16 codes (tensor-core order) [M, lda], sa [G, ldsa];
// W: device-layout codes [N, Kp*bits/8], sw [G, N].  Epilogue:
//   DB_EPI_STORE     y[m, n] = acc
//   DB_EPI_RESIDUAL  y[m, n] = y[m, n] + acc
//   DB_EPI_SWIGLU_QUANT  columns come in blocks of 64 gate + 64 up rows of W; the activation
//                    silu(gate) * up is quantised per 64 to f16 codes (tensor-core order) in
//                    out_codes [M, ldoc] and scales out_scales [N/128, ldos].
// fused = 1: sum = fma(dot, sw*sa, sum) (int8.rs:562-565); 0: sum += dot * (sa*sw) (int8.rs:276-278).
struct DbGemmArgs {
    const void* a_codes;
    int64_t lda;  // elements
    const float* sa;
    int64_t ldsa;
    const uint8_t* w_codes;
    const float* sw;
    int M, N, K, bits;
    int fused;
    int epilogue;
    float* y;
    int64_t ldy;
    void* out_codes;
    int64_t ldoc;
    float* out_scales;
    int64_t ldos;
    const int* nonfinite;  // optional: when *nonfinite != 0 the outputs are NaN (int8.rs:170-173)
    int* dev_error;        // device error word
    int block_n;           // tile width (0 = default)
    int max_ctas;          // persistent grid cap (0 = number of SMs)
    int pair_ctas;         // 1 = CTA pairs with M = 256 MMAs (used for 128-wide tiles when M > 128)
    int block;             // K values per scale group: 0 or 64 (group 64), 32 (Decima int8 blocks, Q8 only)
    const float* bias;     // add_bias = 1: y = acc + bias[n] (bias == nullptr: y = acc + 0)
    int add_bias;
    void* w_scratch;       // dequantised GEMM: f16 [N, Kp] for the unpacked weights (null: cached buffer)
    int overlap_unpack;    // 1: no running kernel reads w_scratch, so the unpack overlaps the previous kernel
    int k_splits;          // dequantised GEMM, store epilogue: 2 = two K halves into y rows 0..M-1, M..2M-1
};
int db_launch_gemm_tc(const DbGemmArgs& args, cudaStream_t stream);
// The same GEMM on int8 activation codes in natural order (DB_CODES_NATURAL_I8, a_codes [M, lda]
// bytes, lda % 16 == 0) with tcgen05 kind::i8 MMAs (gemm_i8.cuh).  Tile widths 64/128/256
// (default 256; the SwiGLU epilogue always 256, writing int8 natural codes to out_codes),
// optional CTA pairs (M = 256 MMAs), scale blocks of 64 or (Q8 only) 32.
int db_launch_gemm_i8(const DbGemmArgs& args, cudaStream_t stream);
// The GEMM on dequantised operands (gemm_dq.cu): a_codes f16 [M, lda] in DB_CODES_DQ_F16
// (sa unused); an unpack pass writes the weights as f16(code * scale) [N, Kp] into w_scratch
// (db_gemm_dq_scratch_bytes; null: a library buffer cached per device and stream), then tcgen05 kind::f16
// with f32 accumulation over the whole K; store or residual epilogue, tile widths 64/128/256.
int db_launch_gemm_dq(const DbGemmArgs& args, cudaStream_t stream);
int db_gemm_dq_default_block_n(int64_t M, int64_t N, int k_splits = 1);
size_t db_gemm_dq_scratch_bytes(int64_t N, int64_t K);

// Small-M path: int8 A codes (GEMV order) [M, lda] + sums [G, ldsa], sa [G, ldsa].
struct DbGemvArgs {
    const int8_t* a_codes;
    int64_t lda;
    const float* sa;
    const int32_t* a_sums;
    int64_t ldsa;
    const uint8_t* w_codes;
    const float* sw;
    int M, N, K, bits;
    int fused;
    int residual;
    float* y;
    int64_t ldy;
    const int* nonfinite;
};
int db_launch_gemv(const DbGemvArgs& args, cudaStream_t stream);
int db_gemv_rows_limit();

int db_num_sms();
// Launches `kernel` with the programmatic-serialization attribute: its CTAs may start on SMs the
// previous kernel in the stream has released, before that kernel completes.  Only for kernels
// that call pdl_wait() before their first access to memory.
template <typename... KArgs, typename... Args>
cudaError_t db_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
// cuTensorMapEncodeTiled, reached through the runtime's driver entry point (null when absent).
typedef CUresult (*DbEncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
DbEncodeTiledFn db_encode_tiled();
// Raises a kernel's dynamic shared-memory limit once per (kernel, device): function attributes
// belong to a device's context, so a process that drives several GPUs sets them on each.
// Thread-safe.
cudaError_t db_set_max_smem(const void* kernel, int bytes);
