// Host entry of the kind::i8 tensor-core GEMM (gemm_i8.cuh): argument checks, tensor maps, and
// the choice of instantiation.
#include <string.h>

#include "gemm_i8.cuh"

int db_gemm_i8_q4(const DbGemmArgs& a, int bn, bool pair, const db::gi8::Maps& mp, cudaStream_t s);
int db_gemm_i8_q8(const DbGemmArgs& a, int bn, bool pair, const db::gi8::Maps& mp, cudaStream_t s);
int db_gemm_i8_swiglu(const DbGemmArgs& a, int bn, bool pair, const db::gi8::Maps& mp, cudaStream_t s);

int db_launch_gemm_i8(const DbGemmArgs& a, cudaStream_t stream) {
    using namespace db::gi8;
    if (a.M <= 0 || a.N <= 0) return 0;
    if (a.K <= 0 || (a.bits != 4 && a.bits != 8)) return (int)cudaErrorInvalidValue;
    if (a.block != 0 && a.block != 64 && !(a.block == 32 && a.bits == 8 && a.epilogue != DB_EPI_SWIGLU_QUANT))
        return (int)cudaErrorInvalidValue;
    DbEncodeTiledFn enc = db_encode_tiled();
    if (!enc) return (int)cudaErrorNotSupported;
    const int G = (a.K + 63) / 64, Kp = G * 64;
    int bn = a.block_n ? a.block_n : 256;
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) {
        if (bn == 64) bn = 128;  // a SwiGLU tile holds whole blocks of 64 gate + 64 up rows
        if (a.N % 128 || !a.out_codes || !a.out_scales || (reinterpret_cast<uintptr_t>(a.out_codes) & 15) ||
            (a.ldoc & 15) || a.ldoc < a.N / 2 || a.ldos < db_scale_stride(a.M))
            return (int)cudaErrorInvalidValue;
    }
    if (bn != 32 && bn != 64 && bn != 128 && bn != 256) return (int)cudaErrorInvalidValue;
    // CTA pairs (M = 256 MMAs) when asked for and there are rows for both CTAs (not at 32-wide tiles)
    const bool pair = a.pair_ctas && a.M > BM && bn != 32;
    if ((reinterpret_cast<uintptr_t>(a.a_codes) & 15) || (a.lda & 15) || a.lda < Kp ||
        (reinterpret_cast<uintptr_t>(a.w_codes) & 15) || (reinterpret_cast<uintptr_t>(a.sa) & 15) ||
        (reinterpret_cast<uintptr_t>(a.sw) & 15) || a.ldsa < db_scale_stride(a.M) || (a.ldsa & 3))
        return (int)cudaErrorMisalignedAddress;
    Maps mp;
    memset(&mp, 0, sizeof(mp));
    mp.G = G;
    {
        cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.lda};
        cuuint32_t box[2] = {KS, BM};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&mp.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a.a_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    {
        const int wr = pair ? bn / 2 : bn;
        const cuuint64_t row_bytes = (cuuint64_t)Kp * a.bits / 8;
        cuuint64_t dims[2] = {row_bytes, (cuuint64_t)a.N};
        cuuint64_t strides[1] = {row_bytes};
        // Q8: the stage's 128 k of each row, 128B swizzle (the MMA operand as loaded); Q4: the
        // raw 64 bytes of nibbles, unswizzled, for the converter warps
        cuuint32_t box[2] = {(cuuint32_t)(a.bits == 8 ? KS : KS / 2), (cuuint32_t)wr};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&mp.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(a.w_codes), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, a.bits == 8 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    // output tensor map for the TMA store / reduce-add (fallback: plain per-thread stores)
    if (a.epilogue != DB_EPI_SWIGLU_QUANT && a.y && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ldy % 4 == 0 &&
        a.ldy >= a.N) {
        cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.ldy * 4};
        cuuint32_t box[2] = {16, 32};
        cuuint32_t estr[2] = {1, 1};
        mp.y_tma = enc(&mp.y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.y, dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (a.epilogue == DB_EPI_SWIGLU_QUANT) return db_gemm_i8_swiglu(a, bn, pair, mp, stream);
    return a.bits == 4 ? db_gemm_i8_q4(a, bn, pair, mp, stream) : db_gemm_i8_q8(a, bn, pair, mp, stream);
}
