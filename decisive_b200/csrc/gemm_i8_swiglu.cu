// Instantiations of the kind::i8 GEMM with the fused SwiGLU + re-quantisation epilogue.
#include "gemm_i8.cuh"

int db_gemm_i8_swiglu(const DbGemmArgs& a, int bn, bool pair, const db::gi8::Maps& mp, cudaStream_t s) {
    using namespace db::gi8;
    if (a.bits == 4)
        return a.fused ? launch_bn<4, DB_EPI_SWIGLU_QUANT, true, 1>(a, bn, pair, mp, s)
                       : launch_bn<4, DB_EPI_SWIGLU_QUANT, false, 1>(a, bn, pair, mp, s);
    return a.fused ? launch_bn<8, DB_EPI_SWIGLU_QUANT, true, 1>(a, bn, pair, mp, s)
                   : launch_bn<8, DB_EPI_SWIGLU_QUANT, false, 1>(a, bn, pair, mp, s);
}
