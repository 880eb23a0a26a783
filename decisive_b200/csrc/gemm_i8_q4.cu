// Instantiations of the kind::i8 GEMM for Q4 weights (store and residual epilogues).
#include "gemm_i8.cuh"

int db_gemm_i8_q4(const DbGemmArgs& a, int bn, bool pair, const db::gi8::Maps& mp, cudaStream_t s) {
    using namespace db::gi8;
    if (a.epilogue == DB_EPI_RESIDUAL)
        return a.fused ? launch_bn<4, DB_EPI_RESIDUAL, true, 1>(a, bn, pair, mp, s)
                       : launch_bn<4, DB_EPI_RESIDUAL, false, 1>(a, bn, pair, mp, s);
    return a.fused ? launch_bn<4, DB_EPI_STORE, true, 1>(a, bn, pair, mp, s)
                   : launch_bn<4, DB_EPI_STORE, false, 1>(a, bn, pair, mp, s);
}
