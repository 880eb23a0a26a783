// Error plumbing shared by the C ABI translation units.
#pragma once
#include <string>

void db_set_error(const char* code, const std::string& message);
int db_fail(int status, const char* code, const std::string& message);
int db_cuda_status(int cuda_error, const char* what);
int* db_device_error_ptr();

// Tuner for one tensor-core GEMM shape (tuner.cu); *report receives the JSON report.
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/decisive_b200.h"
int db_tune_gemm_shape(int64_t M, int64_t N, int64_t K, int bits, int epilogue, const char* cache_path,
                       db_gemm_config* choice, std::string* report, cudaStream_t stream, bool i8);
// Default tile configuration of the int8 (kind::i8) tensor-core GEMM for an M x N output.
db_gemm_config db_gemm_i8_default_config(int64_t M, int64_t N, int epilogue);
