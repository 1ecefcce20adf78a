// Launchers shared between the translation units of the library.
#pragma once
#include "host_common.cuh"

namespace ll {

int check_arch();

int launch_prepare_beta(const uint8_t* s_a, const uint8_t* s_b, int E, int rows, int cols, int64_t sstride,
                        int32_t* beta, int col, cudaStream_t s);

// dst[row] = fp16(src[index[row]] * 2^sigma_row), inv[row] = 2^-sigma_row (index may be null;
// a negative index gives a zero row). src_dtype: 0 fp32, 1 bf16.
int launch_rows_to_half(const void* src, int src_dtype, const int* index, int rows, int K, __half* dst, float* inv,
                        cudaStream_t s);

}  // namespace ll
