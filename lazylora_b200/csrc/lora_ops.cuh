// Host launchers of the LoRA product kernels (k_skinny, k_expand, k_outer8 and their
// fixed-order reductions), defined with the routed-expert layer that uses them most; each
// returns an LL_* status.
#pragma once
#include <cstddef>

#include <cuda_runtime.h>

namespace ll {

// C0 (and C1) = alpha * A[M][K] . B; A dtype adt (0 f32, 1 bf16, 2 f16); B rows ([N][K], B0 the
// first N0, B1 the rest) when brows, else columns ([K][N] in B0); part holds part_floats floats,
// at least M * N. Up to 128 rows with B as rows: one block per column and 16 rows (k_gemv_rows),
// no split partials.
int skinny(const void* A, int adt, bool brows, int M, int K, const float* B0, const float* B1, int N0, int N,
           float alpha, float* C0, float* C1, float* part, size_t part_floats, cudaStream_t s);
// out[T][C] = [sum of Y rows] + alpha * (L0 . R0 + L1 . R1), fp32 (k_expand).
// out1 given: two products in one launch, out = alpha L0 R0 and out1 = alpha L1 R1.
// qz given (with tok_pos, qtw): L0 is q[t][rr] = sum over the token's pairs (ascending expert)
// of qtw[pos] * qz[pos][rr], computed in the kernel and also stored to q_out when given.
int expand(bool rrows, const int* tok_pos, const float* Y, int k, int T, int C, int r, float alpha, const float* L0,
           const float* R0, const float* L1, const float* R1, float* out, cudaStream_t s, float* out1 = nullptr,
           const float* qtw = nullptr, const float* qz = nullptr, float* q_out = nullptr);
// out = sc * sum_n Pm(n, :)^T Q[n][:], [r][C] or transposed [C][r]; part holds nseg_max * r * C floats
int outer(const float* Pm, const int* perm_token, const float* tw, const void* Q, int qdt, int N, const int* n_dev,
          int C, int r, float sc, bool transposed, float* part, int nseg_max, float* out, cudaStream_t s);

}  // namespace ll
