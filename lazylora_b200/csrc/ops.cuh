// Launchers shared between the translation units of the library.
#pragma once
#include "host_common.cuh"

namespace ll {

int check_arch();

int launch_prepare_beta(const uint8_t* s_a, const uint8_t* s_b, int E, int rows, int cols, int64_t sstride,
                        int32_t* beta, int col, cudaStream_t s);

// Transposed codes [E][C][R/2] and fp16 column multipliers [E][C/32][R] of a stack of MXFP4
// matrices W[E][R][C] (bias beta[e*2 + col] folded into the multipliers).
int launch_transpose_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t sstride, int E, int R, int C,
                           const int32_t* beta, int col, uint8_t* codes_t, __half* scales_t, cudaStream_t s);

// chunks[i] = {expert 0, rows i*nmax .. } covering M rows of a single matrix, and their count.
int launch_single_expert_chunks(Chunk* chunks, int* n_chunks, int M, int nmax, cudaStream_t s);

// dst[row] = fp16(src[index[row]] * 2^sigma_row), inv[row] = 2^-sigma_row (index may be null;
// a negative index gives a zero row). src_dtype: 0 fp32, 1 bf16.
int launch_rows_to_half(const void* src, int src_dtype, const int* index, int rows, int K, __half* dst, float* inv,
                        cudaStream_t s, int ld = -1);   // ld: dst row stride (>= K, default K)
// The per-pair rows from the T source rows through tok_pos ([T][k] pair positions, -1 for
// none): one read and one scale per token (falls back to the per-pair conversion through
// perm_token for shapes the vector kernel does not take).
int launch_token_rows_to_half(const void* src, int src_dtype, const int* perm_token, const int* tok_pos, int T, int k,
                              int K, __half* dst, float* inv, cudaStream_t s);

// The block-scaled MMA's weight scales of a stack of MXFP4 matrices W[E][R][C] (R % 128 == 0,
// C % 128 == 0): for every 128-row tile and 128-K stage, a 512-byte block of 32 lines x 16
// bytes, line l holding the 4 scale bytes of rows l, l + 32, l + 64, l + 96 (the layout
// tcgen05.cp copies into tensor memory); bytes >= 253 become 0. out: E * R * C / 32 bytes.
int launch_prepare_sfa(const uint8_t* scales, int64_t sstride, int E, int R, int C, uint8_t* out, cudaStream_t s);

// Rows as three E4M3 terms ([3][rows][K] bytes) with their inverse power-of-two scales
// ([3][rows] floats): per row, term t is the nearest E4M3 values of (x - earlier terms) * 2^e_t,
// e_t bringing that residual's largest entry into [2^7, 2^8). tok_pos given: source rows are
// the T tokens and each is written to its pair positions tok_pos[t][0..k) (-1 skipped);
// otherwise source row p -> row p for p < *n_valid (n_valid may be null: all rows).
// src_dtype: 0 fp32, 1 bf16, 2 fp16. K % 8 == 0, K <= 8192.
int launch_rows_to_e4m3x3(const void* src, int src_dtype, int src_rows, const int* tok_pos, int k,
                          const int* n_valid, int K, int64_t P, uint8_t* dst, float* inv3, cudaStream_t s);

// Rows as four E2M1 terms ([4][rows][K/2] packed bytes), the BS_FP4 activation operand, with
// their E8M0 block-32 scales written straight into the MMA's B scale blocks of each row's chunk
// ([max_chunks][K/128][512], chunk_of[p] = the chunk of pair row p; words no row owns are not
// written: they scale only MMA columns nobody reads); same source / destination rules as
// launch_rows_to_e4m3x3. K % 128 == 0, chunks of at most nmax <= 32 rows.
int launch_rows_to_e2m1x4(const void* src, int src_dtype, int src_rows, const int* tok_pos, int k,
                          const int* n_valid, int K, int64_t P, uint8_t* dst, const Chunk* chunks, const int* chunk_of,
                          int nmax, uint8_t* sfb, cudaStream_t s);

// The few-token sort of the routed pairs (the outputs of k_plan_small: offsets, chunks,
// n_chunks, perm_token, perm_slot, pair_pos, tw, tok_pos, chunk_of; the status word and n_zero
// ints at `zero` cleared) and the T token rows of src as launch_rows_to_e2m1x4 writes them to
// their pair rows, in one launch. E <= 1024, k <= 32, T k <= 2048, nmax <= 32.
int launch_plan_rows_to_e2m1x4(const int64_t* idx, const float* w, int T, int k, int E, int nmax, int* offsets,
                               Chunk* chunks, int* n_chunks, int* perm_token, int* perm_slot, int* pair_pos, float* tw,
                               int* tok_pos, int* chunk_of, DevStatus* st, int* zero, int n_zero, const void* src,
                               int src_dtype, int K, int64_t P, uint8_t* dst, uint8_t* sfb, cudaStream_t s);

// C0 [T][r] (and C1) = x [T][d] (bf16) . W0^T (W1^T) for LoRA projection matrices W [r][d], or
// x . W for W [d][r] when `transposed`, on the tensor cores: W split into three bf16 planes
// (exact), the router's tcgen05 logits kernel split over K to fill the SMs, the splits' fp32
// partials added in order. Workspace project_tc_bytes(T, d, rows = r or 2r); bounded waits
// report to st.
size_t project_tc_bytes(int T, int d, int E);
int project_tc(const void* x, int T, int d, const float* W0, const float* W1, bool transposed, int r, float* out0,
               float* out1, void* ws, size_t ws_bytes, DevStatus* st, cudaStream_t s);

}  // namespace ll
