/*
 * lazylora_b200 — C ABI of the B200 (sm_100a) routed-expert MXFP4 path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no torch types. Every buffer is
 * device memory owned by the caller (the library never allocates or frees); scratch space
 * is a caller-sized workspace whose size the *_workspace_bytes functions return.
 * Every call returns an ll_status; kernels never trap: a bounded wait that runs out is
 * reported as LL_ERR_TIMEOUT through the status word read back after the launch.
 *
 * Weight format (the reference's, lazy_lora/native/mxfp4_gemm.c:12-18): W is [R, K] with K a
 * multiple of 32; packed [R, K/2] bytes, element 2j in the low nibble of byte j; scales
 * [R, K/32] E8M0 bytes, 2^(b-127), bytes >= 253 contribute zero. Here the scale rows may be
 * padded: `scale_stride` is the byte distance between scale rows and must be a multiple of
 * 16 (it equals K/32 whenever K is a multiple of 512, e.g. 7168, 3584, 2048).
 */
#ifndef LAZYLORA_B200_H
#define LAZYLORA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LL_OK = 0,
  LL_ERR_ARG = 1,        /* bad shape, stride, alignment or pointer */
  LL_ERR_CUDA = 2,       /* a CUDA runtime call failed (launch, memcpy, attribute) */
  LL_ERR_TIMEOUT = 3,    /* a device-side bounded wait ran out; the kernel wound down */
  LL_ERR_WORKSPACE = 4,  /* workspace smaller than *_workspace_bytes asked for */
  LL_ERR_RANGE = 5,      /* value outside what the kernel represents exactly */
  LL_ERR_ARCH = 6,       /* device is not sm_100 */
  LL_ERR_IO = 7          /* a host file read failed (ll_pread_batch) */
} ll_status;

/* Human-readable text for a status code (static storage). */
const char* ll_status_string(int status);

/* Last CUDA error text seen by the library on this thread ("" if none). */
const char* ll_last_cuda_error(void);

/* ------------------------------------------------------------------ drop-in kernels
 * Device-pointer versions of the four symbols of lazy_lora/native/mxfp4_gemm.c, with the
 * same argument meaning; `ws` is scratch of ll_mxfp4_workspace_bytes(M, K, R) bytes.
 */

/* Replaces mxfp4_threads (lazy_lora/native/mxfp4_gemm.c:131-138): the parallel width the
 * kernels use (streaming multiprocessors of the current device). */
int ll_mxfp4_threads(void);

size_t ll_mxfp4_workspace_bytes(int M, int K, int R);

/* Replaces mxfp4_gemm (lazy_lora/native/mxfp4_gemm.c:64-94): y[M,R] = x[M,K] . W^T. */
int ll_mxfp4_gemm(float* y, const float* x, const uint8_t* packed, const uint8_t* scales,
                  int M, int K, int R, int64_t scale_stride, void* ws, size_t ws_bytes,
                  void* stream);

/* No counterpart in the reference. ll_mxfp4_gemm without a workspace argument, for callers
 * that cannot allocate device memory (a binding that holds raw pointers and no device
 * allocator, or code running where allocation is not allowed). Its scratch is a static
 * device array of LL_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * exit; M * K must fit it (about M * K * 2 + M * 4 bytes, 8 MiB: e.g. M <= 580 at K = 7168),
 * larger sizes return LL_ERR_WORKSPACE. scale_stride must be >= K/32 and a multiple of 16
 * (such a caller pads its scale rows itself; K a multiple of 512 needs no padding). The
 * first call on a device looks up the array's device address (make it before any stream
 * capture; it is looked up again if the device's context was recreated, e.g. after
 * cudaDeviceReset). The call returns once its GPU work finished (it reads the device status
 * word back). All calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller. Allocates nothing. */
#define LL_NOALLOC_SCRATCH_BYTES (8u << 20)
int ll_mxfp4_gemm_noalloc(float* y, const float* x, const uint8_t* packed, const uint8_t* scales,
                          int M, int K, int R, int64_t scale_stride, void* stream);

/* Replaces mxfp4_gemm_t (lazy_lora/native/mxfp4_gemm.c:96-129): y[M,K] += dy[M,R] . W
 * (accumulates into y, as the reference does). */
int ll_mxfp4_gemm_t(float* y, const float* dy, const uint8_t* packed, const uint8_t* scales,
                    int M, int K, int R, int64_t scale_stride, void* ws, size_t ws_bytes,
                    void* stream);

/* Replaces mxfp4_dequant (lazy_lora/native/mxfp4_gemm.c:142-150): out[R,K] = W, exact.
 * out_dtype: 0 = fp32 (the reference's), 1 = bf16, 2 = fp16 (exact when the scale bytes
 * lie in 104..140). Note the reference's (K, R) argument order. */
int ll_mxfp4_dequant(void* out, const uint8_t* packed, const uint8_t* scales, int K, int R,
                     int64_t scale_stride, int out_dtype, void* stream);

/* ------------------------------------------------------------------------- router
 * KimiK3MoERouter.forward (lazy_lora/core/moe_router.py:80-100): logits = x . Wr^T (fp32),
 * scores = sigmoid(logits), selection on scores + bias (bias may be NULL), top-k in
 * descending order (ties: lower expert id first), weights gathered from the unbiased
 * scores, renormalised by (sum + 1e-20) when renormalize != 0 and k > 1, times scale.
 * x_dtype: 0 = fp32, 1 = bf16. idx is int64 [T,k] like torch.topk's indices.
 * The logits run on the tensor cores with Wr split exactly into three bf16 planes (and fp32
 * x likewise), accumulating in fp32: fp32-level accuracy, another summation order than the
 * reference's F.linear. d must be a multiple of 8, x 16-byte aligned, ws 256-byte aligned.
 */
size_t ll_route_workspace_bytes(int T, int d, int E);
int ll_route_topk(const void* x, int x_dtype, const float* router_w, const float* bias,
                  int T, int d, int E, int k, int renormalize, float routed_scaling_factor,
                  int64_t* idx, float* w, float* scores_out /* optional [T,E] */,
                  void* ws, size_t ws_bytes, void* stream);

/* The router weight is frozen during LoRA training, so its split into the three bf16 planes
 * the logits read can be made once: ll_route_prepare writes planes [3][E][d] (bf16, 16-byte
 * aligned), and ll_route_topk_prepared is ll_route_topk reading them instead of router_w
 * (same results bit for bit). Redo the split whenever the weight changes. */
int ll_route_prepare(const float* router_w, int E, int d, uint16_t* planes, void* stream);
int ll_route_topk_prepared(const void* x, int x_dtype, const uint16_t* planes, const float* bias,
                           int T, int d, int E, int k, int renormalize, float routed_scaling_factor,
                           int64_t* idx, float* w, float* scores_out /* optional [T,E] */,
                           void* ws, size_t ws_bytes, void* stream);

/* The selection half alone (moe_router.py:92-99) from given fp32 scores / scores_for_choice:
 * bit-exact indices and weights for identical inputs. */
int ll_route_select(const float* scores, const float* scores_for_choice, int T, int E, int k,
                    int renormalize, float routed_scaling_factor, int64_t* idx, float* w,
                    void* stream);

/* ------------------------------------------------------------ routed-expert layer
 * One MoE layer's routed experts: the forward sum of LazyLoRATrainer._routed_experts_forward
 * (lazy_lora/trainer/lazy_trainer.py:806-834) and the manual backward of
 * _routed_experts_backward (lazy_trainer.py:836-880), with the layer's shared rank-r LoRA
 * adapters (lazy_lora/core/lora_layer.py) on gate, up and down and the SiTU-GLU activation
 * (lazy_lora/core/situ_activation.py).
 */
typedef struct {
  int d;          /* expert input width (K of gate/up), multiple of 128 */
  int f;          /* expert intermediate width, multiple of 128 */
  int E;          /* experts resident in these arrays (local experts under expert parallelism) */
  int r;          /* LoRA rank, 1..64 */
  float lora_scaling;          /* alpha / r */
  const uint8_t* w1p;  const uint8_t* w1s;   /* gate  [E,f,d/2], scales [E,f,*] */
  const uint8_t* w3p;  const uint8_t* w3s;   /* up    [E,f,d/2], scales [E,f,*] */
  const uint8_t* w2p;  const uint8_t* w2s;   /* down  [E,d,f/2], scales [E,d,*] */
  int64_t s13_stride;          /* scale row stride of gate/up, bytes (>= d/32, %16 == 0) */
  int64_t s2_stride;           /* scale row stride of down, bytes (>= f/32, %16 == 0) */
  const int32_t* beta;         /* [E][2] power-of-two decode bias from ll_moe_prepare */
  const float* A_g; const float* B_g;   /* gate LoRA A [r,d], B [f,r] */
  const float* A_u; const float* B_u;   /* up   LoRA A [r,d], B [f,r] */
  const float* A_d; const float* B_d;   /* down LoRA A [r,f], B [d,r] */
  /* Transposed copies for the backward, built by ll_moe_prepare into caller buffers:
   * codes of W^T ([E,d,f/2] for gate/up, [E,f,d/2] for down) and the per-element scales as
   * fp16 multipliers with the decode bias folded in ([E,d/32,f] gate/up, [E,f/32,d] down).
   * ll_moe_forward does not read them (they may be NULL there); ll_moe_backward needs them. */
  const uint8_t* w1t; const uint8_t* w3t; const uint8_t* w2t;
  const uint16_t* s1t; const uint16_t* s3t; const uint16_t* s2t;
  /* Valid (token, expert) pairs the next forward / backward will see, or 0: taken as T*k. Sets
   * the token-tile width; give it when many slots are -1 (expert parallelism). The forward and
   * the backward that follows must see the same value. */
  int rows_hint;
  /* The forward GEMMs' weight scales in the layout the block-scaled tensor-core MMA reads,
   * built by ll_moe_prepare into caller buffers of ll_mxfp4_sf_bytes(E, rows, cols) bytes:
   * gate and up ([E, f, d]) and down ([E, d, f]). Required by ll_moe_forward. */
  const uint8_t* w1sf; const uint8_t* w3sf; const uint8_t* w2sf;
} ll_moe_layer;

/* Bytes of the block-scaled MMA's scale layout of a stack of E matrices of R rows and C
 * columns (R, C multiples of 128): E * R * C / 32. */
size_t ll_mxfp4_sf_bytes(int E, int R, int C);

/* One-time preparation per weight load (the base weights are frozen): the per-expert
 * decode bias beta (beta[e][0] gate+up, beta[e][1] down, so that every scale byte within 36
 * of the matrix maximum decodes exactly to fp16), then the transposed copies w1t..s2t that
 * L points at (beta_out must be L->beta). It also lays out the scale blocks w1sf, w2sf, w3sf
 * the forward reads. With all six transposed pointers NULL only beta and the scale blocks are
 * built: enough for ll_moe_forward; call again with the buffers set before a backward.
 * Some but not all of them NULL is LL_ERR_ARG. */
int ll_moe_prepare(const ll_moe_layer* L, int32_t* beta_out, void* stream);

/* Bytes of each transposed copy ll_moe_prepare fills: codes (same as the packed stack) and
 * fp16 scale tables, for a stack of E matrices of R rows and C columns. */
size_t ll_mxfp4_transposed_bytes(int E, int R, int C, int which /* 0 codes, 1 scales */);

/* Workspace for a forward + backward of T tokens with top-k routing. The forward leaves
 * the activations the backward needs in it (the role of ctx.save_for_backward). */
size_t ll_moe_workspace_bytes(const ll_moe_layer* L, int T, int k);

/* out[T,d] fp32 = sum over the k selected experts of w * expert(x) (experts ascending).
 * idx int64 [T,k] (values < E, distinct per row; -1 = slot not routed here), w fp32 [T,k].
 * x_dtype: 0 = fp32, 1 = bf16. */
int ll_moe_forward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype,
                   const int64_t* idx, const float* w, float* out, void* ws, size_t ws_bytes,
                   void* stream);
/* ll_moe_forward whose final combine also RMS-normalises each token's row (the latent block's
 * routed_expert_norm after the routed experts' sum, lazy_trainer.py:731-733, with
 * RMSNormFunction.forward, trunk_streamer.py:27-31): out as ll_moe_forward (fp32 [T, d]),
 * normed[t] = bf16(out[t] * rsqrt(mean(out[t]^2) + eps) * norm_w) ([T, d]), rstd[t] the row's
 * rsqrt (fp32 [T]) for ll_rmsnorm_backward. norm_w fp32 [d]; norm_w and normed 8-byte aligned. */
int ll_moe_forward_rmsnorm(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx,
                           const float* w, const float* norm_w, float eps, float* out, void* normed, float* rstd,
                           void* ws, size_t ws_bytes, void* stream);

/* Backward of the forward that last ran in `ws` for upstream gradient g [T,d] (g_dtype as
 * x_dtype): grad_h [T,d], grad_w [T,k] (fp32, overwritten) and the LoRA gradients
 * dA_g [r,d], dB_g [f,r], dA_u [r,d], dB_u [f,r], dA_d [r,f], dB_d [d,r] (fp32, overwritten;
 * the caller adds them into .grad as accumulate_grad does). */
int ll_moe_backward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype,
                    const int64_t* idx, const float* w, const void* g, int g_dtype,
                    float* grad_h, float* grad_w, float* dA_g, float* dB_g, float* dA_u,
                    float* dB_u, float* dA_d, float* dB_d, void* ws, size_t ws_bytes,
                    void* stream);

/* Reads and clears the device status word the layer kernels write into `ws` (a bounded
 * wait that ran out, see LL_ERR_TIMEOUT). Synchronises `stream`. */
int ll_moe_status(const ll_moe_layer* L, int T, int k, void* ws, void* stream);

/* The stable permutation the last ll_moe_forward built in `ws` (device buffers): offsets
 * [E+1] of each expert's rows, then token and slot of each sorted row (expert ascending,
 * tokens ascending within an expert: the row order of lazy_trainer.py:823-827). Rows past
 * offsets[E] are -1. */
int ll_moe_permutation(const ll_moe_layer* L, int T, int k, void* ws, int* offsets,
                       int* perm_token, int* perm_slot, void* stream);

/* ------------------------------------------------------------------ expert parallelism
 * No counterpart in the reference, which runs the routed experts in one process
 * (lazy_trainer.py:806-880 loops over every expert locally); these are the index kernels
 * around the two all-to-all exchanges of an expert-parallel layer. Expert e lives on rank
 * floor(e * n / E). Each rank routes its own T tokens and sends every token row once to each
 * rank owning one of its experts; that rank runs ll_moe_forward / ll_moe_backward on the rows
 * it received and returns per-row fp32 partials, which the origin rank adds in ascending
 * rank order. The exchanges themselves (NCCL all-to-all) are the caller's.
 */

/* First expert id and expert count of `rank` (contiguous blocks). */
int ll_ep_experts_of_rank(int E, int n_ranks, int rank, int* first, int* count);

/* Send plan of this rank's tokens. idx int64 [T,k] global expert ids, w fp32 [T,k].
 * counts int32 [n_ranks + 1]: rows for each destination rank, then the number of slots whose
 * id is outside [0, E) (those slots are routed nowhere; callers treat nonzero as an error).
 * pos int32 [T, n_ranks]: send-buffer row of token t for rank r, or -1.
 * Send rows (at most T * n_ranks) are grouped by destination rank ascending, tokens
 * ascending: send_tok int32 [rows] source token, send_idx int64 [rows, k] expert id local to
 * the destination rank or -1 where that slot's expert is elsewhere, send_w fp32 [rows, k]
 * (0 where send_idx is -1). Deterministic (no order-dependent atomics in the outputs). */
int ll_ep_plan(int T, int k, int E, int n_ranks, const int64_t* idx, const float* w, int* counts, int* pos,
               int* send_tok, int64_t* send_idx, float* send_w, void* stream);

/* dst[i, :] = src[tok[i], :] for i < rows; row_bytes a multiple of 16, 16-byte aligned buffers. */
int ll_ep_gather_rows(void* dst, const void* src, const int* tok, int rows, int64_t row_bytes, void* stream);

/* out[t, :] = sum over r = 0..n_ranks-1 (ascending) of part[pos[t, r], :] where pos >= 0;
 * fp32 rows of width d (a multiple of 4); part holds the returned partials in send order. */
int ll_ep_combine(float* out, const float* part, const int* pos, int T, int n_ranks, int d, void* stream);

/* Packs fp32 partial rows [rows, d] (d a multiple of 4) for the return exchange: each row as
 * d fp16 values scaled by a power of two 2^e that brings its largest magnitude into
 * [2^14, 2^15), then the fp32 2^-e and 12 bytes of padding: 2d + 16 bytes a row (half the
 * fp32 payload; 2^-11 relative rounding). 16-byte aligned buffers. */
int ll_ep_pack_rows(void* dst, const float* src, int rows, int d, void* stream);

/* ll_ep_combine over packed rows (ll_ep_pack_rows layout): out[t, :] = sum over r ascending of
 * the unpacked row pos[t, r], in fp32. */
int ll_ep_combine_packed(float* out, const void* part, const int* pos, int T, int n_ranks, int d, void* stream);

/* grad_w[t, j] = part[pos[t, owner(idx[t, j])], j] (fp32 [rows, k] partials in send order);
 * 0 for a slot whose id is outside [0, E). */
int ll_ep_combine_slots(float* grad_w, const float* part, const int* pos, const int64_t* idx, int T, int k, int E,
                        int n_ranks, void* stream);

/* ------------------------------------------------------------- checkpoint reads
 * Reads n byte ranges of files into host buffers (pinned, when they feed host-to-device
 * copies) with `threads` worker threads: range i is [offsets[i], offsets[i] + sizes[i]) of
 * paths[i] into dsts[i]. Short reads continue; a transient EIO (from the open or a read) is
 * retried up to `retries` times per range, sleeping retry_ms * attempt and reopening the file,
 * the policy of the reference's MmapTensorStreamer._read_range (mmap_loader.py:260-294). On
 * failure returns LL_ERR_IO with the lowest failing range index in *failed_index and the
 * reason in ll_last_cuda_error(); the bytes read are counted in *bytes_done. No CUDA call is
 * made. */
int ll_pread_batch(int n, const char* const* paths, const int64_t* offsets, const int64_t* sizes, void* const* dsts,
                   int threads, int retries, int retry_ms, int64_t* bytes_done, int* failed_index);

/* ------------------------------------------------------------------ shared expert
 * The element-wise middle of the shared expert (dense SiTU-GLU MLP with LoRA on its three
 * projections, lazy_trainer.py:702-707) between its bf16 GEMMs. Forward: from the bf16
 * projections G, U [N, F] and the LoRA A products xa_g, xa_u [N, r] fp32 with B_g, B_u [F, r]
 * fp32: SG = bf16(G + bf16(s xa_g B_g^T)), SU likewise, H = bf16(situ_glu(SG, SU)), all bf16
 * [N, F]. Backward: from Dh (bf16 [N, F], the down projection's input gradient g W_d) and
 * gB = g B_d [N, r] fp32 with A_d [r, F] fp32: dh = bf16(Dh + bf16(s gB A_d)), then the
 * SiTU-GLU gradients DSG, DSU (bf16 [N, F]) at the saved SG, SU. r in {4, 8, 16, 32}. */
int ll_shared_glu_forward(const void* G, const void* U, const float* xa_g, const float* xa_u, const float* B_g,
                          const float* B_u, float scaling, int N, int F, int r, void* SG, void* SU, void* H,
                          void* stream);
int ll_shared_glu_backward(const void* Dh, const float* gB, const float* A_d, float scaling, const void* SG,
                           const void* SU, int N, int F, int r, void* DSG, void* DSU, void* stream);

/* ------------------------------------------------------------------ LoRA products
 * The rank-r products of a LoRA adapter (lora_layer.py:104-123: delta = s (x A^T) B^T) around a
 * bf16 projection, reading the bf16 activations directly (the reference casts them to fp32
 * first). Sums run in a fixed order: results are bitwise reproducible.
 * ll_lora_down: C = alpha X B, X [M, K] (x_dtype 0 fp32, 1 bf16, 2 fp16; 16-byte aligned,
 *   K % 8 == 0). b_rows = 1: B given as rows [n, K] (LoRA A matrices), B0 the first n0 rows
 *   into C0 [M, n0], B1 the other n - n0 into C1 [M, n - n0] (both A_g and A_u of a gate/up
 *   pair in one pass). b_rows = 0: B0 [K, n] (a LoRA B matrix), n0 == n, into C0 [M, n].
 *   Split-K partials go to `workspace` (16-byte aligned, at least 4 M n bytes, else
 *   LL_ERR_WORKSPACE; fewer splits when it is small).
 * ll_lora_outer: out = scale sum_n P[n]^T Q[n], P [N, r] fp32, Q [N, C] (q_dtype as above,
 *   C % 4 == 0), stored [r, C] (dA = s (gB)^T x) or, transposed, [C, r] (dB = s g^T (x A^T)).
 *   `workspace` holds at least 4 r C bytes (else LL_ERR_WORKSPACE).
 * ll_lora_add_bf16: out = bf16(Y + bf16(scale L0 R0) [+ bf16(scale L1 R1)]), Y and out bf16
 *   [N, C] (may be the same buffer), L [N, r] fp32, R(rr, c) = R[rr C + c] ([r, C], r_rows = 1)
 *   or R[c r + rr] ([C, r], r_rows = 0). r in {4, 8, 16, 32}; L1 = NULL for one delta. */
int ll_lora_down(const void* X, int x_dtype, int M, int K, const float* B0, const float* B1, int n0, int n,
                 int b_rows, float alpha, float* C0, float* C1, void* workspace, size_t workspace_bytes,
                 void* stream);
int ll_lora_outer(const float* P, const void* Q, int q_dtype, int N, int C, int r, float scale, int transposed,
                  float* out, void* workspace, size_t workspace_bytes, void* stream);
int ll_lora_add_bf16(const void* Y, const float* L0, const float* R0, const float* L1, const float* R1, int r,
                     int r_rows, float scale, int N, int C, void* out, void* stream);

/* -------------------------------------------------------------- dense bf16 GEMMs
 * The plain projections around the routed experts (the latent block's down / up projections,
 * lazy_trainer.py:722-735, and the shared expert's gate / up / down), whose F.linear products
 * the reference runs as bf16 GEMMs with fp32 accumulation on CUDA; here on tcgen05 tensor
 * cores (no cuBLAS). bf16 operands, fp32 accumulation, C bf16 (c_dtype 1, round to nearest) or
 * fp32 (c_dtype 0), row-major with leading dimension ldc.
 * ll_gemm_bf16: C[M][N] = A[M][K] . B^T with B [N][K] (b_nk = 1, as F.linear's weight), or
 *   A . B with B [K][N] (b_nk = 0, the input gradient through that weight).
 * ll_gemm_bf16_two_outputs: C0 = A op(B0) and C1 = A op(B1) in one launch (gate and up).
 * ll_gemm_bf16_sum2: C = A0 op(B0) + A1 op(B1), both products in one fp32 accumulator and one
 *   rounding (dG W_g + dU W_u).
 * Leading dimensions in elements, multiples of 8 (16-byte rows); pointers 16-byte aligned;
 * M, N, K >= 1 (K need not be a multiple of 64). Waits inside the kernel are bounded; one that
 * runs out sets a per-device status word that ll_gemm_bf16_status returns (after a stream
 * synchronisation) and clears. */
int ll_gemm_bf16(int M, int N, int K, const void* A, int64_t lda, const void* B, int64_t ldb, int b_nk, void* C,
                 int64_t ldc, int c_dtype, void* stream);
int ll_gemm_bf16_two_outputs(int M, int N, int K, const void* A, int64_t lda, const void* B0, const void* B1,
                             int64_t ldb, int b_nk, void* C0, void* C1, int64_t ldc, int c_dtype, void* stream);
int ll_gemm_bf16_sum2(int M, int N, const void* A0, int K0, int64_t lda0, const void* B0, int64_t ldb0, int b0_nk,
                      const void* A1, int K1, int64_t lda1, const void* B1, int64_t ldb1, int b1_nk, void* C,
                      int64_t ldc, int c_dtype, void* stream);
int ll_gemm_bf16_status(void* stream);

/* ------------------------------------------------------------------ latent RMSNorm
 * The norm between the routed-expert sum and the latent up-projection of the Kimi K3 MoE
 * block (lazy_trainer.py:731-733; RMSNormFunction.forward, trunk_streamer.py:27-31):
 * y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w, x fp32 [N, D], w fp32 [D], y fp32 (y_dtype 0)
 * or bf16 (1); rstd fp32 [N] (optional in the forward) receives rsqrt(mean + eps) per row.
 * The backward gives dL/dx for a frozen w from gy (fp32 or bf16) and the saved rstd. Row sums
 * are reduced in a fixed order: bitwise reproducible. */
int ll_rmsnorm_forward(const float* x, const float* w, int N, int D, float eps, void* y, int y_dtype, float* rstd,
                       void* stream);
int ll_rmsnorm_backward(const float* x, const float* w, const float* rstd, const void* gy, int gy_dtype, int N, int D,
                        float* gx, void* stream);

/* Profiling hook: record events[2i] / events[2i+1] (cudaEvent_t handles) on the launching
 * stream around the i-th grouped-GEMM launch that follows on this thread, for the first n/2
 * launches; n = 0 turns it off. Calling it again restarts at i = 0. */
int ll_profile_gemm_events(void* const* events, int n);

/* Number of kernel launches the last ll_moe_forward / ll_moe_backward / ll_route_topk on this
 * thread made. */
int ll_last_launch_count(void);

/* Profiling hook: record events[i] (cudaEvent_t handles), on the stream of the call in
 * progress, right after the i-th kernel launch of this library that follows on this thread,
 * for the first n launches; n = 0 turns it off, calling it again restarts at i = 0. The time
 * from the previous event (or from one the caller recorded before the call) to events[i] is
 * the i-th kernel's time on the stream. ll_profile_launch_recorded: events recorded so far;
 * ll_profile_launch_name(i): the i-th kernel's name (a static string). */
int ll_profile_launch_events(void* const* events, int n);
int ll_profile_launch_recorded(void);
const char* ll_profile_launch_name(int i);

#ifdef __cplusplus
}
#endif

#endif /* LAZYLORA_B200_H */
