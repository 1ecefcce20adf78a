// Routed-expert layer, forward and manual backward, on B200.
//
// Reference: LazyLoRATrainer._routed_experts_forward / _routed_experts_backward
// (lazy_lora/trainer/lazy_trainer.py:806-880) with _expert_forward (:762-791), the shared
// LoRA adapters (lazy_lora/core/lora_layer.py:104-139, 178-226) and SiTU-GLU
// (lazy_lora/core/situ_activation.py:47-134).
//
// The reference loops over experts; here the (token, expert) pairs are sorted once by a
// stable counting sort (expert ascending, tokens ascending within an expert: the row order
// of `mask.any(-1).nonzero()`), and four grouped tcgen05 GEMMs stream every touched
// expert's MXFP4 bytes exactly once per pass:
//   F1  gate/up = W1/W3 . x      epilogue: + LoRA deltas, SiTU-GLU, saves gate/up, h
//   F2  y = W2 . h               epilogue: * routing weight
//   B1  v = g . W2 (+ LoRA)      epilogue: grad_w partials, SiTU-GLU backward -> dg, du
//   B2  dX = dg . W1 + du . W3   (one accumulator)
// The per-token LoRA algebra (the adapter is shared by all experts of the layer):
//   gate/up delta  s (x A^T) B^T is per token, computed once, added in the F1 epilogue;
//   down delta     sum_e w_e s (h_e A_d^T) B_d^T = s q B_d^T with q = sum_e w_e h_e A_d^T;
//   dA_g = s (Dg B_g)^T X,  dB_g = s Dg^T (X A_g^T)  with Dg = sum_e dg_e per token (up alike);
//   dB_d = s G^T q;  dA_d = s sum_pairs w (g B_d)^T h.
// Combines sum a token's experts in ascending expert order, as index_add_ does; no float
// atomics anywhere, so results are bitwise reproducible.
#include <cub/block/block_scan.cuh>

#include "host_common.cuh"
#include "ops.cuh"
#include "lora_aux.cuh"

namespace ll {

constexpr int kTokBlock = 64;   // tokens per block in the counting sort
// The block-scaled GEMMs' balanced split: for up to kSplitUnits units (8 per CTA at 148 SMs),
// with partial slots for up to kSplitCtas CTAs.
constexpr int kSplitUnits = 1280, kSplitCtas = 160;
// Above this many tokens the LoRA projections x . [A_g; A_u]^T and g . B_d run on the tensor
// cores (project_tc) when x / g are bf16; below, on CUDA cores (skinny).
constexpr int kProjTcMin = 128;

// ----------------------------------------------------------------- counting sort
__global__ void k_count(const int64_t* __restrict__ idx, int T, int k, int E, int* __restrict__ cnt) {
  pdl_wait();
  pdl_launch_next();
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int t0 = blockIdx.x * kTokBlock;
  const int t1 = min(T, t0 + kTokBlock);
  for (int q = t0 * k + threadIdx.x; q < t1 * k; q += blockDim.x) {
    const int64_t e = idx[q];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[(int64_t)blockIdx.x * E + e] = hist[e];
}

// Single block: expert offsets, per-(token block, expert) bases (in place over cnt), and the
// chunk list (experts split into runs of at most nmax rows).
__global__ void __launch_bounds__(1024) k_scan(int* __restrict__ cnt, int nblk, int E, int nmax, int* __restrict__ offsets,
                                               Chunk* __restrict__ chunks, int* __restrict__ n_chunks,
                                               int* __restrict__ chunk_of) {
  pdl_wait();
  pdl_launch_next();
  using Scan = cub::BlockScan<int, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int carry_rows, carry_chunks;
  if (threadIdx.x == 0) { carry_rows = 0; carry_chunks = 0; }
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += 1024) {
    const int e = e0 + threadIdx.x;
    int total = 0;
    if (e < E)
      for (int b = 0; b < nblk; b++) total += cnt[(int64_t)b * E + e];
    const int nch = (total + nmax - 1) / nmax;
    int row_off, ch_off, agg_rows, agg_ch;
    Scan(tmp).ExclusiveSum(total, row_off, agg_rows);
    __syncthreads();
    Scan(tmp).ExclusiveSum(nch, ch_off, agg_ch);
    __syncthreads();
    if (e < E) {
      const int base = carry_rows + row_off;
      offsets[e] = base;
      int run = base;
      for (int b = 0; b < nblk; b++) {
        const int c = cnt[(int64_t)b * E + e];
        cnt[(int64_t)b * E + e] = run;
        run += c;
      }
      const int cb = carry_chunks + ch_off;
      for (int i = 0; i < nch; i++) chunks[cb + i] = Chunk{e, base + i * nmax, min(nmax, total - i * nmax), 0};
      for (int i = 0; i < total; i++) chunk_of[base + i] = cb + i / nmax;
    }
    __syncthreads();
    if (threadIdx.x == 0) { carry_rows += agg_rows; carry_chunks += agg_ch; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[E] = carry_rows;
    *n_chunks = carry_chunks;
  }
}

// Positions of every pair; also, per token, its pairs' positions in ascending expert order.
__global__ void k_scatter(const int64_t* __restrict__ idx, const float* __restrict__ w, int T, int k, int E,
                          const int* __restrict__ base, int* __restrict__ perm_token, int* __restrict__ perm_slot,
                          int* __restrict__ pair_pos, float* __restrict__ tw, int* __restrict__ tok_pos) {
  pdl_wait();
  pdl_launch_next();
  extern __shared__ int es[];   // [kTokBlock * k] expert of each pair, -1 if not routed here
  const int t0 = blockIdx.x * kTokBlock;
  const int t1 = min(T, t0 + kTokBlock);
  const int np = (t1 - t0) * k;
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int64_t e = idx[(int64_t)t0 * k + i];
    es[i] = (e >= 0 && e < E) ? (int)e : -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int e = es[i];
    const int q = t0 * k + i;
    if (e < 0) {
      pair_pos[q] = -1;
      continue;
    }
    int rank = 0;
    for (int j = 0; j < i; j++) rank += (es[j] == e);
    const int pos = base[(int64_t)blockIdx.x * E + e] + rank;
    pair_pos[q] = pos;
    perm_token[pos] = q / k;
    perm_slot[pos] = q % k;
    tw[pos] = w[q];
  }
  __syncthreads();
  // per-token ascending-expert order of positions (insertion sort over k <= 32 slots)
  for (int tl = threadIdx.x; tl < t1 - t0; tl += blockDim.x) {
    int ee[32], pp[32];
    int n = 0;
    for (int s = 0; s < k; s++) {
      const int e = es[tl * k + s];
      if (e < 0) continue;
      const int pos = pair_pos[(int64_t)(t0 + tl) * k + s];
      int j = n++;
      while (j > 0 && ee[j - 1] > e) { ee[j] = ee[j - 1]; pp[j] = pp[j - 1]; j--; }
      ee[j] = e;
      pp[j] = pos;
    }
    for (int s = 0; s < k; s++) tok_pos[(int64_t)(t0 + tl) * k + s] = s < n ? pp[s] : -1;
  }
}

// The three kernels above in one block, for a batch of at most kTokBlock tokens (nblk == 1),
// with the same outputs bit for bit (the per-block bases of k_scan are the expert offsets
// here); also clears perm_token (-1), the status word and n_zero ints at `zero` (the split
// GEMMs' arrival counters), so that a few-token forward starts with no copy or memset.
__global__ void __launch_bounds__(1024) k_plan_small(const int64_t* __restrict__ idx, const float* __restrict__ w,
                                                     int T, int k, int E, int nmax, int* __restrict__ offsets,
                                                     Chunk* __restrict__ chunks, int* __restrict__ n_chunks,
                                                     int* __restrict__ perm_token, int* __restrict__ perm_slot,
                                                     int* __restrict__ pair_pos, float* __restrict__ tw,
                                                     int* __restrict__ tok_pos, int* __restrict__ chunk_of,
                                                     DevStatus* __restrict__ st, int* __restrict__ zero,
                                                     int n_zero) {
  pdl_wait();
  pdl_launch_next();
  using Scan = cub::BlockScan<int, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int carry_rows, carry_chunks;
  extern __shared__ int sm[];
  int* hist = sm;          // [E] counts, then each expert's first position
  int* es = sm + E;        // [T k] expert of each pair, -1 if not routed here
  const int np = T * k;
  if (threadIdx.x == 0) {
    carry_rows = 0;
    carry_chunks = 0;
    if (st) *st = DevStatus{0, 0, 0, 0};
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  for (int i = threadIdx.x; i < np; i += blockDim.x) perm_token[i] = -1;
  for (int i = threadIdx.x; i < n_zero; i += blockDim.x) zero[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int64_t e = idx[i];
    const bool ok = e >= 0 && e < E;
    es[i] = ok ? (int)e : -1;
    if (ok) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += 1024) {
    const int e = e0 + threadIdx.x;
    const int total = e < E ? hist[e] : 0;
    const int nch = (total + nmax - 1) / nmax;
    int row_off, ch_off, agg_rows, agg_ch;
    Scan(tmp).ExclusiveSum(total, row_off, agg_rows);
    __syncthreads();
    Scan(tmp).ExclusiveSum(nch, ch_off, agg_ch);
    __syncthreads();
    if (e < E) {
      const int base = carry_rows + row_off;
      offsets[e] = base;
      hist[e] = base;
      const int cb = carry_chunks + ch_off;
      for (int i = 0; i < nch; i++) chunks[cb + i] = Chunk{e, base + i * nmax, min(nmax, total - i * nmax), 0};
      for (int i = 0; i < total; i++) chunk_of[base + i] = cb + i / nmax;
    }
    __syncthreads();
    if (threadIdx.x == 0) { carry_rows += agg_rows; carry_chunks += agg_ch; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[E] = carry_rows;
    *n_chunks = carry_chunks;
  }
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const int e = es[i];
    if (e < 0) {
      pair_pos[i] = -1;
      continue;
    }
    int rank = 0;
    for (int j = 0; j < i; j++) rank += (es[j] == e);
    const int pos = hist[e] + rank;
    pair_pos[i] = pos;
    perm_token[pos] = i / k;
    perm_slot[pos] = i % k;
    tw[pos] = w[i];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    int ee[32], pp[32];
    int n = 0;
    for (int sl = 0; sl < k; sl++) {
      const int e = es[t * k + sl];
      if (e < 0) continue;
      const int pos = pair_pos[(int64_t)t * k + sl];
      int j = n++;
      while (j > 0 && ee[j - 1] > e) { ee[j] = ee[j - 1]; pp[j] = pp[j - 1]; j--; }
      ee[j] = e;
      pp[j] = pos;
    }
    for (int sl = 0; sl < k; sl++) tok_pos[(int64_t)t * k + sl] = sl < n ? pp[sl] : -1;
  }
}

// Per valid pair: one power-of-two scale for both rows of dg / du, fp16 copies for B2.
__global__ void k_pair_rows_half(const float* __restrict__ DG, const float* __restrict__ DU, int f,
                                 const int* __restrict__ n_valid, __half* __restrict__ DGh, __half* __restrict__ DUh,
                                 float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_next();
  const int p = blockIdx.x;
  if (p >= *n_valid) return;
  __shared__ float red[32];
  __shared__ float sh;
  float mx = 0.f;
  for (int m = threadIdx.x; m < f; m += blockDim.x)
    mx = fmaxf(mx, fmaxf(fabsf(DG[(int64_t)p * f + m]), fabsf(DU[(int64_t)p * f + m])));
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); i++) m = fmaxf(m, red[i]);
    const int e = row_scale_exp(m);
    sh = ldexpf(1.f, e);
    inv[p] = ldexpf(1.f, -e);
  }
  __syncthreads();
  for (int m = threadIdx.x; m < f; m += blockDim.x) {
    DGh[(int64_t)p * f + m] = __float2half_rn(DG[(int64_t)p * f + m] * sh);
    DUh[(int64_t)p * f + m] = __float2half_rn(DU[(int64_t)p * f + m] * sh);
  }
}

// D{g,u}[t][m] = sum over the token's pairs (ascending expert) of D{G,U}[pos][m]
__global__ void k_token_sum(const int* __restrict__ tok_pos, const float* __restrict__ DG, const float* __restrict__ DU,
                            int T, int k, int f, float* __restrict__ Dg, float* __restrict__ Du) {
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.y;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= f) return;
  float ag = 0.f, au = 0.f;
  for (int j = 0; j < k; j++) {
    const int p = tok_pos[(int64_t)t * k + j];
    if (p < 0) break;
    ag += DG[(int64_t)p * f + m];
    au += DU[(int64_t)p * f + m];
  }
  Dg[(int64_t)t * f + m] = ag;
  Du[(int64_t)t * f + m] = au;
}

// The two passes over the backward's per-pair gradients of the gate / up pre-activations in
// one: block per token; for each of its pairs in ascending expert order, the pair rows DG, DU
// are read once, converted to fp16 with the pair's power-of-two row scale (the B2 GEMM's
// activation, as k_pair_rows_half) and added to the token sums Dg, Du (as k_token_sum, same
// order, so both results are bitwise those of the two-kernel path). f = 1024, 2048 or 4096.
constexpr int kPTThreads = 256;
template <int NV>   // float4 per thread per row: f = 1024 NV
__global__ void __launch_bounds__(kPTThreads) k_pair_rows_tokens(
    const int* __restrict__ tok_pos, const float* __restrict__ DG, const float* __restrict__ DU, int k, int f,
    __half* __restrict__ DGh, __half* __restrict__ DUh, float* __restrict__ inv, float* __restrict__ Dg,
    float* __restrict__ Du) {
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.x;
  __shared__ float red[kPTThreads / 32];
  __shared__ float sh;
  float4 ag[NV], au[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) ag[i] = au[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < k; j++) {
    const int p = tok_pos[(int64_t)t * k + j];
    if (p < 0) break;
    const float4* g4 = reinterpret_cast<const float4*>(DG + (int64_t)p * f);
    const float4* u4 = reinterpret_cast<const float4*>(DU + (int64_t)p * f);
    float4 gv[NV], uv[NV];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      {
        gv[i] = g4[threadIdx.x + i * kPTThreads];
        uv[i] = u4[threadIdx.x + i * kPTThreads];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(gv[i].x), fabsf(gv[i].y)), fmaxf(fabsf(gv[i].z), fabsf(gv[i].w))));
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(uv[i].x), fabsf(uv[i].y)), fmaxf(fabsf(uv[i].z), fabsf(uv[i].w))));
      }
    }
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = 0.f;
      for (int i = 0; i < kPTThreads / 32; i++) m = fmaxf(m, red[i]);
      const int e = row_scale_exp(m);
      sh = ldexpf(1.f, e);
      inv[p] = ldexpf(1.f, -e);
    }
    __syncthreads();
    const float scl = sh;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      {
        const int64_t o = (int64_t)p * f + 4 * (threadIdx.x + i * kPTThreads);
        const __half2 g01 = __floats2half2_rn(gv[i].x * scl, gv[i].y * scl);
        const __half2 g23 = __floats2half2_rn(gv[i].z * scl, gv[i].w * scl);
        const __half2 u01 = __floats2half2_rn(uv[i].x * scl, uv[i].y * scl);
        const __half2 u23 = __floats2half2_rn(uv[i].z * scl, uv[i].w * scl);
        *reinterpret_cast<uint2*>(DGh + o) = make_uint2(*reinterpret_cast<const uint32_t*>(&g01),
                                                        *reinterpret_cast<const uint32_t*>(&g23));
        *reinterpret_cast<uint2*>(DUh + o) = make_uint2(*reinterpret_cast<const uint32_t*>(&u01),
                                                        *reinterpret_cast<const uint32_t*>(&u23));
        ag[i].x += gv[i].x; ag[i].y += gv[i].y; ag[i].z += gv[i].z; ag[i].w += gv[i].w;
        au[i].x += uv[i].x; au[i].y += uv[i].y; au[i].z += uv[i].z; au[i].w += uv[i].w;
      }
    }
    __syncthreads();                             // sh and red are rewritten by the next pair
  }
#pragma unroll
  for (int i = 0; i < NV; i++) {
    {
      reinterpret_cast<float4*>(Dg + (int64_t)t * f)[threadIdx.x + i * kPTThreads] = ag[i];
      reinterpret_cast<float4*>(Du + (int64_t)t * f)[threadIdx.x + i * kPTThreads] = au[i];
    }
  }
}

__global__ void k_grad_w(const int* __restrict__ pair_pos, const float* __restrict__ parts, int nparts, int P, int Tk,
                         float* __restrict__ grad_w) {
  pdl_wait();
  pdl_launch_next();
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= Tk) return;
  const int pos = pair_pos[q];
  float s = 0.f;
  if (pos >= 0)
    for (int i = 0; i < nparts; i++) s += parts[(int64_t)i * P + pos];
  grad_w[q] = s;
}

// out = s * sum_seg part, stored [r][C] or transposed [C][r]
__global__ void k_outer_reduce(const float* __restrict__ part, int nseg, int r, int C, float s, bool transposed,
                               float* __restrict__ out) {
  pdl_wait();
  pdl_launch_next();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)r * C) return;
  const int rr = (int)(i / C), c = (int)(i % C);
  const float acc = sum_splits(part + i, (int64_t)r * C, nseg);
  if (transposed) out[(int64_t)c * r + rr] = s * acc;
  else out[i] = s * acc;
}

// ------------------------------------------------------------------- workspace
struct LayerWs {
  DevStatus* st;
  int* cnt;
  int* offsets;
  Chunk* chunks;
  int* n_chunks;
  int* perm_token;
  int* perm_slot;
  int* pair_pos;
  int* tok_pos;
  int* chunk_of;      // [P] chunk of each sorted row
  float* tw;
  float* xinv;
  __half* xh;
  // block-scaled forward operands: the activation terms of the pair rows (x for F1, h for F2),
  // 3 E4M3 terms ([3][P][K] bytes) or 4 packed E2M1 terms ([4][P][K/2]), their scales (E4M3: row
  // scales [3][P]; E2M1: block scale bytes [4][P][K/32], laid out per chunk and stage in *sfb)
  uint8_t* xq;
  float* xinv3;
  uint8_t* xsfb;
  uint8_t* hq;
  float* hinv3;
  uint8_t* hsfb;
  int max_chunks;
  float* xa_g;
  float* xa_u;
  float* dlt_g;
  float* dlt_u;
  float* G;
  float* U;
  __half* H;
  float* z;
  float* q;
  float* Y;
  // backward
  float* ginv;
  __half* gh;
  float* gB;
  float* lora_d;
  float* gw_part;
  float* DG;
  float* DU;
  float* rinv;
  __half* DGh;
  __half* DUh;
  float* Dg;
  float* Du;
  float* hg;
  float* hu;
  float* opart;
  float* skpart;
  size_t skpart_floats;
  int nmax;
  int nseg_max;
  // the block-scaled GEMMs' balanced split (few tokens only): partial slots, and the F1 then F2
  // arrival counters (4 per unit each), cleared by k_plan_small
  float* split_part;
  int* split_cnt;
  int split_units;
  // the tensor-core LoRA projections x . [A_g; A_u]^T and g . B_d (more than 128 tokens)
  void* proj_ws;
  size_t proj_bytes;
};

// Token rows per chunk (the MMA N): the smallest tile that holds most experts' rows in one
// chunk, from the mean valid (token, expert) pairs per expert (L->rows_hint when the caller
// knows how many of the T * k slots are routed here, else T * k).
static int choose_nmax(const ll_moe_layer* L, int T, int k) {
  const int64_t slots = (int64_t)T * k;
  const int64_t pairs = L->rows_hint > 0 && L->rows_hint < slots ? L->rows_hint : slots;
  const double mean = (double)pairs / (L->E > 0 ? L->E : 1);
  // the narrowest tile that holds nearly every expert's rows in one chunk (a second chunk
  // re-reads the expert's weights): Poisson-like counts exceed 16 rows for ~1% of experts at a
  // mean of 9, 32 rows for ~0.1% at 18, 64 rows for ~1% at 48
  static const int forced = [] {          // LL_NMAX: a fixed tile width (16, 32, 64 or 128), for tuning
    const char* e = getenv("LL_NMAX");
    const int v = e ? atoi(e) : 0;
    return (v == 16 || v == 32 || v == 64 || v == 128) ? v : 0;
  }();
  if (forced) return forced;
  // a token takes an expert at most once: up to 4 tokens, no expert has more than 4 rows
  if (T <= 4) return 4;
  return mean <= 10.0 ? 16 : mean <= 22.0 ? 32 : (mean <= 48.0 ? 64 : 128);
}

static size_t layer_layout(void* base, const ll_moe_layer* L, int T, int k, LayerWs* out) {
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int64_t P = (int64_t)T * k;
  const int nmax = choose_nmax(L, T, k);
  const int nblk = (T + kTokBlock - 1) / kTokBlock;
  const int nseg_max = 64;
  Carver c(base);
  LayerWs w{};
  w.nmax = nmax;
  w.nseg_max = nseg_max;
  w.st = c.take<DevStatus>(1);
  w.cnt = c.take<int>((size_t)nblk * E);
  w.offsets = c.take<int>(E + 1);
  w.chunks = c.take<Chunk>(E + P / 16 + 2);     // enough for any nmax >= 16
  w.n_chunks = c.take<int>(1);
  w.perm_token = c.take<int>(P);
  w.perm_slot = c.take<int>(P);
  w.pair_pos = c.take<int>(P);
  w.tok_pos = c.take<int>(P);
  w.chunk_of = c.take<int>(P);
  w.tw = c.take<float>(P);
  w.xinv = c.take<float>(P);
  w.xh = c.take<__half>(P * d);
  {
    const int max_chunks = E + (int)(P / 16) + 2;       // the chunk list's capacity
    w.max_chunks = max_chunks;
    w.xq = c.take<uint8_t>((size_t)3 * P * d);          // 3 E4M3 terms or 4 E2M1 terms (2 P d bytes)
    w.xinv3 = c.take<float>((size_t)3 * P);
    w.xsfb = c.take<uint8_t>((size_t)max_chunks * (d / 128) * kBsSfBlock);
    w.hq = c.take<uint8_t>((size_t)3 * P * f);
    w.hinv3 = c.take<float>((size_t)3 * P);
    w.hsfb = c.take<uint8_t>((size_t)max_chunks * (f / 128) * kBsSfBlock);
  }
  w.xa_g = c.take<float>((size_t)T * r);
  w.xa_u = c.take<float>((size_t)T * r);
  w.dlt_g = c.take<float>((size_t)T * f);
  w.dlt_u = c.take<float>((size_t)T * f);
  w.G = c.take<float>(P * f);
  w.U = c.take<float>(P * f);
  w.H = c.take<__half>(P * f);
  w.z = c.take<float>(P * r);
  w.q = c.take<float>((size_t)T * r);
  w.Y = c.take<float>(P * d);
  w.ginv = c.take<float>(P);
  w.gh = c.take<__half>(P * d);
  w.gB = c.take<float>((size_t)T * r);
  w.lora_d = c.take<float>((size_t)T * f);
  w.gw_part = c.take<float>((size_t)((f + 127) / 128) * 4 * P);
  w.DG = c.take<float>(P * f);
  w.DU = c.take<float>(P * f);
  w.rinv = c.take<float>(P);
  w.DGh = c.take<__half>(2 * P * f);            // DG rows then DU rows: one 4-D tensor map reads both
  w.DUh = w.DGh ? w.DGh + P * f : nullptr;
  w.Dg = c.take<float>((size_t)T * f);
  w.Du = c.take<float>((size_t)T * f);
  w.hg = c.take<float>((size_t)T * r);
  w.hu = c.take<float>((size_t)T * r);
  w.opart = c.take<float>((size_t)nseg_max * r * (d > f ? d : f));
  {  // split-K partials of the skinny products: nsplit * mblocks * nblocks <= 4 * SMs +
     // mblocks * nblocks blocks of at most 8192 outputs (BM * NC); SMs <= 160
    const int64_t rows = P > T ? P : T;
    w.skpart_floats = (size_t)4 * 160 * 8192 + (size_t)(rows + 256) * (2 * r + 32);
    w.skpart = c.take<float>(w.skpart_floats);
  }
  if (T > kProjTcMin) {
    w.proj_bytes = project_tc_bytes(T, d, 2 * r);
    w.proj_ws = c.take<uint8_t>(w.proj_bytes);
  }
  if (T <= kTokBlock && nmax <= 64) {   // the one-block plan clears the counters
    w.split_units = kSplitUnits;
    w.split_part = c.take<float>((size_t)2 * kSplitCtas * 2 * nmax * 128);
    w.split_cnt = c.take<int>((size_t)2 * 4 * kSplitUnits);
  }
  if (out) *out = w;
  return c.off + 256;
}

// A second stream (non-blocking) with a fork and a join event, one per device and host thread,
// made on first use: work of a call that does not depend on the call's earlier launches runs
// there, ordered by the events (captured into a graph as a parallel branch).
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
static int side_stream(SideStream** out) {
  constexpr int kMaxDev = 16;
  static thread_local SideStream per_dev[kMaxDev];
  int dev = 0;
  LL_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDev) return LL_ERR_ARG;
  SideStream& ss = per_dev[dev];
  if (!ss.s) {
    LL_CUDA(cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking));
    LL_CUDA(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming));
    LL_CUDA(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming));
  }
  *out = &ss;
  return LL_OK;
}

// The forward reads the weights as stored; only the backward needs the transposed copies.
static int validate(const ll_moe_layer* L, int T, int k, bool backward) {
  if (!L || T <= 0 || k <= 0 || k > 32) return LL_ERR_ARG;
  if (L->d <= 0 || L->f <= 0 || L->d % 128 || L->f % 128 || L->E <= 0 || L->E > 8192) return LL_ERR_ARG;
  if (L->r <= 0 || L->r > kExMaxR) return LL_ERR_ARG;
  if (L->s13_stride < L->d / 32 || L->s13_stride % 16 || L->s2_stride < L->f / 32 || L->s2_stride % 16) return LL_ERR_ARG;
  if (!L->w1p || !L->w1s || !L->w3p || !L->w3s || !L->w2p || !L->w2s || !L->beta) return LL_ERR_ARG;
  if (!L->A_g || !L->B_g || !L->A_u || !L->B_u || !L->A_d || !L->B_d) return LL_ERR_ARG;
  if (!L->w1sf || !L->w3sf || !L->w2sf) return LL_ERR_ARG;
  if (backward && (!L->w1t || !L->w3t || !L->w2t || !L->s1t || !L->s3t || !L->s2t)) return LL_ERR_ARG;
  return LL_OK;
}

template <int EPI, int NMAT, int NB, bool COLSCALE>
static int gemm_nmax(int nmax, const CUtensorMap* pk, const CUtensorMap* sc, const CUtensorMap* act, const GemmArgs& a,
                     cudaStream_t s) {
  if (nmax == 16) return launch_gemm<EPI, NMAT, NB, COLSCALE, 16>(pk, sc, act, a, s);
  if (nmax == 32) return launch_gemm<EPI, NMAT, NB, COLSCALE, 32>(pk, sc, act, a, s);
  if (nmax == 64) return launch_gemm<EPI, NMAT, NB, COLSCALE, 64>(pk, sc, act, a, s);
  return launch_gemm<EPI, NMAT, NB, COLSCALE, 128>(pk, sc, act, a, s);
}

// Stages the block-scaled GEMMs prefetch weight tiles into L2 ahead of their loads
// (LL_BS_PREFETCH_STAGES, for tuning; off by default: measured slower at 4, 8 and 16 stages
// on configs[1], the prefetches competing with the loads for L2).
static int bs_prefetch_stages() {
  static const int v = [] {
    const char* e = getenv("LL_BS_PREFETCH_STAGES");
    return e ? atoi(e) : 0;
  }();
  return v;
}

// Unit counts up to which F1 / F2 run the balanced split (from one unit a CTA up). Measured on
// F1 at 352 units (2.4 a CTA, T = 4) 86 -> 78 us; F1 at 1152 units (7.8 a CTA) 211
// -> 220 us and F2 at 224 / 616 units (16-stage units) 26 -> 28 / 45 -> 47 us, slower; so F1 up
// to 4 units a CTA and not F2. LL_BS_SPLIT_F1 / LL_BS_SPLIT_F2 override (for tuning; 0 = off;
// at most kSplitUnits).
static int bs_split_units(int which) {
  static const int v[2] = {[] {
                             const char* e = getenv("LL_BS_SPLIT_F1");
                             return e ? atoi(e) : -1;
                           }(),
                           [] {
                             const char* e = getenv("LL_BS_SPLIT_F2");
                             return e ? atoi(e) : 0;
                           }()};
  const int u = v[which] >= 0 ? v[which] : 4 * device_info().sms;
  return std::min(u, kSplitUnits);
}

// The token-tile width of the fp16 dequant GEMMs: the layer's, at least 16 (four-row chunks run
// in 16-row tiles there).
static int dq_nmax(const LayerWs& W) { return W.nmax < 16 ? 16 : W.nmax; }

// The block-scaled forward GEMM kind for a token-tile width: E2M1 activation terms up to 32
// rows, E4M3 terms at 64 rows, none (fp16 dequant path) at 128.
static int bs_kind(int nmax) { return nmax <= 32 ? BS_FP4 : nmax <= 64 ? BS_FP8 : -1; }

template <int EPI>
static int bs_launch(int kind, int nmax, const CUtensorMap* a, const CUtensorMap* b, const BsArgs& args,
                     cudaStream_t s) {
  if (kind == BS_FP4)
    return nmax == 4    ? launch_bs_gemm<EPI, 2, 4, BS_FP4>(a, b, args, s)
           : nmax == 16 ? launch_bs_gemm<EPI, 2, 16, BS_FP4>(a, b, args, s)
                        : launch_bs_gemm<EPI, 2, 32, BS_FP4>(a, b, args, s);
  return launch_bs_gemm<EPI, 2, 64, BS_FP8>(a, b, args, s);
}

// The activation operand of a block-scaled GEMM: the rows as the kind's terms (tok_pos given:
// the T token rows written to their pair rows; else pair rows < *n_valid), and for BS_FP4 their
// block scales laid out per chunk and stage, plus the tensor maps of the terms.
static int bs_operand(int kind, const LayerWs& W, const void* src, int src_dtype, int src_rows, const int* tok_pos,
                      int k, const int* n_valid, int K, int64_t P, uint8_t* q, float* inv3, uint8_t* sfb,
                      CUtensorMap* maps, BsArgs& a, cudaStream_t s) {
  if (kind == BS_FP4) {
    LL_TRY(launch_rows_to_e2m1x4(src, src_dtype, src_rows, tok_pos, k, n_valid, K, P, q, W.chunks, W.chunk_of,
                                 W.nmax, sfb, s));
    LL_TRY(make_e2m1x4_maps(maps, W.nmax < 16 ? 1 : W.nmax / 16, q, P, K, W.nmax < 16 ? 4 : 16));
    a.sfb = sfb;
  } else {
    LL_TRY(launch_rows_to_e4m3x3(src, src_dtype, src_rows, tok_pos, k, n_valid, K, P, q, inv3, s));
    LL_TRY(make_e4m3x3_maps(maps, W.nmax / 16, q, P, K));
    a.inv3 = inv3;
  }
  return LL_OK;
}

// C0 (and C1) = alpha * A[M][K] . B, with B given as rows ([N][K], split over B0 / B1 at N0)
// or columns ([K][N]); split-K partials in `part` (room for part_floats floats), summed in a
// fixed order.
int skinny(const void* A, int adt, bool brows, int M, int K, const float* B0, const float* B1, int N0, int N,
           float alpha, float* C0, float* C1, float* part, size_t part_floats, cudaStream_t s) {
  if (K % 8 || M <= 0 || N <= 0) return LL_ERR_ARG;
  const bool al16 = ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B0) |
                      reinterpret_cast<uintptr_t>(B1 ? B1 : B0)) & 15) == 0;
  if (brows && M <= 128 && al16) {        // few rows: one launch, no partials
#define LL_GV(ADT, MR) \
  return launch_pdl("k_gemv_rows", k_gemv_rows<ADT, MR>, dim3(N, (M + MR - 1) / MR), dim3(256), 0, s, A, M, K, B0, B1, \
                    N0, N, alpha, C0, C1)
#define LL_GVM(ADT) \
  do {                                     \
    if (M == 1) LL_GV(ADT, 1);             \
    if (M <= 4) LL_GV(ADT, 4);             \
    LL_GV(ADT, 16);                        \
  } while (0)
    if (adt == 0) LL_GVM(0);
    if (adt == 1) LL_GVM(1);
    LL_GVM(2);
#undef LL_GVM
#undef LL_GV
  }
  if (part_floats < (size_t)M * N) return LL_ERR_ARG;
  const bool nc16 = N <= 16;
  const int BM = nc16 ? SkinnyCfg<16>::BM : SkinnyCfg<32>::BM, NC = nc16 ? 16 : 32;
  const int mblocks = (M + BM - 1) / BM, nblocks = (N + NC - 1) / NC;
  // about four blocks per SM, split over K (a block's 256 threads keep ~1 K-step in flight, so
  // the product is occupancy-bound below that)
  int nsplit = (4 * device_info().sms + mblocks * nblocks - 1) / (mblocks * nblocks);
  nsplit = std::max(1, std::min(nsplit, (K + kSkBK - 1) / kSkBK));
  nsplit = std::min<int64_t>(nsplit, (int64_t)(part_floats / ((size_t)M * N)));
  const int kc = ((K + nsplit - 1) / nsplit + kSkBK - 1) / kSkBK * kSkBK;
  nsplit = (K + kc - 1) / kc;
  dim3 grid(mblocks, nblocks, nsplit);
#define LL_SK(ADT, BR)                                                                             \
  do {                                                                                             \
    if (nc16) LL_TRY(launch_pdl("k_skinny", k_skinny<ADT, BR, 16>, grid, dim3(256), 0, s, A, M, K, K, B0, B1, N0, \
                                N, kc, part));                                                       \
    else LL_TRY(launch_pdl("k_skinny", k_skinny<ADT, BR, 32>, grid, dim3(256), 0, s, A, M, K, K, B0, B1, N0, N,   \
                           kc, part));                                                               \
  } while (0)
  if (brows) {
    if (adt == 0) LL_SK(0, true); else if (adt == 1) LL_SK(1, true); else LL_SK(2, true);
  } else {
    if (adt == 0) LL_SK(0, false); else if (adt == 1) LL_SK(1, false); else LL_SK(2, false);
  }
#undef LL_SK
  const int64_t n = (int64_t)M * N;
  return launch_pdl("k_skinny_reduce", k_skinny_reduce, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part,
                    nsplit, M, N, N0, alpha, C0, C1);
}

// Rank-r expand with the optional ascending-expert sum of per-pair rows (see k_expand).
int expand(bool rrows, const int* tok_pos, const float* Y, int k, int T, int C, int r, float alpha, const float* L0,
           const float* R0, const float* L1, const float* R1, float* out, cudaStream_t s, float* out1,
           const float* qtw, const float* qz, float* q_out) {
  if (C % 4 || r > kExMaxR || k > 32) return LL_ERR_ARG;
  if (out1 && (!L1 || !R1)) return LL_ERR_ARG;
  if (qz && (!tok_pos || !qtw)) return LL_ERR_ARG;
  dim3 grid((C + kExCols - 1) / kExCols, (T + kExTok - 1) / kExTok, out1 ? 2 : 1);
  const bool hasy = Y != nullptr, two = L1 != nullptr && !out1;
  const int smem = r * kExPitch * (int)sizeof(float);  // <= 129 KB at r = 64
  auto attr = [&](const void* f) { return set_smem_attr(f, smem); };
#define LL_EX(RR, HY, TW)                                                                                   \
  do {                                                                                                      \
    LL_TRY(attr(reinterpret_cast<const void*>(k_expand<RR, HY, TW>)));                                     \
    LL_TRY(launch_pdl("k_expand", k_expand<RR, HY, TW>, grid, dim3(kExThreads), smem, s, tok_pos, Y, k, T, C, r,   \
                      alpha, L0, R0, L1, R1, out, out1, qtw, qz, q_out));                                   \
  } while (0)
  if (rrows) {
    if (hasy) { if (two) LL_EX(true, true, true); else LL_EX(true, true, false); }
    else { if (two) LL_EX(true, false, true); else LL_EX(true, false, false); }
  } else {
    if (hasy) { if (two) LL_EX(false, true, true); else LL_EX(false, true, false); }
    else { if (two) LL_EX(false, false, true); else LL_EX(false, false, false); }
  }
#undef LL_EX
  return LL_OK;
}

// out = s * sum_n Pm(n, :)^T Q[n][:], stored [r][C] or transposed [C][r]
int outer(const float* Pm, const int* perm_token, const float* tw, const void* Q, int qdt, int N, const int* n_dev,
          int C, int r, float sc, bool transposed, float* part, int nseg_max, float* out, cudaStream_t s) {
  if (C % 4 || r <= 0) return LL_ERR_ARG;
  const int cblocks = (C + kOuCW - 1) / kOuCW, zb = (r + kOuRB - 1) / kOuRB;
  // about four blocks per SM, two waves of the two that fit (measured against 2, 3, 6 and 8);
  // each warp gets at least one batch of rows
  int nseg = (4 * device_info().sms + cblocks * zb - 1) / (cblocks * zb);
  nseg = std::max(1, std::min(nseg, nseg_max));
  nseg = std::min(nseg, std::max(1, N / (8 * kOuNB)));
  dim3 grid(cblocks, nseg, zb);
  const int smem = 8 * kOuRB * 32 * (int)sizeof(float4);
  const bool pg = perm_token != nullptr;
#define LL_OU(QD, PG)                                                                                \
  do {                                                                                               \
    LL_TRY(set_smem_attr(reinterpret_cast<const void*>(k_outer8<QD, PG>), smem));                   \
    LL_TRY(launch_pdl("k_outer8", k_outer8<QD, PG>, grid, dim3(256), smem, s, Pm, perm_token, tw, Q, N, n_dev, C, \
                      r, nseg, part));                                                               \
  } while (0)
  if (pg) {
    if (qdt == 0) LL_OU(0, true); else if (qdt == 1) LL_OU(1, true); else LL_OU(2, true);
  } else {
    if (qdt == 0) LL_OU(0, false); else if (qdt == 1) LL_OU(1, false); else LL_OU(2, false);
  }
#undef LL_OU
  const int64_t n = (int64_t)r * C;
  return launch_pdl("k_outer_reduce", k_outer_reduce, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part, nseg,
                    r, C, sc, transposed, out);
}

}  // namespace ll

using namespace ll;

extern "C" {

size_t ll_mxfp4_transposed_bytes(int E, int R, int C, int which) {
  if (E <= 0 || R <= 0 || C <= 0) return 0;
  return which == 0 ? (size_t)E * R * C / 2 : (size_t)E * (C / 32) * R * 2;
}

int ll_moe_prepare(const ll_moe_layer* L, int32_t* beta_out, void* stream) {
  if (!L || !beta_out || L->E <= 0 || L->d <= 0 || L->f <= 0 || L->d % 128 || L->f % 128) return LL_ERR_ARG;
  const int n_t = !!L->w1t + !!L->w3t + !!L->w2t + !!L->s1t + !!L->s3t + !!L->s2t;
  if (n_t != 0 && n_t != 6) return LL_ERR_ARG;
  LL_STREAM(stream);
  const int E = L->E, d = L->d, f = L->f;
  LL_TRY(launch_prepare_beta(L->w1s, L->w3s, E, f, d, L->s13_stride, beta_out, 0, s));
  LL_TRY(launch_prepare_beta(L->w2s, nullptr, E, d, f, L->s2_stride, beta_out, 1, s));
  if (L->w1sf || L->w3sf || L->w2sf) {        // the forward's scale blocks
    if (!L->w1sf || !L->w3sf || !L->w2sf) return LL_ERR_ARG;
    auto cw = [](const uint8_t* p) { return const_cast<uint8_t*>(p); };
    LL_TRY(launch_prepare_sfa(L->w1s, L->s13_stride, E, f, d, cw(L->w1sf), s));
    LL_TRY(launch_prepare_sfa(L->w3s, L->s13_stride, E, f, d, cw(L->w3sf), s));
    LL_TRY(launch_prepare_sfa(L->w2s, L->s2_stride, E, d, f, cw(L->w2sf), s));
  }
  if (n_t == 0) return LL_OK;                 // forward-only use: no transposed copies
  auto cw = [](const uint8_t* p) { return const_cast<uint8_t*>(p); };
  auto ch = [](const uint16_t* p) { return reinterpret_cast<__half*>(const_cast<uint16_t*>(p)); };
  LL_TRY(launch_transpose_mxfp4(L->w1p, L->w1s, L->s13_stride, E, f, d, beta_out, 0, cw(L->w1t), ch(L->s1t), s));
  LL_TRY(launch_transpose_mxfp4(L->w3p, L->w3s, L->s13_stride, E, f, d, beta_out, 0, cw(L->w3t), ch(L->s3t), s));
  LL_TRY(launch_transpose_mxfp4(L->w2p, L->w2s, L->s2_stride, E, d, f, beta_out, 1, cw(L->w2t), ch(L->s2t), s));
  return LL_OK;
}

size_t ll_mxfp4_sf_bytes(int E, int R, int C) {
  if (E <= 0 || R <= 0 || C <= 0 || R % 128 || C % 128) return 0;
  return (size_t)E * R * C / 32;
}

size_t ll_moe_workspace_bytes(const ll_moe_layer* L, int T, int k) {
  if (!L || T <= 0 || k <= 0) return 0;
  return layer_layout(nullptr, L, T, k, nullptr);
}

// The forward; with norm_w, the final combine also RMS-normalises each token's row (the latent
// block's routed_expert_norm) into normed (bf16) and rstd.
static int moe_forward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx,
                       const float* w, float* out, const float* norm_w, float eps, void* normed, float* rstd, void* ws,
                       size_t ws_bytes, void* stream) {
  LL_TRY(validate(L, T, k, false));
  if (!x || !idx || !w || !out || !ws || (x_dtype != 0 && x_dtype != 1)) return LL_ERR_ARG;
  if (norm_w && (!normed || !rstd || (reinterpret_cast<uintptr_t>(norm_w) | reinterpret_cast<uintptr_t>(normed)) % 8))
    return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_moe_workspace_bytes(L, T, k)) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int P = T * k;
  const int nblk = (T + kTokBlock - 1) / kTokBlock;
  g_launch_count = 0;

  // The LoRA gate / up deltas depend on x alone: they run on a side stream beside the sort and
  // the operand conversion, joined before F1.
  SideStream* ss = nullptr;
  LL_TRY(side_stream(&ss));
  if (nblk > 1) LL_TRY(reset_status(W.st, s));   // before the fork: the side branch may report to it
  LL_CUDA(cudaEventRecord(ss->fork, s));
  LL_CUDA(cudaStreamWaitEvent(ss->s, ss->fork, 0));
  g_launch_stream = ss->s;
  if (W.proj_ws && x_dtype == 1)
    LL_TRY(project_tc(x, T, d, L->A_g, L->A_u, false, r, W.xa_g, W.xa_u, W.proj_ws, W.proj_bytes, W.st, ss->s));
  else
    LL_TRY(skinny(x, x_dtype, true, T, d, L->A_g, L->A_u, r, 2 * r, 1.f, W.xa_g, W.xa_u, W.skpart, W.skpart_floats,
                  ss->s));
  LL_TRY(expand(false, nullptr, nullptr, k, T, f, r, L->lora_scaling, W.xa_g, L->B_g, W.xa_u, L->B_u, W.dlt_g, ss->s,
                W.dlt_u));
  LL_CUDA(cudaEventRecord(ss->join, ss->s));
  g_launch_stream = s;

  // Tiles up to 64 rows: the forward GEMMs run on the block-scaled MMAs (weights not decoded;
  // E2M1 activation terms up to 32 rows, E4M3 at 64); 128-row tiles (the large-T regime) on the
  // fp16 dequant path.
  const int kind = bs_kind(W.nmax);
  const bool bs = kind >= 0;
  // few tokens with E2M1 terms: the sort and x's terms in one launch
  const bool fused_front = nblk == 1 && kind == BS_FP4 && E <= 1024 && k <= 32 && P <= 2048;
  if (fused_front) {
    LL_TRY(launch_plan_rows_to_e2m1x4(idx, w, T, k, E, W.nmax, W.offsets, W.chunks, W.n_chunks, W.perm_token,
                                      W.perm_slot, W.pair_pos, W.tw, W.tok_pos, W.chunk_of, W.st, W.split_cnt,
                                      W.split_cnt ? 2 * 4 * W.split_units : 0, x, x_dtype, d, P, W.xq, W.xsfb, s));
  } else if (nblk == 1) {    // few tokens: the counting sort in one block, no memset
    LL_TRY(launch_pdl("k_plan_small", k_plan_small, dim3(1), dim3(1024), (size_t)(E + P) * sizeof(int), s, idx, w, T,
                      k, E, W.nmax, W.offsets, W.chunks, W.n_chunks, W.perm_token, W.perm_slot, W.pair_pos, W.tw,
                      W.tok_pos, W.chunk_of, W.st, W.split_cnt, W.split_cnt ? 2 * 4 * W.split_units : 0));
  } else {
    LL_CUDA(cudaMemsetAsync(W.perm_token, 0xFF, sizeof(int) * P, s));
    LL_TRY(launch_pdl("k_count", k_count, dim3(nblk), dim3(256), E * sizeof(int), s, idx, T, k, E, W.cnt));
    LL_TRY(launch_pdl("k_scan", k_scan, dim3(1), dim3(1024), 0, s, W.cnt, nblk, E, W.nmax, W.offsets, W.chunks,
                      W.n_chunks, W.chunk_of));
    LL_TRY(launch_pdl("k_scatter", k_scatter, dim3(nblk), dim3(256), kTokBlock * k * sizeof(int), s, idx, w, T, k, E,
                      W.cnt, W.perm_token, W.perm_slot, W.pair_pos, W.tw, W.tok_pos));
  }
  if (!bs) LL_TRY(launch_token_rows_to_half(x, x_dtype, W.perm_token, W.tok_pos, T, k, d, W.xh, W.xinv, s));
  // F1: gate / up (after the side stream's deltas)
  if (bs) {
    CUtensorMap a[2], b[4];
    if (kind == BS_FP4) {
      LL_TRY(make_fp4_packed_map(&a[0], L->w1p, (int64_t)E * f, d, 128));
      LL_TRY(make_fp4_packed_map(&a[1], L->w3p, (int64_t)E * f, d, 128));
    } else {
      LL_TRY(make_fp4_map(&a[0], L->w1p, (int64_t)E * f, d, 128));
      LL_TRY(make_fp4_map(&a[1], L->w3p, (int64_t)E * f, d, 128));
    }
    BsArgs a1{};
    if (fused_front) {
      LL_TRY(make_e2m1x4_maps(b, W.nmax < 16 ? 1 : W.nmax / 16, W.xq, P, d, W.nmax < 16 ? 4 : 16));
      a1.sfb = W.xsfb;
    } else {
      LL_TRY(bs_operand(kind, W, x, x_dtype, T, W.tok_pos, k, nullptr, d, P, W.xq, W.xinv3, W.xsfb, b, a1, s));
    }
    a1.chunks = W.chunks;
    a1.n_chunks = W.n_chunks;
    a1.chunks_cap = W.max_chunks;
    a1.mtiles = f / 128;
    a1.K = d;
    a1.e_rows = f;
    a1.sfa[0] = L->w1sf;
    a1.sfa[1] = L->w3sf;
    a1.prefetch = bs_prefetch_stages();
    a1.status = W.st;
    a1.split_part = W.split_part;
    a1.split_cnt = W.split_cnt;
    a1.split_units = std::min(W.split_units, bs_split_units(0));
    a1.split_ctas = kSplitCtas;
    a1.epi.perm_token = W.perm_token;
    a1.epi.P = P;
    a1.epi.M = f;
    a1.epi.delta_g = W.dlt_g;
    a1.epi.delta_u = W.dlt_u;
    a1.epi.G = W.G;
    a1.epi.U = W.U;
    a1.epi.H = W.H;
    LL_CUDA(cudaStreamWaitEvent(s, ss->join, 0));
    LL_TRY(bs_launch<EPI_F1>(kind, W.nmax, a, b, a1, s));
  } else {
    CUtensorMap pk[2], sc[2], act[8];
    LL_TRY(make_rowscale_maps(&pk[0], &sc[0], L->w1p, L->w1s, (int64_t)E * f, d, L->s13_stride));
    LL_TRY(make_rowscale_maps(&pk[1], &sc[1], L->w3p, L->w3s, (int64_t)E * f, d, L->s13_stride));
    LL_TRY(make_act_maps(act, dq_nmax(W) / 16, W.xh, P, d));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = f / 128;
    a.K = d;
    a.e_rows = f;
    a.status = W.st;
    a.epi.perm_token = W.perm_token;
    a.epi.row_scale_inv = W.xinv;
    a.epi.beta = L->beta;
    a.epi.beta_col = 0;
    a.epi.P = P;
    a.epi.M = f;
    a.epi.delta_g = W.dlt_g;
    a.epi.delta_u = W.dlt_u;
    a.epi.G = W.G;
    a.epi.U = W.U;
    a.epi.H = W.H;
    LL_CUDA(cudaStreamWaitEvent(s, ss->join, 0));
    LL_TRY((gemm_nmax<EPI_F1, 2, 1, false>(dq_nmax(W), pk, sc, act, a, s)));
  }
  const int* n_valid = W.offsets + E;
  // z = h . A_d^T per pair (h as the fp16 rows the down GEMM reads); with few tokens on the side
  // stream beside the h terms and F2 (which use neither z nor the skinny partials), joined before
  // the combine. (q = the routing-weighted sum of z per token is formed by the combine below.)
  const bool z_side = nblk == 1;
  if (z_side) {
    LL_CUDA(cudaEventRecord(ss->fork, s));
    LL_CUDA(cudaStreamWaitEvent(ss->s, ss->fork, 0));
    g_launch_stream = ss->s;
  }
  LL_TRY(skinny(W.H, 2, true, P, f, L->A_d, nullptr, r, r, 1.f, W.z, nullptr, W.skpart, W.skpart_floats,
                z_side ? ss->s : s));
  if (z_side) {
    LL_CUDA(cudaEventRecord(ss->join, ss->s));
    g_launch_stream = s;
  }
  // F2: down (paired 128-row tiles of the stack: d a multiple of 256)
  if (bs && d % 256 == 0) {
    CUtensorMap a[2], b[4];
    if (kind == BS_FP4)
      LL_TRY(make_fp4_packed_map(&a[0], L->w2p, (int64_t)E * d, f, 256));
    else
      LL_TRY(make_fp4_map(&a[0], L->w2p, (int64_t)E * d, f, 256));
    a[1] = a[0];
    BsArgs a2{};
    LL_TRY(bs_operand(kind, W, W.H, 2, P, nullptr, 0, n_valid, f, P, W.hq, W.hinv3, W.hsfb, b, a2, s));
    a2.chunks = W.chunks;
    a2.n_chunks = W.n_chunks;
    a2.chunks_cap = W.max_chunks;
    a2.mtiles = d / 256;
    a2.K = f;
    a2.e_rows = d;
    a2.sfa[0] = a2.sfa[1] = L->w2sf;
    a2.prefetch = bs_prefetch_stages();
    a2.status = W.st;
    a2.split_part = W.split_part;
    a2.split_cnt = W.split_cnt ? W.split_cnt + 4 * W.split_units : nullptr;
    a2.split_units = std::min(W.split_units, bs_split_units(1));
    a2.split_ctas = kSplitCtas;
    a2.epi.perm_token = W.perm_token;
    a2.epi.tw = W.tw;
    a2.epi.P = P;
    a2.epi.M = d;
    a2.epi.Y = W.Y;
    LL_TRY(bs_launch<EPI_F2>(kind, W.nmax, a, b, a2, s));
  } else {
    CUtensorMap pk[2], sc[2], act[8];
    LL_TRY(make_rowscale_maps(&pk[0], &sc[0], L->w2p, L->w2s, (int64_t)E * d, f, L->s2_stride, 256));
    pk[1] = pk[0];
    sc[1] = sc[0];
    LL_TRY(make_act_maps(act, dq_nmax(W) / 16, W.H, P, f));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = (d + 255) / 256;                 // paired 128-row tiles
    a.K = f;
    a.e_rows = d;
    a.status = W.st;
    a.epi.perm_token = W.perm_token;
    a.epi.tw = W.tw;
    a.epi.beta = L->beta;
    a.epi.beta_col = 1;
    a.epi.P = P;
    a.epi.M = d;
    a.epi.Y = W.Y;
    LL_TRY((gemm_nmax<EPI_F2, 2, 1, false>(dq_nmax(W), pk, sc, act, a, s)));
  }
  if (z_side) LL_CUDA(cudaStreamWaitEvent(s, ss->join, 0));
  if (norm_w) {
    if (d % 2 || r > kExMaxR || k > 32) return LL_ERR_ARG;
    const int smem = r * kExPitch * (int)sizeof(float);
    LL_TRY(set_smem_attr(reinterpret_cast<const void*>(k_expand_norm<false>), smem));
    return launch_pdl("k_expand_norm", k_expand_norm<false>, dim3((T + kExTok - 1) / kExTok), dim3(kExThreads), smem,
                      s, W.tok_pos, W.Y, k, T, d, r, L->lora_scaling, L->B_d, W.tw, W.z, W.q, out, norm_w, eps,
                      static_cast<__nv_bfloat16*>(normed), rstd);
  }
  return expand(false, W.tok_pos, W.Y, k, T, d, r, L->lora_scaling, nullptr, L->B_d, nullptr, nullptr, out, s, nullptr,
                W.tw, W.z, W.q);
}

int ll_moe_forward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx, const float* w,
                   float* out, void* ws, size_t ws_bytes, void* stream) {
  return moe_forward(L, T, k, x, x_dtype, idx, w, out, nullptr, 0.f, nullptr, nullptr, ws, ws_bytes, stream);
}

int ll_moe_forward_rmsnorm(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx,
                           const float* w, const float* norm_w, float eps, float* out, void* normed, float* rstd,
                           void* ws, size_t ws_bytes, void* stream) {
  if (!norm_w) return LL_ERR_ARG;
  return moe_forward(L, T, k, x, x_dtype, idx, w, out, norm_w, eps, normed, rstd, ws, ws_bytes, stream);
}

int ll_moe_backward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx, const float* w,
                    const void* g, int g_dtype, float* grad_h, float* grad_w, float* dA_g, float* dB_g, float* dA_u,
                    float* dB_u, float* dA_d, float* dB_d, void* ws, size_t ws_bytes, void* stream) {
  LL_TRY(validate(L, T, k, true));
  if (!x || !idx || !w || !g || !grad_h || !grad_w || !ws) return LL_ERR_ARG;
  if (!dA_g || !dB_g || !dA_u || !dB_u || !dA_d || !dB_d) return LL_ERR_ARG;
  if ((x_dtype != 0 && x_dtype != 1) || (g_dtype != 0 && g_dtype != 1)) return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_moe_workspace_bytes(L, T, k)) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int P = T * k;
  const float sc_l = L->lora_scaling;
  const int* n_valid = W.offsets + E;
  g_launch_count = 0;

  LL_TRY(launch_token_rows_to_half(g, g_dtype, W.perm_token, W.tok_pos, T, k, d, W.gh, W.ginv, s));
  if (W.proj_ws && g_dtype == 1)
    LL_TRY(project_tc(g, T, d, L->B_d, nullptr, true, r, W.gB, nullptr, W.proj_ws, W.proj_bytes, W.st, s));
  else
    LL_TRY(skinny(g, g_dtype, false, T, d, L->B_d, nullptr, r, r, 1.f, W.gB, nullptr, W.skpart, W.skpart_floats, s));
  // the down adapter's term of dL/dh, once per token: (g B_d) A_d [T][f]
  LL_TRY(expand(true, nullptr, nullptr, k, T, f, r, 1.f, W.gB, L->A_d, nullptr, nullptr, W.lora_d, s));
  // B1: v = g . W2 (+ LoRA down), SiTU-GLU backward
  {
    // paired 128-row tiles, except at 128-token tiles: there two accumulators of 128 columns
    // leave tensor memory for one buffer only, and this epilogue is too heavy to run exposed
    const bool pair = W.nmax < 128;
    CUtensorMap pk[2], sc[2], act[8];
    LL_TRY(make_colscale_maps(&pk[0], &sc[0], L->w2t, reinterpret_cast<const __half*>(L->s2t), (int64_t)E * f, d,
                              pair ? 256 : 128));
    pk[1] = pk[0];
    sc[1] = sc[0];
    LL_TRY(make_act_maps(act, dq_nmax(W) / 16, W.gh, P, d));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = pair ? (f + 255) / 256 : f / 128;
    a.K = d;
    a.e_rows = f;
    a.status = W.st;
    a.epi.perm_token = W.perm_token;
    a.epi.row_scale_inv = W.ginv;
    a.epi.tw = W.tw;
    a.epi.beta = L->beta;
    a.epi.beta_col = 1;
    a.epi.P = P;
    a.epi.M = f;
    a.epi.r = r;
    a.epi.lora_scaling = sc_l;
    a.epi.lora_d = W.lora_d;
    a.epi.Gs = W.G;
    a.epi.Us = W.U;
    a.epi.DG = W.DG;
    a.epi.DU = W.DU;
    a.epi.gw_part = W.gw_part;
    if (!pair)
      LL_TRY((launch_gemm<EPI_B1, 1, 1, true, 128>(pk, sc, act, a, s)));
    else if (dq_nmax(W) == 16)
      LL_TRY((launch_gemm<EPI_B1, 2, 1, true, 16>(pk, sc, act, a, s)));
    else if (dq_nmax(W) == 32)
      LL_TRY((launch_gemm<EPI_B1, 2, 1, true, 32>(pk, sc, act, a, s)));
    else
      LL_TRY((launch_gemm<EPI_B1, 2, 1, true, 64>(pk, sc, act, a, s)));
  }
  // the pairs' fp16 rows for B2 and the per-token sums of the gate / up gradients, one pass
  const int nv = f / (4 * kPTThreads);
  const bool fused_rows = f % (4 * kPTThreads) == 0 && (nv == 1 || nv == 2 || nv == 4);
  if (fused_rows) {
    auto kern = nv == 1 ? k_pair_rows_tokens<1> : nv == 2 ? k_pair_rows_tokens<2> : k_pair_rows_tokens<4>;
    LL_TRY(launch_pdl("k_pair_rows_tokens", kern, dim3(T), dim3(kPTThreads), 0, s, W.tok_pos, W.DG, W.DU, k, f,
                      W.DGh, W.DUh, W.rinv, W.Dg, W.Du));
  } else {
    LL_TRY(launch_pdl("k_pair_rows_half", k_pair_rows_half, dim3(P), dim3(256), 0, s, W.DG, W.DU, f, n_valid, W.DGh,
                      W.DUh, W.rinv));
  }
  // B2: dX = dg . W1 + du . W3
  {
    CUtensorMap pk[2], sc[2], act[8];
    LL_TRY(make_colscale_maps(&pk[0], &sc[0], L->w1t, reinterpret_cast<const __half*>(L->s1t), (int64_t)E * d, f));
    LL_TRY(make_colscale_maps(&pk[1], &sc[1], L->w3t, reinterpret_cast<const __half*>(L->s3t), (int64_t)E * d, f));
    LL_TRY(make_act_maps(act, dq_nmax(W) / 16, W.DGh, P, f, 2, (int64_t)(W.DUh - W.DGh)));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = d / 128;
    a.K = f;
    a.e_rows = d;
    a.status = W.st;
    a.epi.perm_token = W.perm_token;
    a.epi.row_scale_inv = W.rinv;
    a.epi.beta = L->beta;
    a.epi.beta_col = 0;
    a.epi.P = P;
    a.epi.M = d;
    a.epi.Y = W.Y;
    LL_TRY((gemm_nmax<EPI_B2, 2, 2, true>(dq_nmax(W), pk, sc, act, a, s)));
  }
  if (!fused_rows) {
    LL_TRY(launch_pdl("k_token_sum", k_token_sum, dim3((f + 255) / 256, T), dim3(256), 0, s, W.tok_pos, W.DG, W.DU, T,
                      k, f, W.Dg, W.Du));
  }
  LL_TRY(skinny(W.Dg, 0, false, T, f, L->B_g, nullptr, r, r, 1.f, W.hg, nullptr, W.skpart, W.skpart_floats, s));
  LL_TRY(skinny(W.Du, 0, false, T, f, L->B_u, nullptr, r, r, 1.f, W.hu, nullptr, W.skpart, W.skpart_floats, s));
  LL_TRY(expand(true, W.tok_pos, W.Y, k, T, d, r, sc_l, W.hg, L->A_g, W.hu, L->A_u, grad_h, s));
  LL_TRY(launch_pdl("k_grad_w", k_grad_w, dim3((P + 255) / 256), dim3(256), 0, s, W.pair_pos, W.gw_part,
                    (f / 128) * 4, P, P, grad_w));
  // LoRA gradients
  LL_TRY(outer(W.hg, nullptr, nullptr, x, x_dtype, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_g, s));
  LL_TRY(outer(W.xa_g, nullptr, nullptr, W.Dg, 0, T, nullptr, f, r, sc_l, true, W.opart, W.nseg_max, dB_g, s));
  LL_TRY(outer(W.hu, nullptr, nullptr, x, x_dtype, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_u, s));
  LL_TRY(outer(W.xa_u, nullptr, nullptr, W.Du, 0, T, nullptr, f, r, sc_l, true, W.opart, W.nseg_max, dB_u, s));
  LL_TRY(outer(W.gB, W.perm_token, W.tw, W.H, 2, P, n_valid, f, r, sc_l, false, W.opart, W.nseg_max, dA_d, s));
  LL_TRY(outer(W.q, nullptr, nullptr, g, g_dtype, T, nullptr, d, r, sc_l, true, W.opart, W.nseg_max, dB_d, s));
  return LL_OK;
}

// Copies the stable (expert, token) permutation of the last forward out of the workspace:
// offsets [E+1], and for the first offsets[E] sorted rows their token and slot.
int ll_moe_permutation(const ll_moe_layer* L, int T, int k, void* ws, int* offsets, int* perm_token, int* perm_slot,
                       void* stream) {
  if (!L || !ws || !offsets || !perm_token || !perm_slot || T <= 0 || k <= 0) return LL_ERR_ARG;
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  LL_STREAM(stream);
  LL_CUDA(cudaMemcpyAsync(offsets, W.offsets, sizeof(int) * (L->E + 1), cudaMemcpyDeviceToDevice, s));
  LL_CUDA(cudaMemcpyAsync(perm_token, W.perm_token, sizeof(int) * T * k, cudaMemcpyDeviceToDevice, s));
  LL_CUDA(cudaMemcpyAsync(perm_slot, W.perm_slot, sizeof(int) * T * k, cudaMemcpyDeviceToDevice, s));
  return LL_OK;
}

// Reads (and clears) the device status word of a layer workspace; synchronises the stream.
int ll_moe_status(const ll_moe_layer* L, int T, int k, void* ws, void* stream) {
  if (!L || !ws) return LL_ERR_ARG;
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  LL_STREAM(stream);
  LL_CUDA(cudaStreamSynchronize(s));
  LL_CUDA(cudaGetLastError());
  const int rc = read_status(W.st, s);
  LL_TRY(reset_status(W.st, s));
  return rc;
}

}  // extern "C"
