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

namespace ll {

constexpr int kTokBlock = 64;   // tokens per block in the counting sort

// ----------------------------------------------------------------- counting sort
__global__ void k_count(const int64_t* __restrict__ idx, int T, int k, int E, int* __restrict__ cnt) {
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
                                               Chunk* __restrict__ chunks, int* __restrict__ n_chunks) {
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

// ----------------------------------------------------------------- LoRA helpers
// out{0,1}[t][rr] = sum_k X[t][k] * W{0,1}(rr, k); W(rr,k) = W[rr*K + k] (ROWS) or W[k*r + rr].
template <int XD, bool ROWS>
__global__ void k_rowdot(const void* __restrict__ X, int K, int r, const float* __restrict__ W0, const float* __restrict__ W1,
                         float* __restrict__ out0, float* __restrict__ out1) {
  const int t = blockIdx.x;
  float a0[32], a1[32];
#pragma unroll
  for (int i = 0; i < 32; i++) { a0[i] = 0.f; a1[i] = 0.f; }
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float xv = XD == 0 ? reinterpret_cast<const float*>(X)[(int64_t)t * K + k]
                             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(X)[(int64_t)t * K + k]);
#pragma unroll
    for (int i = 0; i < 32; i++) {
      if (i < r) {
        a0[i] = fmaf(xv, ROWS ? W0[(int64_t)i * K + k] : W0[(int64_t)k * r + i], a0[i]);
        if (W1) a1[i] = fmaf(xv, ROWS ? W1[(int64_t)i * K + k] : W1[(int64_t)k * r + i], a1[i]);
      }
    }
  }
  __shared__ float red[2][8][32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    if (i >= r) break;
    float s0 = a0[i], s1 = a1[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    if (lane == 0) { red[0][warp][i] = s0; red[1][warp][i] = s1; }
  }
  __syncthreads();
  if (threadIdx.x < r) {
    float s0 = 0.f, s1 = 0.f;
    for (int wi = 0; wi < (int)(blockDim.x / 32); wi++) { s0 += red[0][wi][threadIdx.x]; s1 += red[1][wi][threadIdx.x]; }
    out0[(int64_t)t * r + threadIdx.x] = s0;
    if (out1) out1[(int64_t)t * r + threadIdx.x] = s1;
  }
}

// delta{g,u}[t][m] = s * sum_rr xa{g,u}[t][rr] * B{g,u}[m][rr]
__global__ void k_lora_delta(const float* __restrict__ xa_g, const float* __restrict__ xa_u, const float* __restrict__ B_g,
                             const float* __restrict__ B_u, int T, int f, int r, float s, float* __restrict__ dg,
                             float* __restrict__ du) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * f) return;
  const int t = (int)(i / f), m = (int)(i % f);
  float ag = 0.f, au = 0.f;
  for (int rr = 0; rr < r; rr++) {
    ag = fmaf(xa_g[(int64_t)t * r + rr], B_g[(int64_t)m * r + rr], ag);
    au = fmaf(xa_u[(int64_t)t * r + rr], B_u[(int64_t)m * r + rr], au);
  }
  dg[i] = s * ag;
  du[i] = s * au;
}

// z[p][rr] = sum_m situ(G[p][m], U[p][m]) * A_d[rr][m] for the valid pairs p < offsets[E]
__global__ void k_z(const float* __restrict__ G, const float* __restrict__ U, const float* __restrict__ A_d, int f, int r,
                    const int* __restrict__ n_valid, float* __restrict__ z) {
  const int p = blockIdx.x;
  if (p >= *n_valid) return;
  float a[32];
#pragma unroll
  for (int i = 0; i < 32; i++) a[i] = 0.f;
  for (int m = threadIdx.x; m < f; m += blockDim.x) {
    const float h = situ_glu_fwd(G[(int64_t)p * f + m], U[(int64_t)p * f + m]);
#pragma unroll
    for (int i = 0; i < 32; i++)
      if (i < r) a[i] = fmaf(h, A_d[(int64_t)i * f + m], a[i]);
  }
  __shared__ float red[8][32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    if (i >= r) break;
    float s0 = a[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s0 += __shfl_xor_sync(0xffffffffu, s0, off);
    if (lane == 0) red[warp][i] = s0;
  }
  __syncthreads();
  if (threadIdx.x < r) {
    float s0 = 0.f;
    for (int wi = 0; wi < (int)(blockDim.x / 32); wi++) s0 += red[wi][threadIdx.x];
    z[(int64_t)p * r + threadIdx.x] = s0;
  }
}

// q[t][rr] = sum over the token's pairs (ascending expert) of tw * z
__global__ void k_q(const int* __restrict__ tok_pos, const float* __restrict__ tw, const float* __restrict__ z, int T, int k,
                    int r, float* __restrict__ q) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * r) return;
  const int t = (int)(i / r), rr = (int)(i % r);
  float acc = 0.f;
  for (int j = 0; j < k; j++) {
    const int pos = tok_pos[(int64_t)t * k + j];
    if (pos < 0) break;
    acc = fmaf(tw[pos], z[(int64_t)pos * r + rr], acc);
  }
  q[i] = acc;
}

// out[t][c] = sum_j Y[pos_j][c] (ascending expert) + s * sum_rr L0[t][rr] * R0(rr, c) (+ L1 R1)
// R(rr, c) = R[c*r + rr] (COLS, B_d [d][r]) or R[rr*C + c] (A [r][C]).
template <bool COLS>
__global__ void k_combine(const int* __restrict__ tok_pos, const float* __restrict__ Y, int k, int C, int r, float s,
                          const float* __restrict__ L0, const float* __restrict__ R0, const float* __restrict__ L1,
                          const float* __restrict__ R1, float* __restrict__ out) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  __shared__ int pos[32];
  __shared__ float l0[32], l1[32];
  if (threadIdx.x < 32) {
    pos[threadIdx.x] = threadIdx.x < k ? tok_pos[(int64_t)t * k + threadIdx.x] : -1;
    l0[threadIdx.x] = threadIdx.x < r ? L0[(int64_t)t * r + threadIdx.x] : 0.f;
    l1[threadIdx.x] = (L1 && threadIdx.x < r) ? L1[(int64_t)t * r + threadIdx.x] : 0.f;
  }
  __syncthreads();
  if (c >= C) return;
  float acc = 0.f;
  for (int j = 0; j < k; j++) {
    const int p = pos[j];
    if (p < 0) break;
    acc += Y[(int64_t)p * C + c];
  }
  float lo = 0.f;
  for (int rr = 0; rr < r; rr++) {
    lo = fmaf(l0[rr], COLS ? R0[(int64_t)c * r + rr] : R0[(int64_t)rr * C + c], lo);
    if (L1) lo = fmaf(l1[rr], COLS ? R1[(int64_t)c * r + rr] : R1[(int64_t)rr * C + c], lo);
  }
  out[(int64_t)t * C + c] = acc + s * lo;
}

// Per valid pair: one power-of-two scale for both rows of dg / du, fp16 copies for B2.
__global__ void k_pair_rows_half(const float* __restrict__ DG, const float* __restrict__ DU, int f,
                                 const int* __restrict__ n_valid, __half* __restrict__ DGh, __half* __restrict__ DUh,
                                 float* __restrict__ inv) {
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

__global__ void k_grad_w(const int* __restrict__ pair_pos, const float* __restrict__ parts, int nparts, int P, int Tk,
                         float* __restrict__ grad_w) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= Tk) return;
  const int pos = pair_pos[q];
  float s = 0.f;
  if (pos >= 0)
    for (int i = 0; i < nparts; i++) s += parts[(int64_t)i * P + pos];
  grad_w[q] = s;
}

// Outer-product reductions for the LoRA gradients:
//   part[seg][rr][c] = sum_{n in seg} Pm(n, rr) * Q(n, c)
// Pm: [N][r] fp32, or (PGATHER) tw[n] * gB[perm_token[n]][rr].
// Q:  QK 0 fp32 [N][C], 1 bf16 [N][C], 2 situ(G, U) from two fp32 [N][C].
template <int QK, bool PGATHER>
__global__ void k_outer(const float* __restrict__ Pm, const int* __restrict__ perm_token, const float* __restrict__ tw,
                        const void* __restrict__ Q, const float* __restrict__ Q2, int N, const int* __restrict__ n_dev,
                        int C, int r, int nseg, float* __restrict__ part) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int seg = blockIdx.y;
  const int n_total = n_dev ? *n_dev : N;
  const int per = (n_total + nseg - 1) / nseg;
  const int n0 = seg * per, n1 = min(n_total, n0 + per);
  __shared__ float ps[32][33];
  float acc[32];
#pragma unroll
  for (int i = 0; i < 32; i++) acc[i] = 0.f;
  for (int nb = n0; nb < n1; nb += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * r; i += blockDim.x) {
      const int nn = i / r, rr = i % r;
      const int n = nb + nn;
      float v = 0.f;
      if (n < n1) v = PGATHER ? tw[n] * Pm[(int64_t)perm_token[n] * r + rr] : Pm[(int64_t)n * r + rr];
      ps[nn][rr] = v;
    }
    __syncthreads();
    if (c < C) {
      const int lim = min(32, n1 - nb);
      for (int nn = 0; nn < lim; nn++) {
        const int64_t o = (int64_t)(nb + nn) * C + c;
        float qv;
        if (QK == 0) qv = reinterpret_cast<const float*>(Q)[o];
        else if (QK == 1) qv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(Q)[o]);
        else qv = situ_glu_fwd(reinterpret_cast<const float*>(Q)[o], Q2[o]);
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (i < r) acc[i] = fmaf(ps[nn][i], qv, acc[i]);
      }
    }
  }
  if (c < C)
    for (int i = 0; i < r; i++) part[((int64_t)seg * r + i) * C + c] = acc[i];
}

// out = s * sum_seg part, stored [r][C] or transposed [C][r]
__global__ void k_outer_reduce(const float* __restrict__ part, int nseg, int r, int C, float s, bool transposed,
                               float* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)r * C) return;
  const int rr = (int)(i / C), c = (int)(i % C);
  float acc = 0.f;
  for (int sg = 0; sg < nseg; sg++) acc += part[((int64_t)sg * r + rr) * C + c];
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
  float* tw;
  float* xinv;
  __half* xh;
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
  int nmax;
  int nseg_max;
};

static int choose_nmax(int T, int k, int E) {
  const double mean = (double)T * k / (E > 0 ? E : 1);
  return mean <= 12.0 ? 32 : 128;
}

static size_t layer_layout(void* base, const ll_moe_layer* L, int T, int k, LayerWs* out) {
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int64_t P = (int64_t)T * k;
  const int nmax = choose_nmax(T, k, E);
  const int nblk = (T + kTokBlock - 1) / kTokBlock;
  const int nseg_max = 64;
  Carver c(base);
  LayerWs w{};
  w.nmax = nmax;
  w.nseg_max = nseg_max;
  w.st = c.take<DevStatus>(1);
  w.cnt = c.take<int>((size_t)nblk * E);
  w.offsets = c.take<int>(E + 1);
  w.chunks = c.take<Chunk>(E + P / nmax + 2);
  w.n_chunks = c.take<int>(1);
  w.perm_token = c.take<int>(P);
  w.perm_slot = c.take<int>(P);
  w.pair_pos = c.take<int>(P);
  w.tok_pos = c.take<int>(P);
  w.tw = c.take<float>(P);
  w.xinv = c.take<float>(P);
  w.xh = c.take<__half>(P * d);
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
  w.gw_part = c.take<float>((size_t)((f + 127) / 128) * 4 * P);
  w.DG = c.take<float>(P * f);
  w.DU = c.take<float>(P * f);
  w.rinv = c.take<float>(P);
  w.DGh = c.take<__half>(P * f);
  w.DUh = c.take<__half>(P * f);
  w.Dg = c.take<float>((size_t)T * f);
  w.Du = c.take<float>((size_t)T * f);
  w.hg = c.take<float>((size_t)T * r);
  w.hu = c.take<float>((size_t)T * r);
  w.opart = c.take<float>((size_t)nseg_max * r * (d > f ? d : f));
  if (out) *out = w;
  return c.off + 256;
}

static int validate(const ll_moe_layer* L, int T, int k) {
  if (!L || T <= 0 || k <= 0 || k > 32) return LL_ERR_ARG;
  if (L->d <= 0 || L->f <= 0 || L->d % 128 || L->f % 128 || L->E <= 0 || L->E > 8192) return LL_ERR_ARG;
  if (L->r <= 0 || L->r > 32) return LL_ERR_ARG;
  if (L->s13_stride < L->d / 32 || L->s13_stride % 16 || L->s2_stride < L->f / 32 || L->s2_stride % 16) return LL_ERR_ARG;
  if (!L->w1p || !L->w1s || !L->w3p || !L->w3s || !L->w2p || !L->w2s || !L->beta) return LL_ERR_ARG;
  if (!L->A_g || !L->B_g || !L->A_u || !L->B_u || !L->A_d || !L->B_d) return LL_ERR_ARG;
  if (!L->w1t || !L->w3t || !L->w2t || !L->s1t || !L->s3t || !L->s2t) return LL_ERR_ARG;
  return LL_OK;
}

template <int EPI, int NMAT, int NB, bool COLSCALE>
static int gemm_nmax(int nmax, const CUtensorMap* pk, const CUtensorMap* sc, const CUtensorMap* act, const GemmArgs& a,
                     cudaStream_t s) {
  if (nmax == 32) return launch_gemm<EPI, NMAT, NB, COLSCALE, 32>(pk, sc, act, a, s);
  return launch_gemm<EPI, NMAT, NB, COLSCALE, 128>(pk, sc, act, a, s);
}

template <int QK, bool PG>
static int outer(const float* Pm, const int* perm_token, const float* tw, const void* Q, const float* Q2, int N,
                 const int* n_dev, int C, int r, float s, bool transposed, float* part, int nseg_max, float* out,
                 cudaStream_t st) {
  const int cblocks = (C + 255) / 256;
  int nseg = (2 * device_info().sms + cblocks - 1) / cblocks;
  nseg = std::max(1, std::min(nseg, nseg_max));
  nseg = std::min(nseg, std::max(1, N / 32));
  k_outer<QK, PG><<<dim3(cblocks, nseg), 256, 0, st>>>(Pm, perm_token, tw, Q, Q2, N, n_dev, C, r, nseg, part);
  LL_TRY(check_launch("k_outer"));
  const int64_t n = (int64_t)r * C;
  k_outer_reduce<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, nseg, r, C, s, transposed, out);
  return check_launch("k_outer_reduce");
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
  if (!L->w1t || !L->w3t || !L->w2t || !L->s1t || !L->s3t || !L->s2t) return LL_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int E = L->E, d = L->d, f = L->f;
  LL_TRY(launch_prepare_beta(L->w1s, L->w3s, E, f, d, L->s13_stride, beta_out, 0, s));
  LL_TRY(launch_prepare_beta(L->w2s, nullptr, E, d, f, L->s2_stride, beta_out, 1, s));
  auto cw = [](const uint8_t* p) { return const_cast<uint8_t*>(p); };
  auto ch = [](const uint16_t* p) { return reinterpret_cast<__half*>(const_cast<uint16_t*>(p)); };
  LL_TRY(launch_transpose_mxfp4(L->w1p, L->w1s, L->s13_stride, E, f, d, beta_out, 0, cw(L->w1t), ch(L->s1t), s));
  LL_TRY(launch_transpose_mxfp4(L->w3p, L->w3s, L->s13_stride, E, f, d, beta_out, 0, cw(L->w3t), ch(L->s3t), s));
  LL_TRY(launch_transpose_mxfp4(L->w2p, L->w2s, L->s2_stride, E, d, f, beta_out, 1, cw(L->w2t), ch(L->s2t), s));
  return LL_OK;
}

size_t ll_moe_workspace_bytes(const ll_moe_layer* L, int T, int k) {
  if (!L || T <= 0 || k <= 0) return 0;
  return layer_layout(nullptr, L, T, k, nullptr);
}

int ll_moe_forward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx, const float* w,
                   float* out, void* ws, size_t ws_bytes, void* stream) {
  LL_TRY(validate(L, T, k));
  if (!x || !idx || !w || !out || !ws || (x_dtype != 0 && x_dtype != 1)) return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_moe_workspace_bytes(L, T, k)) return LL_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int P = T * k;
  const int nblk = (T + kTokBlock - 1) / kTokBlock;
  g_launch_count = 0;

  LL_TRY(reset_status(W.st, s));
  LL_CUDA(cudaMemsetAsync(W.perm_token, 0xFF, sizeof(int) * P, s));
  k_count<<<nblk, 256, E * sizeof(int), s>>>(idx, T, k, E, W.cnt);
  LL_TRY(check_launch("k_count"));
  k_scan<<<1, 1024, 0, s>>>(W.cnt, nblk, E, W.nmax, W.offsets, W.chunks, W.n_chunks);
  LL_TRY(check_launch("k_scan"));
  k_scatter<<<nblk, 256, kTokBlock * k * sizeof(int), s>>>(idx, w, T, k, E, W.cnt, W.perm_token, W.perm_slot,
                                                            W.pair_pos, W.tw, W.tok_pos);
  LL_TRY(check_launch("k_scatter"));
  LL_TRY(launch_rows_to_half(x, x_dtype, W.perm_token, P, d, W.xh, W.xinv, s));
  if (x_dtype == 0)
    k_rowdot<0, true><<<T, 256, 0, s>>>(x, d, r, L->A_g, L->A_u, W.xa_g, W.xa_u);
  else
    k_rowdot<1, true><<<T, 256, 0, s>>>(x, d, r, L->A_g, L->A_u, W.xa_g, W.xa_u);
  LL_TRY(check_launch("k_rowdot"));
  {
    const int64_t n = (int64_t)T * f;
    k_lora_delta<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(W.xa_g, W.xa_u, L->B_g, L->B_u, T, f, r, L->lora_scaling,
                                                             W.dlt_g, W.dlt_u);
    LL_TRY(check_launch("k_lora_delta"));
  }
  // F1: gate / up
  {
    CUtensorMap pk[2], sc[2], act[1];
    LL_TRY(make_rowscale_maps(&pk[0], &sc[0], L->w1p, L->w1s, (int64_t)E * f, d, L->s13_stride));
    LL_TRY(make_rowscale_maps(&pk[1], &sc[1], L->w3p, L->w3s, (int64_t)E * f, d, L->s13_stride));
    LL_TRY(make_act_map(&act[0], W.xh, P, d));
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
    LL_TRY((gemm_nmax<EPI_F1, 2, 1, false>(W.nmax, pk, sc, act, a, s)));
  }
  const int* n_valid = W.offsets + E;
  k_z<<<P, 256, 0, s>>>(W.G, W.U, L->A_d, f, r, n_valid, W.z);
  LL_TRY(check_launch("k_z"));
  {
    const int64_t n = (int64_t)T * r;
    k_q<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(W.tok_pos, W.tw, W.z, T, k, r, W.q);
    LL_TRY(check_launch("k_q"));
  }
  // F2: down
  {
    CUtensorMap pk[1], sc[1], act[1];
    LL_TRY(make_rowscale_maps(&pk[0], &sc[0], L->w2p, L->w2s, (int64_t)E * d, f, L->s2_stride));
    LL_TRY(make_act_map(&act[0], W.H, P, f));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = d / 128;
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
    LL_TRY((gemm_nmax<EPI_F2, 1, 1, false>(W.nmax, pk, sc, act, a, s)));
  }
  k_combine<true><<<dim3((d + 255) / 256, T), 256, 0, s>>>(W.tok_pos, W.Y, k, d, r, L->lora_scaling, W.q, L->B_d,
                                                          nullptr, nullptr, out);
  return check_launch("k_combine");
}

int ll_moe_backward(const ll_moe_layer* L, int T, int k, const void* x, int x_dtype, const int64_t* idx, const float* w,
                    const void* g, int g_dtype, float* grad_h, float* grad_w, float* dA_g, float* dB_g, float* dA_u,
                    float* dB_u, float* dA_d, float* dB_d, void* ws, size_t ws_bytes, void* stream) {
  LL_TRY(validate(L, T, k));
  if (!x || !idx || !w || !g || !grad_h || !grad_w || !ws) return LL_ERR_ARG;
  if (!dA_g || !dB_g || !dA_u || !dB_u || !dA_d || !dB_d) return LL_ERR_ARG;
  if ((x_dtype != 0 && x_dtype != 1) || (g_dtype != 0 && g_dtype != 1)) return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_moe_workspace_bytes(L, T, k)) return LL_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  const int d = L->d, f = L->f, E = L->E, r = L->r;
  const int P = T * k;
  const float sc_l = L->lora_scaling;
  const int* n_valid = W.offsets + E;
  g_launch_count = 0;

  LL_TRY(launch_rows_to_half(g, g_dtype, W.perm_token, P, d, W.gh, W.ginv, s));
  if (g_dtype == 0)
    k_rowdot<0, false><<<T, 256, 0, s>>>(g, d, r, L->B_d, nullptr, W.gB, nullptr);
  else
    k_rowdot<1, false><<<T, 256, 0, s>>>(g, d, r, L->B_d, nullptr, W.gB, nullptr);
  LL_TRY(check_launch("k_rowdot"));
  // B1: v = g . W2 (+ LoRA down), SiTU-GLU backward
  {
    CUtensorMap pk[1], sc[1], act[1];
    LL_TRY(make_colscale_maps(&pk[0], &sc[0], L->w2t, reinterpret_cast<const __half*>(L->s2t), (int64_t)E * f, d));
    LL_TRY(make_act_map(&act[0], W.gh, P, d));
    GemmArgs a{};
    a.chunks = W.chunks;
    a.n_chunks = W.n_chunks;
    a.mtiles = f / 128;
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
    a.epi.gB = W.gB;
    a.epi.A_d = L->A_d;
    a.epi.Gs = W.G;
    a.epi.Us = W.U;
    a.epi.DG = W.DG;
    a.epi.DU = W.DU;
    a.epi.gw_part = W.gw_part;
    LL_TRY((gemm_nmax<EPI_B1, 1, 1, true>(W.nmax, pk, sc, act, a, s)));
  }
  k_pair_rows_half<<<P, 256, 0, s>>>(W.DG, W.DU, f, n_valid, W.DGh, W.DUh, W.rinv);
  LL_TRY(check_launch("k_pair_rows_half"));
  // B2: dX = dg . W1 + du . W3
  {
    CUtensorMap pk[2], sc[2], act[2];
    LL_TRY(make_colscale_maps(&pk[0], &sc[0], L->w1t, reinterpret_cast<const __half*>(L->s1t), (int64_t)E * d, f));
    LL_TRY(make_colscale_maps(&pk[1], &sc[1], L->w3t, reinterpret_cast<const __half*>(L->s3t), (int64_t)E * d, f));
    LL_TRY(make_act_map(&act[0], W.DGh, P, f));
    LL_TRY(make_act_map(&act[1], W.DUh, P, f));
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
    LL_TRY((gemm_nmax<EPI_B2, 2, 2, true>(W.nmax, pk, sc, act, a, s)));
  }
  k_token_sum<<<dim3((f + 255) / 256, T), 256, 0, s>>>(W.tok_pos, W.DG, W.DU, T, k, f, W.Dg, W.Du);
  LL_TRY(check_launch("k_token_sum"));
  k_rowdot<0, false><<<T, 256, 0, s>>>(W.Dg, f, r, L->B_g, nullptr, W.hg, nullptr);
  LL_TRY(check_launch("k_rowdot"));
  k_rowdot<0, false><<<T, 256, 0, s>>>(W.Du, f, r, L->B_u, nullptr, W.hu, nullptr);
  LL_TRY(check_launch("k_rowdot"));
  k_combine<false><<<dim3((d + 255) / 256, T), 256, 0, s>>>(W.tok_pos, W.Y, k, d, r, sc_l, W.hg, L->A_g, W.hu, L->A_u,
                                                           grad_h);
  LL_TRY(check_launch("k_combine"));
  k_grad_w<<<(P + 255) / 256, 256, 0, s>>>(W.pair_pos, W.gw_part, (f / 128) * 4, P, P, grad_w);
  LL_TRY(check_launch("k_grad_w"));
  // LoRA gradients
  if (x_dtype == 0)
    LL_TRY((outer<0, false>(W.hg, nullptr, nullptr, x, nullptr, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_g, s)));
  else
    LL_TRY((outer<1, false>(W.hg, nullptr, nullptr, x, nullptr, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_g, s)));
  LL_TRY((outer<0, false>(W.xa_g, nullptr, nullptr, W.Dg, nullptr, T, nullptr, f, r, sc_l, true, W.opart, W.nseg_max, dB_g, s)));
  if (x_dtype == 0)
    LL_TRY((outer<0, false>(W.hu, nullptr, nullptr, x, nullptr, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_u, s)));
  else
    LL_TRY((outer<1, false>(W.hu, nullptr, nullptr, x, nullptr, T, nullptr, d, r, sc_l, false, W.opart, W.nseg_max, dA_u, s)));
  LL_TRY((outer<0, false>(W.xa_u, nullptr, nullptr, W.Du, nullptr, T, nullptr, f, r, sc_l, true, W.opart, W.nseg_max, dB_u, s)));
  LL_TRY((outer<2, true>(W.gB, W.perm_token, W.tw, W.G, W.U, P, n_valid, f, r, sc_l, false, W.opart, W.nseg_max, dA_d, s)));
  if (g_dtype == 0)
    LL_TRY((outer<0, false>(W.q, nullptr, nullptr, g, nullptr, T, nullptr, d, r, sc_l, true, W.opart, W.nseg_max, dB_d, s)));
  else
    LL_TRY((outer<1, false>(W.q, nullptr, nullptr, g, nullptr, T, nullptr, d, r, sc_l, true, W.opart, W.nseg_max, dB_d, s)));
  return LL_OK;
}

// Copies the stable (expert, token) permutation of the last forward out of the workspace:
// offsets [E+1], and for the first offsets[E] sorted rows their token and slot.
int ll_moe_permutation(const ll_moe_layer* L, int T, int k, void* ws, int* offsets, int* perm_token, int* perm_slot,
                       void* stream) {
  if (!L || !ws || !offsets || !perm_token || !perm_slot || T <= 0 || k <= 0) return LL_ERR_ARG;
  LayerWs W;
  layer_layout(ws, L, T, k, &W);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LL_CUDA(cudaStreamSynchronize(s));
  LL_CUDA(cudaGetLastError());
  const int rc = read_status(W.st, s);
  LL_TRY(reset_status(W.st, s));
  return rc;
}

}  // extern "C"
