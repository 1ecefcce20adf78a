// Small dense kernels around the grouped GEMMs: the rank-r LoRA products and the weighted
// combines. All reductions run in a fixed order (split-K partials summed by a second pass),
// so results are bitwise reproducible.
#pragma once
#include "common.cuh"
#include "lora_ops.cuh"

namespace ll {

template <int DT>
LL_DEV float load_as_float(const void* p, int64_t i) {
  if (DT == 0) return reinterpret_cast<const float*>(p)[i];
  if (DT == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// sum_{sp < n} p[sp * stride], added in split order (the result of the plain loop); the loads of
// 8 splits are issued together instead of one at a time
LL_DEV float sum_splits(const float* __restrict__ p, int64_t stride, int n) {
  float s = 0.f;
  int sp = 0;
  for (; sp + 8 <= n; sp += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = p[(int64_t)(sp + j) * stride];
#pragma unroll
    for (int j = 0; j < 8; j++) s += v[j];
  }
  for (; sp < n; sp++) s += p[(int64_t)sp * stride];
  return s;
}

// ---------------------------------------------------------------- skinny split-K GEMM
// part[split][m][n] = sum_{k in split} A[m][k] * B(k, n) for the NC columns n = blockIdx.y * NC
// .. + NC - 1 (N a few tens: the LoRA rank, or twice it).
// B(k, n): BROWS -> n < N0 ? B0[n*K + k] : B1[(n-N0)*K + k]  ([N][K], e.g. LoRA A matrices)
//          else  -> B0[k*N + n]                             ([K][N], e.g. LoRA B matrices)
// Thread = 4 columns x TM rows (TM = 8 for 32-column blocks, 4 for 16): per k one 16-byte
// read of its 4 B values and TM/4 16-byte reads of its A values (shared by the lanes of the
// warp on the same rows), 4 TM FMAs. The A tile is staged transposed ([k][row]) from 16-byte
// global loads of 8 consecutive k, with the row index XOR-ed by 8 ((k / 8) % 4) so that the
// transposing stores hit 32 distinct banks while 8-row groups stay contiguous and aligned.
// K % 8 == 0; split boundaries are multiples of kSkBK.
constexpr int kSkBK = 32;

template <int NC>
struct SkinnyCfg {
  static constexpr int CQ = NC / 4;           // column quads
  static constexpr int RG = 256 / CQ;         // row groups
  static constexpr int TM = NC == 32 ? 8 : 4; // rows per thread
  static constexpr int BM = RG * TM;          // 256 rows per block
};

// 8 elements held as raw 16-byte words (two for fp32, one for bf16 / fp16) -> fp32
template <int ADT>
LL_DEV void words8_as_float(const uint4 (&u)[ADT == 0 ? 2 : 1], float (&v)[8]) {
  if constexpr (ADT == 0) {
    const uint32_t w[8] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y, u[1].z, u[1].w};
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __uint_as_float(w[j]);
  } else {
    const uint32_t w[4] = {u[0].x, u[0].y, u[0].z, u[0].w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float2 f;
      if (ADT == 1) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      else f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

LL_DEV int sk_swz(int k) { return ((k >> 3) & 3) << 3; }

template <int ADT, bool BROWS, int NC>
__global__ void __launch_bounds__(256) k_skinny(const void* __restrict__ A, int M, int K, int lda,
                                                const float* __restrict__ B0, const float* __restrict__ B1, int N0,
                                                int N, int kc, float* __restrict__ part) {
  pdl_wait();
  pdl_launch_next();
  using SC = SkinnyCfg<NC>;
  constexpr int TM = SC::TM;
  __shared__ __align__(16) float As[kSkBK][SC::BM + 4];
  __shared__ __align__(16) float Bs[kSkBK][NC];
  const int m0 = blockIdx.x * SC::BM, nb0 = blockIdx.y * NC;
  const int k_begin = blockIdx.z * kc, k_end = min(K, k_begin + kc);
  const int cq = threadIdx.x % SC::CQ, rg = threadIdx.x / SC::CQ;
  float acc[TM][4];
#pragma unroll
  for (int i = 0; i < TM; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  // the next k-step's A rows (raw 16-byte words) and B values are fetched into registers before
  // the current step's products, so their latency overlaps the FMAs; they are converted and
  // stored to shared memory at the top of the next step
  constexpr int LD = SC::BM * (kSkBK / 8) / 256;     // 8-element A loads per thread per step
  constexpr int LW = ADT == 0 ? 2 : 1;               // 16-byte words per 8 elements
  constexpr int BLD = NC * kSkBK / 256;              // B values per thread per step
  static_assert(SC::BM * (kSkBK / 8) % 256 == 0 && NC * kSkBK % 256 == 0, "thread cover");
  uint4 raw[LD][LW];
  float bv[BLD];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int l = 0; l < LD; l++) {
      const int i = threadIdx.x + l * 256;
      const int r = i / (kSkBK / 8), c8 = (i % (kSkBK / 8)) * 8;
      const int m = m0 + r, k = k0 + c8;
      const bool in = m < M && k < k_end;
#pragma unroll
      for (int w = 0; w < LW; w++) {
        const char* src = reinterpret_cast<const char*>(A) + ((int64_t)m * lda + k) * (ADT == 0 ? 4 : 2) + 16 * w;
        raw[l][w] = in ? *reinterpret_cast<const uint4*>(src) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int l = 0; l < BLD; l++) {
      const int i = threadIdx.x + l * 256;
      int n, c;
      if (BROWS) { n = i / kSkBK; c = i % kSkBK; } else { c = i / NC; n = i % NC; }
      const int k = k0 + c, ng = nb0 + n;
      float v = 0.f;
      if (ng < N && k < k_end) {
        if (BROWS) v = ng < N0 ? B0[(int64_t)ng * K + k] : B1[(int64_t)(ng - N0) * K + k];
        else v = B0[(int64_t)k * N + ng];
      }
      bv[l] = v;
    }
  };
  if (k_begin < k_end) fetch(k_begin);
  for (int k0 = k_begin; k0 < k_end; k0 += kSkBK) {
#pragma unroll
    for (int l = 0; l < LD; l++) {
      const int i = threadIdx.x + l * 256;
      const int r = i / (kSkBK / 8), c8 = (i % (kSkBK / 8)) * 8;
      float v[8];
      words8_as_float<ADT>(raw[l], v);
      const int rs = r ^ sk_swz(c8);
#pragma unroll
      for (int j = 0; j < 8; j++) As[c8 + j][rs] = v[j];
    }
#pragma unroll
    for (int l = 0; l < BLD; l++) {
      const int i = threadIdx.x + l * 256;
      int n, c;
      if (BROWS) { n = i / kSkBK; c = i % kSkBK; } else { c = i / NC; n = i % NC; }
      Bs[c][n] = bv[l];
    }
    __syncthreads();
    if (k0 + kSkBK < k_end) fetch(k0 + kSkBK);
#pragma unroll 4
    for (int kk = 0; kk < kSkBK; kk++) {
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][cq * 4]);
      const float* ar = &As[kk][(rg * TM) ^ sk_swz(kk)];
      float a[TM];
#pragma unroll
      for (int t = 0; t < TM; t += 4) {
        const float4 v = *reinterpret_cast<const float4*>(ar + t);
        a[t] = v.x; a[t + 1] = v.y; a[t + 2] = v.z; a[t + 3] = v.w;
      }
#pragma unroll
      for (int t = 0; t < TM; t++) {
        acc[t][0] = fmaf(a[t], b.x, acc[t][0]); acc[t][1] = fmaf(a[t], b.y, acc[t][1]);
        acc[t][2] = fmaf(a[t], b.z, acc[t][2]); acc[t][3] = fmaf(a[t], b.w, acc[t][3]);
      }
    }
    __syncthreads();
  }
  float* out = part + (int64_t)blockIdx.z * M * N;
#pragma unroll
  for (int t = 0; t < TM; t++) {
    const int m = m0 + rg * TM + t;
    if (m >= M) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int n = nb0 + cq * 4 + c;
      if (n < N) out[(int64_t)m * N + n] = acc[t][c];
    }
  }
}

// C[m][n] = alpha * sum_split part[split][m][n], split order fixed; n < N0 -> C0, else C1
__global__ void k_skinny_reduce(const float* __restrict__ part, int nsplit, int M, int N, int N0, float alpha,
                                float* __restrict__ C0, float* __restrict__ C1) {
  pdl_wait();
  pdl_launch_next();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  const float s = sum_splits(part + i, (int64_t)M * N, nsplit);
  const int m = (int)(i / N), n = (int)(i % N);
  if (n < N0) C0[(int64_t)m * N0 + n] = alpha * s;
  else C1[(int64_t)m * (N - N0) + (n - N0)] = alpha * s;
}

// ------------------------------------------------------------------ few-row products
// C0 / C1 [m][n] = alpha * sum_k A[m][k] B[n][k] with B given as rows ([N][K], split over B0 /
// B1 at N0), for few rows m: block (n, g) takes column n and rows g MR .. + MR - 1; its 256
// threads stride over K in 8-element steps, the 16-byte loads of UN steps issued before their
// FMAs, and the threads' partial sums are added in a fixed order (lanes by shuffle, then the 8
// warps in order). One launch, no split partials in global memory. K % 8 == 0, A and B 16-byte
// aligned.
template <int ADT, int MR>
__global__ void __launch_bounds__(256) k_gemv_rows(const void* __restrict__ A, int M, int K,
                                                   const float* __restrict__ B0, const float* __restrict__ B1, int N0,
                                                   int N, float alpha, float* __restrict__ C0, float* __restrict__ C1) {
  pdl_wait();
  pdl_launch_next();
  constexpr int LW = ADT == 0 ? 2 : 1;               // 16-byte words per 8 elements of A
  constexpr int ES = ADT == 0 ? 4 : 2;
  constexpr int UN = MR >= 16 ? 1 : MR >= 4 ? 4 : 8;  // K steps whose loads are issued together
  const int n = blockIdx.x, m0 = blockIdx.y * MR;
  const int mr = min(MR, M - m0);
  const float* b = n < N0 ? B0 + (int64_t)n * K : B1 + (int64_t)(n - N0) * K;
  const char* a = reinterpret_cast<const char*>(A) + (int64_t)m0 * K * ES;
  float acc[MR];
#pragma unroll
  for (int m = 0; m < MR; m++) acc[m] = 0.f;
  const int nch = K / 8;
  for (int c0 = threadIdx.x; c0 < nch; c0 += 256 * UN) {
    float4 bq[UN][2];
    uint4 raw[UN][MR][LW];
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const int c = c0 + 256 * u;
      const bool in = c < nch;
      bq[u][0] = in ? *reinterpret_cast<const float4*>(b + 8 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
      bq[u][1] = in ? *reinterpret_cast<const float4*>(b + 8 * c + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < MR; m++)
#pragma unroll
        for (int w = 0; w < LW; w++)
          raw[u][m][w] = (in && m < mr) ? *reinterpret_cast<const uint4*>(a + ((int64_t)m * K + 8 * c) * ES + 16 * w)
                                        : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const float bv[8] = {bq[u][0].x, bq[u][0].y, bq[u][0].z, bq[u][0].w,
                           bq[u][1].x, bq[u][1].y, bq[u][1].z, bq[u][1].w};
#pragma unroll
      for (int m = 0; m < MR; m++) {
        float av[8];
        words8_as_float<ADT>(raw[u][m], av);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[m] = fmaf(av[j], bv[j], acc[m]);
      }
    }
  }
  __shared__ float red[8][MR];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int m = 0; m < MR; m++) {
    float v = acc[m];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[warp][m] = v;
  }
  __syncthreads();
  if ((int)threadIdx.x < mr) {
    float sum = red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < 8; w++) sum += red[w][threadIdx.x];
    const int64_t m = m0 + threadIdx.x;
    if (n < N0) C0[m * N0 + n] = alpha * sum;
    else C1[m * (N - N0) + (n - N0)] = alpha * sum;
  }
}

// -------------------------------------------------------------------- rank-r expand
// out[t][c] = [sum_j Y[pos_j][c], pairs of t in ascending expert order]
//           + alpha * (sum_rr L0[t][rr] R0(rr, c) + sum_rr L1[t][rr] R1(rr, c))
// R(rr, c): RROWS -> R[rr*C + c] ([r][C]);  else R[c*r + rr] ([C][r]).
// Block: 512 columns (2 a thread, 8-byte loads and stores; 8 warps, so that the shared-memory
// bound occupancy of ~6 blocks per SM still keeps 48 warps streaming) x 8 tokens; the R slices
// of the block's columns are staged in shared memory once and reused by the 8 tokens, and a
// token's k rows of Y are all requested before the first is added (k <= 8 per batch).
constexpr int kExTok = 8, kExThreads = 256, kExCols = 2 * kExThreads;
// shared row pitch of the staged R slices: 4 floats of padding keep the float4 reads aligned and
// spread the transposing stores of a [C][r] R (16 consecutive rr of one column) over 8 banks
// instead of one
constexpr int kExPitch = kExCols + 4;

constexpr int kExMaxR = 64;

// The block's R slice into shared memory ([r][kExPitch]; columns >= nc zero), in batches of 8
// 16-byte loads a thread, so one batch's latency is paid once instead of once per element.
// q = the sum over a token's pair positions tp[0..k) (ascending expert; the first -1 ends the
// list) of tw[pos] * z[pos][rr], added in that order; eight positions' loads are issued together
// (one chain of two load latencies per eight pairs instead of two per pair).
LL_DEV float token_q(const int* __restrict__ tp, int k, const float* __restrict__ tw, const float* __restrict__ z,
                     int r, int rr) {
  float l = 0.f;
  for (int j0 = 0; j0 < k; j0 += 8) {
    int pos[8];
#pragma unroll
    for (int u = 0; u < 8; u++) pos[u] = j0 + u < k ? tp[j0 + u] : -1;
    float a[8], b[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      a[u] = pos[u] >= 0 ? tw[pos[u]] : 0.f;
      b[u] = pos[u] >= 0 ? z[(int64_t)pos[u] * r + rr] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      if (pos[u] < 0) return l;
      l = fmaf(a[u], b[u], l);
    }
  }
  return l;
}

template <bool RROWS>
LL_DEV void ex_stage_r(float* Rs, const float* __restrict__ R, int r, int C, int c0, int nc) {
  const int tid = threadIdx.x;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool vec = (reinterpret_cast<uintptr_t>(R) & 15) == 0 && (RROWS || (r & 3) == 0);
  if (RROWS && vec) {
    // 16-byte chunk f: row f / (kExCols / 4) of R, columns 4 (f % (kExCols / 4)) .. + 3
    constexpr int CPR = kExCols / 4;
    const int nchunk = r * CPR;
    for (int f0 = tid; f0 < nchunk; f0 += 8 * kExThreads) {
      float4 v[8];
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const int f = f0 + b * kExThreads;
        const int rr = f / CPR, cc = (f % CPR) * 4;
        v[b] = (f < nchunk && cc < nc) ? *reinterpret_cast<const float4*>(R + (int64_t)rr * C + c0 + cc) : z4;
      }
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const int f = f0 + b * kExThreads;
        if (f < nchunk) *reinterpret_cast<float4*>(Rs + (f / CPR) * kExPitch + (f % CPR) * 4) = v[b];
      }
    }
  } else if (vec) {
    // [C][r]: the block's columns are one contiguous run; 16-byte chunk f holds column 4 f / r,
    // ranks 4 f % r .. + 3 (r % 4 == 0)
    const float* base = R + (int64_t)c0 * r;
    const int nchunk = kExCols * r / 4;
    for (int f0 = tid; f0 < nchunk; f0 += 8 * kExThreads) {
      float4 v[8];
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const int f = f0 + b * kExThreads;
        v[b] = (f < nchunk && (4 * f) / r < nc) ? *reinterpret_cast<const float4*>(base + 4 * (int64_t)f) : z4;
      }
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const int f = f0 + b * kExThreads;
        if (f < nchunk) {
          const int cc = (4 * f) / r, rr = (4 * f) % r;
          Rs[rr * kExPitch + cc] = v[b].x;
          Rs[(rr + 1) * kExPitch + cc] = v[b].y;
          Rs[(rr + 2) * kExPitch + cc] = v[b].z;
          Rs[(rr + 3) * kExPitch + cc] = v[b].w;
        }
      }
    }
  } else if (RROWS) {
    for (int i = tid; i < r * kExCols; i += kExThreads) {
      const int rr = i / kExCols, cc = i % kExCols;
      Rs[rr * kExPitch + cc] = cc < nc ? R[(int64_t)rr * C + c0 + cc] : 0.f;
    }
  } else {
    for (int i = tid; i < r * kExCols; i += kExThreads) {
      const int cc = i / r, rr = i % r;
      Rs[rr * kExPitch + cc] = cc < nc ? R[(int64_t)(c0 + cc) * r + rr] : 0.f;
    }
  }
}

template <bool RROWS, bool HASY, bool TWO>
__global__ void __launch_bounds__(kExThreads) k_expand(const int* __restrict__ tok_pos, const float* __restrict__ Y, int k,
                                                   int T, int C, int r, float alpha, const float* __restrict__ L0,
                                                   const float* __restrict__ R0, const float* __restrict__ L1,
                                                   const float* __restrict__ R1, float* __restrict__ out,
                                                   float* __restrict__ out1, const float* __restrict__ qtw,
                                                   const float* __restrict__ qz, float* __restrict__ q_out) {
  // gridDim.z == 2 (one product, TWO false): blocks z = 1 compute out1 = alpha L1 R1 instead
  if (!TWO && blockIdx.z == 1) {
    L0 = L1;
    R0 = R1;
    out = out1;
  }
  extern __shared__ float Rs[];                          // [r][kExPitch], one R at a time
  __shared__ float Ls[kExTok][kExMaxR];
  __shared__ int ps[kExTok][32];
  const int c0 = blockIdx.x * kExCols, t0 = blockIdx.y * kExTok;
  const int nc = min(kExCols, C - c0);
  const int c = 2 * threadIdx.x;
  // The first R is a LoRA weight (every caller passes the layer's adapters), written before the
  // kernels this launch follows had passed their own waits: its slice is staged before the wait,
  // overlapping the predecessor.
  ex_stage_r<RROWS>(Rs, R0, r, C, c0, nc);
  pdl_wait();
  pdl_launch_next();
  if (HASY)
    for (int i = threadIdx.x; i < kExTok * k; i += kExThreads) {
      const int tt = i / k, j = i % k;
      ps[tt][j] = (t0 + tt < T) ? tok_pos[(int64_t)(t0 + tt) * k + j] : -1;
    }
  float2 lo[kExTok];
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) lo[tt] = make_float2(0.f, 0.f);
  for (int w = 0; w < (TWO ? 2 : 1); w++) {
    const float* Lm = w == 0 ? L0 : L1;
    if (w > 0) {
      __syncthreads();                                   // the previous R is no longer read
      ex_stage_r<RROWS>(Rs, R1, r, C, c0, nc);
    }
    for (int i = threadIdx.x; i < kExTok * r; i += kExThreads) {
      const int tt = i / r, rr = i % r;
      float l = 0.f;
      if (t0 + tt < T) {
        if (qz) {
          // L0 = q: q[t][rr] = sum over the token's pairs (ascending expert) of tw * z
          l = token_q(tok_pos + (int64_t)(t0 + tt) * k, k, qtw, qz, r, rr);
          if (q_out && blockIdx.x == 0) q_out[(int64_t)(t0 + tt) * r + rr] = l;
        } else {
          l = Lm[(int64_t)(t0 + tt) * r + rr];
        }
      }
      Ls[tt][rr] = l;
    }
    __syncthreads();
    if (c < nc)
      for (int rr = 0; rr < r; rr++) {
        const float2 rv = *reinterpret_cast<const float2*>(Rs + rr * kExPitch + c);
#pragma unroll
        for (int tt = 0; tt < kExTok; tt++) {
          const float l = Ls[tt][rr];
          lo[tt].x = fmaf(l, rv.x, lo[tt].x); lo[tt].y = fmaf(l, rv.y, lo[tt].y);
        }
      }
  }
  if (c >= nc) return;
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) {
    if (t0 + tt >= T) break;
    float2 acc = make_float2(0.f, 0.f);
    if (HASY) {
      for (int j0 = 0; j0 < k; j0 += 8) {
        float2 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // all requests first
          const int p = j0 + j < k ? ps[tt][j0 + j] : -1;
          v[j] = p >= 0 ? *reinterpret_cast<const float2*>(Y + (int64_t)p * C + c0 + c) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // then the sum, in slot order
          acc.x += v[j].x; acc.y += v[j].y;
        }
      }
    }
    float2 o;
    o.x = acc.x + alpha * lo[tt].x; o.y = acc.y + alpha * lo[tt].y;
    *reinterpret_cast<float2*>(out + (int64_t)(t0 + tt) * C + c0 + c) = o;
  }
}

// The latent block's combine with its RMSNorm in one pass (the sum of a token's expert rows,
// lazy_trainer.py:729-731, then routed_expert_norm, :731-733): a block takes 8 tokens and every
// column, in 512-column slices (the R slice staged in shared memory per slice, as k_expand):
//   out[t][c]    = [sum_j Y[pos_j][c], pairs of t in ascending expert order] + alpha (q[t] . R)(c),
//                  q[t] = sum over the token's pairs of qtw * qz (stored to q_out by the block);
//   rstd[t]      = rsqrt(mean_c out[t][c]^2 + eps), the squares summed per thread over its
//                  columns, then across the block in a fixed order;
//   normed[t][c] = bf16(out[t][c] * rstd[t] * norm_w[c]).
// The sums of each out element are those of k_expand, bit for bit. A thread re-reads only the
// columns it wrote.
template <bool RROWS>
__global__ void __launch_bounds__(kExThreads) k_expand_norm(const int* __restrict__ tok_pos, const float* __restrict__ Y,
                                                        int k, int T, int C, int r, float alpha,
                                                        const float* __restrict__ R0, const float* __restrict__ qtw,
                                                        const float* __restrict__ qz, float* __restrict__ q_out,
                                                        float* __restrict__ out, const float* __restrict__ norm_w,
                                                        float eps, __nv_bfloat16* __restrict__ normed,
                                                        float* __restrict__ rstd) {
  pdl_wait();
  pdl_launch_next();
  extern __shared__ float Rs[];                          // [r][kExPitch], one slice at a time
  __shared__ float Ls[kExTok][kExMaxR];
  __shared__ int ps[kExTok][32];
  __shared__ float red[kExThreads / 32][kExTok];
  __shared__ float rs[kExTok];
  const int t0 = blockIdx.x * kExTok;
  const int c = 2 * threadIdx.x;
  for (int i = threadIdx.x; i < kExTok * k; i += kExThreads) {
    const int tt = i / k, j = i % k;
    ps[tt][j] = (t0 + tt < T) ? tok_pos[(int64_t)(t0 + tt) * k + j] : -1;
  }
  for (int i = threadIdx.x; i < kExTok * r; i += kExThreads) {
    const int tt = i / r, rr = i % r;
    float l = 0.f;
    if (t0 + tt < T) {
      l = token_q(tok_pos + (int64_t)(t0 + tt) * k, k, qtw, qz, r, rr);
      if (q_out) q_out[(int64_t)(t0 + tt) * r + rr] = l;
    }
    Ls[tt][rr] = l;
  }
  float ss[kExTok];
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) ss[tt] = 0.f;
  for (int c0 = 0; c0 < C; c0 += kExCols) {
    const int nc = min(kExCols, C - c0);
    __syncthreads();                                     // Ls / ps ready; the previous slice no longer read
    ex_stage_r<RROWS>(Rs, R0, r, C, c0, nc);
    __syncthreads();
    if (c >= nc) continue;
    float2 lo[kExTok];
#pragma unroll
    for (int tt = 0; tt < kExTok; tt++) lo[tt] = make_float2(0.f, 0.f);
    for (int rr = 0; rr < r; rr++) {
      const float2 rv = *reinterpret_cast<const float2*>(Rs + rr * kExPitch + c);
#pragma unroll
      for (int tt = 0; tt < kExTok; tt++) {
        const float l = Ls[tt][rr];
        lo[tt].x = fmaf(l, rv.x, lo[tt].x); lo[tt].y = fmaf(l, rv.y, lo[tt].y);
      }
    }
#pragma unroll
    for (int tt = 0; tt < kExTok; tt++) {
      if (t0 + tt >= T) break;
      float2 acc = make_float2(0.f, 0.f);
      for (int j0 = 0; j0 < k; j0 += 8) {
        float2 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // all requests first
          const int p = j0 + j < k ? ps[tt][j0 + j] : -1;
          v[j] = p >= 0 ? *reinterpret_cast<const float2*>(Y + (int64_t)p * C + c0 + c) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // then the sum, in slot order
          acc.x += v[j].x; acc.y += v[j].y;
        }
      }
      float2 o;
      o.x = acc.x + alpha * lo[tt].x; o.y = acc.y + alpha * lo[tt].y;
      *reinterpret_cast<float2*>(out + (int64_t)(t0 + tt) * C + c0 + c) = o;
      ss[tt] = fmaf(o.y, o.y, fmaf(o.x, o.x, ss[tt]));
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) {
    float v = ss[tt];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[warp][tt] = v;
  }
  __syncthreads();
  if (threadIdx.x < kExTok) {
    const int tt = threadIdx.x;
    float tot = red[0][tt];
    for (int wi = 1; wi < kExThreads / 32; wi++) tot += red[wi][tt];
    const float rv = rsqrtf(tot / (float)C + eps);
    rs[tt] = rv;
    if (t0 + tt < T) rstd[t0 + tt] = rv;
  }
  __syncthreads();
  for (int c0 = 0; c0 < C; c0 += kExCols) {
    const int nc = min(kExCols, C - c0);
    if (c >= nc) continue;
    const float2 wv = *reinterpret_cast<const float2*>(norm_w + c0 + c);
#pragma unroll
    for (int tt = 0; tt < kExTok; tt++) {
      if (t0 + tt >= T) break;
      const float2 o = *reinterpret_cast<const float2*>(out + (int64_t)(t0 + tt) * C + c0 + c);
      const float rv = rs[tt];
      *reinterpret_cast<__nv_bfloat162*>(normed + (int64_t)(t0 + tt) * C + c0 + c) =
          __floats2bfloat162_rn(o.x * rv * wv.x, o.y * rv * wv.y);
    }
  }
}

// --------------------------------------------------------------- outer-product sums
// part[seg][rr][c] = sum_{n in seg} Pm(n, rr) * Q[n][c] for the ranks rr = kOuRB blockIdx.z ..
// + kOuRB - 1 and the 128 columns of blockIdx.x. Pm: [N][r] fp32, or (PGATHER) tw[n] *
// Pm[perm_token[n]][rr]. Q dtype QDT (0 f32, 1 bf16, 2 f16), C % 4 == 0.
// Block = 8 warps, lane = 4 consecutive columns; the 8 warps take interleaved batches of
// kOuNB rows n of the segment (a batch's Q loads issued before its FMAs, and for 16-bit Q the
// next batch's during them), then their sums are added in warp order through shared memory.
constexpr int kOuRB = 16, kOuCW = 128, kOuNB = 4;

// 4 consecutive Q elements as raw words (fp32: uint4; bf16 / fp16: uint2), loaded now and
// converted by raw4_as_float when used, so the conversion does not wait on the load
template <int QDT>
struct QRaw {
  using T = uint2;
};
template <>
struct QRaw<0> {
  using T = uint4;
};

template <int QDT>
LL_DEV typename QRaw<QDT>::T load4_raw(const void* Q, int64_t off) {
  if constexpr (QDT == 0) return *reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(Q) + off);
  else return *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(Q) + off);
}

template <int QDT>
LL_DEV typename QRaw<QDT>::T raw_zero() {
  if constexpr (QDT == 0) return make_uint4(0u, 0u, 0u, 0u);
  else return make_uint2(0u, 0u);
}

template <int QDT>
LL_DEV float4 raw4_as_float(const typename QRaw<QDT>::T v) {
  if constexpr (QDT == 0) {
    return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
  } else {
    float2 a, b;
    if (QDT == 1) {
      a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
      b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
    } else {
      a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    }
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

template <int QDT, bool PGATHER>
__global__ void __launch_bounds__(256) k_outer8(const float* __restrict__ Pm, const int* __restrict__ perm_token,
                                                const float* __restrict__ tw, const void* __restrict__ Q, int N,
                                                const int* __restrict__ n_dev, int C, int r, int nseg,
                                                float* __restrict__ part) {
  pdl_wait();
  pdl_launch_next();
  extern __shared__ float4 red4[];                    // [8 warps][kOuRB][32 lanes] float4
  __shared__ __align__(16) float ps[8][kOuNB][kOuRB];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = blockIdx.x * kOuCW + lane * 4;
  const bool cok = c < C;
  const int seg = blockIdx.y;
  const int rb = blockIdx.z * kOuRB, rn = min(kOuRB, r - rb);
  const int n_total = n_dev ? *n_dev : N;
  const int per = (n_total + nseg - 1) / nseg;
  const int n0 = seg * per, n1 = min(n_total, n0 + per);
  float4 acc[kOuRB];
#pragma unroll
  for (int i = 0; i < kOuRB; i++) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  // software pipeline over this warp's batches of kOuNB rows: the next batch's Q words and Pm
  // values are requested before the current batch's FMAs (16-bit Q; fp32 Q, twice the
  // registers, requests each batch's rows just before staging its Pm)
  constexpr bool PIPE = QDT != 0;
  auto pm_val = [&](int nb, int i) {
    const int nn = i / kOuRB, rr = i % kOuRB;
    const int n = nb + nn;
    float v = 0.f;
    if (n < n1 && rr < rn) v = PGATHER ? tw[n] * Pm[(int64_t)perm_token[n] * r + rb + rr] : Pm[(int64_t)n * r + rb + rr];
    return v;
  };
  constexpr int PV = kOuNB * kOuRB / 32;              // Pm values a lane stages per batch
  typename QRaw<QDT>::T qr[kOuNB];
  float pv[PV];
  int nb = n0 + warp * kOuNB;
  if (PIPE && nb < n1) {
#pragma unroll
    for (int nn = 0; nn < kOuNB; nn++)
      qr[nn] = (cok && nb + nn < n1) ? load4_raw<QDT>(Q, (int64_t)(nb + nn) * C + c) : raw_zero<QDT>();
#pragma unroll
    for (int j = 0; j < PV; j++) pv[j] = pm_val(nb, lane + 32 * j);
  }
  for (; nb < n1; nb += 8 * kOuNB) {
    if (!PIPE) {
#pragma unroll
      for (int nn = 0; nn < kOuNB; nn++)
        qr[nn] = (cok && nb + nn < n1) ? load4_raw<QDT>(Q, (int64_t)(nb + nn) * C + c) : raw_zero<QDT>();
#pragma unroll
      for (int j = 0; j < PV; j++) pv[j] = pm_val(nb, lane + 32 * j);
    }
#pragma unroll
    for (int j = 0; j < PV; j++) {
      const int i = lane + 32 * j;
      ps[warp][i / kOuRB][i % kOuRB] = pv[j];
    }
    __syncwarp();
    typename QRaw<QDT>::T qc[kOuNB];
#pragma unroll
    for (int nn = 0; nn < kOuNB; nn++) qc[nn] = qr[nn];
    const int nx = nb + 8 * kOuNB;                   // this warp's next batch
    if (PIPE && nx < n1) {
#pragma unroll
      for (int nn = 0; nn < kOuNB; nn++)
        qr[nn] = (cok && nx + nn < n1) ? load4_raw<QDT>(Q, (int64_t)(nx + nn) * C + c) : raw_zero<QDT>();
#pragma unroll
      for (int j = 0; j < PV; j++) pv[j] = pm_val(nx, lane + 32 * j);
    }
#pragma unroll
    for (int nn = 0; nn < kOuNB; nn++) {
      const float4 q = raw4_as_float<QDT>(qc[nn]);
#pragma unroll
      for (int i = 0; i < kOuRB; i += 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(&ps[warp][nn][i]);
        const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
          acc[i + u].x = fmaf(pp[u], q.x, acc[i + u].x);
          acc[i + u].y = fmaf(pp[u], q.y, acc[i + u].y);
          acc[i + u].z = fmaf(pp[u], q.z, acc[i + u].z);
          acc[i + u].w = fmaf(pp[u], q.w, acc[i + u].w);
        }
      }
    }
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < kOuRB; i++) red4[(warp * kOuRB + i) * 32 + lane] = acc[i];
  __syncthreads();
  // thread -> (rank i, lane l): the 8 warps' sums in warp order
  for (int o = threadIdx.x; o < kOuRB * 32; o += 256) {
    const int i = o / 32, l = o % 32;
    const int cc = blockIdx.x * kOuCW + l * 4;
    if (i >= rn || cc >= C) continue;
    float4 s = red4[i * 32 + l];
#pragma unroll
    for (int w = 1; w < 8; w++) {
      const float4 t = red4[(w * kOuRB + i) * 32 + l];
      s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
    }
    *reinterpret_cast<float4*>(part + ((int64_t)seg * r + rb + i) * C + cc) = s;
  }
}

}  // namespace ll
