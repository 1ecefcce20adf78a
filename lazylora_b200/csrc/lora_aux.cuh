// Small dense kernels around the grouped GEMMs: the rank-r LoRA products and the weighted
// combines. All reductions run in a fixed order (split-K partials summed by a second pass),
// so results are bitwise reproducible.
#pragma once
#include "common.cuh"

namespace ll {

template <int DT>
LL_DEV float load_as_float(const void* p, int64_t i) {
  if (DT == 0) return reinterpret_cast<const float*>(p)[i];
  if (DT == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// ---------------------------------------------------------------- skinny split-K GEMM
// part[split][m][n] = sum_{k in split} A[m][k] * B(k, n); blockIdx.y picks 32 of the N columns.
// B(k, n): BROWS -> n < N0 ? B0[n*K + k] : B1[(n-N0)*K + k]  ([N][K], e.g. LoRA A matrices)
//          else  -> B0[k*N + n]                             ([K][N], e.g. LoRA B matrices)
// Tile 64 rows x 32 columns x 64 k per step; thread = 2 rows x 4 columns.
constexpr int kSkBM = 64, kSkBN = 32, kSkBK = 64;

template <int ADT, bool BROWS>
__global__ void __launch_bounds__(256) k_skinny(const void* __restrict__ A, int M, int K, int lda,
                                                const float* __restrict__ B0, const float* __restrict__ B1, int N0,
                                                int N, int kc, float* __restrict__ part) {
  __shared__ float As[kSkBK][kSkBM + 4];
  __shared__ float Bs[kSkBK][kSkBN + 4];
  const int m0 = blockIdx.x * kSkBM, nb0 = blockIdx.y * kSkBN;
  const int k_begin = blockIdx.z * kc, k_end = min(K, k_begin + kc);
  const int tm = threadIdx.x / 8, tn = threadIdx.x % 8;   // rows tm, tm+32; columns 4tn..4tn+3
  float acc[2][4] = {};
  for (int k0 = k_begin; k0 < k_end; k0 += kSkBK) {
    for (int i = threadIdx.x; i < kSkBM * kSkBK; i += 256) {
      const int r = i / kSkBK, c = i % kSkBK;
      const int m = m0 + r, k = k0 + c;
      As[c][r] = (m < M && k < k_end) ? load_as_float<ADT>(A, (int64_t)m * lda + k) : 0.f;
    }
    for (int i = threadIdx.x; i < kSkBN * kSkBK; i += 256) {
      int n, c;
      if (BROWS) { n = i / kSkBK; c = i % kSkBK; } else { c = i / kSkBN; n = i % kSkBN; }
      const int k = k0 + c, ng = nb0 + n;
      float v = 0.f;
      if (ng < N && k < k_end) {
        if (BROWS) v = ng < N0 ? B0[(int64_t)ng * K + k] : B1[(int64_t)(ng - N0) * K + k];
        else v = B0[(int64_t)k * N + ng];
      }
      Bs[c][n] = v;
    }
    __syncthreads();
#pragma unroll 16
    for (int kk = 0; kk < kSkBK; kk++) {
      const float a0 = As[kk][tm], a1 = As[kk][tm + 32];
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tn * 4]);
      acc[0][0] = fmaf(a0, b.x, acc[0][0]); acc[0][1] = fmaf(a0, b.y, acc[0][1]);
      acc[0][2] = fmaf(a0, b.z, acc[0][2]); acc[0][3] = fmaf(a0, b.w, acc[0][3]);
      acc[1][0] = fmaf(a1, b.x, acc[1][0]); acc[1][1] = fmaf(a1, b.y, acc[1][1]);
      acc[1][2] = fmaf(a1, b.z, acc[1][2]); acc[1][3] = fmaf(a1, b.w, acc[1][3]);
    }
    __syncthreads();
  }
  float* out = part + (int64_t)blockIdx.z * M * N;
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int m = m0 + tm + 32 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = nb0 + tn * 4 + j;
      if (n < N) out[(int64_t)m * N + n] = acc[i][j];
    }
  }
}

// C[m][n] = alpha * sum_split part[split][m][n], split order fixed; n < N0 -> C0, else C1
__global__ void k_skinny_reduce(const float* __restrict__ part, int nsplit, int M, int N, int N0, float alpha,
                                float* __restrict__ C0, float* __restrict__ C1) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  float s = 0.f;
  for (int sp = 0; sp < nsplit; sp++) s += part[(int64_t)sp * M * N + i];
  const int m = (int)(i / N), n = (int)(i % N);
  if (n < N0) C0[(int64_t)m * N0 + n] = alpha * s;
  else C1[(int64_t)m * (N - N0) + (n - N0)] = alpha * s;
}

// -------------------------------------------------------------------- rank-r expand
// out[t][c] = [sum_j Y[pos_j][c], pairs of t in ascending expert order]
//           + alpha * (sum_rr L0[t][rr] R0(rr, c) + sum_rr L1[t][rr] R1(rr, c))
// R(rr, c): RROWS -> R[rr*C + c] ([r][C]);  else R[c*r + rr] ([C][r]).
// Block: 512 columns (4 a thread, 16-byte loads and stores) x 8 tokens; the R slices of the
// block's columns are staged in shared memory once and reused by the 8 tokens, and a
// token's k rows of Y are all requested before the first is added (k <= 8 per batch), so the
// kernel streams Y at memory speed instead of one dependent load at a time.
constexpr int kExTok = 8, kExThreads = 128, kExCols = 4 * kExThreads;

constexpr int kExMaxR = 64;

template <bool RROWS, bool HASY, bool TWO>
__global__ void __launch_bounds__(kExThreads) k_expand(const int* __restrict__ tok_pos, const float* __restrict__ Y, int k,
                                                   int T, int C, int r, float alpha, const float* __restrict__ L0,
                                                   const float* __restrict__ R0, const float* __restrict__ L1,
                                                   const float* __restrict__ R1, float* __restrict__ out) {
  extern __shared__ float Rs[];                          // [r][kExCols], one R at a time
  __shared__ float Ls[kExTok][kExMaxR];
  __shared__ int ps[kExTok][32];
  const int c0 = blockIdx.x * kExCols, t0 = blockIdx.y * kExTok;
  const int nc = min(kExCols, C - c0);
  const int c = 4 * threadIdx.x;
  if (HASY)
    for (int i = threadIdx.x; i < kExTok * k; i += kExThreads) {
      const int tt = i / k, j = i % k;
      ps[tt][j] = (t0 + tt < T) ? tok_pos[(int64_t)(t0 + tt) * k + j] : -1;
    }
  float4 lo[kExTok];
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) lo[tt] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int w = 0; w < (TWO ? 2 : 1); w++) {
    const float* R = w == 0 ? R0 : R1;
    const float* Lm = w == 0 ? L0 : L1;
    __syncthreads();                                     // the previous R is no longer read
    if (RROWS) {
      for (int i = threadIdx.x; i < r * kExCols; i += kExThreads) {
        const int rr = i / kExCols, cc = i % kExCols;
        Rs[rr * kExCols + cc] = cc < nc ? R[(int64_t)rr * C + c0 + cc] : 0.f;
      }
    } else {   // [C][r]: the block's columns are one contiguous run of kExCols * r floats
      for (int i = threadIdx.x; i < r * kExCols; i += kExThreads) {
        const int cc = i / r, rr = i % r;
        Rs[rr * kExCols + cc] = cc < nc ? R[(int64_t)(c0 + cc) * r + rr] : 0.f;
      }
    }
    for (int i = threadIdx.x; i < kExTok * r; i += kExThreads) {
      const int tt = i / r, rr = i % r;
      Ls[tt][rr] = (t0 + tt < T) ? Lm[(int64_t)(t0 + tt) * r + rr] : 0.f;
    }
    __syncthreads();
    if (c < nc)
      for (int rr = 0; rr < r; rr++) {
        const float4 rv = *reinterpret_cast<const float4*>(Rs + rr * kExCols + c);
#pragma unroll
        for (int tt = 0; tt < kExTok; tt++) {
          const float l = Ls[tt][rr];
          lo[tt].x = fmaf(l, rv.x, lo[tt].x); lo[tt].y = fmaf(l, rv.y, lo[tt].y);
          lo[tt].z = fmaf(l, rv.z, lo[tt].z); lo[tt].w = fmaf(l, rv.w, lo[tt].w);
        }
      }
  }
  if (c >= nc) return;
#pragma unroll
  for (int tt = 0; tt < kExTok; tt++) {
    if (t0 + tt >= T) break;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (HASY) {
      for (int j0 = 0; j0 < k; j0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // all requests first
          const int p = j0 + j < k ? ps[tt][j0 + j] : -1;
          v[j] = p >= 0 ? *reinterpret_cast<const float4*>(Y + (int64_t)p * C + c0 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {                    // then the sum, in slot order
          acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
        }
      }
    }
    float4 o;
    o.x = acc.x + alpha * lo[tt].x; o.y = acc.y + alpha * lo[tt].y;
    o.z = acc.z + alpha * lo[tt].z; o.w = acc.w + alpha * lo[tt].w;
    *reinterpret_cast<float4*>(out + (int64_t)(t0 + tt) * C + c0 + c) = o;
  }
}

// --------------------------------------------------------------- outer-product sums
// part[seg][rr][c] = sum_{n in seg} Pm(n, rr) * Q[n][c]; 4 consecutive columns per thread,
// ranks rr = 32 blockIdx.z .. + 31 (any r, 32 at a time).
// Pm: [N][r] fp32, or (PGATHER) tw[n] * Pm[perm_token[n]][rr]. Q dtype QDT (0 f32, 1 bf16, 2 f16).
template <int QDT, bool PGATHER>
__global__ void __launch_bounds__(64) k_outer4(const float* __restrict__ Pm, const int* __restrict__ perm_token,
                                               const float* __restrict__ tw, const void* __restrict__ Q, int N,
                                               const int* __restrict__ n_dev, int C, int r, int nseg,
                                               float* __restrict__ part) {
  const int c = (blockIdx.x * 64 + threadIdx.x) * 4;
  const int seg = blockIdx.y;
  const int rb = blockIdx.z * 32, rn = min(32, r - rb);   // this block's ranks
  const int n_total = n_dev ? *n_dev : N;
  const int per = (n_total + nseg - 1) / nseg;
  const int n0 = seg * per, n1 = min(n_total, n0 + per);
  __shared__ float ps[16][33];
  float acc[32][4];
#pragma unroll
  for (int i = 0; i < 32; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  for (int nb = n0; nb < n1; nb += 16) {
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * rn; i += 64) {
      const int nn = i / rn, rr = i % rn;
      const int n = nb + nn;
      float v = 0.f;
      if (n < n1) v = PGATHER ? tw[n] * Pm[(int64_t)perm_token[n] * r + rb + rr] : Pm[(int64_t)n * r + rb + rr];
      ps[nn][rr] = v;
    }
    __syncthreads();
    if (c < C) {
      const int lim = min(16, n1 - nb);
#pragma unroll 4
      for (int nn = 0; nn < lim; nn++) {
        const int64_t o = (int64_t)(nb + nn) * C + c;
        float q0, q1, q2, q3;
        if (QDT == 0) {
          const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(Q) + o);
          q0 = v.x; q1 = v.y; q2 = v.z; q3 = v.w;
        } else if (QDT == 1) {
          const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(Q) + o);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
          q0 = a.x; q1 = a.y; q2 = b.x; q3 = b.y;
        } else {
          const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(Q) + o);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
          const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
          q0 = a.x; q1 = a.y; q2 = b.x; q3 = b.y;
        }
#pragma unroll
        for (int i = 0; i < 32; i++) {
          if (i < rn) {
            const float p = ps[nn][i];
            acc[i][0] = fmaf(p, q0, acc[i][0]);
            acc[i][1] = fmaf(p, q1, acc[i][1]);
            acc[i][2] = fmaf(p, q2, acc[i][2]);
            acc[i][3] = fmaf(p, q3, acc[i][3]);
          }
        }
      }
    }
  }
  if (c < C) {
#pragma unroll
    for (int i = 0; i < 32; i++)
      if (i < rn)
        *reinterpret_cast<float4*>(part + ((int64_t)seg * r + rb + i) * C + c) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
}

}  // namespace ll
