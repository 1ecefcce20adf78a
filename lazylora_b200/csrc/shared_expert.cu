// The element-wise middle of the shared expert (Kimi K3's dense SiTU-GLU MLP with LoRA on its
// three projections, lazy_lora/trainer/lazy_trainer.py:702-707), between its bf16 GEMMs:
//
// forward:  sg = bf16(G + bf16(s * xa_g . B_g^T)),  su = bf16(U + bf16(s * xa_u . B_u^T)),
//           h  = bf16(situ_glu(sg, su))
//   G, U: the bf16 gate / up projections x W^T; xa = x A^T [N, r] fp32 (the LoRA A product);
//   B [F, r] fp32; the LoRA deltas are added in bf16 as the reference adds the two bf16
//   tensors; SiTU-GLU in fp32 on the bf16 inputs, rounded to bf16 (situ_activation.py:47-75).
// backward: dh = bf16(Dh + bf16(s * gB . A_d)),  (dsg, dsu) = bf16(situ_glu_backward(dh, sg, su))
//   Dh: the bf16 input gradient of the down projection (g W_d); gB = g B_d [N, r] fp32;
//   A_d [r, F] fp32 (the down adapter's A, whose input is h).
// Block: 256 columns x 32 tokens; a thread keeps its column's r adapter values in registers and
// reads the tokens' r-vectors from shared memory.
//
// Also here, the C-ABI of the LoRA products around such bf16 GEMMs (the shared expert's, or any
// dense projection's), which read the bf16 activations directly instead of an fp32 copy:
//   ll_lora_down      C = alpha * X . B   (X [M][K] bf16/f16/f32; B: the rank-r A matrices as
//                     rows, or a B matrix as columns), split-K with a fixed-order sum
//   ll_lora_outer     out = scale * sum_n P[n]^T Q[n]  (the adapter gradients dA, dB)
//   ll_lora_add_bf16  out = bf16(Y + bf16(scale * L0 . R0) [+ bf16(scale * L1 . R1)]): the bf16
//                     projection output plus its rounded LoRA delta(s), as the reference adds
//                     the two bf16 tensors (lora_layer.py:104-123)
#include "host_common.cuh"
#include "lora_ops.cuh"

namespace ll {

constexpr int kSgCols = 256, kSgTok = 32, kSgB = 4;

LL_DEV float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Tokens t0 .. t0 + kSgTok - 1 in batches of kSgB: a batch's bf16 inputs are all requested
// (predicated, no early exit) before the first is used, so kSgB loads per input are in flight.
template <int R>
__global__ void __launch_bounds__(kSgCols) k_shared_glu_fwd(const __nv_bfloat16* __restrict__ G,
                                                            const __nv_bfloat16* __restrict__ U,
                                                            const float* __restrict__ xa_g, const float* __restrict__ xa_u,
                                                            const float* __restrict__ Bg, const float* __restrict__ Bu,
                                                            float s, int N, int F, __nv_bfloat16* __restrict__ SG,
                                                            __nv_bfloat16* __restrict__ SU, __nv_bfloat16* __restrict__ H) {
  __shared__ float la[kSgTok][2 * R];
  const int j = blockIdx.x * kSgCols + threadIdx.x;
  const int t0 = blockIdx.y * kSgTok;
  for (int i = threadIdx.x; i < kSgTok * 2 * R; i += kSgCols) {
    const int tt = i / (2 * R), rr = i % (2 * R);
    const int t = t0 + tt;
    la[tt][rr] = t < N ? (rr < R ? xa_g[(int64_t)t * R + rr] : xa_u[(int64_t)t * R + rr - R]) : 0.f;
  }
  __syncthreads();
  if (j >= F) return;
  float bg[R], bu[R];
#pragma unroll
  for (int rr = 0; rr < R; rr++) {
    bg[rr] = Bg[(int64_t)j * R + rr];
    bu[rr] = Bu[(int64_t)j * R + rr];
  }
  for (int tb = 0; tb < kSgTok && t0 + tb < N; tb += kSgB) {
    float gv[kSgB], uv[kSgB];
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      const int64_t o = (int64_t)t * F + j;
      gv[q] = t < N ? __bfloat162float(G[o]) : 0.f;
      uv[q] = t < N ? __bfloat162float(U[o]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      if (t >= N) break;
      float dg = 0.f, du = 0.f;
#pragma unroll
      for (int rr = 0; rr < R; rr++) {
        dg = fmaf(la[tb + q][rr], bg[rr], dg);
        du = fmaf(la[tb + q][R + rr], bu[rr], du);
      }
      const int64_t o = (int64_t)t * F + j;
      const float sg = bf16r(gv[q] + bf16r(s * dg));
      const float su = bf16r(uv[q] + bf16r(s * du));
      SG[o] = __float2bfloat16_rn(sg);
      SU[o] = __float2bfloat16_rn(su);
      H[o] = __float2bfloat16_rn(situ_glu_fwd(sg, su));
    }
  }
}

template <int R>
__global__ void __launch_bounds__(kSgCols) k_shared_glu_bwd(const __nv_bfloat16* __restrict__ Dh,
                                                            const float* __restrict__ gB, const float* __restrict__ Ad,
                                                            float s, const __nv_bfloat16* __restrict__ SG,
                                                            const __nv_bfloat16* __restrict__ SU, int N, int F,
                                                            __nv_bfloat16* __restrict__ DSG,
                                                            __nv_bfloat16* __restrict__ DSU) {
  __shared__ float lg[kSgTok][R];
  const int j = blockIdx.x * kSgCols + threadIdx.x;
  const int t0 = blockIdx.y * kSgTok;
  for (int i = threadIdx.x; i < kSgTok * R; i += kSgCols) {
    const int tt = i / R, rr = i % R;
    const int t = t0 + tt;
    lg[tt][rr] = t < N ? gB[(int64_t)t * R + rr] : 0.f;
  }
  __syncthreads();
  if (j >= F) return;
  float ad[R];
#pragma unroll
  for (int rr = 0; rr < R; rr++) ad[rr] = Ad[(int64_t)rr * F + j];
  for (int tb = 0; tb < kSgTok && t0 + tb < N; tb += kSgB) {
    float hv[kSgB], gv[kSgB], uv[kSgB];
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      const int64_t o = (int64_t)t * F + j;
      hv[q] = t < N ? __bfloat162float(Dh[o]) : 0.f;
      gv[q] = t < N ? __bfloat162float(SG[o]) : 0.f;
      uv[q] = t < N ? __bfloat162float(SU[o]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      if (t >= N) break;
      float dl = 0.f;
#pragma unroll
      for (int rr = 0; rr < R; rr++) dl = fmaf(lg[tb + q][rr], ad[rr], dl);
      const int64_t o = (int64_t)t * F + j;
      const float go = bf16r(hv[q] + bf16r(s * dl));
      float dsg, dsu;
      situ_glu_bwd(go, gv[q], uv[q], dsg, dsu);
      DSG[o] = __float2bfloat16_rn(dsg);
      DSU[o] = __float2bfloat16_rn(dsu);
    }
  }
}

// out[t][c] = bf16(Y[t][c] + bf16(s * sum_rr L0[t][rr] R0(rr, c)) [+ bf16(s * L1[t] . R1(:, c))])
// R(rr, c): RROWS -> R[rr * C + c] ([r][C]); else R[c * r + rr] ([C][r]). Y may alias out.
// Block: 256 columns x 32 tokens (batches of 4 as above); a thread keeps its column's adapter
// values in registers.
template <int R, bool TWO, bool RROWS>
__global__ void __launch_bounds__(kSgCols) k_lora_add_bf16(const __nv_bfloat16* Y, const float* __restrict__ L0,
                                                           const float* __restrict__ R0, const float* __restrict__ L1,
                                                           const float* __restrict__ R1, float s, int N, int C,
                                                           __nv_bfloat16* out) {
  constexpr int NW = TWO ? 2 : 1;
  __shared__ float ls[kSgTok][NW * R];
  const int j = blockIdx.x * kSgCols + threadIdx.x;
  const int t0 = blockIdx.y * kSgTok;
  for (int i = threadIdx.x; i < kSgTok * NW * R; i += kSgCols) {
    const int tt = i / (NW * R), rr = i % (NW * R);
    const int t = t0 + tt;
    ls[tt][rr] = t < N ? (rr < R ? L0[(int64_t)t * R + rr] : L1[(int64_t)t * R + rr - R]) : 0.f;
  }
  __syncthreads();
  if (j >= C) return;
  float rv[NW][R];
#pragma unroll
  for (int w = 0; w < NW; w++) {
    const float* Rm = w == 0 ? R0 : R1;
#pragma unroll
    for (int rr = 0; rr < R; rr++) rv[w][rr] = RROWS ? Rm[(int64_t)rr * C + j] : Rm[(int64_t)j * R + rr];
  }
  for (int tb = 0; tb < kSgTok && t0 + tb < N; tb += kSgB) {
    float yv[kSgB];
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      yv[q] = t < N ? __bfloat162float(Y[(int64_t)t * C + j]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kSgB; q++) {
      const int t = t0 + tb + q;
      if (t >= N) break;
      float v = yv[q];
#pragma unroll
      for (int w = 0; w < NW; w++) {
        float dl = 0.f;
#pragma unroll
        for (int rr = 0; rr < R; rr++) dl = fmaf(ls[tb + q][w * R + rr], rv[w][rr], dl);
        v += bf16r(s * dl);
      }
      out[(int64_t)t * C + j] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace ll

using namespace ll;

extern "C" {

int ll_shared_glu_forward(const void* G, const void* U, const float* xa_g, const float* xa_u, const float* B_g,
                          const float* B_u, float scaling, int N, int F, int r, void* SG, void* SU, void* H,
                          void* stream) {
  if (N < 0 || F <= 0 || !(r == 4 || r == 8 || r == 16 || r == 32)) return LL_ERR_ARG;
  if (N == 0) return LL_OK;
  if (!G || !U || !xa_g || !xa_u || !B_g || !B_u || !SG || !SU || !H) return LL_ERR_ARG;
  LL_STREAM(stream);
  const dim3 grid((F + kSgCols - 1) / kSgCols, (N + kSgTok - 1) / kSgTok);
  auto g = static_cast<const __nv_bfloat16*>(G);
  auto u = static_cast<const __nv_bfloat16*>(U);
  auto sg = static_cast<__nv_bfloat16*>(SG);
  auto su = static_cast<__nv_bfloat16*>(SU);
  auto h = static_cast<__nv_bfloat16*>(H);
#define LL_SGF(RR) k_shared_glu_fwd<RR><<<grid, kSgCols, 0, s>>>(g, u, xa_g, xa_u, B_g, B_u, scaling, N, F, sg, su, h)
  if (r == 4) LL_SGF(4); else if (r == 8) LL_SGF(8); else if (r == 16) LL_SGF(16); else LL_SGF(32);
#undef LL_SGF
  return check_launch("k_shared_glu_fwd");
}

int ll_shared_glu_backward(const void* Dh, const float* gB, const float* A_d, float scaling, const void* SG,
                           const void* SU, int N, int F, int r, void* DSG, void* DSU, void* stream) {
  if (N < 0 || F <= 0 || !(r == 4 || r == 8 || r == 16 || r == 32)) return LL_ERR_ARG;
  if (N == 0) return LL_OK;
  if (!Dh || !gB || !A_d || !SG || !SU || !DSG || !DSU) return LL_ERR_ARG;
  LL_STREAM(stream);
  const dim3 grid((F + kSgCols - 1) / kSgCols, (N + kSgTok - 1) / kSgTok);
  auto dh = static_cast<const __nv_bfloat16*>(Dh);
  auto sg = static_cast<const __nv_bfloat16*>(SG);
  auto su = static_cast<const __nv_bfloat16*>(SU);
  auto dsg = static_cast<__nv_bfloat16*>(DSG);
  auto dsu = static_cast<__nv_bfloat16*>(DSU);
#define LL_SGB(RR) k_shared_glu_bwd<RR><<<grid, kSgCols, 0, s>>>(dh, gB, A_d, scaling, sg, su, N, F, dsg, dsu)
  if (r == 4) LL_SGB(4); else if (r == 8) LL_SGB(8); else if (r == 16) LL_SGB(16); else LL_SGB(32);
#undef LL_SGB
  return check_launch("k_shared_glu_bwd");
}

int ll_lora_down(const void* X, int x_dtype, int M, int K, const float* B0, const float* B1, int n0, int n,
                 int b_rows, float alpha, float* C0, float* C1, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (M < 0 || K <= 0 || K % 8 || n <= 0 || n0 <= 0 || n0 > n || x_dtype < 0 || x_dtype > 2) return LL_ERR_ARG;
  if (M == 0) return LL_OK;
  if (!X || !B0 || !C0 || !workspace || (reinterpret_cast<uintptr_t>(X) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15))
    return LL_ERR_ARG;
  if (b_rows ? (n0 < n && (!B1 || !C1)) : n0 != n) return LL_ERR_ARG;
  if (workspace_bytes / sizeof(float) < (size_t)M * n) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  return skinny(X, x_dtype, b_rows != 0, M, K, B0, B1, n0, n, alpha, C0, C1, static_cast<float*>(workspace),
                workspace_bytes / sizeof(float), s);
}

int ll_lora_outer(const float* P, const void* Q, int q_dtype, int N, int C, int r, float scale, int transposed,
                  float* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (N < 0 || C <= 0 || C % 4 || r <= 0 || q_dtype < 0 || q_dtype > 2) return LL_ERR_ARG;
  if (!out || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 15)) return LL_ERR_ARG;
  if (N > 0 && (!P || !Q || (reinterpret_cast<uintptr_t>(Q) & (q_dtype == 0 ? 15 : 7)))) return LL_ERR_ARG;
  const size_t per_seg = (size_t)r * C;
  const size_t nseg_max = workspace_bytes / sizeof(float) / per_seg;
  if (nseg_max < 1) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  return outer(P, nullptr, nullptr, Q, q_dtype, N, nullptr, C, r, scale, transposed != 0,
               static_cast<float*>(workspace), (int)(nseg_max > 64 ? 64 : nseg_max), out, s);
}

int ll_lora_add_bf16(const void* Y, const float* L0, const float* R0, const float* L1, const float* R1, int r,
                     int r_rows, float scale, int N, int C, void* out, void* stream) {
  if (N < 0 || C <= 0 || !(r == 4 || r == 8 || r == 16 || r == 32)) return LL_ERR_ARG;
  if (N == 0) return LL_OK;
  if (!Y || !L0 || !R0 || !out || (L1 && !R1)) return LL_ERR_ARG;
  LL_STREAM(stream);
  const dim3 grid((C + kSgCols - 1) / kSgCols, (N + kSgTok - 1) / kSgTok);
  auto y = static_cast<const __nv_bfloat16*>(Y);
  auto o = static_cast<__nv_bfloat16*>(out);
#define LL_LA(RR, TW, RW) k_lora_add_bf16<RR, TW, RW><<<grid, kSgCols, 0, s>>>(y, L0, R0, L1, R1, scale, N, C, o)
#define LL_LA_R(TW, RW)                                                                          \
  do {                                                                                           \
    if (r == 4) LL_LA(4, TW, RW); else if (r == 8) LL_LA(8, TW, RW);                             \
    else if (r == 16) LL_LA(16, TW, RW); else LL_LA(32, TW, RW);                                 \
  } while (0)
  if (L1) {
    if (r_rows) LL_LA_R(true, true); else LL_LA_R(true, false);
  } else {
    if (r_rows) LL_LA_R(false, true); else LL_LA_R(false, false);
  }
#undef LL_LA_R
#undef LL_LA
  return check_launch("k_lora_add_bf16");
}

}  // extern "C"
