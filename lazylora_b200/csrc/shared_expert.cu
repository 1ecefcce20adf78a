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
// Block: 256 columns x 8 tokens; a thread keeps its column's r adapter values in registers and
// reads the 8 tokens' r-vectors from shared memory.
#include "host_common.cuh"

namespace ll {

constexpr int kSgCols = 256, kSgTok = 8;

LL_DEV float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

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
#pragma unroll 2
  for (int tt = 0; tt < kSgTok; tt++) {
    const int t = t0 + tt;
    if (t >= N) break;
    float dg = 0.f, du = 0.f;
#pragma unroll
    for (int rr = 0; rr < R; rr++) {
      dg = fmaf(la[tt][rr], bg[rr], dg);
      du = fmaf(la[tt][R + rr], bu[rr], du);
    }
    const int64_t o = (int64_t)t * F + j;
    const float sg = bf16r(__bfloat162float(G[o]) + bf16r(s * dg));
    const float su = bf16r(__bfloat162float(U[o]) + bf16r(s * du));
    SG[o] = __float2bfloat16_rn(sg);
    SU[o] = __float2bfloat16_rn(su);
    H[o] = __float2bfloat16_rn(situ_glu_fwd(sg, su));
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
#pragma unroll 2
  for (int tt = 0; tt < kSgTok; tt++) {
    const int t = t0 + tt;
    if (t >= N) break;
    float dl = 0.f;
#pragma unroll
    for (int rr = 0; rr < R; rr++) dl = fmaf(lg[tt][rr], ad[rr], dl);
    const int64_t o = (int64_t)t * F + j;
    const float go = bf16r(__bfloat162float(Dh[o]) + bf16r(s * dl));
    float dsg, dsu;
    situ_glu_bwd(go, __bfloat162float(SG[o]), __bfloat162float(SU[o]), dsg, dsu);
    DSG[o] = __float2bfloat16_rn(dsg);
    DSU[o] = __float2bfloat16_rn(dsu);
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

}  // extern "C"
