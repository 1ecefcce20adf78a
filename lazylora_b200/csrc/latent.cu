// Row RMSNorm of the latent MoE block (the step between the routed-expert sum and the latent
// up-projection of Kimi K3, lazy_lora/trainer/lazy_trainer.py:731-733, with the reference's
// RMSNormFunction.forward, lazy_lora/streaming/trunk_streamer.py:27-31):
//   y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w          (x: the fp32 routed sum)
// and its gradient with respect to x for a frozen w (LoRA training leaves the norm weight
// fixed):
//   r = rsqrt(mean(x^2) + eps), u = gy * w,
//   gx[j] = r * u[j] - r^3 * x[j] * (sum_i u[i] x[i]) / D.
// One block per row; the row's sums are reduced in a fixed order (per-thread strided partial,
// warp shuffle tree, then the warps in order), so results are bitwise reproducible. The
// forward also stores r per row for the backward.
#include "host_common.cuh"

namespace ll {

constexpr int kNormThreads = 256;

LL_DEV float block_sum_fixed(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < kNormThreads / 32; i++) s += red[i];
  __syncthreads();
  return s;
}

template <int YDT>
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_fwd(const float* __restrict__ x, const float* __restrict__ w,
                                                              int D, float eps, void* __restrict__ y,
                                                              float* __restrict__ rstd) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += kNormThreads) ss = fmaf(xr[i], xr[i], ss);
  const float tot = block_sum_fixed(ss, red);
  const float r = rsqrtf(tot / (float)D + eps);
  if (threadIdx.x == 0 && rstd) rstd[row] = r;
  for (int i = threadIdx.x; i < D; i += kNormThreads) {
    const float v = xr[i] * r * w[i];
    if (YDT == 0) reinterpret_cast<float*>(y)[row * D + i] = v;
    else reinterpret_cast<__nv_bfloat16*>(y)[row * D + i] = __float2bfloat16_rn(v);
  }
}

template <int GDT>
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_bwd(const float* __restrict__ x, const float* __restrict__ w,
                                                              const float* __restrict__ rstd,
                                                              const void* __restrict__ gy, int D,
                                                              float* __restrict__ gx) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * D;
  auto g_at = [&](int i) {
    return GDT == 0 ? reinterpret_cast<const float*>(gy)[row * D + i]
                    : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(gy)[row * D + i]);
  };
  float dot = 0.f;
  for (int i = threadIdx.x; i < D; i += kNormThreads) dot = fmaf(g_at(i) * w[i], xr[i], dot);
  const float tot = block_sum_fixed(dot, red);
  const float r = rstd[row];
  const float c = r * r * r * tot / (float)D;
  for (int i = threadIdx.x; i < D; i += kNormThreads) gx[row * D + i] = r * (g_at(i) * w[i]) - c * xr[i];
}

}  // namespace ll

using namespace ll;

extern "C" {

int ll_rmsnorm_forward(const float* x, const float* w, int N, int D, float eps, void* y, int y_dtype, float* rstd,
                       void* stream) {
  if (N < 0 || D <= 0 || (y_dtype != 0 && y_dtype != 1)) return LL_ERR_ARG;
  if (N == 0) return LL_OK;
  if (!x || !w || !y) return LL_ERR_ARG;
  LL_STREAM(stream);
  if (y_dtype == 0) k_rmsnorm_fwd<0><<<N, kNormThreads, 0, s>>>(x, w, D, eps, y, rstd);
  else k_rmsnorm_fwd<1><<<N, kNormThreads, 0, s>>>(x, w, D, eps, y, rstd);
  return check_launch("k_rmsnorm_fwd");
}

int ll_rmsnorm_backward(const float* x, const float* w, const float* rstd, const void* gy, int gy_dtype, int N, int D,
                        float* gx, void* stream) {
  if (N < 0 || D <= 0 || (gy_dtype != 0 && gy_dtype != 1)) return LL_ERR_ARG;
  if (N == 0) return LL_OK;
  if (!x || !w || !rstd || !gy || !gx) return LL_ERR_ARG;
  LL_STREAM(stream);
  if (gy_dtype == 0) k_rmsnorm_bwd<0><<<N, kNormThreads, 0, s>>>(x, w, rstd, gy, D, gx);
  else k_rmsnorm_bwd<1><<<N, kNormThreads, 0, s>>>(x, w, rstd, gy, D, gx);
  return check_launch("k_rmsnorm_bwd");
}

}  // extern "C"
