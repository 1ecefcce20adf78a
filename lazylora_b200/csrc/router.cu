// Router of the routed-expert layer: KimiK3MoERouter.forward (lazy_lora/core/moe_router.py:80-100).
//   logits = x . Wr^T (fp32), scores = sigmoid(logits), choice = scores + bias,
//   top-k of choice (descending; ties: lower expert id), weights = scores at those ids,
//   renormalised by (sum + 1e-20) when asked and k > 1, times the routed scaling factor.
#include "host_common.cuh"
#include "ops.cuh"

namespace ll {

// logits[T][E] = x[T][d] . W[E][d]^T in fp32, 64 x 64 tiles, 4 x 4 outputs per thread.
template <int XD>  // x dtype: 0 fp32, 1 bf16
__global__ void __launch_bounds__(256) k_router_logits(const void* __restrict__ xv, const float* __restrict__ W,
                                                       float* __restrict__ out, int T, int d, int E) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int t0 = blockIdx.y * BM, e0 = blockIdx.x * BN;
  float acc[4][4] = {};
  const int lr = threadIdx.x / 4;          // 0..63 row within tile
  const int lk = (threadIdx.x % 4) * 4;    // 0,4,8,12
  for (int k0 = 0; k0 < d; k0 += BK) {
    {
      const int t = t0 + lr;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (t < T) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int k = k0 + lk + i;
          if (k < d)
            v[i] = XD == 0 ? reinterpret_cast<const float*>(xv)[(int64_t)t * d + k]
                           : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(xv)[(int64_t)t * d + k]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; i++) xs[lk + i][lr] = v[i];
      const int e = e0 + lr;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int k = k0 + lk + i;
        ws[lk + i][lr] = (e < E && k < d) ? W[(int64_t)e * d + k] : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int e = e0 + tx * 4 + j;
      if (e < E) out[(int64_t)t * E + e] = acc[i][j];
    }
  }
}

// One warp per token. MODE 0: `a` holds logits (scores = sigmoid, choice = scores + bias).
// MODE 1: `a` holds scores and `b` the scores used for the choice, as given.
template <int MODE, int PER_LANE>
__global__ void k_route_select(const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ bias,
                               int T, int E, int k, int renorm, float rsf, int64_t* __restrict__ idx,
                               float* __restrict__ w, float* __restrict__ scores_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const int t = warp;
  float sc[PER_LANE], ch[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; i++) {
    const int e = lane + 32 * i;
    sc[i] = 0.f;
    ch[i] = -INFINITY;
    if (e < E) {
      if (MODE == 0) {
        const float s = 1.0f / (1.0f + expf(-a[(int64_t)t * E + e]));
        sc[i] = s;
        ch[i] = bias ? s + bias[e] : s;
        if (scores_out) scores_out[(int64_t)t * E + e] = s;
      } else {
        sc[i] = a[(int64_t)t * E + e];
        ch[i] = b[(int64_t)t * E + e];
      }
    }
  }
  uint64_t taken = 0;
  float wsel[32];
  int esel[32];
  for (int kk = 0; kk < k; kk++) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1) && (ch[i] > bv || (ch[i] == bv && e < be))) {
        bv = ch[i];
        be = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; i++)
      if (lane + 32 * i == be) {
        taken |= (uint64_t)1 << i;
        mine = sc[i];
      }
    const float sv = __shfl_sync(0xffffffffu, mine, be & 31);
    if (kk < 32) {
      wsel[kk] = sv;
      esel[kk] = be;
    }
  }
  if (lane == 0) {
    // Sum in the order torch's CPU reduction uses for a short row (moe_router.py:97): eight
    // lane accumulators (element i into lane i % 8, in order), then the lanes in order.
    // For k <= 8 that is the plain left-to-right sum; for k = 16 it is sum_i (v_i + v_{i+8}).
    float denom = 0.f;
    if (k > 1 && renorm) {
      float lanes[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int kk = 0; kk < k; kk++) lanes[kk & 7] += wsel[kk];
      denom = lanes[0];
      for (int i = 1; i < 8; i++) denom += lanes[i];
      denom += 1e-20f;
    }
    for (int kk = 0; kk < k; kk++) {
      float v = wsel[kk];
      if (k > 1 && renorm) v = v / denom;
      idx[(int64_t)t * k + kk] = esel[kk];
      w[(int64_t)t * k + kk] = v * rsf;
    }
  }
}

template <int MODE>
static int launch_select(const float* a, const float* b, const float* bias, int T, int E, int k, int renorm, float rsf,
                         int64_t* idx, float* w, float* scores_out, cudaStream_t s) {
  const int blocks = (T * 32 + 255) / 256;
  if (E <= 32 * 32)
    k_route_select<MODE, 32><<<blocks, 256, 0, s>>>(a, b, bias, T, E, k, renorm, rsf, idx, w, scores_out);
  else
    k_route_select<MODE, 64><<<blocks, 256, 0, s>>>(a, b, bias, T, E, k, renorm, rsf, idx, w, scores_out);
  return check_launch("k_route_select");
}

}  // namespace ll

using namespace ll;

extern "C" {

size_t ll_route_workspace_bytes(int T, int E) { return ((size_t)T * E * sizeof(float) + 255) & ~size_t(255); }

int ll_route_topk(const void* x, int x_dtype, const float* router_w, const float* bias, int T, int d, int E, int k,
                  int renormalize, float routed_scaling_factor, int64_t* idx, float* w, float* scores_out, void* ws,
                  size_t ws_bytes, void* stream) {
  if (T <= 0 || d <= 0 || E <= 0 || k <= 0 || k > 32 || k > E || E > 2048) return LL_ERR_ARG;
  if (!x || !router_w || !idx || !w || !ws || (x_dtype != 0 && x_dtype != 1)) return LL_ERR_ARG;
  if (ws_bytes < ll_route_workspace_bytes(T, E)) return LL_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* logits = static_cast<float*>(ws);
  dim3 grid((E + 63) / 64, (T + 63) / 64);
  if (x_dtype == 0)
    k_router_logits<0><<<grid, 256, 0, s>>>(x, router_w, logits, T, d, E);
  else
    k_router_logits<1><<<grid, 256, 0, s>>>(x, router_w, logits, T, d, E);
  LL_TRY(check_launch("k_router_logits"));
  return launch_select<0>(logits, nullptr, bias, T, E, k, renormalize, routed_scaling_factor, idx, w, scores_out, s);
}

int ll_route_select(const float* scores, const float* scores_for_choice, int T, int E, int k, int renormalize,
                    float routed_scaling_factor, int64_t* idx, float* w, void* stream) {
  if (T <= 0 || E <= 0 || k <= 0 || k > 32 || k > E || E > 2048 || !scores || !scores_for_choice || !idx || !w)
    return LL_ERR_ARG;
  return launch_select<1>(scores, scores_for_choice, nullptr, T, E, k, renormalize, routed_scaling_factor, idx, w,
                          nullptr, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
