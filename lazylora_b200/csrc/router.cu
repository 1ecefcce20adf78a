// Router of the routed-expert layer: KimiK3MoERouter.forward (lazy_lora/core/moe_router.py:80-100).
//   logits = x . Wr^T (fp32), scores = sigmoid(logits), choice = scores + bias,
//   top-k of choice (descending; ties: lower expert id), weights = scores at those ids,
//   renormalised by (sum + 1e-20) when asked and k > 1, times the routed scaling factor.
#include "host_common.cuh"
#include "ops.cuh"
#include "router_tc.cuh"

namespace ll {

// One warp per token. MODE 0: `a` holds logits (scores = sigmoid, choice = scores + bias).
// MODE 1: `a` holds scores and `b` the scores used for the choice, as given.
// In MODE 0 the logits are the sum of `nsplit` fp32 partials [nsplit][T][E], added in order.
template <int MODE, int PER_LANE>
__global__ void k_route_select(const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ bias,
                               int T, int E, int k, int renorm, float rsf, int64_t* __restrict__ idx,
                               float* __restrict__ w, float* __restrict__ scores_out, int nsplit) {
  pdl_wait();
  pdl_launch_next();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const int t = warp;
  float sc[PER_LANE], ch[PER_LANE];
  if (MODE == 0) {
    // the K-split partials of the lane's logits, added in split order; each split's PER_LANE
    // loads are issued together (one round of latency per split, not one per element)
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {                   // sc[] holds the logits first
      const int e = lane + 32 * i;
      sc[i] = e < E ? a[(int64_t)t * E + e] : 0.f;
    }
    for (int sp = 1; sp < nsplit; sp++) {
      const float* ap = a + ((int64_t)sp * T + t) * E;
#pragma unroll
      for (int i = 0; i < PER_LANE; i++) {
        const int e = lane + 32 * i;
        if (e < E) sc[i] += ap[e];
      }
    }
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
      const int e = lane + 32 * i;
      ch[i] = -INFINITY;
      if (e < E) {
        const float s = 1.0f / (1.0f + expf(-sc[i]));
        sc[i] = s;
        ch[i] = bias ? s + bias[e] : s;
        if (scores_out) scores_out[(int64_t)t * E + e] = s;
      } else {
        sc[i] = 0.f;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
      const int e = lane + 32 * i;
      sc[i] = e < E ? a[(int64_t)t * E + e] : 0.f;
      ch[i] = e < E ? b[(int64_t)t * E + e] : -INFINITY;
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

// The same selection for few tokens, one block per token: each of the 8 warps takes the top k of
// its slice of experts (expert e = 256 i + 32 w + lane), then warp 0 merges the 8 lists. The
// top k of the union of the slices' top k is the top k overall, with the same order and tie
// rule (higher value, then lower id), and every score is computed in the same order as above,
// so indices and weights are bit for bit those of k_route_select.
constexpr int kSelWarps = 8;
template <int MODE, int PL>
__global__ void __launch_bounds__(kSelWarps * 32) k_route_select_block(
    const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ bias, int T, int E, int k,
    int renorm, float rsf, int64_t* __restrict__ idx, float* __restrict__ w, float* __restrict__ scores_out,
    int nsplit) {
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int wp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __shared__ float c_ch[kSelWarps][32], c_sc[kSelWarps][32];
  __shared__ int c_e[kSelWarps][32];
  float sc[PL], ch[PL];
#pragma unroll
  for (int i = 0; i < PL; i++) sc[i] = 0.f;
  if (MODE == 0) {     // the splits' partial logits, added in split order, a split's loads together
#pragma unroll
    for (int i = 0; i < PL; i++) {
      const int e = 256 * i + 32 * wp + lane;
      if (e < E) sc[i] = a[(int64_t)t * E + e];
    }
    int sp = 1;
    for (; sp + 8 <= nsplit; sp += 8) {        // eight splits' loads in flight, added in order
      float v[8][PL];
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int i = 0; i < PL; i++) {
          const int e = 256 * i + 32 * wp + lane;
          v[u][i] = e < E ? a[((int64_t)(sp + u) * T + t) * E + e] : 0.f;
        }
#pragma unroll
      for (int u = 0; u < 8; u++)
#pragma unroll
        for (int i = 0; i < PL; i++)
          if (256 * i + 32 * wp + lane < E) sc[i] += v[u][i];
    }
    for (; sp < nsplit; sp++) {
      const float* ap = a + ((int64_t)sp * T + t) * E;
#pragma unroll
      for (int i = 0; i < PL; i++) {
        const int e = 256 * i + 32 * wp + lane;
        if (e < E) sc[i] += ap[e];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PL; i++) {
    const int e = 256 * i + 32 * wp + lane;
    ch[i] = -INFINITY;
    const float l = sc[i];
    sc[i] = 0.f;
    if (e >= E) continue;
    if (MODE == 0) {
      const float sg = 1.0f / (1.0f + expf(-l));
      sc[i] = sg;
      ch[i] = bias ? sg + bias[e] : sg;
      if (scores_out) scores_out[(int64_t)t * E + e] = sg;
    } else {
      sc[i] = a[(int64_t)t * E + e];
      ch[i] = b[(int64_t)t * E + e];
    }
  }
  // this warp's top k
  uint32_t taken = 0;
  for (int kk = 0; kk < k; kk++) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PL; i++) {
      const int e = 256 * i + 32 * wp + lane;
      if (e < E && !((taken >> i) & 1) && (ch[i] > bv || (ch[i] == bv && e < be))) { bv = ch[i]; be = e; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < PL; i++)
      if (256 * i + 32 * wp + lane == be) { taken |= 1u << i; mine = sc[i]; }
    const float sv = __shfl_sync(0xffffffffu, mine, (be & 31));
    if (lane == 0) { c_ch[wp][kk] = bv; c_sc[wp][kk] = sv; c_e[wp][kk] = be; }
  }
  __syncthreads();
  if (wp != 0) return;
  // merge: lane j holds candidate j of every warp's list
  float mch[kSelWarps], msc[kSelWarps];
  int me[kSelWarps];
#pragma unroll
  for (int v = 0; v < kSelWarps; v++) {
    const bool ok = lane < k;
    mch[v] = ok ? c_ch[v][lane] : -INFINITY;
    msc[v] = ok ? c_sc[v][lane] : 0.f;
    me[v] = ok ? c_e[v][lane] : 0x7fffffff;
  }
  uint32_t used = 0;
  float wsel = 0.f, denom_l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int esel = 0;
  for (int kk = 0; kk < k; kk++) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int v = 0; v < kSelWarps; v++)
      if (!((used >> v) & 1) && me[v] < E && (mch[v] > bv || (mch[v] == bv && me[v] < be))) { bv = mch[v]; be = me[v]; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    float mine = 0.f;
    bool found = false;
#pragma unroll
    for (int v = 0; v < kSelWarps; v++)
      if (me[v] == be && !((used >> v) & 1)) { used |= 1u << v; mine = msc[v]; found = true; }
    const uint32_t holder = __ballot_sync(0xffffffffu, found);
    const float sv = __shfl_sync(0xffffffffu, mine, holder ? __ffs(holder) - 1 : 0);
    denom_l[kk & 7] += sv;            // every lane, in the order of the warp kernel's lane 0
    if (lane == kk) { wsel = sv; esel = be; }
  }
  float denom = 0.f;
  if (k > 1 && renorm) {
    denom = denom_l[0];
    for (int i = 1; i < 8; i++) denom += denom_l[i];
    denom += 1e-20f;
  }
  if (lane < k) {
    float v = wsel;
    if (k > 1 && renorm) v = v / denom;
    idx[(int64_t)t * k + lane] = esel;
    w[(int64_t)t * k + lane] = v * rsf;
  }
}

// Few tokens: a block of 8 warps per token (k_route_select_block), else a warp per token.
static bool select_by_block(int T, int E, int k) { return T <= 256 && k <= 32 && E <= 256 * 4; }

template <int MODE>
static int launch_select(const float* a, const float* b, const float* bias, int T, int E, int k, int renorm, float rsf,
                         int64_t* idx, float* w, float* scores_out, cudaStream_t s, int nsplit = 1) {
  if (select_by_block(T, E, k))
    return launch_pdl("k_route_select", k_route_select_block<MODE, 4>, dim3(T), dim3(kSelWarps * 32), 0, s, a, b,
                      bias, T, E, k, renorm, rsf, idx, w, scores_out, nsplit);
  const dim3 blocks((T * 32 + 255) / 256);
  if (E <= 32 * 32)
    return launch_pdl("k_route_select", k_route_select<MODE, 32>, blocks, dim3(256), 0, s, a, b, bias, T, E, k, renorm,
                      rsf, idx, w, scores_out, nsplit);
  return launch_pdl("k_route_select", k_route_select<MODE, 64>, blocks, dim3(256), 0, s, a, b, bias, T, E, k, renorm,
                    rsf, idx, w, scores_out, nsplit);
}

// logits[i] = sum over the nsplit partials of element i, added in split order.
__global__ void k_sum_partials(const float* __restrict__ part, int nsplit, int64_t n, float* __restrict__ logits) {
  pdl_wait();
  pdl_launch_next();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = part[i];
#pragma unroll 8
  for (int sp = 1; sp < nsplit; sp++) acc += part[(int64_t)sp * n + i];
  logits[i] = acc;
}

// ------------------------------------------------------------ tensor-core logits: plan + launch
struct RouterPlan {
  int BN = 16, NP = 1, mt = 1, nt = 1, nsplit = 1, kbps = 1, kb_total = 1;
  size_t off_w = 0, off_x = 0, off_part = 0, off_logits = 0, off_st = 0, bytes = 0;
};

static RouterPlan router_plan(int T, int d, int E, int x_dtype) {
  RouterPlan p;
  p.BN = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
  p.NP = x_dtype == 0 ? 3 : 1;
  p.mt = (E + 127) / 128;
  p.nt = (T + p.BN - 1) / p.BN;
  p.kb_total = (d + 63) / 64;
  const int sms = device_info().sms > 0 ? device_info().sms : 148;
  const int tiles = p.mt * p.nt;
  int want = tiles >= sms ? 1 : sms / tiles;                 // K splits that fill the SMs once
  if (want > p.kb_total) want = p.kb_total;
  p.kbps = (p.kb_total + want - 1) / want;
  p.nsplit = (p.kb_total + p.kbps - 1) / p.kbps;               // every split non-empty
  {
    size_t off = 0;
    auto take = [&](size_t n) { off = (off + 255) & ~size_t(255); const size_t o = off; off += n; return o; };
    p.off_w = take((size_t)3 * E * d * 2);
    p.off_x = take(p.NP == 3 ? (size_t)3 * T * d * 2 : 0);
    p.off_part = take((size_t)p.nsplit * T * E * 4);
    p.off_logits = take((size_t)T * E * 4);
    p.off_st = take(sizeof(DevStatus));
    p.bytes = (off + 255) & ~size_t(255);
  }
  return p;
}

template <int NP, int BN>
static int launch_router_mma(const RouterMaps& maps, float* part, int T, int E, const RouterPlan& p, DevStatus* st,
                             cudaStream_t s) {
  using Cf = RouterCfg<NP, BN>;
  auto kern = k_router_mma<NP, BN>;
  LL_TRY(set_smem_attr(reinterpret_cast<const void*>(kern), Cf::SMEM));
  return launch_pdl("k_router_mma", kern, dim3(p.mt, p.nt, p.nsplit), dim3(kRtWarps * 32), Cf::SMEM, s, maps, part, T,
                    E, p.kb_total, p.kbps, st);
}

// planes: the router weight split into its three bf16 planes (hi, lo, lo2; [3][E][d]), or null
// to split W into the workspace on this call.
static int router_logits_tc(const void* x, int x_dtype, const float* W, const __nv_bfloat16* planes, int T, int d,
                            int E, void* ws, const RouterPlan& p, cudaStream_t s) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  const int64_t nw = (int64_t)E * d;
  const __nv_bfloat16* wp = planes;
  if (!wp) {
    __nv_bfloat16* split = reinterpret_cast<__nv_bfloat16*>(base + p.off_w);
    k_split_bf16x3<<<148 * 4, 256, 0, s>>>(W, split, split + nw, split + 2 * nw, nw);
    LL_TRY(check_launch("k_split_bf16x3"));
    wp = split;
  }
  const __nv_bfloat16* xp[3] = {static_cast<const __nv_bfloat16*>(x), nullptr, nullptr};
  if (p.NP == 3) {
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(base + p.off_x);
    const int64_t nx = (int64_t)T * d;
    k_split_bf16x3<<<148 * 4, 256, 0, s>>>(static_cast<const float*>(x), xs, xs + nx, xs + 2 * nx, nx);
    LL_TRY(check_launch("k_split_bf16x3"));
    xp[0] = xs; xp[1] = xs + nx; xp[2] = xs + 2 * nx;
  }
  RouterMaps maps;
  for (int i = 0; i < 3; i++)
    LL_TRY(make_map_2d(&maps.a[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wp + i * nw, (uint64_t)d, (uint64_t)E,
                       (uint64_t)d * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  for (int i = 0; i < p.NP; i++)
    LL_TRY(make_map_2d(&maps.b[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xp[i], (uint64_t)d, (uint64_t)T,
                       (uint64_t)d * 2, 64, p.BN, CU_TENSOR_MAP_SWIZZLE_128B));
  if (p.NP == 1) maps.b[1] = maps.b[2] = maps.b[0];
  DevStatus* st = reinterpret_cast<DevStatus*>(base + p.off_st);
  LL_TRY(reset_status(st, s));
  float* part = reinterpret_cast<float*>(base + p.off_part);
#define LL_RT(NPv, BNv) \
  if (p.NP == NPv && p.BN == BNv) return launch_router_mma<NPv, BNv>(maps, part, T, E, p, st, s);
  LL_RT(1, 16) LL_RT(1, 32) LL_RT(1, 64) LL_RT(1, 128)
  LL_RT(3, 16) LL_RT(3, 32) LL_RT(3, 64) LL_RT(3, 128)
#undef LL_RT
  return LL_ERR_ARG;
}

}  // namespace ll

using namespace ll;

extern "C" {

size_t ll_route_workspace_bytes(int T, int d, int E) {
  if (T <= 0 || d <= 0 || E <= 0) return 0;
  return router_plan(T, d, E, 0).bytes;     // fp32 activations need the most (their planes)
}

static int route_topk(const void* x, int x_dtype, const float* router_w, const __nv_bfloat16* planes,
                      const float* bias, int T, int d, int E, int k, int renormalize, float routed_scaling_factor,
                      int64_t* idx, float* w, float* scores_out, void* ws, size_t ws_bytes, void* stream) {
  if (T <= 0 || d <= 0 || E <= 0 || k <= 0 || k > 32 || k > E || E > 2048 || d % 8) return LL_ERR_ARG;
  if (!x || (!router_w && !planes) || !idx || !w || !ws || (x_dtype != 0 && x_dtype != 1)) return LL_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(ws) % 256) return LL_ERR_ARG;
  if (planes && reinterpret_cast<uintptr_t>(planes) % 16) return LL_ERR_ARG;
  const RouterPlan p = router_plan(T, d, E, x_dtype);
  if (ws_bytes < p.bytes) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  g_launch_count = 0;
  LL_TRY(router_logits_tc(x, x_dtype, router_w, planes, T, d, E, ws, p, s));
  const float* part = reinterpret_cast<const float*>(static_cast<uint8_t*>(ws) + p.off_part);
  if (p.nsplit > 1 && !select_by_block(T, E, k)) {   // the K splits' partials, summed in split order by a wide kernel
    float* logits = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.off_logits);
    const int64_t n = (int64_t)T * E;
    LL_TRY(launch_pdl("k_sum_partials", k_sum_partials, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part,
                      p.nsplit, n, logits));
    return launch_select<0>(logits, nullptr, bias, T, E, k, renormalize, routed_scaling_factor, idx, w, scores_out, s,
                            1);
  }
  // few tokens: the selection kernel adds the splits' partials itself (in split order)
  return launch_select<0>(part, nullptr, bias, T, E, k, renormalize, routed_scaling_factor, idx, w, scores_out, s,
                          p.nsplit);
}

int ll_route_topk(const void* x, int x_dtype, const float* router_w, const float* bias, int T, int d, int E, int k,
                  int renormalize, float routed_scaling_factor, int64_t* idx, float* w, float* scores_out, void* ws,
                  size_t ws_bytes, void* stream) {
  return route_topk(x, x_dtype, router_w, nullptr, bias, T, d, E, k, renormalize, routed_scaling_factor, idx, w,
                    scores_out, ws, ws_bytes, stream);
}

int ll_route_prepare(const float* router_w, int E, int d, uint16_t* planes, void* stream) {
  if (!router_w || !planes || E <= 0 || d <= 0 || d % 8 || reinterpret_cast<uintptr_t>(planes) % 16) return LL_ERR_ARG;
  LL_STREAM(stream);
  g_launch_count = 0;
  __nv_bfloat16* wp = reinterpret_cast<__nv_bfloat16*>(planes);
  const int64_t nw = (int64_t)E * d;
  k_split_bf16x3<<<148 * 4, 256, 0, s>>>(router_w, wp, wp + nw, wp + 2 * nw, nw);
  return check_launch("k_split_bf16x3");
}

int ll_route_topk_prepared(const void* x, int x_dtype, const uint16_t* planes, const float* bias, int T, int d, int E,
                           int k, int renormalize, float routed_scaling_factor, int64_t* idx, float* w,
                           float* scores_out, void* ws, size_t ws_bytes, void* stream) {
  return route_topk(x, x_dtype, nullptr, reinterpret_cast<const __nv_bfloat16*>(planes), bias, T, d, E, k,
                    renormalize, routed_scaling_factor, idx, w, scores_out, ws, ws_bytes, stream);
}

int ll_route_select(const float* scores, const float* scores_for_choice, int T, int E, int k, int renormalize,
                    float routed_scaling_factor, int64_t* idx, float* w, void* stream) {
  if (T <= 0 || E <= 0 || k <= 0 || k > 32 || k > E || E > 2048 || !scores || !scores_for_choice || !idx || !w)
    return LL_ERR_ARG;
  LL_STREAM(stream);
  return launch_select<1>(scores, scores_for_choice, nullptr, T, E, k, renormalize, routed_scaling_factor, idx, w,
                          nullptr, s);
}

}  // extern "C"
