// Router of the routed-expert layer: KimiK3MoERouter.forward (lazy_lora/core/moe_router.py:80-100).
//   logits = x . Wr^T (fp32), scores = sigmoid(logits), choice = scores + bias,
//   top-k of choice (descending; ties: lower expert id), weights = scores at those ids,
//   renormalised by (sum + 1e-20) when asked and k > 1, times the routed scaling factor.
#include <algorithm>

#include "host_common.cuh"
#include "ops.cuh"
#include "router_tc.cuh"

namespace ll {

// Values compared as order-preserving unsigned words (-0 as +0; NaN as 0, below every number,
// never preferred to a number): a > b as floats iff f32_order(a) > f32_order(b).
LL_DEV uint32_t f32_order(float f) {
  if (isnan(f)) return 0u;
  const uint32_t u = f == 0.f ? 0u : __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-wide best of each lane's candidate (value word bo, expert be): the highest value, then the
// lowest id, by two hardware reductions. Every lane gets the winner's value word and id.
LL_DEV void warp_best(uint32_t bo, int be, uint32_t& vmax, int& emin) {
  vmax = __reduce_max_sync(0xffffffffu, bo);
  const uint32_t idw = bo == vmax ? 0x7fffffffu - (uint32_t)be : 0u;
  emin = (int)(0x7fffffffu - __reduce_max_sync(0xffffffffu, idw));
}

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
    {   // the warp's best: highest value, then lowest id (a lane with nothing left offers 0)
      uint32_t vmax;
      warp_best(be == 0x7fffffff ? 0u : f32_order(bv), be, vmax, be);
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

// ------------------------------------------------------- block-wide top k of one token
constexpr int kSelWarps = 8;
struct SelShared {
  float sc[kSelWarps * 32 * 4];          // score of every expert (E <= 1024)
  uint32_t cv[kSelWarps][32];            // each warp's top k: value words
  int ce[kSelWarps][32];                 //                     expert ids
};

// The top k (k <= 32) of one token by a block of 8 warps (all 256 threads call it, and the block
// synchronises before reusing `sh`): thread (w, lane) holds the scores sc[i] and choice values
// ch[i] of experts e = 256 i + 32 w + lane (i < 4, E <= 1024). Each warp takes its slice's top k
// in k rounds (a lane's best of 4, then the warp's best by reduction); warp 0 merges the 8 lists
// in k more rounds (lane j holding entry j of each list), and lane 0 writes the k ids and
// weights (renormalised in torch's CPU order for a short row, times rsf) to idx / w. Order: the
// highest value first, ties to the lower id, as k_route_select.
LL_DEV void block_select_token(const float (&sc)[4], const float (&ch)[4], int E, int k, int renorm, float rsf,
                               SelShared& sh, int64_t* __restrict__ idx, float* __restrict__ w) {
  const int wp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint32_t ov[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int e = 256 * i + 32 * wp + lane;
    ov[i] = e < E ? f32_order(ch[i]) : 0u;
    if (e < E) sh.sc[e] = sc[i];
  }
  uint32_t taken = 0;
  for (int kk = 0; kk < k; kk++) {
    uint32_t bo = 0;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int e = 256 * i + 32 * wp + lane;
      if (e < E && !((taken >> i) & 1) && (ov[i] > bo || (ov[i] == bo && e < be))) { bo = ov[i]; be = e; }
    }
    uint32_t vmax;
    int emin;
    warp_best(bo, be, vmax, emin);
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (256 * i + 32 * wp + lane == emin) taken |= 1u << i;
    if (lane == 0) { sh.cv[wp][kk] = vmax; sh.ce[wp][kk] = emin; }
  }
  __syncthreads();
  if (wp != 0) return;
  uint32_t mv[kSelWarps];
  int me[kSelWarps];
#pragma unroll
  for (int v = 0; v < kSelWarps; v++) {
    mv[v] = lane < k ? sh.cv[v][lane] : 0u;
    me[v] = lane < k ? sh.ce[v][lane] : 0x7fffffff;
  }
  uint32_t used = 0;
  float denom_l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float wsel = 0.f;
  int esel = 0;
  for (int kk = 0; kk < k; kk++) {
    uint32_t bo = 0;
    int be = 0x7fffffff;
#pragma unroll
    for (int v = 0; v < kSelWarps; v++)
      if (!((used >> v) & 1) && me[v] < E && (mv[v] > bo || (mv[v] == bo && me[v] < be))) { bo = mv[v]; be = me[v]; }
    uint32_t vmax;
    int emin;
    warp_best(bo, be, vmax, emin);
#pragma unroll
    for (int v = 0; v < kSelWarps; v++)
      if (me[v] == emin) used |= 1u << v;
    const float sv = emin < E ? sh.sc[emin] : 0.f;
    denom_l[kk & 7] += sv;           // every lane, in the order of k_route_select's lane 0
    if (lane == kk) { wsel = sv; esel = emin; }
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
    idx[lane] = esel;
    w[lane] = v * rsf;
  }
}

// The same selection for few tokens, one block per token (block_select_token), with every
// score computed in the same order as k_route_select: indices and weights are bit for bit
// those of k_route_select.
template <int MODE, int PL>
__global__ void __launch_bounds__(kSelWarps * 32) k_route_select_block(
    const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ bias, int T, int E, int k,
    int renorm, float rsf, int64_t* __restrict__ idx, float* __restrict__ w, float* __restrict__ scores_out,
    int nsplit) {
  static_assert(PL == 4, "four experts a thread");
  const int wp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the bias was written before the router's first kernel, which had passed its own wait before
  // this launch could start: its loads go before the wait and overlap it
  float bv[PL];
#pragma unroll
  for (int i = 0; i < PL; i++) {
    const int e = 256 * i + 32 * wp + lane;
    bv[i] = (MODE == 0 && bias && e < E) ? bias[e] : 0.f;
  }
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ SelShared sh;
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
      ch[i] = bias ? sg + bv[i] : sg;
      if (scores_out) scores_out[(int64_t)t * E + e] = sg;
    } else {
      sc[i] = a[(int64_t)t * E + e];
      ch[i] = b[(int64_t)t * E + e];
    }
  }
  block_select_token(sc, ch, E, k, renorm, rsf, sh, idx + (int64_t)t * k, w + (int64_t)t * k);
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

// ------------------------------------------------------------------ few-token logits
// For a handful of tokens the router is a matrix-vector product bound by reading W. Block = 8
// warps = 2 experts x 4 warps; warp q of an expert takes the runs q, q + 4, ... of 32 16-byte
// chunks of the expert's row (four runs' loads issued together, two from planes), W read as
// stored (fp32) or rebuilt from its three bf16 planes (hi + lo + lo2, which is W exactly); per
// token, the lanes' sums go through a shuffle tree and the 4 warps' sums are added in warp
// order. At most 64 registers a thread, so that four blocks fit an SM and the 448 blocks of 896
// experts run as one wave (at three a SM the last four blocks ran as a second wave). The logits
// are left for k_route_select_block (a block per token): selecting in the last block of this
// kernel to finish, behind a counter, measured slower (one token: 30.7 us against 28.7 us).
constexpr int kRgTok = 8;
template <bool PLANES, int XT>
__global__ void __launch_bounds__(256, 4) k_router_gemv(const void* __restrict__ x, const void* __restrict__ W, int T,
                                                       int d, int E, float* __restrict__ logits) {
  // runs whose loads are issued together: 4 (fp32 W), 2 (three planes: the registers of 4 spill);
  // a lane adds its chunks in the same order either way
  constexpr int kRgRun = PLANES ? 2 : 4;
  pdl_wait();
  pdl_launch_next();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int e = blockIdx.x * 2 + warp / 4, q = warp % 4;
  const int nch = d / 8;
  float acc[kRgTok];
#pragma unroll
  for (int t = 0; t < kRgTok; t++) acc[t] = 0.f;
  if (e < E) {
    for (int g0 = q; g0 * 32 < nch; g0 += 4 * kRgRun) {
      float wv[kRgRun][8];
#pragma unroll
      for (int u = 0; u < kRgRun; u++) {
        const int ch = (g0 + 4 * u) * 32 + lane;
        const bool in = ch < nch;
        if (PLANES) {
          const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(W);
          const int64_t nw = (int64_t)E * d, o = (int64_t)e * d + 8 * ch;
          uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h, l2 = h;
          if (in) {
            h = *reinterpret_cast<const uint4*>(wp + o);
            l = *reinterpret_cast<const uint4*>(wp + nw + o);
            l2 = *reinterpret_cast<const uint4*>(wp + 2 * nw + o);
          }
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w}, l2w[4] = {l2.x, l2.y, l2.z, l2.w};
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hw[j]));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lw[j]));
            const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&l2w[j]));
            wv[u][2 * j] = (a.x + b.x) + c.x;
            wv[u][2 * j + 1] = (a.y + b.y) + c.y;
          }
        } else {
          const float* wf = static_cast<const float*>(W) + (int64_t)e * d + 8 * ch;
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 a = in ? *reinterpret_cast<const float4*>(wf) : z;
          const float4 b = in ? *reinterpret_cast<const float4*>(wf + 4) : z;
          wv[u][0] = a.x; wv[u][1] = a.y; wv[u][2] = a.z; wv[u][3] = a.w;
          wv[u][4] = b.x; wv[u][5] = b.y; wv[u][6] = b.z; wv[u][7] = b.w;
        }
      }
#pragma unroll
      for (int t = 0; t < kRgTok; t++) {
        if (t >= T) break;
#pragma unroll
        for (int u = 0; u < kRgRun; u++) {
          const int ch = (g0 + 4 * u) * 32 + lane;
          if (ch >= nch) continue;
          float xv[8];
          if (XT == 0) {
            const float* xf = static_cast<const float*>(x) + (int64_t)t * d + 8 * ch;
            const float4 a = *reinterpret_cast<const float4*>(xf), b = *reinterpret_cast<const float4*>(xf + 4);
            xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w; xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
          } else {
            const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + (int64_t)t * d + 8 * ch);
            const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rw[j]));
              xv[2 * j] = f.x;
              xv[2 * j + 1] = f.y;
            }
          }
#pragma unroll
          for (int j = 0; j < 8; j++) acc[t] = fmaf(xv[j], wv[u][j], acc[t]);
        }
      }
    }
  }
  __shared__ float red[8][kRgTok];
#pragma unroll
  for (int t = 0; t < kRgTok; t++) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[warp][t] = v;
  }
  __syncthreads();
  if ((int)threadIdx.x < 2 * T) {
    const int el = threadIdx.x / T, t = threadIdx.x % T;
    const int ee = blockIdx.x * 2 + el;
    if (ee < E) {
      float v = red[4 * el][t];
#pragma unroll
      for (int qq = 1; qq < 4; qq++) v += red[4 * el + qq][t];
      logits[(int64_t)t * E + ee] = v;
    }
  }
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
    p.off_st = take(32);              // the status word
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
                            int E, void* ws, const RouterPlan& p, cudaStream_t s, DevStatus* status = nullptr) {
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
  DevStatus* st = status;
  if (!st) {   // its own status word (the caller's, when given, is reset by the caller)
    st = reinterpret_cast<DevStatus*>(base + p.off_st);
    LL_TRY(reset_status(st, s));
  }
  float* part = reinterpret_cast<float*>(base + p.off_part);
#define LL_RT(NPv, BNv) \
  if (p.NP == NPv && p.BN == BNv) return launch_router_mma<NPv, BNv>(maps, part, T, E, p, st, s);
  LL_RT(1, 16) LL_RT(1, 32) LL_RT(1, 64) LL_RT(1, 128)
  LL_RT(3, 16) LL_RT(3, 32) LL_RT(3, 64) LL_RT(3, 128)
#undef LL_RT
  return LL_ERR_ARG;
}

// out0 [T][r] (and out1 [T][r]) = the columns 0..r-1 (r..2r-1) of the sum of the nsplit
// partials [nsplit][T][E], added in split order.
__global__ void k_sum_split_cols(const float* __restrict__ part, int nsplit, int T, int E, int r,
                                 float* __restrict__ out0, float* __restrict__ out1) {
  pdl_wait();
  pdl_launch_next();
  const int64_t n = (int64_t)T * E;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = part[i];
#pragma unroll 8
  for (int sp = 1; sp < nsplit; sp++) acc += part[(int64_t)sp * n + i];
  const int t = (int)(i / E), e = (int)(i % E);
  if (e < r) out0[(int64_t)t * r + e] = acc;
  else out1[(int64_t)t * r + (e - r)] = acc;
}

size_t project_tc_bytes(int T, int d, int E) { return router_plan(T, d, E, 1).bytes; }

int project_tc(const void* x, int T, int d, const float* W0, const float* W1, bool transposed, int r, float* out0,
               float* out1, void* ws, size_t ws_bytes, DevStatus* st, cudaStream_t s) {
  const int E = W1 ? 2 * r : r;
  if (T <= 0 || d <= 0 || r <= 0 || d % 64 || !x || !W0 || !out0 || (W1 && !out1) || !ws) return LL_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(ws) % 256) return LL_ERR_ARG;
  const RouterPlan p = router_plan(T, d, E, 1);
  if (ws_bytes < p.bytes) return LL_ERR_WORKSPACE;
  uint8_t* base = static_cast<uint8_t*>(ws);
  __nv_bfloat16* planes = reinterpret_cast<__nv_bfloat16*>(base + p.off_w);
  k_split_lora_planes<<<(unsigned)std::min<int64_t>(((int64_t)E * d + 255) / 256, 148 * 4), 256, 0, s>>>(
      W0, W1, transposed, r, d, planes);
  LL_TRY(check_launch("k_split_lora_planes"));
  LL_TRY(router_logits_tc(x, 1, nullptr, planes, T, d, E, ws, p, s, st));
  const float* part = reinterpret_cast<const float*>(base + p.off_part);
  const int64_t n = (int64_t)T * E;
  return launch_pdl("k_sum_split_cols", k_sum_split_cols, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part,
                    p.nsplit, T, E, r, out0, out1);
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
  if (T <= kRgTok && E <= 1024 && (reinterpret_cast<uintptr_t>(planes ? (const void*)planes : (const void*)router_w) % 16) == 0) {
    // few tokens: logits on CUDA cores, then the selection
    float* logits = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.off_logits);
    const void* wsrc = planes ? static_cast<const void*>(planes) : static_cast<const void*>(router_w);
#define LL_RG(PL, XTv)                                                                                   \
  LL_TRY(launch_pdl("k_router_gemv", k_router_gemv<PL, XTv>, dim3((E + 1) / 2), dim3(256), 0, s, x, wsrc, T, d, E, \
                    logits))
    if (planes) { if (x_dtype == 0) LL_RG(true, 0); else LL_RG(true, 1); }
    else { if (x_dtype == 0) LL_RG(false, 0); else LL_RG(false, 1); }
#undef LL_RG
    return launch_select<0>(logits, nullptr, bias, T, E, k, renormalize, routed_scaling_factor, idx, w, scores_out, s,
                            1);
  }
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
