// Expert parallelism: the index work around the two all-to-all exchanges.
//
// Experts are split over n ranks in contiguous blocks, expert e on rank floor(e * n / E), the
// first expert of rank r being ceil(r * E / n). Tokens stay data-parallel: each rank routes its
// own tokens and sends every token row ONCE to each rank that owns at least one of its k
// experts, with a header of k slots (the expert's id local to that rank, or -1 where the slot's
// expert lives elsewhere) and the k routing weights. The receiving rank runs the unchanged
// single-GPU layer on the rows it received (slots with -1 are skipped by the layer) and
// returns per-row fp32 partial sums; the origin rank adds the partials of each token in
// ascending rank order, which keeps the result deterministic.
//
// The exchanges themselves are the caller's (NCCL all-to-all through torch.distributed in
// lazylora_b200.trainer.expert_parallel); these kernels build the send plan, gather the rows
// and reduce what comes back. The partial sums travel back packed: fp16 with a power-of-two
// row scale (half the bytes of fp32, 2^-11 relative rounding), unpacked by the combine. Send rows are grouped by destination rank (ascending), tokens
// ascending inside a group, so a rank receives its rows grouped by source rank, and the
// reverse exchange returns the partials in exactly the send order.
#include <cub/block/block_scan.cuh>

#include "host_common.cuh"

namespace ll {

LL_DEV int ep_owner(int64_t e, int E, int n) { return (int)((e * n) / E); }
LL_DEV int64_t ep_first(int r, int E, int n) { return ((int64_t)r * E + n - 1) / n; }

constexpr int kPlanThreads = 1024;

// One block. Pass 1 counts the rows for every destination rank (and the invalid slots);
// pass 2 assigns each (token, rank) pair its row: rank block offset + rank of the token among
// the tokens that go to that rank (block-wide exclusive scan, tile by tile).
__global__ void __launch_bounds__(kPlanThreads) k_ep_plan(const int64_t* __restrict__ idx, const float* __restrict__ w,
                                                          int T, int k, int E, int n, int* __restrict__ counts,
                                                          int* __restrict__ pos, int* __restrict__ send_tok,
                                                          int64_t* __restrict__ send_idx, float* __restrict__ send_w) {
  using Scan = cub::BlockScan<int, kPlanThreads>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int s_count[65];
  __shared__ int s_base[65];
  __shared__ int s_tile_total;
  for (int r = threadIdx.x; r <= n; r += blockDim.x) s_count[r] = 0;
  __syncthreads();
  // ---- pass 1: rows per destination rank, invalid slots in s_count[n]
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    uint64_t mask = 0;
    int bad = 0;
    for (int j = 0; j < k; j++) {
      const int64_t e = idx[(int64_t)t * k + j];
      if (e < 0 || e >= E) { bad++; continue; }
      mask |= 1ull << ep_owner(e, E, n);
    }
    for (int r = 0; r < n; r++)
      if (mask >> r & 1) atomicAdd(&s_count[r], 1);
    if (bad) atomicAdd(&s_count[n], bad);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int r = 0; r < n; r++) { s_base[r] = acc; acc += s_count[r]; }
  }
  __syncthreads();
  for (int r = threadIdx.x; r <= n; r += blockDim.x) counts[r] = s_count[r];
  // ---- pass 2: positions, one rank at a time so a tile needs one scan per rank
  for (int r = 0; r < n; r++) {
    const int64_t lo = ep_first(r, E, n);
    for (int t0 = 0; t0 < T; t0 += kPlanThreads) {
      const int t = t0 + threadIdx.x;
      int has = 0;
      if (t < T)
        for (int j = 0; j < k; j++) {
          const int64_t e = idx[(int64_t)t * k + j];
          if (e >= 0 && e < E && ep_owner(e, E, n) == r) has = 1;
        }
      int rank_in_tile, tile_total;
      Scan(tmp).ExclusiveSum(has, rank_in_tile, tile_total);
      if (t < T) {
        const int row = s_base[r] + rank_in_tile;
        pos[(int64_t)t * n + r] = has ? row : -1;
        if (has) {
          send_tok[row] = t;
          for (int j = 0; j < k; j++) {
            const int64_t e = idx[(int64_t)t * k + j];
            const bool here = e >= 0 && e < E && ep_owner(e, E, n) == r;
            send_idx[(int64_t)row * k + j] = here ? e - lo : -1;
            send_w[(int64_t)row * k + j] = here ? w[(int64_t)t * k + j] : 0.f;
          }
        }
      }
      if (threadIdx.x == 0) s_tile_total = tile_total;
      __syncthreads();
      if (threadIdx.x == 0) s_base[r] += s_tile_total;
      __syncthreads();
    }
  }
}

// dst[i, :] = src[tok[i], :], rows of `vecs` 16-byte vectors.
__global__ void k_ep_gather_rows(uint4* __restrict__ dst, const uint4* __restrict__ src, const int* __restrict__ tok,
                                 int rows, int vecs) {
  for (int i = blockIdx.x; i < rows; i += gridDim.x) {
    const uint4* s = src + (int64_t)tok[i] * vecs;
    uint4* o = dst + (int64_t)i * vecs;
    for (int v = threadIdx.x; v < vecs; v += blockDim.x) o[v] = s[v];
  }
}

// out[t, :] = sum over ranks r ascending of part[pos[t, r], :] (fp32 rows of d4 float4).
__global__ void k_ep_combine(float4* __restrict__ out, const float4* __restrict__ part, const int* __restrict__ pos,
                             int T, int n, int d4) {
  __shared__ int s_pos[64];
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    __syncthreads();
    if (threadIdx.x < n) s_pos[threadIdx.x] = pos[(int64_t)t * n + threadIdx.x];
    __syncthreads();
    for (int v = threadIdx.x; v < d4; v += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < n; r++) {
        const int p = s_pos[r];
        if (p < 0) continue;
        const float4 x = part[(int64_t)p * d4 + v];
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      out[(int64_t)t * d4 + v] = acc;
    }
  }
}

// grad_w[t, j] = part[pos[t, owner(idx[t, j])], j]: each slot was computed on its expert's rank.
__global__ void k_ep_combine_slots(float* __restrict__ grad_w, const float* __restrict__ part,
                                   const int* __restrict__ pos, const int64_t* __restrict__ idx, int T, int k, int E,
                                   int n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)T * k) return;
  const int64_t t = i / k;
  const int j = (int)(i % k);
  const int64_t e = idx[i];
  float v = 0.f;
  if (e >= 0 && e < E) {
    const int p = pos[t * n + ep_owner(e, E, n)];
    if (p >= 0) v = part[(int64_t)p * k + j];
  }
  grad_w[i] = v;
}

// Packed partial rows for the return exchanges: row i of `src` (fp32, d4 float4) as d fp16
// values times 2^e_i, e_i the power of two that brings max|row| into [2^14, 2^15), followed
// by the fp32 2^-e_i and 12 bytes of padding (2d + 16 bytes a row). One warp per row.
__global__ void k_ep_pack_rows(uint8_t* __restrict__ dst, const float4* __restrict__ src, int rows, int d4) {
  const int warps = blockDim.x / 32, lane = threadIdx.x % 32;
  const int64_t row_bytes = (int64_t)d4 * 8 + 16;
  for (int64_t i = (int64_t)blockIdx.x * warps + threadIdx.x / 32; i < rows; i += (int64_t)gridDim.x * warps) {
    const float4* s = src + i * d4;
    float mx = 0.f;
    for (int v = lane; v < d4; v += 32) {
      const float4 x = s[v];
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const int e = row_scale_exp(mx);
    const float sc = ldexpf(1.f, e);
    uint2* o = reinterpret_cast<uint2*>(dst + i * row_bytes);
    for (int v = lane; v < d4; v += 32) {
      const float4 x = s[v];
      const __half2 a = __floats2half2_rn(x.x * sc, x.y * sc), b = __floats2half2_rn(x.z * sc, x.w * sc);
      o[v] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
    if (lane == 0)
      *reinterpret_cast<float4*>(dst + i * row_bytes + (int64_t)d4 * 8) = make_float4(ldexpf(1.f, -e), 0.f, 0.f, 0.f);
  }
}

// out[t, :] = sum over ranks r ascending of the packed row pos[t, r] (fp16 x its 2^-e, in fp32).
__global__ void k_ep_combine_packed(float4* __restrict__ out, const uint8_t* __restrict__ part,
                                    const int* __restrict__ pos, int T, int n, int d4) {
  __shared__ int s_pos[64];
  __shared__ float s_inv[64];
  const int64_t row_bytes = (int64_t)d4 * 8 + 16;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    __syncthreads();
    if (threadIdx.x < n) {
      const int p = pos[(int64_t)t * n + threadIdx.x];
      s_pos[threadIdx.x] = p;
      s_inv[threadIdx.x] = p < 0 ? 0.f : *reinterpret_cast<const float*>(part + p * row_bytes + (int64_t)d4 * 8);
    }
    __syncthreads();
    for (int v = threadIdx.x; v < d4; v += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < n; r++) {
        const int p = s_pos[r];
        if (p < 0) continue;
        const uint2 h = reinterpret_cast<const uint2*>(part + p * row_bytes)[v];
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        const float iv = s_inv[r];
        acc.x += a.x * iv; acc.y += a.y * iv; acc.z += b.x * iv; acc.w += b.y * iv;
      }
      out[(int64_t)t * d4 + v] = acc;
    }
  }
}

}  // namespace ll

using namespace ll;

extern "C" {

int ll_ep_experts_of_rank(int E, int n_ranks, int rank, int* first, int* count) {
  if (E <= 0 || n_ranks <= 0 || n_ranks > 64 || rank < 0 || rank >= n_ranks || !first || !count) return LL_ERR_ARG;
  const int64_t lo = ((int64_t)rank * E + n_ranks - 1) / n_ranks;
  const int64_t hi = ((int64_t)(rank + 1) * E + n_ranks - 1) / n_ranks;
  *first = (int)lo;
  *count = (int)(hi - lo);
  return LL_OK;
}

int ll_ep_plan(int T, int k, int E, int n_ranks, const int64_t* idx, const float* w, int* counts, int* pos,
               int* send_tok, int64_t* send_idx, float* send_w, void* stream) {
  if (T < 0 || k <= 0 || k > 64 || E <= 0 || n_ranks <= 0 || n_ranks > 64) return LL_ERR_ARG;
  if (!counts || (T > 0 && (!idx || !w || !pos || !send_tok || !send_idx || !send_w))) return LL_ERR_ARG;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_plan<<<1, kPlanThreads, 0, static_cast<cudaStream_t>(stream)>>>(idx, w, T, k, E, n_ranks, counts, pos,
                                                                         send_tok, send_idx, send_w);
  return check_launch("k_ep_plan");
}

int ll_ep_gather_rows(void* dst, const void* src, const int* tok, int rows, int64_t row_bytes, void* stream) {
  if (rows < 0 || row_bytes <= 0 || row_bytes % 16) return LL_ERR_ARG;
  if (rows == 0) return LL_OK;
  if (!dst || !src || !tok || (reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) % 16)
    return LL_ERR_ARG;
  const int vecs = (int)(row_bytes / 16);
  const int grid = rows < 148 * 16 ? rows : 148 * 16;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_gather_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(dst), static_cast<const uint4*>(src), tok, rows, vecs);
  return check_launch("k_ep_gather_rows");
}

int ll_ep_combine(float* out, const float* part, const int* pos, int T, int n_ranks, int d, void* stream) {
  if (T < 0 || n_ranks <= 0 || n_ranks > 64 || d <= 0 || d % 4) return LL_ERR_ARG;
  if (T == 0) return LL_OK;
  if (!out || !pos || (reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(part)) % 16) return LL_ERR_ARG;
  const int grid = T < 148 * 8 ? T : 148 * 8;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_combine<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4*>(out), reinterpret_cast<const float4*>(part), pos, T, n_ranks, d / 4);
  return check_launch("k_ep_combine");
}

int ll_ep_pack_rows(void* dst, const float* src, int rows, int d, void* stream) {
  if (rows < 0 || d <= 0 || d % 4) return LL_ERR_ARG;
  if (rows == 0) return LL_OK;
  if (!dst || !src || (reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) % 16) return LL_ERR_ARG;
  const int grid = (rows + 7) / 8 < 148 * 8 ? (rows + 7) / 8 : 148 * 8;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_pack_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(dst), reinterpret_cast<const float4*>(src), rows, d / 4);
  return check_launch("k_ep_pack_rows");
}

int ll_ep_combine_packed(float* out, const void* part, const int* pos, int T, int n_ranks, int d, void* stream) {
  if (T < 0 || n_ranks <= 0 || n_ranks > 64 || d <= 0 || d % 4) return LL_ERR_ARG;
  if (T == 0) return LL_OK;
  if (!out || !pos || (reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(part)) % 16) return LL_ERR_ARG;
  const int grid = T < 148 * 8 ? T : 148 * 8;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_combine_packed<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4*>(out), static_cast<const uint8_t*>(part), pos, T, n_ranks, d / 4);
  return check_launch("k_ep_combine_packed");
}

int ll_ep_combine_slots(float* grad_w, const float* part, const int* pos, const int64_t* idx, int T, int k, int E,
                        int n_ranks, void* stream) {
  if (T < 0 || k <= 0 || E <= 0 || n_ranks <= 0 || n_ranks > 64) return LL_ERR_ARG;
  if (T == 0) return LL_OK;
  if (!grad_w || !pos || !idx) return LL_ERR_ARG;
  const int64_t n = (int64_t)T * k;
  g_launch_stream = static_cast<cudaStream_t>(stream);
  k_ep_combine_slots<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      grad_w, part, pos, idx, T, k, E, n_ranks);
  return check_launch("k_ep_combine_slots");
}

}  // extern "C"
