// Operand preparation for the block-scaled forward GEMMs (bs_gemm.cuh): the weights' E8M0
// scale blocks in the layout tcgen05.cp copies into tensor memory (once per weight load), and
// activation rows as low-precision terms (once per GEMM input): four E2M1 terms with E8M0
// block-32 scales (BS_FP4, their scales then laid out per chunk and stage) or three E4M3 terms
// with power-of-two row scales (BS_FP8).
#include <algorithm>

#include "host_common.cuh"
#include "ops.cuh"

#include <cub/block/block_scan.cuh>

namespace ll {

// One thread per (row, 128-K stage): the row's 4 scale bytes of that stage, bytes >= 253 (the
// reference's "contributes zero") replaced by 0, written to line (row % 32), word
// ((row % 128) / 32) of the stage's block of the row's 128-row tile.
__global__ void k_prepare_sfa(const uint8_t* __restrict__ scales, int64_t sstride, int64_t rows_total, int R,
                              int n_stage, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows_total * n_stage) return;
  const int64_t row = i / n_stage;
  const int ks = (int)(i % n_stage);
  uint32_t w = *reinterpret_cast<const uint32_t*>(scales + row * sstride + 4 * ks);
  uint32_t fixed = 0;
#pragma unroll
  for (int b = 0; b < 4; b++) {
    const uint32_t byte = (w >> (8 * b)) & 0xffu;
    fixed |= (byte >= 253u ? 0u : byte) << (8 * b);
  }
  const int64_t e = row / R;
  const int r = (int)(row % R);
  const int64_t tile = e * (R / 128) + r / 128;
  const int m = r % 128;
  uint32_t* blk = reinterpret_cast<uint32_t*>(out + (tile * n_stage + ks) * kBsSfBlock);
  blk[(m % 32) * 4 + m / 32] = fixed;
}

int launch_prepare_sfa(const uint8_t* scales, int64_t sstride, int E, int R, int C, uint8_t* out, cudaStream_t s) {
  if (E <= 0 || R <= 0 || R % 128 || C <= 0 || C % 128 || sstride < C / 32 || sstride % 4 || !scales || !out)
    return LL_ERR_ARG;
  const int64_t rows = (int64_t)E * R;
  const int n_stage = C / 128;
  const int64_t n = rows * n_stage;
  k_prepare_sfa<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(scales, sstride, rows, R, n_stage, out);
  return check_launch("k_prepare_sfa");
}

// ------------------------------------------------------------------------------------
constexpr int kE3Threads = 256;
constexpr int kE3Chunks = 4;       // 8-element chunks a thread holds: K <= 8 * 4 * 256
constexpr int kBsTermsFp4 = BsTerms<BS_FP4>::value;

template <int SRC>   // 0 fp32, 1 bf16, 2 fp16
LL_DEV void load8(const void* src, int64_t row, int K, int ch, float (&v)[8]) {
  if (SRC == 0) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + row * K) + 2 * ch;
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + row * K)[ch];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 f = SRC == 1 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]))
                                : __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// Block-wide max of v (every thread gets it); `red` holds kE3Threads / 32 floats.
LL_DEV float block_max(float v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  __syncthreads();                                   // red is reused term after term
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kE3Threads / 32; i++) m = fmaxf(m, red[i]);
  return m;
}

// One block per source row: the row in registers, three rounds of (block max, scale, round to
// E4M3, subtract), each term stored to every destination row.
template <int SRC, bool TOK>
__global__ void __launch_bounds__(kE3Threads) k_rows_to_e4m3x3(const void* __restrict__ src, int src_rows,
                                                               const int* __restrict__ tok_pos, int k,
                                                               const int* __restrict__ n_valid, int K, int64_t P,
                                                               uint8_t* __restrict__ dst, float* __restrict__ inv3) {
  pdl_wait();
  pdl_launch_next();
  const int r = blockIdx.x;
  if (r >= src_rows) return;
  if (!TOK && n_valid && r >= *n_valid) return;
  __shared__ float red[kE3Threads / 32];
  const int nch = K / 8;
  float v[kE3Chunks][8];
#pragma unroll
  for (int i = 0; i < kE3Chunks; i++) {
    const int ch = threadIdx.x + i * kE3Threads;
#pragma unroll
    for (int j = 0; j < 8; j++) v[i][j] = 0.f;
    if (ch < nch) load8<SRC>(src, r, K, ch, v[i]);
  }
#pragma unroll 1
  for (int t = 0; t < BsTerms<BS_FP8>::value; t++) {
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < kE3Chunks; i++)
#pragma unroll
      for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[i][j]));
    const int e = e4m3_scale_exp(block_max(mx, red));
    const float sc = ldexpf(1.f, e), inv = ldexpf(1.f, -e);
    uint2 q[kE3Chunks];
#pragma unroll
    for (int i = 0; i < kE3Chunks; i++) {
      uint32_t b[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        b[j] = f32x2_to_e4m3x2(v[i][2 * j] * sc, v[i][2 * j + 1] * sc);
        const float2 d = e4m3x2_to_f32x2(b[j]);
        v[i][2 * j] -= d.x * inv;                // the residual the next term takes
        v[i][2 * j + 1] -= d.y * inv;
      }
      q[i] = make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
    }
    for (int j = 0; j < (TOK ? k : 1); j++) {
      const int p = TOK ? tok_pos[(int64_t)r * k + j] : r;
      if (p < 0) continue;
      if (threadIdx.x == 0) inv3[t * P + p] = inv;
      uint2* row = reinterpret_cast<uint2*>(dst + ((int64_t)t * P + p) * K);
#pragma unroll
      for (int i = 0; i < kE3Chunks; i++) {
        const int ch = threadIdx.x + i * kE3Threads;
        if (ch < nch) row[ch] = q[i];
      }
    }
  }
}

// The four E2M1 term rounds of one thread's 8 source values (8-element chunk ch of the row):
// term t's packed codes word[t] and its stage's four scale bytes sw[t] (the blocks of this
// thread and the threads + 4, 8, 12; meaningful in the stage's lead thread). Every lane of the
// warp takes part (shuffles). See k_rows_to_e2m1x4 for the formats.
LL_DEV void e2m1x4_terms(float (&v)[8], uint32_t (&word)[kBsTermsFp4], uint32_t (&sw)[kBsTermsFp4]) {
#pragma unroll
  for (int t = 0; t < kBsTermsFp4; t++) {
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[j]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    // smallest e with mx / 2^e <= 6
    int e = -127;
    if (mx > 0.f && isfinite(mx)) {
      int E;
      const float m = frexpf(mx, &E);            // mx = m 2^E, m in [0.5, 1)
      e = m <= 0.75f ? E - 3 : E - 2;
      e = e < -127 ? -127 : (e > 127 ? 127 : e);
    }
    const uint32_t sbyte = (uint32_t)(e + 127);
    const float inv = ldexpf(1.f, -e), scl = ldexpf(1.f, e);
    uint32_t wd = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t b = f32x2_to_e2m1x2(v[2 * j] * inv, v[2 * j + 1] * inv);
      wd |= b << (8 * j);
      const uint32_t h = e2m1x2_to_half2(b);
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&h));
      v[2 * j] -= d.x * scl;                     // the residual the next term takes
      v[2 * j + 1] -= d.y * scl;
    }
    // the stage's four scale bytes (blocks of the threads + 0, 4, 8, 12), lowest block first
    const uint32_t s1 = __shfl_down_sync(0xffffffffu, sbyte, 4);
    const uint32_t s2 = __shfl_down_sync(0xffffffffu, sbyte, 8);
    const uint32_t s3 = __shfl_down_sync(0xffffffffu, sbyte, 12);
    word[t] = wd;
    sw[t] = sbyte | (s1 << 8) | (s2 << 16) | (s3 << 24);
  }
}

// The terms of e2m1x4_terms stored to the nd destination pair rows s_p[] (skipping -1), and the
// stage's scale word to their chunks' B scale blocks (chunk s_c[], row s_jr[] of s_npad[] rows).
LL_DEV void e2m1x4_put(const uint32_t (&word)[kBsTermsFp4], const uint32_t (&sw)[kBsTermsFp4], int ch, int nch,
                       int K, int64_t P, int nd, const int* s_p, const int* s_c, const int* s_jr, const int* s_npad,
                       uint8_t* __restrict__ dst, uint32_t* __restrict__ sfb) {
  if (ch >= nch) return;
  const int n_stage = K / 128;
  const int ks = ch / 16;                        // stage of this thread's chunk
  const bool lead = (ch & 15) == 0;              // writes the stage's scale word
  constexpr int WPB = kBsSfBlock / 4;            // words per scale block
  for (int j = 0; j < nd; j++) {
    const int p = s_p[j];
    if (p < 0) continue;
#pragma unroll
    for (int t = 0; t < kBsTermsFp4; t++) {
      reinterpret_cast<uint32_t*>(dst + ((int64_t)t * P + p) * (K / 2))[ch] = word[t];
      if (lead) {
        const int n = t * s_npad[j] + s_jr[j];
        sfb[((int64_t)s_c[j] * n_stage + ks) * WPB + (n % 32) * 4 + (n % 128) / 32] = sw[t];
      }
    }
  }
}

LL_DEV void e2m1x4_store(float (&v)[8], int ch, int nch, int K, int64_t P, int nd, const int* s_p, const int* s_c,
                         const int* s_jr, const int* s_npad, uint8_t* __restrict__ dst, uint32_t* __restrict__ sfb) {
  uint32_t word[kBsTermsFp4], sw[kBsTermsFp4];
  e2m1x4_terms(v, word, sw);
  e2m1x4_put(word, sw, ch, nch, K, P, nd, s_p, s_c, s_jr, s_npad, dst, sfb);
}

// The BS_FP4 activation terms: per row, four rounds of (per 32-element block: max |r|, scale
// 2^e with e the smallest exponent bringing that max into [-6, 6], round r / 2^e to E2M1,
// subtract). Term t of pair row p: packed codes dst[t][p][K/2] (two per byte, even element in
// the low nibble). A 32-element block is 4 neighbouring threads' 8 values, so the block max is
// two shuffles, and a row splits over blocks with no reduction: block (x, y) takes source row x,
// 8-element chunks [256 y, 256 y + 256) (16 stages of 128 K).
// The E8M0 scale bytes go straight into the MMA's B scale blocks of the row's chunk: block
// (chunk c, stage ks) of 512 bytes holds, for B row n = t npad + j (term t, chunk row j; npad =
// the chunk's rows padded to rp = 16, or to 4 for four-row tiles), the row's 4 scale bytes of the
// stage at word (n % 32) * 4 + (n % 128) / 32 (the tcgen05.cp layout).
// The other words are left as they are: they only scale B rows past the chunk's rows (MMA
// columns the epilogue never reads, as the MMA's columns are independent) or past the MMA's N.
template <int SRC, bool TOK>
__global__ void __launch_bounds__(kE3Threads) k_rows_to_e2m1x4(const void* __restrict__ src, int src_rows,
                                                               const int* __restrict__ tok_pos, int k,
                                                               const int* __restrict__ n_valid, int K, int64_t P,
                                                               uint8_t* __restrict__ dst,
                                                               const Chunk* __restrict__ chunks,
                                                               const int* __restrict__ chunk_of,
                                                               uint32_t* __restrict__ sfb, int rp) {
  pdl_wait();
  pdl_launch_next();
  const int r = blockIdx.x;
  if (r >= src_rows) return;
  if (!TOK && n_valid && r >= *n_valid) return;
  const int nch = K / 8;
  const int ch = blockIdx.y * kE3Threads + threadIdx.x;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = 0.f;
  if (ch < nch) load8<SRC>(src, r, K, ch, v);
  // destinations (pair row, chunk, row in the chunk, padded chunk rows), looked up by one thread
  // each so that their loads overlap
  __shared__ int s_p[32], s_c[32], s_jr[32], s_npad[32];
  const int nd = TOK ? k : 1;
  if ((int)threadIdx.x < nd) {
    const int j = threadIdx.x;
    const int p = TOK ? tok_pos[(int64_t)r * k + j] : r;
    s_p[j] = p;
    if (p >= 0) {
      const int c = chunk_of[p];
      const Chunk cc = chunks[c];
      s_c[j] = c;
      s_jr[j] = p - cc.p0;
      s_npad[j] = (cc.n + rp - 1) & ~(rp - 1);
    }
  }
  __syncthreads();
  e2m1x4_store(v, ch, nch, K, P, nd, s_p, s_c, s_jr, s_npad, dst, sfb);
}

// The few-token sort and the x terms in one launch (k_plan_small, then k_rows_to_e2m1x4 on the
// token rows, with the same outputs bit for bit). Every block takes one token row r and 8-element
// chunks [256 y, 256 y + 256) of it, and works out from idx the sort it needs: the experts'
// counts (shared-memory histogram of every pair), their row and chunk offsets (two block scans),
// then for its own token's pairs the position in the sorted order (pairs of one expert keep
// their order), chunk and row in the chunk. The blocks with y = 0 write their token's entries of
// the sort (pair_pos, perm_token, perm_slot, tw, chunk_of, tok_pos); block (0, 0) writes the
// per-expert outputs (offsets, chunks, n_chunks), the -1 of perm_token past the valid pairs, and
// clears the status word; the n_zero ints at `zero` are cleared by all blocks together. Needs
// E <= 4 * kE3Threads and k <= 32.
template <int SRC>
__global__ void __launch_bounds__(kE3Threads) k_plan_rows_to_e2m1x4(
    const int64_t* __restrict__ idx, const float* __restrict__ w, int T, int k, int E, int nmax,
    int* __restrict__ offsets, Chunk* __restrict__ chunks, int* __restrict__ n_chunks, int* __restrict__ perm_token,
    int* __restrict__ perm_slot, int* __restrict__ pair_pos, float* __restrict__ tw, int* __restrict__ tok_pos,
    int* __restrict__ chunk_of, DevStatus* __restrict__ st, int* __restrict__ zero, int n_zero,
    const void* __restrict__ src, int K, int64_t P, uint8_t* __restrict__ dst, uint32_t* __restrict__ sfb) {
  using Scan = cub::BlockScan<int, kE3Threads>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int cnt[4 * kE3Threads], rbase[4 * kE3Threads], cbase[4 * kE3Threads];
  __shared__ int s_p[32], s_c[32], s_jr[32], s_npad[32], s_e[32];
  extern __shared__ int es[];                    // [T k] expert of each pair, -1 if not routed here
  pdl_wait();
  pdl_launch_next();
  const int r = blockIdx.x, tid = threadIdx.x;
  const bool first = blockIdx.x == 0 && blockIdx.y == 0;
  const int np = T * k, nch = K / 8;
  const int ch = blockIdx.y * kE3Threads + tid;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = 0.f;
  if (ch < nch) load8<SRC>(src, r, K, ch, v);
  if (first && tid == 0 && st) *st = DevStatus{0, 0, 0, 0};
  {
    const int nb = gridDim.x * gridDim.y, b = blockIdx.y * gridDim.x + blockIdx.x;
    for (int i = b * kE3Threads + tid; i < n_zero; i += nb * kE3Threads) zero[i] = 0;
  }
  for (int e = tid; e < E; e += kE3Threads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < np; i += kE3Threads) {
    const int64_t e = idx[i];
    const bool ok = e >= 0 && e < E;
    es[i] = ok ? (int)e : -1;
    if (ok) atomicAdd(&cnt[e], 1);
  }
  // x's terms (they depend on x alone), while the idx loads above are answered
  uint32_t word[kBsTermsFp4], swd[kBsTermsFp4];
  e2m1x4_terms(v, word, swd);
  __syncthreads();
  int c4[4], n4[4], ro[4], co[4], agg_rows, agg_ch;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int e = 4 * tid + j;
    c4[j] = e < E ? cnt[e] : 0;
    n4[j] = (c4[j] + nmax - 1) / nmax;
  }
  Scan(tmp).ExclusiveSum(c4, ro, agg_rows);
  __syncthreads();
  Scan(tmp).ExclusiveSum(n4, co, agg_ch);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int e = 4 * tid + j;
    if (e >= E) continue;
    rbase[e] = ro[j];
    cbase[e] = co[j];
    if (first) {
      offsets[e] = ro[j];
      for (int i = 0; i < n4[j]; i++) chunks[co[j] + i] = Chunk{e, ro[j] + i * nmax, min(nmax, c4[j] - i * nmax), 0};
    }
  }
  if (first) {
    if (tid == 0) {
      offsets[E] = agg_rows;
      *n_chunks = agg_ch;
    }
    for (int p = agg_rows + tid; p < np; p += kE3Threads) perm_token[p] = -1;
  }
  __syncthreads();
  // this token's pairs
  if (tid < k) {
    const int i = r * k + tid;
    const int e = es[i];
    int p = -1;
    if (e >= 0) {
      int rank = 0;
      for (int j = 0; j < i; j++) rank += es[j] == e;
      p = rbase[e] + rank;
      const int cr = rank / nmax;
      s_c[tid] = cbase[e] + cr;
      s_jr[tid] = rank - cr * nmax;
      const int rp = nmax < 16 ? 4 : 16;
      s_npad[tid] = (min(nmax, cnt[e] - cr * nmax) + rp - 1) & ~(rp - 1);
      if (blockIdx.y == 0) {
        perm_token[p] = r;
        perm_slot[p] = tid;
        tw[p] = w[i];
        chunk_of[p] = s_c[tid];
      }
    }
    s_p[tid] = p;
    s_e[tid] = e;
    if (blockIdx.y == 0) pair_pos[i] = p;
  }
  __syncthreads();
  e2m1x4_put(word, swd, ch, nch, K, P, k, s_p, s_c, s_jr, s_npad, dst, sfb);
  if (blockIdx.y == 0 && tid < 32) {
    // the token's pair positions by ascending expert id (equal ids in slot order), then -1 for
    // the slots routed elsewhere: lane l's place is the number of valid slots ahead of it
    const int lane = tid;
    const int el = lane < k ? s_e[lane] : -1;
    const int n = __popc(__ballot_sync(0xffffffffu, el >= 0));
    int rank = 0;
    for (int i = 0; i < k; i++) {
      const int ei = __shfl_sync(0xffffffffu, el, i);
      rank += ei >= 0 && (ei < el || (ei == el && i < lane));
    }
    if (lane < k) {
      if (el >= 0) tok_pos[(int64_t)r * k + rank] = s_p[lane];
      if (lane >= n) tok_pos[(int64_t)r * k + lane] = -1;
    }
  }
}

int launch_plan_rows_to_e2m1x4(const int64_t* idx, const float* w, int T, int k, int E, int nmax, int* offsets,
                               Chunk* chunks, int* n_chunks, int* perm_token, int* perm_slot, int* pair_pos, float* tw,
                               int* tok_pos, int* chunk_of, DevStatus* st, int* zero, int n_zero, const void* src,
                               int src_dtype, int K, int64_t P, uint8_t* dst, uint8_t* sfb, cudaStream_t s) {
  if (T <= 0) return LL_OK;
  if (!idx || !w || !src || !dst || !sfb || E <= 0 || E > 4 * kE3Threads || k <= 0 || k > 32 || nmax <= 0 ||
      nmax > 32 || K <= 0 || K % 128 || src_dtype < 0 || src_dtype > 2 || (int64_t)T * k > 2048)
    return LL_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(sfb)) % 16)
    return LL_ERR_ARG;
  uint32_t* sw = reinterpret_cast<uint32_t*>(sfb);
  const dim3 grid(T, (K / 8 + kE3Threads - 1) / kE3Threads);
  const size_t smem = (size_t)T * k * sizeof(int);
#define LL_PE(SRC)                                                                                               \
  return launch_pdl("k_plan_rows_to_e2m1x4", k_plan_rows_to_e2m1x4<SRC>, grid, dim3(kE3Threads), smem, s, idx, w, T, \
                    k, E, nmax, offsets, chunks, n_chunks, perm_token, perm_slot, pair_pos, tw, tok_pos, chunk_of, st, \
                    zero, n_zero, src, K, P, dst, sw)
  if (src_dtype == 0) LL_PE(0);
  if (src_dtype == 1) LL_PE(1);
  LL_PE(2);
#undef LL_PE
}

int launch_rows_to_e2m1x4(const void* src, int src_dtype, int src_rows, const int* tok_pos, int k,
                          const int* n_valid, int K, int64_t P, uint8_t* dst, const Chunk* chunks, const int* chunk_of,
                          int nmax, uint8_t* sfb, cudaStream_t s) {
  if (src_rows <= 0) return LL_OK;
  if (!src || !dst || !chunks || !chunk_of || !sfb || K <= 0 || K % 128 || src_dtype < 0 || src_dtype > 2 ||
      k > 32 || nmax > 32 || 4 * nmax > 128)
    return LL_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(sfb)) % 16)
    return LL_ERR_ARG;
  const bool tok = tok_pos != nullptr;
  uint32_t* sw = reinterpret_cast<uint32_t*>(sfb);
#define LL_E2(SRC, TOKV)                                                                                      \
  LL_TRY(launch_pdl("k_rows_to_e2m1x4", k_rows_to_e2m1x4<SRC, TOKV>,                                        \
                    dim3(src_rows, (K / 8 + kE3Threads - 1) / kE3Threads), dim3(kE3Threads), 0, s, src, src_rows, \
                    tok_pos, k, n_valid, K, P, dst, chunks, chunk_of, sw, nmax < 16 ? 4 : 16))
  if (tok) {
    if (src_dtype == 0) LL_E2(0, true); else if (src_dtype == 1) LL_E2(1, true); else LL_E2(2, true);
  } else {
    if (src_dtype == 0) LL_E2(0, false); else if (src_dtype == 1) LL_E2(1, false); else LL_E2(2, false);
  }
#undef LL_E2
  return LL_OK;
}

int launch_rows_to_e4m3x3(const void* src, int src_dtype, int src_rows, const int* tok_pos, int k,
                          const int* n_valid, int K, int64_t P, uint8_t* dst, float* inv3, cudaStream_t s) {
  if (src_rows <= 0) return LL_OK;
  if (!src || !dst || !inv3 || K <= 0 || K % 8 || K > 8 * kE3Chunks * kE3Threads || src_dtype < 0 || src_dtype > 2)
    return LL_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16) return LL_ERR_ARG;
  const bool tok = tok_pos != nullptr;
#define LL_E3(SRC, TOKV)                                                                              \
  LL_TRY(launch_pdl("k_rows_to_e4m3x3", k_rows_to_e4m3x3<SRC, TOKV>, dim3(src_rows), dim3(kE3Threads), 0, s, src, \
                    src_rows, tok_pos, k, n_valid, K, P, dst, inv3))
  if (tok) {
    if (src_dtype == 0) LL_E3(0, true); else if (src_dtype == 1) LL_E3(1, true); else LL_E3(2, true);
  } else {
    if (src_dtype == 0) LL_E3(0, false); else if (src_dtype == 1) LL_E3(1, false); else LL_E3(2, false);
  }
#undef LL_E3
  return LL_OK;
}

}  // namespace ll
