// Router logits on the tensor cores with fp32-level accuracy: logits[T][E] = x[T][d] . W[E][d]^T.
//
// W (fp32) is split exactly into three bf16 planes, W = W_hi + W_lo + W_lo2 (each plane the
// bf16 rounding of what the planes before it left over; the three carry 24 significant bits,
// all of fp32's). bf16 activations are exact in bf16 and need one plane; fp32 activations are
// split the same way into three planes. The products accumulated in fp32 tensor memory are
//   bf16 x:  W_hi.x + W_lo.x + W_lo2.x                            (all of x.W)
//   fp32 x:  the six plane pairs whose orders sum to at most 2 (hi.hi, lo.hi, lo2.hi, hi.lo,
//            lo.lo, hi.lo2); the three dropped pairs are below 2^-24 relative
// so the logits carry fp32-level error, like the reference's fp32 F.linear, with a different
// summation order.
//
// Tiles: M = 128 experts (the A operand, weight planes from shared memory), N = BN tokens
// (B operand), K = 64 per pipeline stage (128-byte rows, 128-byte swizzle, TMA). The K range
// is split over blockIdx.z when the output tiles alone would leave SMs idle; each split
// writes its own fp32 partial [split][T][E], summed in split order by the selection kernel.
// Warps: 0 TMA producer, 1 MMA issuer (owns the tensor-memory allocation), 2..5 epilogue.
#pragma once
#include "common.cuh"

namespace ll {

constexpr int kRtWarps = 6;

template <int NP, int BN>
struct RouterCfg {
  static constexpr int A_TILE = 128 * 64 * 2;        // one weight plane, 128 rows x 64 k, bf16
  static constexpr int B_TILE = BN * 64 * 2;         // one activation plane
  static constexpr int STAGE = 3 * A_TILE + NP * B_TILE;
  static constexpr int S0 = (200 * 1024) / STAGE;
  static constexpr int STAGES = S0 > 6 ? 6 : S0;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(STAGES >= 2, "shared memory");
};

struct RouterMaps {
  CUtensorMap a[3];   // W_hi, W_lo, W_lo2: [E][d] bf16, box {64, 128}
  CUtensorMap b[3];   // x (or x_hi, x_lo, x_lo2): [T][d] bf16, box {64, BN}
};

LL_DEV uint32_t idesc_bf16_m128(uint32_t n) {
  uint32_t d = 0;
  d |= 1u << 4;          // D format F32
  d |= 1u << 7;          // A format BF16
  d |= 1u << 10;         // B format BF16 (same type as A)
  d |= (n >> 3) << 17;   // both operands K-major
  d |= (128u >> 4) << 24;
  return d;
}

template <int NP, int BN>
__global__ void __launch_bounds__(kRtWarps * 32, 1)
k_router_mma(const __grid_constant__ RouterMaps maps, float* __restrict__ part, int T, int E, int kb_total,
             int kb_per_split, DevStatus* st) {
  using C = RouterCfg<NP, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accfull = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * BN;
  const int kb0 = blockIdx.z * kb_per_split;
  const int kb1 = min(kb_total, kb0 + kb_per_split);
  const int nkb = kb1 - kb0;     // >= 1 by construction of the grid

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_next();                        // (after the allocation)
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < 3; i++) tma_prefetch_desc(&maps.a[i]);
      for (int i = 0; i < NP; i++) tma_prefetch_desc(&maps.b[i]);
      int s = 0;
      uint32_t ph = 0;
      for (int kb = 0; kb < nkb; kb++) {
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, st, 21)) break;
        uint8_t* stage = smem + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        const int kc = (kb0 + kb) * 64;
        for (int i = 0; i < 3; i++) tma_load_2d(stage + i * C::A_TILE, &maps.a[i], &full[s], kc, m0);
        for (int i = 0; i < NP; i++) tma_load_2d(stage + 3 * C::A_TILE + i * C::B_TILE, &maps.b[i], &full[s], kc, n0);
        if (++s == C::STAGES) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_m128(BN);
      int s = 0;
      uint32_t ph = 0;
      bool first = true;
      bool ok = true;
      for (int kb = 0; kb < nkb; kb++) {
        if (!(ok = mbar_wait(&full[s], ph, abort_flag, st, 22))) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * C::STAGE);
        const uint32_t b0 = a0 + 3 * C::A_TILE;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          // (A plane, B plane) products, largest first
          constexpr int NPROD = NP == 1 ? 3 : 6;
#pragma unroll
          for (int p = 0; p < NPROD; p++) {
            const int ai = p < 3 ? p : (p == 4 ? 1 : 0);      // 0 1 2 0 1 0
            const int bi = p < 3 ? 0 : (p == 5 ? 2 : 1);      // 0 0 0 1 1 2
            const uint64_t ad = umma_desc(a0 + ai * C::A_TILE + kk * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = umma_desc(b0 + bi * C::B_TILE + kk * 32, 16, 1024, kSwizzle128B);
            mma_f16_ss(tmem, ad, bd, idesc, first ? 0u : 1u);
            first = false;
          }
        }
        mma_commit(&empty[s]);
        if (++s == C::STAGES) { s = 0; ph ^= 1; }
      }
      mma_commit(accfull);
      // the tensor memory is freed below only once every MMA issued above has completed
      // (a bounded wait that an abort elsewhere does not cut short)
      volatile int keep_waiting = 0;
      mbar_wait(accfull, 0, &keep_waiting, st, 24);
      (void)ok;
    }
  } else {
    // epilogue: warp (2..5) may read TMEM lanes 32 * (warp % 4) .. + 31 = experts of the tile
    const int q = warp & 3;
    const int e = m0 + q * 32 + lane;
    const bool ok = mbar_wait(accfull, 0, abort_flag, st, 23);
    tc_fence_after();
    if (ok) {
      float* out = part + (size_t)blockIdx.z * T * E;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c, v);
        tmem_ld_wait();
        if (e < E) {
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const int t = n0 + c + j;
            if (t < T) out[(size_t)t * E + e] = v[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// An fp32 value as three bf16 planes whose sum is the value exactly (round-to-nearest at each step).
LL_DEV void split_bf16x3(float v, __nv_bfloat16& h, __nv_bfloat16& l, __nv_bfloat16& l2) {
  h = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(h);
  l = __float2bfloat16_rn(r1);
  l2 = __float2bfloat16_rn(r1 - __bfloat162float(l));
}

// W fp32 -> three bf16 planes whose sum is W exactly.
__global__ void k_split_bf16x3(const float* __restrict__ w, __nv_bfloat16* __restrict__ hi,
                               __nv_bfloat16* __restrict__ lo, __nv_bfloat16* __restrict__ lo2, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    split_bf16x3(w[i], hi[i], lo[i], lo2[i]);
}

// The planes [3][E][d] of a LoRA projection matrix for the logits kernel: rows 0..r-1 from W0,
// rows r..2r-1 from W1 (when given); W0 / W1 stored [r][d], or [d][r] when `transposed` (the
// matrix read as its transpose).
__global__ void k_split_lora_planes(const float* __restrict__ W0, const float* __restrict__ W1, bool transposed,
                                    int r, int d, __nv_bfloat16* __restrict__ planes) {
  const int E = W1 ? 2 * r : r;
  const int64_t n = (int64_t)E * d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)(i / d), c = (int)(i % d);
    const float* W = e < r ? W0 : W1;
    const int j = e < r ? e : e - r;
    split_bf16x3(transposed ? W[(int64_t)c * r + j] : W[(int64_t)j * d + c], planes[i], planes[n + i],
                 planes[2 * n + i]);
  }
}

}  // namespace ll
