// Grouped MXFP4 GEMM on the block-scaled tcgen05 MMA (kind::mxf8f6f4), one persistent CTA per
// SM: the forward GEMMs of the routed-expert layer (gate/up with SiTU-GLU, down).
//
// The weights are never decoded. Their E2M1 codes go from HBM to shared memory by TMA (the
// 16 x 4-bit, 16-byte-aligned form the MMA reads: each 8 packed bytes land in 16), their E8M0
// block-32 scales go into tensor memory (tcgen05.cp from a 512-byte block per 128 rows x 128 K,
// laid out once per weight load by ll_moe_prepare), and the MMA applies them itself: W row m,
// K block b contributes code * 2^(scale - 127) exactly. An E8M0 byte >= 253, which the
// reference treats as "this group contributes zero", is laid out as byte 0 (2^-127): its
// products stay below 2^-116 of the activation scale and vanish in the fp32 sums.
//
// The activations (the B operand) are E4M3 and carry no exponent of their own beyond a power
// of two per row, so a row x is held as three E4M3 terms x = (q0 2^-e0 + q1 2^-e1 + q2 2^-e2):
// each term the nearest E4M3 values of what the previous terms left, scaled by a power of two
// that brings the residual's largest entry into [2^7, 2^8). Three terms keep ~12 significant
// bits of every entry (fp16 keeps 11). The terms are stacked along N: the B tile of a chunk of
// n rows is [term][npad rows][128 K], so one MMA of N = 3 npad computes all three partial
// products into adjacent accumulator columns, and the epilogue adds them with their row
// scales: y[m, j] = sum_t D[m, t npad + j] 2^-e_t(j). The B scale factors are all 1.0 (one
// constant block in tensor memory for the whole kernel).
//
// Work units are (chunk of <= N_MAX rows of one expert, m-tile) as in grouped_gemm.cuh, with two
// weight tiles per unit (gate and up for F1; two adjacent 128-row tiles of one stack for F2).
// Warp roles (7 warps): 0 TMA producer (weights, activations, scale blocks of a stage on one
// mbarrier), 1 MMA issuer (tcgen05.cp of the stage's scales, then 4 K-steps x 2 tiles of MMAs,
// one commit releasing the stage), 2..5 epilogue (one TMEM lane quarter each), 6 watcher (waits
// on the mbarriers the issuer depends on and publishes a count it polls). Accumulators are
// double-buffered when tensor memory allows, so the epilogue of a unit overlaps the next unit's
// MMAs. Every wait is bounded (see common.cuh).
#pragma once
#include "grouped_gemm.cuh"

namespace ll {

constexpr int kBsTerms = 3;          // E4M3 terms per activation row
constexpr int kBsSfBlock = 512;      // scale bytes of 128 rows x 128 K (4 per row), tcgen05.cp layout

struct BsArgs {
  const Chunk* chunks;
  const int* n_chunks;
  int mtiles;                 // units per chunk
  int K;                      // reduction length, a multiple of 128
  int e_rows;                 // weight rows per expert
  const uint8_t* sfa[2];      // prepared scale blocks [E][e_rows/128][K/128][512] of tile 0 / 1
  const float* inv3;          // [3][P] 2^-e_t of each activation row's term t
  int prefetch;               // stages the L2 prefetch of weight tiles runs ahead of the loads
  DevStatus* status;
  EpiParams epi;
};

template <int NMAT, int N_MAX>
struct BsCfg {
  static constexpr int kThreads = 7 * 32;
  static constexpr int kEpWarp0 = 2, kEpWarps = 4, kWatchWarp = 6;
  static constexpr int BN = kBsTerms * N_MAX;            // MMA N of a full chunk
  static constexpr int A_TILE = 128 * 128;               // shared bytes of a 128 x 128-K weight tile
  static constexpr int A_TX = 128 * 64;                  // its transaction (packed global) bytes
  static constexpr int B_TILE = BN * 128;
  static constexpr int STAGE0 = NMAT * A_TILE + B_TILE + NMAT * kBsSfBlock;
  static constexpr int STAGE = (STAGE0 + 1023) / 1024 * 1024;
  static constexpr int S0 = (227 * 1024 - 4096) / STAGE;
  static constexpr int S = S0 > 8 ? 8 : S0;
  static_assert(S >= 2, "shared memory budget");
  static constexpr int OFF_SFB = S * STAGE;              // 512 bytes of 0x7f: every B scale 1.0
  static constexpr int OFF_BAR = OFF_SFB + kBsSfBlock;
  static constexpr int N_BARS = 2 * S + 5;
  static constexpr int SMEM = OFF_BAR + N_BARS * 8 + 32 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // tensor memory: accumulators [buffer][tile][BN], then a scale slot (4 columns: 128 rows) per
  // stage and tile, then the constant B scale slot (8 columns: B rows up to 256)
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int SF_COLS = S * NMAT * 4 + 8;
  static_assert(ACC_COLS + SF_COLS <= 512, "tensor memory budget");
  static constexpr int NACC = 2 * ACC_COLS + SF_COLS <= 512 ? 2 : 1;
  static constexpr int SFA_BASE = NACC * ACC_COLS;
  static constexpr int SFB_BASE = SFA_BASE + S * NMAT * 4;
  static constexpr int TMEM_COLS0 = SFB_BASE + 8;
  static constexpr int TMEM_COLS = TMEM_COLS0 <= 32 ? 32 : TMEM_COLS0 <= 64 ? 64 : TMEM_COLS0 <= 128 ? 128
                                   : TMEM_COLS0 <= 256 ? 256 : 512;
  static_assert(N_MAX % 16 == 0 && BN <= 256, "MMA N");
};

template <int NMAT, int N_MAX>
struct BsTma {
  CUtensorMap a[NMAT];          // weight codes, 16 x 4-bit 16-byte-aligned, 128-byte swizzle
  CUtensorMap b[N_MAX / 16];    // b[c - 1]: [3 terms][16 c rows][128 K] E4M3, 128-byte swizzle
};

template <int EPI, int NMAT, int N_MAX>
__global__ void __launch_bounds__(BsCfg<NMAT, N_MAX>::kThreads, 1)
grouped_mxfp4_bs_gemm(const __grid_constant__ BsTma<NMAT, N_MAX> tm, const BsArgs args) {
  using C = BsCfg<NMAT, N_MAX>;
  static_assert(EPI == EPI_F1 || EPI == EPI_F2 || EPI == EPI_STORE, "epilogue");
  // a single-product epilogue takes two adjacent 128-row tiles of one stack as its two tiles
  constexpr bool PAIR = NMAT == 2 && EPI != EPI_F1;
  constexpr int TILE_ROWS = PAIR ? 256 : 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + C::S;
  uint64_t* accfull = empty + C::S;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* ready_seq = tmem_slot + 2;      // events the watcher has seen complete (see below)

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_units = (*args.n_chunks) * args.mtiles;
  if ((int)blockIdx.x >= n_units || args.K <= 0 || args.K % 128) return;   // uniform: nothing allocated yet
  const int n_stage = args.K / 128;
  const int tiles128 = args.e_rows / 128;      // 128-row tiles per expert (scale-block index)

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], C::kEpWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *ready_seq = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < kBsSfBlock / 4) reinterpret_cast<uint32_t*>(smem + C::OFF_SFB)[threadIdx.x] = 0x7f7f7f7fu;
  fence_async_smem();                       // the constant block is read by tcgen05.cp (async proxy)
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  DevStatus* st = args.status;

  if (warp == 0) {
    // ------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      for (int i = 0; i < NMAT; i++) tma_prefetch_desc(&tm.a[i]);
      for (int i = 0; i < N_MAX / 16; i++) tma_prefetch_desc(&tm.b[i]);
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      // weight tiles and scale blocks are prefetched into L2 args.prefetch stages ahead of their
      // loads: the shared-memory ring alone holds too few bytes to cover the DRAM latency
      int pu = blockIdx.x, pks = 0;
      auto prefetch_next = [&]() {
        if (pu >= n_units) return;
        const Chunk pc = args.chunks[pu / args.mtiles];
        const int pmt = pu % args.mtiles;
        const int prow = pc.e * args.e_rows + pmt * TILE_ROWS;
        const int ptile = pc.e * tiles128 + pmt * (TILE_ROWS / 128);
#pragma unroll
        for (int i = 0; i < (PAIR ? 1 : NMAT); i++) tma_prefetch_l2_2d(&tm.a[i], pks * 128, prow);
#pragma unroll
        for (int i = 0; i < NMAT; i++)
          bulk_prefetch_l2(PAIR ? args.sfa[0] + ((size_t)(ptile + i) * n_stage + pks) * kBsSfBlock
                                : args.sfa[i] + ((size_t)ptile * n_stage + pks) * kBsSfBlock, kBsSfBlock);
        if (++pks == n_stage) { pks = 0; pu += gridDim.x; }
      };
      for (int i = 0; i < args.prefetch; i++) prefetch_next();
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int mt = u % args.mtiles;
        const int row = ch.e * args.e_rows + mt * TILE_ROWS;
        const int tile0 = ch.e * tiles128 + mt * (TILE_ROWS / 128);
        const int npad = (ch.n + 15) & ~15;
        const uint32_t tx = NMAT * C::A_TX + kBsTerms * npad * 128 + NMAT * kBsSfBlock;
        for (int ks = 0; ks < n_stage && ok; ks++) {
          if (!(ok = mbar_wait_sleep(&empty[s], ph ^ 1, abort_flag, st, 21, 256))) break;
          uint8_t* stage = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], tx);
          if (PAIR) {
            tma_load_2d(stage, &tm.a[0], &full[s], ks * 128, row);     // 256 rows: both tiles
          } else {
#pragma unroll
            for (int i = 0; i < NMAT; i++) tma_load_2d(stage + i * C::A_TILE, &tm.a[i], &full[s], ks * 128, row);
          }
          tma_load_3d(stage + NMAT * C::A_TILE, &tm.b[npad / 16 - 1], &full[s], ks * 128, ch.p0, 0);
#pragma unroll
          for (int i = 0; i < NMAT; i++) {
            const uint8_t* src = PAIR ? args.sfa[0] + ((size_t)(tile0 + i) * n_stage + ks) * kBsSfBlock
                                      : args.sfa[i] + ((size_t)tile0 * n_stage + ks) * kBsSfBlock;
            bulk_load(stage + NMAT * C::A_TILE + C::B_TILE + i * kBsSfBlock, src, kBsSfBlock, &full[s]);
          }
          issued++;
          if (args.prefetch > 0) prefetch_next();
          if (++s == C::S) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < C::S && i < issued; i++) {   // drain: the last stages' bytes landed
        if (--s < 0) { s = C::S - 1; ph ^= 1; }
        mbar_wait_sleep(&full[s], ph, abort_flag, st, 22, 256);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // B rows 0..127 and 128..255 (an MMA of N > 128 reads the second block)
      tmem_cp_32x128b_x4(tmem + C::SFB_BASE, umma_desc(smem_u32(smem + C::OFF_SFB), 128, 128, kSwizzleNone));
      tmem_cp_32x128b_x4(tmem + C::SFB_BASE + 4, umma_desc(smem_u32(smem + C::OFF_SFB), 128, 128, kSwizzleNone));
      // The issuer never waits on an mbarrier (a wait in the thread that issues tcgen05.mma
      // stalls its MMA stream by hundreds of cycles): the watcher warp waits for each event (an
      // accumulator buffer drained, a stage's bytes landed) in the order the issuer needs them
      // and counts them in ready_seq, which the issuer polls.
      int s = 0, ab = 0;
      uint32_t ev = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int npad = (ch.n + 15) & ~15;
        const uint32_t n_mma = kBsTerms * npad;
        if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 23))) break;
        tc_fence_after();
        for (int ks = 0; ks < n_stage; ks++) {
          if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 24))) break;
          tc_fence_after();
          uint8_t* stage = smem + s * C::STAGE;
          const uint32_t a0 = smem_u32(stage), b0 = smem_u32(stage + NMAT * C::A_TILE);
          const uint32_t sf0 = smem_u32(stage + NMAT * C::A_TILE + C::B_TILE);
#pragma unroll
          for (int i = 0; i < NMAT; i++)
            tmem_cp_32x128b_x4(tmem + C::SFA_BASE + (s * NMAT + i) * 4,
                               umma_desc(sf0 + i * kBsSfBlock, 128, 128, kSwizzleNone));
          const uint64_t bdesc0 = umma_desc(b0, 16, 1024, kSwizzle128B);
#pragma unroll
          for (int kb = 0; kb < 4; kb++) {
            const uint32_t idesc = idesc_mxf4xe4m3_m128(n_mma, kb, kb);
#pragma unroll
            for (int i = 0; i < NMAT; i++) {
              const uint64_t adesc = umma_desc(a0 + i * C::A_TILE, 16, 1024, kSwizzle128B) + kb * 2;
              mma_mxf8f6f4_bs(tmem + ab * C::ACC_COLS + i * C::BN, adesc, bdesc0 + kb * 2, idesc,
                              tmem + C::SFA_BASE + (s * NMAT + i) * 4 + ((uint32_t)kb << 30),
                              tmem + C::SFB_BASE + ((uint32_t)kb << 30), (ks | kb) ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);                 // stage (and its scale slots) free once these finish
          if (++s == C::S) s = 0;
        }
        if (!ok) break;
        mma_commit(&accfull[ab]);
        if (++ab == C::NACC) ab = 0;
      }
      mma_commit(drain);                         // completes once every MMA issued above finished
      volatile int keep_waiting = 0;             // wait for them even after an abort
      mbar_wait_sleep(drain, 0, &keep_waiting, st, 25, 256);
    }
    __syncwarp();
  } else if (warp == C::kWatchWarp) {
    // ---------------------------------------------------------------------- watcher
    // The issuer's events in its order: per unit, its accumulator buffer drained by the
    // epilogue, then each stage's bytes landed. Bounded waits; after an abort the count still
    // advances (the issuer sees the abort flag and stops).
    if (lane == 0) {
      int s = 0, ab = 0;
      uint32_t ph = 0, abph = 0, ev = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 27);
        seq_publish(ready_seq, ++ev);
        for (int ks = 0; ks < n_stage; ks++) {
          mbar_wait(&full[s], ph, abort_flag, st, 28);
          seq_publish(ready_seq, ++ev);
          if (++s == C::S) { s = 0; ph ^= 1; }
        }
        if (++ab == C::NACC) { ab = 0; abph ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------------ epilogue
    const int q = warp & 3;                      // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const EpiParams& ep = args.epi;
    const int* __restrict__ perm = ep.perm_token;
    const float* __restrict__ inv3 = args.inv3;
    const float* __restrict__ tw = ep.tw;
    const float* __restrict__ dlt_g = ep.delta_g;
    const float* __restrict__ dlt_u = ep.delta_u;
    float* __restrict__ Go = ep.G;
    float* __restrict__ Uo = ep.U;
    __half* __restrict__ Ho = ep.H;
    float* __restrict__ Yo = ep.Y;
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Chunk ch = args.chunks[u / args.mtiles];
      const int npad = (ch.n + 15) & ~15;
      if (!(ok = mbar_wait_sleep(&accfull[ab], abph, abort_flag, st, 26, 512))) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * C::ACC_COLS;
#pragma unroll 1
      for (int pm = 0; pm < (PAIR ? 2 : 1); pm++) {
        const int mt = (u % args.mtiles) * (PAIR ? 2 : 1) + pm;    // 128-row tile of the output
        const int m = mt * 128 + row;
        const bool mvalid = m < ep.M;
        const uint32_t c0 = tbase + (PAIR ? pm : 0) * C::BN;        // this product's accumulator
        for (int j0 = 0; j0 < npad; j0 += 16) {
          // the three terms' partial products of 16 tokens (and of the up projection for F1)
          uint32_t d0[16], d1[16], d2[16], e0[16], e1[16], e2[16];
          tmem_ld16_u(c0 + j0, d0);
          tmem_ld16_u(c0 + npad + j0, d1);
          tmem_ld16_u(c0 + 2 * npad + j0, d2);
          if (EPI == EPI_F1) {                   // the up projection: tile 1's accumulator
            tmem_ld16_u(c0 + C::BN + j0, e0);
            tmem_ld16_u(c0 + C::BN + npad + j0, e1);
            tmem_ld16_u(c0 + C::BN + 2 * npad + j0, e2);
          }
          tmem_ld_wait();
          tmem_regs_ready(d0);
          tmem_regs_ready(d1);
          tmem_regs_ready(d2);
          if (EPI == EPI_F1) {
            tmem_regs_ready(e0);
            tmem_regs_ready(e1);
            tmem_regs_ready(e2);
          }
#pragma unroll
          for (int jj = 0; jj < 16; jj++) {
            const int j = j0 + jj;
            if (j >= ch.n || !mvalid) continue;
            const int p = ch.p0 + j;
            const float i0 = inv3[p], i1 = inv3[ep.P + p], i2 = inv3[2 * ep.P + p];
            const float v = fmaf(__uint_as_float(d2[jj]), i2,
                                 fmaf(__uint_as_float(d1[jj]), i1, __uint_as_float(d0[jj]) * i0));
            const size_t o = (size_t)p * ep.M + m;
            if (EPI == EPI_F1) {
              const int t = perm ? perm[p] : p;
              const size_t tmo = (size_t)t * ep.M + m;
              const float gate = v + dlt_g[tmo];
              const float up = fmaf(__uint_as_float(e2[jj]), i2,
                                    fmaf(__uint_as_float(e1[jj]), i1, __uint_as_float(e0[jj]) * i0)) + dlt_u[tmo];
              Go[o] = gate;
              Uo[o] = up;
              Ho[o] = __float2half_rn(situ_glu_fwd(gate, up));
            } else if (EPI == EPI_F2) {
              Yo[o] = v * tw[p];
            } else {
              Yo[o] = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[ab]);
      if (++ab == C::NACC) { ab = 0; abph ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ll
