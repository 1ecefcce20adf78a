// Grouped MXFP4 GEMM on the block-scaled tcgen05 MMAs, one persistent CTA per SM: the forward
// GEMMs of the routed-expert layer (gate/up with SiTU-GLU, down).
//
// The weights are never decoded. Their E2M1 codes go from HBM to shared memory by TMA and their
// E8M0 block-32 scales into tensor memory (tcgen05.cp from a 512-byte block per 128 rows x 128
// K, laid out once per weight load by ll_moe_prepare); the MMA applies the scales itself: W row
// m, K block b contributes code * 2^(scale - 127) exactly. An E8M0 byte >= 253, which the
// reference treats as "this group contributes zero", is laid out as byte 0 (2^-127): its
// products vanish in the fp32 sums.
//
// The activations (the B operand) are a short sum of low-precision terms stacked along N: the B
// tile of a chunk of n rows is [term][npad rows][K] (n padded to 16 rows, or to 4 for tiles of at
// most 4 rows), so one MMA of N = terms * npad computes every term's partial product into
// adjacent accumulator columns, and the epilogue adds them.
// Two kinds:
//   BS_FP4  kind::mxf4 (K = 64 per MMA): the weights stay packed in shared memory (half the
//           bytes the tensor core reads per weight element), and the activations are four E2M1
//           terms, each with its own E8M0 scale per 32 K elements (the nearest E2M1 values of
//           what the earlier terms left, scaled into [-6, 6] block by block); four terms keep an
//           activation row to ~4e-5 relative. The B scales come per stage from blocks laid out
//           per chunk (bs_ops.cu). Used for chunks of up to 32 rows.
//   BS_FP8  kind::mxf8f6f4 (K = 32 per MMA): the weights' codes unpacked to one per byte (TMA
//           16 x 4-bit 16-byte-aligned form), the activations three E4M3 terms with one
//           power-of-two scale per row and term (applied in the epilogue; the B scale factors
//           are a constant 1.0 block). Three terms keep ~12 significant bits. Used for chunks of
//           up to 64 rows (four E2M1 terms of 64 rows would need 2 x 256 accumulator columns).
//
// Work units are (chunk of <= N_MAX rows of one expert, m-tile) as in grouped_gemm.cuh, with two
// weight tiles per unit (gate and up for F1; two adjacent 128-row tiles of one stack for F2).
// With few units (decode) the units' K stages are shared out evenly over the CTAs instead and a
// unit cut between CTAs is finished from fp32 partials (BsSegs).
// Warp roles (7 warps): 0 TMA producer (weights, activations, scale blocks of a stage on one
// mbarrier), 1 MMA issuer (tcgen05.cp of the stage's scales, then the K-steps x 2 tiles of
// MMAs, one commit releasing the stage), 2..5 epilogue (one TMEM lane quarter each), 6 watcher
// (waits on the mbarriers the issuer depends on and publishes a count it polls). Accumulators
// are double-buffered when tensor memory allows, so the epilogue of a unit overlaps the next
// unit's MMAs. Every wait is bounded (see common.cuh).
#pragma once
#include "grouped_gemm.cuh"

namespace ll {

enum BsKind : int { BS_FP8 = 0, BS_FP4 = 1 };

constexpr int kBsSfBlock = 512;      // scale bytes of 128 rows x 128 K (4 per row), tcgen05.cp layout

template <int KIND>
struct BsTerms {
  static constexpr int value = KIND == BS_FP4 ? 4 : 3;
};

struct BsArgs {
  const Chunk* chunks;
  const int* n_chunks;
  int mtiles;                 // units per chunk
  int K;                      // reduction length, a multiple of 128
  int e_rows;                 // weight rows per expert
  const uint8_t* sfa[2];      // prepared weight scale blocks [E][e_rows/128][K/128][512] of tile 0 / 1
  const uint8_t* sfb;         // BS_FP4: activation scale blocks [chunk][K/128][blocks][512]
  const float* inv3;          // BS_FP8: [3][P] 2^-e_t of each activation row's term t
  int prefetch;               // stages the L2 prefetch of weight tiles runs ahead of the loads
  DevStatus* status;
  EpiParams epi;
  // Balanced split (few units, see BsSegs): partial sums of the units several CTAs share, two
  // slots per CTA [slot][2 products][N_MAX][128 rows] fp32, and four arrival counters per unit
  // (one per epilogue warp; zero before the launch, the last arrival sets its counter back to
  // zero). Off when split_part is null.
  float* split_part;
  int* split_cnt;
  int split_units;            // units the counters cover: the split runs only for n_units <= this
  int split_ctas;             // CTAs split_part has slots for
  int chunks_cap;             // entries the chunk list has room for (0: unknown)
};

// The (unit, K-stage range) pieces a CTA runs. Without the split, CTA b takes whole units b,
// b + G, b + 2G, ... (G = gridDim.x). With it, the n_units * n_stage stages in unit order are cut
// into G contiguous ranges of equal length (+-1), CTA b taking stages [b tot / G, (b+1) tot / G):
// every CTA streams the same number of weight bytes however few units there are. A range is
// whole units plus at most a partial first and a partial last piece; a unit cut across CTAs
// b0..b1 (b0 = the owner of its first stage) is finished by whichever of them arrives last,
// which adds the pieces' fp32 partials in the order b0, b0 + 1, ..., b1.
struct BsSeg {
  int u, ks0, ks1;            // unit and its stages [ks0, ks1)
  int piece;                  // 0: the first piece of this CTA's range, 1: a later one
};
struct BsSegs {
  long long g, end, tot;
  int ns, G;
  bool split, first = true;
  LL_DEV BsSegs(bool sp, int n_units, int n_stage) : ns(n_stage), G((int)gridDim.x), split(sp) {
    tot = (long long)n_units * n_stage;
    if (sp) {
      g = begin_of(blockIdx.x);
      end = begin_of(blockIdx.x + 1);
    } else {
      g = (long long)blockIdx.x * n_stage;
      end = tot;
    }
  }
  LL_DEV long long begin_of(int b) const { return tot * b / G; }
  // the CTA whose range holds stage gs: the largest b with begin_of(b) <= gs
  LL_DEV int owner(long long gs) const { return (int)(((gs + 1) * G - 1) / tot); }
  LL_DEV bool next(BsSeg& s) {
    if (g >= end) return false;
    s.u = (int)(g / ns);
    const long long u0 = (long long)s.u * ns, u1 = u0 + ns;
    s.ks0 = (int)(g - u0);
    s.ks1 = (int)((u1 < end ? u1 : end) - u0);
    s.piece = first ? 0 : 1;
    first = false;
    g = split ? u1 : u1 + (long long)(G - 1) * ns;
    return true;
  }
  // slot of the o-th piece of unit u (o = 0 .. nseg-1, CTAs b0 + o)
  LL_DEV int slot(int u, int o, int b0) const {
    return 2 * (b0 + o) + ((o == 0 && begin_of(b0) < (long long)u * ns) ? 1 : 0);
  }
};

// Row padding of a chunk's activation rows in the B tile (the MMA N is terms x padded rows):
// 16 rows, or 4 for the four-row tiles of tiny batches (a chunk of at most 4 rows; MMA N = 16,
// a quarter of the B bytes a stage of a 16-row tile moves), and the tensor maps per tile height.
template <int N_MAX>
struct BsRows {
  static constexpr int rp = N_MAX < 16 ? 4 : 16;
  static constexpr int maps = N_MAX / rp;
  static LL_DEV int pad(int n) { return (n + rp - 1) & ~(rp - 1); }
};

template <int NMAT, int N_MAX, int KIND>
struct BsCfg {
  static constexpr int kThreads = 7 * 32;
  static constexpr int kEpWarp0 = 2, kEpWarps = 4, kWatchWarp = 6;
  static constexpr bool FP4 = KIND == BS_FP4;
  static constexpr int NT = BsTerms<KIND>::value;         // activation terms
  static constexpr int BN = NT * N_MAX;                   // MMA N of a full chunk
  static constexpr int KMMA = FP4 ? 64 : 32;              // K per MMA instruction
  static constexpr int ROWB = FP4 ? 64 : 128;             // shared bytes of one operand row (128 K)
  static constexpr int A_TILE = 128 * ROWB;               // shared bytes of a 128 x 128-K weight tile
  static constexpr int A_TX = 128 * 64;                   // its transaction (packed global) bytes
  static constexpr int B_TILE = BN * ROWB;
  static constexpr int SFB_BLKS = FP4 ? (BN + 127) / 128 : 0;   // B scale blocks per stage
  static constexpr int STAGE0 = NMAT * A_TILE + B_TILE + (NMAT + SFB_BLKS) * kBsSfBlock;
  static constexpr int STAGE = (STAGE0 + 1023) / 1024 * 1024;
  static constexpr int S0 = (227 * 1024 - 4096) / STAGE;
  static constexpr int S = S0 > 12 ? 12 : S0;
  static_assert(S >= 2, "shared memory budget");
  static constexpr int OFF_SFB = S * STAGE;               // BS_FP8: 512 bytes of 0x7f (every B scale 1.0)
  static constexpr int OFF_BAR = OFF_SFB + kBsSfBlock;
  static constexpr int N_BARS = 2 * S + 5;
  static constexpr int SMEM = OFF_BAR + N_BARS * 8 + 32 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // tensor memory: accumulators [buffer][tile][BN], the A scale slots (4 columns: 128 rows) per
  // stage and tile, then the B scale slots (8 columns: B rows up to 256), one per stage (BS_FP4)
  // or one constant slot (BS_FP8)
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int SFB_SLOTS = FP4 ? S : 1;
  static constexpr int SF_COLS = S * NMAT * 4 + SFB_SLOTS * 8;
  static_assert(ACC_COLS + SF_COLS <= 512, "tensor memory budget");
  static constexpr int NACC = 2 * ACC_COLS + SF_COLS <= 512 ? 2 : 1;
  static constexpr int SFA_BASE = NACC * ACC_COLS;
  static constexpr int SFB_BASE = SFA_BASE + S * NMAT * 4;
  static constexpr int TMEM_COLS0 = SFB_BASE + SFB_SLOTS * 8;
  static constexpr int TMEM_COLS = TMEM_COLS0 <= 32 ? 32 : TMEM_COLS0 <= 64 ? 64 : TMEM_COLS0 <= 128 ? 128
                                   : TMEM_COLS0 <= 256 ? 256 : 512;
  static_assert((N_MAX % 16 == 0 || (N_MAX == 4 && FP4)) && BN <= 256, "MMA N");
  static_assert(A_TILE % 1024 == 0 && (16 * ROWB) % 1024 == 0, "1024-byte aligned operand tiles and terms");
};

template <int NMAT, int N_MAX, int KIND>
struct BsTma {
  CUtensorMap a[NMAT];          // weight codes (BS_FP4 packed, 64-byte swizzle; BS_FP8 unpacked, 128)
  CUtensorMap b[BsRows<N_MAX>::maps];   // b[c - 1]: [terms][RP c rows][128 K] activation terms
};

// UMMA descriptor of a K-major operand tile (rows of ROWB bytes, the swizzle of that width).
template <int KIND>
LL_DEV uint64_t bs_desc(uint32_t addr) {
  return KIND == BS_FP4 ? umma_desc(addr, 16, 512, kSwizzle64B) : umma_desc(addr, 16, 1024, kSwizzle128B);
}

template <int EPI, int NMAT, int N_MAX, int KIND>
__global__ void __launch_bounds__(BsCfg<NMAT, N_MAX, KIND>::kThreads, 1)
grouped_mxfp4_bs_gemm(const __grid_constant__ BsTma<NMAT, N_MAX, KIND> tm, const BsArgs args) {
  using C = BsCfg<NMAT, N_MAX, KIND>;
  constexpr int NT = C::NT;
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
  if (args.K <= 0 || args.K % 128) {   // uniform: nothing allocated yet
    pdl_wait();
    return;
  }
  const int n_stage = args.K / 128;
  const int tiles128 = args.e_rows / 128;      // 128-row tiles per expert (scale-block index)

  // Prologue (barriers, tensor memory, descriptor prefetch) before the wait for the kernels
  // this one depends on: it reads nothing they write.
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], C::kEpWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *ready_seq = 0;
    fence_barrier_init();
  }
  if (!C::FP4 && threadIdx.x < kBsSfBlock / 4) reinterpret_cast<uint32_t*>(smem + C::OFF_SFB)[threadIdx.x] = 0x7f7f7f7fu;
  fence_async_smem();                       // the constant block is read by tcgen05.cp (async proxy)
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < NMAT; i++) tma_prefetch_desc(&tm.a[i]);
    for (int i = 0; i < BsRows<N_MAX>::maps; i++) tma_prefetch_desc(&tm.b[i]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  DevStatus* st = args.status;
  pdl_launch_next();                        // (after the allocation: see pdl_launch_next)
  pdl_wait();
  const int n_units = (*args.n_chunks) * args.mtiles;
  // the chunk of this CTA's first unit without the split (unit blockIdx.x), loaded beside the
  // count instead of after it (inside the chunk list's capacity; used only if that unit exists)
  const int c_first_i = (int)blockIdx.x / args.mtiles;
  Chunk c_first{};
  if (warp == 0 && lane == 0 && c_first_i < args.chunks_cap) c_first = args.chunks[c_first_i];
  // the balanced split for a few waves of units (at least one unit a CTA: with fewer it measured
  // slower, the partial sums' round trip costing more than the bytes it evens out)
  const bool split = args.split_part != nullptr && n_units >= (int)gridDim.x && n_units <= args.split_units &&
                     (int)gridDim.x <= args.split_ctas;
  if (!split && (int)blockIdx.x >= n_units) {   // uniform per block: no unit for this one
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
    return;
  }

  if (warp == 0) {
    // ------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      // A x coordinate of a stage: packed bytes (BS_FP4, uint8 map) or 4-bit elements (BS_FP8)
      constexpr int AX = C::FP4 ? 64 : 128;
      // weight tiles and scale blocks are prefetched into L2 args.prefetch stages ahead of their
      // loads (off by default: measured slower on configs[1])
      int pu = blockIdx.x, pks = 0;
      const int prefetch = split ? 0 : args.prefetch;
      auto prefetch_next = [&]() {
        if (pu >= n_units) return;
        const Chunk pc = args.chunks[pu / args.mtiles];
        const int pmt = pu % args.mtiles;
        const int prow = pc.e * args.e_rows + pmt * TILE_ROWS;
        const int ptile = pc.e * tiles128 + pmt * (TILE_ROWS / 128);
#pragma unroll
        for (int i = 0; i < (PAIR ? 1 : NMAT); i++) tma_prefetch_l2_2d(&tm.a[i], pks * AX, prow);
#pragma unroll
        for (int i = 0; i < NMAT; i++)
          bulk_prefetch_l2(PAIR ? args.sfa[0] + ((size_t)(ptile + i) * n_stage + pks) * kBsSfBlock
                                : args.sfa[i] + ((size_t)ptile * n_stage + pks) * kBsSfBlock, kBsSfBlock);
        if (++pks == n_stage) { pks = 0; pu += gridDim.x; }
      };
      for (int i = 0; i < prefetch; i++) prefetch_next();
      BsSegs segs(split, n_units, n_stage);
      BsSeg sg;
      while (ok && segs.next(sg)) {
        const int u = sg.u;
        const int ci = u / args.mtiles;
        const Chunk ch = (!split && u == (int)blockIdx.x && ci < args.chunks_cap) ? c_first : args.chunks[ci];
        const int mt = u % args.mtiles;
        const int row = ch.e * args.e_rows + mt * TILE_ROWS;
        const int tile0 = ch.e * tiles128 + mt * (TILE_ROWS / 128);
        const int npad = BsRows<N_MAX>::pad(ch.n);
        const uint32_t tx = NMAT * C::A_TX + NT * npad * C::ROWB + (NMAT + C::SFB_BLKS) * kBsSfBlock;
        for (int ks = sg.ks0; ks < sg.ks1 && ok; ks++) {
          if (!(ok = mbar_wait_sleep(&empty[s], ph ^ 1, abort_flag, st, 21, 256))) break;
          uint8_t* stage = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], tx);
          if (PAIR) {
            tma_load_2d(stage, &tm.a[0], &full[s], ks * AX, row);     // 256 rows: both tiles
          } else {
#pragma unroll
            for (int i = 0; i < NMAT; i++) tma_load_2d(stage + i * C::A_TILE, &tm.a[i], &full[s], ks * AX, row);
          }
          tma_load_3d(stage + NMAT * C::A_TILE, &tm.b[npad / BsRows<N_MAX>::rp - 1], &full[s], ks * C::ROWB, ch.p0,
                      0);
          uint8_t* sf = stage + NMAT * C::A_TILE + C::B_TILE;
#pragma unroll
          for (int i = 0; i < NMAT; i++) {
            const uint8_t* src = PAIR ? args.sfa[0] + ((size_t)(tile0 + i) * n_stage + ks) * kBsSfBlock
                                      : args.sfa[i] + ((size_t)tile0 * n_stage + ks) * kBsSfBlock;
            bulk_load(sf + i * kBsSfBlock, src, kBsSfBlock, &full[s]);
          }
          if (C::FP4)
            bulk_load(sf + NMAT * kBsSfBlock, args.sfb + ((size_t)ci * n_stage + ks) * C::SFB_BLKS * kBsSfBlock,
                      C::SFB_BLKS * kBsSfBlock, &full[s]);
          issued++;
          if (prefetch > 0) prefetch_next();
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
      if (!C::FP4) {   // constant B scales: rows 0..127 and 128..255 (an MMA of N > 128 reads both)
        tmem_cp_32x128b_x4(tmem + C::SFB_BASE, umma_desc(smem_u32(smem + C::OFF_SFB), 128, 128, kSwizzleNone));
        tmem_cp_32x128b_x4(tmem + C::SFB_BASE + 4, umma_desc(smem_u32(smem + C::OFF_SFB), 128, 128, kSwizzleNone));
      }
      // The issuer never waits on an mbarrier (a wait in the thread that issues tcgen05.mma
      // stalls its MMA stream by hundreds of cycles): the watcher warp waits for each event (an
      // accumulator buffer drained, a stage's bytes landed) in the order the issuer needs them
      // and counts them in ready_seq, which the issuer polls.
      int s = 0, ab = 0;
      uint32_t ev = 0;
      bool ok = true;
      BsSegs segs(split, n_units, n_stage);
      BsSeg sg;
      while (ok && segs.next(sg)) {
        const Chunk ch = args.chunks[sg.u / args.mtiles];
        const int npad = BsRows<N_MAX>::pad(ch.n);
        const uint32_t n_mma = NT * npad;
        if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 23))) break;
        tc_fence_after();
        for (int ks = sg.ks0; ks < sg.ks1; ks++) {
          if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 24))) break;
          tc_fence_after();
          uint8_t* stage = smem + s * C::STAGE;
          const uint32_t a0 = smem_u32(stage), b0 = smem_u32(stage + NMAT * C::A_TILE);
          const uint32_t sf0 = smem_u32(stage + NMAT * C::A_TILE + C::B_TILE);
#pragma unroll
          for (int i = 0; i < NMAT; i++)
            tmem_cp_32x128b_x4(tmem + C::SFA_BASE + (s * NMAT + i) * 4,
                               umma_desc(sf0 + i * kBsSfBlock, 128, 128, kSwizzleNone));
          const uint32_t sfb = C::FP4 ? tmem + C::SFB_BASE + s * 8 : tmem + C::SFB_BASE;
          if (C::FP4) {
#pragma unroll
            for (int bl = 0; bl < C::SFB_BLKS; bl++)
              tmem_cp_32x128b_x4(sfb + bl * 4, umma_desc(sf0 + (NMAT + bl) * kBsSfBlock, 128, 128, kSwizzleNone));
          }
          const uint64_t bdesc0 = bs_desc<KIND>(b0);
#pragma unroll
          for (int kk = 0; kk < 128 / C::KMMA; kk++) {
            const uint32_t sfid = C::FP4 ? 2 * kk : kk;      // first scale byte this MMA reads
            const uint32_t idesc =
                C::FP4 ? idesc_mxf4_m128(n_mma, sfid, sfid) : idesc_mxf4xe4m3_m128(n_mma, sfid, sfid);
#pragma unroll
            for (int i = 0; i < NMAT; i++) {
              const uint64_t adesc = bs_desc<KIND>(a0 + i * C::A_TILE) + kk * 2;   // + 32 bytes of K
              const uint32_t d = tmem + ab * C::ACC_COLS + i * C::BN;
              const uint32_t sfa = tmem + C::SFA_BASE + (s * NMAT + i) * 4 + (sfid << 30);
              if (C::FP4)
                mma_mxf4_bs(d, adesc, bdesc0 + kk * 2, idesc, sfa, sfb + (sfid << 30), (ks != sg.ks0 || kk) ? 1u : 0u);
              else
                mma_mxf8f6f4_bs(d, adesc, bdesc0 + kk * 2, idesc, sfa, sfb + (sfid << 30),
                                (ks != sg.ks0 || kk) ? 1u : 0u);
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
      BsSegs segs(split, n_units, n_stage);
      BsSeg sg;
      while (segs.next(sg)) {
        mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 27);
        seq_publish(ready_seq, ++ev);
        for (int ks = sg.ks0; ks < sg.ks1; ks++) {
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
    // the per-row output of a finished (token row p, output row m) from its accumulator sums, for
    // the units finished from split partials (the whole-unit path below has the same lines inline)
    auto finish = [&](int p, int m, float v, float up) {
      const size_t o = (size_t)p * ep.M + m;
      if (EPI == EPI_F1) {
        const int tk = perm ? perm[p] : p;
        const size_t tmo = (size_t)tk * ep.M + m;
        const float gate = v + dlt_g[tmo];
        up += dlt_u[tmo];
        Go[o] = gate;
        Uo[o] = up;
        Ho[o] = __float2half_rn(situ_glu_fwd(gate, up));
      } else if (EPI == EPI_F2) {
        Yo[o] = v * tw[p];
      } else {
        Yo[o] = v;
      }
    };
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    BsSegs segs(split, n_units, n_stage);
    BsSeg sg;
    while (ok && segs.next(sg)) {
      const int u = sg.u;
      const Chunk ch = args.chunks[u / args.mtiles];
      const int npad = BsRows<N_MAX>::pad(ch.n);
      // a piece of a split unit: its partial sums go to this CTA's slot
      const bool whole = sg.ks0 == 0 && sg.ks1 == n_stage;
      float* part = whole ? nullptr : args.split_part + (size_t)(2 * blockIdx.x + sg.piece) * 2 * N_MAX * 128;
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
          // the terms' partial products of 16 tokens (and of the up projection for F1)
          uint32_t d[NT][16], e[EPI == EPI_F1 ? NT : 1][16];
          if (BsRows<N_MAX>::rp == 4) {
            // four rows a term: one 16-column load holds every term's columns (term t at 4 t)
            uint32_t rd[16], re[16];
            tmem_ld16_u(c0, rd);
            if (EPI == EPI_F1) tmem_ld16_u(c0 + C::BN, re);
            tmem_ld_wait();
            tmem_regs_ready(rd);
            if (EPI == EPI_F1) tmem_regs_ready(re);
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
              for (int jj = 0; jj < 4; jj++) {
                d[t][jj] = rd[4 * t + jj];
                if (EPI == EPI_F1) e[t][jj] = re[4 * t + jj];
              }
          } else {
#pragma unroll
            for (int t = 0; t < NT; t++) tmem_ld16_u(c0 + t * npad + j0, d[t]);
            if (EPI == EPI_F1) {                 // the up projection: tile 1's accumulator
#pragma unroll
              for (int t = 0; t < NT; t++) tmem_ld16_u(c0 + C::BN + t * npad + j0, e[t]);
            }
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < NT; t++) tmem_regs_ready(d[t]);
            if (EPI == EPI_F1) {
#pragma unroll
              for (int t = 0; t < NT; t++) tmem_regs_ready(e[t]);
            }
          }
#pragma unroll
          for (int jj = 0; jj < (BsRows<N_MAX>::rp == 4 ? 4 : 16); jj++) {
            const int j = j0 + jj;
            if (j >= ch.n || !mvalid) continue;
            const int p = ch.p0 + j;
            float sc[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) sc[t] = C::FP4 ? 1.f : inv3[t * ep.P + p];
            // terms added from the smallest up (the last term first)
            float v = __uint_as_float(d[NT - 1][jj]) * sc[NT - 1];
#pragma unroll
            for (int t = NT - 2; t >= 0; t--) v = fmaf(__uint_as_float(d[t][jj]), sc[t], v);
            float up = 0.f;
            if (EPI == EPI_F1) {
              up = __uint_as_float(e[NT - 1][jj]) * sc[NT - 1];
#pragma unroll
              for (int t = NT - 2; t >= 0; t--) up = fmaf(__uint_as_float(e[t][jj]), sc[t], up);
            }
            if (whole) {                         // (inline: the pointers keep their __restrict__)
              const size_t o = (size_t)p * ep.M + m;
              if (EPI == EPI_F1) {
                const int tk = perm ? perm[p] : p;
                const size_t tmo = (size_t)tk * ep.M + m;
                const float gate = v + dlt_g[tmo];
                up += dlt_u[tmo];
                Go[o] = gate;
                Uo[o] = up;
                Ho[o] = __float2half_rn(situ_glu_fwd(gate, up));
              } else if (EPI == EPI_F2) {
                Yo[o] = v * tw[p];
              } else {
                Yo[o] = v;
              }
            } else if (EPI == EPI_F1) {
              __stcg(part + (size_t)j * 128 + row, v);
              __stcg(part + (size_t)(N_MAX + j) * 128 + row, up);
            } else {
              __stcg(part + (size_t)(pm * N_MAX + j) * 128 + row, v);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[ab]);
      if (++ab == C::NACC) { ab = 0; abph ^= 1; }
      if (!whole) {
        // count this warp's quarter of the piece in (a counter per unit and quarter: no barrier
        // across warps); the last of the unit's pieces adds them all, in CTA order, and writes
        // that quarter's outputs
        const long long us = (long long)u * n_stage;
        const int b0 = segs.owner(us), nseg = segs.owner(us + n_stage - 1) - b0 + 1;
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int* cnt = args.split_cnt + 4 * u + q;
          last = atomicAdd(cnt, 1) == nseg - 1;
          if (last) *cnt = 0;                    // ready for the next launch
          __threadfence();
        }
        if (__shfl_sync(0xffffffffu, last, 0)) {
          __threadfence();
#pragma unroll 1
          for (int pm = 0; pm < (PAIR ? 2 : 1); pm++) {
            const int m = ((u % args.mtiles) * (PAIR ? 2 : 1) + pm) * 128 + row;
            if (m >= ep.M) continue;
#pragma unroll 1
            for (int j0 = 0; j0 < ch.n; j0 += 16) {
              // 16 rows' sums at a time, each piece's loads issued together
              float v[16], up[16];
#pragma unroll
              for (int jj = 0; jj < 16; jj++) v[jj] = up[jj] = 0.f;
#pragma unroll 1
              for (int o = 0; o < nseg; o++) {
                const float* pp = args.split_part + (size_t)segs.slot(u, o, b0) * 2 * N_MAX * 128;
                const float* pv = pp + (size_t)((EPI == EPI_F1 ? 0 : pm) * N_MAX + j0) * 128 + row;
#pragma unroll
                for (int jj = 0; jj < 16; jj++) {
                  if (j0 + jj < ch.n) {
                    v[jj] += __ldcg(pv + jj * 128);
                    if (EPI == EPI_F1) up[jj] += __ldcg(pv + (N_MAX + jj) * 128);
                  }
                }
              }
#pragma unroll
              for (int jj = 0; jj < 16; jj++)
                if (j0 + jj < ch.n) finish(ch.p0 + j0 + jj, m, v[jj], up[jj]);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ll
