// Grouped MXFP4 x fp16 GEMM on tcgen05, one persistent CTA per SM.
//
// A unit of work is (chunk, m-tile): a chunk is up to N_MAX consecutive rows of the
// expert-sorted activation matrix that belong to one expert e; the m-tile is 128 output
// rows. For every unit the CTA computes D[128, N] = W_e'[m-tile, :] . Act[chunk rows, :]^T
// in fp32 in tensor memory, where W_e' is the expert's MXFP4 weight decoded exactly to
// fp16 (times a per-expert power of two that keeps fp16 in range) and the activations are
// fp16 rows carrying their own power-of-two row scale. Weights are the A operand (M = 128
// weight rows), tokens the B operand (N = 16..N_MAX), so the few tokens an expert gets do
// not waste a 128-wide MMA dimension.
//
// Data path per 128-element K stage: TMA brings the packed E2M1 bytes (and the scales) of
// the weight tile into shared memory; each dequant thread owns one weight row (one TMEM
// lane), decodes 32 consecutive K elements of it (one cvt.e2m1x2 and one fp16x2 multiply
// per byte) and writes them into tensor memory with a single tcgen05.st; the MMA reads A
// from tensor memory and the activations from shared memory (TMA, 128-byte swizzle). The
// decoded weights never touch shared memory, which keeps the per-element shared-memory
// traffic to the packed bytes.
//
// Scales. ROWSCALE (COLSCALE = false): the reference layout, one E8M0 byte per (row, 32
// K elements), used for W as stored (forward: gate/up rows = f, down rows = d).
// COLSCALE: the transposed copy of W that the backward reads (ll_moe_prepare builds it
// once per weight load): codes [cols][rows/2], and one fp16 multiplier per (32-row group,
// k) with the decode bias folded in, so the dequant thread multiplies each element pair by
// its own pair of scales.
//
// Warp roles (25 warps): 0 packed/scale TMA, 1 activation TMA, 2 and 3 MMA issuers (warp 2
// owns the TMEM allocation), 4..19 dequant (four warps per TMEM lane quarter, one per 32-K
// segment of a 128-K stage), 20..23 epilogue, 24 stage watcher (waits on the mbarriers for
// the issuers and releases them through named barriers). With four issuers (27 warps) the
// extra two are warps 24 and 25 and the watcher is warp 26.
// A product with one weight matrix (the down projection, its backward, the drop-ins) can
// run with NMAT = 2 over two adjacent 128-row tiles of the same stack (PAIR below).
// The issuers accumulate into separate accumulators (chains: gate / up and even / odd K
// stages, or K stages mod 4), so none waits on another and the sums stay deterministic; the
// epilogue adds the chains of one product in a fixed order.
// Packed weights move in 128-K TMA stages through a deep shared-memory ring; the
// tensor-memory A stages and the activation slots move in a shorter ring of 128-K stages,
// each with one "full" barrier (the 16 dequant warps + the activation TMA) and one "empty"
// commit per consuming chain. A dequant warp decodes stage s + 1 while its tensor-memory
// store of stage s completes.
#pragma once
#include "common.cuh"

namespace ll {

struct Chunk {
  int e;    // expert (index into the weight stacks)
  int p0;   // first row of the chunk in the expert-sorted activation matrix
  int n;    // rows, 1..N_MAX
  int pad;
};

enum EpiKind : int {
  EPI_F1 = 0,     // gate/up -> SiTU-GLU, saves gate/up fp32 and h fp16
  EPI_F2 = 1,     // down -> tw * y per pair (fp32)
  EPI_B1 = 2,     // g . W2 -> d_situ, SiTU-GLU backward, grad_w partials
  EPI_B2 = 3,     // dg . W1 + du . W3 -> dX per pair (fp32)
  EPI_STORE = 4,  // plain y[row, m] = D (drop-in mxfp4_gemm)
  EPI_ACCUM = 5,  // y[row, m] += D (drop-in mxfp4_gemm_t)
};

struct EpiParams {
  const int* perm_token;      // [P] token of each sorted row (nullptr: identity)
  const float* row_scale_inv; // [P] 2^-(power-of-two scale of each sorted activation row)
  const float* tw;            // [P] routing weight of each sorted row
  const int32_t* beta;        // [E][2]
  int beta_col;               // 0 = gate/up bias, 1 = down bias
  int P;                      // rows of the sorted activation matrix
  int M;                      // output width (rows of D)
  int r;                      // LoRA rank
  float lora_scaling;
  // F1
  const float* delta_g;       // [T][M] s*(x A_g^T) B_g^T
  const float* delta_u;
  float* G;                   // [P][M] gate pre-activation
  float* U;                   // [P][M] up pre-activation
  __half* H;                  // [P][M] SiTU-GLU output (fp16, B operand of the down GEMM)
  // F2 / B2 / STORE / ACCUM
  float* Y;                   // [P][M] (or [rows][M] for STORE / ACCUM)
  // B1
  const float* lora_d;        // [T][M] (g B_d) A_d: the down adapter's term of dL/dh per token
  const float* Gs;            // saved G
  const float* Us;            // saved U
  float* DG;                  // [P][M]
  float* DU;                  // [P][M]
  float* gw_part;             // [mtiles * 4][P] (one partial per epilogue warp)
};

struct GemmArgs {
  const Chunk* chunks;
  const int* n_chunks;
  int mtiles;        // units per chunk: ceil(M / 128), ceil(M / 256) with paired tiles
  int K;             // reduction length
  int e_rows;        // stored weight rows per expert (= M)
  DevStatus* status;
  EpiParams epi;
};


template <int NMAT, int NB, bool COLSCALE, int N_MAX>
struct GemmCfg {
  static constexpr int kIssuerWarpX = 24;                 // issuers 2 and 3 (when present): warps 24, 25
  // Independent accumulation chains, one MMA issuer warp each: a warp issues one tcgen05.mma
  // per ~50 cycles at small N however many accumulators it rotates, so small-N tiles need
  // several issuing warps.
#ifndef LL_CHAINS_SMALL_N
#define LL_CHAINS_SMALL_N 2
#endif
  // (N = 128 MMAs are long enough for one chain per weight matrix, which leaves room for two
  // accumulator buffers when there is one matrix, so its epilogue overlaps the next unit)
  // At 16-row tiles four chains fit in tensor memory next to a 3-deep A ring, and the issue
  // rate of one warp (not the tensor pipe) bounds a 16-wide MMA.
  static constexpr int CH = N_MAX <= 16 ? 4 : N_MAX <= 32 ? LL_CHAINS_SMALL_N : (N_MAX >= 128 ? NMAT : 2);
  static constexpr int PM = CH / NMAT;                    // chains per weight matrix
  static constexpr int kThreads = (CH > 2 ? 27 : 25) * 32;
  // with four issuers each sits on its own SM sub-partition (warp % 4), away from the others'
  // instruction issue; the watcher then moves to warp 26
  static constexpr int kWatchWarp = CH > 2 ? 26 : 24;
  static constexpr int kIssuerWarp0 = 2;
  static constexpr int kDqWarp0 = 4, kDqWarps = 16;
  static constexpr int kEpWarp0 = 20, kEpWarps = 4;
  static constexpr int BK = 128;                          // K per packed (TMA) stage
  static constexpr int KS = LL_KS;                        // K per A/B ring stage (64 or 128)
  static constexpr int SUBS = BK / KS;                    // ring stages per packed stage
  static_assert(KS == 64 || KS == 128, "ring stage");
  static constexpr int PK_BYTES = 128 * 64;               // 128 rows x 64 packed bytes
  static constexpr int SC_BYTES = COLSCALE ? 4 * 128 * 2  // 4 row groups x 128 k x fp16
                                           : 128 * 16;    // 128 rows x 16 scale bytes
  static constexpr int P_STAGE = NMAT * (PK_BYTES + SC_BYTES);
  static constexpr int B_HALF = N_MAX * 128;              // one 64-K half of one operand
  static constexpr int B_SLOT = NB * (KS / 64) * B_HALF;
  // tensor memory: two accumulators per buffer (one per issuer), then the A stages
  static constexpr int ACC_COLS = CH * N_MAX;
  static constexpr int A_STAGE_COLS = NMAT * KS / 2;      // fp16 pairs: KS/2 columns per matrix
  static constexpr int NACC = (2 * ACC_COLS + 2 * A_STAGE_COLS <= 512) ? 2 : 1;
  static constexpr int A_BASE = NACC * ACC_COLS;
  static constexpr int S_AB0 = (512 - A_BASE) / A_STAGE_COLS;
  static constexpr int S_AB = S_AB0 > 7 ? 7 : S_AB0;     // 2 named barriers a slot, ids 1..14
  static_assert(S_AB >= 2, "tensor memory budget");
  // Dequant stage groups: group j of dequant warps fills ring stages g with g % GROUPS == j,
  // SEGW 32-K segments per warp, so GROUPS stages fill at once and a warp pays its barrier
  // round trip once per SEGW segments.
  static constexpr int GROUPS = KS == 64 ? 2 : (S_AB >= 5 ? 4 : (S_AB >= 3 ? 2 : 1));
  static constexpr int SEGW = (KS / 32) * GROUPS / 4;     // segments a warp decodes per stage
  static_assert(SEGW >= 1 && (kDqWarps / 4) % GROUPS == 0 && (kDqWarps / 4 / GROUPS) * SEGW == KS / 32,
                "segment cover");
  static constexpr int kDqPerStage = kDqWarps / GROUPS;   // warps that fill one ring stage
  // a dequant group may wait on a stage up to GROUPS - 1 stages ahead of the others; a ring
  // shorter than that would let a parity wait match a phase one ring cycle early
  static constexpr int TMEM_COLS0 = A_BASE + S_AB * A_STAGE_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS0 <= 32 ? 32 : TMEM_COLS0 <= 64 ? 64 : TMEM_COLS0 <= 128 ? 128
                                   : TMEM_COLS0 <= 256 ? 256 : 512;
  // shared memory: the activation (B) ring and the packed-weight ring, each with its own
  // barriers and as deep as half the budget allows: the activation tiles come through L2
  // with a latency of a few microseconds under the weight stream, so they are fetched many
  // stages ahead of the tensor-memory A ring
  static constexpr int AVAIL = 227 * 1024 - 2048;
  static constexpr int S_B0 = (AVAIL / 2) / B_SLOT;
  static constexpr int S_B = S_B0 > 16 ? 16 : (S_B0 < 2 ? 2 : S_B0);
  static constexpr int S_P0 = (AVAIL - S_B * B_SLOT) / P_STAGE;
  static constexpr int S_P = S_P0 > 10 ? 10 : S_P0;
  static_assert(S_P >= 2, "shared memory budget");
  static_assert(S_P >= GROUPS && S_AB >= GROUPS, "ring shorter than the dequant stage groups");
  static constexpr int OFF_B = 0;
  static constexpr int OFF_P = OFF_B + S_B * B_SLOT;
  static constexpr int OFF_BAR = OFF_P + S_P * P_STAGE;
  static constexpr int N_BARS = 2 * S_P + 2 * S_AB + 2 * S_B + 4 + 1;
  static constexpr int SMEM = OFF_BAR + N_BARS * 8 + 64 + 1024;  // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(N_MAX % 16 == 0 && N_MAX <= 128, "N_MAX");
  // a ring slot is reused only after every chain that could share its named barrier moved on
  static_assert(S_AB >= PM, "ring shorter than the chains of one matrix");
  // named barrier releasing the chain of weight matrix `mat` that takes the stage in ring
  // slot s (ids 1..14; id 0 is __syncthreads)
  static __device__ __forceinline__ int ready_bar(int s, int mat) { return 1 + 2 * s + mat; }
};

template <int NMAT, int N_MAX>
struct TmaSet {
  CUtensorMap pk[NMAT];
  CUtensorMap sc[NMAT];
  CUtensorMap act[N_MAX / 16];   // act[c - 1]: one ring stage of a 16 c-row chunk (all operands)
};

template <int EPI, int NMAT, int NB, bool COLSCALE, int N_MAX>
__global__ void __launch_bounds__(GemmCfg<NMAT, NB, COLSCALE, N_MAX>::kThreads, 1)
grouped_mxfp4_gemm(const __grid_constant__ TmaSet<NMAT, N_MAX> tm, const GemmArgs args) {
  using C = GemmCfg<NMAT, NB, COLSCALE, N_MAX>;
  // A single-product epilogue with two weight matrices takes two adjacent 128-row tiles of
  // one stack as its two matrices (both maps name the same stack): one activation stage then
  // feeds twice the weight bytes, and the per-stage barrier work is paid once per 256 rows.
  constexpr bool PAIR = NMAT == 2 && EPI != EPI_F1 && EPI != EPI_B2;
  constexpr int TILE_ROWS = PAIR ? 256 : 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* pfull = bars;
  uint64_t* pempty = pfull + C::S_P;
  uint64_t* full = pempty + C::S_P;
  uint64_t* empty = full + C::S_AB;
  uint64_t* bfull = empty + C::S_AB;
  uint64_t* bempty = bfull + C::S_B;
  uint64_t* accfull = bempty + C::S_B;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (args.K <= 0) {                        // uniform over the CTA: nothing allocated yet
    pdl_wait();
    return;
  }

  const int K = args.K;
  const int n_stage = (K + C::BK - 1) / C::BK;   // packed (TMA) stages per unit
  const int n_sub = n_stage * C::SUBS;          // A/B ring stages per unit (a K tail past the
                                                 // last 64 columns decodes zeros)
  // with one weight matrix the two issuers take alternate stages; a 1-stage K leaves one idle
  const int chains_used = n_sub < C::PM ? n_sub : C::PM;   // chains of a matrix that got a stage

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::S_P; i++) { mbar_init(&pfull[i], 1); mbar_init(&pempty[i], C::kDqPerStage * C::SUBS); }
    for (int i = 0; i < C::S_AB; i++) { mbar_init(&full[i], C::kDqPerStage); mbar_init(&empty[i], NMAT); }
    for (int i = 0; i < C::S_B; i++) { mbar_init(&bfull[i], 1); mbar_init(&bempty[i], NMAT); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], C::CH); mbar_init(&accempty[i], C::kEpWarps); }
    mbar_init(drain, C::CH);
    *abort_flag = 0;
    fence_barrier_init();
    fence_async_smem();
  }
  if (warp == C::kIssuerWarp0) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  DevStatus* st = args.status;
  // the prologue above reads nothing another kernel writes; the chunk list below does
  pdl_launch_next();                        // (after the allocation)
  pdl_wait();
  const int n_units = (*args.n_chunks) * args.mtiles;
  if ((int)blockIdx.x >= n_units) {         // uniform per block: no unit for this one
    if (warp == C::kIssuerWarp0) tmem_dealloc(tmem, C::TMEM_COLS);
    return;
  }

  if (warp == 0) {
    // ------------------------------------------------ packed weights + scales producer
    if (lane == 0) {
      for (int i = 0; i < NMAT; i++) { tma_prefetch_desc(&tm.pk[i]); tma_prefetch_desc(&tm.sc[i]); }
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int mt = u % args.mtiles;
        const int row = ch.e * args.e_rows + mt * TILE_ROWS;
        const int grp = (ch.e * args.e_rows) / 32 + mt * (TILE_ROWS / 32);
        for (int ks = 0; ks < n_stage && ok; ks++) {
          if (!(ok = mbar_wait_sleep(&pempty[s], ph ^ 1, abort_flag, st, 1, 256))) break;
          uint8_t* stage = smem + C::OFF_P + s * C::P_STAGE;
          mbar_arrive_expect_tx(&pfull[s], C::P_STAGE);
          // stage layout: the NMAT packed tiles, then their NMAT scale tiles; paired tiles are
          // adjacent rows of one stack, so one box of 256 rows (8 column groups) brings both
          for (int i = 0; i < (PAIR ? 1 : NMAT); i++) {
            uint8_t* pk = stage + i * C::PK_BYTES;
            uint8_t* sc = stage + NMAT * C::PK_BYTES + i * C::SC_BYTES;
            tma_load_2d(pk, &tm.pk[i], &pfull[s], ks * (C::BK / 2), row);
            if (COLSCALE)
              tma_load_2d(sc, &tm.sc[i], &pfull[s], ks * C::BK, grp);
            else
              tma_load_2d(sc, &tm.sc[i], &pfull[s], ((ks * C::BK) / 32) & ~15, row);
          }
          issued++;
          if (++s == C::S_P) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < C::S_P && i < issued; i++) {   // drain: bytes of the last stages landed
        if (--s < 0) { s = C::S_P - 1; ph ^= 1; }
        mbar_wait_sleep(&pfull[s], ph, abort_flag, st, 11, 256);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- activation (B) producer
    if (lane == 0) {
      for (int i = 0; i < N_MAX / 16; i++) tma_prefetch_desc(&tm.act[i]);
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int npad = (ch.n + 15) & ~15;
        for (int sb = 0; sb < n_sub && ok; sb++) {
          if (!(ok = mbar_wait_sleep(&bempty[s], ph ^ 1, abort_flag, st, 2, 256))) break;
          uint8_t* slot = smem + C::OFF_B + s * C::B_SLOT;
          // one instruction: [operand][64-K half][npad rows][128 bytes]
          mbar_arrive_expect_tx(&bfull[s], NB * (C::KS / 64) * npad * 128);
          if (NB == 2)
            tma_load_4d(slot, &tm.act[npad / 16 - 1], &bfull[s], 0, ch.p0, sb * (C::KS / 64), 0);
          else
            tma_load_3d(slot, &tm.act[npad / 16 - 1], &bfull[s], 0, ch.p0, sb * (C::KS / 64));
          issued++;
          if (++s == C::S_B) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < C::S_B && i < issued; i++) {   // drain: bytes of the last stages landed
        if (--s < 0) { s = C::S_B - 1; ph ^= 1; }
        mbar_wait_sleep(&bfull[s], ph, abort_flag, st, 12, 256);
      }
    }
  } else if (warp < C::kDqWarp0 || (warp >= C::kIssuerWarpX && warp != C::kWatchWarp)) {
    // ---------------------------------------------------------------- MMA issuers
    // Chain c = mat * PM + k accumulates weight matrix `mat` over the stages sb with
    // sb % PM == k. The whole warp takes part in the named barriers the watcher releases
    // stages on; lane 0 issues. An issuer never touches an mbarrier in its loop: an mbarrier
    // wait in the thread that issues tcgen05.mma stalls the MMA stream by hundreds of cycles.
    const int c = warp < C::kDqWarp0 ? warp - C::kIssuerWarp0 : 2 + warp - C::kIssuerWarpX;
    if (c < C::CH) {
      const int mat = c / C::PM, kc = c % C::PM;
      int s = 0, bs = 0, ab = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int npad = (ch.n + 15) & ~15;
        const uint32_t idesc = idesc_f16_m128(npad, false, false);
        const uint32_t d = tmem + (ab * C::CH + c) * N_MAX;
        bool first = true;
        for (int sb = 0; sb < n_sub; sb++) {
          if (sb % C::PM == kc) {
            if (*abort_flag) { ok = false; break; }   // the watcher may run ahead after an abort
            named_bar_sync(C::ready_bar(s, mat), 64);
            if (lane == 0) {
              tc_fence_after();
              const uint32_t a_tmem = tmem + C::A_BASE + s * C::A_STAGE_COLS + mat * (C::KS / 2);
              const uint32_t half_bytes = (uint32_t)npad * 128;   // one 64-K half of the chunk's rows
              const uint32_t b_addr =
                  smem_u32(smem + C::OFF_B + bs * C::B_SLOT) + (NB == 2 ? mat : 0) * (C::KS / 64) * half_bytes;
              // the descriptor's address field is addr >> 4 in its low bits (shared memory is
              // below 256 KB, so the sums stay in the field): one base descriptor per stage
              const uint64_t bdesc0 = umma_desc(b_addr, 16, 1024, kSwizzle128B);
              const uint64_t half16 = half_bytes >> 4;
#pragma unroll
              for (int kk = 0; kk < C::KS / 16; kk++) {
                const uint64_t bdesc = bdesc0 + (kk >> 2) * half16 + (kk & 3) * 2;
                mma_f16_ts(d, a_tmem + kk * 8, bdesc, idesc, first ? 0u : 1u);
                first = false;
              }
              mma_commit(&empty[s]);    // A slot free once these MMAs completed
              mma_commit(&bempty[bs]);  // and the activation slot
            }
            __syncwarp();
          }
          if (++s == C::S_AB) s = 0;
          if (++bs == C::S_B) bs = 0;
        }
        if (lane == 0) mma_commit(&accfull[ab]);
        __syncwarp();
        if (++ab == C::NACC) ab = 0;
      }
      if (lane == 0) {
        mma_commit(drain);              // completes once every MMA issued above has finished
        volatile int keep_waiting = 0;  // wait for them even after an abort
        mbar_wait_sleep(drain, 0, &keep_waiting, st, 13, 256);
      }
    }
  } else if (warp == C::kWatchWarp) {
    // ------------------------------------------------------------------ stage watcher
    // Waits (bounded) for each ring stage to fill (A: dequant warps; B: activation TMA) and for
    // each unit's accumulator buffer to drain (epilogue), then releases the issuer(s) of that
    // stage through named barrier (stage slot, issuer). It never leaves the loop early and
    // never blocks without a bound, so every barrier an issuer syncs on gets its arrival,
    // also after an abort (when the waits return at once).
    int s = 0, bs = 0, ab = 0;
    uint32_t ph = 0, bph = 0, abph = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
      if (lane == 0) mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 3);
      __syncwarp();
      for (int sb = 0; sb < n_sub; sb++) {
        if (lane == 0) {
          mbar_wait(&bfull[bs], bph, abort_flag, st, 5);
          mbar_wait(&full[s], ph, abort_flag, st, 4);
        }
        __syncwarp();
        for (int mat = 0; mat < NMAT; mat++) named_bar_arrive(C::ready_bar(s, mat), 64);
        if (++s == C::S_AB) { s = 0; ph ^= 1; }
        if (++bs == C::S_B) { bs = 0; bph ^= 1; }
      }
      if (++ab == C::NACC) { ab = 0; abph ^= 1; }
    }
  } else if (warp < C::kEpWarp0) {
    // ---------------------------------------------------------------- dequant warps
    // warp -> (TMEM lane quarter q, stage group grp, segments seg0 .. seg0 + SEGW - 1 of the
    // 128-K stages of that group); thread -> weight row. Each 32-K segment is decoded to
    // registers and stored to tensor memory at once; the stage is marked full after the
    // last store of the warp completes.
    const int dw = warp - C::kDqWarp0;           // 0..15
    const int q = warp & 3;
    const int sub = dw >> 2;                     // 0..3
    const int grp = sub % C::GROUPS;
    const int seg0 = (sub / C::GROUPS) * C::SEGW;
    const int m = q * 32 + lane;                 // weight row within the 128-row tile
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int32_t* beta = args.epi.beta;
    const int bcol = args.epi.beta_col;
    int g = grp;                                 // ring stage index over this CTA's stages
    int u = blockIdx.x, kss = grp;               // kss: ring stage within the unit
    while (kss >= n_sub) { kss -= n_sub; u += gridDim.x; }
    int bias = (u < n_units && !COLSCALE && beta) ? beta[args.chunks[u / args.mtiles].e * 2 + bcol] : 0;
    while (u < n_units) {
      const int gp = g / C::SUBS;                // packed stage (global over the CTA's stages)
      const int ks = kss / C::SUBS;              // packed stage within the unit
      const int segb = (g % C::SUBS) * (C::KS / 32);   // first 32-K segment of this ring stage
      const int ps = gp % C::S_P, as = g % C::S_AB;
      const uint32_t pph = (uint32_t)(gp / C::S_P) & 1u, aph = (uint32_t)(g / C::S_AB) & 1u;
      if (!mbar_wait(&pfull[ps], pph, abort_flag, st, 6)) break;
      const uint8_t* stage = smem + C::OFF_P + ps * C::P_STAGE;
      bool waited = false, ok = true;
#pragma unroll
      for (int j = 0; j < C::SEGW; j++) {
        const int seg = segb + seg0 + j;         // 32-K segment within the packed stage
#pragma unroll
        for (int i = 0; i < NMAT; i++) {
          const uint8_t* pk = stage + i * C::PK_BYTES;
          const uint8_t* sc = stage + NMAT * C::PK_BYTES + i * C::SC_BYTES;
          const uint4 raw = ld_shared_v4(smem_u32(pk + m * 64 + ((seg ^ ((m >> 1) & 3)) << 4)));
          uint32_t o[16];
          if (COLSCALE) {
            // fp16 multipliers of k = 32 seg .. 32 seg + 31 for this warp's 32-row group q
            const uint32_t sa = smem_u32(sc + (q * 128 + seg * 32) * 2);
            const uint4 s0 = ld_shared_v4(sa), s1 = ld_shared_v4(sa + 16);
            const uint4 s2 = ld_shared_v4(sa + 32), s3 = ld_shared_v4(sa + 48);
            const uint32_t sv[16] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w,
                                     s2.x, s2.y, s2.z, s2.w, s3.x, s3.y, s3.z, s3.w};
            decode8v(raw.x, &sv[0], &o[0]);
            decode8v(raw.y, &sv[4], &o[4]);
            decode8v(raw.z, &sv[8], &o[8]);
            decode8v(raw.w, &sv[12], &o[12]);
          } else {
            const uint32_t sbyte = sc[m * 16 + (((ks * C::BK) / 32) & 15) + seg];
            const uint32_t s2 = e8m0_to_half2_bits(sbyte, bias);
            decode8(raw.x, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[0]));
            decode8(raw.y, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[4]));
            decode8(raw.z, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[8]));
            decode8(raw.w, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[12]));
          }
          if (!waited) {                         // the slot's previous MMAs are done
            if (!(ok = mbar_wait(&empty[as], aph ^ 1, abort_flag, st, 7))) break;
            tc_fence_after();
            waited = true;
          }
          tmem_st16(tmem + lane_base + C::A_BASE + as * C::A_STAGE_COLS + i * (C::KS / 2) + (seg0 + j) * 16, o);
        }
        if (!ok) break;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[ps]);   // packed bytes consumed
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[as]);
      g += C::GROUPS;
      kss += C::GROUPS;
      while (kss >= n_sub) {                     // into the next unit(s)
        kss -= n_sub;
        u += gridDim.x;
        if (u < n_units && !COLSCALE && beta) bias = beta[args.chunks[u / args.mtiles].e * 2 + bcol];
      }
    }
  } else {
    // ------------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;          // accumulator row = M index within the tile
    const EpiParams& ep = args.epi;
    const int* __restrict__ perm = ep.perm_token;
    const float* __restrict__ rsi = ep.row_scale_inv;
    const float* __restrict__ tw = ep.tw;
    const float* __restrict__ dlt_g = ep.delta_g;
    const float* __restrict__ dlt_u = ep.delta_u;
    const float* __restrict__ lora_d = ep.lora_d;
    const float* __restrict__ Gs = ep.Gs;
    const float* __restrict__ Us = ep.Us;
    float* __restrict__ Go = ep.G;
    float* __restrict__ Uo = ep.U;
    __half* __restrict__ Ho = ep.H;
    float* __restrict__ Yo = ep.Y;
    float* __restrict__ DGo = ep.DG;
    float* __restrict__ DUo = ep.DU;
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Chunk ch = args.chunks[u / args.mtiles];
      const int npad = (ch.n + 15) & ~15;
      const int bias = ep.beta ? ep.beta[ch.e * 2 + ep.beta_col] : 0;
      const float wunscale = exp2f((float)(-bias));
      if (!(ok = mbar_wait_sleep(&accfull[ab], abph, abort_flag, st, 8, 512))) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * C::CH * N_MAX;
#pragma unroll 1
      for (int pm = 0; pm < (PAIR ? 2 : 1); pm++) {
        const int mt = (u % args.mtiles) * (PAIR ? 2 : 1) + pm;   // 128-row tile of the output
        const int m = mt * 128 + row;
        const bool mvalid = m < ep.M;
        const int c0 = PAIR ? pm * C::PM : 0;                     // first chain of this product
        const int c1 = PAIR ? c0 + C::PM : C::CH;
        for (int j0 = 0; j0 < npad; j0 += 16) {
          // v0 = sum of matrix 0's chains (all chains unless F1 or paired tiles), v1 = matrix
          // 1's (F1: up)
          float v0[16], v1[16], t[16];
          tmem_ld16(tbase + c0 * N_MAX + j0, v0);
          tmem_ld_wait();
          if (EPI == EPI_F1) {
            tmem_ld16(tbase + C::PM * N_MAX + j0, v1);
            tmem_ld_wait();
          }
          for (int cc = c0 + 1; cc < c1; cc++) {
            const int kc = cc % C::PM;
            if (kc >= chains_used) continue;        // a chain that got no stage holds no sum
            if (EPI == EPI_F1 && kc == 0) continue; // first chain of matrix 1, loaded above
            tmem_ld16(tbase + cc * N_MAX + j0, t);
            tmem_ld_wait();
            if (EPI == EPI_F1 && cc >= C::PM) {
#pragma unroll
              for (int jj = 0; jj < 16; jj++) v1[jj] += t[jj];
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; jj++) v0[jj] += t[jj];
            }
          }
          float gwp[16];
          // Batches of EB tokens: the per-token indices and scalars of a batch, then its
          // per-element loads, are all requested before anything is computed or stored (the
          // pointers are restrict-qualified, so loads are not held behind the stores).
          constexpr int EB = (EPI == EPI_F1 || (EPI == EPI_B1 && PAIR)) ? 2 : (EPI == EPI_B1 ? 4 : 8);
#pragma unroll
          for (int h = 0; h < 16; h += EB) {
            int pp[EB];
            size_t tm[EB];
            float sc[EB], a0[EB], a1[EB], a2[EB];
#pragma unroll
            for (int i = 0; i < EB; i++) {
              const int j = j0 + h + i;
              const bool ok = j < ch.n && mvalid;
              const int p = ch.p0 + j;
              pp[i] = ok ? p : -1;
              const int t = ok ? (perm ? perm[p] : p) : 0;
              tm[i] = (size_t)t * ep.M + m;
              if (EPI == EPI_F2) sc[i] = ok ? tw[p] : 0.f;
              else if (EPI == EPI_B1) { sc[i] = ok ? rsi[p] : 0.f; a2[i] = ok ? tw[p] : 0.f; }
              else sc[i] = ok ? rsi[p] : 0.f;
            }
#pragma unroll
            for (int i = 0; i < EB; i++) {
              const size_t o = (size_t)(pp[i] < 0 ? 0 : pp[i]) * ep.M + m;
              if (pp[i] < 0) { a0[i] = a1[i] = 0.f; continue; }
              if (EPI == EPI_F1) { a0[i] = dlt_g[tm[i]]; a1[i] = dlt_u[tm[i]]; }
              else if (EPI == EPI_B1) { a0[i] = Gs[o]; a1[i] = Us[o]; sc[i] = sc[i] * wunscale; }
              else if (EPI == EPI_ACCUM) a0[i] = Yo[o];
            }
            float ld[EB];
            if (EPI == EPI_B1) {
#pragma unroll
              for (int i = 0; i < EB; i++) ld[i] = pp[i] < 0 ? 0.f : lora_d[tm[i]];
            }
#pragma unroll
            for (int i = 0; i < EB; i++) {
              const int jj = h + i;
              gwp[jj] = 0.f;
              if (pp[i] < 0) continue;
              const size_t o = (size_t)pp[i] * ep.M + m;
              if (EPI == EPI_F1) {
                const float cs = sc[i] * wunscale;
                const float gate = v0[jj] * cs + a0[i];
                const float up = v1[jj] * cs + a1[i];
                Go[o] = gate;
                Uo[o] = up;
                Ho[o] = __float2half_rn(situ_glu_fwd(gate, up));
              } else if (EPI == EPI_F2) {
                Yo[o] = v0[jj] * wunscale * sc[i];
              } else if (EPI == EPI_B1) {
                const float v = v0[jj] * sc[i] + ep.lora_scaling * ld[i];
                const float g = a0[i], uu = a1[i];
                gwp[jj] = situ_glu_fwd(g, uu) * v;
                float dg, du;
                situ_glu_bwd(a2[i] * v, g, uu, dg, du);
                DGo[o] = dg;
                DUo[o] = du;
              } else if (EPI == EPI_B2 || EPI == EPI_STORE) {
                Yo[o] = v0[jj] * sc[i] * wunscale;
              } else if (EPI == EPI_ACCUM) {
                Yo[o] = a0[i] + v0[jj] * sc[i] * wunscale;
              }
            }
          }
          if (EPI == EPI_B1) {
            // grad_w partial over this warp's 32 rows (fixed shuffle order); the four warps of
            // the tile write separate partials, summed later in a fixed order.
            float mine = 0.f;
#pragma unroll
            for (int jj = 0; jj < 16; jj++) {
              float s = gwp[jj];
#pragma unroll
              for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
              if (jj == lane) mine = s;
            }
            if (lane < 16 && j0 + lane < ch.n && mt * 128 < ep.M)
              ep.gw_part[((size_t)mt * 4 + q) * ep.P + ch.p0 + j0 + lane] = mine;
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
  if (warp == C::kIssuerWarp0) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ll
