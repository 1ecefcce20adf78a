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
// Warp roles (15 warps): 0 packed/scale TMA, 1 activation TMA, 2 MMA issue + TMEM owner,
// 3..10 dequant (two warps per TMEM lane quarter, one per 32-element half of a 64-K
// sub-chunk), 11..14 epilogue.
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
  const float* gB;            // [T][r] g . B_d
  const float* A_d;           // [r][M]
  const float* Gs;            // saved G
  const float* Us;            // saved U
  float* DG;                  // [P][M]
  float* DU;                  // [P][M]
  float* gw_part;             // [mtiles * 4][P] (one partial per epilogue warp)
};

struct GemmArgs {
  const Chunk* chunks;
  const int* n_chunks;
  int mtiles;        // ceil(M / 128)
  int K;             // reduction length
  int e_rows;        // stored weight rows per expert (= M)
  DevStatus* status;
  EpiParams epi;
};

template <int NMAT, int NB, int ND, bool COLSCALE, int N_MAX>
struct GemmCfg {
  static constexpr int kThreads = 15 * 32;
  static constexpr int kDqWarp0 = 3, kDqWarps = 8;
  static constexpr int kEpWarp0 = 11, kEpWarps = 4;
  static constexpr int BK = 128;                          // K per packed stage
  static constexpr int SUBS = 2;                          // 64-K A sub-chunks per stage
  static constexpr int PK_BYTES = 128 * 64;               // 128 rows x 64 packed bytes
  static constexpr int SC_BYTES = COLSCALE ? 4 * 128 * 2  // 4 row groups x 128 k x fp16
                                           : 128 * 16;    // 128 rows x 16 scale bytes
  static constexpr int P_STAGE = NMAT * (PK_BYTES + SC_BYTES);
  static constexpr int B_SLOT = NB * N_MAX * 128;
  // tensor memory: accumulators first, then the A stages (32 columns per matrix and stage)
  static constexpr int S_A = NMAT == 2 ? 3 : 4;
  static constexpr int A_COLS = S_A * NMAT * 32;
  static constexpr int NACC = (2 * ND * N_MAX + A_COLS <= 512) ? 2 : 1;
  static constexpr int A_BASE = NACC * ND * N_MAX;
  static constexpr int TMEM_COLS0 = A_BASE + A_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS0 <= 32 ? 32 : TMEM_COLS0 <= 64 ? 64 : TMEM_COLS0 <= 128 ? 128
                                   : TMEM_COLS0 <= 256 ? 256 : 512;
  static_assert(TMEM_COLS0 <= 512, "tensor memory budget");
  // shared memory: B ring and packed ring
  static constexpr int AVAIL = 227 * 1024 - 2048;
  static constexpr int S_B0 = (AVAIL * 2 / 5) / B_SLOT;
  static constexpr int S_B = S_B0 < 3 ? 3 : (S_B0 > 8 ? 8 : S_B0);
  static constexpr int S_P0 = (AVAIL - S_B * B_SLOT) / P_STAGE;
  static constexpr int S_P = S_P0 < 2 ? 2 : (S_P0 > 12 ? 12 : S_P0);
  static constexpr int OFF_B = 0;
  static constexpr int OFF_P = OFF_B + S_B * B_SLOT;
  static constexpr int OFF_BAR = OFF_P + S_P * P_STAGE;
  static constexpr int N_BARS = 2 * S_P + 2 * S_A + 2 * S_B + 4 + 1;
  static constexpr int SMEM = OFF_BAR + N_BARS * 8 + 64 + 1024;  // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(N_MAX % 16 == 0 && N_MAX <= 256, "N_MAX");
};

template <int NMAT, int NB>
struct TmaSet {
  CUtensorMap pk[NMAT];
  CUtensorMap sc[NMAT];
  CUtensorMap act[NB];
};

template <int EPI, int NMAT, int NB, int ND, bool COLSCALE, int N_MAX>
__global__ void __launch_bounds__(15 * 32, 1)
grouped_mxfp4_gemm(const __grid_constant__ TmaSet<NMAT, NB> tm, const GemmArgs args) {
  using C = GemmCfg<NMAT, NB, ND, COLSCALE, N_MAX>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* pfull = bars;
  uint64_t* pempty = pfull + C::S_P;
  uint64_t* afull = pempty + C::S_P;
  uint64_t* aempty = afull + C::S_A;
  uint64_t* bfull = aempty + C::S_A;
  uint64_t* bempty = bfull + C::S_B;
  uint64_t* accfull = bempty + C::S_B;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_units = (*args.n_chunks) * args.mtiles;
  if ((int)blockIdx.x >= n_units) return;   // uniform over the CTA: nothing allocated yet

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::S_P; i++) { mbar_init(&pfull[i], 1); mbar_init(&pempty[i], C::kDqWarps); }
    for (int i = 0; i < C::S_A; i++) { mbar_init(&afull[i], C::kDqWarps); mbar_init(&aempty[i], 1); }
    for (int i = 0; i < C::S_B; i++) { mbar_init(&bfull[i], 1); mbar_init(&bempty[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], C::kEpWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_async_smem();
  }
  if (warp == 2) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int K = args.K;
  const int n_sub = (K + 63) / 64;
  const int n_stage = (K + C::BK - 1) / C::BK;
  DevStatus* st = args.status;

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
        const int row = ch.e * args.e_rows + mt * 128;
        const int grp = (ch.e * args.e_rows) / 32 + mt * 4;
        for (int ks = 0; ks < n_stage && ok; ks++) {
          if (!(ok = mbar_wait(&pempty[s], ph ^ 1, abort_flag, st, 1))) break;
          uint8_t* stage = smem + C::OFF_P + s * C::P_STAGE;
          mbar_arrive_expect_tx(&pfull[s], C::P_STAGE);
          for (int i = 0; i < NMAT; i++) {
            uint8_t* pk = stage + i * (C::PK_BYTES + C::SC_BYTES);
            tma_load_2d(pk, &tm.pk[i], &pfull[s], ks * (C::BK / 2), row);
            if (COLSCALE)
              tma_load_2d(pk + C::PK_BYTES, &tm.sc[i], &pfull[s], ks * C::BK, grp);
            else
              tma_load_2d(pk + C::PK_BYTES, &tm.sc[i], &pfull[s], ((ks * C::BK) / 32) & ~15, row);
          }
          issued++;
          if (++s == C::S_P) { s = 0; ph ^= 1; }
        }
      }
      // drain: wait for the bytes of the last issued stages to land before exiting
      for (int i = 0; i < C::S_P && i < issued; i++) {
        if (--s < 0) { s = C::S_P - 1; ph ^= 1; }
        mbar_wait(&pfull[s], ph, abort_flag, st, 11);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- activation (B) producer
    if (lane == 0) {
      for (int i = 0; i < NB; i++) tma_prefetch_desc(&tm.act[i]);
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int npad = (ch.n + 15) & ~15;
        for (int sb = 0; sb < n_sub && ok; sb++) {
          if (!(ok = mbar_wait(&bempty[s], ph ^ 1, abort_flag, st, 2))) break;
          uint8_t* slot = smem + C::OFF_B + s * C::B_SLOT;
          mbar_arrive_expect_tx(&bfull[s], NB * npad * 128);
          for (int b = 0; b < NB; b++)
            for (int rb = 0; rb < npad; rb += 16)
              tma_load_2d(slot + b * N_MAX * 128 + rb * 128, &tm.act[b], &bfull[s], sb * 64, ch.p0 + rb);
          issued++;
          if (++s == C::S_B) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < C::S_B && i < issued; i++) {
        if (--s < 0) { s = C::S_B - 1; ph ^= 1; }
        mbar_wait(&bfull[s], ph, abort_flag, st, 12);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int as = 0, bs = 0, ab = 0;
      uint32_t aph = 0, bph = 0, abph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Chunk ch = args.chunks[u / args.mtiles];
        const int npad = (ch.n + 15) & ~15;
        const uint32_t idesc = idesc_f16_m128(npad, false, false);
        if (!(ok = mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 3))) break;
        tc_fence_after();
        const uint32_t d0 = tmem + ab * ND * N_MAX;
        for (int sb = 0; sb < n_sub && ok; sb++) {
          if (!(ok = mbar_wait(&afull[as], aph, abort_flag, st, 4))) break;
          if (!(ok = mbar_wait(&bfull[bs], bph, abort_flag, st, 5))) break;
          tc_fence_after();
          const uint32_t b_base = smem_u32(smem + C::OFF_B + bs * C::B_SLOT);
#pragma unroll
          for (int i = 0; i < NMAT; i++) {
            const uint32_t d = d0 + (ND == 2 ? i : 0) * N_MAX;
            const uint32_t a_tmem = tmem + C::A_BASE + (as * NMAT + i) * 32;
            const uint32_t b_addr = b_base + (NB == 2 ? i : 0) * N_MAX * 128;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
              const uint64_t bdesc = umma_desc(b_addr + kk * 32, 16, 1024, kSwizzle128B);
              const uint32_t acc = (sb > 0 || kk > 0 || (ND == 1 && i > 0)) ? 1u : 0u;
              mma_f16_ts(d, a_tmem + kk * 8, bdesc, idesc, acc);
            }
          }
          mma_commit(&aempty[as]);
          mma_commit(&bempty[bs]);
          if (++as == C::S_A) { as = 0; aph ^= 1; }
          if (++bs == C::S_B) { bs = 0; bph ^= 1; }
        }
        mma_commit(&accfull[ab]);
        if (++ab == C::NACC) { ab = 0; abph ^= 1; }
      }
      mma_commit(drain);            // completes once every MMA issued above has finished
      mbar_wait(drain, 0, abort_flag, st, 13);
    }
  } else if (warp < C::kEpWarp0) {
    // ---------------------------------------------------------------- dequant warps
    // warp -> (TMEM lane quarter q, 32-element half h of each 64-K sub-chunk); thread -> row
    const int dw = warp - C::kDqWarp0;           // 0..7
    const int q = warp & 3;
    const int h = dw >> 2;
    const int m = q * 32 + lane;                 // weight row within the 128-row tile
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int32_t* beta = args.epi.beta;
    const int bcol = args.epi.beta_col;
    int ps = 0, as = 0;
    uint32_t pph = 0, aph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Chunk ch = args.chunks[u / args.mtiles];
      const int bias = (!COLSCALE && beta) ? beta[ch.e * 2 + bcol] : 0;
      for (int ks = 0; ks < n_stage && ok; ks++) {
        if (!(ok = mbar_wait(&pfull[ps], pph, abort_flag, st, 6))) break;
        const uint8_t* stage = smem + C::OFF_P + ps * C::P_STAGE;
        for (int sub = 0; sub < C::SUBS; sub++) {
          if (ks * C::SUBS + sub >= n_sub) break;
          if (!(ok = mbar_wait(&aempty[as], aph ^ 1, abort_flag, st, 7))) break;
          tc_fence_after();
          const int c = sub * 2 + h;                   // 16-byte chunk (32 K) in the 64-byte row
#pragma unroll
          for (int i = 0; i < NMAT; i++) {
            const uint8_t* pk = stage + i * (C::PK_BYTES + C::SC_BYTES);
            const uint8_t* sc = pk + C::PK_BYTES;
            const uint4 raw = ld_shared_v4(smem_u32(pk + m * 64 + ((c ^ ((m >> 1) & 3)) << 4)));
            uint32_t o[16];
            if (COLSCALE) {
              // fp16 multipliers of k = 32c .. 32c+31 for this warp's 32-row group q
              const uint32_t sa = smem_u32(sc + (q * 128 + c * 32) * 2);
              const uint4 s0 = ld_shared_v4(sa), s1 = ld_shared_v4(sa + 16);
              const uint4 s2 = ld_shared_v4(sa + 32), s3 = ld_shared_v4(sa + 48);
              const uint32_t sv[16] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w,
                                       s2.x, s2.y, s2.z, s2.w, s3.x, s3.y, s3.z, s3.w};
              decode8v(raw.x, &sv[0], &o[0]);
              decode8v(raw.y, &sv[4], &o[4]);
              decode8v(raw.z, &sv[8], &o[8]);
              decode8v(raw.w, &sv[12], &o[12]);
            } else {
              const uint32_t sbyte = sc[m * 16 + (((ks * C::BK) / 32) & 15) + c];
              const uint32_t s1 = e8m0_to_half_bits(sbyte, bias);
              const uint32_t s2 = s1 | (s1 << 16);
              decode8(raw.x, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[0]));
              decode8(raw.y, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[4]));
              decode8(raw.z, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[8]));
              decode8(raw.w, s2, *reinterpret_cast<uint32_t(*)[4]>(&o[12]));
            }
            tmem_st16(tmem + lane_base + C::A_BASE + (as * NMAT + i) * 32 + h * 16, o);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[as]);
          if (++as == C::S_A) { as = 0; aph ^= 1; }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[ps]);
        if (++ps == C::S_P) { ps = 0; pph ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;          // accumulator row = M index within the tile
    const EpiParams& ep = args.epi;
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const Chunk ch = args.chunks[u / args.mtiles];
      const int mt = u % args.mtiles;
      const int m = mt * 128 + row;
      const bool mvalid = m < ep.M;
      const int npad = (ch.n + 15) & ~15;
      const int bias = ep.beta ? ep.beta[ch.e * 2 + ep.beta_col] : 0;
      const float wunscale = exp2f((float)(-bias));
      if (!(ok = mbar_wait(&accfull[ab], abph, abort_flag, st, 8))) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * ND * N_MAX;
      float ad[32];
      if (EPI == EPI_B1) {
#pragma unroll
        for (int rr = 0; rr < 32; rr++) ad[rr] = (rr < ep.r && mvalid) ? ep.A_d[rr * ep.M + m] : 0.f;
      }
      for (int j0 = 0; j0 < npad; j0 += 16) {
        float v0[16], v1[16];
        tmem_ld16(tbase + j0, v0);
        if (ND == 2) tmem_ld16(tbase + N_MAX + j0, v1);
        tmem_ld_wait();
        float gwp[16];
#pragma unroll
        for (int jj = 0; jj < 16; jj++) {
          gwp[jj] = 0.f;
          const int j = j0 + jj;
          if (j >= ch.n || !mvalid) continue;
          const int p = ch.p0 + j;
          const int t = ep.perm_token ? ep.perm_token[p] : p;
          const size_t o = (size_t)p * ep.M + m;
          if (EPI == EPI_F1) {
            const float cs = ep.row_scale_inv[p] * wunscale;
            const float gate = v0[jj] * cs + ep.delta_g[(size_t)t * ep.M + m];
            const float up = v1[jj] * cs + ep.delta_u[(size_t)t * ep.M + m];
            ep.G[o] = gate;
            ep.U[o] = up;
            ep.H[o] = __float2half_rn(situ_glu_fwd(gate, up));
          } else if (EPI == EPI_F2) {
            ep.Y[o] = v0[jj] * wunscale * ep.tw[p];
          } else if (EPI == EPI_B1) {
            const float ys = v0[jj] * ep.row_scale_inv[p] * wunscale;
            float lorad = 0.f;
#pragma unroll
            for (int rr = 0; rr < 32; rr++)
              if (rr < ep.r) lorad += ep.gB[(size_t)t * ep.r + rr] * ad[rr];
            const float v = ys + ep.lora_scaling * lorad;
            const float g = ep.Gs[o], uu = ep.Us[o];
            gwp[jj] = situ_glu_fwd(g, uu) * v;
            float dg, du;
            situ_glu_bwd(ep.tw[p] * v, g, uu, dg, du);
            ep.DG[o] = dg;
            ep.DU[o] = du;
          } else if (EPI == EPI_B2) {
            ep.Y[o] = v0[jj] * ep.row_scale_inv[p] * wunscale;
          } else if (EPI == EPI_STORE) {
            ep.Y[o] = v0[jj] * ep.row_scale_inv[p] * wunscale;
          } else if (EPI == EPI_ACCUM) {
            ep.Y[o] += v0[jj] * ep.row_scale_inv[p] * wunscale;
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
          if (lane < 16 && j0 + lane < ch.n)
            ep.gw_part[((size_t)mt * 4 + q) * ep.P + ch.p0 + j0 + lane] = mine;
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
  if (warp == 2) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ll
