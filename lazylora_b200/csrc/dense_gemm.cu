// Dense bf16 GEMMs on the tensor cores for the projections around the routed experts: the
// latent block's down / up projections (lazy_lora/trainer/lazy_trainer.py:722-735) and the
// shared expert's gate / up / down (its F.linear calls), forward and input-gradient backward.
//
// C[M][N] = sum over a job's operand pairs p of A_p . op(B_p), bf16 operands, fp32 accumulation
// in tensor memory, C written as bf16 (round to nearest) or fp32. A_p is row-major [M][K_p];
// B_p is either [N][K_p] (C = A B^T, the layout of a weight in F.linear) or [K_p][N] (C = A B,
// the input gradient through that weight). A launch runs up to two jobs (two outputs of one A,
// e.g. the gate and up projections, or one output of two pairs, e.g. dG W_g + dU W_u summed in
// tensor memory before the single rounding).
//
// One persistent CTA per SM, 7 warps: 0 TMA producer (A tile 128 x 64 and B tile BN x 64 of a
// K block per stage, 128-byte swizzle; a [K][N] B arrives as BN/64 boxes of 64 N x 64 K),
// 1 MMA issuer (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = BN, K = 16, four per stage;
// A K-major, B K-major or MN-major by the instruction descriptor), 2..5 epilogue (tcgen05.ld of
// their lane quarter, 16 columns at a time, 16-byte stores), 6 watcher (waits on the mbarriers
// and publishes an event count the issuer polls, so the issuing thread never waits on an
// mbarrier). Accumulators double-buffered (2 x BN columns), so a tile's epilogue overlaps the
// next tile's main loop. Tiles are ordered M-fastest, so the CTAs working at the same time share
// B tiles (the weight slices) through L2; A (the activations) stays in L2. Every wait is
// bounded (common.cuh). No cluster; every TMA load fills only the issuing CTA's shared memory.
#include <algorithm>
#include <cmath>

#include "host_common.cuh"
#include "ops.cuh"

namespace ll {

constexpr int kDnThreads = 7 * 32;
constexpr int kDnBK = 64;                       // K per stage: one 128-byte bf16 row of the swizzle
constexpr int kDnAStage = 128 * kDnBK * 2;      // 16 KB
constexpr int kDnMaxStages = 8;
constexpr int kDnSmemBudget = 225 * 1024;

struct DenseJob {
  void* C;
  int64_t ldc;
  int n_pairs;      // 1 or 2
  int map[2];       // tensor-map index (a[map], b[map]) of each pair
  int kb[2];        // 64-wide K blocks of each pair
  int b_mn[2];      // 1: B of the pair is [K][N] (N-major)
  int nt;           // tiles along N
};

struct DenseArgs {
  int M, N, BN, mt, S, stage_bytes;
  int n_jobs, tiles0, tiles;   // tiles of job 0, all tiles
  int c_bf16;
  DenseJob job[2];
};

// Status word of these launches (one per device; a wait that runs out records itself here and
// the word stays set until ll_gemm_bf16_status reads and clears it).
__device__ DevStatus g_dn_status;

struct DenseTma {
  CUtensorMap a[2], b[2];
};

// Instruction descriptor, kind::f16: bf16 A and B, fp32 D, M = 128, N = n; B MN-major when asked.
LL_DEV uint32_t idesc_bf16_m128_major(uint32_t n, bool b_mn_major) {
  uint32_t d = 0;
  d |= 1u << 4;                       // D format F32
  d |= 1u << 7;                       // A format BF16
  d |= 1u << 10;                      // B format BF16
  d |= (b_mn_major ? 1u : 0u) << 16;  // B major
  d |= (n >> 3) << 17;
  d |= (128u >> 4) << 24;
  return d;
}

__global__ void __launch_bounds__(kDnThreads, 1) k_dense_gemm(const __grid_constant__ DenseTma tm, const DenseArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base);
  uint64_t* full = bars;
  uint64_t* empty = full + kDnMaxStages;
  uint64_t* accfull = empty + kDnMaxStages;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* ready_seq = tmem_slot + 2;
  uint8_t* stages = base + 1024;
  const int S = args.S, STG = args.stage_bytes, BN = args.BN;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], 4); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *ready_seq = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; i++) { tma_prefetch_desc(&tm.a[i]); tma_prefetch_desc(&tm.b[i]); }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  DevStatus* st = &g_dn_status;
  pdl_launch_next();                        // (after the allocation)
  pdl_wait();

  auto tile_of = [&](int u, int& j, int& m0, int& n0) {
    j = u < args.tiles0 ? 0 : 1;
    const int v = j ? u - args.tiles0 : u;
    m0 = (v % args.mt) * 128;
    n0 = (v / args.mt) * BN;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t tx = kDnAStage + BN * kDnBK * 2;
      for (int u = blockIdx.x; u < args.tiles && ok; u += gridDim.x) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        for (int p = 0; p < jb.n_pairs && ok; p++) {
          const CUtensorMap* am = &tm.a[jb.map[p]];
          const CUtensorMap* bm = &tm.b[jb.map[p]];
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            if (!(ok = mbar_wait_sleep(&empty[s], ph ^ 1, abort_flag, st, 41, 256))) break;
            uint8_t* a_s = stages + s * STG;
            uint8_t* b_s = a_s + kDnAStage;
            mbar_arrive_expect_tx(&full[s], tx);
            tma_load_2d(a_s, am, &full[s], kb * kDnBK, m0);
            if (!jb.b_mn[p]) {
              tma_load_2d(b_s, bm, &full[s], kb * kDnBK, n0);
            } else {
              for (int c = 0; c < BN / 64; c++) tma_load_2d(b_s + c * 64 * 128, bm, &full[s], n0 + 64 * c, kb * kDnBK);
            }
            issued++;
            if (++s == S) { s = 0; ph ^= 1; }
          }
        }
      }
      for (int i = 0; i < S && i < issued; i++) {   // drain: the last stages' bytes landed
        if (--s < 0) { s = S - 1; ph ^= 1; }
        mbar_wait_sleep(&full[s], ph, abort_flag, st, 42, 256);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int s = 0, ab = 0;
      uint32_t ev = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < args.tiles && ok; u += gridDim.x) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 43))) break;   // accumulator ab drained
        tc_fence_after();
        const uint32_t d = tmem + ab * 256;
        bool first = true;
        for (int p = 0; p < jb.n_pairs && ok; p++) {
          const bool bmn = jb.b_mn[p] != 0;
          const uint32_t idesc = idesc_bf16_m128_major(BN, bmn);
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 44))) break;
            tc_fence_after();
            const uint32_t a0 = smem_u32(stages + s * STG), b0 = a0 + kDnAStage;
#pragma unroll
            for (int kk = 0; kk < kDnBK / 16; kk++) {
              const uint64_t adesc = umma_desc(a0 + kk * 32, 16, 1024, kSwizzle128B);
              // K-major B: the next 16 K are 32 bytes along the row; MN-major B: 16 rows of 128
              // bytes further, the 64-column boxes 64 x 128 bytes apart (leading offset)
              const uint64_t bdesc = bmn ? umma_desc(b0 + kk * 16 * 128, 64 * 128, 1024, kSwizzle128B)
                                         : umma_desc(b0 + kk * 32, 16, 1024, kSwizzle128B);
              mma_f16_ss(d, adesc, bdesc, idesc, first ? 0u : 1u);
              first = false;
            }
            mma_commit(&empty[s]);
            if (++s == S) s = 0;
          }
        }
        if (!ok) break;
        mma_commit(&accfull[ab]);
        ab ^= 1;
      }
      mma_commit(drain);                         // completes once every MMA issued above finished
      volatile int keep_waiting = 0;             // wait for them even after an abort
      mbar_wait_sleep(drain, 0, &keep_waiting, st, 45, 256);
    }
    __syncwarp();
  } else if (warp == 6) {
    // ---------------------------------------------------------------------- watcher
    if (lane == 0) {
      int s = 0, ab = 0;
      uint32_t ph = 0, abph = 0, ev = 0;
      for (int u = blockIdx.x; u < args.tiles; u += gridDim.x) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 46);
        seq_publish(ready_seq, ++ev);
        for (int p = 0; p < jb.n_pairs; p++)
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            mbar_wait(&full[s], ph, abort_flag, st, 47);
            seq_publish(ready_seq, ++ev);
            if (++s == S) { s = 0; ph ^= 1; }
          }
        if (++ab == 2) { ab = 0; abph ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------------ epilogue
    const int q = warp & 3;                      // TMEM lane quarter this warp may access
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < args.tiles && ok; u += gridDim.x) {
      int j, m0, n0;
      tile_of(u, j, m0, n0);
      const DenseJob& jb = args.job[j];
      if (!(ok = mbar_wait_sleep(&accfull[ab], abph, abort_flag, st, 48, 512))) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * 256;
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(tbase + c, v);
        tmem_ld_wait();
        const int col = n0 + c;
        if (row >= args.M || col >= args.N) continue;
        if (args.c_bf16) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(jb.C) + (int64_t)row * jb.ldc + col;
          if (col + 16 <= args.N) {
            uint4 w[2];
            uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
              wp[i] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            reinterpret_cast<uint4*>(out)[0] = w[0];
            reinterpret_cast<uint4*>(out)[1] = w[1];
          } else {
            for (int i = 0; i < 16 && col + i < args.N; i++) out[i] = __float2bfloat16_rn(v[i]);
          }
        } else {
          float* out = static_cast<float*>(jb.C) + (int64_t)row * jb.ldc + col;
          if (col + 16 <= args.N) {
#pragma unroll
            for (int i = 0; i < 4; i++)
              reinterpret_cast<float4*>(out)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            for (int i = 0; i < 16 && col + i < args.N; i++) out[i] = v[i];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[ab]);
      ab ^= 1;
      if (ab == 0) abph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- CTA-pair variant
// The same GEMM with tiles of 256 rows on a CTA pair (a cluster of 2): tcgen05.mma.cta_group::2
// with M = 256 reads A's rows from both CTAs' shared memory (rows 0..127 from CTA 0, 128..255
// from CTA 1, at the same offset) and B's N/2-row halves likewise, and writes each CTA's 128
// accumulator rows to its own tensor memory. Each CTA loads only its own halves (one destination):
// per CTA a stage is A 16 KB + B BN/2 x 128 B, so a ring of 6 stages fits and each byte brought
// from L2 feeds twice the MMA work of the single-CTA kernel. CTA 0 issues the MMAs; its stage
// barrier expects both CTAs' bytes (CTA 1's TMA completes on CTA 0's barrier), and each commit
// is made to the barriers of both CTAs (two plain commits); CTA 1's epilogue arrives on CTA 0's
// accumulator-empty barrier remotely. Cluster barriers after the set-up and before the
// tensor-memory release keep both CTAs alive while the other still uses their memory.
LL_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
LL_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of this CTA's shared variable at `p` in cluster CTA `rank`.
LL_DEV uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
LL_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
LL_DEV void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
LL_DEV void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
LL_DEV void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
LL_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {   // whole warp, both CTAs
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
LL_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {     // whole warp, both CTAs
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Instruction descriptor for the pair: M = 256.
LL_DEV uint32_t idesc_bf16_m256_major(uint32_t n, bool b_mn_major) {
  return (idesc_bf16_m128_major(n, b_mn_major) & ~(0x1Fu << 24)) | ((256u >> 4) << 24);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kDnThreads, 1)
    k_dense_gemm_pair(const __grid_constant__ DenseTma tm, const DenseArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base);
  uint64_t* full = bars;
  uint64_t* empty = full + kDnMaxStages;
  uint64_t* accfull = empty + kDnMaxStages;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* ready_seq = tmem_slot + 2;
  uint8_t* stages = base + 1024;
  const int S = args.S, STG = args.stage_bytes, BN = args.BN, HB = args.BN / 2;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x / 2, n_pairs_grid = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], 8); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *ready_seq = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; i++) { tma_prefetch_desc(&tm.a[i]); tma_prefetch_desc(&tm.b[i]); }
  }
  tc_fence_before();
  cluster_sync();                           // both CTAs' barriers initialised, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  DevStatus* st = &g_dn_status;
  pdl_launch_next();
  pdl_wait();

  auto tile_of = [&](int u, int& j, int& m0, int& n0) {
    j = u < args.tiles0 ? 0 : 1;
    const int v = j ? u - args.tiles0 : u;
    m0 = (v % args.mt) * 256;
    n0 = (v / args.mt) * BN;
  };

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs, own halves)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t tx_cta = kDnAStage + HB * kDnBK * 2;
      for (int u = pair; u < args.tiles && ok; u += n_pairs_grid) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        const int am0 = m0 + 128 * (int)rank, bn0 = n0 + HB * (int)rank;
        for (int p = 0; p < jb.n_pairs && ok; p++) {
          const CUtensorMap* am = &tm.a[jb.map[p]];
          const CUtensorMap* bm = &tm.b[jb.map[p]];
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            if (!(ok = mbar_wait_sleep(&empty[s], ph ^ 1, abort_flag, st, 51, 256))) break;
            uint8_t* a_s = stages + s * STG;
            uint8_t* b_s = a_s + kDnAStage;
            const uint32_t fb = peer_addr(&full[s], 0);        // CTA 0's stage barrier
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * tx_cta);
            tma_load_2d_pair(a_s, am, fb, kb * kDnBK, am0);
            if (!jb.b_mn[p]) {
              tma_load_2d_pair(b_s, bm, fb, kb * kDnBK, bn0);
            } else {
              for (int c = 0; c < HB / 64; c++) tma_load_2d_pair(b_s + c * 64 * 128, bm, fb, bn0 + 64 * c, kb * kDnBK);
            }
            if (++s == S) { s = 0; ph ^= 1; }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer (CTA 0 only)
    if (leader && lane == 0) {
      int s = 0, ab = 0;
      uint32_t ev = 0;
      bool ok = true;
      for (int u = pair; u < args.tiles && ok; u += n_pairs_grid) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 53))) break;   // accumulator ab drained
        tc_fence_after();
        const uint32_t d = tmem + ab * 256;
        bool first = true;
        for (int p = 0; p < jb.n_pairs && ok; p++) {
          const bool bmn = jb.b_mn[p] != 0;
          const uint32_t idesc = idesc_bf16_m256_major(BN, bmn);
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            if (!(ok = seq_wait(ready_seq, ++ev, abort_flag, st, 54))) break;
            tc_fence_after();
            const uint32_t a0 = smem_u32(stages + s * STG), b0 = a0 + kDnAStage;
#pragma unroll
            for (int kk = 0; kk < kDnBK / 16; kk++) {
              const uint64_t adesc = umma_desc(a0 + kk * 32, 16, 1024, kSwizzle128B);
              const uint64_t bdesc = bmn ? umma_desc(b0 + kk * 16 * 128, 64 * 128, 1024, kSwizzle128B)
                                         : umma_desc(b0 + kk * 32, 16, 1024, kSwizzle128B);
              mma_f16_ss_pair(d, adesc, bdesc, idesc, first ? 0u : 1u);
              first = false;
            }
            mma_commit_pair(peer_addr(&empty[s], 0));           // the stage is free in both CTAs
            mma_commit_pair(peer_addr(&empty[s], 1));
            if (++s == S) s = 0;
          }
        }
        if (!ok) break;
        mma_commit_pair(peer_addr(&accfull[ab], 0));
        mma_commit_pair(peer_addr(&accfull[ab], 1));
        ab ^= 1;
      }
      mma_commit_pair(peer_addr(drain, 0));   // completes once every MMA issued above finished
      volatile int keep_waiting = 0;          // wait for them even after an abort
      mbar_wait_sleep(drain, 0, &keep_waiting, st, 55, 256);
    }
    __syncwarp();
  } else if (warp == 6) {
    // -------------------------------------------------------------- watcher (CTA 0 only)
    if (leader && lane == 0) {
      int s = 0, ab = 0;
      uint32_t ph = 0, abph = 0, ev = 0;
      for (int u = pair; u < args.tiles; u += n_pairs_grid) {
        int j, m0, n0;
        tile_of(u, j, m0, n0);
        const DenseJob& jb = args.job[j];
        mbar_wait(&accempty[ab], abph ^ 1, abort_flag, st, 56);
        seq_publish(ready_seq, ++ev);
        for (int p = 0; p < jb.n_pairs; p++)
          for (int kb = 0; kb < jb.kb[p]; kb++) {
            mbar_wait(&full[s], ph, abort_flag, st, 57);
            seq_publish(ready_seq, ++ev);
            if (++s == S) { s = 0; ph ^= 1; }
          }
        if (++ab == 2) { ab = 0; abph ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- epilogue (both CTAs, own rows)
    const int q = warp & 3;
    int ab = 0;
    uint32_t abph = 0;
    bool ok = true;
    for (int u = pair; u < args.tiles && ok; u += n_pairs_grid) {
      int j, m0, n0;
      tile_of(u, j, m0, n0);
      const DenseJob& jb = args.job[j];
      if (!(ok = mbar_wait_sleep(&accfull[ab], abph, abort_flag, st, 58, 512))) break;
      tc_fence_after();
      const int row = m0 + 128 * (int)rank + q * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * 256;
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(tbase + c, v);
        tmem_ld_wait();
        const int col = n0 + c;
        if (row >= args.M || col >= args.N) continue;
        if (args.c_bf16) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(jb.C) + (int64_t)row * jb.ldc + col;
          if (col + 16 <= args.N) {
            uint4 w[2];
            uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
              wp[i] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            reinterpret_cast<uint4*>(out)[0] = w[0];
            reinterpret_cast<uint4*>(out)[1] = w[1];
          } else {
            for (int i = 0; i < 16 && col + i < args.N; i++) out[i] = __float2bfloat16_rn(v[i]);
          }
        } else {
          float* out = static_cast<float*>(jb.C) + (int64_t)row * jb.ldc + col;
          if (col + 16 <= args.N) {
#pragma unroll
            for (int i = 0; i < 4; i++)
              reinterpret_cast<float4*>(out)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            for (int i = 0; i < 16 && col + i < args.N; i++) out[i] = v[i];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_addr(&accempty[ab], 0));
      ab ^= 1;
      if (ab == 0) abph ^= 1;
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();                           // both CTAs done with every barrier, stage and column
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

// The tile width: the multiple of 16 (of 64 when a B operand is N-major; for CTA pairs 32 and
// 128) up to 256 that minimises (waves of tiles over the units) x (a tile's time). A tile's time
// grows only as BN^0.23: the narrower tile brings the same A bytes for fewer MMAs, and the
// measured rates per column at BN = 128 / 192 / 256 are 0.59 / 0.82 / 1 of the widest's.
// units: the SMs (single-CTA tiles of 128 rows) or the CTA pairs (tiles of 256 rows).
static int pick_bn(int M, int N, int jobs, bool any_mn, int units, bool pair) {
  const int rows = pair ? 256 : 128;
  const int mt = (M + rows - 1) / rows;
  const int step = pair ? (any_mn ? 128 : 32) : (any_mn ? 64 : 16);
  int best = 256;
  double best_cost = 1e30;
  for (int bn = step < 32 ? 32 : step; bn <= 256; bn += step) {
    const long long tiles = (long long)mt * ((N + bn - 1) / bn) * jobs;
    const long long waves = (tiles + units - 1) / units;
    const double cost = (double)waves * pow((double)bn, 0.23);
    if (cost < best_cost - 1e-9) { best_cost = cost; best = bn; }
  }
  return best;
}

struct DenseOperand {
  const void* A;
  int64_t lda;
  int K;
  const void* B;
  int64_t ldb;
  int b_nk;        // 1: B is [N][K]
};

static int dense_gemm(int M, int N, int n_jobs, const int* pairs_per_job, const DenseOperand* ops, void* const* C,
                      const int64_t* ldc, int c_bf16, cudaStream_t s) {
  if (M <= 0 || N <= 0 || n_jobs < 1 || n_jobs > 2) return LL_ERR_ARG;
  int n_ops = 0;
  bool any_mn = false;
  for (int j = 0; j < n_jobs; j++) {
    if (pairs_per_job[j] < 1 || pairs_per_job[j] > 2) return LL_ERR_ARG;
    n_ops += pairs_per_job[j];
  }
  if (n_ops > 2) return LL_ERR_ARG;             // two tensor-map pairs per launch
  for (int i = 0; i < n_ops; i++) {
    const DenseOperand& o = ops[i];
    if (!o.A || !o.B || o.K <= 0 || o.lda < o.K || o.lda % 8 || o.ldb % 8) return LL_ERR_ARG;
    if (o.b_nk ? o.ldb < o.K : o.ldb < N) return LL_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(o.A) | reinterpret_cast<uintptr_t>(o.B)) % 16) return LL_ERR_ARG;
    any_mn |= !o.b_nk;
  }
  for (int j = 0; j < n_jobs; j++) {
    if (!C[j] || ldc[j] < N || ldc[j] % 8 || reinterpret_cast<uintptr_t>(C[j]) % 16) return LL_ERR_ARG;
  }
  const DeviceInfo di = device_info();
  // tuning overrides: LL_DENSE_PAIR=0 (single-CTA tiles only), LL_DENSE_BN (the tile width, a
  // multiple the chosen variant takes, <= 256) and LL_DENSE_STAGES (ring depth, at most what
  // shared memory holds)
  static const int env_pair = [] { const char* e = getenv("LL_DENSE_PAIR"); return e ? atoi(e) : 1; }();
  static const int env_bn = [] { const char* e = getenv("LL_DENSE_BN"); return e ? atoi(e) : 0; }();
  static const int env_st = [] { const char* e = getenv("LL_DENSE_STAGES"); return e ? atoi(e) : 0; }();
  // CTA pairs (256-row tiles) once there are more than 128 rows
  const bool pair = env_pair != 0 && M > 128 && di.sms >= 2;
  const int units = pair ? di.sms / 2 : di.sms;
  DenseArgs a{};
  a.M = M;
  a.N = N;
  a.BN = pick_bn(M, N, n_jobs, any_mn, units, pair);
  const int bn_step = pair ? (any_mn ? 128 : 32) : (any_mn ? 64 : 16);
  if (env_bn >= bn_step && env_bn <= 256 && env_bn % bn_step == 0) a.BN = env_bn;
  a.mt = (M + (pair ? 255 : 127)) / (pair ? 256 : 128);
  a.stage_bytes = kDnAStage + (pair ? a.BN / 2 : a.BN) * kDnBK * 2;
  a.S = std::min(kDnMaxStages, (kDnSmemBudget - 1024 - 1024) / a.stage_bytes);
  if (env_st >= 2 && env_st < a.S) a.S = env_st;
  if (a.S < 2) return LL_ERR_ARG;
  a.n_jobs = n_jobs;
  a.c_bf16 = c_bf16;
  DenseTma tm;
  int op = 0;
  for (int j = 0; j < n_jobs; j++) {
    DenseJob& jb = a.job[j];
    jb.C = C[j];
    jb.ldc = ldc[j];
    jb.n_pairs = pairs_per_job[j];
    jb.nt = (N + a.BN - 1) / a.BN;
    for (int p = 0; p < jb.n_pairs; p++, op++) {
      const DenseOperand& o = ops[op];
      jb.map[p] = op;
      jb.kb[p] = (o.K + kDnBK - 1) / kDnBK;
      jb.b_mn[p] = o.b_nk ? 0 : 1;
      LL_TRY(make_map_2d(&tm.a[op], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, o.A, (uint64_t)o.K, (uint64_t)M,
                         (uint64_t)o.lda * 2, kDnBK, 128, CU_TENSOR_MAP_SWIZZLE_128B));
      if (o.b_nk)   // a CTA of a pair loads half of the tile's B rows
        LL_TRY(make_map_2d(&tm.b[op], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, o.B, (uint64_t)o.K, (uint64_t)N,
                           (uint64_t)o.ldb * 2, kDnBK, pair ? a.BN / 2 : a.BN, CU_TENSOR_MAP_SWIZZLE_128B));
      else
        LL_TRY(make_map_2d(&tm.b[op], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, o.B, (uint64_t)N, (uint64_t)o.K,
                           (uint64_t)o.ldb * 2, 64, kDnBK, CU_TENSOR_MAP_SWIZZLE_128B));
    }
  }
  for (int i = op; i < 2; i++) { tm.a[i] = tm.a[0]; tm.b[i] = tm.b[0]; }
  a.tiles0 = a.mt * a.job[0].nt;
  a.tiles = a.tiles0 + (n_jobs == 2 ? a.mt * a.job[1].nt : 0);
  const int smem = 1024 + 1024 + a.S * a.stage_bytes;
  if (pair) {
    LL_TRY(set_smem_attr(reinterpret_cast<const void*>(k_dense_gemm_pair), smem));
    const int grid = 2 * std::min(a.tiles, units);
    return launch_pdl("k_dense_gemm_pair", k_dense_gemm_pair, dim3(grid), dim3(kDnThreads), smem, s, tm, a);
  }
  LL_TRY(set_smem_attr(reinterpret_cast<const void*>(k_dense_gemm), smem));
  const int grid = std::min(a.tiles, di.sms);
  return launch_pdl("k_dense_gemm", k_dense_gemm, dim3(grid), dim3(kDnThreads), smem, s, tm, a);
}

}  // namespace ll

using namespace ll;

extern "C" {

int ll_gemm_bf16(int M, int N, int K, const void* A, int64_t lda, const void* B, int64_t ldb, int b_nk, void* C,
                 int64_t ldc, int c_dtype, void* stream) {
  if (c_dtype != 0 && c_dtype != 1) return LL_ERR_ARG;
  LL_TRY(check_arch());
  LL_STREAM(stream);
  g_launch_count = 0;
  const int pairs[1] = {1};
  const DenseOperand ops[1] = {{A, lda, K, B, ldb, b_nk}};
  void* const cs[1] = {C};
  const int64_t lc[1] = {ldc};
  return dense_gemm(M, N, 1, pairs, ops, cs, lc, c_dtype, s);
}

int ll_gemm_bf16_two_outputs(int M, int N, int K, const void* A, int64_t lda, const void* B0, const void* B1,
                             int64_t ldb, int b_nk, void* C0, void* C1, int64_t ldc, int c_dtype, void* stream) {
  if (c_dtype != 0 && c_dtype != 1) return LL_ERR_ARG;
  LL_TRY(check_arch());
  LL_STREAM(stream);
  g_launch_count = 0;
  const int pairs[2] = {1, 1};
  const DenseOperand ops[2] = {{A, lda, K, B0, ldb, b_nk}, {A, lda, K, B1, ldb, b_nk}};
  void* const cs[2] = {C0, C1};
  const int64_t lc[2] = {ldc, ldc};
  return dense_gemm(M, N, 2, pairs, ops, cs, lc, c_dtype, s);
}

int ll_gemm_bf16_sum2(int M, int N, const void* A0, int K0, int64_t lda0, const void* B0, int64_t ldb0, int b0_nk,
                      const void* A1, int K1, int64_t lda1, const void* B1, int64_t ldb1, int b1_nk, void* C,
                      int64_t ldc, int c_dtype, void* stream) {
  if (c_dtype != 0 && c_dtype != 1) return LL_ERR_ARG;
  LL_TRY(check_arch());
  LL_STREAM(stream);
  g_launch_count = 0;
  const int pairs[1] = {2};
  const DenseOperand ops[2] = {{A0, lda0, K0, B0, ldb0, b0_nk}, {A1, lda1, K1, B1, ldb1, b1_nk}};
  void* const cs[1] = {C};
  const int64_t lc[1] = {ldc};
  return dense_gemm(M, N, 1, pairs, ops, cs, lc, c_dtype, s);
}

int ll_gemm_bf16_status(void* stream) {
  LL_STREAM(stream);
  DevStatus h{};
  LL_CUDA(cudaMemcpyFromSymbolAsync(&h, g_dn_status, sizeof(DevStatus), 0, cudaMemcpyDeviceToHost, s));
  LL_CUDA(cudaStreamSynchronize(s));
  if (h.code != 0) {
    const DevStatus zero{};
    LL_CUDA(cudaMemcpyToSymbolAsync(g_dn_status, &zero, sizeof(DevStatus), 0, cudaMemcpyHostToDevice, s));
    LL_CUDA(cudaStreamSynchronize(s));
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "device status %d at site %d (info %d)", h.code, h.where,
             h.info);
    return h.code;
  }
  return LL_OK;
}

}  // extern "C"
