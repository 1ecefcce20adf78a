// Host-side helpers shared by the entry points: CUDA error capture, device properties,
// TMA tensor-map encoding (through the driver entry point, so the library does not link
// libcuda directly), workspace carving and the grouped-GEMM launcher.
#pragma once
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "grouped_gemm.cuh"
#include "bs_gemm.cuh"

namespace ll {

extern thread_local char g_last_cuda_error[256];
extern thread_local int g_launch_count;
// Optional CUDA events recorded around each grouped-GEMM launch (profiling hook).
extern thread_local cudaEvent_t* g_prof_events;
extern thread_local int g_prof_n;
extern thread_local int g_prof_i;
// Optional CUDA event recorded after every kernel launch (profiling hook), on the stream of
// the C call in progress, with the kernel's name.
extern thread_local cudaStream_t g_launch_stream;
extern thread_local cudaEvent_t* g_lev;
extern thread_local const char** g_lev_names;
extern thread_local int g_lev_n;
extern thread_local int g_lev_i;

inline int cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", what, cudaGetErrorString(e));
  return LL_ERR_CUDA;
}

#define LL_CUDA(call)                                      \
  do {                                                     \
    cudaError_t e_ = (call);                               \
    if (e_ != cudaSuccess) return ::ll::cuda_fail(e_, #call); \
  } while (0)

#define LL_TRY(call)             \
  do {                           \
    int s_ = (call);             \
    if (s_ != LL_OK) return s_;  \
  } while (0)

inline int check_launch(const char* what) {
  g_launch_count++;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (g_lev && g_lev_i < g_lev_n) {
    g_lev_names[g_lev_i] = what;
    // inside a stream capture the event becomes an event-record node of the graph (timed on replay)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    LL_CUDA(cudaStreamIsCapturing(g_launch_stream, &cs));
    LL_CUDA(cudaEventRecordWithFlags(g_lev[g_lev_i++], g_launch_stream,
                                     cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0));
  }
  return LL_OK;
}

// Whether launch_pdl sets the programmatic-serialization attribute (environment LL_PDL=0
// turns it off; the kernels then run strictly one after another, as with <<<>>>).
bool pdl_enabled();

// A launch that lets the kernel start before its predecessor on the stream has finished
// (the kernel must call pdl_wait(): see common.cuh), checked and counted like check_launch.
template <typename... KArgs, typename... Args>
inline int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return check_launch(what);
}

// The stream argument of a C entry point, remembered for the launch-event hook.
#define LL_STREAM(stream_arg) \
  cudaStream_t s = static_cast<cudaStream_t>(stream_arg); \
  ::ll::g_launch_stream = s

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
};

DeviceInfo device_info();   // of the current device, cached

// ------------------------------------------------------------------------ tensor maps
int make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0, uint64_t dim1,
                uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw);

// Packed weight bytes [rows_total][cols/2] (boxes of `box_rows` rows x 64 bytes, 64-byte
// swizzle) with the reference's E8M0 scale bytes [rows_total][scale_stride] (boxes of
// box_rows x 16 bytes). box_rows: 128, or 256 for a pair of adjacent 128-row tiles.
inline int make_rowscale_maps(CUtensorMap* pk, CUtensorMap* sc, const uint8_t* packed, const uint8_t* scales,
                              int64_t rows_total, int cols, int64_t scale_stride, int box_rows = 128) {
  LL_TRY(make_map_2d(pk, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, (uint64_t)cols / 2, (uint64_t)rows_total,
                     (uint64_t)cols / 2, 64, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_64B));
  LL_TRY(make_map_2d(sc, CU_TENSOR_MAP_DATA_TYPE_UINT8, scales, (uint64_t)cols / 32, (uint64_t)rows_total,
                     (uint64_t)scale_stride, 16, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
  return LL_OK;
}

// Transposed codes [rows_total][K/2] with the fp16 column-scale table [rows_total/32][K]
// (boxes of box_rows / 32 row groups x 128 k).
inline int make_colscale_maps(CUtensorMap* pk, CUtensorMap* sc, const uint8_t* codes, const __half* cscales,
                              int64_t rows_total, int K, int box_rows = 128) {
  LL_TRY(make_map_2d(pk, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)K / 2, (uint64_t)rows_total, (uint64_t)K / 2,
                     64, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_64B));
  LL_TRY(make_map_2d(sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, cscales, (uint64_t)K, (uint64_t)rows_total / 32,
                     (uint64_t)K * 2, 128, (uint32_t)box_rows / 32, CU_TENSOR_MAP_SWIZZLE_NONE));
  return LL_OK;
}

int make_map_nd(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle sw);

// fp16 activation rows [rows][K] (K % 64 == 0), one map per tile height 16 c (c = 1..n): a
// box holds one ring stage (LL_KS columns) as 64-column halves, [half][16 c rows][128 bytes], K-major
// with the 128-byte swizzle, so a stage of a chunk of up to 16 c rows is one TMA instruction.
// The halves are a third dimension of stride 128 bytes. With nb = 2 a fourth dimension of
// stride mat_stride elements reaches the second operand (the gate and up gradients), and the
// box is [operand][half][rows][128 bytes].
inline int make_act_maps(CUtensorMap* maps, int n, const __half* base, int64_t rows, int K, int nb = 1,
                         int64_t mat_stride = 0) {
  if (K <= 0 || K % 64 || n < 1 || n > 8 || (nb != 1 && nb != 2)) return LL_ERR_ARG;
  const uint64_t dims[4] = {64, (uint64_t)rows, (uint64_t)K / 64, (uint64_t)nb};
  const uint64_t strides[3] = {(uint64_t)K * 2, 128, (uint64_t)mat_stride * 2};
  for (int c = 1; c <= n; c++) {
    const uint32_t box[4] = {64, (uint32_t)(16 * c), LL_KS / 64, (uint32_t)nb};
    LL_TRY(make_map_nd(&maps[c - 1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, nb == 2 ? 4 : 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B));
  }
  return LL_OK;
}

int set_smem_attr(const void* func, int bytes);

template <int EPI, int NMAT, int NB, bool COLSCALE, int N_MAX>
int launch_gemm(const CUtensorMap* pk, const CUtensorMap* sc, const CUtensorMap* act, const GemmArgs& a,
                cudaStream_t stream) {
  using Cfg = GemmCfg<NMAT, NB, COLSCALE, N_MAX>;
  TmaSet<NMAT, N_MAX> tm;
  for (int i = 0; i < NMAT; i++) { tm.pk[i] = pk[i]; tm.sc[i] = sc[i]; }
  for (int i = 0; i < N_MAX / 16; i++) tm.act[i] = act[i];
  auto kern = grouped_mxfp4_gemm<EPI, NMAT, NB, COLSCALE, N_MAX>;
  LL_TRY(set_smem_attr(reinterpret_cast<const void*>(kern), Cfg::SMEM));
  const DeviceInfo di = device_info();
  const bool prof = g_prof_events && g_prof_i + 2 <= g_prof_n;
  if (prof) LL_CUDA(cudaEventRecord(g_prof_events[g_prof_i], stream));
  const int rc = launch_pdl(EPI == EPI_F1   ? "grouped_mxfp4_gemm F1 gate/up"
                            : EPI == EPI_F2 ? "grouped_mxfp4_gemm F2 down"
                            : EPI == EPI_B1 ? "grouped_mxfp4_gemm B1 g.W2"
                            : EPI == EPI_B2 ? "grouped_mxfp4_gemm B2 dg.W1+du.W3"
                                            : "grouped_mxfp4_gemm",
                            kern, dim3(di.sms), dim3(Cfg::kThreads), Cfg::SMEM, stream, tm, a);
  if (prof) {
    LL_CUDA(cudaEventRecord(g_prof_events[g_prof_i + 1], stream));
    g_prof_i += 2;
  }
  return rc;
}

// Weight codes [rows_total][K/2] bytes as the block-scaled MMA reads them: 16 x 4-bit values
// per 16-byte chunk in shared memory (TMA unpacks each 8 packed bytes into 16), boxes of
// box_rows rows x 128 K, 128-byte swizzle. K a multiple of 128; the row stride (K/2 bytes)
// and the base must be 32-byte aligned.
inline int make_fp4_map(CUtensorMap* m, const uint8_t* packed, int64_t rows_total, int K, int box_rows) {
  if (K % 128 || (reinterpret_cast<uintptr_t>(packed) & 31)) return LL_ERR_ARG;
  return make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, packed, (uint64_t)K, (uint64_t)rows_total,
                     (uint64_t)K / 2, 128, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// E4M3 activation terms [3][rows][K] bytes (BS_FP8), one map per chunk height 16 c (c = 1..n):
// a box is [3 terms][16 c rows][128 K], 128-byte swizzle.
inline int make_e4m3x3_maps(CUtensorMap* maps, int n, const uint8_t* base, int64_t rows, int K) {
  constexpr int NT = BsTerms<BS_FP8>::value;
  if (K % 128 || n < 1 || n > 4) return LL_ERR_ARG;
  const uint64_t dims[3] = {(uint64_t)K, (uint64_t)rows, (uint64_t)NT};
  const uint64_t strides[2] = {(uint64_t)K, (uint64_t)rows * K};
  for (int c = 1; c <= n; c++) {
    const uint32_t box[3] = {128, (uint32_t)(16 * c), (uint32_t)NT};
    LL_TRY(make_map_nd(&maps[c - 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, base, 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B));
  }
  return LL_OK;
}

// Packed E2M1 activation terms [4][rows][K/2] bytes (BS_FP4): a box is [4 terms][rp c rows][64
// bytes = 128 K] (rp = 16, or 4 for four-row tiles), 64-byte swizzle.
inline int make_e2m1x4_maps(CUtensorMap* maps, int n, const uint8_t* base, int64_t rows, int K, int rp = 16) {
  constexpr int NT = BsTerms<BS_FP4>::value;
  if (K % 128 || n < 1 || n > 4 || (rp != 4 && rp != 16)) return LL_ERR_ARG;
  const uint64_t dims[3] = {(uint64_t)K / 2, (uint64_t)rows, (uint64_t)NT};
  const uint64_t strides[2] = {(uint64_t)K / 2, (uint64_t)rows * K / 2};
  for (int c = 1; c <= n; c++) {
    const uint32_t box[3] = {64, (uint32_t)(rp * c), (uint32_t)NT};
    LL_TRY(make_map_nd(&maps[c - 1], CU_TENSOR_MAP_DATA_TYPE_UINT8, base, 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_64B));
  }
  return LL_OK;
}

// Packed weight codes [rows_total][K/2] bytes as BS_FP4 reads them: boxes of box_rows rows x 64
// bytes (128 K), 64-byte swizzle.
inline int make_fp4_packed_map(CUtensorMap* m, const uint8_t* packed, int64_t rows_total, int K, int box_rows) {
  if (K % 128) return LL_ERR_ARG;
  return make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, (uint64_t)K / 2, (uint64_t)rows_total,
                     (uint64_t)K / 2, 64, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_64B);
}

template <int EPI, int NMAT, int N_MAX, int KIND>
int launch_bs_gemm(const CUtensorMap* a, const CUtensorMap* b, const BsArgs& args, cudaStream_t stream) {
  using Cfg = BsCfg<NMAT, N_MAX, KIND>;
  BsTma<NMAT, N_MAX, KIND> tm;
  for (int i = 0; i < NMAT; i++) tm.a[i] = a[i];
  for (int i = 0; i < BsRows<N_MAX>::maps; i++) tm.b[i] = b[i];
  auto kern = grouped_mxfp4_bs_gemm<EPI, NMAT, N_MAX, KIND>;
  LL_TRY(set_smem_attr(reinterpret_cast<const void*>(kern), Cfg::SMEM));
  const DeviceInfo di = device_info();
  const bool prof = g_prof_events && g_prof_i + 2 <= g_prof_n;
  if (prof) LL_CUDA(cudaEventRecord(g_prof_events[g_prof_i], stream));
  const int rc = launch_pdl(EPI == EPI_F1   ? "grouped_mxfp4_bs_gemm F1 gate/up"
                            : EPI == EPI_F2 ? "grouped_mxfp4_bs_gemm F2 down"
                                            : "grouped_mxfp4_bs_gemm",
                            kern, dim3(di.sms), dim3(Cfg::kThreads), Cfg::SMEM, stream, tm, args);
  if (prof) {
    LL_CUDA(cudaEventRecord(g_prof_events[g_prof_i + 1], stream));
    g_prof_i += 2;
  }
  return rc;
}

// ----------------------------------------------------------------------- workspace
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

// Status word + reset, read back after a sequence of launches.
int reset_status(DevStatus* st, cudaStream_t s);
int read_status(DevStatus* st, cudaStream_t s);

}  // namespace ll
