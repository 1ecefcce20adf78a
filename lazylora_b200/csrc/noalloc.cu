// An allocation-free variant of ll_mxfp4_gemm.
//
// Some callers cannot allocate device memory: a host binding that holds raw pointers and no
// device allocator of its own (the reference binds its kernels through ctypes with plain
// pointers), or code that runs where allocating is not allowed. ll_mxfp4_gemm asks such a
// caller for a workspace; this entry point needs none. Its scratch space (the status word,
// the chunk list, the decode bias, the fp16 activation rows and their scales) lives in the
// file-scope device array below, LL_NOALLOC_SCRATCH_BYTES bytes that every GPU which loads
// the library keeps until the process exits.
//
// In host code the array's name is only a host-side handle, not a device address, so the
// address passed to the kernels comes from cudaGetSymbolAddress, looked up once per device
// (with that device current) on the entry point's first call there, and again if that
// device's context was created anew since (after cudaDeviceReset). Make the first call on a
// device before any stream capture. A call returns after its GPU work finished: it reads the
// device status word back, so it waits on its stream.
//
// Every call shares the one array and leaves its contents behind; each call re-initialises
// what it reads (status word, chunk list, bias, activation rows). Calls that overlap on the
// GPU (different streams, or different host threads on one device) race on the array and
// must be serialised by the caller.
#include <mutex>

#include "host_common.cuh"
#include "ops.cuh"

using namespace ll;

static __device__ __align__(256) uint8_t g_noalloc_scratch[LL_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoAllocNmax = 128;

struct NoAllocLayout {
  DevStatus* st;
  Chunk* chunks;
  int* n_chunks;
  int32_t* beta;
  float* inv;
  __half* act;
};

size_t noalloc_layout(void* base, int M, int K, NoAllocLayout* out) {
  Carver c(base);
  NoAllocLayout w;
  w.st = c.take<DevStatus>(1);
  w.chunks = c.take<Chunk>((M + kNoAllocNmax - 1) / kNoAllocNmax + 1);
  w.n_chunks = c.take<int>(1);
  w.beta = c.take<int32_t>(2);
  w.inv = c.take<float>(M);
  w.act = c.take<__half>((size_t)M * ((K + 63) / 64 * 64));   // rows padded to whole 64-K halves
  if (out) *out = w;
  return c.off;
}

// The current CUDA context (driver API, reached through the runtime's entry-point query).
CUcontext current_context() {
  typedef CUresult (*CtxGetCurrent)(CUcontext*);
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetCurrent>(p) : nullptr;
  }();
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Device address of the scratch array for the current device, looked up once per device and
// context: a context created anew on that device (after cudaDeviceReset) loads the module
// again, so the address is looked up again then.
int scratch_address(void** out) {
  struct Entry { CUcontext ctx; void* addr; };
  static Entry cache[64] = {};
  static std::mutex mu;
  int dev = 0;
  LL_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return LL_ERR_ARG;
  std::lock_guard<std::mutex> lock(mu);
  const CUcontext ctx = current_context();
  if (!cache[dev].addr || !ctx || cache[dev].ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    cache[dev] = Entry{current_context(), p};     // the lookup made the device's context current
  }
  *out = cache[dev].addr;
  return LL_OK;
}

}  // namespace

extern "C" int ll_mxfp4_gemm_noalloc(float* y, const float* x, const uint8_t* packed, const uint8_t* scales, int M,
                                     int K, int R, int64_t scale_stride, void* stream) {
  if (M <= 0 || K <= 0 || R <= 0 || K % 32 || scale_stride < K / 32 || scale_stride % 16) return LL_ERR_ARG;
  if (!y || !x || !packed || !scales) return LL_ERR_ARG;
  const size_t need = noalloc_layout(nullptr, M, K, nullptr);
  if (need > LL_NOALLOC_SCRATCH_BYTES) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
             "ll_mxfp4_gemm_noalloc: M=%d x K=%d needs %zu bytes of scratch, the static array holds %zu", M, K, need,
             (size_t)LL_NOALLOC_SCRATCH_BYTES);
    return LL_ERR_WORKSPACE;
  }
  LL_TRY(check_arch());
  void* base = nullptr;
  LL_TRY(scratch_address(&base));
  NoAllocLayout w;
  noalloc_layout(base, M, K, &w);
  LL_STREAM(stream);
  g_launch_count = 0;
  LL_TRY(reset_status(w.st, s));
  LL_TRY(launch_single_expert_chunks(w.chunks, w.n_chunks, M, kNoAllocNmax, s));
  LL_TRY(launch_prepare_beta(scales, nullptr, 1, R, K, scale_stride, w.beta, 0, s));
  const int Kp = (K + 63) / 64 * 64;
  LL_TRY(launch_rows_to_half(x, 0, nullptr, M, K, w.act, w.inv, s, Kp));
  CUtensorMap pk, sc, act[kNoAllocNmax / 16];
  LL_TRY(make_rowscale_maps(&pk, &sc, packed, scales, R, K, scale_stride));
  LL_TRY(make_act_maps(act, kNoAllocNmax / 16, w.act, M, Kp));
  GemmArgs a{};
  a.chunks = w.chunks;
  a.n_chunks = w.n_chunks;
  a.mtiles = (R + 127) / 128;
  a.K = K;
  a.e_rows = R;
  a.status = w.st;
  a.epi.row_scale_inv = w.inv;
  a.epi.beta = w.beta;
  a.epi.beta_col = 0;
  a.epi.P = M;
  a.epi.M = R;
  a.epi.Y = y;
  LL_TRY((launch_gemm<EPI_STORE, 1, 1, false, kNoAllocNmax>(&pk, &sc, act, a, s)));
  return read_status(w.st, s);
}
