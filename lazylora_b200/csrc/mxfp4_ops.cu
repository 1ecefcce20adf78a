// Drop-in MXFP4 kernels (device-pointer versions of lazy_lora/native/mxfp4_gemm.c) and the
// host plumbing every entry point shares.
#include <cuda_runtime.h>

#include "host_common.cuh"
#include "ops.cuh"

namespace ll {

thread_local char g_last_cuda_error[256] = "";
thread_local int g_launch_count = 0;
thread_local cudaEvent_t* g_prof_events = nullptr;
thread_local int g_prof_n = 0;
thread_local int g_prof_i = 0;
static thread_local cudaEvent_t g_prof_store[64];
thread_local cudaStream_t g_launch_stream = nullptr;
thread_local cudaEvent_t* g_lev = nullptr;
thread_local const char** g_lev_names = nullptr;
thread_local int g_lev_n = 0;
thread_local int g_lev_i = 0;
static thread_local cudaEvent_t g_lev_store[512];
static thread_local const char* g_lev_name_store[512];

DeviceInfo device_info() {
  static DeviceInfo cache[64];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = cache[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
  }
  return d;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_map_nd(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled unavailable");
    return LL_ERR_CUDA;
  }
  if (rank < 1 || rank > 5 || (reinterpret_cast<uintptr_t>(base) & 15)) return LL_ERR_ARG;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], estr[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] & 15) return LL_ERR_ARG;
      st[i] = strides_bytes[i];
    }
  }
  CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LL_ERR_ARG;
  }
  return LL_OK;
}

int make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0, uint64_t dim1,
                uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  const uint64_t dims[2] = {dim0, dim1};
  const uint32_t box[2] = {box0, box1};
  return make_map_nd(m, dt, base, 2, dims, &stride1_bytes, box, sw);
}

int set_smem_attr(const void* func, int bytes) {
  LL_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return LL_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("LL_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int reset_status(DevStatus* st, cudaStream_t s) {
  LL_CUDA(cudaMemsetAsync(st, 0, sizeof(DevStatus), s));
  return LL_OK;
}

int read_status(DevStatus* st, cudaStream_t s) {
  DevStatus h;
  LL_CUDA(cudaMemcpyAsync(&h, st, sizeof(DevStatus), cudaMemcpyDeviceToHost, s));
  LL_CUDA(cudaStreamSynchronize(s));
  if (h.code != 0) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "device status %d at site %d (info %d)", h.code,
             h.where, h.info);
    return h.code;
  }
  return LL_OK;
}

int check_arch() {
  const DeviceInfo d = device_info();
  if (d.major != 10) return LL_ERR_ARCH;
  return LL_OK;
}

// ------------------------------------------------------------------------- kernels

// out[R,K] = W (exact). One thread per packed byte pair of elements; 16 bytes per thread.
template <int OUT>  // 0 fp32, 1 bf16, 2 fp16
__global__ void k_dequant(void* out, const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                          int K, int R, int64_t sstride) {
  const int64_t groups = (int64_t)R * (K / 32);
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = gi / (K / 32);
    const int g = (int)(gi % (K / 32));
    const uint4 raw = *reinterpret_cast<const uint4*>(packed + r * (K / 2) + g * 16);
    const uint32_t b = scales[r * sstride + g];
    const float s = b >= 253u ? 0.f : ldexpf(1.f, (int)b - 127);
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    const int64_t o = r * K + (int64_t)g * 32;
#pragma unroll
    for (int wi = 0; wi < 4; wi++) {
      uint32_t h[4];
      decode8(words[wi], 0x3C003C00u /* fp16 1.0 splat */, h);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&h[j]));
        const float v0 = v.x * s, v1 = v.y * s;   // exact: a 2-significant-bit value times 2^e
        const int64_t idx = o + wi * 8 + j * 2;
        if (OUT == 0) {
          reinterpret_cast<float*>(out)[idx] = v0;
          reinterpret_cast<float*>(out)[idx + 1] = v1;
        } else if (OUT == 1) {
          reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v0);
          reinterpret_cast<__nv_bfloat16*>(out)[idx + 1] = __float2bfloat16_rn(v1);
        } else {
          reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v0);
          reinterpret_cast<__half*>(out)[idx + 1] = __float2half_rn(v1);
        }
      }
    }
  }
}

// beta[e*2 + col] = 140 - (largest scale byte < 253 of the expert's matrices), so that
// 6 * 2^(b - 127 + beta) <= 2^15 for every byte: fp16 holds each decoded weight exactly for
// bytes within 36 of that maximum. Matrices with no usable byte get beta 0.
__global__ void k_prepare_beta(const uint8_t* __restrict__ s_a, const uint8_t* __restrict__ s_b, int rows, int ngroups,
                               int64_t sstride, int32_t* beta, int col) {
  const int e = blockIdx.x;
  int mx = -1;
  for (const uint8_t* s : {s_a, s_b}) {
    if (!s) continue;
    const uint8_t* base = s + (int64_t)e * rows * sstride;
    for (int64_t i = threadIdx.x; i < (int64_t)rows * ngroups; i += blockDim.x) {
      const int v = base[(i / ngroups) * sstride + (i % ngroups)];
      if (v < 253 && v > mx) mx = v;
    }
  }
  __shared__ int red[32];
  for (int off = 16; off > 0; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    int m = -1;
    for (int i = 0; i < (int)(blockDim.x / 32); i++) m = max(m, red[i]);
    beta[e * 2 + col] = m < 0 ? 0 : 140 - m;
  }
}

// Row scaling into fp16: for each of `rows` output rows, src row = index ? index[row] : row,
// sigma = row_scale_exp(max|src row|); dst = fp16(src * 2^sigma); inv[row] = 2^-sigma.
// A row index < 0 yields a zero row. SRC: 0 fp32, 1 bf16. dst rows are ld >= K elements apart,
// columns K..ld-1 written as 0.
template <int SRC>
__global__ void k_rows_to_half(const void* __restrict__ src, const int* __restrict__ index, int rows, int K,
                               int ld, __half* __restrict__ dst, float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_next();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int sr = index ? index[row] : row;
  __shared__ float red[32];
  __shared__ float sh_scale;
  float mx = 0.f;
  if (sr >= 0) {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = SRC == 0 ? reinterpret_cast<const float*>(src)[(int64_t)sr * K + k]
                               : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[(int64_t)sr * K + k]);
      mx = fmaxf(mx, fabsf(v));
    }
  }
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); i++) m = fmaxf(m, red[i]);
    const int e = row_scale_exp(m);
    sh_scale = ldexpf(1.f, e);
    if (inv) inv[row] = ldexpf(1.f, -e);
  }
  __syncthreads();
  const float sc = sh_scale;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = 0.f;
    if (sr >= 0)
      v = SRC == 0 ? reinterpret_cast<const float*>(src)[(int64_t)sr * K + k]
                   : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[(int64_t)sr * K + k]);
    dst[(int64_t)row * ld + k] = __float2half_rn(v * sc);
  }
  for (int k = K + threadIdx.x; k < ld; k += blockDim.x) dst[(int64_t)row * ld + k] = __float2half_rn(0.f);
}

// The same, one pass: each thread holds up to 4 chunks of 8 values of the row in registers
// (16- or 32-byte loads, 16-byte stores), K % 8 == 0, ld % 8 == 0 and K <= 8 * 4 * blockDim.x.
template <int SRC>
__global__ void __launch_bounds__(256) k_rows_to_half_v(const void* __restrict__ src, const int* __restrict__ index,
                                                        int rows, int K, int ld, __half* __restrict__ dst,
                                                        float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_next();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int sr = index ? index[row] : row;
  const int nch = K / 8;
  float v[4][8];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int ch = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; j++) v[i][j] = 0.f;
    if (ch < nch && sr >= 0) {
      if (SRC == 0) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + (int64_t)sr * K) + 2 * ch;
        const float4 a = p[0], b = p[1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
      } else {
        const uint4 u = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src) + (int64_t)sr * K)[ch];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          v[i][2 * j] = f.x;
          v[i][2 * j + 1] = f.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[i][j]));
    }
  }
  __shared__ float red[32];
  __shared__ float sh_scale;
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); i++) m = fmaxf(m, red[i]);
    const int e = row_scale_exp(m);
    sh_scale = ldexpf(1.f, e);
    if (inv) inv[row] = ldexpf(1.f, -e);
  }
  __syncthreads();
  const float sc = sh_scale;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int ch = threadIdx.x + i * blockDim.x;
    if (ch >= nch) continue;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __half2 h = __floats2half2_rn(v[i][2 * j] * sc, v[i][2 * j + 1] * sc);
      o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(dst + (int64_t)row * ld)[ch] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int ch = nch + threadIdx.x; ch < ld / 8; ch += blockDim.x)
    reinterpret_cast<uint4*>(dst + (int64_t)row * ld)[ch] = make_uint4(0, 0, 0, 0);
}

// Transposed copy of an MXFP4 stack for the backward GEMMs. For every expert:
//   codes_t[c][r/2]  = the E2M1 codes of W[r][c], transposed (element 2j of a row still in
//                      the low nibble of byte j), and
//   scales_t[c/32][r] = fp16 of 2^(b - 127 + beta) for the scale byte b of (r, c/32): the
//                      multiplier of every element of that group, decode bias included
//                      (0 for bytes >= 253).
// One 64 x 64 element tile per block.
__global__ void k_transpose_mxfp4(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                  int64_t sstride, int R, int C, const int32_t* __restrict__ beta, int col,
                                  uint8_t* __restrict__ codes_t, __half* __restrict__ scales_t) {
  __shared__ uint8_t tile[64][65];
  const int e = blockIdx.z;
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const uint8_t* pe = packed + (int64_t)e * R * (C / 2);
  for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
    const int r = i / 32, b = i % 32;
    uint8_t v = 0;
    if (r0 + r < R && c0 + 2 * b < C) v = pe[(int64_t)(r0 + r) * (C / 2) + c0 / 2 + b];
    tile[r][2 * b] = v & 0x0F;
    tile[r][2 * b + 1] = v >> 4;
  }
  __syncthreads();
  uint8_t* te = codes_t + (int64_t)e * C * (R / 2);
  for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
    const int c = i / 32, j = i % 32;
    if (c0 + c < C && r0 + 2 * j < R)
      te[(int64_t)(c0 + c) * (R / 2) + r0 / 2 + j] = (uint8_t)(tile[2 * j][c] | (tile[2 * j + 1][c] << 4));
  }
  const int bias = beta ? beta[e * 2 + col] : 0;
  const uint8_t* se = scales + (int64_t)e * R * sstride;
  __half* ste = scales_t + (int64_t)e * (C / 32) * R;
  for (int i = threadIdx.x; i < 2 * 64; i += blockDim.x) {
    const int g = i / 64, r = i % 64;
    const int cg = c0 / 32 + g;
    if (r0 + r < R && cg * 32 < C) {
      const uint32_t bits = e8m0_to_half_bits(se[(int64_t)(r0 + r) * sstride + cg], bias);
      ste[(int64_t)cg * R + r0 + r] = __ushort_as_half((unsigned short)bits);
    }
  }
}

__global__ void k_single_expert_chunks(Chunk* chunks, int* n_chunks, int M, int nmax) {
  const int n = (M + nmax - 1) / nmax;
  for (int i = threadIdx.x; i < n; i += blockDim.x) chunks[i] = Chunk{0, i * nmax, min(nmax, M - i * nmax), 0};
  if (threadIdx.x == 0) *n_chunks = n;
}

// --------------------------------------------------------------------- launchers

int launch_prepare_beta(const uint8_t* s_a, const uint8_t* s_b, int E, int rows, int cols, int64_t sstride,
                        int32_t* beta, int col, cudaStream_t s) {
  k_prepare_beta<<<E, 256, 0, s>>>(s_a, s_b, rows, cols / 32, sstride, beta, col);
  return check_launch("k_prepare_beta");
}

int launch_transpose_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t sstride, int E, int R, int C,
                           const int32_t* beta, int col, uint8_t* codes_t, __half* scales_t, cudaStream_t s) {
  dim3 grid((C + 63) / 64, (R + 63) / 64, E);
  k_transpose_mxfp4<<<grid, 256, 0, s>>>(packed, scales, sstride, R, C, beta, col, codes_t, scales_t);
  return check_launch("k_transpose_mxfp4");
}

int launch_single_expert_chunks(Chunk* chunks, int* n_chunks, int M, int nmax, cudaStream_t s) {
  k_single_expert_chunks<<<1, 128, 0, s>>>(chunks, n_chunks, M, nmax);
  return check_launch("k_single_expert_chunks");
}

int launch_rows_to_half(const void* src, int src_dtype, const int* index, int rows, int K, __half* dst, float* inv,
                        cudaStream_t s, int ld) {
  if (rows <= 0) return LL_OK;
  if (ld < 0) ld = K;
  if (ld < K) return LL_ERR_ARG;
  const bool vec = K % 8 == 0 && ld % 8 == 0 && K <= 8 * 4 * 256 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dst) % 16 == 0;
  auto kern = vec ? (src_dtype == 0 ? k_rows_to_half_v<0> : k_rows_to_half_v<1>)
                  : (src_dtype == 0 ? k_rows_to_half<0> : k_rows_to_half<1>);
  return launch_pdl("k_rows_to_half", kern, dim3(rows), dim3(256), 0, s, src, index, rows, K, ld, dst, inv);
}

// The same conversion, one block per source token: the token's row is read and its scale found
// once, then written to each of its k pair rows (tok_pos[t * k + j], -1 for none). The pair
// rows match k_rows_to_half_v's bit for bit; rows no token maps to are left as they are.
template <int SRC>
__global__ void __launch_bounds__(256) k_token_rows_to_half(const void* __restrict__ src, const int* __restrict__ tok_pos,
                                                            int T, int k, int K, __half* __restrict__ dst,
                                                            float* __restrict__ inv) {
  pdl_wait();
  pdl_launch_next();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int nch = K / 8;
  float v[4][8];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int ch = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; j++) v[i][j] = 0.f;
    if (ch < nch) {
      if (SRC == 0) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + (int64_t)t * K) + 2 * ch;
        const float4 a = p[0], b = p[1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
      } else {
        const uint4 u = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src) + (int64_t)t * K)[ch];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          v[i][2 * j] = f.x;
          v[i][2 * j + 1] = f.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) mx = fmaxf(mx, fabsf(v[i][j]));
    }
  }
  __shared__ float red[32];
  __shared__ float sh_scale, sh_inv;
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); i++) m = fmaxf(m, red[i]);
    const int e = row_scale_exp(m);
    sh_scale = ldexpf(1.f, e);
    sh_inv = ldexpf(1.f, -e);
  }
  __syncthreads();
  const float sc = sh_scale;
  uint4 o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint32_t h2[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __half2 h = __floats2half2_rn(v[i][2 * j] * sc, v[i][2 * j + 1] * sc);
      h2[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    o[i] = make_uint4(h2[0], h2[1], h2[2], h2[3]);
  }
  for (int j = 0; j < k; j++) {
    const int p = tok_pos[(int64_t)t * k + j];
    if (p < 0) continue;
    if (threadIdx.x == 0) inv[p] = sh_inv;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int ch = threadIdx.x + i * blockDim.x;
      if (ch < nch) reinterpret_cast<uint4*>(dst + (int64_t)p * K)[ch] = o[i];
    }
  }
}

int launch_token_rows_to_half(const void* src, int src_dtype, const int* perm_token, const int* tok_pos, int T, int k,
                              int K, __half* dst, float* inv, cudaStream_t s) {
  if (T <= 0) return LL_OK;
  const bool vec = K % 8 == 0 && K <= 8 * 4 * 256 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dst) % 16 == 0;
  if (!vec) return launch_rows_to_half(src, src_dtype, perm_token, T * k, K, dst, inv, s);
  return launch_pdl("k_rows_to_half", src_dtype == 0 ? k_token_rows_to_half<0> : k_token_rows_to_half<1>, dim3(T),
                    dim3(256), 0, s, src, tok_pos, T, k, K, dst, inv);
}


}  // namespace ll

using namespace ll;

static constexpr int kDropInNmax = 128;

struct DropInWs {
  DevStatus* st;
  Chunk* chunks;
  int* n_chunks;
  int32_t* beta;
  float* inv;
  __half* act;
  uint8_t* codes_t;    // gemm_t: transposed codes [K][R/2]
  __half* scales_t;    // gemm_t: fp16 column multipliers [K/32][R]
};

// rows: activation rows (M); width: activation row length; R, K: the weight's shape
static size_t dropin_layout(void* base, int rows, int width, int R, int K, DropInWs* w) {
  Carver c(base);
  DropInWs t;
  t.st = c.take<DevStatus>(1);
  t.chunks = c.take<Chunk>((rows + kDropInNmax - 1) / kDropInNmax + 1);
  t.n_chunks = c.take<int>(1);
  t.beta = c.take<int32_t>(2);
  t.inv = c.take<float>(rows);
  t.act = c.take<__half>((size_t)rows * ((width + 63) / 64 * 64));   // rows padded to whole 64-K halves
  t.codes_t = c.take<uint8_t>((size_t)R * K / 2);
  t.scales_t = c.take<__half>((size_t)(K / 32) * R);
  if (w) *w = t;
  return c.off + 256;
}

extern "C" {

const char* ll_status_string(int status) {
  switch (status) {
    case LL_OK: return "ok";
    case LL_ERR_ARG: return "invalid argument (shape, stride, alignment or pointer)";
    case LL_ERR_CUDA: return "CUDA runtime error";
    case LL_ERR_TIMEOUT: return "device-side wait timed out";
    case LL_ERR_WORKSPACE: return "workspace too small";
    case LL_ERR_RANGE: return "value outside the exactly representable range";
    case LL_ERR_ARCH: return "device is not sm_100 (B200)";
    case LL_ERR_IO: return "host file read failed";
    default: return "unknown status";
  }
}

const char* ll_last_cuda_error(void) { return g_last_cuda_error; }

int ll_last_launch_count(void) { return g_launch_count; }

int ll_profile_launch_events(void* const* events, int n) {
  if (n < 0 || n > 512 || (n > 0 && !events)) return LL_ERR_ARG;
  for (int i = 0; i < n; i++) g_lev_store[i] = static_cast<cudaEvent_t>(events[i]);
  g_lev = n > 0 ? g_lev_store : nullptr;
  g_lev_names = g_lev_name_store;
  g_lev_n = n;
  g_lev_i = 0;
  return LL_OK;
}

int ll_profile_launch_recorded(void) { return g_lev_i; }

const char* ll_profile_launch_name(int i) { return (i >= 0 && i < g_lev_i) ? g_lev_name_store[i] : ""; }

int ll_mxfp4_threads(void) { return device_info().sms; }

int ll_profile_gemm_events(void* const* events, int n) {
  if (n < 0 || n > 64 || (n > 0 && !events)) return LL_ERR_ARG;
  for (int i = 0; i < n; i++) g_prof_store[i] = static_cast<cudaEvent_t>(events[i]);
  g_prof_events = n > 0 ? g_prof_store : nullptr;
  g_prof_n = n;
  g_prof_i = 0;
  return LL_OK;
}

size_t ll_mxfp4_workspace_bytes(int M, int K, int R) {
  return dropin_layout(nullptr, M, K > R ? K : R, R, K, nullptr);
}

int ll_mxfp4_dequant(void* out, const uint8_t* packed, const uint8_t* scales, int K, int R, int64_t scale_stride,
                     int out_dtype, void* stream) {
  if (K <= 0 || R <= 0 || K % 32 || !out || !packed || !scales || scale_stride < K / 32) return LL_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(packed) & 15)) return LL_ERR_ARG;
  LL_STREAM(stream);
  const int64_t groups = (int64_t)R * (K / 32);
  const int grid = (int)std::min<int64_t>((groups + 255) / 256, 148 * 16);
  if (out_dtype == 0) k_dequant<0><<<grid, 256, 0, s>>>(out, packed, scales, K, R, scale_stride);
  else if (out_dtype == 1) k_dequant<1><<<grid, 256, 0, s>>>(out, packed, scales, K, R, scale_stride);
  else if (out_dtype == 2) k_dequant<2><<<grid, 256, 0, s>>>(out, packed, scales, K, R, scale_stride);
  else return LL_ERR_ARG;
  return check_launch("k_dequant");
}

int ll_mxfp4_gemm(float* y, const float* x, const uint8_t* packed, const uint8_t* scales, int M, int K, int R,
                  int64_t scale_stride, void* ws, size_t ws_bytes, void* stream) {
  if (M <= 0 || K <= 0 || R <= 0 || K % 32 || scale_stride < K / 32 || scale_stride % 16) return LL_ERR_ARG;
  if (!y || !x || !packed || !scales || !ws) return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_mxfp4_workspace_bytes(M, K, R)) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  DropInWs w;
  dropin_layout(ws, M, K > R ? K : R, R, K, &w);
  g_launch_count = 0;
  LL_TRY(reset_status(w.st, s));
  k_single_expert_chunks<<<1, 128, 0, s>>>(w.chunks, w.n_chunks, M, kDropInNmax);
  LL_TRY(check_launch("k_single_expert_chunks"));
  LL_TRY(launch_prepare_beta(scales, nullptr, 1, R, K, scale_stride, w.beta, 0, s));
  const int Kp = (K + 63) / 64 * 64;
  LL_TRY(launch_rows_to_half(x, 0, nullptr, M, K, w.act, w.inv, s, Kp));
  CUtensorMap pk, sc, act[kDropInNmax / 16];
  LL_TRY(make_rowscale_maps(&pk, &sc, packed, scales, R, K, scale_stride));
  LL_TRY(make_act_maps(act, kDropInNmax / 16, w.act, M, Kp));
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
  LL_TRY((launch_gemm<EPI_STORE, 1, 1, false, kDropInNmax>(&pk, &sc, act, a, s)));
  return read_status(w.st, s);
}

int ll_mxfp4_gemm_t(float* y, const float* dy, const uint8_t* packed, const uint8_t* scales, int M, int K, int R,
                    int64_t scale_stride, void* ws, size_t ws_bytes, void* stream) {
  if (M <= 0 || K <= 0 || R <= 0 || K % 32 || R % 32 || scale_stride < K / 32 || scale_stride % 16) return LL_ERR_ARG;
  if (!y || !dy || !packed || !scales || !ws) return LL_ERR_ARG;
  LL_TRY(check_arch());
  if (ws_bytes < ll_mxfp4_workspace_bytes(M, K, R)) return LL_ERR_WORKSPACE;
  LL_STREAM(stream);
  DropInWs w;
  dropin_layout(ws, M, K > R ? K : R, R, K, &w);
  g_launch_count = 0;
  LL_TRY(reset_status(w.st, s));
  k_single_expert_chunks<<<1, 128, 0, s>>>(w.chunks, w.n_chunks, M, kDropInNmax);
  LL_TRY(check_launch("k_single_expert_chunks"));
  LL_TRY(launch_prepare_beta(scales, nullptr, 1, R, K, scale_stride, w.beta, 0, s));
  const int Rp = (R + 63) / 64 * 64;
  LL_TRY(launch_rows_to_half(dy, 0, nullptr, M, R, w.act, w.inv, s, Rp));
  // the backward orientation reads a transposed copy: codes [K][R/2], fp16 multipliers [K/32][R]
  LL_TRY(launch_transpose_mxfp4(packed, scales, scale_stride, 1, R, K, w.beta, 0, w.codes_t, w.scales_t, s));
  CUtensorMap pk, sc, act[kDropInNmax / 16];
  LL_TRY(make_colscale_maps(&pk, &sc, w.codes_t, w.scales_t, K, R));
  LL_TRY(make_act_maps(act, kDropInNmax / 16, w.act, M, Rp));
  GemmArgs a{};
  a.chunks = w.chunks;
  a.n_chunks = w.n_chunks;
  a.mtiles = (K + 127) / 128;
  a.K = R;
  a.e_rows = K;
  a.status = w.st;
  a.epi.row_scale_inv = w.inv;
  a.epi.beta = w.beta;
  a.epi.beta_col = 0;
  a.epi.P = M;
  a.epi.M = K;
  a.epi.Y = y;
  LL_TRY((launch_gemm<EPI_ACCUM, 1, 1, true, kDropInNmax>(&pk, &sc, act, a, s)));
  return read_status(w.st, s);
}

}  // extern "C"
