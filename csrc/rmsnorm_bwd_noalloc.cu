// RMSNorm backward with its weight-gradient scratch in a fixed file-scope device array, for
// callers that cannot allocate device memory (the header tdsv_noalloc.h says who and why).
// No counterpart in the reference implementation.
//
// Work split: at most TDSV_NOALLOC_MAX_PARTS blocks; block b takes the 32-row chunks
// b, b + parts, b + 2 * parts, ... and keeps its weight-gradient partial for all h columns in
// registers (256 threads x 8 columns x up to 4 passes), writing it once to scratch row b.  A
// second kernel sums the `parts` scratch rows per column in fixed order.  Every scratch row the
// sum reads is written by the first kernel of the same call (blocks without a chunk write
// zeros), so nothing in the array needs clearing between calls.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "tdsv_noalloc.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 32;  // rows per chunk
constexpr int kCols = kThreads * 8;
constexpr int kPasses = TDSV_NOALLOC_MAX_HIDDEN / kCols;
constexpr int kMaxDevices = 64;

// The scratch.  In host code `g_noalloc_partial` is only a host-side stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress on the current device.
static __device__ __align__(256) float g_noalloc_partial[TDSV_NOALLOC_MAX_PARTS * TDSV_NOALLOC_MAX_HIDDEN];

std::atomic<float*> g_scratch[kMaxDevices];
std::mutex g_setup_mutex;

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ float wload(const float* w, int c) { return w[c]; }
__device__ __forceinline__ float wload(const __nv_bfloat16* w, int c) { return __bfloat162float(w[c]); }

template <typename WT>
__global__ void __launch_bounds__(kThreads) rmsnorm_bwd_parts_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
    const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx, float* __restrict__ partial, int64_t rows,
    int h) {
  __shared__ float dots[kRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunks = (rows + kRows - 1) / kRows;
  float acc[kPasses][8];
#pragma unroll
  for (int p = 0; p < kPasses; ++p)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[p][i] = 0.f;
  for (int64_t chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x) {
    const int64_t row0 = chunk * kRows;
    for (int rr = warp; rr < kRows; rr += kWarps) {  // per-row <w * dy, x>
      const int64_t row = row0 + rr;
      float dot = 0.f;
      if (row < rows) {
        for (int c = lane * 8; c < h; c += 256) {
          float g[8], v[8];
          load8(dy + row * h + c, g);
          load8(x + row * h + c, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) dot += wload(w, c + i) * g[i] * v[i];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (lane == 0) dots[rr] = dot;
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int c0 = p * kCols + threadIdx.x * 8;
      if (c0 >= h) continue;
      float wv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) wv[i] = wload(w, c0 + i);
      for (int rr = 0; rr < kRows; ++rr) {
        const int64_t row = row0 + rr;
        if (row >= rows) break;
        const float r = rstd[row];
        const float coef = dots[rr] * r * r * r / static_cast<float>(h);
        float g[8], v[8], o[8];
        load8(dy + row * h + c0, g);
        load8(x + row * h + c0, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = r * wv[i] * g[i] - coef * v[i];
          acc[p][i] += g[i] * __bfloat162float(__float2bfloat16_rn(v[i] * r));
        }
        store8(dx + row * h + c0, o);
      }
    }
    __syncthreads();  // dots[] is rewritten by the next chunk
  }
  if (partial == nullptr) return;
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int c0 = p * kCols + threadIdx.x * 8;
    if (c0 >= h) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i) partial[static_cast<int64_t>(blockIdx.x) * h + c0 + i] = acc[p][i];
  }
}

__global__ void parts_sum_kernel(const float* __restrict__ partial, float* __restrict__ out, int parts, int h) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= h) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[static_cast<int64_t>(p) * h + c];
  out[c] = s;
}

int fail(int code, const char* what) {
  std::fprintf(stderr, "tdsv_rmsnorm_bwd_noalloc: %s\n", what);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  std::fprintf(stderr, "tdsv_rmsnorm_bwd_noalloc: %s: %s\n", what, cudaGetErrorString(err));
  return TDSV_NOALLOC_ECUDA;
}

// Device address of the scratch array on the current device, looked up once per device.
int scratch_for_current_device(float** out) {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice failed");
  if (device < 0 || device >= kMaxDevices) return fail(TDSV_NOALLOC_EINVAL, "device ordinal out of range");
  float* ptr = g_scratch[device].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    ptr = g_scratch[device].load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      err = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_partial);
      if (err != cudaSuccess || ptr == nullptr) return cuda_fail(err, "cudaGetSymbolAddress of the scratch failed");
      g_scratch[device].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return TDSV_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int tdsv_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, int weight_is_bf16, const float* rstd, void* dx, float* dw,
    int64_t rows, int h, void* stream) {
  if (rows < 0 || h <= 0 || h % 8 != 0) return fail(TDSV_NOALLOC_EINVAL, "rows >= 0 and h a positive multiple of 8");
  if (h > TDSV_NOALLOC_MAX_HIDDEN)
    return fail(TDSV_NOALLOC_ETOOBIG, "h exceeds TDSV_NOALLOC_MAX_HIDDEN (8192), the scratch array's row width");
  if (rows > 0 && (dy == nullptr || x == nullptr || w == nullptr || rstd == nullptr || dx == nullptr))
    return fail(TDSV_NOALLOC_EINVAL, "null input or output pointer");
  if (!aligned16(dy) || !aligned16(x) || !aligned16(dx))
    return fail(TDSV_NOALLOC_EINVAL, "dy, x and dx must be 16-byte aligned");
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != TDSV_NOALLOC_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (dw != nullptr) {
      const cudaError_t err = cudaMemsetAsync(dw, 0, sizeof(float) * static_cast<size_t>(h), s);
      if (err != cudaSuccess) return cuda_fail(err, "zeroing dw failed");
    }
    return TDSV_NOALLOC_OK;
  }
  const int64_t chunks = (rows + kRows - 1) / kRows;
  const int parts = static_cast<int>(chunks < TDSV_NOALLOC_MAX_PARTS ? chunks : TDSV_NOALLOC_MAX_PARTS);
  float* partial = dw != nullptr ? scratch : nullptr;
  const __nv_bfloat16* dyp = static_cast<const __nv_bfloat16*>(dy);
  const __nv_bfloat16* xp = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* dxp = static_cast<__nv_bfloat16*>(dx);
  if (weight_is_bf16) {
    rmsnorm_bwd_parts_kernel<__nv_bfloat16><<<parts, kThreads, 0, s>>>(
        dyp, xp, static_cast<const __nv_bfloat16*>(w), rstd, dxp, partial, rows, h);
  } else {
    rmsnorm_bwd_parts_kernel<float><<<parts, kThreads, 0, s>>>(dyp, xp, static_cast<const float*>(w), rstd, dxp,
                                                                partial, rows, h);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, "kernel launch failed");
  if (dw != nullptr) {
    parts_sum_kernel<<<(h + 255) / 256, 256, 0, s>>>(scratch, dw, parts, h);
    err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "kernel launch failed");
  }
  return TDSV_NOALLOC_OK;
}
