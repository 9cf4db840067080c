// Block fake quantization of activations, matching how an FP8 / FP4 KV cache stores them
// (quantize, then dequantize back to the input dtype). Used by the DeepSeek-V4 scoring path so
// the learner sees the same cached values as the sampler (reference:
// dsv41_train/rl/_native_runtime/c3868011979ca/dsv41_train/models/dsv4/quantization.py).
//
//   kind 0  fp8        blocks of 32, scale = 2^ceil(log2(max(amax, 1e-4) / 448)), E4M3 values
//   kind 1  fp4_index  blocks of 32, scale = 2^ceil(log2(max(amax, 6 * 2^-126) / 6)), E2M1 values
//   kind 2  fp4_kv     blocks of 16, scale = E4M3(max(amax, 6 * 2^-9) / 6), E2M1 values
//
// E2M1 rounds to nearest with ties to the even code (magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; the even
// codes are 0, 1, 2, 4). One lane per value; the lanes of a block reduce the maximum by shuffles.
#include "common.cuh"

#include <cuda_fp8.h>

namespace tdsv {

namespace {

__device__ __forceinline__ float pow2_ceil(float v) {  // v > 0, normal
  const int bits = __float_as_int(v);
  const int e = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0 ? 1 : 0);
  return ldexpf(1.f, e);
}

__device__ __forceinline__ float e4m3_round(float v) {
  const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(q, __NV_E4M3)));
}

__device__ __forceinline__ float e2m1_round(float v) {  // |v| <= 6
  const float a = fabsf(v);
  // ties: 0.25 -> 0, 0.75 -> 1, 1.25 -> 1, 1.75 -> 2, 2.5 -> 2, 3.5 -> 4, 5 -> 4
  float m;
  if (a <= 0.25f) m = 0.f;
  else if (a < 0.75f) m = 0.5f;
  else if (a <= 1.25f) m = 1.f;
  else if (a < 1.75f) m = 1.5f;
  else if (a <= 2.5f) m = 2.f;
  else if (a < 3.5f) m = 3.f;
  else if (a <= 5.f) m = 4.f;
  else m = 6.f;
  return copysignf(m, v);
}

template <typename T, int B>
__global__ void fake_quant_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n, int kind) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // n is a multiple of B and the grid covers whole blocks per iteration (blockDim % 32 == 0)
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i - (threadIdx.x & 31) < n;
       i += stride) {
    const bool live = i < n;
    const float v = live ? to_float(x[i]) : 0.f;
    float amax = fabsf(v);
#pragma unroll
    for (int m = B / 2; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m, B));
    float q;
    if (kind == 0) {
      const float scale = pow2_ceil(fmaxf(amax, 1e-4f) / 448.f);
      q = e4m3_round(fminf(fmaxf(v / scale, -448.f), 448.f)) * scale;
    } else {
      const float scale = kind == 1 ? pow2_ceil(fmaxf(amax, 6.f * 0x1p-126f) / 6.f)
                                    : e4m3_round(fmaxf(amax, 6.f * 0x1p-9f) / 6.f);
      q = e2m1_round(fminf(fmaxf(v / scale, -6.f), 6.f)) * scale;
    }
    if (live) y[i] = from_float<T>(q);
  }
}

}  // namespace

// kind: 0 fp8 (blocks of 32), 1 fp4_index (blocks of 32), 2 fp4_kv (blocks of 16, E4M3 scales).
// Blocks run along the last dimension; a last dimension that is not a multiple of the block size
// returns the input unchanged.
at::Tensor cache_fake_quant(const at::Tensor& x, int64_t kind) {
  check_cuda_tensor(x, "fake-quant input");
  TDSV_CHECK(kind >= 0 && kind <= 2, "fake-quant kind must be 0 (fp8), 1 (fp4_index) or 2 (fp4_kv)");
  TDSV_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "fake-quant input: bf16 or fp32");
  const int block = kind == 2 ? 16 : 32;
  if (x.dim() == 0 || x.size(-1) % block != 0) return x;
  auto y = at::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return y;
  c10::cuda::CUDAGuard guard(x.device());
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + threads - 1) / threads, num_sms() * 16));
  if (x.scalar_type() == at::kBFloat16) {
    auto* in = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    auto* out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
    if (block == 16) fake_quant_kernel<__nv_bfloat16, 16><<<grid, threads, 0, stream()>>>(in, out, n, static_cast<int>(kind));
    else fake_quant_kernel<__nv_bfloat16, 32><<<grid, threads, 0, stream()>>>(in, out, n, static_cast<int>(kind));
  } else {
    if (block == 16) fake_quant_kernel<float, 16><<<grid, threads, 0, stream()>>>(x.data_ptr<float>(), y.data_ptr<float>(), n, static_cast<int>(kind));
    else fake_quant_kernel<float, 32><<<grid, threads, 0, stream()>>>(x.data_ptr<float>(), y.data_ptr<float>(), n, static_cast<int>(kind));
  }
  TDSV_LAUNCH_CHECK();
  return y;
}

}  // namespace tdsv
