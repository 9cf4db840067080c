// MXFP4 (E2M1 values, one E8M0 power-of-two scale per 32 values) -> bf16, for frozen expert weights
// kept packed in HBM (4.25 bits per weight instead of 16) and expanded per layer just in time.
//
// Layout (the released DeepSeek-V4.1 expert layout): rows of `cols` values; each byte holds two
// codes, low nibble first; scale[r, b] applies to values [32 b, 32 b + 32) of row r and encodes
// 2^(s - 127). One thread expands one 32-value block: a 16-byte load of codes, one scale byte,
// four 16-byte stores.
#include "common.cuh"

namespace tdsv {

namespace {

__device__ __forceinline__ float e2m1(uint32_t code) {
  // magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 (OCP microscaling E2M1); bit 3 is the sign
  const uint32_t m = code & 7u;
  // m < 4: 0.5 m; m = 4..7: 2, 3, 4, 6 = (2 or 4) x (1 or 1.5)
  const float mag = m < 4u ? 0.5f * static_cast<float>(m)
                           : static_cast<float>(2u << ((m >> 1) & 1u)) * ((m & 1u) ? 1.5f : 1.f);
  return (code & 8u) ? -mag : mag;
}

__global__ void fp4_dequant_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scale,
                                   __nv_bfloat16* __restrict__ out, int64_t blocks) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < blocks; b += stride) {
    const uint4 raw = reinterpret_cast<const uint4*>(packed)[b];
    const float s = ldexpf(1.f, static_cast<int>(scale[b]) - 127);
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    __nv_bfloat16* dst = out + b * 32;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = e2m1((words[w] >> (4 * i)) & 0xFu) * s;
      store_bf16x8(dst + w * 8, v);
    }
  }
}

}  // namespace

// packed uint8 [..., cols / 2], scale uint8 [..., cols / 32] -> bf16 [..., cols]
at::Tensor fp4_dequant(const at::Tensor& packed, const at::Tensor& scale) {
  check_cuda_tensor(packed, "packed");
  check_cuda_tensor(scale, "scale");
  TDSV_CHECK(packed.scalar_type() == at::kByte && scale.scalar_type() == at::kByte, "fp4_dequant: uint8 codes/scales");
  const int64_t cols = packed.size(-1) * 2;
  TDSV_CHECK(cols % 32 == 0 && scale.size(-1) * 32 == cols && packed.numel() / packed.size(-1) == scale.numel() / scale.size(-1),
             "fp4_dequant: one scale per 32 values of every row");
  auto sizes = packed.sizes().vec();
  sizes.back() = cols;
  auto out = at::empty(sizes, packed.options().dtype(at::kBFloat16));
  const int64_t blocks = scale.numel();
  if (blocks == 0) return out;
  c10::cuda::CUDAGuard guard(packed.device());
  const int threads = 256;
  const int64_t want = (blocks + threads - 1) / threads;
  const int grid = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * 8));
  fp4_dequant_kernel<<<grid, threads, 0, stream()>>>(packed.data_ptr<uint8_t>(), scale.data_ptr<uint8_t>(),
                                                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), blocks);
  TDSV_LAUNCH_CHECK();
  return out;
}

}  // namespace tdsv
