// RMSNorm forward/backward (memory-bound; one warp per row, 16-byte vector accesses).
//
// Semantics follow the reference modules (dsv41_train/models/qwen/model.py:45-57 and
// dsv41_train/models/dsv4/attention/module.py:20-30): the statistics are fp32, the normalised
// row is rounded to the activation dtype and only then multiplied by the weight:
//     y = w * bf16(x * rsqrt(mean(x^2) + eps))
// The backward treats that intermediate rounding as identity and reduces the weight gradient
// deterministically (per-block partials, then a fixed-order column sum).
#include "common.cuh"

namespace tdsv {

namespace {

constexpr int kWarps = 8;

template <typename WT>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int64_t rows,
                                   int h, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + row * h;
  __nv_bfloat16* yr = y + row * h;
  float ss = 0.f;
  for (int c = lane * 8; c < h; c += 256) {
    float v[8];
    load_bf16x8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(h) + eps);
  if (lane == 0 && rstd_out != nullptr) rstd_out[row] = r;
  for (int c = lane * 8; c < h; c += 256) {
    float v[8], o[8];
    load_bf16x8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float n = bf2f(f2bf(v[i] * r));
      o[i] = to_float<WT>(w[c + i]) * n;
    }
    store_bf16x8(yr + c, o);
  }
}

// Block handles kRowsPerBlock rows; each thread owns 8 columns per pass of 2048 columns.
constexpr int kRowsPerBlock = 32;

template <typename WT>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const WT* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_partial, int64_t rows,
                                   int h) {
  __shared__ float dots[kRowsPerBlock];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock;
  // Phase A: per-row dot(w*dy, x).
  for (int rr = warp; rr < kRowsPerBlock; rr += kWarps) {
    const int64_t row = row0 + rr;
    float dot = 0.f;
    if (row < rows) {
      for (int c = lane * 8; c < h; c += 256) {
        float g[8], v[8];
        load_bf16x8(dy + row * h + c, g);
        load_bf16x8(x + row * h + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += to_float<WT>(w[c + i]) * g[i] * v[i];
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) dots[rr] = dot;
  }
  __syncthreads();
  // Phase B: dx and the weight-gradient partial for this block of rows.
  for (int c0 = threadIdx.x * 8; c0 < h; c0 += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = to_float<WT>(w[c0 + i]);
    for (int rr = 0; rr < kRowsPerBlock; ++rr) {
      const int64_t row = row0 + rr;
      if (row >= rows) break;
      const float r = rstd[row];
      const float coef = dots[rr] * r * r * r / static_cast<float>(h);
      float g[8], v[8], o[8];
      load_bf16x8(dy + row * h + c0, g);
      load_bf16x8(x + row * h + c0, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i] = r * wv[i] * g[i] - coef * v[i];
        acc[i] += g[i] * bf2f(f2bf(v[i] * r));
      }
      store_bf16x8(dx + row * h + c0, o);
    }
    if (dw_partial != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) dw_partial[static_cast<int64_t>(blockIdx.x) * h + c0 + i] = acc[i];
    }
  }
}

// Fixed-order column sum of [parts, h] fp32 partials.
__global__ void column_sum_kernel(const float* __restrict__ partial, float* __restrict__ out, int parts, int h) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= h) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[static_cast<int64_t>(p) * h + c];
  out[c] = s;
}

}  // namespace

std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, double eps) {
  check_cuda_tensor(x, "x");
  check_cuda_tensor(w, "w");
  TDSV_CHECK(x.scalar_type() == at::kBFloat16, "rmsnorm: x must be bf16");
  const int h = static_cast<int>(x.size(-1));
  TDSV_CHECK(h % 8 == 0, "rmsnorm: hidden size must be a multiple of 8");
  TDSV_CHECK(w.numel() == h, "rmsnorm: weight size mismatch");
  const int64_t rows = x.numel() / h;
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, rstd};
  const dim3 grid((rows + kWarps - 1) / kWarps);
  c10::cuda::CUDAGuard guard(x.device());
  if (w.scalar_type() == at::kFloat) {
    rmsnorm_fwd_kernel<float><<<grid, kWarps * 32, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), rows, h, static_cast<float>(eps));
  } else {
    TDSV_CHECK(w.scalar_type() == at::kBFloat16, "rmsnorm: weight must be fp32 or bf16");
    rmsnorm_fwd_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), rows, h, static_cast<float>(eps));
  }
  TDSV_LAUNCH_CHECK();
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                    const at::Tensor& rstd, bool need_dw) {
  check_cuda_tensor(dy, "dy");
  check_cuda_tensor(x, "x");
  check_cuda_tensor(w, "w");
  check_cuda_tensor(rstd, "rstd");
  const int h = static_cast<int>(x.size(-1));
  const int64_t rows = x.numel() / h;
  auto dx = at::empty_like(x);
  auto dw = at::zeros({h}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dw};
  const int blocks = static_cast<int>((rows + kRowsPerBlock - 1) / kRowsPerBlock);
  at::Tensor partial;
  if (need_dw) partial = at::empty({blocks, h}, x.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(x.device());
  const int threads = 256;
  if (w.scalar_type() == at::kFloat) {
    rmsnorm_bwd_kernel<float><<<blocks, threads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        w.data_ptr<float>(), rstd.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()),
        need_dw ? partial.data_ptr<float>() : nullptr, rows, h);
  } else {
    rmsnorm_bwd_kernel<__nv_bfloat16><<<blocks, threads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), need_dw ? partial.data_ptr<float>() : nullptr, rows, h);
  }
  TDSV_LAUNCH_CHECK();
  if (need_dw) {
    column_sum_kernel<<<(h + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                            blocks, h);
    TDSV_LAUNCH_CHECK();
  }
  return {dx, dw};
}

// Fixed-order sum over the leading dimension of a [parts, n] fp32 tensor.
at::Tensor column_sum(const at::Tensor& partial) {
  check_cuda_tensor(partial, "partial");
  TDSV_CHECK(partial.scalar_type() == at::kFloat && partial.dim() == 2, "column_sum: [parts, n] fp32");
  const int parts = static_cast<int>(partial.size(0));
  const int n = static_cast<int>(partial.size(1));
  auto out = at::empty({n}, partial.options());
  if (n == 0) return out;
  c10::cuda::CUDAGuard guard(partial.device());
  column_sum_kernel<<<(n + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), out.data_ptr<float>(), parts,
                                                          n);
  TDSV_LAUNCH_CHECK();
  return out;
}

}  // namespace tdsv
