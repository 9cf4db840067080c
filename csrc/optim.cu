// Fused optimizer updates over flat parameter buffers.
//
// adamw_step implements torch.optim.AdamW (decoupled weight decay, bias-corrected moments) on an
// fp32 master buffer, reading fp32 or bf16 gradients, keeping the moments in fp32 or bf16, and
// writing the bf16 compute copy of the parameters in the same pass. An optional device scalar
// multiplies the gradient (global-norm clipping coefficient, 1/world, loss-scale undo) without a
// host synchronisation.
//
// sgd_step implements the reference's SGD-in-backward update (dsv41_train/optim.py:13-82): plain
// SGD on an fp32 master (or directly on the parameter), with a finite flag raised per launch.
//
// grad_sq_norm writes per-block partial sums of squares; the caller reduces them in fixed order.
#include "common.cuh"

namespace tdsv {

namespace {

// Four consecutive elements of T as one vector access (16 B for fp32, 8 B for bf16).
template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  using type = float4;
  __device__ static void load(const float* p, float (&o)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
  __device__ static void store(float* p, const float (&o)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&o)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
  __device__ static void store(__nv_bfloat16* p, const float (&o)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(o[2], o[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t*>(&a);
    raw.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
  }
};

// Element-wise AdamW; `vectorized` requires 16-byte aligned fp32 and 8-byte aligned bf16 arrays
// (n is handled with a scalar tail either way).
template <typename GT, typename MT>
__global__ void adamw_kernel(float* __restrict__ master, const GT* __restrict__ grad, MT* __restrict__ m,
                             MT* __restrict__ v, __nv_bfloat16* __restrict__ out, int64_t n, float lr, float beta1,
                             float beta2, float eps, float weight_decay, float bc1, float bc2_sqrt,
                             float grad_scale, const float* __restrict__ grad_scale_ptr, bool vectorized,
                             const int* __restrict__ step_ptr) {
  const float gs = grad_scale * (grad_scale_ptr != nullptr ? *grad_scale_ptr : 1.f);
  if (step_ptr != nullptr) {  // step count kept on the device (CUDA-graph replays): bias corrections here
    const double st = static_cast<double>(*step_ptr);
    bc1 = static_cast<float>(1.0 - pow(static_cast<double>(beta1), st));
    bc2_sqrt = static_cast<float>(sqrt(1.0 - pow(static_cast<double>(beta2), st)));
  }
  const float step_size = lr / bc1;
  const float decay = 1.f - lr * weight_decay;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t tail = 0;
  if (vectorized) {
    const int64_t n4 = n / 4;
    for (int64_t q = tid; q < n4; q += stride) {
      const int64_t i = q * 4;
      float g[4], p[4], mi[4], vi[4];
      Vec4<GT>::load(grad + i, g);
      Vec4<float>::load(master + i, p);
      Vec4<MT>::load(m + i, mi);
      Vec4<MT>::load(v + i, vi);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float gk = g[k] * gs;
        mi[k] = beta1 * mi[k] + (1.f - beta1) * gk;
        vi[k] = beta2 * vi[k] + (1.f - beta2) * gk * gk;
        p[k] = p[k] * decay - step_size * mi[k] / (sqrtf(vi[k]) / bc2_sqrt + eps);
      }
      Vec4<float>::store(master + i, p);
      Vec4<MT>::store(m + i, mi);
      Vec4<MT>::store(v + i, vi);
      if (out != nullptr) Vec4<__nv_bfloat16>::store(out + i, p);
    }
    tail = n4 * 4;
  }
  for (int64_t i = tail + tid; i < n; i += stride) {
    const float g = to_float<GT>(grad[i]) * gs;
    float p = master[i] * decay;
    const float mi = beta1 * to_float<MT>(m[i]) + (1.f - beta1) * g;
    const float vi = beta2 * to_float<MT>(v[i]) + (1.f - beta2) * g * g;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    p -= step_size * mi / denom;
    master[i] = p;
    m[i] = from_float<MT>(mi);
    v[i] = from_float<MT>(vi);
    if (out != nullptr) out[i] = f2bf(p);
  }
}

template <typename GT, typename PT>
__global__ void sgd_kernel(PT* __restrict__ param, const GT* __restrict__ grad, __nv_bfloat16* __restrict__ out,
                           int64_t n, float lr, float grad_scale, int* __restrict__ nonfinite) {
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float g = to_float<GT>(grad[i]) * grad_scale;
    bad |= !isfinite(g);
    const float p = to_float<PT>(param[i]) - lr * g;
    param[i] = from_float<PT>(p);
    if (out != nullptr) out[i] = f2bf(p);
  }
  if (bad && nonfinite != nullptr) atomicExch(nonfinite, 1);
}

template <typename GT>
__global__ void sq_norm_kernel(const GT* __restrict__ g, float* __restrict__ partial, int64_t n) {
  __shared__ float scratch[32];
  float s = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = to_float<GT>(g[i]);
    s += x * x;
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

int grid_for(int64_t n) {
  const int64_t blocks = (n + 255) / 256;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(num_sms()) * 8)));
}

}  // namespace

void adamw_step(at::Tensor& master, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& out, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step, double grad_scale, const c10::optional<at::Tensor>& grad_scale_t,
                const c10::optional<at::Tensor>& step_t, int64_t max_blocks) {
  check_cuda_tensor(master, "master");
  check_cuda_tensor(grad, "grad");
  check_cuda_tensor(m, "m");
  check_cuda_tensor(v, "v");
  TDSV_CHECK(master.scalar_type() == at::kFloat, "adamw: fp32 master");
  const int64_t n = master.numel();
  TDSV_CHECK(grad.numel() == n && m.numel() == n && v.numel() == n, "adamw: size mismatch");
  TDSV_CHECK(m.scalar_type() == v.scalar_type(), "adamw: moments share a dtype");
  __nv_bfloat16* outp = nullptr;
  if (out.has_value() && out->defined()) {
    check_cuda_tensor(*out, "out");
    TDSV_CHECK(out->scalar_type() == at::kBFloat16 && out->numel() == n, "adamw: bf16 out copy");
    outp = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
  }
  const float* gsp = nullptr;
  if (grad_scale_t.has_value() && grad_scale_t->defined()) gsp = grad_scale_t->data_ptr<float>();
  const int* stp = nullptr;
  if (step_t.has_value() && step_t->defined()) {
    check_cuda_tensor(*step_t, "step_t");
    TDSV_CHECK(step_t->scalar_type() == at::kInt, "adamw: step_t is an int32 device scalar");
    stp = step_t->data_ptr<int>();
  }
  if (n == 0) return;
  const float bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  const float bc2s = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  c10::cuda::CUDAGuard guard(master.device());
  // max_blocks > 0 caps the CTAs (an update running on a side stream next to compute kernels)
  const int grid = max_blocks > 0 ? std::min<int>(grid_for((n + 3) / 4), static_cast<int>(max_blocks))
                                  : grid_for((n + 3) / 4);
  auto aligned = [](const void* p, int bytes) { return reinterpret_cast<uintptr_t>(p) % bytes == 0; };
  const bool vec = aligned(master.data_ptr(), 16) && aligned(grad.data_ptr(), 16) && aligned(m.data_ptr(), 16) &&
                   aligned(v.data_ptr(), 16) && (outp == nullptr || aligned(outp, 8));
#define TDSV_ADAMW(GT, MT, gptr, mptr, vptr)                                                                   \
  adamw_kernel<GT, MT><<<grid, 256, 0, stream()>>>(master.data_ptr<float>(), gptr, mptr, vptr, outp, n,       \
                                                   static_cast<float>(lr), static_cast<float>(beta1),         \
                                                   static_cast<float>(beta2), static_cast<float>(eps),        \
                                                   static_cast<float>(weight_decay), bc1, bc2s,               \
                                                   static_cast<float>(grad_scale), gsp, vec, stp)
  const bool g32 = grad.scalar_type() == at::kFloat;
  const bool m32 = m.scalar_type() == at::kFloat;
  auto gbf = reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr());
  auto mbf = reinterpret_cast<__nv_bfloat16*>(m.data_ptr());
  auto vbf = reinterpret_cast<__nv_bfloat16*>(v.data_ptr());
  if (g32 && m32) TDSV_ADAMW(float, float, grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>());
  else if (g32) TDSV_ADAMW(float, __nv_bfloat16, grad.data_ptr<float>(), mbf, vbf);
  else if (m32) TDSV_ADAMW(__nv_bfloat16, float, gbf, m.data_ptr<float>(), v.data_ptr<float>());
  else TDSV_ADAMW(__nv_bfloat16, __nv_bfloat16, gbf, mbf, vbf);
#undef TDSV_ADAMW
  TDSV_LAUNCH_CHECK();
}

void sgd_step(at::Tensor& param, const at::Tensor& grad, const c10::optional<at::Tensor>& out, double lr,
              double grad_scale, const c10::optional<at::Tensor>& nonfinite) {
  check_cuda_tensor(param, "param");
  check_cuda_tensor(grad, "grad");
  const int64_t n = param.numel();
  TDSV_CHECK(grad.numel() == n, "sgd: size mismatch");
  __nv_bfloat16* outp = nullptr;
  if (out.has_value() && out->defined()) outp = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
  int* flag = nullptr;
  if (nonfinite.has_value() && nonfinite->defined()) flag = nonfinite->data_ptr<int>();
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(param.device());
  const int grid = grid_for(n);
  const bool g32 = grad.scalar_type() == at::kFloat;
  const bool p32 = param.scalar_type() == at::kFloat;
  auto gbf = reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr());
  auto pbf = reinterpret_cast<__nv_bfloat16*>(param.data_ptr());
  const float lrf = static_cast<float>(lr), gsf = static_cast<float>(grad_scale);
  if (g32 && p32) sgd_kernel<float, float><<<grid, 256, 0, stream()>>>(param.data_ptr<float>(), grad.data_ptr<float>(), outp, n, lrf, gsf, flag);
  else if (g32) sgd_kernel<float, __nv_bfloat16><<<grid, 256, 0, stream()>>>(pbf, grad.data_ptr<float>(), outp, n, lrf, gsf, flag);
  else if (p32) sgd_kernel<__nv_bfloat16, float><<<grid, 256, 0, stream()>>>(param.data_ptr<float>(), gbf, outp, n, lrf, gsf, flag);
  else sgd_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, stream()>>>(pbf, gbf, outp, n, lrf, gsf, flag);
  TDSV_LAUNCH_CHECK();
}

at::Tensor column_sum(const at::Tensor& partial);

// Sum of squares of a tensor as a 0-d fp32 device tensor (fixed-order reduction).
at::Tensor grad_sq_norm(const at::Tensor& g) {
  check_cuda_tensor(g, "g");
  const int64_t n = g.numel();
  const int grid = std::min(grid_for(n), 1024);
  auto partial = at::empty({grid, 1}, g.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(g.device());
  if (g.scalar_type() == at::kFloat) {
    sq_norm_kernel<float><<<grid, 256, 0, stream()>>>(g.data_ptr<float>(), partial.data_ptr<float>(), n);
  } else {
    TDSV_CHECK(g.scalar_type() == at::kBFloat16, "grad_sq_norm: fp32 or bf16");
    sq_norm_kernel<__nv_bfloat16><<<grid, 256, 0, stream()>>>(reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
                                                              partial.data_ptr<float>(), n);
  }
  TDSV_LAUNCH_CHECK();
  return column_sum(partial).view({});
}

}  // namespace tdsv
