// SwiGLU activation for the expert MLPs, forward and backward.
//
// Qwen3 experts (dsv41_train/models/qwen/model.py:231-238): h = silu(gate) * up, with gate and up
// the two halves of the gate_up projection ("split" layout, [R, 2I] = [gate | up]).
// DSV4 experts (dsv41_train/models/dsv4/moe/kernels.py:15-27, 31-162): gate/up interleaved per
// column ("interleaved" layout, [R, I, 2]); gate is clamped to <= limit, up to [-limit, limit],
// SiLU(-inf) = 0, and the result is multiplied by the per-row route weight. The route-weight
// gradient is a per-row dot product reduced in a fixed order (no atomics).
#include "common.cuh"

namespace tdsv {

namespace {

__device__ __forceinline__ void load_gu(const __nv_bfloat16* gu, int64_t row, int i, int inter, bool interleaved,
                                        float& g, float& u) {
  if (interleaved) {
    const __nv_bfloat162 p = reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * inter)[i];
    g = __low2float(p);
    u = __high2float(p);
  } else {
    g = bf2f(gu[row * 2 * inter + i]);
    u = bf2f(gu[row * 2 * inter + inter + i]);
  }
}

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, const float* __restrict__ w,
                                  __nv_bfloat16* __restrict__ out, int64_t rows, int inter, bool interleaved,
                                  float limit, const int32_t* __restrict__ row_limit) {
  const int64_t row = blockIdx.x;
  if (row >= rows || (row_limit != nullptr && row >= *row_limit)) return;
  const float ws = w != nullptr ? w[row] : 1.f;
  for (int i = threadIdx.x; i < inter; i += blockDim.x) {
    float g, u;
    load_gu(gu, row, i, inter, interleaved, g, u);
    if (limit > 0.f) {
      g = fminf(g, limit);
      u = fminf(fmaxf(u, -limit), limit);
    }
    const float s = (g == -INFINITY) ? 0.f : silu_f(g);
    out[row * inter + i] = f2bf(s * u * ws);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ gu,
                                  const float* __restrict__ w, __nv_bfloat16* __restrict__ dgu,
                                  float* __restrict__ dw, int64_t rows, int inter, bool interleaved, float limit,
                                  const int32_t* __restrict__ row_limit) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  if (row >= rows || (row_limit != nullptr && row >= *row_limit)) return;
  const float ws = w != nullptr ? w[row] : 1.f;
  float dot = 0.f;
  for (int i = threadIdx.x; i < inter; i += blockDim.x) {
    float g0, u0;
    load_gu(gu, row, i, inter, interleaved, g0, u0);
    float g = g0, u = u0;
    bool g_pass = true, u_pass = true;
    if (limit > 0.f) {
      g_pass = g0 <= limit;
      u_pass = (u0 >= -limit) && (u0 <= limit);
      g = fminf(g0, limit);
      u = fminf(fmaxf(u0, -limit), limit);
    }
    const float d = bf2f(dout[row * inter + i]);
    float s, ds;
    if (g == -INFINITY) {
      s = 0.f;
      ds = 0.f;
    } else {
      const float sg = sigmoid_f(g);
      s = g * sg;
      ds = sg * (1.f + g * (1.f - sg));
    }
    dot += d * s * u;
    const float dg = g_pass ? d * ws * u * ds : 0.f;
    const float du = u_pass ? d * ws * s : 0.f;
    if (interleaved) {
      reinterpret_cast<__nv_bfloat162*>(dgu + row * 2 * inter)[i] = __floats2bfloat162_rn(dg, du);
    } else {
      dgu[row * 2 * inter + i] = f2bf(dg);
      dgu[row * 2 * inter + inter + i] = f2bf(du);
    }
  }
  if (dw != nullptr) {
    dot = block_sum(dot, scratch);
    if (threadIdx.x == 0) dw[row] = dot;
  }
}


// Warp-per-row variants for inter % 8 == 0: 16-byte accesses, a grid-stride loop over the rows in
// use (the expert-major buffer is capacity-sized; only the first *row_limit rows are live), and a
// fixed-order warp reduction for the route-weight gradient.
__device__ __forceinline__ void load_gu8(const __nv_bfloat16* row, int c, int inter, bool interleaved, float* g,
                                         float* u) {
  if (interleaved) {
    float a[8], b[8];
    load_bf16x8(row + 2 * c, a);
    load_bf16x8(row + 2 * c + 8, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      g[i] = a[2 * i];
      u[i] = a[2 * i + 1];
      g[4 + i] = b[2 * i];
      u[4 + i] = b[2 * i + 1];
    }
  } else {
    load_bf16x8(row + c, g);
    load_bf16x8(row + inter + c, u);
  }
}

__global__ void swiglu_fwd_vec_kernel(const __nv_bfloat16* __restrict__ gu, const float* __restrict__ w,
                                      __nv_bfloat16* __restrict__ out, int64_t rows, int inter, bool interleaved,
                                      float limit, const int32_t* __restrict__ row_limit) {
  const int lane = threadIdx.x & 31;
  const int64_t live = row_limit != nullptr ? min(rows, static_cast<int64_t>(*row_limit)) : rows;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < live;
       row += warps) {
    const float ws = w != nullptr ? w[row] : 1.f;
    const __nv_bfloat16* src = gu + row * 2 * inter;
    for (int c = lane * 8; c < inter; c += 256) {
      float g[8], u[8], o[8];
      load_gu8(src, c, inter, interleaved, g, u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float gg = g[i], uu = u[i];
        if (limit > 0.f) {
          gg = fminf(gg, limit);
          uu = fminf(fmaxf(uu, -limit), limit);
        }
        const float sv = (gg == -INFINITY) ? 0.f : silu_f(gg);
        o[i] = sv * uu * ws;
      }
      store_bf16x8(out + row * inter + c, o);
    }
  }
}

__global__ void swiglu_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ gu,
                                      const float* __restrict__ w, __nv_bfloat16* __restrict__ dgu,
                                      float* __restrict__ dw, int64_t rows, int inter, bool interleaved, float limit,
                                      const int32_t* __restrict__ row_limit) {
  const int lane = threadIdx.x & 31;
  const int64_t live = row_limit != nullptr ? min(rows, static_cast<int64_t>(*row_limit)) : rows;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < live;
       row += warps) {
    const float ws = w != nullptr ? w[row] : 1.f;
    const __nv_bfloat16* src = gu + row * 2 * inter;
    __nv_bfloat16* dst = dgu + row * 2 * inter;
    float dot = 0.f;
    for (int c = lane * 8; c < inter; c += 256) {
      float g[8], u[8], d[8], dg[8], du[8];
      load_gu8(src, c, inter, interleaved, g, u);
      load_bf16x8(dout + row * inter + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g0 = g[i], u0 = u[i];
        bool g_pass = true, u_pass = true;
        float gg = g0, uu = u0;
        if (limit > 0.f) {
          g_pass = g0 <= limit;
          u_pass = (u0 >= -limit) && (u0 <= limit);
          gg = fminf(g0, limit);
          uu = fminf(fmaxf(u0, -limit), limit);
        }
        float sv = 0.f, ds = 0.f;
        if (gg != -INFINITY) {
          const float sg = sigmoid_f(gg);
          sv = gg * sg;
          ds = sg * (1.f + gg * (1.f - sg));
        }
        dot += d[i] * sv * uu;
        dg[i] = g_pass ? d[i] * ws * uu * ds : 0.f;
        du[i] = u_pass ? d[i] * ws * sv : 0.f;
      }
      if (interleaved) {
        float a[8], b[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[2 * i] = dg[i];
          a[2 * i + 1] = du[i];
          b[2 * i] = dg[4 + i];
          b[2 * i + 1] = du[4 + i];
        }
        store_bf16x8(dst + 2 * c, a);
        store_bf16x8(dst + 2 * c + 8, b);
      } else {
        store_bf16x8(dst + c, dg);
        store_bf16x8(dst + inter + c, du);
      }
    }
    if (dw != nullptr) {
      dot = warp_sum(dot);
      if (lane == 0) dw[row] = dot;
    }
  }
}

constexpr int kVecThreads = 256;

int vec_grid(int64_t rows) {
  const int64_t want = (rows + (kVecThreads / 32) - 1) / (kVecThreads / 32);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * 8)));
}

bool vec_ok(const at::Tensor& gu, int inter) {
  return inter % 8 == 0 && reinterpret_cast<uintptr_t>(gu.data_ptr()) % 16 == 0;
}

}  // namespace

static const int32_t* limit_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<int32_t>() : nullptr;
}

at::Tensor swiglu_fwd(const at::Tensor& gu, const c10::optional<at::Tensor>& w, bool interleaved, double limit,
                      const c10::optional<at::Tensor>& row_limit) {
  check_cuda_tensor(gu, "gate_up");
  TDSV_CHECK(gu.scalar_type() == at::kBFloat16 && gu.dim() == 2 && gu.size(1) % 2 == 0, "swiglu: bf16 [R, 2I]");
  const int64_t rows = gu.size(0);
  const int inter = static_cast<int>(gu.size(1) / 2);
  auto out = at::empty({rows, inter}, gu.options());
  if (rows == 0) return out;
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    check_cuda_tensor(*w, "w");
    TDSV_CHECK(w->scalar_type() == at::kFloat && w->numel() == rows, "swiglu: fp32 weight per row");
    wp = w->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(gu.device());
  if (vec_ok(gu, inter)) {
    swiglu_fwd_vec_kernel<<<vec_grid(rows), kVecThreads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), wp, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        rows, inter, interleaved, static_cast<float>(limit), limit_ptr(row_limit));
    TDSV_LAUNCH_CHECK();
    return out;
  }
  const int threads = std::min(1024, std::max(32, ((inter + 31) / 32) * 32 / 2));
  swiglu_fwd_kernel<<<rows, threads, 0, stream()>>>(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), wp,
                                                    reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, inter,
                                                    interleaved, static_cast<float>(limit), limit_ptr(row_limit));
  TDSV_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu, const c10::optional<at::Tensor>& w,
                                   bool interleaved, double limit, bool need_dw,
                                   const c10::optional<at::Tensor>& row_limit) {
  check_cuda_tensor(dout, "dout");
  check_cuda_tensor(gu, "gate_up");
  const int64_t rows = gu.size(0);
  const int inter = static_cast<int>(gu.size(1) / 2);
  auto dgu = at::empty_like(gu);
  auto dw = at::zeros({rows}, gu.options().dtype(at::kFloat));
  if (rows == 0) return {dgu, dw};
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) wp = w->data_ptr<float>();
  c10::cuda::CUDAGuard guard(gu.device());
  if (vec_ok(gu, inter) && reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0) {
    swiglu_bwd_vec_kernel<<<vec_grid(rows), kVecThreads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        wp, reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), need_dw ? dw.data_ptr<float>() : nullptr, rows, inter,
        interleaved, static_cast<float>(limit), limit_ptr(row_limit));
    TDSV_LAUNCH_CHECK();
    return {dgu, dw};
  }
  const int threads = std::min(1024, std::max(32, ((inter + 31) / 32) * 32 / 2));
  swiglu_bwd_kernel<<<rows, threads, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), wp,
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), need_dw ? dw.data_ptr<float>() : nullptr, rows, inter,
      interleaved, static_cast<float>(limit), limit_ptr(row_limit));
  TDSV_LAUNCH_CHECK();
  return {dgu, dw};
}

}  // namespace tdsv
