// mHC hyper-connection mixing kernels for 4 residual streams (DeepSeek-V4.1).
//
// Semantics of dsv41_train/models/dsv4/mhc.py (K5-K10 there):
//   sinkhorn : P = softmax_row(C) + eps, column-normalise, then (iters-1) x (row, column)
//              normalisations, each dividing by (sum + eps). One thread per token; the backward
//              recomputes the forward iterates instead of keeping a 2*iters*16 float workspace.
//   collapse : out[t] = sum_j w[t,j] * s[t,j]                         (fp32 accumulate)
//   expand   : out[t,k] = post[t,k] * v[t] + sum_j comb[t,j,k] * r[t,j]
// The backward reductions over the hidden dimension (weight gradients) are per-token block
// reductions with a fixed order, so they are deterministic without atomics.
#include "common.cuh"

namespace tdsv {

namespace {

// ---- Sinkhorn ----------------------------------------------------------------------------
// Normalisation step index s in [0, 2*iters): s = 0 is the first column normalisation that
// follows the row softmax; afterwards odd s are row and even s are column normalisations.
__device__ __forceinline__ bool step_is_row(int s) { return (s & 1) == 1; }

__device__ __forceinline__ void normalize(float (&p)[16], bool rows, float eps) {
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    float sum = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) sum += rows ? p[a * 4 + b] : p[b * 4 + a];
    const float inv = 1.f / (sum + eps);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      if (rows) p[a * 4 + b] *= inv; else p[b * 4 + a] *= inv;
    }
  }
}

__device__ __forceinline__ void softmax_rows(const float (&x)[16], float (&p)[16], float eps) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float mx = x[i * 4];
#pragma unroll
    for (int j = 1; j < 4; ++j) mx = fmaxf(mx, x[i * 4 + j]);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[i * 4 + j] = __expf(x[i * 4 + j] - mx);
      sum += p[i * 4 + j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) p[i * 4 + j] = p[i * 4 + j] / sum + eps;
  }
}

// state after `steps` normalisation steps (steps = 0: softmax + eps only)
__device__ __forceinline__ void sinkhorn_state(const float (&x)[16], int steps, float eps, float (&p)[16]) {
  softmax_rows(x, p, eps);
  for (int s = 0; s < steps; ++s) normalize(p, step_is_row(s), eps);
}

__global__ void sinkhorn_fwd_kernel(const float* __restrict__ comb, float* __restrict__ out, int64_t rows,
                                    int iters, float eps) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  float x[16], p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = comb[t * 16 + i];
  sinkhorn_state(x, 2 * iters - 1, eps, p);
#pragma unroll
  for (int i = 0; i < 16; ++i) out[t * 16 + i] = p[i];
}

__global__ void sinkhorn_bwd_kernel(const float* __restrict__ comb, const float* __restrict__ grad,
                                    float* __restrict__ dcomb, int64_t rows, int iters, float eps) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  float x[16], g[16], p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    x[i] = comb[t * 16 + i];
    g[i] = grad[t * 16 + i];
  }
  const int steps = 2 * iters - 1;
  for (int s = steps - 1; s >= 0; --s) {
    // p = input of step s; y = p / (sum + eps) along rows or columns
    sinkhorn_state(x, s, eps, p);
    const bool rows_step = step_is_row(s);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float sum = 0.f, dot = 0.f;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int idx = rows_step ? a * 4 + b : b * 4 + a;
        sum += p[idx];
      }
      const float d = sum + eps;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int idx = rows_step ? a * 4 + b : b * 4 + a;
        dot += g[idx] * p[idx];
      }
      const float corr = dot / (d * d);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int idx = rows_step ? a * 4 + b : b * 4 + a;
        g[idx] = g[idx] / d - corr;
      }
    }
  }
  // softmax rows backward (+eps is constant): dx = q * (g - sum(g q)) with q = softmax
  float q[16];
  softmax_rows(x, q, 0.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) dot += g[i * 4 + j] * q[i * 4 + j];
#pragma unroll
    for (int j = 0; j < 4; ++j) dcomb[t * 16 + i * 4 + j] = q[i * 4 + j] * (g[i * 4 + j] - dot);
  }
}

// ---- collapse / expand --------------------------------------------------------------------
constexpr int kThreads = 256;

__global__ void collapse_fwd_kernel(const __nv_bfloat16* __restrict__ s, const float* __restrict__ w,
                                    __nv_bfloat16* __restrict__ out, int h) {
  const int64_t t = blockIdx.x;
  float wv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) wv[j] = w[t * 4 + j];
  for (int c = threadIdx.x * 8; c < h; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v[8];
      load_bf16x8(s + (t * 4 + j) * h + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += wv[j] * v[i];
    }
    store_bf16x8(out + t * h + c, acc);
  }
}

__global__ void collapse_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ s,
                                    const float* __restrict__ w, __nv_bfloat16* __restrict__ ds,
                                    float* __restrict__ dw, int h) {
  __shared__ float red[kThreads / 32][4];
  const int64_t t = blockIdx.x;
  float wv[4], part[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) wv[j] = w[t * 4 + j];
  for (int c = threadIdx.x * 8; c < h; c += blockDim.x * 8) {
    float gv[8];
    load_bf16x8(g + t * h + c, gv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v[8], o[8];
      load_bf16x8(s + (t * 4 + j) * h + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        part[j] += gv[i] * v[i];
        o[i] = wv[j] * gv[i];
      }
      store_bf16x8(ds + (t * 4 + j) * h + c, o);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float r = warp_sum(part[j]);
    if (lane == 0) red[warp][j] = r;
  }
  __syncthreads();
  if (threadIdx.x < 4) {
    float sum = 0.f;
    for (int wi = 0; wi < static_cast<int>(blockDim.x / 32); ++wi) sum += red[wi][threadIdx.x];
    dw[t * 4 + threadIdx.x] = sum;
  }
}

__global__ void expand_fwd_kernel(const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ r,
                                  const float* __restrict__ post, const float* __restrict__ comb,
                                  __nv_bfloat16* __restrict__ out, int h) {
  const int64_t t = blockIdx.x;
  float pw[4], cw[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) pw[k] = post[t * 4 + k];
#pragma unroll
  for (int i = 0; i < 16; ++i) cw[i] = comb[t * 16 + i];
  for (int c = threadIdx.x * 8; c < h; c += blockDim.x * 8) {
    float vv[8], rr[4][8];
    load_bf16x8(v + t * h + c, vv);
#pragma unroll
    for (int j = 0; j < 4; ++j) load_bf16x8(r + (t * 4 + j) * h + c, rr[j]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float acc = pw[k] * vv[i];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc += cw[j * 4 + k] * rr[j][i];
        o[i] = acc;
      }
      store_bf16x8(out + (t * 4 + k) * h + c, o);
    }
  }
}

__global__ void expand_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ v,
                                  const __nv_bfloat16* __restrict__ r, const float* __restrict__ post,
                                  const float* __restrict__ comb, __nv_bfloat16* __restrict__ dv,
                                  __nv_bfloat16* __restrict__ dr, float* __restrict__ dpost,
                                  float* __restrict__ dcomb, int h) {
  __shared__ float red[kThreads / 32][20];
  const int64_t t = blockIdx.x;
  float pw[4], cw[16], part[20];
#pragma unroll
  for (int k = 0; k < 4; ++k) pw[k] = post[t * 4 + k];
#pragma unroll
  for (int i = 0; i < 16; ++i) cw[i] = comb[t * 16 + i];
#pragma unroll
  for (int i = 0; i < 20; ++i) part[i] = 0.f;
  for (int c = threadIdx.x * 8; c < h; c += blockDim.x * 8) {
    float gg[4][8], vv[8], rr[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) load_bf16x8(g + (t * 4 + k) * h + c, gg[k]);
    load_bf16x8(v + t * h + c, vv);
#pragma unroll
    for (int j = 0; j < 4; ++j) load_bf16x8(r + (t * 4 + j) * h + c, rr[j]);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) acc += pw[k] * gg[k][i];
      o[i] = acc;
    }
    store_bf16x8(dv + t * h + c, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) acc += cw[j * 4 + k] * gg[k][i];
        o[i] = acc;
      }
      store_bf16x8(dr + (t * 4 + j) * h + c, o);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        part[k] += gg[k][i] * vv[i];
#pragma unroll
        for (int j = 0; j < 4; ++j) part[4 + j * 4 + k] += gg[k][i] * rr[j][i];
      }
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 20; ++i) {
    const float s = warp_sum(part[i]);
    if (lane == 0) red[warp][i] = s;
  }
  __syncthreads();
  if (threadIdx.x < 20) {
    float sum = 0.f;
    for (int wi = 0; wi < static_cast<int>(blockDim.x / 32); ++wi) sum += red[wi][threadIdx.x];
    if (threadIdx.x < 4) dpost[t * 4 + threadIdx.x] = sum;
    else dcomb[t * 16 + threadIdx.x - 4] = sum;
  }
}

int threads_for(int h) { return std::min(kThreads, std::max(32, ((h / 8 + 31) / 32) * 32)); }

}  // namespace

at::Tensor mhc_sinkhorn_fwd(const at::Tensor& comb, int64_t iters, double eps) {
  check_cuda_tensor(comb, "comb");
  TDSV_CHECK(comb.scalar_type() == at::kFloat && comb.size(-1) == 16, "sinkhorn: fp32 [rows, 16]");
  const int64_t rows = comb.numel() / 16;
  auto out = at::empty_like(comb);
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(comb.device());
  sinkhorn_fwd_kernel<<<(rows + 127) / 128, 128, 0, stream()>>>(comb.data_ptr<float>(), out.data_ptr<float>(), rows,
                                                                 static_cast<int>(iters), static_cast<float>(eps));
  TDSV_LAUNCH_CHECK();
  return out;
}

at::Tensor mhc_sinkhorn_bwd(const at::Tensor& comb, const at::Tensor& grad, int64_t iters, double eps) {
  check_cuda_tensor(comb, "comb");
  check_cuda_tensor(grad, "grad");
  const int64_t rows = comb.numel() / 16;
  auto out = at::empty_like(comb);
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(comb.device());
  sinkhorn_bwd_kernel<<<(rows + 127) / 128, 128, 0, stream()>>>(comb.data_ptr<float>(), grad.data_ptr<float>(),
                                                                 out.data_ptr<float>(), rows, static_cast<int>(iters),
                                                                 static_cast<float>(eps));
  TDSV_LAUNCH_CHECK();
  return out;
}

at::Tensor mhc_collapse_fwd(const at::Tensor& s, const at::Tensor& w) {
  check_cuda_tensor(s, "streams");
  check_cuda_tensor(w, "weights");
  const int64_t rows = s.size(0);
  const int h = static_cast<int>(s.size(2));
  TDSV_CHECK(h % 8 == 0 && s.size(1) == 4, "collapse: [rows, 4, H] with H % 8 == 0");
  auto out = at::empty({rows, h}, s.options());
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(s.device());
  collapse_fwd_kernel<<<rows, threads_for(h), 0, stream()>>>(reinterpret_cast<const __nv_bfloat16*>(s.data_ptr()),
                                                            w.data_ptr<float>(),
                                                            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), h);
  TDSV_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> mhc_collapse_bwd(const at::Tensor& g, const at::Tensor& s, const at::Tensor& w) {
  check_cuda_tensor(g, "grad");
  const int64_t rows = s.size(0);
  const int h = static_cast<int>(s.size(2));
  auto ds = at::empty_like(s);
  auto dw = at::empty({rows, 4}, w.options());
  if (rows == 0) return {ds, dw};
  c10::cuda::CUDAGuard guard(s.device());
  collapse_bwd_kernel<<<rows, threads_for(h), 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(s.data_ptr()),
      w.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(ds.data_ptr()), dw.data_ptr<float>(), h);
  TDSV_LAUNCH_CHECK();
  return {ds, dw};
}

at::Tensor mhc_expand_fwd(const at::Tensor& v, const at::Tensor& r, const at::Tensor& post, const at::Tensor& comb) {
  check_cuda_tensor(v, "value");
  check_cuda_tensor(r, "residual");
  const int64_t rows = r.size(0);
  const int h = static_cast<int>(r.size(2));
  TDSV_CHECK(h % 8 == 0 && r.size(1) == 4, "expand: [rows, 4, H] with H % 8 == 0");
  auto out = at::empty_like(r);
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(r.device());
  expand_fwd_kernel<<<rows, threads_for(h), 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(r.data_ptr()),
      post.data_ptr<float>(), comb.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), h);
  TDSV_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> mhc_expand_bwd(const at::Tensor& g, const at::Tensor& v, const at::Tensor& r,
                                       const at::Tensor& post, const at::Tensor& comb) {
  check_cuda_tensor(g, "grad");
  const int64_t rows = r.size(0);
  const int h = static_cast<int>(r.size(2));
  auto dv = at::empty_like(v);
  auto dr = at::empty_like(r);
  auto dpost = at::empty({rows, 4}, post.options());
  auto dcomb = at::empty({rows, 16}, comb.options());
  if (rows == 0) return {dv, dr, dpost, dcomb};
  c10::cuda::CUDAGuard guard(r.device());
  expand_bwd_kernel<<<rows, threads_for(h), 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(r.data_ptr()), post.data_ptr<float>(), comb.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dr.data_ptr()),
      dpost.data_ptr<float>(), dcomb.data_ptr<float>(), h);
  TDSV_LAUNCH_CHECK();
  return {dv, dr, dpost, dcomb};
}

}  // namespace tdsv
