// Fused per-head RMSNorm + rotary embedding for Qwen3 attention inputs, and the interleaved
// (even/odd) rotary embedding used by DeepSeek-V4.1 CSA2 attention.
//
// Qwen3 (dsv41_train/models/qwen/model.py:19-35, 114-123): q and k heads are RMS-normalised over
// head_dim with their own weights, then rotated with the "rotate half" convention
//     out = y * cos + cat(-y[D/2:], y[:D/2]) * sin,   angle_i = pos * theta^(-2i/D).
// The kernel reads the fused [T, (Hq + 2 Hkv) * D] projection output directly and writes
// contiguous q [T, Hq, D] and k [T, Hkv, D]; v stays a strided view of the projection output.
//
// DSV4 (dsv41_train/models/dsv4/attention/module.py:72-85): the last `rope_dim` channels are
// rotated as (even, odd) pairs; `inverse` rotates by -angle (used on the attention output).
#include "common.cuh"

namespace tdsv {

namespace {

constexpr int kWarps = 8;

// One warp per (token, head); D = 128 -> four consecutive elements per lane.
__global__ void qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ wq,
                                        const __nv_bfloat16* __restrict__ wk, const int64_t* __restrict__ pos,
                                        const float* __restrict__ inv_freq, __nv_bfloat16* __restrict__ q_out,
                                        __nv_bfloat16* __restrict__ k_out, int64_t tokens, int hq, int hkv,
                                        float eps) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int heads = hq + hkv;
  if (item >= tokens * heads) return;
  const int64_t t = item / heads;
  const int h = static_cast<int>(item % heads);
  const bool is_q = h < hq;
  const int64_t row_stride = static_cast<int64_t>(hq + 2 * hkv) * D;
  const __nv_bfloat16* src = qkv + t * row_stride + static_cast<int64_t>(h) * D;
  const __nv_bfloat16* w = is_q ? wq : wk;
  float x[4];
  {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(src + lane * 4);
    float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  }
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float n = bf2f(f2bf(x[i] * r));
    y[i] = bf2f(f2bf(bf2f(w[lane * 4 + i]) * n));
  }
  // rotate-half partner lives 16 lanes away.
  float partner[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
  const float p = static_cast<float>(pos[t]);
  float out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane * 4 + i;
    const int f = d & (D / 2 - 1);
    float s, c;
    sincosf(p * inv_freq[f], &s, &c);
    const float rh = d < D / 2 ? -partner[i] : partner[i];
    out[i] = y[i] * c + rh * s;
  }
  __nv_bfloat16* dst = is_q ? q_out + (t * hq + h) * D : k_out + (t * hkv + (h - hq)) * D;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(dst + lane * 4);
  o[0] = __floats2bfloat162_rn(out[0], out[1]);
  o[1] = __floats2bfloat162_rn(out[2], out[3]);
}

constexpr int kTokensPerBlock = 16;

// Backward: inverse rotation, RMSNorm backward per head, weight-gradient partials per block.
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk,
                                        const __nv_bfloat16* __restrict__ dv, const __nv_bfloat16* __restrict__ qkv,
                                        const __nv_bfloat16* __restrict__ wq, const __nv_bfloat16* __restrict__ wk,
                                        const int64_t* __restrict__ pos, const float* __restrict__ inv_freq,
                                        __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dwq_part,
                                        float* __restrict__ dwk_part, int64_t tokens, int hq, int hkv, float eps) {
  constexpr int D = 128;
  __shared__ float red_q[kWarps][D];
  __shared__ float red_k[kWarps][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int heads = hq + hkv;
  const int64_t row_stride = static_cast<int64_t>(hq + 2 * hkv) * D;
  float accq[4] = {0, 0, 0, 0}, acck[4] = {0, 0, 0, 0};
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTokensPerBlock;
  for (int item = warp; item < kTokensPerBlock * heads; item += kWarps) {
    const int64_t t = t0 + item / heads;
    const int h = item % heads;
    if (t >= tokens) break;
    const bool is_q = h < hq;
    const __nv_bfloat16* src = qkv + t * row_stride + static_cast<int64_t>(h) * D;
    const __nv_bfloat16* g_src = is_q ? dq + (t * hq + h) * D : dk + (t * hkv + (h - hq)) * D;
    const __nv_bfloat16* w = is_q ? wq : wk;
    float x[4], g[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = bf2f(src[lane * 4 + i]);
      g[i] = bf2f(g_src[lane * 4 + i]);
    }
    float gp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) gp[i] = __shfl_xor_sync(0xffffffffu, g[i], 16);
    const float p = static_cast<float>(pos[t]);
    float dy[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane * 4 + i;
      const int f = d & (D / 2 - 1);
      float s, c;
      sincosf(p * inv_freq[f], &s, &c);
      // out_lo = y_lo c - y_hi s ; out_hi = y_hi c + y_lo s
      dy[i] = d < D / 2 ? g[i] * c + gp[i] * s : g[i] * c - gp[i] * s;
    }
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    float dn[4], dot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float wv = bf2f(w[lane * 4 + i]);
      dn[i] = wv * dy[i];
      dot += dn[i] * x[i];
      const float n = bf2f(f2bf(x[i] * r));
      if (is_q) accq[i] += dy[i] * n; else acck[i] += dy[i] * n;
    }
    dot = warp_sum(dot);
    const float coef = dot * r * r * r / D;
    __nv_bfloat16* dst = dqkv + t * row_stride + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = f2bf(r * dn[i] - coef * x[i]);
  }
  // v gradient is a plain copy into its slot.
  for (int64_t idx = threadIdx.x; idx < static_cast<int64_t>(kTokensPerBlock) * hkv * D; idx += blockDim.x) {
    const int64_t t = t0 + idx / (hkv * D);
    if (t >= tokens) break;
    const int64_t rem = idx % (hkv * D);
    dqkv[t * row_stride + static_cast<int64_t>(hq + hkv) * D + rem] = dv[t * hkv * D + rem];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    red_q[warp][lane * 4 + i] = accq[i];
    red_k[warp][lane * 4 + i] = acck[i];
  }
  __syncthreads();
  if (threadIdx.x < D) {
    float sq = 0.f, sk = 0.f;
    for (int wv = 0; wv < kWarps; ++wv) {
      sq += red_q[wv][threadIdx.x];
      sk += red_k[wv][threadIdx.x];
    }
    dwq_part[static_cast<int64_t>(blockIdx.x) * D + threadIdx.x] = sq;
    dwk_part[static_cast<int64_t>(blockIdx.x) * D + threadIdx.x] = sk;
  }
}

// DSV4 interleaved rotary on the last `rope_dim` channels of [rows, heads, D] (in place allowed).
__global__ void rope_interleaved_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                        const int64_t* __restrict__ pos, const float* __restrict__ inv_freq,
                                        int64_t rows, int heads, int d, int rope_dim, float sign) {
  const int64_t pairs_per_row = static_cast<int64_t>(heads) * (d / 2);
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * pairs_per_row) return;
  const int64_t row = idx / pairs_per_row;
  const int64_t rem = idx % pairs_per_row;
  const int head = static_cast<int>(rem / (d / 2));
  const int pair = static_cast<int>(rem % (d / 2));
  const int64_t base = (row * heads + head) * d + 2 * pair;
  const int first_rot_pair = (d - rope_dim) / 2;
  const float a = bf2f(x[base]), b = bf2f(x[base + 1]);
  if (pair < first_rot_pair) {
    if (x != y) {
      y[base] = x[base];
      y[base + 1] = x[base + 1];
    }
    return;
  }
  const int f = pair - first_rot_pair;
  float s, c;
  sincosf(static_cast<float>(pos[row]) * inv_freq[f], &s, &c);
  s *= sign;
  y[base] = f2bf(a * c - b * s);
  y[base + 1] = f2bf(a * s + b * c);
}

}  // namespace

std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk,
                                         const at::Tensor& pos, const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                         double eps) {
  check_cuda_tensor(qkv, "qkv");
  TDSV_CHECK(qkv.scalar_type() == at::kBFloat16, "qk_norm_rope: bf16 input");
  TDSV_CHECK(wq.scalar_type() == at::kBFloat16 && wk.scalar_type() == at::kBFloat16, "qk_norm_rope: bf16 weights");
  TDSV_CHECK(pos.scalar_type() == at::kLong, "qk_norm_rope: int64 positions");
  constexpr int D = 128;
  TDSV_CHECK(qkv.size(-1) == (hq + 2 * hkv) * D, "qk_norm_rope: head_dim must be 128");
  const int64_t tokens = qkv.numel() / qkv.size(-1);
  TDSV_CHECK(pos.numel() == tokens, "qk_norm_rope: one position per token");
  auto q = at::empty({tokens, hq, D}, qkv.options());
  auto k = at::empty({tokens, hkv, D}, qkv.options());
  const int64_t items = tokens * (hq + hkv);
  if (items == 0) return {q, k};
  c10::cuda::CUDAGuard guard(qkv.device());
  qk_norm_rope_fwd_kernel<<<(items + kWarps - 1) / kWarps, kWarps * 32, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(wq.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(wk.data_ptr()), pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k.data_ptr()), tokens,
      static_cast<int>(hq), static_cast<int>(hkv), static_cast<float>(eps));
  TDSV_LAUNCH_CHECK();
  return {q, k};
}

at::Tensor column_sum(const at::Tensor& partial);

std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv,
                                         const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk,
                                         const at::Tensor& pos, const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                         double eps) {
  check_cuda_tensor(dq, "dq");
  check_cuda_tensor(dk, "dk");
  check_cuda_tensor(dv, "dv");
  check_cuda_tensor(qkv, "qkv");
  constexpr int D = 128;
  const int64_t tokens = qkv.numel() / qkv.size(-1);
  auto dqkv = at::empty_like(qkv);
  const int blocks = static_cast<int>((tokens + kTokensPerBlock - 1) / kTokensPerBlock);
  auto pq = at::empty({std::max(blocks, 1), D}, qkv.options().dtype(at::kFloat));
  auto pk = at::empty({std::max(blocks, 1), D}, qkv.options().dtype(at::kFloat));
  if (tokens == 0) return {dqkv, pq.zero_().sum(0), pk.zero_().sum(0)};
  c10::cuda::CUDAGuard guard(qkv.device());
  qk_norm_rope_bwd_kernel<<<blocks, kWarps * 32, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(wq.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(wk.data_ptr()),
      pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
      pq.data_ptr<float>(), pk.data_ptr<float>(), tokens, static_cast<int>(hq), static_cast<int>(hkv),
      static_cast<float>(eps));
  TDSV_LAUNCH_CHECK();
  return {dqkv, column_sum(pq), column_sum(pk)};
}

at::Tensor rope_interleaved(const at::Tensor& x, const at::Tensor& pos, const at::Tensor& inv_freq, int64_t rope_dim,
                            bool inverse) {
  check_cuda_tensor(x, "x");
  TDSV_CHECK(x.dim() == 3, "rope_interleaved: x must be [rows, heads, D]");
  TDSV_CHECK(x.scalar_type() == at::kBFloat16, "rope_interleaved: bf16 input");
  const int64_t rows = x.size(0);
  const int heads = static_cast<int>(x.size(1)), d = static_cast<int>(x.size(2));
  TDSV_CHECK(rope_dim % 2 == 0 && rope_dim <= d, "rope_interleaved: bad rope_dim");
  TDSV_CHECK(pos.numel() == rows, "rope_interleaved: one position per row");
  auto y = at::empty_like(x);
  const int64_t n = rows * heads * (d / 2);
  if (n == 0) return y;
  c10::cuda::CUDAGuard guard(x.device());
  rope_interleaved_kernel<<<(n + 255) / 256, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
      pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(), rows, heads, d, static_cast<int>(rope_dim),
      inverse ? -1.f : 1.f);
  TDSV_LAUNCH_CHECK();
  return y;
}

}  // namespace tdsv
