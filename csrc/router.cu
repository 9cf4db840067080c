// MoE router: score function, (biased) top-k selection and weight normalisation, one warp per
// token, plus its backward (including the load-balancing auxiliary gradient).
//
// Qwen3-MoE (dsv41_train/models/qwen/model.py:246-257): softmax -> top-k -> renormalise.
// DSV4 TopKRouter (dsv41_train/models/dsv4/moe/module.py:22-41): score = sqrtsoftplus |
// softmax | sigmoid of fp32 logits; top-k of (score + selection_bias); weights are the unbiased
// scores, renormalised with +1e-20 and multiplied by routed_scaling_factor.
//
// The auxiliary load-balancing loss of both families is E * sum_e f_e * P_e where P_e is the mean
// softmax probability; its gradient w.r.t. each token's softmax is a per-expert constant vector
// (`aux_coef`, computed on the host from the global expert counts), folded into dlogits here.
#include "common.cuh"

namespace tdsv {

namespace {

constexpr int kMaxPerLane = 16;  // up to 512 experts
constexpr int kWarps = 8;

enum ScoreFunc : int { kSoftmax = 0, kSigmoid = 1, kSqrtSoftplus = 2 };

__device__ __forceinline__ float softplus_f(float x) {
  // log1p(exp(x)) with the same threshold torch uses for large inputs.
  return x > 20.f ? x : log1pf(__expf(x));
}

template <typename LT>
__global__ void router_fwd_kernel(const LT* __restrict__ logits, const float* __restrict__ bias,
                                  int32_t* __restrict__ ids, float* __restrict__ weights, float* __restrict__ scores,
                                  int64_t tokens, int e, int k, int func, bool normalize, float norm_eps,
                                  float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;
  float s[kMaxPerLane], sel[kMaxPerLane];
  const int per_lane = (e + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = i * 32 + lane;
    s[i] = (i < per_lane && c < e) ? to_float<LT>(logits[t * e + c]) : -INFINITY;
    mx = fmaxf(mx, s[i]);
  }
  if (func == kSoftmax) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      s[i] = (s[i] == -INFINITY) ? 0.f : __expf(s[i] - mx);
      sum += s[i];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) s[i] *= inv;
  } else {
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      if (s[i] == -INFINITY) { s[i] = 0.f; continue; }
      s[i] = func == kSigmoid ? sigmoid_f(s[i]) : sqrtf(softplus_f(s[i]));
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = i * 32 + lane;
    const bool valid = i < per_lane && c < e;
    sel[i] = valid ? s[i] + (bias != nullptr ? bias[c] : 0.f) : -INFINITY;
    if (valid) scores[t * e + c] = s[i];
  }
  float chosen_score = 0.f;
  int chosen_id = 0;
  float total = 0.f;
  for (int j = 0; j < k; ++j) {
    // arg-max over (sel) with the lowest index winning ties.
    float best = -INFINITY;
    int best_id = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = i * 32 + lane;
      if (sel[i] > best || (sel[i] == best && c < best_id)) {
        best = sel[i];
        best_id = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_id, o);
      if (ob > best || (ob == best && oi < best_id)) {
        best = ob;
        best_id = oi;
      }
    }
    // the owner lane knocks it out and broadcasts the unbiased score.
    float sc = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      if (i * 32 + lane == best_id) {
        sc = s[i];
        sel[i] = -INFINITY;
      }
    }
    sc = __shfl_sync(0xffffffffu, sc, best_id & 31);
    total += sc;
    if (lane == j) {
      chosen_score = sc;
      chosen_id = best_id;
    }
  }
  if (lane < k) {
    float w = chosen_score;
    if (normalize && k > 1) w = w / (total + norm_eps);
    ids[t * k + lane] = chosen_id;
    weights[t * k + lane] = w * scale;
  }
}

template <typename LT>
__global__ void router_bwd_kernel(const float* __restrict__ dweights, const int32_t* __restrict__ ids,
                                  const float* __restrict__ scores, const LT* __restrict__ logits,
                                  const float* __restrict__ aux_coef, LT* __restrict__ dlogits, int64_t tokens, int e,
                                  int k, int func, bool normalize, float norm_eps, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;
  // gradient w.r.t. the selected scores
  float total = 0.f, wdot = 0.f;
  float dw = 0.f, sk = 0.f;
  int id = -1;
  if (lane < k) {
    id = ids[t * k + lane];
    sk = scores[t * e + id];
    dw = dweights[t * k + lane];
  }
  total = warp_sum(sk);
  wdot = warp_sum(dw * sk);
  float dsel = 0.f;
  if (lane < k) {
    if (normalize && k > 1) {
      const float denom = total + norm_eps;
      dsel = scale * (dw / denom - wdot / (denom * denom));
    } else {
      dsel = scale * dw;
    }
  }
  const int per_lane = (e + 31) / 32;
  float ds[kMaxPerLane], sv[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    ds[i] = 0.f;
    const int c = i * 32 + lane;
    sv[i] = (i < per_lane && c < e) ? scores[t * e + c] : 0.f;
  }
  for (int j = 0; j < k; ++j) {
    const int jid = __shfl_sync(0xffffffffu, id, j);
    const float jd = __shfl_sync(0xffffffffu, dsel, j);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (i * 32 + lane == jid) ds[i] += jd;
  }
  float dl[kMaxPerLane];
  if (func == kSoftmax) {
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) dot += sv[i] * ds[i];
    dot = warp_sum(dot);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) dl[i] = sv[i] * (ds[i] - dot);
  } else {
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = i * 32 + lane;
      float x = (i < per_lane && c < e) ? to_float<LT>(logits[t * e + c]) : 0.f;
      if (func == kSigmoid) {
        dl[i] = ds[i] * sv[i] * (1.f - sv[i]);
      } else {
        dl[i] = sv[i] > 0.f ? ds[i] * sigmoid_f(x) / (2.f * sv[i]) : 0.f;
      }
    }
  }
  if (aux_coef != nullptr) {
    // softmax(logits) backward of the per-expert auxiliary gradient vector.
    float p[kMaxPerLane], mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = i * 32 + lane;
      p[i] = (i < per_lane && c < e) ? to_float<LT>(logits[t * e + c]) : -INFINITY;
      mx = fmaxf(mx, p[i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      p[i] = p[i] == -INFINITY ? 0.f : __expf(p[i] - mx);
      sum += p[i];
    }
    sum = warp_sum(sum);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = i * 32 + lane;
      p[i] /= sum;
      dot += (i < per_lane && c < e) ? p[i] * aux_coef[c] : 0.f;
    }
    dot = warp_sum(dot);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = i * 32 + lane;
      if (i < per_lane && c < e) dl[i] += p[i] * (aux_coef[c] - dot);
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = i * 32 + lane;
    if (i < per_lane && c < e) dlogits[t * e + c] = from_float<LT>(dl[i]);
  }
}

}  // namespace

std::vector<at::Tensor> router_fwd(const at::Tensor& logits, const c10::optional<at::Tensor>& bias, int64_t k,
                                   int64_t func, bool normalize, double norm_eps, double scale) {
  check_cuda_tensor(logits, "logits");
  TDSV_CHECK(logits.dim() == 2, "router: logits must be [tokens, experts]");
  const int64_t tokens = logits.size(0);
  const int e = static_cast<int>(logits.size(1));
  TDSV_CHECK(e <= 32 * kMaxPerLane, "router: at most 512 experts");
  TDSV_CHECK(k >= 1 && k <= 32 && k <= e, "router: 1 <= k <= min(32, experts)");
  auto ids = at::empty({tokens, k}, logits.options().dtype(at::kInt));
  auto weights = at::empty({tokens, k}, logits.options().dtype(at::kFloat));
  auto scores = at::empty({tokens, e}, logits.options().dtype(at::kFloat));
  if (tokens == 0) return {ids, weights, scores};
  const float* bias_ptr = nullptr;
  if (bias.has_value() && bias->defined()) {
    check_cuda_tensor(*bias, "bias");
    TDSV_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == e, "router: bias must be fp32 [experts]");
    bias_ptr = bias->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(logits.device());
  const dim3 grid((tokens + kWarps - 1) / kWarps);
  if (logits.scalar_type() == at::kFloat) {
    router_fwd_kernel<float><<<grid, kWarps * 32, 0, stream()>>>(
        logits.data_ptr<float>(), bias_ptr, ids.data_ptr<int32_t>(), weights.data_ptr<float>(),
        scores.data_ptr<float>(), tokens, e, static_cast<int>(k), static_cast<int>(func), normalize,
        static_cast<float>(norm_eps), static_cast<float>(scale));
  } else {
    TDSV_CHECK(logits.scalar_type() == at::kBFloat16, "router: logits fp32 or bf16");
    router_fwd_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), bias_ptr, ids.data_ptr<int32_t>(),
        weights.data_ptr<float>(), scores.data_ptr<float>(), tokens, e, static_cast<int>(k), static_cast<int>(func),
        normalize, static_cast<float>(norm_eps), static_cast<float>(scale));
  }
  TDSV_LAUNCH_CHECK();
  return {ids, weights, scores};
}

at::Tensor router_bwd(const at::Tensor& dweights, const at::Tensor& ids, const at::Tensor& scores,
                      const at::Tensor& logits, const c10::optional<at::Tensor>& aux_coef, int64_t func,
                      bool normalize, double norm_eps, double scale) {
  check_cuda_tensor(dweights, "dweights");
  check_cuda_tensor(ids, "ids");
  check_cuda_tensor(scores, "scores");
  check_cuda_tensor(logits, "logits");
  const int64_t tokens = logits.size(0);
  const int e = static_cast<int>(logits.size(1));
  const int k = static_cast<int>(ids.size(1));
  auto dlogits = at::empty_like(logits);
  if (tokens == 0) return dlogits;
  const float* aux_ptr = nullptr;
  if (aux_coef.has_value() && aux_coef->defined()) {
    check_cuda_tensor(*aux_coef, "aux_coef");
    TDSV_CHECK(aux_coef->scalar_type() == at::kFloat && aux_coef->numel() == e, "router: aux_coef fp32 [experts]");
    aux_ptr = aux_coef->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(logits.device());
  const dim3 grid((tokens + kWarps - 1) / kWarps);
  if (logits.scalar_type() == at::kFloat) {
    router_bwd_kernel<float><<<grid, kWarps * 32, 0, stream()>>>(
        dweights.data_ptr<float>(), ids.data_ptr<int32_t>(), scores.data_ptr<float>(), logits.data_ptr<float>(),
        aux_ptr, dlogits.data_ptr<float>(), tokens, e, k, static_cast<int>(func), normalize,
        static_cast<float>(norm_eps), static_cast<float>(scale));
  } else {
    router_bwd_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, stream()>>>(
        dweights.data_ptr<float>(), ids.data_ptr<int32_t>(), scores.data_ptr<float>(),
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), aux_ptr,
        reinterpret_cast<__nv_bfloat16*>(dlogits.data_ptr()), tokens, e, k, static_cast<int>(func), normalize,
        static_cast<float>(norm_eps), static_cast<float>(scale));
  }
  TDSV_LAUNCH_CHECK();
  return dlogits;
}

}  // namespace tdsv
