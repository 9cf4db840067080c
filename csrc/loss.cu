// Cross entropy and selected-token log-probabilities over vocabulary-sized rows.
//
// cross_entropy_fused: for each row with a target != ignore_index computes
//     loss = logsumexp(l) - l[target]
// and overwrites the (bf16) logits row in place with  scale * (softmax(l) - onehot(target)),
// i.e. the gradient of `scale * loss`; ignored rows get loss 0 and a zero gradient. This lets the
// LM head run chunk by chunk (dsv41_train/models/dsv4/model.py:670-677 computes the same CE in fp32
// over materialised logits).
//
// token_logprob: log_softmax(l / T)[target] for RL scoring (dsv41_train/models/dsv4/model.py:679-684)
// with its backward  dl = dlogp * (onehot - softmax(l / T)) / T.
#include "common.cuh"

namespace tdsv {

namespace {

constexpr int kThreads = 512;

template <typename LT>
__device__ void row_stats(const LT* __restrict__ row, int v, float inv_t, float* scratch, float& mx, float& lse) {
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < v; i += blockDim.x) {
    const float x = to_float<LT>(row[i]) * inv_t;
    if (x > m) {
      s = s * __expf(m - x) + 1.f;
      m = x;
    } else {
      s += __expf(x - m);
    }
  }
  const float gm = block_max(m, scratch);
  s = (m == -INFINITY) ? 0.f : s * __expf(m - gm);
  const float gs = block_sum(s, scratch);
  mx = gm;
  lse = gm + logf(gs);
}

template <typename LT>
__global__ void ce_fused_kernel(LT* __restrict__ logits, const int64_t* __restrict__ targets,
                                float* __restrict__ loss, float* __restrict__ lse_out, int64_t rows, int v,
                                float scale, int64_t ignore_index, bool write_grad) {
  __shared__ float scratch[32];
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  LT* row = logits + r * v;
  const int64_t tgt = targets[r];
  if (tgt == ignore_index) {
    if (threadIdx.x == 0) {
      loss[r] = 0.f;
      if (lse_out) lse_out[r] = 0.f;
    }
    if (write_grad)
      for (int i = threadIdx.x; i < v; i += blockDim.x) row[i] = from_float<LT>(0.f);
    return;
  }
  float mx, lse;
  row_stats<LT>(row, v, 1.f, scratch, mx, lse);
  const float xt = to_float<LT>(row[tgt]);
  __syncthreads();
  if (threadIdx.x == 0) {
    loss[r] = lse - xt;
    if (lse_out) lse_out[r] = lse;
  }
  if (write_grad) {
    for (int i = threadIdx.x; i < v; i += blockDim.x) {
      const float p = __expf(to_float<LT>(row[i]) - lse);
      row[i] = from_float<LT>(scale * (p - (i == tgt ? 1.f : 0.f)));
    }
  }
}

template <typename LT>
__global__ void logprob_fwd_kernel(const LT* __restrict__ logits, const int64_t* __restrict__ targets,
                                   float* __restrict__ logp, float* __restrict__ lse_out, int64_t rows, int v,
                                   float inv_t) {
  __shared__ float scratch[32];
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const LT* row = logits + r * v;
  float mx, lse;
  row_stats<LT>(row, v, inv_t, scratch, mx, lse);
  if (threadIdx.x == 0) {
    logp[r] = to_float<LT>(row[targets[r]]) * inv_t - lse;
    lse_out[r] = lse;
  }
}

template <typename LT>
__global__ void logprob_bwd_kernel(const LT* __restrict__ logits, const int64_t* __restrict__ targets,
                                   const float* __restrict__ lse, const float* __restrict__ dlogp,
                                   LT* __restrict__ dlogits, int64_t rows, int v, float inv_t) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const LT* row = logits + r * v;
  LT* out = dlogits + r * v;
  const float g = dlogp[r];
  const float l = lse[r];
  const int64_t tgt = targets[r];
  for (int i = threadIdx.x; i < v; i += blockDim.x) {
    const float p = __expf(to_float<LT>(row[i]) * inv_t - l);
    out[i] = from_float<LT>(g * ((i == tgt ? 1.f : 0.f) - p) * inv_t);
  }
}

}  // namespace

std::vector<at::Tensor> cross_entropy_fused(at::Tensor& logits, const at::Tensor& targets, double scale,
                                            int64_t ignore_index, bool write_grad) {
  check_cuda_tensor(logits, "logits");
  check_cuda_tensor(targets, "targets");
  TDSV_CHECK(logits.dim() == 2, "cross_entropy: logits [rows, V]");
  TDSV_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "cross_entropy: int64 targets");
  const int64_t rows = logits.size(0);
  const int v = static_cast<int>(logits.size(1));
  auto loss = at::empty({rows}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({rows}, logits.options().dtype(at::kFloat));
  if (rows == 0) return {loss, lse};
  c10::cuda::CUDAGuard guard(logits.device());
  if (logits.scalar_type() == at::kBFloat16) {
    ce_fused_kernel<__nv_bfloat16><<<rows, kThreads, 0, stream()>>>(
        reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), loss.data_ptr<float>(),
        lse.data_ptr<float>(), rows, v, static_cast<float>(scale), ignore_index, write_grad);
  } else {
    TDSV_CHECK(logits.scalar_type() == at::kFloat, "cross_entropy: bf16 or fp32 logits");
    ce_fused_kernel<float><<<rows, kThreads, 0, stream()>>>(logits.data_ptr<float>(), targets.data_ptr<int64_t>(),
                                                          loss.data_ptr<float>(), lse.data_ptr<float>(), rows, v,
                                                          static_cast<float>(scale), ignore_index, write_grad);
  }
  TDSV_LAUNCH_CHECK();
  return {loss, lse};
}

std::vector<at::Tensor> token_logprob_fwd(const at::Tensor& logits, const at::Tensor& targets, double temperature) {
  check_cuda_tensor(logits, "logits");
  check_cuda_tensor(targets, "targets");
  const int64_t rows = logits.size(0);
  const int v = static_cast<int>(logits.size(1));
  auto logp = at::empty({rows}, logits.options().dtype(at::kFloat));
  auto lse = at::empty({rows}, logits.options().dtype(at::kFloat));
  if (rows == 0) return {logp, lse};
  c10::cuda::CUDAGuard guard(logits.device());
  const float inv_t = static_cast<float>(1.0 / temperature);
  if (logits.scalar_type() == at::kBFloat16) {
    logprob_fwd_kernel<__nv_bfloat16><<<rows, kThreads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), logp.data_ptr<float>(),
        lse.data_ptr<float>(), rows, v, inv_t);
  } else {
    logprob_fwd_kernel<float><<<rows, kThreads, 0, stream()>>>(logits.data_ptr<float>(), targets.data_ptr<int64_t>(),
                                                             logp.data_ptr<float>(), lse.data_ptr<float>(), rows, v,
                                                             inv_t);
  }
  TDSV_LAUNCH_CHECK();
  return {logp, lse};
}

at::Tensor token_logprob_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                             const at::Tensor& dlogp, double temperature) {
  check_cuda_tensor(logits, "logits");
  const int64_t rows = logits.size(0);
  const int v = static_cast<int>(logits.size(1));
  auto dlogits = at::empty_like(logits);
  if (rows == 0) return dlogits;
  c10::cuda::CUDAGuard guard(logits.device());
  const float inv_t = static_cast<float>(1.0 / temperature);
  auto g = dlogp.contiguous().to(at::kFloat);
  if (logits.scalar_type() == at::kBFloat16) {
    logprob_bwd_kernel<__nv_bfloat16><<<rows, kThreads, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
        g.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dlogits.data_ptr()), rows, v, inv_t);
  } else {
    logprob_bwd_kernel<float><<<rows, kThreads, 0, stream()>>>(logits.data_ptr<float>(), targets.data_ptr<int64_t>(),
                                                             lse.data_ptr<float>(), g.data_ptr<float>(),
                                                             dlogits.data_ptr<float>(), rows, v, inv_t);
  }
  TDSV_LAUNCH_CHECK();
  return dlogits;
}

}  // namespace tdsv
