// Token <-> expert-major row movement for MoE layers on one GPU.
//
// The expert-major buffer holds each expert's routed rows in one contiguous segment whose start
// is a multiple of 128 rows (the tcgen05 GEMM M tile), padding rows are zero, so the grouped GEMMs
// never straddle two experts and their weight-gradient reductions over rows need no masking.
//
//   gather : rows[r]      = x[src[r]]             (src[r] < 0 -> zero row)
//   combine: out[t]       = sum_slot w[t,slot] * rows[idx[t,slot]]   (fp32, fixed slot order)
//   combine backward: drows[idx[t,s]] = w[t,s] * dout[t] ; dw[t,s] = <dout[t], rows[idx[t,s]]>
//
// The fixed slot order makes the reduction deterministic, as the reference requires
// (dsv41_train/models/dsv4/moe/dispatch.py:57-63 restores router-slot order before summing).
#include "common.cuh"

namespace tdsv {

namespace {

__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ src,
                                   __nv_bfloat16* __restrict__ out, int64_t rows, int h,
                                   const int32_t* __restrict__ row_limit, int64_t src_rows, int* status) {
  // one warp per row, 16B vectors, grid-stride over the live rows
  const int lane = threadIdx.x & 31;
  const int64_t live = row_limit != nullptr ? min(rows, static_cast<int64_t>(*row_limit)) : rows;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int vecs = h / 8;
  bf16x8 z;
#pragma unroll
  for (int i = 0; i < 4; ++i) z.v[i] = __floats2bfloat162_rn(0.f, 0.f);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < live; r += warps) {
    int s = src[r];
    if (s >= 0 && !TDSV_IN_BOUNDS(s < src_rows, status)) s = -1;
    bf16x8* dst = reinterpret_cast<bf16x8*>(out + r * h);
    if (s < 0) {
      for (int v = lane; v < vecs; v += 32) dst[v] = z;
      continue;
    }
    const bf16x8* sp = reinterpret_cast<const bf16x8*>(x + static_cast<int64_t>(s) * h);
    for (int v = lane; v < vecs; v += 32) dst[v] = sp[v];
  }
}

// One warp per token (grid-stride); each lane owns 8 columns per pass.
__global__ void combine_rows_kernel(const __nv_bfloat16* __restrict__ rows, const int32_t* __restrict__ idx,
                                    const float* __restrict__ w, __nv_bfloat16* __restrict__ out, int64_t tokens,
                                    int k, int h, int64_t row_cap, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens;
       t += warps)
  for (int c = lane * 8; c < h; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < k; ++s) {
      const int r = idx[t * k + s];
      if (r < 0 || !TDSV_IN_BOUNDS(r < row_cap, status)) continue;
      const float ws = w != nullptr ? w[t * k + s] : 1.f;
      float v[8];
      load_bf16x8(rows + static_cast<int64_t>(r) * h + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += ws * v[i];
    }
    store_bf16x8(out + t * h + c, acc);
  }
}

// Backward of combine: scatter weighted dout into the row buffer and compute dweights.
// One warp per token (grid-stride); unrouted slots cost one index read.
__global__ void combine_rows_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ rows,
                                        const int32_t* __restrict__ idx, const float* __restrict__ w,
                                        __nv_bfloat16* __restrict__ drows, float* __restrict__ dw, int64_t tokens,
                                        int k, int h, int64_t row_cap, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens;
       t += warps)
  for (int s = 0; s < k; ++s) {
    int r = idx[t * k + s];
    if (r >= 0 && !TDSV_IN_BOUNDS(r < row_cap, status)) r = -1;
    float dot = 0.f;
    if (r >= 0) {
      const float ws = w != nullptr ? w[t * k + s] : 1.f;
      for (int c = lane * 8; c < h; c += 256) {
        float g[8], v[8], o[8];
        load_bf16x8(dout + t * h + c, g);
        if (dw != nullptr) {
          load_bf16x8(rows + static_cast<int64_t>(r) * h + c, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) dot += g[i] * v[i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = ws * g[i];
        store_bf16x8(drows + static_cast<int64_t>(r) * h + c, o);
      }
    }
    if (dw != nullptr && r >= 0) {
      dot = warp_sum(dot);
      if (lane == 0) dw[t * k + s] = dot;
    }
  }
}

// Zero the padding rows of the expert-major buffer (rows whose source index is negative).
__global__ void zero_rows_kernel(__nv_bfloat16* __restrict__ buf, const int32_t* __restrict__ src, int64_t rows,
                                 int h, const int32_t* __restrict__ row_limit) {
  const int lane = threadIdx.x & 31;
  const int64_t live = row_limit != nullptr ? min(rows, static_cast<int64_t>(*row_limit)) : rows;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  bf16x8 z;
#pragma unroll
  for (int i = 0; i < 4; ++i) z.v[i] = __floats2bfloat162_rn(0.f, 0.f);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < live; r += warps) {
    if (src[r] >= 0) continue;
    bf16x8* dst = reinterpret_cast<bf16x8*>(buf + r * h);
    for (int v = lane; v < h / 8; v += 32) dst[v] = z;
  }
}

}  // namespace

// Blocks of 8 warps for `items` warp-sized work items, at most 8 blocks per SM (grid-stride).
static int warp_grid(int64_t items) {
  const int64_t want = (items + 7) / 8;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * 8)));
}

static const int32_t* limit_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<int32_t>() : nullptr;
}

at::Tensor moe_gather(const at::Tensor& x, const at::Tensor& src, const c10::optional<at::Tensor>& row_limit) {
  check_cuda_tensor(x, "x");
  check_cuda_tensor(src, "src");
  TDSV_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2, "moe_gather: x must be bf16 [T, H]");
  TDSV_CHECK(src.scalar_type() == at::kInt, "moe_gather: int32 index");
  const int h = static_cast<int>(x.size(1));
  TDSV_CHECK(h % 8 == 0, "moe_gather: H % 8 == 0");
  const int64_t rows = src.numel();
  auto out = at::empty({rows, h}, x.options());
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(x.device());
  gather_rows_kernel<<<warp_grid(rows), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), src.data_ptr<int32_t>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, h, limit_ptr(row_limit), x.size(0), status_word_ptr());
  TDSV_LAUNCH_CHECK();
  return out;
}

at::Tensor moe_combine(const at::Tensor& rows, const at::Tensor& idx, const c10::optional<at::Tensor>& w) {
  check_cuda_tensor(rows, "rows");
  check_cuda_tensor(idx, "idx");
  TDSV_CHECK(rows.scalar_type() == at::kBFloat16 && rows.dim() == 2, "moe_combine: rows bf16 [R, H]");
  const int64_t tokens = idx.size(0);
  const int k = static_cast<int>(idx.size(1));
  const int h = static_cast<int>(rows.size(1));
  TDSV_CHECK(h % 8 == 0, "moe_combine: H % 8 == 0");
  auto out = at::empty({tokens, h}, rows.options());
  if (tokens == 0) return out;
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    check_cuda_tensor(*w, "w");
    TDSV_CHECK(w->scalar_type() == at::kFloat, "moe_combine: fp32 weights");
    wp = w->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(rows.device());
  combine_rows_kernel<<<warp_grid(tokens), 256, 0, stream()>>>(reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()),
                                                        idx.data_ptr<int32_t>(), wp,
                                                        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), tokens, k, h,
                                                        rows.size(0), status_word_ptr());
  TDSV_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> moe_combine_bwd(const at::Tensor& dout, const at::Tensor& rows, const at::Tensor& idx,
                                        const c10::optional<at::Tensor>& w, bool need_dw) {
  check_cuda_tensor(dout, "dout");
  check_cuda_tensor(rows, "rows");
  check_cuda_tensor(idx, "idx");
  const int64_t tokens = idx.size(0);
  const int k = static_cast<int>(idx.size(1));
  const int h = static_cast<int>(rows.size(1));
  auto drows = at::empty_like(rows);
  auto dw = at::zeros({tokens, k}, rows.options().dtype(at::kFloat));
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) wp = w->data_ptr<float>();
  c10::cuda::CUDAGuard guard(rows.device());
  if (tokens > 0) {
    combine_rows_bwd_kernel<<<warp_grid(tokens), 256, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()),
        idx.data_ptr<int32_t>(), wp, reinterpret_cast<__nv_bfloat16*>(drows.data_ptr()),
        need_dw ? dw.data_ptr<float>() : nullptr, tokens, k, h, rows.size(0), status_word_ptr());
    TDSV_LAUNCH_CHECK();
  }
  return {drows, dw};
}

// Zeroes rows of `buf` whose `src` entry is negative (segment padding) in place.
void moe_zero_padding(at::Tensor& buf, const at::Tensor& src, const c10::optional<at::Tensor>& row_limit) {
  check_cuda_tensor(buf, "buf");
  check_cuda_tensor(src, "src");
  const int64_t rows = src.numel();
  const int h = static_cast<int>(buf.size(1));
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(buf.device());
  zero_rows_kernel<<<warp_grid(rows), 256, 0, stream()>>>(reinterpret_cast<__nv_bfloat16*>(buf.data_ptr()),
                                                          src.data_ptr<int32_t>(), rows, h, limit_ptr(row_limit));
  TDSV_LAUNCH_CHECK();
}

}  // namespace tdsv
