// Routing plans built on the GPU in a few launches, with no host synchronisation.
//
// moe_route_plan: the expert-major layout of a [N, k] id matrix (ids < 0 are unrouted). Each
// expert's rows form one segment whose start is a multiple of 128 (the tcgen05 GEMM M tile);
// within a segment rows keep the flat (item, slot) order, so the layout is deterministic and
// equals a stable sort by expert. Three kernels: per-chunk histograms, one block that scans
// them into segment and chunk bases, and a scatter that ranks entries inside a chunk with warp
// match masks. Optionally, items whose position inside their slab of `slab` items is at or above
// that slab's live count are treated as unrouted (the NVLink receive buffer is laid out as
// [sources, slab] with `slab_counts[source]` live rows each).
//
// ep_dest_plan: for token-level expert-parallel dispatch, which ranks each token goes to
// (dest[t, r]), the token's slot in each destination's receive slab (running count), and the
// per-destination totals. One block per destination scans the tokens in order.
#include "common.cuh"

namespace tdsv {

namespace {

constexpr int kChunk = 4096;  // entries per histogram / scatter block
constexpr int kThreads = 1024;

__device__ __forceinline__ int entry_expert(const int32_t* ids, int64_t i, int k, int num_experts,
                                            const int32_t* slab_counts, int64_t slab) {
  int e = ids[i];
  if (e < 0 || e >= num_experts) return -1;
  if (slab_counts != nullptr) {
    const int64_t item = i / k;
    if (item % slab >= slab_counts[item / slab]) return -1;
  }
  return e;
}

__global__ void __launch_bounds__(kThreads) route_hist_kernel(const int32_t* __restrict__ ids, int64_t n, int k,
                                                              int num_experts, const int32_t* __restrict__ slab_counts,
                                                              int64_t slab, int32_t* __restrict__ chunk_hist) {
  extern __shared__ int32_t hist[];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  for (int j = threadIdx.x; j < kChunk; j += blockDim.x) {
    const int64_t i = base + j;
    if (i >= n) break;
    const int e = entry_expert(ids, i, k, num_experts, slab_counts, slab);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    chunk_hist[static_cast<int64_t>(blockIdx.x) * num_experts + e] = hist[e];
}

// One block: per-expert totals -> padded segment sizes -> segment offsets (exclusive scan over
// experts) -> per-chunk bases (running sums over chunks, in chunk order).
__global__ void __launch_bounds__(kThreads) route_scan_kernel(int32_t* __restrict__ chunk_hist, int chunks,
                                                              int num_experts, int block, int32_t* __restrict__ offsets,
                                                              int32_t* __restrict__ seg_rows,
                                                              int64_t* __restrict__ counts, int32_t* __restrict__ total) {
  __shared__ int32_t warp_tot[32];
  const int e = threadIdx.x;
  int32_t count = 0;
  if (e < num_experts)
    for (int c = 0; c < chunks; ++c) count += chunk_hist[static_cast<int64_t>(c) * num_experts + e];
  const int32_t pad = (count + block - 1) / block * block;
  // block-wide exclusive scan of `pad` over experts
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t incl = pad;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t t = lane < (blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t v = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += v;
    }
    warp_tot[lane] = t;  // inclusive totals per warp
  }
  __syncthreads();
  const int32_t excl = incl - pad + (warp > 0 ? warp_tot[warp - 1] : 0);
  if (e < num_experts) {
    offsets[e] = excl;
    seg_rows[e] = pad;
    counts[e] = count;
    int32_t run = excl;  // chunk bases, in place of the histogram
    for (int c = 0; c < chunks; ++c) {
      const int64_t at = static_cast<int64_t>(c) * num_experts + e;
      const int32_t h = chunk_hist[at];
      chunk_hist[at] = run;
      run += h;
    }
  }
  if (threadIdx.x == blockDim.x - 1) total[0] = warp_tot[(blockDim.x >> 5) - 1];
}

__global__ void __launch_bounds__(kThreads) route_scatter_kernel(const int32_t* __restrict__ ids, int64_t n, int k,
                                                                 int num_experts, const int32_t* __restrict__ slab_counts,
                                                                 int64_t slab, const int32_t* __restrict__ chunk_base,
                                                                 int32_t* __restrict__ route_rows,
                                                                 int32_t* __restrict__ src) {
  extern __shared__ int32_t sm[];
  int32_t* running = sm;                   // [E]
  int32_t* warp_cnt = sm + num_experts;    // [32][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    running[e] = chunk_base[static_cast<int64_t>(blockIdx.x) * num_experts + e];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  for (int round = 0; round < kChunk; round += blockDim.x) {
    for (int j = threadIdx.x; j < warps * num_experts; j += blockDim.x) warp_cnt[j] = 0;
    __syncthreads();
    const int64_t i = base + round + threadIdx.x;
    const int e = i < n ? entry_expert(ids, i, k, num_experts, slab_counts, slab) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) warp_cnt[warp * num_experts + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int32_t pos = running[e] + rank;
      for (int w = 0; w < warp; ++w) pos += warp_cnt[w * num_experts + e];
      route_rows[i] = pos;
      src[pos] = static_cast<int32_t>(i / k);
    } else if (i < n) {
      route_rows[i] = -1;
    }
    __syncthreads();
    for (int ex = threadIdx.x; ex < num_experts; ex += blockDim.x) {
      int32_t add = 0;
      for (int w = 0; w < warps; ++w) add += warp_cnt[w * num_experts + ex];
      running[ex] += add;
    }
    __syncthreads();
  }
}

// dest[t, r] = token t has a selected expert on rank r; slot[t, r] = number of earlier tokens with
// dest[., r] (its row in rank r's receive slab); counts[r] = tokens sent to r.
__global__ void __launch_bounds__(kThreads) ep_dest_plan_kernel(const int32_t* __restrict__ ids, int64_t tokens, int k,
                                                                int experts_per_rank, int ranks,
                                                                uint8_t* __restrict__ dest, int32_t* __restrict__ slot,
                                                                int32_t* __restrict__ counts) {
  __shared__ int32_t warp_tot[32];
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t carry = 0;
  for (int64_t t0 = 0; t0 < tokens; t0 += blockDim.x) {
    const int64_t t = t0 + threadIdx.x;
    int32_t flag = 0;
    if (t < tokens) {
      for (int j = 0; j < k; ++j) {
        const int e = ids[t * k + j];
        if (e >= 0 && e / experts_per_rank == r) flag = 1;
      }
    }
    int32_t incl = flag;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int32_t s = lane < (blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t v = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += v;
      }
      warp_tot[lane] = s;
    }
    __syncthreads();
    const int32_t before = carry + incl - flag + (warp > 0 ? warp_tot[warp - 1] : 0);
    if (t < tokens) {
      dest[t * ranks + r] = static_cast<uint8_t>(flag);
      slot[t * ranks + r] = before + flag - 1;  // the token's row when flag == 1
    }
    carry += warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[r] = carry;
}

}  // namespace

// Returns route_rows [N, k] int32, src [capacity] int32, offsets [E] int32, rows [E] int32,
// counts [E] int64, total [1] int32.
std::vector<at::Tensor> moe_route_plan(const at::Tensor& ids, int64_t num_experts, int64_t block,
                                       const c10::optional<at::Tensor>& slab_counts, int64_t slab) {
  check_cuda_tensor(ids, "ids");
  TDSV_CHECK(ids.scalar_type() == at::kInt && ids.dim() == 2, "moe_route_plan: int32 ids [N, k]");
  TDSV_CHECK(num_experts > 0 && num_experts <= 1024, "moe_route_plan: 1..1024 experts");
  TDSV_CHECK(block > 0, "moe_route_plan: positive block");
  const int k = static_cast<int>(ids.size(1));
  const int64_t n = ids.numel();
  const int64_t capacity = (n + num_experts * (block - 1) + block - 1) / block * block;
  auto opts = ids.options();
  auto route_rows = at::empty({ids.size(0), k}, opts);
  auto src = at::empty({capacity}, opts);
  auto offsets = at::empty({num_experts}, opts);
  auto seg_rows = at::empty({num_experts}, opts);
  auto counts = at::empty({num_experts}, opts.dtype(at::kLong));
  auto total = at::empty({1}, opts);
  const int32_t* slab_ptr = nullptr;
  if (slab_counts.has_value() && slab_counts->defined()) {
    check_cuda_tensor(*slab_counts, "slab_counts");
    TDSV_CHECK(slab_counts->scalar_type() == at::kInt && slab > 0, "moe_route_plan: int32 slab counts");
    TDSV_CHECK(ids.size(0) % slab == 0 && slab_counts->numel() == ids.size(0) / slab,
               "moe_route_plan: items must be whole slabs");
    slab_ptr = slab_counts->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard guard(ids.device());
  cudaStream_t s = stream();
  TDSV_CUDA_CHECK(cudaMemsetAsync(src.data_ptr(), 0xff, capacity * sizeof(int32_t), s));  // -1 = padding
  const int chunks = static_cast<int>(std::max<int64_t>(1, (n + kChunk - 1) / kChunk));
  auto chunk_hist = at::empty({chunks, num_experts}, opts);
  const int e = static_cast<int>(num_experts);
  route_hist_kernel<<<chunks, kThreads, e * sizeof(int32_t), s>>>(ids.data_ptr<int32_t>(), n, k, e, slab_ptr, slab,
                                                                    chunk_hist.data_ptr<int32_t>());
  TDSV_LAUNCH_CHECK();
  route_scan_kernel<<<1, kThreads, 0, s>>>(chunk_hist.data_ptr<int32_t>(), chunks, e, static_cast<int>(block),
                                           offsets.data_ptr<int32_t>(), seg_rows.data_ptr<int32_t>(),
                                           counts.data_ptr<int64_t>(), total.data_ptr<int32_t>());
  TDSV_LAUNCH_CHECK();
  const size_t smem = static_cast<size_t>(e) * (1 + kThreads / 32) * sizeof(int32_t);
  if (smem > 48 * 1024) {
    TDSV_CUDA_CHECK(cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
  }
  if (n > 0) {
    route_scatter_kernel<<<chunks, kThreads, smem, s>>>(ids.data_ptr<int32_t>(), n, k, e, slab_ptr, slab,
                                                        chunk_hist.data_ptr<int32_t>(), route_rows.data_ptr<int32_t>(),
                                                        src.data_ptr<int32_t>());
    TDSV_LAUNCH_CHECK();
  }
  return {route_rows, src, offsets, seg_rows, counts, total};
}

// Returns dest [T, ranks] uint8, slot [T, ranks] int32, counts [ranks] int32.
std::vector<at::Tensor> ep_dest_plan(const at::Tensor& ids, int64_t experts_per_rank, int64_t ranks) {
  check_cuda_tensor(ids, "ids");
  TDSV_CHECK(ids.scalar_type() == at::kInt && ids.dim() == 2, "ep_dest_plan: int32 ids [T, k]");
  TDSV_CHECK(experts_per_rank > 0 && ranks > 0, "ep_dest_plan: positive sizes");
  const int64_t tokens = ids.size(0);
  auto dest = at::empty({tokens, ranks}, ids.options().dtype(at::kByte));
  auto slot = at::empty({tokens, ranks}, ids.options());
  auto counts = at::empty({ranks}, ids.options());
  c10::cuda::CUDAGuard guard(ids.device());
  ep_dest_plan_kernel<<<static_cast<int>(ranks), kThreads, 0, stream()>>>(
      ids.data_ptr<int32_t>(), tokens, static_cast<int>(ids.size(1)), static_cast<int>(experts_per_rank),
      static_cast<int>(ranks), dest.data_ptr<uint8_t>(), slot.data_ptr<int32_t>(), counts.data_ptr<int32_t>());
  TDSV_LAUNCH_CHECK();
  return {dest, slot, counts};
}

}  // namespace tdsv
