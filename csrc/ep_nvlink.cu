// Expert-parallel token exchange over NVLink / NVSwitch peer memory (no NCCL on this path).
//
// Every rank owns symmetric buffers (same layout on all ranks, peers' base addresses known):
//   recv [ep][T_cap][H]  rows pushed *to* this rank (dispatch direction), one slab per source
//   ret  [ep][T_cap][H]  rows pushed *back* to this rank (combine direction), one slab per owner
//   meta [ep][T_cap][2k] per pushed row: k local expert ids (-1 = not on this rank), k weights
//   flags: ready/free epochs per source for each buffer, and per-source row counts.
//
// Dispatch sends each token once per destination rank that owns any of its experts (dedupe; the
// reference sends one copy per (token, expert)), into the destination's slab of the source at a
// position fixed by a prefix count, so the layout - and every later reduction - is deterministic.
// Combine returns one pre-reduced row per (token, destination) and the source sums the
// destinations in rank order in fp32.
//
// Synchronisation: the last CTA of a push kernel fences (system scope) and raises the peer's
// ready flag with a release store; receivers acquire-poll their flags. Before pushing, a sender
// waits until the peer has released the previous contents (free flag). All polls are bounded by
// wall time and report kTimeoutPeer in the status word instead of hanging.
#include "common.cuh"

namespace tdsv {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epoch of an exchange: `offset` alone, or added to a device-resident base. With a base the host
// passes per-step offsets and advances the base once per step on the stream, so a captured CUDA
// graph replays with fresh epochs instead of the ones baked in at capture.
__device__ __forceinline__ uint32_t epoch_at(const uint32_t* base, uint32_t offset) {
  return base == nullptr ? offset : *reinterpret_cast<const volatile uint32_t*>(base) + offset;
}

// Wait until flags[s] >= epoch for every s != skip (or all s). One thread per source.
__global__ void wait_flags_kernel(const uint32_t* __restrict__ flags, int ep, const uint32_t* base, uint32_t offset,
                                  int* status, uint64_t limit_ns) {
  const int s = threadIdx.x;
  if (s >= ep) return;
  const uint32_t epoch = epoch_at(base, offset);
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (static_cast<int32_t>(ld_acquire_sys(flags + s) - epoch) >= 0) return;
    if ((i & 63u) == 63u && global_timer_ns() - start > limit_ns) {
      report_status(status, kTimeoutPeer);
      return;
    }
  }
}

// Raise flag slot `my_rank` of every peer's flag array to `epoch` (optionally writing counts first).
__global__ void signal_peers_kernel(const int64_t* __restrict__ peer_flags, const int64_t* __restrict__ peer_counts,
                                    const int32_t* __restrict__ counts, int ep, int my_rank, const uint32_t* base,
                                    uint32_t offset) {
  const int d = threadIdx.x;
  if (d >= ep) return;
  const uint32_t epoch = epoch_at(base, offset);
  __threadfence_system();
  if (peer_counts != nullptr) {
    reinterpret_cast<int32_t*>(peer_counts[d])[my_rank] = counts[d];
    __threadfence_system();
  }
  st_release_sys(reinterpret_cast<uint32_t*>(peer_flags[d]) + my_rank, epoch);
}

// Push token rows to their destination ranks' recv slabs (+ routing metadata).
// Grid: one warp per token. After all CTAs finished, the last one raises the ready flags.
__global__ void push_rows_kernel(const __nv_bfloat16* __restrict__ x, const uint8_t* __restrict__ dest_mask,
                                 const int32_t* __restrict__ slot, const int64_t* __restrict__ peer_recv,
                                 const int64_t* __restrict__ peer_meta, const int32_t* __restrict__ ids,
                                 const float* __restrict__ weights, int64_t tokens, int h, int ep, int my_rank,
                                 int64_t t_cap, int k, int e_local, unsigned int* __restrict__ done_counter,
                                 const int64_t* __restrict__ peer_flags, const int64_t* __restrict__ peer_counts,
                                 const int32_t* __restrict__ counts, const uint32_t* base, uint32_t offset,
                                 int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t < tokens) {
    const uint4* src = reinterpret_cast<const uint4*>(x + t * h);
    const int vecs = h / 8;
    for (int d = 0; d < ep; ++d) {
      if (!dest_mask[t * ep + d]) continue;
      const int sl = slot[t * ep + d];
      if (!TDSV_IN_BOUNDS(sl >= 0 && sl < t_cap, status)) continue;  // a peer-memory write: never out of range
      const int64_t row = static_cast<int64_t>(my_rank) * t_cap + sl;
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peer_recv[d]) + row * h);
      for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
      if (peer_meta != nullptr && lane < k) {
        const int gid = ids[t * k + lane];
        const int owner = gid / e_local;
        int32_t* meta = reinterpret_cast<int32_t*>(peer_meta[d]) + row * 2 * k;
        meta[lane] = owner == d ? gid - d * e_local : -1;
        reinterpret_cast<float*>(meta)[k + lane] = owner == d ? weights[t * k + lane] : 0.f;
      }
    }
  }
  // completion: every thread fences its peer stores, then the last CTA signals all peers
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(done_counter, 1u);
    if (prev == gridDim.x - 1) {
      *done_counter = 0;  // reset for the next launch (stream order protects reuse)
      const uint32_t epoch = epoch_at(base, offset);
      __threadfence_system();
      for (int d = 0; d < ep; ++d) {
        if (peer_counts != nullptr) reinterpret_cast<int32_t*>(peer_counts[d])[my_rank] = counts[d];
      }
      __threadfence_system();
      for (int d = 0; d < ep; ++d) st_release_sys(reinterpret_cast<uint32_t*>(peer_flags[d]) + my_rank, epoch);
    }
  }
}

constexpr int kCombineWarps = 8;  // warps per block of combine_push_kernel (one received row each)

// For every received row (source s, index i < counts[s]) compute sum_j w_j * y[route[s,i,j]]
// (fp32; w = 1 when weights is null) and store it into source s's ret slab `my_rank`, row i.
__global__ void combine_push_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ route,
                                    const float* __restrict__ weights, const int32_t* __restrict__ counts,
                                    const int64_t* __restrict__ peer_ret, const float* __restrict__ row_extra,
                                    const int64_t* __restrict__ peer_retw, int64_t t_cap, int h, int ep, int my_rank,
                                    int k, unsigned int* __restrict__ done_counter,
                                    const int64_t* __restrict__ peer_flags, const uint32_t* base, uint32_t offset,
                                    int64_t y_rows, int* status) {
  __shared__ int s_rows[kCombineWarps][32];
  __shared__ float s_w[kCombineWarps][32];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + wib;
  const int s = static_cast<int>(r / t_cap);
  const int64_t i = r % t_cap;
  if (s < ep && i < counts[s]) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peer_ret[s]) + (static_cast<int64_t>(my_rank) * t_cap + i) * h;
    // the row's routes, compacted once (in route order) into a per-warp table
    int my_row = -1;
    float my_w = 0.f;
    if (lane < k) {
      my_row = route[r * k + lane];
      my_w = weights != nullptr ? weights[r * k + lane] : 1.f;
      if (my_row >= 0 && !TDSV_IN_BOUNDS(my_row < y_rows, status)) my_row = -1;
    }
    const unsigned valid = __ballot_sync(0xffffffffu, my_row >= 0);
    if (my_row >= 0) {
      const int slot = __popc(valid & ((1u << lane) - 1u));
      s_rows[wib][slot] = my_row;
      s_w[wib][slot] = my_w;
    }
    __syncwarp();
    const int n = __popc(valid);
    for (int c = lane * 8; c < h; c += 256) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int j = 0;
      for (; j + 4 <= n; j += 4) {  // four independent 16-byte loads in flight per lane
        float v[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) load_bf16x8(y + static_cast<int64_t>(s_rows[wib][j + u]) * h + c, v[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float w = s_w[wib][j + u];
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += w * v[u][q];
        }
      }
      for (; j < n; ++j) {
        float v[8];
        load_bf16x8(y + static_cast<int64_t>(s_rows[wib][j]) * h + c, v);
        const float w = s_w[wib][j];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += w * v[q];
      }
      store_bf16x8(dst + c, acc);
    }
    if (row_extra != nullptr && lane < k) {
      float* wdst = reinterpret_cast<float*>(peer_retw[s]) + (static_cast<int64_t>(my_rank) * t_cap + i) * k;
      wdst[lane] = row_extra[r * k + lane];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(done_counter, 1u);
    if (prev == gridDim.x - 1) {
      *done_counter = 0;
      const uint32_t epoch = epoch_at(base, offset);
      __threadfence_system();
      for (int d = 0; d < ep; ++d) st_release_sys(reinterpret_cast<uint32_t*>(peer_flags[d]) + my_rank, epoch);
    }
  }
}

// out[t] = sum over destination ranks d (ascending) with dest_mask[t,d] of ret[d][slot[t,d]].
__global__ void reduce_returned_kernel(const __nv_bfloat16* __restrict__ ret, const uint8_t* __restrict__ dest_mask,
                                       const int32_t* __restrict__ slot, __nv_bfloat16* __restrict__ out,
                                       int64_t tokens, int64_t t_cap, int h, int ep, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  for (int c = lane * 8; c < h; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int d = 0; d < ep; ++d) {
      if (!dest_mask[t * ep + d]) continue;
      const int sl = slot[t * ep + d];
      if (!TDSV_IN_BOUNDS(sl >= 0 && sl < t_cap, status)) continue;
      float v[8];
      load_bf16x8(ret + (static_cast<int64_t>(d) * t_cap + sl) * h + c, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += v[q];
    }
    store_bf16x8(out + t * h + c, acc);
  }
}

constexpr int kWarpsPerBlock = 8;
static_assert(kWarpsPerBlock == kCombineWarps, "combine_push_kernel's route tables are sized per warp");

}  // namespace

namespace {
const uint32_t* epoch_base_ptr(const c10::optional<at::Tensor>& base) {
  if (!base.has_value() || !base->defined()) return nullptr;
  check_cuda_tensor(*base, "epoch_base");
  TDSV_CHECK(base->scalar_type() == at::kInt && base->numel() >= 1, "epoch_base: int32 device scalar");
  return reinterpret_cast<const uint32_t*>(base->data_ptr());
}
}  // namespace

void ep_wait(const at::Tensor& flags, int64_t epoch, const c10::optional<at::Tensor>& epoch_base) {
  check_cuda_tensor(flags, "flags");
  const int ep = static_cast<int>(flags.numel());
  TDSV_CHECK(ep <= 1024, "ep_wait: too many ranks");
  c10::cuda::CUDAGuard guard(flags.device());
  wait_flags_kernel<<<1, std::max(32, ep), 0, stream()>>>(reinterpret_cast<const uint32_t*>(flags.data_ptr()), ep,
                                                          epoch_base_ptr(epoch_base), static_cast<uint32_t>(epoch),
                                                          status_word_ptr(), peer_wait_limit_ns());
  TDSV_LAUNCH_CHECK();
}

void ep_signal(const at::Tensor& peer_flags, const c10::optional<at::Tensor>& peer_counts,
               const c10::optional<at::Tensor>& counts, int64_t my_rank, int64_t epoch,
               const c10::optional<at::Tensor>& epoch_base) {
  check_cuda_tensor(peer_flags, "peer_flags");
  const int ep = static_cast<int>(peer_flags.numel());
  const int64_t* pc = nullptr;
  const int32_t* cnt = nullptr;
  if (peer_counts.has_value() && peer_counts->defined()) {
    pc = peer_counts->data_ptr<int64_t>();
    cnt = counts->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard guard(peer_flags.device());
  signal_peers_kernel<<<1, std::max(32, ep), 0, stream()>>>(peer_flags.data_ptr<int64_t>(), pc, cnt, ep,
                                                            static_cast<int>(my_rank), epoch_base_ptr(epoch_base),
                                                            static_cast<uint32_t>(epoch));
  TDSV_LAUNCH_CHECK();
}

void ep_push_rows(const at::Tensor& x, const at::Tensor& dest_mask, const at::Tensor& slot,
                  const at::Tensor& peer_recv, const c10::optional<at::Tensor>& peer_meta,
                  const c10::optional<at::Tensor>& ids, const c10::optional<at::Tensor>& weights, int64_t t_cap,
                  int64_t e_local, at::Tensor& done_counter, const at::Tensor& peer_flags,
                  const c10::optional<at::Tensor>& peer_counts, const c10::optional<at::Tensor>& counts,
                  int64_t my_rank, int64_t epoch, const c10::optional<at::Tensor>& epoch_base) {
  check_cuda_tensor(x, "x");
  const int64_t tokens = x.size(0);
  const int h = static_cast<int>(x.size(1));
  const int ep = static_cast<int>(dest_mask.size(1));
  TDSV_CHECK(h % 8 == 0, "ep_push_rows: H % 8 == 0");
  TDSV_CHECK(tokens <= t_cap, "ep_push_rows: more tokens than the buffer capacity");
  const int64_t* meta = nullptr;
  const int32_t* idp = nullptr;
  const float* wp = nullptr;
  int k = 0;
  if (peer_meta.has_value() && peer_meta->defined()) {
    meta = peer_meta->data_ptr<int64_t>();
    idp = ids->data_ptr<int32_t>();
    wp = weights->data_ptr<float>();
    k = static_cast<int>(ids->size(1));
    TDSV_CHECK(k <= 32, "ep_push_rows: top-k must be <= 32");
  }
  const int64_t* pc = nullptr;
  const int32_t* cnt = nullptr;
  if (peer_counts.has_value() && peer_counts->defined()) {
    pc = peer_counts->data_ptr<int64_t>();
    cnt = counts->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t blocks = std::max<int64_t>(1, (tokens + kWarpsPerBlock - 1) / kWarpsPerBlock);
  push_rows_kernel<<<blocks, kWarpsPerBlock * 32, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), dest_mask.data_ptr<uint8_t>(), slot.data_ptr<int32_t>(),
      peer_recv.data_ptr<int64_t>(), meta, idp, wp, tokens, h, ep, static_cast<int>(my_rank), t_cap, k,
      static_cast<int>(e_local), reinterpret_cast<unsigned int*>(done_counter.data_ptr()),
      peer_flags.data_ptr<int64_t>(), pc, cnt, epoch_base_ptr(epoch_base), static_cast<uint32_t>(epoch),
      status_word_ptr());
  TDSV_LAUNCH_CHECK();
}

void ep_combine_push(const at::Tensor& y, const at::Tensor& route, const c10::optional<at::Tensor>& weights,
                     const at::Tensor& counts, const at::Tensor& peer_ret, const c10::optional<at::Tensor>& row_extra,
                     const c10::optional<at::Tensor>& peer_retw, int64_t t_cap, at::Tensor& done_counter,
                     const at::Tensor& peer_flags, int64_t my_rank, int64_t epoch,
                     const c10::optional<at::Tensor>& epoch_base) {
  check_cuda_tensor(y, "y");
  check_cuda_tensor(route, "route");
  const int h = static_cast<int>(y.size(1));
  const int ep = static_cast<int>(counts.numel());
  const int k = static_cast<int>(route.size(1));
  TDSV_CHECK(route.size(0) == ep * t_cap, "ep_combine_push: route must be [ep * t_cap, k]");
  TDSV_CHECK(k >= 1 && k <= 32, "ep_combine_push: 1 <= k <= 32");
  const float* wp = nullptr;
  if (weights.has_value() && weights->defined()) wp = weights->data_ptr<float>();
  const float* extra = nullptr;
  const int64_t* retw = nullptr;
  if (row_extra.has_value() && row_extra->defined()) {
    check_cuda_tensor(*row_extra, "row_extra");
    TDSV_CHECK(row_extra->scalar_type() == at::kFloat && row_extra->size(1) == k, "row_extra: fp32 [rows, k]");
    extra = row_extra->data_ptr<float>();
    retw = peer_retw->data_ptr<int64_t>();
  }
  c10::cuda::CUDAGuard guard(y.device());
  const int64_t rows = ep * t_cap;
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  combine_push_kernel<<<blocks, kWarpsPerBlock * 32, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), route.data_ptr<int32_t>(), wp, counts.data_ptr<int32_t>(),
      peer_ret.data_ptr<int64_t>(), extra, retw, t_cap, h, ep, static_cast<int>(my_rank), k,
      reinterpret_cast<unsigned int*>(done_counter.data_ptr()), peer_flags.data_ptr<int64_t>(),
      epoch_base_ptr(epoch_base), static_cast<uint32_t>(epoch), y.size(0), status_word_ptr());
  TDSV_LAUNCH_CHECK();
}

at::Tensor ep_reduce_returned(const at::Tensor& ret, const at::Tensor& dest_mask, const at::Tensor& slot,
                              int64_t tokens) {
  check_cuda_tensor(ret, "ret");
  const int ep = static_cast<int>(ret.size(0));
  const int64_t t_cap = ret.size(1);
  const int h = static_cast<int>(ret.size(2));
  auto out = at::empty({tokens, h}, ret.options());
  if (tokens == 0) return out;
  c10::cuda::CUDAGuard guard(ret.device());
  reduce_returned_kernel<<<(tokens + kWarpsPerBlock - 1) / kWarpsPerBlock, kWarpsPerBlock * 32, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(ret.data_ptr()), dest_mask.data_ptr<uint8_t>(), slot.data_ptr<int32_t>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), tokens, t_cap, h, ep, status_word_ptr());
  TDSV_LAUNCH_CHECK();
  return out;
}

}  // namespace tdsv
