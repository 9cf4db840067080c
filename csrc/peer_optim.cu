// Fused gradient reduce-scatter + optimizer update + parameter all-gather over NVLink peer memory.
//
// Dense (non-expert) parameters are kept as a bf16 replica on every rank, in a symmetric buffer
// (the "parameter pool"); their gradients are staged in a second symmetric buffer (the "gradient
// pool"). The fp32 master weights and the optimizer moments are sharded: rank r owns elements
// [offset + r * shard, offset + (r + 1) * shard) of every unit (a unit is a group of parameters
// that becomes ready together in backward, e.g. one decoder layer).
//
// One kernel per unit and step does what FSDP does with three collectives and an optimizer pass:
//   1. raise this rank's "gradients of this unit are staged" flag on every peer, then wait
//      (bounded) until every peer has raised its own;
//   2. reduce: read the owned slice of the gradient from every rank's pool with 16-byte peer
//      loads, summed in fp32 in rank order (deterministic, the same on every run);
//   3. scale (1 / world, or a device scalar) and apply AdamW (fp32 master, fp32 or bf16 moments;
//      torch.optim.AdamW semantics) or SGD to the owned slice;
//   4. gather: store the rounded bf16 result into every rank's parameter pool with 16-byte peer
//      stores, so no all-gather runs before the next forward.
// Bytes over NVLink per rank and unit: (world - 1) / world of the unit's gradient in bf16 and as
// much again of its parameters - half of what an fp32 reduce-scatter plus a bf16 all-gather move.
//
// Reuse of the pools across steps is ordered by a per-step barrier over the same flag array
// (ep_signal / ep_wait), run by the caller after the last unit of the step.
//
// Replaces the FSDP2 all-gather / reduce-scatter of the dense weights and the optimizer update of
// dsv41_train/models/qwen/parallel.py:28-45 and dsv41_train/optim.py:85-137 (reference paths).
#include "common.cuh"

namespace tdsv {

namespace {

__device__ __forceinline__ void flag_store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t flag_load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kMaxWorld = 8;
constexpr int kThreads = 256;

__device__ __forceinline__ void bf16x8_to_float(const uint4& raw, float (&o)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(h[q]);
    o[2 * q] = f.x;
    o[2 * q + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 float_to_bf16x8(const float (&o)[8]) {
  uint4 raw;
  uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __nv_bfloat162 b = __floats2bfloat162_rn(o[2 * q], o[2 * q + 1]);
    w[q] = *reinterpret_cast<uint32_t*>(&b);
  }
  return raw;
}

template <typename MT>
__device__ __forceinline__ void load8(const MT* p, float (&o)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&o)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) {
  bf16x8_to_float(*reinterpret_cast<const uint4*>(p), o);
}
template <typename MT>
__device__ __forceinline__ void store8(MT* p, const float (&o)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&o)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(o[0], o[1], o[2], o[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(o[4], o[5], o[6], o[7]);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&o)[8]) {
  *reinterpret_cast<uint4*>(p) = float_to_bf16x8(o);
}

struct PeerTables {
  int64_t grad[kMaxWorld];   // base of every rank's gradient pool (bf16)
  int64_t param[kMaxWorld];  // base of every rank's parameter pool (bf16)
  int64_t flags[kMaxWorld];  // base of every rank's flag array (uint32 [rows][world])
};

struct OptimArgs {
  float lr, beta1, beta2, eps, decay, step_size, bc2_sqrt, grad_scale;
  const int* step;       // device step count (bias corrections computed here) or null
  const uint32_t* base;  // device epoch base added to the epoch argument, or null
};

// Steps 1-4 above for one unit. kAdam = false: SGD on the fp32 master (m, v unused).
template <bool kAdam, typename MT>
__global__ void __launch_bounds__(kThreads) peer_update_kernel(
    PeerTables peers, const uint32_t* __restrict__ my_flags, int flag_row, int world, int my_rank, uint32_t epoch,
    int64_t offset, int64_t n, float* __restrict__ master, MT* __restrict__ m, MT* __restrict__ v, OptimArgs a,
    const float* __restrict__ grad_scale_ptr, int* __restrict__ nonfinite, int* status, uint64_t limit_ns) {
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  if (a.base != nullptr) epoch += *reinterpret_cast<const volatile uint32_t*>(a.base);
  if (kAdam && a.step != nullptr) {  // step count kept on the device (CUDA-graph replays)
    const double st = static_cast<double>(*a.step);
    a.step_size = static_cast<float>(a.lr / (1.0 - pow(static_cast<double>(a.beta1), st)));
    a.bc2_sqrt = static_cast<float>(sqrt(1.0 - pow(static_cast<double>(a.beta2), st)));
  }
  // 1. announce (every block stores the same value, so no block depends on another being
  //    resident), then every block waits for all ranks' announcements
  if (threadIdx.x < world) {
    __threadfence_system();
    uint32_t* peer = reinterpret_cast<uint32_t*>(peers.flags[threadIdx.x]);
    flag_store_release(peer + flag_row * world + my_rank, epoch);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* f = my_flags + flag_row * world + threadIdx.x;
    const uint64_t start = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
      if (static_cast<int32_t>(flag_load_acquire(f) - epoch) >= 0) break;
      if ((i & 63u) == 63u && global_timer_ns() - start > limit_ns) {
        report_status(status, kTimeoutPeer);
        atomicExch(&s_abort, 1);
        break;
      }
    }
  }
  __syncthreads();
  if (s_abort) return;  // a peer never staged its gradients: leave every buffer as it is

  const float gs = a.grad_scale * (grad_scale_ptr != nullptr ? *grad_scale_ptr : 1.f);
  bool bad = false;
  const int64_t vecs = n / 8;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; q < vecs;
       q += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t e = offset + q * 8;  // element index in the pools
    // 2. fixed-order fp32 sum over ranks (all loads issued before the first add)
    uint4 raw[kMaxWorld];
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p < world) raw[p] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers.grad[p]) + e);
    }
    float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p < world) {
        float t[8];
        bf16x8_to_float(raw[p], t);
#pragma unroll
        for (int k = 0; k < 8; ++k) g[k] += t[k];
      }
    }
    // 3. optimizer on the owned slice
    const int64_t i = q * 8;  // element index in this rank's shard state
    float w[8];
    load8<float>(master + i, w);
    if constexpr (kAdam) {
      float mi[8], vi[8];
      load8<MT>(m + i, mi);
      load8<MT>(v + i, vi);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gk = g[k] * gs;
        mi[k] = a.beta1 * mi[k] + (1.f - a.beta1) * gk;
        vi[k] = a.beta2 * vi[k] + (1.f - a.beta2) * gk * gk;
        w[k] = w[k] * a.decay - a.step_size * mi[k] / (sqrtf(vi[k]) / a.bc2_sqrt + a.eps);
      }
      store8<MT>(m + i, mi);
      store8<MT>(v + i, vi);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gk = g[k] * gs;
        bad |= !isfinite(gk);
        w[k] -= a.lr * gk;
      }
    }
    store8<float>(master + i, w);
    // 4. the rounded parameter into every rank's replica
    const uint4 out = float_to_bf16x8(w);
#pragma unroll
    for (int p = 0; p < kMaxWorld; ++p) {
      if (p < world) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers.param[p]) + e) = out;
    }
  }
  if (bad && nonfinite != nullptr) atomicExch(nonfinite, 1);
  // this thread's peer stores are visible to every GPU before the kernel counts as complete, so a
  // barrier signalled by a later launch on the stream orders after them
  __threadfence_system();
}

PeerTables make_tables(const at::Tensor& peer_grad, const at::Tensor& peer_param, const at::Tensor& peer_flags,
                       int world) {
  TDSV_CHECK(peer_grad.device().is_cpu() && peer_param.device().is_cpu() && peer_flags.device().is_cpu(),
             "peer pointer tables are host int64 tensors");
  TDSV_CHECK(peer_grad.numel() == world && peer_param.numel() == world && peer_flags.numel() == world,
             "one pointer per rank");
  PeerTables t{};
  for (int p = 0; p < world; ++p) {
    t.grad[p] = peer_grad.data_ptr<int64_t>()[p];
    t.param[p] = peer_param.data_ptr<int64_t>()[p];
    t.flags[p] = peer_flags.data_ptr<int64_t>()[p];
    TDSV_CHECK(t.grad[p] % 16 == 0 && t.param[p] % 16 == 0 && t.flags[p] % 4 == 0, "peer pools must be 16-byte aligned");
  }
  return t;
}

int update_grid(int64_t vecs, int64_t max_blocks) {
  const int64_t want = (vecs + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, max_blocks)));
}

}  // namespace

// One unit's fused update. `offset` is the element offset of this rank's shard in the pools and
// `n` its length (a multiple of 8); master / m / v hold exactly that shard. `algo` 0 = AdamW,
// 1 = SGD. `max_blocks` bounds the CTAs the update takes from the compute running beside it.
void peer_update(const at::Tensor& peer_grad, const at::Tensor& peer_param, const at::Tensor& peer_flags,
                 const at::Tensor& my_flags, int64_t flag_row, int64_t my_rank, int64_t epoch, int64_t offset,
                 at::Tensor& master, const c10::optional<at::Tensor>& m, const c10::optional<at::Tensor>& v,
                 int64_t algo, double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
                 double grad_scale, const c10::optional<at::Tensor>& grad_scale_t,
                 const c10::optional<at::Tensor>& nonfinite, int64_t max_blocks,
                 const c10::optional<at::Tensor>& step_t, const c10::optional<at::Tensor>& epoch_base) {
  check_cuda_tensor(master, "master");
  check_cuda_tensor(my_flags, "my_flags");
  const int world = static_cast<int>(peer_grad.numel());
  TDSV_CHECK(world >= 1 && world <= kMaxWorld, "peer_update: 1..8 ranks");
  TDSV_CHECK(my_rank >= 0 && my_rank < world, "peer_update: rank out of range");
  TDSV_CHECK(master.scalar_type() == at::kFloat, "peer_update: fp32 master");
  const int64_t n = master.numel();
  TDSV_CHECK(n % 8 == 0 && offset % 8 == 0, "peer_update: shard offset and length must be multiples of 8");
  TDSV_CHECK(my_flags.scalar_type() == at::kInt && (flag_row + 1) * world <= my_flags.numel(),
             "peer_update: flag row out of range");
  TDSV_CHECK(reinterpret_cast<uintptr_t>(master.data_ptr()) % 16 == 0, "peer_update: master must be 16-byte aligned");
  PeerTables tables = make_tables(peer_grad, peer_param, peer_flags, world);
  const float* gsp = nullptr;
  if (grad_scale_t.has_value() && grad_scale_t->defined()) gsp = grad_scale_t->data_ptr<float>();
  int* nf = nullptr;
  if (nonfinite.has_value() && nonfinite->defined()) nf = nonfinite->data_ptr<int>();
  OptimArgs a{};  // NOLINT
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.decay = static_cast<float>(1.0 - lr * weight_decay);
  a.grad_scale = static_cast<float>(grad_scale);
  auto dev_scalar = [](const c10::optional<at::Tensor>& t, const char* name) -> const void* {
    if (!t.has_value() || !t->defined()) return nullptr;
    check_cuda_tensor(*t, name);
    TDSV_CHECK(t->scalar_type() == at::kInt && t->numel() >= 1, name, ": int32 device scalar");
    return t->data_ptr();
  };
  a.step = static_cast<const int*>(dev_scalar(step_t, "step_t"));
  a.base = static_cast<const uint32_t*>(dev_scalar(epoch_base, "epoch_base"));
  if (algo == 0) {
    const double bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
    a.step_size = static_cast<float>(lr / bc1);
    a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  }
  c10::cuda::CUDAGuard guard(master.device());
  const int grid = update_grid(n / 8, std::max<int64_t>(1, max_blocks));
  const auto fl = reinterpret_cast<const uint32_t*>(my_flags.data_ptr());
  const auto ep = static_cast<uint32_t>(epoch);
  const uint64_t limit = peer_wait_limit_ns();
  if (algo == 1) {
    peer_update_kernel<false, float><<<grid, kThreads, 0, stream()>>>(
        tables, fl, static_cast<int>(flag_row), world, static_cast<int>(my_rank), ep, offset, n,
        master.data_ptr<float>(), nullptr, nullptr, a, gsp, nf, status_word_ptr(), limit);
  } else {
    TDSV_CHECK(algo == 0, "peer_update: algo 0 (AdamW) or 1 (SGD)");
    TDSV_CHECK(m.has_value() && v.has_value(), "peer_update: AdamW needs both moments");
    check_cuda_tensor(*m, "m");
    check_cuda_tensor(*v, "v");
    TDSV_CHECK(m->numel() == n && v->numel() == n && m->scalar_type() == v->scalar_type(),
               "peer_update: moments match the master");
    if (m->scalar_type() == at::kFloat) {
      peer_update_kernel<true, float><<<grid, kThreads, 0, stream()>>>(
          tables, fl, static_cast<int>(flag_row), world, static_cast<int>(my_rank), ep, offset, n,
          master.data_ptr<float>(), m->data_ptr<float>(), v->data_ptr<float>(), a, gsp, nf, status_word_ptr(), limit);
    } else {
      TDSV_CHECK(m->scalar_type() == at::kBFloat16, "peer_update: fp32 or bf16 moments");
      peer_update_kernel<true, __nv_bfloat16><<<grid, kThreads, 0, stream()>>>(
          tables, fl, static_cast<int>(flag_row), world, static_cast<int>(my_rank), ep, offset, n,
          master.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(m->data_ptr()),
          reinterpret_cast<__nv_bfloat16*>(v->data_ptr()), a, gsp, nf, status_word_ptr(), limit);
    }
  }
  TDSV_LAUNCH_CHECK();
}

}  // namespace tdsv
