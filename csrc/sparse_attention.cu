// DeepSeek-V4 sparse attention forward on the 5th-generation tensor cores (sm_100a).
//
// Each query token attends, with all of its heads, to a short list of keys of its own: W window
// rows of the raw KV (window_indices / window_mask) and K selected rows of the compressed KV
// (compressed_indices, -1 = none), plus one sink logit per head that takes part in the softmax but
// carries no value. KV is one latent tensor [B, S, D] that serves as keys and values (MQA).
//
// Orientation: the gathered keys are the M side of every MMA, the heads the N side, so a token's
// heads share each gathered key tile and its D-wide accumulators fit tensor memory:
//   S^T[k, h] = K[k, :] . Q[h, :]          M = 128 keys, N = 64 heads, K = D   (K-major A and B)
//   O^T[d, h] += sum_k V^T[d, k] P^T[k, h]  M = 128 dims (D / 128 tiles), N = 64, K = 128 keys
//                                           (A = the same key tile read MN-major, B = P^T MN-major)
// One CTA per (token, batch row, group of 64 heads), 288 threads:
//   warps 0-3  softmax: thread i owns key row i of S^T (TMEM lane i). Per-head maxima and sums run
//              over the 128 rows with a halving shuffle reduction (62 shuffles for 64 columns)
//              and one shared-memory step across the four warps, in a fixed order. Online softmax in
//              the exp2 domain, seeded with the sink logit (m = sink, l = 1); the running maximum is
//              raised only when a tile exceeds it by more than 2^8, and only then is O^T rescaled
//              in tensor memory. P^T (bf16) goes to shared memory as the B operand of O^T. At the
//              end O / l is staged through shared memory and written as one contiguous
//              [64 heads x D] block; lse = (m + log2 l) ln 2 per head (natural log, sink included).
//   warp 4     MMA issuer (one elected thread). With two key buffers (D <= 256) S^T of tile t+1 is
//              issued before O^T of tile t, so the next score tile overlaps this tile's softmax.
//   warps 5-8  gather: key rows are copied with 16-byte cp.async straight into the 128-byte
//              swizzled operand layout (invalid rows are zero-filled and masked in the softmax).
// TMEM: S^T double-buffered at columns [0, 64) and [64, 128), O^T tile m at [128 + 64 m, +64).
// Every mbarrier wait is bounded: a timeout records a status code and the CTA drains.
//
// Replaces the Triton forward kernel _attention_forward_kernel of
// dsv41_train/models/dsv4/attention/sparse_attention.py:17-151 (reference path).
#include "common.cuh"
#include "tc_util.cuh"

namespace tdsv {

namespace {

constexpr int kKeys = 128;      // key tile (MMA M)
constexpr int kHeadsCta = 64;   // heads per CTA (MMA N)
constexpr int kKAtom = 128 * 128;  // [128 key rows x 64 dims] bf16, swizzled, bytes
constexpr int kQAtom = 64 * 128;   // [64 head rows x 64 dims]
constexpr int kSaThreads = 288;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.f;  // raise the running maximum only when a tile exceeds it by 2^8

enum : int { kSaWaitQ = 501, kSaWaitK, kSaWaitKEmpty, kSaWaitS, kSaWaitSFree, kSaWaitP, kSaWaitPV };

template <int D>
struct SaCfg {
  static constexpr int kAtoms = D / 64;
  static constexpr int kBufs = D <= 256 ? 2 : 1;  // key tiles in flight
  static constexpr int kOTiles = D / 128;
  static constexpr uint32_t kColO = 2 * kHeadsCta;
  static constexpr uint32_t kTmemCols = kColO + kOTiles * kHeadsCta <= 256 ? 256 : 512;
};

template <int D>
struct SaSmem {
  alignas(1024) uint8_t q[SaCfg<D>::kAtoms * kQAtom];
  alignas(1024) uint8_t k[SaCfg<D>::kBufs][SaCfg<D>::kAtoms * kKAtom];
  alignas(1024) uint8_t p[SaCfg<D>::kBufs][kKeys * 128];
  uint64_t q_full;
  uint64_t k_full[SaCfg<D>::kBufs];
  uint64_t k_empty[SaCfg<D>::kBufs];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t pv_done;
  const __nv_bfloat16* key_src[kKeys];  // gather table of the tile being loaded
  uint32_t key_ok[kKeys];
  float red[4][kHeadsCta];
  float m_run[kHeadsCta];
  float l_run[kHeadsCta];
  float alpha[kHeadsCta];
  int any_rescale;
  int fail;  // a softmax warp's bounded wait gave up: the four warps leave together
  uint32_t tmem_base;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void producer_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Reduce 64 per-thread columns over the 32 lanes of a warp by halving: afterwards lane l holds the
// results for columns 2l and 2l + 1 in v[0], v[1]. Fixed order, so sums are reproducible.
template <bool kMax>
__device__ __forceinline__ void halving_reduce64(float (&v)[64], int lane) {
#pragma unroll
  for (int w = 32, o = 16; o >= 1; w >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const float send = upper ? v[j] : v[j + w];
      const float keep = upper ? v[j + w] : v[j];
      const float recv = __shfl_xor_sync(0xffffffffu, send, o);
      v[j] = kMax ? fmaxf(keep, recv) : keep + recv;
    }
  }
}

struct SaParams {
  const __nv_bfloat16* q;        // [B, L, H, D]
  const __nv_bfloat16* kv;       // [B, S, D]
  const int64_t* win_idx;        // [B, L, W]
  const uint8_t* win_mask;       // [B, L, W]
  const __nv_bfloat16* comp;     // [B, C, D] or null
  const int64_t* comp_idx;       // [B, L, K] or null
  const float* sinks;            // [H]
  __nv_bfloat16* out;            // [B, L, H, D]
  float* lse;                    // [B, L, H]
  int L, H, S, W, C, K;
  float scale_log2;              // D^-1/2 log2(e)
  int* status;
};

// Global source row of entry j of token (b, t): window entries first, then the selected ones.
template <int D>
__device__ __forceinline__ const __nv_bfloat16* key_row(const SaParams& p, int b, int t, int j, bool& ok) {
  const int64_t tok = static_cast<int64_t>(b) * p.L + t;
  if (j < p.W) {
    const int64_t idx = p.win_idx[tok * p.W + j];
    ok = p.win_mask[tok * p.W + j] != 0 && idx >= 0 && idx < p.S;
    return p.kv + (static_cast<int64_t>(b) * p.S + (ok ? idx : 0)) * D;
  }
  if (j < p.W + p.K) {
    const int64_t idx = p.comp_idx[tok * p.K + (j - p.W)];
    ok = idx >= 0 && idx < p.C;
    return p.comp + (static_cast<int64_t>(b) * p.C + (ok ? idx : 0)) * D;
  }
  ok = false;
  return p.kv;
}

template <int D>
__global__ void __launch_bounds__(kSaThreads, 1) sparse_attn_fwd_kernel(const SaParams p) {
  using Cfg = SaCfg<D>;
  constexpr int kBufs = Cfg::kBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SaSmem<D>& sm = *reinterpret_cast<SaSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int t = blockIdx.x, b = blockIdx.y, hg = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int entries = p.W + p.K;
  const int tiles = (entries + kKeys - 1) / kKeys;
  const int64_t tok = static_cast<int64_t>(b) * p.L + t;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 128);
    for (int i = 0; i < kBufs; ++i) {
      mbar_init(&sm.k_full[i], 128);
      mbar_init(&sm.k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 128);
    }
    mbar_init(&sm.p_full, 128);
    mbar_init(&sm.pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&sm.tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) sm.fail = 0;
  if (threadIdx.x < kHeadsCta) {
    const int h = hg * kHeadsCta + threadIdx.x;
    sm.m_run[threadIdx.x] = h < p.H ? p.sinks[h] * kLog2e : 0.f;
    sm.l_run[threadIdx.x] = 1.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  bool failed = false;

  if (warp >= 5) {
    // ---------------- gather producers ----------------
    const int pt = threadIdx.x - 160;  // 0..127
    {
      const __nv_bfloat16* qsrc = p.q + (tok * p.H + hg * kHeadsCta) * D;
      const uint32_t qbase = smem_u32(sm.q);
      for (int c = pt; c < kHeadsCta * (D / 8); c += 128) {
        const int row = c / (D / 8), ch = c % (D / 8);
        const bool ok = hg * kHeadsCta + row < p.H;
        cp_async16(qbase + (ch >> 3) * kQAtom + swz(row, ch & 7), qsrc + (ok ? row * D + ch * 8 : 0), ok);
      }
      cp_async_commit();
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&sm.q_full);
    }
    for (int it = 0; it < tiles; ++it) {
      const int buf = it % kBufs;
      if (it >= kBufs && !warp_wait(&sm.k_empty[buf], ((it / kBufs) - 1) & 1, p.status, kSaWaitKEmpty)) {
        failed = true;
        break;
      }
      const uint32_t kbase = smem_u32(sm.k[buf]);
      {  // one source row per thread, then consecutive threads copy consecutive chunks of a row
        bool ok;
        sm.key_src[pt] = key_row<D>(p, b, t, it * kKeys + pt, ok);
        sm.key_ok[pt] = ok ? 1u : 0u;
      }
      producer_sync();
      for (int c = pt; c < kKeys * (D / 8); c += 128) {
        const int row = c / (D / 8), ch = c % (D / 8);
        cp_async16(kbase + (ch >> 3) * kKAtom + swz(row, ch & 7), sm.key_src[row] + ch * 8, sm.key_ok[row] != 0);
      }
      cp_async_commit();
      cp_async_wait_all();
      fence_proxy_async_smem();
      producer_sync();  // the gather table is read by every producer before the next tile rewrites it
      mbar_arrive(&sm.k_full[buf]);
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    const bool leader = elect_one();
    const uint32_t idesc_s = make_idesc_bf16(kKeys, kHeadsCta, false, false);
    const uint32_t idesc_o = make_idesc_bf16(128, kHeadsCta, true, true);
    const uint32_t qbase = smem_u32(sm.q);
    auto issue_s = [&](int it) -> bool {
      const int buf = it % kBufs;
      if (!warp_wait(&sm.k_full[buf], (it / kBufs) & 1, p.status, kSaWaitK)) return false;
      if (it >= 2 && !warp_wait(&sm.s_free[it & 1], ((it >> 1) - 1) & 1, p.status, kSaWaitSFree)) return false;
      tc_fence_after();
      if (leader) {
        const uint32_t kb = smem_u32(sm.k[buf]);
#pragma unroll 4
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16(tmem + (it & 1) * kHeadsCta, kmajor_desc(kb, kk, kKAtom), kmajor_desc(qbase, kk, kQAtom), idesc_s,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[it & 1]);
      }
      __syncwarp();
      return true;
    };
    bool ok = warp_wait(&sm.q_full, 0, p.status, kSaWaitQ);
    if (ok) ok = issue_s(0);
    for (int it = 0; ok && it < tiles; ++it) {
      if (kBufs == 2 && it + 1 < tiles && !issue_s(it + 1)) {
        ok = false;
        break;
      }
      if (!warp_wait(&sm.p_full, it & 1, p.status, kSaWaitP)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int buf = it % kBufs;
      if (leader) {
        const uint32_t kb = smem_u32(sm.k[buf]);
        const uint32_t pb = smem_u32(sm.p[buf]);
#pragma unroll
        for (int m = 0; m < Cfg::kOTiles; ++m) {
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            umma_f16(tmem + Cfg::kColO + m * kHeadsCta, mnmajor_desc(kb + 2 * m * kKAtom, kk, kKAtom),
                     mnmajor_desc(pb, kk, kKeys * 128), idesc_o, (it > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&sm.k_empty[buf]);
        umma_commit(&sm.pv_done);
      }
      __syncwarp();
      if (kBufs == 1 && it + 1 < tiles && !issue_s(it + 1)) {
        ok = false;
        break;
      }
    }
    failed = !ok;
  } else {
    // ---------------- softmax (warps 0-3, thread = key row = TMEM lane) ----------------
    const int row = threadIdx.x;  // 0..127
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    for (int it = 0; it < tiles; ++it) {
      const int buf = it % kBufs;
      if (!warp_wait(&sm.s_full[it & 1], (it >> 1) & 1, p.status, kSaWaitS)) sm.fail = 1;
      softmax_sync();
      if (sm.fail) {
        failed = true;
        break;
      }
      tc_fence_after();
      float s[64];
      {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + (it & 1) * kHeadsCta, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(r[j]);
        tmem_ld_32x32b_x32(lane_base + (it & 1) * kHeadsCta + 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) s[32 + j] = __uint_as_float(r[j]);
      }
      tc_fence_before();
      mbar_arrive(&sm.s_free[it & 1]);
      bool valid;
      (void)key_row<D>(p, b, t, it * kKeys + row, valid);
#pragma unroll
      for (int j = 0; j < 64; ++j) s[j] = valid ? s[j] * p.scale_log2 : -INFINITY;
      // per-head tile maximum
      float v[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = s[j];
      halving_reduce64<true>(v, lane);
      sm.red[warp][2 * lane] = v[0];
      sm.red[warp][2 * lane + 1] = v[1];
      if (row == 0) sm.any_rescale = 0;
      softmax_sync();
      if (row < kHeadsCta) {
        const float tmax = fmaxf(fmaxf(sm.red[0][row], sm.red[1][row]), fmaxf(sm.red[2][row], sm.red[3][row]));
        const float mold = sm.m_run[row];
        float a = 1.f;
        if (tmax > mold + kRescaleLog2) {
          a = ex2_approx(mold - tmax);
          sm.m_run[row] = tmax;
          sm.any_rescale = 1;
        }
        sm.alpha[row] = a;
      }
      softmax_sync();
      // P = 2^(s - m) (bf16) into the MN-major P^T tile: row = key, 64 head columns
      float pr[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) pr[j] = ex2_approx(s[j] - sm.m_run[j]);
      // the previous PV MMA has finished with O^T and with this P buffer
      if (it > 0 && !warp_wait(&sm.pv_done, (it - 1) & 1, p.status, kSaWaitPV)) sm.fail = 1;
      softmax_sync();
      if (sm.fail) {
        failed = true;
        break;
      }
      {
        uint8_t* prow = sm.p[buf] + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(pr[8 * c + 2 * q], pr[8 * c + 2 * q + 1]);
            wp[q] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = w;
        }
      }
      if (it > 0 && sm.any_rescale) {
        tc_fence_after();
#pragma unroll
        for (int m = 0; m < Cfg::kOTiles; ++m) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t r[32];
            const uint32_t addr = lane_base + Cfg::kColO + m * kHeadsCta + half * 32;
            tmem_ld_32x32b_x32(addr, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * sm.alpha[half * 32 + j]);
            tmem_st_32x32b_x32(addr, r);
          }
        }
        tmem_st_wait();
      }
      // per-head sums of this tile's probabilities (the bf16-rounded values the MMA uses)
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(pr[j]));
      halving_reduce64<false>(v, lane);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full);
      sm.red[warp][2 * lane] = v[0];
      sm.red[warp][2 * lane + 1] = v[1];
      softmax_sync();
      if (row < kHeadsCta) {
        const float tsum = ((sm.red[0][row] + sm.red[1][row]) + sm.red[2][row]) + sm.red[3][row];
        sm.l_run[row] = sm.l_run[row] * sm.alpha[row] + tsum;
      }
      softmax_sync();
    }
    if (!failed && !warp_wait(&sm.pv_done, (tiles - 1) & 1, p.status, kSaWaitPV)) sm.fail = 1;
    softmax_sync();
    if (!sm.fail) {
      tc_fence_after();
      // O / l staged as bf16 [64 heads x D] over the (now idle) key buffer, then one contiguous store
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(sm.k[0]);
#pragma unroll 1
      for (int m = 0; m < Cfg::kOTiles; ++m) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_base + Cfg::kColO + m * kHeadsCta + half * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int h = half * 32 + j;
            stage[h * D + m * 128 + row] = __float2bfloat16_rn(__uint_as_float(r[j]) / sm.l_run[h]);
          }
        }
      }
      softmax_sync();
      const int heads_here = min(kHeadsCta, p.H - hg * kHeadsCta);
      const uint4* src = reinterpret_cast<const uint4*>(stage);
      uint4* dst = reinterpret_cast<uint4*>(p.out + (tok * p.H + hg * kHeadsCta) * D);
      for (int i = row; i < heads_here * D / 8; i += 128) dst[i] = src[i];
      if (row < heads_here) {
        p.lse[tok * p.H + hg * kHeadsCta + row] = (sm.m_run[row] + __log2f(sm.l_run[row])) * kLn2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  (void)failed;
}

template <int D>
void launch_fwd(const SaParams& prm, int L, int B, int groups) {
  const size_t smem = sizeof(SaSmem<D>) + 1024;
  static bool configured = false;
  if (!configured) {
    TDSV_CUDA_CHECK(cudaFuncSetAttribute(sparse_attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    configured = true;
  }
  sparse_attn_fwd_kernel<D><<<dim3(L, B, groups), kSaThreads, smem, stream()>>>(prm);
}

}  // namespace

// out [B, L, H, D] bf16, lse [B, L, H] fp32.
std::vector<at::Tensor> sparse_attention_fwd(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx,
                                             const at::Tensor& win_mask, const c10::optional<at::Tensor>& comp,
                                             const c10::optional<at::Tensor>& comp_idx, const at::Tensor& sinks) {
  check_cuda_tensor(q, "q");
  check_cuda_tensor(kv, "kv");
  check_cuda_tensor(win_idx, "window_indices");
  check_cuda_tensor(win_mask, "window_mask");
  check_cuda_tensor(sinks, "sinks");
  TDSV_CHECK(q.dim() == 4 && kv.dim() == 3, "sparse_attention_fwd: q [B, L, H, D], kv [B, S, D]");
  const int B = static_cast<int>(q.size(0)), L = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2));
  const int D = static_cast<int>(q.size(3));
  TDSV_CHECK(q.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16, "sparse_attention_fwd: bf16");
  TDSV_CHECK(D == 128 || D == 256 || D == 512, "sparse_attention_fwd: head dim 128, 256 or 512");
  TDSV_CHECK(kv.size(0) == B && kv.size(2) == D, "sparse_attention_fwd: kv shape");
  TDSV_CHECK(win_idx.scalar_type() == at::kLong && win_idx.dim() == 3 && win_idx.size(0) == B && win_idx.size(1) == L,
             "sparse_attention_fwd: window_indices int64 [B, L, W]");
  TDSV_CHECK(win_mask.scalar_type() == at::kBool && win_mask.sizes() == win_idx.sizes(),
             "sparse_attention_fwd: window_mask bool [B, L, W]");
  TDSV_CHECK(sinks.scalar_type() == at::kFloat && sinks.numel() == H, "sparse_attention_fwd: sinks fp32 [H]");
  SaParams prm{};
  prm.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  prm.kv = reinterpret_cast<const __nv_bfloat16*>(kv.data_ptr());
  prm.win_idx = win_idx.data_ptr<int64_t>();
  prm.win_mask = reinterpret_cast<const uint8_t*>(win_mask.data_ptr());
  prm.sinks = sinks.data_ptr<float>();
  prm.L = L;
  prm.H = H;
  prm.S = static_cast<int>(kv.size(1));
  prm.W = static_cast<int>(win_idx.size(2));
  prm.K = 0;
  prm.C = 0;
  if (comp.has_value() && comp->defined() && comp_idx.has_value() && comp_idx->defined()) {
    check_cuda_tensor(*comp, "compressed_kv");
    check_cuda_tensor(*comp_idx, "compressed_indices");
    TDSV_CHECK(comp->scalar_type() == at::kBFloat16 && comp->dim() == 3 && comp->size(0) == B && comp->size(2) == D,
               "sparse_attention_fwd: compressed_kv bf16 [B, C, D]");
    TDSV_CHECK(comp_idx->scalar_type() == at::kLong && comp_idx->dim() == 3 && comp_idx->size(0) == B &&
                   comp_idx->size(1) == L,
               "sparse_attention_fwd: compressed_indices int64 [B, L, K]");
    prm.comp = reinterpret_cast<const __nv_bfloat16*>(comp->data_ptr());
    prm.comp_idx = comp_idx->data_ptr<int64_t>();
    prm.C = static_cast<int>(comp->size(1));
    prm.K = static_cast<int>(comp_idx->size(2));
  }
  TDSV_CHECK(prm.W + prm.K > 0, "sparse_attention_fwd: no keys");
  prm.scale_log2 = static_cast<float>(std::pow(static_cast<double>(D), -0.5)) * kLog2e;
  prm.status = status_word_ptr();
  auto out = at::empty({B, L, H, D}, q.options());
  auto lse = at::empty({B, L, H}, q.options().dtype(at::kFloat));
  prm.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  prm.lse = lse.data_ptr<float>();
  if (B * L == 0) return {out, lse};
  c10::cuda::CUDAGuard guard(q.device());
  const int groups = (H + kHeadsCta - 1) / kHeadsCta;
  if (D == 128) launch_fwd<128>(prm, L, B, groups);
  else if (D == 256) launch_fwd<256>(prm, L, B, groups);
  else launch_fwd<512>(prm, L, B, groups);
  TDSV_LAUNCH_CHECK();
  return {out, lse};
}

}  // namespace tdsv
