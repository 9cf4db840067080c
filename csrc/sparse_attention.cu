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
  uint64_t table_full;  // the producers finished the token's entry table
  uint64_t k_full[SaCfg<D>::kBufs];
  uint64_t k_empty[SaCfg<D>::kBufs];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t pv_done;
  float red[4][kHeadsCta];
  float m_run[kHeadsCta];
  float l_run[kHeadsCta];
  float alpha[kHeadsCta];
  int any_rescale;
  int fail;   // a softmax warp's bounded wait gave up: the four warps leave together
  int pfail;  // the same for the four producer warps
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

// The token's entry table, built once per CTA in its prologue (dynamic shared memory after the
// fixed part): entry j < W is window row win_idx[j] of the raw KV, entry j >= W is compressed row
// comp_idx[j - W]; -1 marks a masked, negative or out-of-range entry. The gather and the softmax
// read it instead of the index arrays in global memory.
__device__ __forceinline__ int32_t entry_of(const SaParams& p, int b, int t, int j) {
  const int64_t tok = static_cast<int64_t>(b) * p.L + t;
  if (j < p.W) {
    const int64_t idx = p.win_idx[tok * p.W + j];
    return p.win_mask[tok * p.W + j] != 0 && idx >= 0 && idx < p.S ? static_cast<int32_t>(idx) : -1;
  }
  const int64_t idx = p.comp_idx[tok * p.K + (j - p.W)];
  return idx >= 0 && idx < p.C ? static_cast<int32_t>(idx) : -1;
}
// The 128 producer threads fill the table; the index loads of up to eight entries per thread are
// issued before any of them is used, so a token pays about one global-memory latency for it.
__device__ __forceinline__ void build_table(const SaParams& p, int b, int t, int32_t* ent, int pt) {
  const int entries = p.W + p.K;
  for (int base = pt; base < entries; base += 128 * 8) {
    int32_t e[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = base + u * 128;
      e[u] = j < entries ? entry_of(p, b, t, j) : -1;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = base + u * 128;
      if (j < entries) ent[j] = e[u];
    }
  }
}
__device__ __forceinline__ int32_t entry_at(const SaParams& p, const int32_t* ent, int j) {
  return j < p.W + p.K ? ent[j] : -1;
}
// Global row of entry j (a valid in-range row even for e < 0, whose copy is zero-filled).
template <int D>
__device__ __forceinline__ const __nv_bfloat16* entry_src(const SaParams& p, int b, int j, int32_t e) {
  const int64_t row = e < 0 ? 0 : e;
  return j < p.W ? p.kv + (static_cast<int64_t>(b) * p.S + row) * D : p.comp + (static_cast<int64_t>(b) * p.C + row) * D;
}

template <int D>
__global__ void __launch_bounds__(kSaThreads, 1) sparse_attn_fwd_kernel(const SaParams p) {
  using Cfg = SaCfg<D>;
  constexpr int kBufs = Cfg::kBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SaSmem<D>& sm = *reinterpret_cast<SaSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int32_t* ent = reinterpret_cast<int32_t*>(&sm + 1);
  const int t = blockIdx.x, b = blockIdx.y, hg = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int entries = p.W + p.K;
  const int tiles = (entries + kKeys - 1) / kKeys;
  const int64_t tok = static_cast<int64_t>(b) * p.L + t;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 128);
    mbar_init(&sm.table_full, 128);
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
  if (threadIdx.x == 0) {
    sm.fail = 0;
    sm.pfail = 0;
  }
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
      // the entry table is built while Q is in flight; the softmax warps wait for it on table_full
      build_table(p, b, t, ent, pt);
      mbar_arrive(&sm.table_full);
      producer_sync();
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&sm.q_full);
    }
    for (int it = 0; it < tiles; ++it) {
      const int buf = it % kBufs;
      // every producer warp waits, then the four agree before any named barrier below
      if (it >= kBufs && !warp_wait(&sm.k_empty[buf], ((it / kBufs) - 1) & 1, p.status, kSaWaitKEmpty)) sm.pfail = 1;
      producer_sync();
      if (sm.pfail) {
        failed = true;
        break;
      }
      const uint32_t kbase = smem_u32(sm.k[buf]);
      // consecutive threads copy consecutive 16-byte chunks of a key row
      for (int c = pt; c < kKeys * (D / 8); c += 128) {
        const int row = c / (D / 8), ch = c % (D / 8);
        const int j = it * kKeys + row;
        const int32_t e = entry_at(p, ent, j);
        cp_async16(kbase + (ch >> 3) * kKAtom + swz(row, ch & 7), entry_src<D>(p, b, j, e) + ch * 8, e >= 0);
      }
      cp_async_commit();
      cp_async_wait_all();
      fence_proxy_async_smem();
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
    if (!warp_wait(&sm.table_full, 0, p.status, kSaWaitQ)) sm.fail = 1;
    softmax_sync();
    failed = sm.fail != 0;
    for (int it = 0; it < tiles && !failed; ++it) {
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
      const bool valid = entry_at(p, ent, it * kKeys + row) >= 0;
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

// =============================================================================================
// Backward
// =============================================================================================
// One CTA per (token, batch row, group of 64 heads), 288 threads, the same roles as the forward.
// Per key tile (with P = exp2(S c - lse log2 e), Delta[h] = O[h] . dO[h], dS = P (dP - Delta)):
//   S^T = K Q^T, dP^T = V dO^T        M = 128 keys, N = 64 heads, K = D       (TMEM [0,64), [64,128))
//   dQ^T += K^T (scale dS^T)          M = 128 dims (D / 128 tiles), N = 64, K = 128 keys
//   dKV[:, chunk] = P^T dO[:, chunk] + (scale dS^T) Q[:, chunk]
//                                     M = 128 keys, N = 64 dims per chunk, K = 64 heads
// P^T (bf16) goes to tensor memory as the A operand of dKV; scale dS^T (bf16) to shared memory,
// where it is both the MN-major B operand of dQ^T and the K-major A operand of dKV. Key rows are
// gathered D / 2 dims at a time: with D = 512 one half-buffer is resident and the first half is
// gathered again for its dQ^T tiles (shared memory holds Q, dO, one half and dS^T); with D <= 256
// both halves stay resident. The compute warps drain each dKV chunk from tensor memory and add it
// to the fp32 gradient of its KV row with 16-byte vector reductions (the rows a tile shares with
// other tokens meet there, as in the reference's default atomic path). dQ is written once per
// (token, head) and the sink gradient partial -exp(sink - lse) Delta per (token, head).
// TMEM: S [0,64), dP [64,128), dQ^T [128, 128 + 64 D/128), dKV chunk (64 cols), P^T (32 cols).
//
// Replaces _attention_backward_kernel of dsv41_train/models/dsv4/attention/sparse_attention.py:152-323.
enum : int { kSbWaitQ = 521, kSbWaitK, kSbWaitKEmpty, kSbWaitS, kSbWaitSFree, kSbWaitDs, kSbWaitDsFree, kSbWaitDkv,
             kSbWaitDkvFree, kSbWaitDq };

template <int D>
struct SbCfg {
  static constexpr int kAtoms = D / 64;
  static constexpr int kHalfAtoms = kAtoms / 2;          // atoms of one gathered half (D / 2 dims)
  static constexpr int kBufs = D <= 256 ? 2 : 1;          // resident halves
  static constexpr int kOTiles = D / 128;                 // dQ^T tiles
  static constexpr int kChunks = D / 64;                  // dKV chunks of 64 dims
  static constexpr uint32_t kColS = 0, kColDp = 64, kColDq = 128;
  static constexpr uint32_t kColDkv = kColDq + kOTiles * 64;
  static constexpr uint32_t kColP = kColDkv + 64;
  static_assert(kColP + 32 <= 512, "tensor memory budget");
};

template <int D>
struct SbSmem {
  alignas(1024) uint8_t q[SbCfg<D>::kAtoms * kQAtom];
  alignas(1024) uint8_t dout[SbCfg<D>::kAtoms * kQAtom];
  alignas(1024) uint8_t k[SbCfg<D>::kBufs][SbCfg<D>::kHalfAtoms * kKAtom];  // contiguous halves
  alignas(1024) uint8_t ds[kKeys * 128];
  uint64_t qd_full;
  uint64_t table_full;
  uint64_t k_full[SbCfg<D>::kBufs];
  uint64_t k_empty[SbCfg<D>::kBufs];
  uint64_t s_full, s_free, ds_full, ds_free, dkv_full, dkv_free, dq_full;
  float lse2[kHeadsCta];
  float delta[kHeadsCta];
  float dpart[2][kHeadsCta];
  int fail;   // compute warps leave together after a failed wait
  int pfail;  // producer warps likewise
  uint32_t tmem_base;
};

struct SbParams {
  SaParams f;                     // inputs as in the forward (out / lse are read here)
  const __nv_bfloat16* dout;      // [B, L, H, D]
  __nv_bfloat16* dq;              // [B, L, H, D]
  float* dkv;                     // [B, S, D] fp32, accumulated
  float* dcomp;                   // [B, C, D] fp32, accumulated, or null
  float* dsink_part;              // [B, L, H]
  float scale;                    // D^-1/2
  // ordered (deterministic) mode: per-edge dKV rows [B, chunk, W + K, groups, D] fp32 instead of
  // reductions; the CTAs cover tokens [t0, t0 + chunk) and ordered_edge_reduce sums the edges
  float* edges;
  int t0, chunk;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

template <int D>
__global__ void __launch_bounds__(kSaThreads, 1) sparse_attn_bwd_kernel(const SbParams sp) {
  using Cfg = SbCfg<D>;
  constexpr int kBufs = Cfg::kBufs;
  constexpr int kLoadsPerTile = kBufs == 1 ? 3 : 2;  // D = 512: half 0, half 1, half 0 again
  const SaParams& p = sp.f;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SbSmem<D>& sm = *reinterpret_cast<SbSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int32_t* ent = reinterpret_cast<int32_t*>(&sm + 1);
  const int t = sp.t0 + blockIdx.x, b = blockIdx.y, hg = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.W + p.K + kKeys - 1) / kKeys;
  const int64_t tok = static_cast<int64_t>(b) * p.L + t;
  const int heads_here = min(kHeadsCta, p.H - hg * kHeadsCta);

  if (threadIdx.x == 0) {
    mbar_init(&sm.qd_full, 128);
    mbar_init(&sm.table_full, 128);
    for (int i = 0; i < kBufs; ++i) {
      mbar_init(&sm.k_full[i], 128);
      mbar_init(&sm.k_empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, 128);
    mbar_init(&sm.ds_full, 128);
    mbar_init(&sm.ds_free, 1);
    mbar_init(&sm.dkv_full, 1);
    mbar_init(&sm.dkv_free, 128);
    mbar_init(&sm.dq_full, 1);
    fence_barrier_init();
    sm.fail = 0;
    sm.pfail = 0;
  }
  if (warp == 4) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // which half a load carries, and into which buffer
  auto load_half = [&](int n) { return kBufs == 1 ? ((n % 3) == 1 ? 1 : 0) : (n % 2); };
  auto load_buf = [&](int n) { return kBufs == 1 ? 0 : (n % 2); };
  auto load_use = [&](int n) { return kBufs == 1 ? n : n / 2; };  // earlier loads into the same buffer

  if (warp >= 5) {
    // ---------------- gather producers ----------------
    const int pt = threadIdx.x - 160;
    {
      const __nv_bfloat16* qsrc = p.q + (tok * p.H + hg * kHeadsCta) * D;
      const __nv_bfloat16* dsrc = sp.dout + (tok * p.H + hg * kHeadsCta) * D;
      const uint32_t qb = smem_u32(sm.q), db = smem_u32(sm.dout);
      for (int c = pt; c < kHeadsCta * (D / 8); c += 128) {
        const int row = c / (D / 8), ch = c % (D / 8);
        const bool ok = row < heads_here;
        const uint32_t off = (ch >> 3) * kQAtom + swz(row, ch & 7);
        cp_async16(qb + off, qsrc + (ok ? row * D + ch * 8 : 0), ok);
        cp_async16(db + off, dsrc + (ok ? row * D + ch * 8 : 0), ok);
      }
      cp_async_commit();
      build_table(p, b, t, ent, pt);
      mbar_arrive(&sm.table_full);
      producer_sync();
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&sm.qd_full);
    }
    for (int it = 0; it < tiles; ++it) {
      for (int j = 0; j < kLoadsPerTile; ++j) {
        const int n = it * kLoadsPerTile + j;
        const int buf = load_buf(n), half = load_half(n), use = load_use(n);
        if (use >= 1 && !warp_wait(&sm.k_empty[buf], (use - 1) & 1, p.status, kSbWaitKEmpty)) sm.pfail = 1;
        producer_sync();
        if (sm.pfail) break;
        const uint32_t kb = smem_u32(sm.k[buf]);
        constexpr int kHalfChunks = D / 16;  // 16-byte chunks per half row
        for (int c = pt; c < kKeys * kHalfChunks; c += 128) {
          const int row = c / kHalfChunks, ch = c % kHalfChunks;
          const int entry = it * kKeys + row;
          const int32_t e = entry_at(p, ent, entry);
          cp_async16(kb + (ch >> 3) * kKAtom + swz(row, ch & 7), entry_src<D>(p, b, entry, e) + half * (D / 2) + ch * 8,
                     e >= 0);
        }
        cp_async_commit();
        cp_async_wait_all();
        fence_proxy_async_smem();
        mbar_arrive(&sm.k_full[buf]);
      }
      if (sm.pfail) break;
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    const bool leader = elect_one();
    const uint32_t idesc_sdp = make_idesc_bf16(kKeys, kHeadsCta, false, false);
    const uint32_t idesc_dq = make_idesc_bf16(128, kHeadsCta, true, true);
    const uint32_t idesc_dkv = make_idesc_bf16(kKeys, 64, false, true);
    const uint32_t qb = smem_u32(sm.q), db = smem_u32(sm.dout), dsb = smem_u32(sm.ds);
    bool ok = warp_wait(&sm.qd_full, 0, p.status, kSbWaitQ);
    auto wait_load = [&](int n) {
      return warp_wait(&sm.k_full[load_buf(n)], load_use(n) & 1, p.status, kSbWaitK);
    };
    // S^T and dP^T over the dims of one gathered half
    auto issue_sdp = [&](int n, bool first) {
      const int half = load_half(n);
      const uint32_t kb = smem_u32(sm.k[load_buf(n)]);
      if (leader) {
#pragma unroll 4
        for (int kk = 0; kk < D / 32; ++kk) {
          const uint64_t a = kmajor_desc(kb, kk, kKAtom);
          const int gk = half * (D / 32) + kk;  // k-step in the full head dim
          umma_f16(tmem + Cfg::kColS, a, kmajor_desc(qb, gk, kQAtom), idesc_sdp, (first && kk == 0) ? 0u : 1u);
          umma_f16(tmem + Cfg::kColDp, a, kmajor_desc(db, gk, kQAtom), idesc_sdp, (first && kk == 0) ? 0u : 1u);
        }
      }
    };
    // dQ^T tiles whose dims lie in the resident half(s)
    auto issue_dq = [&](int n, int m_lo, int m_hi, bool first_tile) {
      const uint32_t kb0 = smem_u32(sm.k[0]);
      if (leader) {
        for (int m = m_lo; m < m_hi; ++m) {
          // atom of dims [128 m, 128 m + 64): with one buffer it is relative to the resident half
          const int atom = kBufs == 1 ? 2 * m - load_half(n) * Cfg::kHalfAtoms : 2 * m;
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            umma_f16(tmem + Cfg::kColDq + m * 64, mnmajor_desc(kb0 + atom * kKAtom, kk, kKAtom),
                     mnmajor_desc(dsb, kk, kKeys * 128), idesc_dq, (first_tile && kk == 0) ? 0u : 1u);
          }
        }
      }
    };
    int g = 0;  // dKV chunk counter
    for (int it = 0; ok && it < tiles; ++it) {
      const int n0 = it * kLoadsPerTile;
      if (it > 0 && !warp_wait(&sm.s_free, (it - 1) & 1, p.status, kSbWaitSFree)) { ok = false; break; }
      // S^T, dP^T: half 0 then half 1
      if (!wait_load(n0)) { ok = false; break; }
      tc_fence_after();
      issue_sdp(n0, true);
      if (kBufs == 1 && leader) umma_commit(&sm.k_empty[0]);
      __syncwarp();
      if (!wait_load(n0 + 1)) { ok = false; break; }
      tc_fence_after();
      issue_sdp(n0 + 1, false);
      if (leader) umma_commit(&sm.s_full);
      __syncwarp();
      // P^T (TMEM) and dS^T (shared) are ready
      if (!warp_wait(&sm.ds_full, it & 1, p.status, kSbWaitDs)) { ok = false; break; }
      tc_fence_after();
      if (kBufs == 1) {
        issue_dq(n0 + 1, Cfg::kOTiles / 2, Cfg::kOTiles, it == 0);  // tiles of the resident half 1
        if (leader) umma_commit(&sm.k_empty[0]);
      } else {
        issue_dq(n0 + 1, 0, Cfg::kOTiles, it == 0);                 // both halves resident
        if (leader) {
          umma_commit(&sm.k_empty[0]);
          umma_commit(&sm.k_empty[1]);
        }
      }
      __syncwarp();
      // dKV chunks of 64 dims
      for (int c = 0; c < Cfg::kChunks; ++c, ++g) {
        if (g > 0 && !warp_wait(&sm.dkv_free, (g - 1) & 1, p.status, kSbWaitDkvFree)) { ok = false; break; }
        tc_fence_after();
        if (leader) {
          const uint32_t bq = qb + c * kQAtom, bd = db + c * kQAtom;
#pragma unroll
          for (int kk = 0; kk < kHeadsCta / 16; ++kk) {
            umma_f16_ts(tmem + Cfg::kColDkv, tmem + Cfg::kColP + kk * 8, mnmajor_desc(bd, kk, kQAtom), idesc_dkv,
                        kk > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < kHeadsCta / 16; ++kk) {
            umma_f16(tmem + Cfg::kColDkv, kmajor_desc(dsb, kk, kKeys * 128), mnmajor_desc(bq, kk, kQAtom), idesc_dkv,
                     1u);
          }
          umma_commit(&sm.dkv_full);
          if (c == Cfg::kChunks - 1) umma_commit(&sm.ds_free);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (kBufs == 1) {  // half 0 again for its dQ^T tiles
        if (!wait_load(n0 + 2)) { ok = false; break; }
        tc_fence_after();
        issue_dq(n0 + 2, 0, Cfg::kOTiles / 2, it == 0);
        if (leader) umma_commit(&sm.k_empty[0]);
        __syncwarp();
      }
    }
    if (ok && leader) umma_commit(&sm.dq_full);
    __syncwarp();
  } else {
    // ---------------- compute warps 0-3 (thread = key row = TMEM lane) ----------------
    const int row = threadIdx.x;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    // Delta[h] = O[h] . dO[h] (two threads per head), lse in the exp2 domain, sink-gradient partial
    {
      const int h = row >> 1, part = row & 1;
      float acc = 0.f;
      if (h < heads_here) {
        const __nv_bfloat16* o = p.out + (tok * p.H + hg * kHeadsCta + h) * D + part * (D / 2);
        const __nv_bfloat16* g = sp.dout + (tok * p.H + hg * kHeadsCta + h) * D + part * (D / 2);
        for (int d = 0; d < D / 2; d += 8) {
          float a[8], c[8];
          load_bf16x8(o + d, a);
          load_bf16x8(g + d, c);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc += a[q] * c[q];
        }
      }
      sm.dpart[part][h] = acc;
      softmax_sync();
      if (row < kHeadsCta) {
        const float dlt = sm.dpart[0][row] + sm.dpart[1][row];
        sm.delta[row] = dlt;
        if (row < heads_here) {
          const int64_t hi = tok * p.H + hg * kHeadsCta + row;
          const float l = p.lse[hi];
          sm.lse2[row] = l * kLog2e;
          sp.dsink_part[hi] = -__expf(p.sinks[hg * kHeadsCta + row] - l) * dlt;
        } else {
          sm.lse2[row] = 0.f;
        }
      }
      softmax_sync();
    }
    bool failed = false;
    if (!warp_wait(&sm.table_full, 0, p.status, kSbWaitQ)) sm.fail = 1;
    softmax_sync();
    failed = sm.fail != 0;
    int g = 0;
    for (int it = 0; it < tiles && !failed; ++it) {
      if (!warp_wait(&sm.s_full, it & 1, p.status, kSbWaitS)) sm.fail = 1;
      softmax_sync();
      if (sm.fail) break;
      tc_fence_after();
      float sv[64], dp[64];
      {
        uint32_t r[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          tmem_ld_32x32b_x32(lane_base + Cfg::kColS + hh * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[hh * 32 + j] = __uint_as_float(r[j]);
          tmem_ld_32x32b_x32(lane_base + Cfg::kColDp + hh * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) dp[hh * 32 + j] = __uint_as_float(r[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.s_free);
      const int32_t e_row = entry_at(p, ent, it * kKeys + row);
      const bool valid = e_row >= 0;
      const __nv_bfloat16* src = entry_src<D>(p, b, it * kKeys + row, e_row);
      // P and scale * dS
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        float p0 = valid && j < heads_here ? ex2_approx(sv[j] * p.scale_log2 - sm.lse2[j]) : 0.f;
        float p1 = valid && j + 1 < heads_here ? ex2_approx(sv[j + 1] * p.scale_log2 - sm.lse2[j + 1]) : 0.f;
        __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        pk[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
        dp[j] = p0 * (dp[j] - sm.delta[j]) * sp.scale;
        dp[j + 1] = p1 * (dp[j + 1] - sm.delta[j + 1]) * sp.scale;
      }
      if (it > 0 && !warp_wait(&sm.ds_free, (it - 1) & 1, p.status, kSbWaitDsFree)) sm.fail = 1;
      softmax_sync();
      if (sm.fail) break;
      tc_fence_after();
      tmem_st_32x32b_x32(lane_base + Cfg::kColP, pk);
      {
        uint8_t* drow = sm.ds + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(dp[8 * c + 2 * q], dp[8 * c + 2 * q + 1]);
            wp[q] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(drow + ((c ^ (row & 7)) << 4)) = w;
        }
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.ds_full);
      // drain the dKV chunks into the fp32 gradient of this key's row
      const int j = it * kKeys + row;
      float* dst = nullptr;
      const bool ordered = sp.edges != nullptr;
      if (valid) {
        if (ordered) {  // this (token, entry, head group)'s own edge row: plain stores
          dst = sp.edges + (((static_cast<int64_t>(b) * sp.chunk + (t - sp.t0)) * (p.W + p.K) + j) * gridDim.z + hg) * D;
        } else if (j < p.W) {
          dst = sp.dkv + (src - p.kv);
        } else {
          dst = sp.dcomp + (src - p.comp);
        }
      }
      for (int c = 0; c < Cfg::kChunks; ++c, ++g) {
        if (!warp_wait(&sm.dkv_full, g & 1, p.status, kSbWaitDkv)) sm.fail = 1;
        softmax_sync();
        if (sm.fail) {
          failed = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_base + Cfg::kColDkv + hh * 32, r);
          tmem_ld_wait();
          if (dst != nullptr && ordered) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              *reinterpret_cast<float4*>(dst + c * 64 + hh * 32 + q) =
                  make_float4(__uint_as_float(r[q]), __uint_as_float(r[q + 1]), __uint_as_float(r[q + 2]),
                              __uint_as_float(r[q + 3]));
            }
          } else if (dst != nullptr) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              red_add_v4(dst + c * 64 + hh * 32 + q, __uint_as_float(r[q]), __uint_as_float(r[q + 1]),
                         __uint_as_float(r[q + 2]), __uint_as_float(r[q + 3]));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&sm.dkv_free);
      }
    }
    if (!failed && !sm.fail && !warp_wait(&sm.dq_full, 0, p.status, kSbWaitDq)) sm.fail = 1;
    softmax_sync();
    if (!sm.fail) {
      tc_fence_after();
      // dQ staged as bf16 [64 heads x D] over the idle key buffer(s), then one contiguous store
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(sm.k[0]);
#pragma unroll 1
      for (int m = 0; m < Cfg::kOTiles; ++m) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(lane_base + Cfg::kColDq + m * 64 + hh * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 32; ++q) stage[(hh * 32 + q) * D + m * 128 + row] = __float2bfloat16_rn(__uint_as_float(r[q]));
        }
      }
      softmax_sync();
      const uint4* from = reinterpret_cast<const uint4*>(stage);
      uint4* to = reinterpret_cast<uint4*>(sp.dq + (tok * p.H + hg * kHeadsCta) * D);
      for (int i = row; i < heads_here * D / 8; i += 128) to[i] = from[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
void launch_bwd(const SbParams& prm, int tokens, int B, int groups) {
  const size_t smem = sizeof(SbSmem<D>) + 1024 + static_cast<size_t>(prm.f.W + prm.f.K) * sizeof(int32_t);
  static const int limit = [] {  // configured once at the device's opt-in maximum
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncSetAttribute(sparse_attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
    return v;
  }();
  TDSV_CHECK(smem <= static_cast<size_t>(limit), "sparse attention: too many keys per token for shared memory (",
             smem, " > ", limit, " bytes)");
  sparse_attn_bwd_kernel<D><<<dim3(tokens, B, groups), kSaThreads, smem, stream()>>>(prm);
}

// Deterministic sum of per-edge dKV rows: one CTA per destination row r (window rows first, then
// compressed rows), its edges in `order[offsets[r] .. offsets[r + 1])` (ascending edge id, the
// stable sort of the chunk's destinations) and, within an edge, the head groups in order. The sum
// is added to the row's fp32 gradient by its only writer.
__global__ void ordered_edge_reduce_kernel(const float* __restrict__ edges, const int64_t* __restrict__ order,
                                           const int64_t* __restrict__ offsets, float* __restrict__ dkv,
                                           float* __restrict__ dcomp, int64_t kv_rows, int groups, int D) {
  const int64_t r = blockIdx.x;
  const int64_t lo = offsets[r], hi = offsets[r + 1];
  if (lo == hi) return;
  float* out = r < kv_rows ? dkv + r * D : dcomp + (r - kv_rows) * D;
  for (int d = threadIdx.x * 4; d < D; d += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t e = lo; e < hi; ++e) {
      const float* row = edges + order[e] * groups * D + d;
      for (int g = 0; g < groups; ++g) {
        const float4 v = *reinterpret_cast<const float4*>(row + g * D);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    float4 cur = *reinterpret_cast<float4*>(out + d);
    cur.x += acc.x;
    cur.y += acc.y;
    cur.z += acc.z;
    cur.w += acc.w;
    *reinterpret_cast<float4*>(out + d) = cur;
  }
}

template <int D>
void launch_fwd(const SaParams& prm, int L, int B, int groups) {
  const size_t smem = sizeof(SaSmem<D>) + 1024 + static_cast<size_t>(prm.W + prm.K) * sizeof(int32_t);
  static const int limit = [] {  // configured once at the device's opt-in maximum
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncSetAttribute(sparse_attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
    return v;
  }();
  TDSV_CHECK(smem <= static_cast<size_t>(limit), "sparse attention: too many keys per token for shared memory (",
             smem, " > ", limit, " bytes)");
  sparse_attn_fwd_kernel<D><<<dim3(L, B, groups), kSaThreads, smem, stream()>>>(prm);
}

}  // namespace

namespace {

// Shared argument checks of the forward and backward entry points.
SaParams make_params(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx, const at::Tensor& win_mask,
                     const c10::optional<at::Tensor>& comp, const c10::optional<at::Tensor>& comp_idx,
                     const at::Tensor& sinks) {
  check_cuda_tensor(q, "q");
  check_cuda_tensor(kv, "kv");
  check_cuda_tensor(win_idx, "window_indices");
  check_cuda_tensor(win_mask, "window_mask");
  check_cuda_tensor(sinks, "sinks");
  TDSV_CHECK(q.dim() == 4 && kv.dim() == 3, "sparse_attention: q [B, L, H, D], kv [B, S, D]");
  const int B = static_cast<int>(q.size(0)), L = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2));
  const int D = static_cast<int>(q.size(3));
  TDSV_CHECK(q.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16, "sparse_attention: bf16");
  TDSV_CHECK(D == 128 || D == 256 || D == 512, "sparse_attention: head dim 128, 256 or 512");
  TDSV_CHECK(kv.size(0) == B && kv.size(2) == D, "sparse_attention: kv shape");
  TDSV_CHECK(win_idx.scalar_type() == at::kLong && win_idx.dim() == 3 && win_idx.size(0) == B && win_idx.size(1) == L,
             "sparse_attention: window_indices int64 [B, L, W]");
  TDSV_CHECK(win_mask.scalar_type() == at::kBool && win_mask.sizes() == win_idx.sizes(),
             "sparse_attention: window_mask bool [B, L, W]");
  TDSV_CHECK(sinks.scalar_type() == at::kFloat && sinks.numel() == H, "sparse_attention: sinks fp32 [H]");
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
  if (comp.has_value() && comp->defined() && comp_idx.has_value() && comp_idx->defined()) {
    check_cuda_tensor(*comp, "compressed_kv");
    check_cuda_tensor(*comp_idx, "compressed_indices");
    TDSV_CHECK(comp->scalar_type() == at::kBFloat16 && comp->dim() == 3 && comp->size(0) == B && comp->size(2) == D,
               "sparse_attention: compressed_kv bf16 [B, C, D]");
    TDSV_CHECK(comp_idx->scalar_type() == at::kLong && comp_idx->dim() == 3 && comp_idx->size(0) == B &&
                   comp_idx->size(1) == L,
               "sparse_attention: compressed_indices int64 [B, L, K]");
    prm.comp = reinterpret_cast<const __nv_bfloat16*>(comp->data_ptr());
    prm.comp_idx = comp_idx->data_ptr<int64_t>();
    prm.C = static_cast<int>(comp->size(1));
    prm.K = static_cast<int>(comp_idx->size(2));
  }
  TDSV_CHECK(prm.W + prm.K > 0, "sparse_attention: no keys");
  prm.scale_log2 = static_cast<float>(std::pow(static_cast<double>(D), -0.5)) * kLog2e;
  prm.status = status_word_ptr();
  return prm;
}

}  // namespace

// out [B, L, H, D] bf16, lse [B, L, H] fp32 (natural log, sink included).
std::vector<at::Tensor> sparse_attention_fwd(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx,
                                             const at::Tensor& win_mask, const c10::optional<at::Tensor>& comp,
                                             const c10::optional<at::Tensor>& comp_idx, const at::Tensor& sinks) {
  SaParams prm = make_params(q, kv, win_idx, win_mask, comp, comp_idx, sinks);
  const int B = static_cast<int>(q.size(0)), L = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2));
  const int D = static_cast<int>(q.size(3));
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

// dq [B, L, H, D] bf16, dkv [B, S, D] fp32, dcompressed [B, C, D] fp32 (empty without compressed
// keys), dsink partials [B, L, H] fp32 (sum over B and L for the sink gradient).
std::vector<at::Tensor> sparse_attention_bwd(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx,
                                             const at::Tensor& win_mask, const c10::optional<at::Tensor>& comp,
                                             const c10::optional<at::Tensor>& comp_idx, const at::Tensor& sinks,
                                             const at::Tensor& out, const at::Tensor& lse, const at::Tensor& dout,
                                             c10::optional<int64_t> ordered_chunk) {
  SbParams sp{};
  sp.f = make_params(q, kv, win_idx, win_mask, comp, comp_idx, sinks);
  check_cuda_tensor(out, "out");
  check_cuda_tensor(lse, "lse");
  check_cuda_tensor(dout, "dout");
  TDSV_CHECK(out.sizes() == q.sizes() && dout.sizes() == q.sizes() && dout.scalar_type() == at::kBFloat16 &&
                 out.scalar_type() == at::kBFloat16,
             "sparse_attention_bwd: out / dout bf16 like q");
  const int B = static_cast<int>(q.size(0)), L = static_cast<int>(q.size(1)), H = static_cast<int>(q.size(2));
  const int D = static_cast<int>(q.size(3));
  TDSV_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == static_cast<int64_t>(B) * L * H,
             "sparse_attention_bwd: lse fp32 [B, L, H]");
  sp.f.out = const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()));
  sp.f.lse = const_cast<float*>(lse.data_ptr<float>());
  sp.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  auto dq = at::empty_like(q);
  auto dkv = at::zeros(kv.sizes(), kv.options().dtype(at::kFloat));
  at::Tensor dcomp;
  if (sp.f.comp != nullptr) {
    dcomp = at::zeros(comp->sizes(), comp->options().dtype(at::kFloat));
    sp.dcomp = dcomp.data_ptr<float>();
  }
  auto dsink = at::empty({B, L, H}, q.options().dtype(at::kFloat));
  sp.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  sp.dkv = dkv.data_ptr<float>();
  sp.dsink_part = dsink.data_ptr<float>();
  sp.scale = static_cast<float>(std::pow(static_cast<double>(D), -0.5));
  sp.chunk = L;
  if (B * L == 0) return {dq, dkv, dcomp, dsink};
  c10::cuda::CUDAGuard guard(q.device());
  const int groups = (H + kHeadsCta - 1) / kHeadsCta;
  if (!ordered_chunk.has_value()) {
    if (D == 128) launch_bwd<128>(sp, L, B, groups);
    else if (D == 256) launch_bwd<256>(sp, L, B, groups);
    else launch_bwd<512>(sp, L, B, groups);
    TDSV_LAUNCH_CHECK();
    return {dq, dkv, dcomp, dsink};
  }
  // Deterministic KV gradients: token chunks in order; per chunk, every (token, entry, head group)
  // stores its own dKV row, then each destination row sums its edges in ascending edge order.
  const int chunk = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(*ordered_chunk, L)));
  const int slots = sp.f.W + sp.f.K;
  const int64_t kv_rows = static_cast<int64_t>(B) * sp.f.S;
  const int64_t rows = kv_rows + static_cast<int64_t>(B) * sp.f.C;
  auto edges = at::empty({B, chunk, slots, groups, D}, q.options().dtype(at::kFloat));
  sp.edges = edges.data_ptr<float>();
  sp.chunk = chunk;
  // destination row of every edge of the whole sequence (rows = invalid)
  auto opts = win_idx.options();
  auto wvalid = win_mask & (win_idx >= 0) & (win_idx < sp.f.S);
  auto batch_kv = at::arange(B, opts).view({B, 1, 1}) * sp.f.S;
  auto wdest = at::where(wvalid, win_idx + batch_kv, at::full({}, rows, opts));
  at::Tensor dest = wdest;
  if (sp.f.K > 0) {
    auto cvalid = (*comp_idx >= 0) & (*comp_idx < sp.f.C);
    auto batch_c = at::arange(B, opts).view({B, 1, 1}) * sp.f.C + kv_rows;
    dest = at::cat({wdest, at::where(cvalid, *comp_idx + batch_c, at::full({}, rows, opts))}, 2);
  }
  for (int t0 = 0; t0 < L; t0 += chunk) {
    const int n = std::min(chunk, L - t0);
    sp.t0 = t0;
    if (D == 128) launch_bwd<128>(sp, n, B, groups);
    else if (D == 256) launch_bwd<256>(sp, n, B, groups);
    else launch_bwd<512>(sp, n, B, groups);
    TDSV_LAUNCH_CHECK();
    // edge ids local to the chunk buffer: (b * chunk + (t - t0)) * slots + j
    auto d = dest.narrow(1, t0, n);                                       // [B, n, slots]
    if (n < chunk) d = at::cat({d, at::full({B, chunk - n, slots}, rows, opts)}, 1);
    auto flat = d.reshape({-1});
    auto order = std::get<1>(at::sort(flat, /*stable=*/true, /*dim=*/0, /*descending=*/false));
    auto counts = at::bincount(flat, /*weights=*/{}, rows + 1).narrow(0, 0, rows);
    auto offsets = at::cat({at::zeros({1}, counts.options()), counts.cumsum(0)});
    ordered_edge_reduce_kernel<<<static_cast<unsigned>(rows), 128, 0, stream()>>>(
        edges.data_ptr<float>(), order.data_ptr<int64_t>(), offsets.data_ptr<int64_t>(), dkv.data_ptr<float>(),
        sp.f.C > 0 ? dcomp.data_ptr<float>() : nullptr, kv_rows, groups, D);
    TDSV_LAUNCH_CHECK();
  }
  return {dq, dkv, dcomp, dsink};
}

}  // namespace tdsv
