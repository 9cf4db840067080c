// Causal GQA flash attention on the 5th-generation tensor cores (sm_100a), forward and backward.
//
// Layout: q / out / dout [B, L, H, 128], k / v [B, L, Hkv, 128] bf16, token-major (the layout the
// QKV projection writes, so no transposed copies); lse [B, H, L] fp32 (natural log). Every tile
// moves by TMA through 3-D tensor maps {128 dims, heads, tokens} with 128-byte swizzle, every
// contraction is a tcgen05.mma with its fp32 accumulator in tensor memory, and every mbarrier wait
// is bounded (a timeout records a status code and the CTA drains instead of spinning forever).
//
// Forward: one CTA per (128-query tile, head, batch), 192 threads.
//   warp 0     TMA producer: Q once, then K_j / V_j tiles through a two-stage ring
//   warp 1     MMA issuer: S_{j+1} = Q K_{j+1}^T is issued before P_j is ready, so the next score
//              tile overlaps the softmax of this one (S is double-buffered in tensor memory)
//   warps 2-5  softmax, one thread per query row: online softmax in the exp2 domain; the running
//              maximum is raised only when it grows by more than 2^8, so O (in tensor memory) is
//              rescaled rarely; P goes to shared memory in the swizzled K-major layout the PV MMA
//              reads; at the end O / l is stored as bf16 and the row's log-sum-exp as fp32.
//   TMEM: S0 [0, 128), S1 [128, 256), O [256, 384).
//
// Backward: one CTA per (128-key tile, query head, batch), looping over 64-query blocks, 192 threads.
//   S^T = K Q^T and dP^T = V dO^T put one key per TMEM lane, so the thread that owns key row r
//   computes P^T = exp2(S^T c - lse2) and dS^T = P^T (dP^T - D) for its row and writes both to
//   shared memory (K-major); then dV += P^T dO, dK += dS^T Q (both accumulated in TMEM over the
//   whole loop) and dQ^T = K^T dS^T (fresh per block, reduced into an fp32 [B, H, 128, L] buffer by
//   TMA reduce-add). D = rowsum(dO * O) and lse2 = lse log2(e) come from a small prep kernel;
//   dK / dV of the query heads of one GQA group meet in fp32 buffers (TMA reduce-add) and a
//   finalize kernel scales and converts dQ / dK / dV to bf16.
//   Issue order per block i: dP_i, S_{i+1}, [P_i, dS_i ready] dV, dK, dQ_i; the softmax of block
//   i+1 overlaps the dV / dK / dQ MMAs of block i.
//   TMEM: S0 [0, 64), S1 [64, 128), dP [128, 192), dQ^T [192, 256), dV [256, 384), dK [384, 512).
//
// No reference counterpart: the reference runs torch's scaled_dot_product_attention
// (dsv41_train/models/qwen/model.py:162) and an eager sparse-attention path for DeepSeek-V4.
#include "common.cuh"

#include <mutex>

namespace tdsv {

namespace {

constexpr int kDim = 128;           // head dim
constexpr int kTile = 128;          // forward query tile / key tile; backward key tile
constexpr int kQBlk = 64;           // backward query block
constexpr int kAtom = 128 * 128;    // [128 rows x 64 bf16] swizzled atom, bytes
constexpr int kHalfAtom = 64 * 128; // [64 rows x 64 bf16]
constexpr float kLog2e = 1.4426950408889634f;

// ---- wait-site codes (reported through the status word) -----------------------------------
enum : int {
  kFwdWaitKvEmpty = 301, kFwdWaitQ, kFwdWaitKv0, kFwdWaitKv, kFwdWaitSFree, kFwdWaitP, kFwdWaitS, kFwdWaitPV,
  kFwdWaitLast,
  kBwdWaitQEmpty = 321, kBwdWaitKv, kBwdWaitQ, kBwdWaitDpFree, kBwdWaitSFree, kBwdWaitPds, kBwdWaitDqFree,
  kBwdWaitS, kBwdWaitDp, kBwdWaitPdsFree, kBwdWaitDq, kBwdWaitQc,
};

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Plain bulk copy global -> shared (no multicast), completion on an mbarrier. 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// K-major operand of `rows` x 128 columns stored as two 64-column atoms of `atom_bytes`:
// descriptor of MMA k-step kk (16 columns).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk, uint32_t atom_bytes) {
  return make_smem_desc_sw128(base + (kk >> 2) * atom_bytes + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (K rows x MN columns, MN split into 64-column atoms `atom_bytes` apart):
// k-step kk covers rows 16kk .. 16kk+15.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk, uint32_t atom_bytes) {
  return make_smem_desc_sw128(base + kk * 2048, atom_bytes, 1024);
}

// Bounded wait taken by a whole warp: every lane reaches the vote, so the warp leaves converged
// (tcgen05.ld / st are warp-collective) and takes a timeout branch together.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status, code));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled atom.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// =============================================================================================
// Forward
// =============================================================================================
struct FwdSmem {
  alignas(1024) uint8_t q[2 * kAtom];
  alignas(1024) uint8_t k[2][2 * kAtom];
  alignas(1024) uint8_t v[2][2 * kAtom];
  alignas(1024) uint8_t p[2 * kAtom];
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(192, 1) attn_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                          const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv,
                                                          __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                                                          int seq, int heads, int kv_heads, float scale_log2,
                                                          int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_q = seq / kTile;
  const int h = blockIdx.x;
  const int qi = n_q - 1 - static_cast<int>(blockIdx.y);  // longest causal rows in the first wave
  const int b = blockIdx.z;
  const int hk = h / (heads / kv_heads);
  const int n_kv = qi + 1;
  const int row0 = b * seq + qi * kTile;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
    }
    mbar_init(&sm.p_full, 128);
    mbar_init(&sm.pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(&sm.q_full, 2 * kAtom);
      tma_load_3d(sm.q, &tq, &sm.q_full, 0, h, row0);
      tma_load_3d(sm.q + kAtom, &tq, &sm.q_full, 64, h, row0);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&sm.kv_empty[s], ((j >> 1) - 1) & 1, status, kFwdWaitKvEmpty)) break;
        mbar_arrive_expect_tx(&sm.kv_full[s], 4 * kAtom);
        const int key0 = b * seq + j * kTile;
        tma_load_3d(sm.k[s], &tk, &sm.kv_full[s], 0, hk, key0);
        tma_load_3d(sm.k[s] + kAtom, &tk, &sm.kv_full[s], 64, hk, key0);
        tma_load_3d(sm.v[s], &tv, &sm.kv_full[s], 0, hk, key0);
        tma_load_3d(sm.v[s] + kAtom, &tv, &sm.kv_full[s], 64, hk, key0);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc_s = make_idesc_bf16(kTile, kTile, false, false);
      const uint32_t idesc_pv = make_idesc_bf16(kTile, kDim, false, true);
      const uint32_t qa = smem_u32(sm.q), pa = smem_u32(sm.p);
      bool ok = mbar_wait(&sm.q_full, 0, status, kFwdWaitQ) && mbar_wait(&sm.kv_full[0], 0, status, kFwdWaitKv0);
      if (ok) {
        tc_fence_after();
        const uint32_t ka = smem_u32(sm.k[0]);
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk)
          umma_f16(tmem, kmajor_desc(qa, kk, kAtom), kmajor_desc(ka, kk, kAtom), idesc_s, kk > 0);
        umma_commit(&sm.s_full[0]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv) {
          const int sn = (j + 1) & 1;
          ok = mbar_wait(&sm.kv_full[sn], ((j + 1) >> 1) & 1, status, kFwdWaitKv);
          if (ok && j + 1 >= 2) ok = mbar_wait(&sm.s_free[sn], (((j + 1) >> 1) - 1) & 1, status, kFwdWaitSFree);
          if (!ok) break;
          tc_fence_after();
          const uint32_t ka = smem_u32(sm.k[sn]);
#pragma unroll
          for (int kk = 0; kk < kDim / 16; ++kk)
            umma_f16(tmem + sn * kTile, kmajor_desc(qa, kk, kAtom), kmajor_desc(ka, kk, kAtom), idesc_s, kk > 0);
          umma_commit(&sm.s_full[sn]);
        }
        if (!(ok = mbar_wait(&sm.p_full, j & 1, status, kFwdWaitP))) break;
        tc_fence_after();
        const uint32_t va = smem_u32(sm.v[j & 1]);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_f16(tmem + 2 * kTile, kmajor_desc(pa, kk, kAtom), mnmajor_desc(va, kk, kAtom), idesc_pv,
                   (j > 0 || kk > 0));
        umma_commit(&sm.pv_done);
        umma_commit(&sm.kv_empty[j & 1]);
      }
    }
  } else {
    // softmax: thread <-> query row (TMEM lane)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int q_pos = qi * kTile + r;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int buf = j & 1;
      if (!(ok = warp_wait(&sm.s_full[buf], (j >> 1) & 1, status, kFwdWaitS))) break;
      tc_fence_after();
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the per-thread wait loop
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(lane_addr + buf * kTile + c * 32, sv[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free[buf]);
      // scores in the log2 domain, causal mask on the diagonal tile
      float mx = -INFINITY;
      const bool diag = j == qi;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = __uint_as_float(sv[c][i]) * scale_log2;
          if (diag && j * kTile + c * 32 + i > q_pos) x = -INFINITY;
          sv[c][i] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      float alpha = 1.f;
      if (mx > m_used + 8.f) {  // raise the reference maximum only when it grows by more than 2^8
        alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - mx);
        m_used = mx;
      }
      float rowsum = 0.f;
      uint32_t packed[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = exp2f(__uint_as_float(sv[c][i]) - m_used);
          const float p1 = exp2f(__uint_as_float(sv[c][i + 1]) - m_used);
          const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
          rowsum += __low2float(pb) + __high2float(pb);  // the sum of exactly what the PV MMA multiplies
          packed[c][i / 2] = *reinterpret_cast<const uint32_t*>(&pb);
        }
      l = l * alpha + rowsum;
      if (j > 0) {
        // PV_{j-1} complete: O may be rescaled and P overwritten
        if (!(ok = warp_wait(&sm.pv_done, (j - 1) & 1, status, kFwdWaitPV))) break;
        tc_fence_after();
        __syncwarp();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(lane_addr + 2 * kTile + c * 32, ov);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st_32x32b_x32(lane_addr + 2 * kTile + c * 32, ov);
          }
          tmem_st_wait();
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int col = c * 32 + g * 8;  // first key of this 16-byte chunk
          const uint4 val = make_uint4(packed[c][g * 4], packed[c][g * 4 + 1], packed[c][g * 4 + 2],
                                       packed[c][g * 4 + 3]);
          *reinterpret_cast<uint4*>(sm.p + (col >> 6) * kAtom + swz(r, (col & 63) >> 3)) = val;
        }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full);
    }
    if (ok && warp_wait(&sm.pv_done, (n_kv - 1) & 1, status, kFwdWaitLast)) {
      tc_fence_after();
      __syncwarp();
      const float inv = 1.f / l;
      __nv_bfloat16* dst = out + (static_cast<int64_t>(row0 + r) * heads + h) * kDim;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(lane_addr + 2 * kTile + c * 32, ov);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(ov[g * 8 + i]) * inv;
          store_bf16x8(dst + c * 32 + g * 8, o);
        }
      }
      lse[(static_cast<int64_t>(b) * heads + h) * seq + q_pos] = (m_used + log2f(l)) * 0.69314718055994531f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

// =============================================================================================
// Backward
// =============================================================================================
struct BwdSmem {
  alignas(1024) uint8_t k[2 * kAtom];           // [128 keys x 128 dims]
  alignas(1024) uint8_t v[2 * kAtom];
  alignas(1024) uint8_t q[2][2 * kHalfAtom];    // per stage [64 queries x 128 dims]
  alignas(1024) uint8_t dout[2][2 * kHalfAtom];
  alignas(1024) uint8_t pt[kAtom];              // P^T  [128 keys x 64 queries]
  alignas(1024) uint8_t dst[kAtom];             // dS^T [128 keys x 64 queries]
  alignas(1024) uint8_t stage[4][2][32 * 128];  // per epilogue warp: two [32 x 32 fp32] reduce boxes
  alignas(16) float lse2[2][kQBlk];
  alignas(16) float dvec[2][kQBlk];
  uint64_t kv_full;
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t dp_full;
  uint64_t dp_free;
  uint64_t pds_ready;
  uint64_t pds_free;
  uint64_t dq_full;
  uint64_t dq_free;
  uint32_t tmem_base;
};

constexpr uint32_t kColS = 0, kColDp = 128, kColDq = 192, kColDv = 256, kColDk = 384;

// One warp drains `chunks` x 32 fp32 columns of its 32 TMEM lanes and reduce-adds them into global
// memory through two 4 KB staging boxes (lane 0 issues every bulk group, so it alone waits on them).
template <typename IssueFn>
__device__ __forceinline__ void drain_reduce(uint32_t taddr, int chunks, uint8_t (*stage)[32 * 128], int lane,
                                             int& slot, IssueFn issue) {
  for (int c = 0; c < chunks; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c * 32, v);
    tmem_ld_wait();
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
    uint8_t* box = stage[slot];
#pragma unroll
    for (int g = 0; g < 8; ++g)
      *reinterpret_cast<uint4*>(box + swz(lane, g)) = make_uint4(v[g * 4], v[g * 4 + 1], v[g * 4 + 2], v[g * 4 + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      issue(smem_u32(box), c);
      bulk_commit_group();
    }
    __syncwarp();
    slot ^= 1;
  }
}

__global__ void __launch_bounds__(192, 1) attn_bwd_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
    const __grid_constant__ CUtensorMap tdq_acc, const __grid_constant__ CUtensorMap tdk_acc,
    const __grid_constant__ CUtensorMap tdv_acc, const float* __restrict__ lse2, const float* __restrict__ dvec,
    int seq, int heads, int kv_heads, float scale_log2, int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int j = blockIdx.y;  // key tile; j = 0 sees every query block, so it is scheduled first
  const int b = blockIdx.z;
  const int hk = h / (heads / kv_heads);
  const int i0 = j * (kTile / kQBlk);
  const int n_it = seq / kQBlk - i0;
  const int key0 = b * seq + j * kTile;
  const int64_t stat_row = (static_cast<int64_t>(b) * heads + h) * seq;

  if (threadIdx.x == 0) {
    mbar_init(&sm.kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
    }
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.dp_free, 128);
    mbar_init(&sm.pds_ready, 128);
    mbar_init(&sm.pds_free, 1);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_free, 128);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      tma_prefetch_desc(&tdo);
      mbar_arrive_expect_tx(&sm.kv_full, 4 * kAtom);
      tma_load_3d(sm.k, &tk, &sm.kv_full, 0, hk, key0);
      tma_load_3d(sm.k + kAtom, &tk, &sm.kv_full, 64, hk, key0);
      tma_load_3d(sm.v, &tv, &sm.kv_full, 0, hk, key0);
      tma_load_3d(sm.v + kAtom, &tv, &sm.kv_full, 64, hk, key0);
      for (int it = 0; it < n_it; ++it) {
        const int s = it & 1;
        if (it >= 2 && !mbar_wait(&sm.q_empty[s], ((it >> 1) - 1) & 1, status, kBwdWaitQEmpty)) break;
        const int qrow = b * seq + (i0 + it) * kQBlk;
        mbar_arrive_expect_tx(&sm.q_full[s], 4 * kHalfAtom + 2 * kQBlk * 4);
        tma_load_3d(sm.q[s], &tq, &sm.q_full[s], 0, h, qrow);
        tma_load_3d(sm.q[s] + kHalfAtom, &tq, &sm.q_full[s], 64, h, qrow);
        tma_load_3d(sm.dout[s], &tdo, &sm.q_full[s], 0, h, qrow);
        tma_load_3d(sm.dout[s] + kHalfAtom, &tdo, &sm.q_full[s], 64, h, qrow);
        const int64_t off = stat_row + (i0 + it) * kQBlk;
        bulk_load_1d(sm.lse2[s], lse2 + off, kQBlk * 4, &sm.q_full[s]);
        bulk_load_1d(sm.dvec[s], dvec + off, kQBlk * 4, &sm.q_full[s]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc_sp = make_idesc_bf16(kTile, kQBlk, false, false);  // S^T, dP^T: M keys, N queries
      const uint32_t idesc_kv = make_idesc_bf16(kTile, kDim, false, true);    // dV, dK: M keys, N dims
      const uint32_t idesc_q = make_idesc_bf16(kDim, kQBlk, true, true);      // dQ^T: M dims, N queries
      const uint32_t ka = smem_u32(sm.k), va = smem_u32(sm.v), pta = smem_u32(sm.pt), dsa = smem_u32(sm.dst);
      bool ok = mbar_wait(&sm.kv_full, 0, status, kBwdWaitKv) && mbar_wait(&sm.q_full[0], 0, status, kBwdWaitQ);
      if (ok) {
        tc_fence_after();
        const uint32_t qa = smem_u32(sm.q[0]);
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk)
          umma_f16(tmem + kColS, kmajor_desc(ka, kk, kAtom), kmajor_desc(qa, kk, kHalfAtom), idesc_sp, kk > 0);
        umma_commit(&sm.s_full[0]);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const int s = it & 1;
        // dP^T_it = V dO_it^T
        if (it >= 1 && !(ok = mbar_wait(&sm.dp_free, (it - 1) & 1, status, kBwdWaitDpFree))) break;
        tc_fence_after();
        const uint32_t doa = smem_u32(sm.dout[s]), qa = smem_u32(sm.q[s]);
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk)
          umma_f16(tmem + kColDp, kmajor_desc(va, kk, kAtom), kmajor_desc(doa, kk, kHalfAtom), idesc_sp, kk > 0);
        umma_commit(&sm.dp_full);
        // S^T_{it+1} = K Q_{it+1}^T into the other S buffer
        if (it + 1 < n_it) {
          const int sn = (it + 1) & 1;
          ok = mbar_wait(&sm.q_full[sn], ((it + 1) >> 1) & 1, status, kBwdWaitQ);
          if (ok && it + 1 >= 2) ok = mbar_wait(&sm.s_free[sn], (((it + 1) >> 1) - 1) & 1, status, kBwdWaitSFree);
          if (!ok) break;
          tc_fence_after();
          const uint32_t qn = smem_u32(sm.q[sn]);
#pragma unroll
          for (int kk = 0; kk < kDim / 16; ++kk)
            umma_f16(tmem + kColS + sn * kQBlk, kmajor_desc(ka, kk, kAtom), kmajor_desc(qn, kk, kHalfAtom), idesc_sp,
                     kk > 0);
          umma_commit(&sm.s_full[sn]);
        }
        // P^T_it, dS^T_it in shared memory
        if (!(ok = mbar_wait(&sm.pds_ready, it & 1, status, kBwdWaitPds))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kQBlk / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          umma_f16(tmem + kColDv, make_smem_desc_sw128(pta + kk * 32, 16, 1024), mnmajor_desc(doa, kk, kHalfAtom),
                   idesc_kv, acc);
          umma_f16(tmem + kColDk, make_smem_desc_sw128(dsa + kk * 32, 16, 1024), mnmajor_desc(qa, kk, kHalfAtom),
                   idesc_kv, acc);
        }
        umma_commit(&sm.q_empty[s]);
        // dQ^T_it = K^T dS^T_it (the previous block's dQ^T must have been drained)
        if (it >= 1 && !(ok = mbar_wait(&sm.dq_free, (it - 1) & 1, status, kBwdWaitDqFree))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_f16(tmem + kColDq, mnmajor_desc(ka, kk, kAtom), mnmajor_desc(dsa, kk, kAtom), idesc_q, kk > 0);
        umma_commit(&sm.dq_full);
        umma_commit(&sm.pds_free);
      }
    }
  } else {
    // thread <-> key row r of this tile (TMEM lane r); for dQ^T, TMEM lane r is head dim r
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int key_pos = j * kTile + r;
    uint8_t (*stage)[32 * 128] = sm.stage[quarter];
    int slot = 0;
    const int dq_row = (b * heads + h) * kDim + quarter * 32;
    auto drain_dq = [&](int it) {
      const int q0 = (i0 + it) * kQBlk;
      drain_reduce(lane_addr + kColDq, kQBlk / 32, stage, lane, slot, [&](uint32_t src, int c) {
        tma_reduce_add_2d(&tdq_acc, src, q0 + c * 32, dq_row);
      });
    };
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int s = it & 1;
      const int q0 = (i0 + it) * kQBlk;
      if (!(ok = warp_wait(&sm.q_full[s], (it >> 1) & 1, status, kBwdWaitQc))) break;
      if (!(ok = warp_wait(&sm.s_full[s], (it >> 1) & 1, status, kBwdWaitS))) break;
      tc_fence_after();
      __syncwarp();
      uint32_t sv[2][32];
      tmem_ld_32x32b_x32(lane_addr + kColS + s * kQBlk, sv[0]);
      tmem_ld_32x32b_x32(lane_addr + kColS + s * kQBlk + 32, sv[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free[s]);
      const bool diag = q0 < (j + 1) * kTile;
      float p[64];
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int q = c * 32 + i;
          const float x = fmaf(__uint_as_float(sv[c][i]), scale_log2, -sm.lse2[s][q]);
          p[q] = (diag && key_pos > q0 + q) ? 0.f : exp2f(x);
        }
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const __nv_bfloat162 t = __floats2bfloat162_rn(p[2 * i], p[2 * i + 1]);
        pk[i] = *reinterpret_cast<const uint32_t*>(&t);
      }
      if (!(ok = warp_wait(&sm.dp_full, it & 1, status, kBwdWaitDp))) break;
      tc_fence_after();
      __syncwarp();
      tmem_ld_32x32b_x32(lane_addr + kColDp, sv[0]);
      tmem_ld_32x32b_x32(lane_addr + kColDp + 32, sv[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.dp_free);
      uint32_t dk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int q = 2 * i;
        const float d0 = p[q] * (__uint_as_float(sv[q >> 5][q & 31]) - sm.dvec[s][q]);
        const float d1 = p[q + 1] * (__uint_as_float(sv[(q + 1) >> 5][(q + 1) & 31]) - sm.dvec[s][q + 1]);
        const __nv_bfloat162 t = __floats2bfloat162_rn(d0, d1);
        dk[i] = *reinterpret_cast<const uint32_t*>(&t);
      }
      if (it >= 1 && !(ok = warp_wait(&sm.pds_free, (it - 1) & 1, status, kBwdWaitPdsFree))) break;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        *reinterpret_cast<uint4*>(sm.pt + swz(r, g)) = make_uint4(pk[g * 4], pk[g * 4 + 1], pk[g * 4 + 2], pk[g * 4 + 3]);
        *reinterpret_cast<uint4*>(sm.dst + swz(r, g)) = make_uint4(dk[g * 4], dk[g * 4 + 1], dk[g * 4 + 2], dk[g * 4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.pds_ready);
      if (it >= 1) {
        if (!(ok = warp_wait(&sm.dq_full, (it - 1) & 1, status, kBwdWaitDq))) break;
        tc_fence_after();
        __syncwarp();
        drain_dq(it - 1);
        tc_fence_before();
        mbar_arrive(&sm.dq_free);
      }
    }
    if (ok && warp_wait(&sm.dq_full, (n_it - 1) & 1, status, kBwdWaitDq)) {
      // the last dQ^T MMA was the last MMA of the CTA: dV and dK are final too
      tc_fence_after();
      __syncwarp();
      drain_dq(n_it - 1);
      const int row = b * seq + j * kTile + quarter * 32;
      drain_reduce(lane_addr + kColDk, kDim / 32, stage, lane, slot, [&](uint32_t src, int c) {
        tma_reduce_add_3d(&tdk_acc, src, c * 32, hk, row);
      });
      drain_reduce(lane_addr + kColDv, kDim / 32, stage, lane, slot, [&](uint32_t src, int c) {
        tma_reduce_add_3d(&tdv_acc, src, c * 32, hk, row);
      });
    }
    if (lane == 0) bulk_wait_group0();  // reductions complete before the CTA exits
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

// D = rowsum(dO * O) and lse2 = lse * log2(e), both [B, H, L]. One 16-lane group per (token, head).
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout,
                                     const float* __restrict__ lse, float* __restrict__ dvec,
                                     float* __restrict__ lse2, int64_t rows, int seq, int heads) {
  const int64_t groups = (static_cast<int64_t>(gridDim.x) * blockDim.x) / 16;
  const int sub = threadIdx.x & 15;
  for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 16; row < rows; row += groups) {
    float o[8], d[8];
    load_bf16x8(out + row * kDim + sub * 8, o);
    load_bf16x8(dout + row * kDim + sub * 8, d);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(o[i], d[i], acc);
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m, 16);
    if (sub == 0) {
      const int64_t token = row / heads;
      const int h = static_cast<int>(row % heads);
      const int64_t b = token / seq, l = token % seq;
      const int64_t idx = (b * heads + h) * seq + l;
      dvec[idx] = acc;
      lse2[idx] = lse[idx] * kLog2e;
    }
  }
}

// dq [B, L, H, 128] bf16 = scale * transpose(dq_acc [B, H, 128, L]); one block per (32 tokens, head, batch).
__global__ void attn_dq_finalize_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int seq,
                                        int heads, float scale) {
  __shared__ float tile[kDim][33];
  const int l0 = blockIdx.x * 32, h = blockIdx.y, b = blockIdx.z;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 256 threads
  const float* src = acc + ((static_cast<int64_t>(b) * heads + h) * kDim) * seq + l0;
  for (int d = ty; d < kDim; d += 8) tile[d][tx] = src[static_cast<int64_t>(d) * seq + tx];
  __syncthreads();
  // each thread writes 16 consecutive dims of one token: 32 tokens x 8 groups
  const int t = threadIdx.x >> 3, g = threadIdx.x & 7;
  float v[8];
  __nv_bfloat16* dst = dq + ((static_cast<int64_t>(b) * seq + l0 + t) * heads + h) * kDim + g * 16;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = tile[g * 16 + half * 8 + i][t] * scale;
    store_bf16x8(dst + half * 8, v);
  }
}

// dk = scale * dk_acc, dv = dv_acc (fp32 -> bf16), 8 values per thread.
__global__ void attn_dkv_finalize_kernel(const float* __restrict__ dk_acc, const float* __restrict__ dv_acc,
                                         __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                                         int64_t n8, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const float4 a0 = reinterpret_cast<const float4*>(dk_acc)[2 * i];
    const float4 a1 = reinterpret_cast<const float4*>(dk_acc)[2 * i + 1];
    const float4 b0 = reinterpret_cast<const float4*>(dv_acc)[2 * i];
    const float4 b1 = reinterpret_cast<const float4*>(dv_acc)[2 * i + 1];
    const float k8[8] = {a0.x * scale, a0.y * scale, a0.z * scale, a0.w * scale,
                         a1.x * scale, a1.y * scale, a1.z * scale, a1.w * scale};
    const float v8[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    store_bf16x8(dk + i * 8, k8);
    store_bf16x8(dv + i * 8, v8);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
// Token-major [tokens, heads, 128] tensor, box {64 bf16 or 32 fp32 columns, 1 head, box_rows tokens}.
CUtensorMap head_major_map(const at::Tensor& t, int heads, int box_rows) {
  bind_primary_context();
  const bool bf16 = t.scalar_type() == at::kBFloat16;
  const int esize = bf16 ? 2 : 4;
  TDSV_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "attention tensor base must be 16-byte aligned");
  const int64_t tokens = t.numel() / (static_cast<int64_t>(heads) * kDim);
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kDim) * esize, static_cast<cuuint64_t>(heads) * kDim * esize};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / esize), 1, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = encode_fn()(&map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                           t.data_ptr(), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

// fp32 [rows, cols] tensor, box {32 columns, 32 rows}.
CUtensorMap rows_map_f32(const at::Tensor& t, int64_t rows, int64_t cols) {
  bind_primary_context();
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

void check_operands(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  for (const auto* t : {&q, &k, &v}) {
    check_cuda_tensor(*t, "attention operand");
    TDSV_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4 && t->size(3) == kDim,
               "attention: bf16 [B, L, H, 128] operands");
  }
  TDSV_CHECK(k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(1) == q.size(1),
             "attention: k / v shapes must match and share q's batch and length");
  TDSV_CHECK(q.size(2) % k.size(2) == 0, "attention: query heads must be a multiple of key/value heads");
  TDSV_CHECK(q.size(1) % kTile == 0, "attention: sequence length must be a multiple of 128");
  TDSV_CHECK(q.size(1) <= (1 << 30) / q.size(0), "attention: too many tokens");
}

template <typename Kernel>
void set_smem(Kernel kernel, size_t bytes) {
  TDSV_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
}

}  // namespace

// q [B, L, H, 128], k/v [B, L, Hkv, 128] bf16 -> (out [B, L, H, 128] bf16, lse [B, H, L] fp32)
std::vector<at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  check_operands(q, k, v);
  const int64_t batch = q.size(0), seq = q.size(1);
  const int heads = static_cast<int>(q.size(2)), kv_heads = static_cast<int>(k.size(2));
  auto out = at::empty_like(q);
  auto lse = at::empty({batch, heads, seq}, q.options().dtype(at::kFloat));
  if (batch == 0 || seq == 0) return {out, lse};
  c10::cuda::CUDAGuard guard(q.device());
  const CUtensorMap mq = head_major_map(q, heads, kTile), mk = head_major_map(k, kv_heads, kTile),
                    mv = head_major_map(v, kv_heads, kTile);
  const size_t smem = sizeof(FwdSmem) + 1024;
  static std::once_flag once;
  std::call_once(once, [&] { set_smem(attn_fwd_kernel, smem); });
  dim3 grid(static_cast<unsigned>(heads), static_cast<unsigned>(seq / kTile), static_cast<unsigned>(batch));
  attn_fwd_kernel<<<grid, 192, smem, stream()>>>(mq, mk, mv, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                 lse.data_ptr<float>(), static_cast<int>(seq), heads, kv_heads,
                                                 kLog2e / sqrtf(static_cast<float>(kDim)), status_word_ptr());
  TDSV_LAUNCH_CHECK();
  return {out, lse};
}

// Gradients of attn_fwd: (dq, dk, dv) in the layouts of q, k, v.
std::vector<at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                 const at::Tensor& v, const at::Tensor& out, const at::Tensor& lse) {
  check_operands(q, k, v);
  check_cuda_tensor(dout, "attention dout");
  check_cuda_tensor(out, "attention out");
  check_cuda_tensor(lse, "attention lse");
  TDSV_CHECK(dout.sizes() == q.sizes() && out.sizes() == q.sizes() && dout.scalar_type() == at::kBFloat16 &&
                 out.scalar_type() == at::kBFloat16,
             "attention backward: dout / out must be bf16 shaped like q");
  const int64_t batch = q.size(0), seq = q.size(1);
  const int heads = static_cast<int>(q.size(2)), kv_heads = static_cast<int>(k.size(2));
  TDSV_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == batch * heads * seq, "attention backward: lse [B, H, L]");
  auto dq = at::empty_like(q), dk = at::empty_like(k), dv = at::empty_like(v);
  if (batch == 0 || seq == 0) return {dq, dk, dv};
  c10::cuda::CUDAGuard guard(q.device());
  const float scale = 1.f / sqrtf(static_cast<float>(kDim));
  // one fp32 workspace: dq_acc [B, H, 128, L], dk_acc, dv_acc [B, L, Hkv, 128], then D and lse2 [B, H, L]
  const int64_t n_q = batch * heads * seq * kDim, n_kv = k.numel(), n_stat = batch * heads * seq;
  auto ws = at::empty({n_q + 2 * n_kv + 2 * n_stat}, q.options().dtype(at::kFloat));
  TDSV_CUDA_CHECK(cudaMemsetAsync(ws.data_ptr(), 0, (n_q + 2 * n_kv) * sizeof(float), stream()));
  auto dq_acc = ws.narrow(0, 0, n_q);
  auto dk_acc = ws.narrow(0, n_q, n_kv).view(k.sizes());
  auto dv_acc = ws.narrow(0, n_q + n_kv, n_kv).view(k.sizes());
  float* dvec = ws.data_ptr<float>() + n_q + 2 * n_kv;
  float* lse2 = dvec + n_stat;

  const int64_t rows = batch * seq * heads;
  attn_bwd_prep_kernel<<<static_cast<unsigned>(std::min<int64_t>((rows + 15) / 16, 148 * 16)), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      lse.data_ptr<float>(), dvec, lse2, rows, static_cast<int>(seq), heads);
  TDSV_LAUNCH_CHECK();

  const CUtensorMap mq = head_major_map(q, heads, kQBlk), mdo = head_major_map(dout, heads, kQBlk);
  const CUtensorMap mk = head_major_map(k, kv_heads, kTile), mv = head_major_map(v, kv_heads, kTile);
  const CUtensorMap mdq = rows_map_f32(dq_acc, batch * heads * kDim, seq);
  const CUtensorMap mdk = head_major_map(dk_acc, kv_heads, 32), mdv = head_major_map(dv_acc, kv_heads, 32);
  const size_t smem = sizeof(BwdSmem) + 1024;
  static std::once_flag once;
  std::call_once(once, [&] { set_smem(attn_bwd_kernel, smem); });
  dim3 grid(static_cast<unsigned>(heads), static_cast<unsigned>(seq / kTile), static_cast<unsigned>(batch));
  attn_bwd_kernel<<<grid, 192, smem, stream()>>>(mq, mk, mv, mdo, mdq, mdk, mdv, lse2, dvec, static_cast<int>(seq),
                                                 heads, kv_heads, kLog2e * scale, status_word_ptr());
  TDSV_LAUNCH_CHECK();

  attn_dq_finalize_kernel<<<dim3(static_cast<unsigned>(seq / 32), static_cast<unsigned>(heads),
                                 static_cast<unsigned>(batch)),
                            256, 0, stream()>>>(dq_acc.data_ptr<float>(),
                                                reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                                static_cast<int>(seq), heads, scale);
  TDSV_LAUNCH_CHECK();
  const int64_t n8 = n_kv / 8;
  attn_dkv_finalize_kernel<<<static_cast<unsigned>(std::min<int64_t>((n8 + 255) / 256, 148 * 8)), 256, 0,
                             stream()>>>(dk_acc.data_ptr<float>(), dv_acc.data_ptr<float>(),
                                         reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
                                         reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), n8, scale);
  TDSV_LAUNCH_CHECK();
  return {dq, dk, dv};
}

}  // namespace tdsv
