// DeepSeek-V4 sparse-indexer scores on the 5th-generation tensor cores (sm_100a).
//
//   score[b, l, c] = d^-1/2 * sum_h w[b, l, h] * relu(q[b, l, h, :] . k[b, starts[b, l] + c, :])
//   for c in [0, width); -inf where starts + c >= ends[b, l] or the candidate mask is false.
//
// One CTA per block of QB = 128 / Hi consecutive queries of one batch row. The block's 128
// (query, head) rows are the MMA's N operand; keys stream through in 128-row tiles as the M
// operand, so S^T = K Q^T puts one key per TMEM lane and each epilogue thread reduces the heads
// of every query of the block for its key in registers (no [B, L, width, Hi] tensor, no
// cross-thread reduction). The key range of the block is [min starts, max starts + width); inside
// one packed sequence every query shares `starts`, so the range is exactly `width` keys.
//
//   warp 0     TMA producer: the Q block once, then key tiles through a three-stage ring
//   warp 1     MMA issuer (M = 128 keys, N = 128 rows, K = head dim), TMEM double-buffered
//   warps 2-9  epilogue, two per TMEM lane quarter (each owns half of the block's queries): relu,
//              head weights, head reduction in registers, masked coalesced stores
//
// Reference: dsv41_train/models/dsv4/attention/sparse_indexer.py:17-78 (Triton, one program per
// query and 64 keys) and its PyTorch restatement at lines 156-172.
#include "common.cuh"
#include "tc_util.cuh"

#include <climits>
#include <mutex>

namespace tdsv {

namespace {

constexpr int kRows = 128;            // (query, head) rows per CTA and keys per tile
constexpr int kStages = 3;
constexpr int kAtomBytes = 128 * 128; // [128 rows x 64 bf16]
constexpr int kMaxDim = 128;

enum : int { kWaitEmpty = 401, kWaitQ, kWaitFull, kWaitAccFree, kWaitAcc };

struct IdxSmem {
  alignas(1024) uint8_t q[kMaxDim / 64][kAtomBytes];
  alignas(1024) uint8_t k[kStages][kMaxDim / 64][kAtomBytes];
  float w[kRows];
  int start[kRows];
  int end[kRows];
  int kmin, ntiles;
  uint64_t q_full;
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_free[2];
  uint32_t tmem_base;
};

constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps (two per TMEM lane quarter)

template <int H>
__global__ void __launch_bounds__(kThreads, 1) index_scores_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, const float* __restrict__ weights,
    const int* __restrict__ starts, const int* __restrict__ ends, const bool* __restrict__ candidates,
    float* __restrict__ out, int seq, int key_len, int dim, int width, float scale, int* __restrict__ status) {
  constexpr int heads = H;
  extern __shared__ uint8_t smem_raw[];
  IdxSmem& sm = *reinterpret_cast<IdxSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = kRows / heads;  // queries per CTA
  const int b = blockIdx.y;
  const int l0 = blockIdx.x * qb;
  const int atoms = dim / 64;
  const int64_t qrow0 = static_cast<int64_t>(b) * seq + l0;

  // per-query metadata; the key range is computed by warp 0
  for (int i = threadIdx.x; i < kRows; i += blockDim.x) {
    const int q = i / heads;
    const bool live = l0 + q < seq;
    sm.w[i] = live ? weights[(qrow0 + q) * heads + (i % heads)] : 0.f;
    if (i < qb) {
      sm.start[i] = live ? starts[qrow0 + i] : 0;
      sm.end[i] = live ? ends[qrow0 + i] : 0;
    }
  }
  if (warp == 0) {
    int lo = INT_MAX, hi = INT_MIN;
    for (int q = lane; q < qb; q += 32)
      if (l0 + q < seq) {
        const int s = starts[qrow0 + q];
        lo = min(lo, s);
        hi = max(hi, s + width);
      }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, m));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, m));
    }
    if (lane == 0) {
      sm.kmin = lo;
      sm.ntiles = (hi - lo + kRows - 1) / kRows;
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_free[s], 256);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 2 * kRows);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int kmin = sm.kmin, ntiles = sm.ntiles;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      mbar_arrive_expect_tx(&sm.q_full, atoms * kAtomBytes);
      for (int a = 0; a < atoms; ++a) tma_load_2d(sm.q[a], &tq, &sm.q_full, a * 64, static_cast<int>(qrow0 * heads));
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&sm.empty[s], ((t / kStages) - 1) & 1, status, kWaitEmpty)) break;
        mbar_arrive_expect_tx(&sm.full[s], atoms * kAtomBytes);
        for (int a = 0; a < atoms; ++a) tma_load_3d(sm.k[s][a], &tk, &sm.full[s], a * 64, kmin + t * kRows, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = make_idesc_bf16(kRows, kRows, false, false);
      const uint32_t qa = smem_u32(sm.q[0]);
      bool ok = mbar_wait(&sm.q_full, 0, status, kWaitQ);
      for (int t = 0; ok && t < ntiles; ++t) {
        const int s = t % kStages, buf = t & 1;
        if (!(ok = mbar_wait(&sm.full[s], (t / kStages) & 1, status, kWaitFull))) break;
        if (t >= 2 && !(ok = mbar_wait(&sm.acc_free[buf], ((t >> 1) - 1) & 1, status, kWaitAccFree))) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(sm.k[s][0]);
        for (int kk = 0; kk < dim / 16; ++kk)
          umma_f16(tmem + buf * kRows, kmajor_desc(ka, kk, kAtomBytes), kmajor_desc(qa, kk, kAtomBytes), idesc, kk > 0);
        umma_commit(&sm.empty[s]);
        umma_commit(&sm.acc_full[buf]);
      }
    }
  } else {
    // thread <-> key (TMEM lane); `half` owns accumulator columns [64 half, 64 half + 64), i.e. the
    // queries [64 half / H, (64 half + 64) / H) of the block (all heads of a query in one half)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + half * 64;
    const int64_t out_row0 = qrow0 * width;
    constexpr int G = H < 32 ? H : 32;  // heads of one query inside a 32-column chunk
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (!warp_wait(&sm.acc_full[buf], (t >> 1) & 1, status, kWaitAcc)) break;
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(lane_addr + buf * kRows, v[0]);
      tmem_ld_32x32b_x32(lane_addr + buf * kRows + 32, v[1]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.acc_free[buf]);
      const int key = kmin + t * kRows + quarter * 32 + lane;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int g0 = 0; g0 < 32; g0 += G) {
          const int n0 = half * 64 + c * 32 + g0;  // first accumulator column of this head group
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int i = 0; i < G; i += 2) {
            s0 = fmaf(sm.w[n0 + i], fmaxf(__uint_as_float(v[c][g0 + i]), 0.f), s0);
            s1 = fmaf(sm.w[n0 + i + 1], fmaxf(__uint_as_float(v[c][g0 + i + 1]), 0.f), s1);
          }
          acc += s0 + s1;
          if ((n0 + G) % H == 0) {  // last head group of query n0 / H
            const int q = n0 / H;
            const int col = key - sm.start[q];
            if (l0 + q < seq && col >= 0 && col < width) {
              const int64_t o = out_row0 + static_cast<int64_t>(q) * width + col;
              const bool valid = key < sm.end[q] && (candidates == nullptr || candidates[o]);
              out[o] = valid ? acc * scale : -INFINITY;
            }
            acc = 0.f;
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 2 * kRows);
  }
}

CUtensorMap bf16_map(const at::Tensor& t, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                     const cuuint32_t* box) {
  bind_primary_context();
  TDSV_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "index scores: tensor base must be 16-byte aligned");
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

}  // namespace

// query [B, L, Hi, D] bf16, keys [B, Lk, D] bf16, weights [B, L, Hi] fp32, starts / ends [B, L] int32,
// candidates [B, L, width] bool (optional) -> scores [B, L, width] fp32.
at::Tensor index_scores(const at::Tensor& query, const at::Tensor& keys, const at::Tensor& weights,
                        const at::Tensor& starts, const at::Tensor& ends, int64_t width,
                        const c10::optional<at::Tensor>& candidates) {
  check_cuda_tensor(query, "index query");
  check_cuda_tensor(keys, "index keys");
  check_cuda_tensor(weights, "index weights");
  check_cuda_tensor(starts, "index starts");
  check_cuda_tensor(ends, "index ends");
  TDSV_CHECK(query.dim() == 4 && keys.dim() == 3 && query.scalar_type() == at::kBFloat16 &&
                 keys.scalar_type() == at::kBFloat16,
             "index scores: bf16 query [B, L, H, D] and keys [B, Lk, D]");
  const int64_t batch = query.size(0), seq = query.size(1), heads = query.size(2), dim = query.size(3);
  const int64_t key_len = keys.size(1);
  TDSV_CHECK(keys.size(0) == batch && keys.size(2) == dim, "index scores: keys must share batch and head dim");
  TDSV_CHECK(dim == 64 || dim == 128, "index scores: head dim 64 or 128");
  TDSV_CHECK(heads >= 4 && heads <= 64 && (heads & (heads - 1)) == 0, "index scores: heads a power of two in [4, 64]");
  TDSV_CHECK(weights.scalar_type() == at::kFloat && weights.numel() == batch * seq * heads, "index weights [B, L, H] fp32");
  TDSV_CHECK(starts.scalar_type() == at::kInt && ends.scalar_type() == at::kInt && starts.numel() == batch * seq &&
                 ends.numel() == batch * seq,
             "index starts / ends: int32 [B, L]");
  TDSV_CHECK(width >= 0 && width < (1 << 30) && key_len < (1 << 30) && batch * seq * heads < (int64_t(1) << 31),
             "index scores: sizes out of range");
  const bool* cand = nullptr;
  if (candidates.has_value() && candidates->defined()) {
    check_cuda_tensor(*candidates, "index candidates");
    TDSV_CHECK(candidates->scalar_type() == at::kBool && candidates->numel() == batch * seq * width,
               "index candidates: bool [B, L, width]");
    cand = candidates->data_ptr<bool>();
  }
  auto out = at::empty({batch, seq, width}, query.options().dtype(at::kFloat));
  if (batch == 0 || seq == 0 || width == 0) return out;
  c10::cuda::CUDAGuard guard(query.device());
  const cuuint64_t qdims[2] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(batch * seq * heads)};
  const cuuint64_t qstr[1] = {static_cast<cuuint64_t>(dim) * 2};
  const cuuint32_t qbox[2] = {64, kRows};
  const cuuint64_t kdims[3] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(key_len),
                               static_cast<cuuint64_t>(batch)};
  const cuuint64_t kstr[2] = {static_cast<cuuint64_t>(dim) * 2, static_cast<cuuint64_t>(key_len * dim) * 2};
  const cuuint32_t kbox[3] = {64, kRows, 1};
  const CUtensorMap mq = bf16_map(query, 2, qdims, qstr, qbox);
  const CUtensorMap mk = bf16_map(keys, 3, kdims, kstr, kbox);
  const size_t smem = sizeof(IdxSmem) + 1024;
  const int qb = static_cast<int>(kRows / heads);
  dim3 grid(static_cast<unsigned>((seq + qb - 1) / qb), static_cast<unsigned>(batch));
  auto launch = [&](auto kernel) {
    static std::once_flag once[7];
    std::call_once(once[__builtin_ctz(static_cast<unsigned>(heads))], [&] {
      TDSV_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    });
    kernel<<<grid, kThreads, smem, stream()>>>(mq, mk, weights.data_ptr<float>(), starts.data_ptr<int>(),
                                               ends.data_ptr<int>(), cand, out.data_ptr<float>(), static_cast<int>(seq),
                                               static_cast<int>(key_len), static_cast<int>(dim), static_cast<int>(width),
                                               1.f / sqrtf(static_cast<float>(dim)), status_word_ptr());
  };
  switch (heads) {
    case 4: launch(index_scores_kernel<4>); break;
    case 8: launch(index_scores_kernel<8>); break;
    case 16: launch(index_scores_kernel<16>); break;
    case 32: launch(index_scores_kernel<32>); break;
    default: launch(index_scores_kernel<64>); break;
  }
  TDSV_LAUNCH_CHECK();
  return out;
}

}  // namespace tdsv
