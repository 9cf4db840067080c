// Persistent warp-specialised tcgen05 GEMM for sm_100a (B200).
//
//   C[M, N] (+)= A[M, K] * B[N, K]^T      bf16 operands, fp32 accumulation in tensor memory.
//
// Roles inside one CTA (192 threads, one CTA per SM):
//   warp 0     TMA producer: 128B-swizzled tiles of A and B into a ring of shared-memory stages
//   warp 1     MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM accumulator
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (each warp owns its 32-lane TMEM quarter),
//              conversion and global stores; the accumulator is double buffered so the epilogue
//              of tile i overlaps the MMAs of tile i+1.
//
// Operand majors: A is K-major ([M, K] row-major) or M-major ([K, M] row-major); B is K-major
// ([N, K]) or N-major ([K, N]). The MN-major forms are what the backward passes need (dX = dY W,
// dW = dY^T X) without any transposition kernel.
//
// Scheduling modes:
//   kDense   one problem
//   kGroupM  expert-grouped along M (MoE forward and dX): group g owns rows [off_g, off_g + rows_g)
//            of A and C (rows_g a multiple of 128) and uses B[g] of a [G, N, K] (or [G, K, N]) tensor
//   kGroupK  expert-grouped along K (MoE weight gradients): C[g] = A_g^T B_g where A_g, B_g are rows
//            [off_g, off_g + rows_g) of [R, M] and [R, N] tensors (both MN-major).
// Group sizes live on the device, so no host synchronisation is needed between routing and GEMMs.
//
// Every mbarrier wait is bounded (see common.cuh); a timeout records a status code and the CTA
// drains and exits instead of spinning forever.
#include "common.cuh"

#include <mutex>

namespace tdsv {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle atom row
constexpr int kThreads = 192;
constexpr int kMaxGroups = 512;

enum Mode : int { kDense = 0, kGroupM = 1, kGroupK = 2 };
enum Epi : int { kStoreBF16 = 0, kStoreF32 = 1, kAccumF32 = 2 };

struct Params {
  int M, N, K;           // dense problem (kGroupM: N, K used; kGroupK: M, N used)
  int num_groups;
  const int* group_off;  // [G] start row of each group
  const int* group_rows; // [G] rows of each group (kGroupM: multiple of 128; kGroupK: multiple of 64)
  void* C;
  int64_t ldc;           // row stride of C (elements)
  int64_t group_stride_c;// kGroupK: elements between consecutive groups' outputs
  int epi;
  int* status;
};

constexpr int kStageC = 32 * 128;  // one warp's epilogue chunk: 32 rows x 128 bytes

template <int BN>
struct Smem {
  static constexpr int kStageA = BM * BK * 2;
  static constexpr int kStageB = BN * BK * 2;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kBytes = kStages * (kStageA + kStageB) + 4 * kStageC + 1024 /*align*/ + 512 /*barriers*/ +
                                kMaxGroups * 4 /*group tile prefix*/;
};

struct TileInfo {
  int group;
  int m0;      // row offset into A/C (kDense/kGroupM) or output row block (kGroupK)
  int n0;
  int k_begin; // first K index (kGroupK: absolute row)
  int k_len;
  int m_limit; // exclusive row bound for stores
};

template <int MODE, int BN>
__device__ __forceinline__ bool tile_info(const Params& p, const int* prefix, int total_tiles, int tile,
                                          TileInfo& ti) {
  if (tile >= total_tiles) return false;
  const int n_blocks = (p.N + BN - 1) / BN;
  if (MODE == kDense) {
    const int m_blocks = (p.M + BM - 1) / BM;
    int mb, nb;
    if (m_blocks <= n_blocks) {  // the smaller dimension varies fastest -> operand reuse in L2
      mb = tile % m_blocks;
      nb = tile / m_blocks;
    } else {
      nb = tile % n_blocks;
      mb = tile / n_blocks;
    }
    ti.group = 0;
    ti.m0 = mb * BM;
    ti.n0 = nb * BN;
    ti.k_begin = 0;
    ti.k_len = p.K;
    ti.m_limit = p.M;
  } else if (MODE == kGroupM) {
    // prefix[g] = first tile of group g (exclusive scan of (rows_g/128) * n_blocks)
    int lo = 0, hi = p.num_groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int local = tile - prefix[g];
    const int m_blocks_g = p.group_rows[g] / BM;
    const int mb = local % m_blocks_g;
    const int nb = local / m_blocks_g;
    ti.group = g;
    ti.m0 = p.group_off[g] + mb * BM;
    ti.n0 = nb * BN;
    ti.k_begin = 0;
    ti.k_len = p.K;
    ti.m_limit = p.group_off[g] + p.group_rows[g];
  } else {
    const int m_blocks = (p.M + BM - 1) / BM;
    const int per_group = m_blocks * n_blocks;
    const int g = tile / per_group;
    const int local = tile % per_group;
    const int mb = local % m_blocks;
    const int nb = local / m_blocks;
    ti.group = g;
    ti.m0 = mb * BM;
    ti.n0 = nb * BN;
    ti.k_begin = p.group_off[g];
    ti.k_len = p.group_rows[g];
    ti.m_limit = p.M;
  }
  return true;
}

template <bool A_MN, bool B_MN, int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const Params p) {
  using S = Smem<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kStages * S::kStageA;
  uint8_t* smem_c = smem_b + kStages * S::kStageB;  // 4 x kStageC epilogue staging (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_c + 4 * kStageC);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;   // [2]
  uint64_t* tempty = tfull + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* aborted = reinterpret_cast<int*>(tmem_slot + 1);
  int* total_tiles_s = aborted + 1;
  int* prefix = reinterpret_cast<int*>(full + 64);  // after the 512-byte barrier area

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *aborted = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  // tile prefix for grouped-M scheduling
  if (MODE == kGroupM) {
    if (threadIdx.x == 32) {
      const int n_blocks = (p.N + BN - 1) / BN;
      int acc = 0;
      for (int g = 0; g < p.num_groups; ++g) {
        prefix[g] = acc;
        acc += (p.group_rows[g] / BM) * n_blocks;
      }
      *total_tiles_s = acc;
    }
  } else if (threadIdx.x == 32) {
    const int n_blocks = (p.N + BN - 1) / BN;
    const int m_blocks = (p.M + BM - 1) / BM;
    *total_tiles_s = MODE == kDense ? m_blocks * n_blocks : m_blocks * n_blocks * p.num_groups;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = *total_tiles_s;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      uint32_t it = 0;
      TileInfo ti;
      for (int tile = blockIdx.x; tile_info<MODE, BN>(p, prefix, total_tiles, tile, ti); tile += gridDim.x) {
        const int kb_count = (ti.k_len + BK - 1) / BK;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, kTimeoutEmpty)) { *aborted = 1; break; }
          if (*(volatile int*)aborted) break;
          mbar_arrive_expect_tx(&full[s], S::kStageA + S::kStageB);
          const int k0 = ti.k_begin + kb * BK;
          uint8_t* sa = smem_a + s * S::kStageA;
          uint8_t* sb = smem_b + s * S::kStageB;
          if (!A_MN) {
            tma_load_2d(sa, &tma_a, &full[s], k0, ti.m0);
          } else {
            tma_load_2d(sa, &tma_a, &full[s], ti.m0, k0);
            tma_load_2d(sa + 8192, &tma_a, &full[s], ti.m0 + 64, k0);
          }
          if (!B_MN) {
            if (MODE == kGroupM) tma_load_3d(sb, &tma_b, &full[s], k0, ti.n0, ti.group);
            else tma_load_2d(sb, &tma_b, &full[s], k0, ti.n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) {
              if (MODE == kGroupM) tma_load_3d(sb + c * 8192, &tma_b, &full[s], ti.n0 + 64 * c, k0, ti.group);
              else tma_load_2d(sb + c * 8192, &tma_b, &full[s], ti.n0 + 64 * c, k0);
            }
          }
        }
        if (*(volatile int*)aborted) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      uint32_t it = 0, tcount = 0;
      TileInfo ti;
      for (int tile = blockIdx.x; tile_info<MODE, BN>(p, prefix, total_tiles, tile, ti);
           tile += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1, p.status, kTimeoutAccumFree)) { *aborted = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kb_count = (ti.k_len + BK - 1) / BK;
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[s], ph, p.status, kTimeoutFull)) { *aborted = 1; ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem_a + s * S::kStageA);
          const uint32_t sb = smem_u32(smem_b + s * S::kStageB);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if (!A_MN) adesc = make_smem_desc_sw128(sa + kk * 32, 16, 1024);
            else adesc = make_smem_desc_sw128(sa + kk * 2048, 8192, 1024);
            if (!B_MN) bdesc = make_smem_desc_sw128(sb + kk * 32, 16, 1024);
            else bdesc = make_smem_desc_sw128(sb + kk * 2048, 8192, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    // Each warp drains its 32 TMEM lanes in chunks of 128-byte rows (64 bf16 or 32 fp32 columns),
    // writes them 128B-swizzled into its own shared staging buffer and issues one TMA store (or
    // TMA reduce-add for accumulation) per chunk; the TMA clips rows/columns outside the output.
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    uint8_t* stage = smem_c + quarter * kStageC;
    const uint32_t stage_u32 = smem_u32(stage);
    const bool bf16_out = p.epi == kStoreBF16;
    const int cols_per_chunk = bf16_out ? 64 : 32;
    uint32_t tcount = 0;
    TileInfo ti;
    for (int tile = blockIdx.x; tile_info<MODE, BN>(p, prefix, total_tiles, tile, ti);
         tile += gridDim.x, ++tcount) {
      const int buf = tcount & 1;
      const uint32_t tph = (tcount >> 1) & 1;
      if (!mbar_wait(&tfull[buf], tph, p.status, kTimeoutAccum)) { *aborted = 1; break; }
      tc_fence_after();
      const bool zero = ti.k_len <= 0;
      const uint32_t t_addr = tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row0 = ti.m0 + quarter * 32;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += cols_per_chunk) {
        uint32_t r[64];
        tmem_ld_32x32b_x32(t_addr + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (bf16_out) tmem_ld_32x32b_x32(t_addr + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        // the previous chunk's TMA must have finished reading the staging buffer
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
        uint8_t* my_row = stage + lane * 128;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint4 v;
          if (bf16_out) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float a = zero ? 0.f : __uint_as_float(r[g * 8 + 2 * i]);
              const float b = zero ? 0.f : __uint_as_float(r[g * 8 + 2 * i + 1]);
              h[i] = __floats2bfloat162_rn(a, b);
            }
            v = *reinterpret_cast<uint4*>(h);
          } else {
            v.x = zero ? 0u : r[g * 4 + 0];
            v.y = zero ? 0u : r[g * 4 + 1];
            v.z = zero ? 0u : r[g * 4 + 2];
            v.w = zero ? 0u : r[g * 4 + 3];
          }
          *reinterpret_cast<uint4*>(my_row + ((g ^ (lane & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && ti.n0 + c0 < p.N && row0 < ti.m_limit) {
          const int x = ti.n0 + c0;
          if (MODE == kGroupK) {
            if (p.epi == kAccumF32) tma_reduce_add_3d(&tma_c, stage_u32, x, row0, ti.group);
            else tma_store_3d(&tma_c, stage_u32, x, row0, ti.group);
          } else {
            if (p.epi == kAccumF32) tma_reduce_add_2d(&tma_c, stage_u32, x, row0);
            else tma_store_2d(&tma_c, stage_u32, x, row0);
          }
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no libcuda link dependency).
// ---------------------------------------------------------------------------------------------
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    TDSV_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// The driver API needs a current context; a fresh host thread (the autograd engine's worker,
// a Python thread) has none until a runtime call binds the primary context of its device.
void bind_primary_context() {
  static thread_local int bound_device = -1;
  int dev = 0;
  TDSV_CUDA_CHECK(cudaGetDevice(&dev));
  if (bound_device != dev) {
    TDSV_CUDA_CHECK(cudaSetDevice(dev));
    TDSV_CUDA_CHECK(cudaFree(nullptr));
    bound_device = dev;
  }
}

namespace {

// Row-major tensor [outer..., rows, inner] with a box of {box_inner, box_rows, 1...}, 128B swizzle.
CUtensorMap make_map(const at::Tensor& t, int box_rows, int box_inner = 64) {
  bind_primary_context();
  check_cuda_tensor(t, "gemm operand");
  const bool bf16 = t.scalar_type() == at::kBFloat16;
  TDSV_CHECK(bf16 || t.scalar_type() == at::kFloat, "gemm tensors must be bf16 (operands) or fp32 (outputs)");
  const int esize = bf16 ? 2 : 4;
  TDSV_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "gemm tensor base must be 16-byte aligned");
  const int rank = static_cast<int>(t.dim());
  TDSV_CHECK(rank == 2 || rank == 3, "gemm tensors must be 2-D or 3-D");
  cuuint64_t dims[3];
  cuuint64_t strides[2];
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  dims[0] = static_cast<cuuint64_t>(t.size(rank - 1));
  dims[1] = static_cast<cuuint64_t>(t.size(rank - 2));
  TDSV_CHECK((dims[0] * esize) % 16 == 0, "gemm inner dimension must be a multiple of 16 bytes");
  strides[0] = dims[0] * esize;
  if (rank == 3) {
    dims[2] = static_cast<cuuint64_t>(t.size(0));
    strides[1] = dims[0] * dims[1] * esize;
  }
  CUtensorMap map;
  CUresult r = encode_fn()(&map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank,
                           t.data_ptr(), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

// Output map: 32-row boxes of 128 bytes (64 bf16 or 32 fp32 columns).
CUtensorMap make_out_map(const at::Tensor& out) {
  return make_map(out, 32, out.scalar_type() == at::kBFloat16 ? 64 : 32);
}

template <bool A_MN, bool B_MN, int BN, int MODE>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const Params& p, int max_tiles) {
  using S = Smem<BN>;
  auto kern = gemm_tc_kernel<A_MN, B_MN, BN, MODE>;
  static bool configured = false;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured) {
      TDSV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
      configured = true;
    }
  }
  const int grid = std::max(1, std::min(num_sms(), max_tiles));
  // Launch through an argument array that points at our own 64-byte aligned tensor maps rather
  // than through the <<<>>> stub, which passes the over-aligned CUtensorMap by value.
  void* args[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mb), const_cast<CUtensorMap*>(&mc),
                  const_cast<Params*>(&p)};
  TDSV_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), args,
                                   S::kBytes, stream()));
}

template <int MODE>
void dispatch(bool a_mn, bool b_mn, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
              const Params& p, int max_tiles) {
#define TDSV_GEMM_CASE(AM, BMN, BNV)                                        \
  if (a_mn == AM && b_mn == BMN && bn == BNV) {                             \
    launch<AM, BMN, BNV, MODE>(ma, mb, mc, p, max_tiles);                   \
    return;                                                                 \
  }
  if constexpr (MODE == kDense) {
    TDSV_GEMM_CASE(false, false, 256)
    TDSV_GEMM_CASE(false, false, 128)
    TDSV_GEMM_CASE(false, true, 256)
    TDSV_GEMM_CASE(false, true, 128)
    TDSV_GEMM_CASE(true, true, 256)
    TDSV_GEMM_CASE(true, true, 128)
    TDSV_GEMM_CASE(true, false, 256)
    TDSV_GEMM_CASE(true, false, 128)
  } else if constexpr (MODE == kGroupM) {
    TDSV_GEMM_CASE(false, false, 256)
    TDSV_GEMM_CASE(false, false, 128)
    TDSV_GEMM_CASE(false, true, 256)
    TDSV_GEMM_CASE(false, true, 128)
  } else {
    TDSV_GEMM_CASE(true, true, 256)
    TDSV_GEMM_CASE(true, true, 128)
  }
#undef TDSV_GEMM_CASE
  TORCH_CHECK(false, "unsupported gemm configuration");
}

int epi_code(const at::Tensor& out, bool accumulate) {
  if (out.scalar_type() == at::kBFloat16) {
    TDSV_CHECK(!accumulate, "gemm: accumulation needs an fp32 output");
    return kStoreBF16;
  }
  TDSV_CHECK(out.scalar_type() == at::kFloat, "gemm: output must be bf16 or fp32");
  return accumulate ? kAccumF32 : kStoreF32;
}

}  // namespace

// out[M, N] (+)= A * B^T with A [M, K] (a_mn=false) or [K, M] (a_mn=true) and
// B [N, K] (b_mn=false) or [K, N] (b_mn=true).
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn, bool accumulate) {
  check_cuda_tensor(a, "a");
  check_cuda_tensor(b, "b");
  check_cuda_tensor(out, "out");
  TDSV_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm: 2-D operands");
  const int M = static_cast<int>(a_mn ? a.size(1) : a.size(0));
  const int K = static_cast<int>(a_mn ? a.size(0) : a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(1) : b.size(0));
  TDSV_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: K mismatch");
  TDSV_CHECK(out.size(0) == M && out.size(1) == N, "gemm: output shape mismatch");
  TDSV_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const int bn = N >= 256 ? 256 : 128;
  const CUtensorMap ma = make_map(a, a_mn ? BK : BM);
  const CUtensorMap mb = make_map(b, b_mn ? BK : bn);
  const CUtensorMap mc = make_out_map(out);
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_groups = 1;
  p.C = out.data_ptr();
  p.ldc = out.stride(0);
  p.epi = epi_code(out, accumulate);
  p.status = status_word_ptr();
  if (K == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  dispatch<kDense>(a_mn, b_mn, bn, ma, mb, mc, p, tiles);
}

// Expert-grouped along M: out[off_g : off_g + rows_g] = A[off_g : ...] * B[g]^T.
// b is [G, N, K] (b_mn=false) or [G, K, N] (b_mn=true); rows_g must be multiples of 128.
void grouped_gemm_m(const at::Tensor& a, const at::Tensor& b, const at::Tensor& group_off,
                    const at::Tensor& group_rows, at::Tensor& out, bool b_mn, int64_t max_rows) {
  check_cuda_tensor(a, "a");
  check_cuda_tensor(b, "b");
  check_cuda_tensor(out, "out");
  TDSV_CHECK(a.dim() == 2 && b.dim() == 3 && out.dim() == 2, "grouped_gemm_m: a [R,K], b [G,*,*], out [R,N]");
  const int G = static_cast<int>(b.size(0));
  TDSV_CHECK(G <= kMaxGroups, "grouped_gemm_m: too many groups");
  TDSV_CHECK(group_off.numel() == G && group_rows.numel() == G, "grouped_gemm_m: group metadata size");
  TDSV_CHECK(group_off.scalar_type() == at::kInt && group_rows.scalar_type() == at::kInt, "int32 group metadata");
  const int K = static_cast<int>(a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(2) : b.size(1));
  TDSV_CHECK((b_mn ? b.size(1) : b.size(2)) == K, "grouped_gemm_m: K mismatch");
  TDSV_CHECK(out.size(1) == N && out.size(0) == a.size(0), "grouped_gemm_m: output shape");
  TDSV_CHECK(N % 8 == 0, "grouped_gemm_m: N must be a multiple of 8");
  if (a.size(0) == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const int bn = N >= 256 ? 256 : 128;
  const CUtensorMap ma = make_map(a, BM);
  const CUtensorMap mb = make_map(b, b_mn ? BK : bn);
  const CUtensorMap mc = make_out_map(out);
  Params p{};
  p.M = static_cast<int>(a.size(0));
  p.N = N;
  p.K = K;
  p.num_groups = G;
  p.group_off = group_off.data_ptr<int>();
  p.group_rows = group_rows.data_ptr<int>();
  p.C = out.data_ptr();
  p.ldc = out.stride(0);
  p.epi = epi_code(out, false);
  p.status = status_word_ptr();
  const int64_t rows = max_rows > 0 ? max_rows : a.size(0);
  const int max_tiles = static_cast<int>(((rows + BM - 1) / BM) * ((N + bn - 1) / bn));
  dispatch<kGroupM>(false, b_mn, bn, ma, mb, mc, p, max_tiles);
}

// Expert-grouped along K (weight gradients): out[g] = A_g^T * B_g with A_g = a[off_g : off_g + rows_g]
// ([R, M] row-major) and B_g = b[off_g : ...] ([R, N]); out is [G, M, N] fp32 (optionally accumulated)
// or bf16. rows_g must be multiples of 64.
void grouped_gemm_k(const at::Tensor& a, const at::Tensor& b, const at::Tensor& group_off,
                    const at::Tensor& group_rows, at::Tensor& out, bool accumulate) {
  check_cuda_tensor(a, "a");
  check_cuda_tensor(b, "b");
  check_cuda_tensor(out, "out");
  TDSV_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 3, "grouped_gemm_k: a [R,M], b [R,N], out [G,M,N]");
  const int G = static_cast<int>(out.size(0));
  TDSV_CHECK(group_off.numel() == G && group_rows.numel() == G, "grouped_gemm_k: group metadata size");
  const int M = static_cast<int>(a.size(1));
  const int N = static_cast<int>(b.size(1));
  TDSV_CHECK(out.size(1) == M && out.size(2) == N, "grouped_gemm_k: output shape");
  TDSV_CHECK(a.size(0) == b.size(0), "grouped_gemm_k: row mismatch");
  TDSV_CHECK(N % 8 == 0, "grouped_gemm_k: N must be a multiple of 8");
  if (G == 0 || M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const int bn = N >= 256 ? 256 : 128;
  const CUtensorMap ma = make_map(a, BK);
  const CUtensorMap mb = make_map(b, BK);
  const CUtensorMap mc = make_out_map(out);
  Params p{};
  p.M = M;
  p.N = N;
  p.K = 0;
  p.num_groups = G;
  p.group_off = group_off.data_ptr<int>();
  p.group_rows = group_rows.data_ptr<int>();
  p.C = out.data_ptr();
  p.ldc = out.stride(1);
  p.group_stride_c = out.stride(0);
  p.epi = epi_code(out, accumulate);
  p.status = status_word_ptr();
  const int tiles = G * ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  dispatch<kGroupK>(true, true, bn, ma, mb, mc, p, tiles);
}

}  // namespace tdsv
