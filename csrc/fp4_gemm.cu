// Expert-grouped tcgen05 GEMM against frozen MXFP4 weights, read packed (sm_100a).
//
//   out[off_g : off_g + rows_g] = A[off_g : off_g + rows_g] * W_g^T      (forward, B K-major)
//   out[off_g : off_g + rows_g] = A[off_g : off_g + rows_g] * W_g        (input gradient, B N-major)
//
// W_g is stored as E2M1 codes (two per byte, low nibble first) with one E8M0 scale per 32
// consecutive values along the packed (last) dimension: codes [G, rows, cols / 2], scales
// [G, rows, cols / 32]. This is the released checkpoint's expert layout
// (dsv41_train/models/dsv4/checkpoint.py:258-279 dequantises it the same way, to bf16 at load
// time). Nothing is expanded in global memory: the weight crosses HBM at 4.25 bits per value.
//
// Roles inside one CTA (448 threads, one CTA per SM):
//   warp 0       TMA producer of the activation tiles (bf16, 128B-swizzled)
//   warp 1       MMA issuer: two tcgen05.mma kind::f16 (M = 128, N = 128, K = 16) per k-step, one per
//                128-row half of the 256-row tile, both reading the same converted weight stage,
//                into double-buffered TMEM accumulators (2 x 256 columns)
//   warps 2-5    epilogue: tcgen05.ld, bf16 conversion, swizzled staging, TMA store
//   warps 6-13   weight producers in two teams of four warps on alternate stages: each thread
//                copies its own 16-byte code pieces (32 values) and the 4-byte word holding each
//                piece's scale into a private slot of its team's raw ring with cp.async, two team
//                stages ahead of the stage it converts, so global latency does not stall the
//                conversion; it then converts the pieces to bf16 with byte permutes
//                and one packed multiply and writes them into the 128B-swizzled layout a TMA load
//                of a bf16 weight would give.
// The 256 x 128 tile halves the conversion work per MMA against a 128 x 256 tile (the weight is
// converted once for twice the rows); an expert's last tile may have only its first half in the
// group, whose second half is computed and not stored.
// Activations and converted weights have separate rings (A deeper, since its TMA loads see the
// full L2/HBM latency; B shallower, since its producers work from shared memory). A B stage's full
// barrier completes when the four warps of the team that owns the stage have arrived after fencing their shared-memory
// writes for the async proxy.
//
// E2M1 -> bf16: the magnitude (3 bits) selects the high and low byte of the unscaled bf16 value
// from two 8-entry byte tables (one prmt each for four values); the sign bits are replicated into
// the high bytes with prmt's sign mode; a prmt pair interleaves the bytes into bf16x2 words; the
// E8M0 scale 2^(s-127) is exact in bf16, so one bf16x2 multiply applies it with no rounding
// (value * scale is exact in fp32 as well, the reference's order of operations, except at the
// far ends of the scale range where a product leaves bf16's normal range).
//
// Every mbarrier wait is bounded: a timeout records a status code, sets the CTA's abort flag and
// every role leaves its loop, so the CTA reaches its final barrier and frees its TMEM.
#include "common.cuh"
#include "tc_util.cuh"

#include <mutex>

namespace tdsv {

namespace {

constexpr int BM = 128;               // rows of one MMA (one TMEM lane per row)
constexpr int kHalves = 2;            // a tile is two MMA row blocks sharing each converted B stage
constexpr int BMT = BM * kHalves;     // rows of a tile
constexpr int BK = 64;
constexpr int kWarpsBase = 6;
constexpr int kProducerWarps = 8;
constexpr int kProducers = kProducerWarps * 32;
constexpr int kThreads = kWarpsBase * 32 + kProducers;
constexpr int kTeams = 2;                        // producer teams, taking alternate pipeline stages
constexpr int kTeamThreads = kProducers / kTeams;
constexpr int kRaw = 3;  // raw slots per team: copies for the team's next kRaw - 1 stages fly while one converts
constexpr int kMaxGroups = 512;
constexpr int kStageC = 32 * 128;

template <int BN>
struct Fp4Smem {
  static constexpr int kStageA = BMT * BK * 2;
  static constexpr int kStageB = BN * BK * 2;
  static constexpr int kStagesA = 4;
  static constexpr int kStagesB = 3;
  static constexpr int kPieces = BN * BK / 32 / kTeamThreads;  // pieces per producer thread per stage
  static_assert(kPieces >= 1 && BN * BK / 32 % kTeamThreads == 0, "whole pieces per producer thread");
  static constexpr int kCodeBytes = kPieces * kTeamThreads * 16;
  static constexpr int kRawSlot = kCodeBytes + kPieces * kTeamThreads * 4;
  static constexpr int kRawBytes = kTeams * kRaw * kRawSlot;
  static constexpr int kBytes = kStagesA * kStageA + kStagesB * kStageB + kRawBytes + 4 * kStageC + 1024 +
                                512 + kMaxGroups * 4;
  static_assert(kRawBytes % 1024 == 0, "epilogue staging must stay 1024-byte aligned");
  static_assert(kBytes <= 232448, "shared memory over the per-CTA opt-in limit");
};

struct Fp4Params {
  int N, K;               // output columns, contraction length
  int num_groups;
  const int* group_off;
  const int* group_rows;  // multiples of 128
  const uint8_t* codes;   // forward: [G, N, K/2]; input gradient: [G, K, N/2]
  const uint8_t* scales;  // forward: [G, N, K/32]; input gradient: [G, K, N/32]
  int* status;
};

struct Tile {
  int group, m0, n0, m_limit;
};

template <int BN>
__device__ __forceinline__ bool tile_at(const Fp4Params& p, const int* prefix, int total, int tile, Tile& t) {
  if (tile >= total) return false;
  int lo = 0, hi = p.num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int local = tile - prefix[lo];
  const int m_blocks = (p.group_rows[lo] + BMT - 1) / BMT;
  t.group = lo;
  t.m0 = p.group_off[lo] + (local % m_blocks) * BMT;
  t.n0 = (local / m_blocks) * BN;
  t.m_limit = p.group_off[lo] + p.group_rows[lo];
  return true;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  __nv_bfloat162 z = __hmul2(x, y);
  return *reinterpret_cast<uint32_t*>(&z);
}

// bf16 bit pattern of 2^(s - 127) for an E8M0 byte (0xFF is NaN; 0 is the subnormal 2^-127).
__device__ __forceinline__ uint32_t e8m0_bf16x2(uint32_t s) {
  const uint32_t h = s == 0xFFu ? 0x7FC0u : (s == 0u ? 0x0040u : (s << 7));
  return h | (h << 16);
}

// Unscaled bf16 of each E2M1 magnitude, split into high and low bytes: 0, .5, 1, 1.5, 2, 3, 4, 6.
constexpr uint32_t kHi0 = 0x3F3F3F00u, kHi1 = 0x40404040u;
constexpr uint32_t kLo0 = 0xC0800000u, kLo1 = 0xC0804000u;

// Eight E2M1 values (one code word, value e in nibble e) -> eight scaled bf16 values.
__device__ __forceinline__ uint4 e2m1x8_to_bf16(uint32_t w, uint32_t scale2) {
  const uint32_t mag = w & 0x77777777u;
  const uint32_t w4 = w << 4;  // byte k's msb = sign of value 2k; w's byte k msb = sign of value 2k+1
  const uint32_t mag_hi = mag >> 16;
  uint32_t hi_a = prmt(kHi0, kHi1, mag);
  const uint32_t lo_a = prmt(kLo0, kLo1, mag);
  uint32_t hi_b = prmt(kHi0, kHi1, mag_hi);
  const uint32_t lo_b = prmt(kLo0, kLo1, mag_hi);
  hi_a |= prmt(w, w4, 0x9D8Cu) & 0x80808080u;
  hi_b |= prmt(w, w4, 0xBFAEu) & 0x80808080u;
  uint4 o;
  o.x = bf16x2_mul(prmt(lo_a, hi_a, 0x5140u), scale2);
  o.y = bf16x2_mul(prmt(lo_a, hi_a, 0x7362u), scale2);
  o.z = bf16x2_mul(prmt(lo_b, hi_b, 0x5140u), scale2);
  o.w = bf16x2_mul(prmt(lo_b, hi_b, 0x7362u), scale2);
  return o;
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Piece u of a stage (32 weight values sharing one scale): B K-major (forward) has two pieces per
// weight row n (the two k halves of the 64-wide stage); B N-major (input gradient) has BN/32
// pieces per contraction row k. Gives the global offsets of its codes and its scale byte, and
// where its four 16-byte bf16 chunks go in the swizzled stage.
struct Piece {
  int64_t code_off, scale_off;
  bool valid;
  int row;     // swizzle row inside its 64-column block
  int block;   // 64-column block (8 KB apart; N-major only)
  int chunk0;  // first of its four 16-byte chunks in the 128-byte row
};

template <bool B_MN, int BN>
__device__ __forceinline__ Piece piece_at(const Fp4Params& p, const Tile& t, int kb, int u) {
  Piece q;
  const int k0 = kb * BK;
  if (!B_MN) {
    const int n = t.n0 + (u >> 1);
    const int h = u & 1;
    q.valid = n < p.N;
    const int64_t row = static_cast<int64_t>(t.group) * p.N + n;
    q.code_off = row * (p.K / 2) + k0 / 2 + 16 * h;
    q.scale_off = row * (p.K / 32) + k0 / 32 + h;
    q.row = u >> 1;
    q.block = 0;
    q.chunk0 = 4 * h;
  } else {
    constexpr int per_row = BN / 32;
    const int r = u / per_row;
    const int piece = u % per_row;
    const int n = t.n0 + 32 * piece;
    q.valid = n < p.N;
    const int64_t row = static_cast<int64_t>(t.group) * p.K + k0 + r;
    q.code_off = row * (p.N / 2) + n / 2;
    q.scale_off = row * (p.N / 32) + n / 32;
    q.row = r;
    q.block = piece >> 1;
    q.chunk0 = 4 * (piece & 1);
  }
  return q;
}

// Copies of one stage's pieces of this thread into its raw slot: codes at [i][tid] x 16 bytes,
// then the aligned 4-byte word holding each scale at [i][tid] x 4 bytes (rows beyond N are
// zero-filled, which converts to 0 whatever the scale).
template <bool B_MN, int BN>
__device__ __forceinline__ void issue_pieces(const Fp4Params& p, const Tile& t, int kb, int tid, uint32_t slot) {
  using S = Fp4Smem<BN>;
#pragma unroll
  for (int i = 0; i < S::kPieces; ++i) {
    const Piece q = piece_at<B_MN, BN>(p, t, kb, tid + kTeamThreads * i);
    cp_async_16(slot + (i * kTeamThreads + tid) * 16, q.valid ? p.codes + q.code_off : p.codes, q.valid);
    cp_async_4(slot + S::kCodeBytes + (i * kTeamThreads + tid) * 4,
               q.valid ? p.scales + (q.scale_off & ~int64_t(3)) : p.scales, q.valid);
  }
}

template <bool B_MN, int BN>
__device__ __forceinline__ void convert_pieces(const Fp4Params& p, const Tile& t, int kb, int tid,
                                               const uint8_t* slot, uint8_t* sb) {
  using S = Fp4Smem<BN>;
#pragma unroll
  for (int i = 0; i < S::kPieces; ++i) {
    const Piece q = piece_at<B_MN, BN>(p, t, kb, tid + kTeamThreads * i);
    const uint4 c = *reinterpret_cast<const uint4*>(slot + (i * kTeamThreads + tid) * 16);
    const uint32_t word = *reinterpret_cast<const uint32_t*>(slot + S::kCodeBytes + (i * kTeamThreads + tid) * 4);
    const uint32_t s2 = e8m0_bf16x2((word >> (8 * static_cast<uint32_t>(q.scale_off & 3))) & 0xFFu);
    uint8_t* row = sb + q.block * 8192 + q.row * 128;
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      *reinterpret_cast<uint4*>(row + (((q.chunk0 + k) ^ (q.row & 7)) << 4)) = e2m1x8_to_bf16(words[k], s2);
    }
  }
}

template <bool B_MN, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    fp4_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_c,
                            const Fp4Params p) {
  using S = Fp4Smem<BN>;
  constexpr int kSA = S::kStagesA, kSB = S::kStagesB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem_a + kSA * S::kStageA;
  uint8_t* smem_raw_ring = smem_b + kSB * S::kStageB;
  uint8_t* smem_c = smem_raw_ring + S::kRawBytes;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem_c + 4 * kStageC);
  uint64_t* empty_a = full_a + kSA;
  uint64_t* full_b = empty_a + kSA;
  uint64_t* empty_b = full_b + kSB;
  uint64_t* tfull = empty_b + kSB;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* aborted = reinterpret_cast<int*>(tmem_slot + 1);
  int* total_s = aborted + 1;
  int* prefix = reinterpret_cast<int*>(full_a + 64);  // after the 512-byte barrier area

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_count = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSA; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kSB; ++s) {
      mbar_init(&full_b[s], kProducerWarps / kTeams);
      mbar_init(&empty_b[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *aborted = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 2 * kHalves * BN);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    const int n_blocks = (p.N + BN - 1) / BN;
    int acc = 0;
    for (int g = 0; g < p.num_groups; ++g) {
      prefix[g] = acc;
      acc += ((p.group_rows[g] + BMT - 1) / BMT) * n_blocks;
    }
    *total_s = acc;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = *total_s;

  if (warp == 0) {
    // ------------------------------------------------------------ activation TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      uint32_t it = 0;
      Tile t;
      for (int tile = blockIdx.x; tile_at<BN>(p, prefix, total, tile, t); tile += gridDim.x) {
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int s = it % kSA;
          if (!mbar_wait(&empty_a[s], ((it / kSA) & 1) ^ 1, p.status, kTimeoutEmpty)) { *aborted = 1; break; }
          if (*(volatile int*)aborted) break;
          mbar_arrive_expect_tx(&full_a[s], S::kStageA);
          tma_load_2d(smem_a + s * S::kStageA, &tma_a, &full_a[s], kb * BK, t.m0);
        }
        if (*(volatile int*)aborted) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, false, B_MN);
      uint32_t it = 0, tcount = 0;
      Tile t;
      for (int tile = blockIdx.x; tile_at<BN>(p, prefix, total, tile, t); tile += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        if (!mbar_wait(&tempty[buf], ((tcount >> 1) & 1) ^ 1, p.status, kTimeoutAccumFree)) { *aborted = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * (kHalves * BN);
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb, ++it) {
          const int sa_i = it % kSA, sb_i = it % kSB;
          if (!mbar_wait(&full_a[sa_i], (it / kSA) & 1, p.status, kTimeoutFull) ||
              !mbar_wait(&full_b[sb_i], (it / kSB) & 1, p.status, kTimeoutFull)) {
            *aborted = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem_a + sa_i * S::kStageA);
          const uint32_t sb = smem_u32(smem_b + sb_i * S::kStageB);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bdesc = !B_MN ? make_smem_desc_sw128(sb + kk * 32, 16, 1024)
                                         : make_smem_desc_sw128(sb + kk * 2048, 8192, 1024);
#pragma unroll
            for (int h = 0; h < kHalves; ++h) {
              const uint64_t adesc = make_smem_desc_sw128(sa + h * (BM * 128) + kk * 32, 16, 1024);
              umma_f16(d_tmem + h * BN, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty_a[sa_i]);
          umma_commit(&empty_b[sb_i]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else if (warp < kWarpsBase) {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    uint8_t* stage = smem_c + quarter * kStageC;
    const uint32_t stage_u32 = smem_u32(stage);
    uint32_t tcount = 0;
    Tile t;
    for (int tile = blockIdx.x; tile_at<BN>(p, prefix, total, tile, t); tile += gridDim.x, ++tcount) {
      const int buf = tcount & 1;
      if (!warp_wait(&tfull[buf], (tcount >> 1) & 1, p.status, kTimeoutAccum)) {
        if (lane == 0) *aborted = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_addr = tmem_base + buf * (kHalves * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int cc = 0; cc < kHalves * BN; cc += 64) {
        const int h = cc / BN, c0 = cc % BN;
        const int row0 = t.m0 + h * BM + quarter * 32;
        uint32_t r[64];
        tmem_ld_32x32b_x32(t_addr + cc, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(t_addr + cc + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
        uint8_t* my_row = stage + lane * 128;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          __nv_bfloat162 h[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            h[i] = __floats2bfloat162_rn(__uint_as_float(r[g * 8 + 2 * i]), __uint_as_float(r[g * 8 + 2 * i + 1]));
          *reinterpret_cast<uint4*>(my_row + ((g ^ (lane & 7)) << 4)) = *reinterpret_cast<uint4*>(h);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && t.n0 + c0 < p.N && row0 < t.m_limit) {
          tma_store_2d(&tma_c, stage_u32, t.n0 + c0, row0);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  } else {
    // ------------------------------------------------------------ weight producers (warps 6..13)
    // Two teams of four warps take alternate pipeline stages, so one team's conversion overlaps the
    // other's and each has two stage times for its own. Per thread, two cursors walk the team's
    // stages in the pipeline's (tile, k-block) order: one issues raw copies kRaw - 1 team stages
    // ahead, the other converts. A thread reads back only the raw bytes it copied itself, so its
    // own cp.async groups are the only synchronisation the raw ring needs.
    const int pw = warp - kWarpsBase;
    const int team = pw / (kProducerWarps / kTeams);
    const int tid = (pw % (kProducerWarps / kTeams)) * 32 + lane;
    const uint32_t raw0 = smem_u32(smem_raw_ring) + team * kRaw * S::kRawSlot;
    uint8_t* raw0_ptr = smem_raw_ring + team * kRaw * S::kRawSlot;
    struct Cursor {
      int tile, kb;
      Tile t;
      bool have;
    };
    auto step = [&](Cursor& c) {
      if (++c.kb == kb_count) {
        c.kb = 0;
        c.tile += gridDim.x;
        c.have = tile_at<BN>(p, prefix, total, c.tile, c.t);
      }
    };
    auto advance = [&](Cursor& c) {  // to the team's next stage
      for (int k = 0; k < kTeams && c.have; ++k) step(c);
    };
    Cursor ld{static_cast<int>(blockIdx.x), 0, Tile{}, false};
    ld.have = tile_at<BN>(p, prefix, total, ld.tile, ld.t);
    for (int k = 0; k < team && ld.have; ++k) step(ld);
    Cursor cv = ld;
    uint32_t lit = 0;
    auto issue_next = [&]() {
      if (ld.have) {
        issue_pieces<B_MN, BN>(p, ld.t, ld.kb, tid, raw0 + (lit % kRaw) * S::kRawSlot);
        ++lit;
        advance(ld);
      }
      cp_async_commit();  // possibly empty: group j always belongs to the team's stage j
    };
#pragma unroll 1
    for (int j = 0; j < kRaw - 1; ++j) issue_next();
#pragma unroll 1
    for (uint32_t j = 0, it = team; cv.have; ++j, it += kTeams) {
      issue_next();
      cp_async_wait<kRaw - 1>();  // this thread's copies of the team's stage j have landed
      const int s = it % kSB;
      if (!warp_wait(&empty_b[s], ((it / kSB) & 1) ^ 1, p.status, kTimeoutEmpty)) {
        if (lane == 0) *aborted = 1;
        break;
      }
      if (*(volatile int*)aborted) break;
      convert_pieces<B_MN, BN>(p, cv.t, cv.kb, tid, raw0_ptr + (j % kRaw) * S::kRawSlot, smem_b + s * S::kStageB);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_b[s]);
      advance(cv);
    }
    cp_async_wait<0>();  // no copy may still target shared memory when the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kHalves * BN);
  }
}

CUtensorMap bf16_map(const at::Tensor& t, int box_rows) {
  bind_primary_context();
  TDSV_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 2, "fp4 gemm: 2-D bf16 activation / output");
  TDSV_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "fp4 gemm: 16-byte aligned base");
  TDSV_CHECK((t.size(1) * 2) % 16 == 0, "fp4 gemm: row bytes must be a multiple of 16");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(t.size(1)), static_cast<cuuint64_t>(t.size(0))};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(t.size(1)) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

template <bool B_MN, int BN>
void launch_fp4(const CUtensorMap& ma, const CUtensorMap& mc, const Fp4Params& p, int max_tiles) {
  using S = Fp4Smem<BN>;
  auto kern = fp4_grouped_gemm_kernel<B_MN, BN>;
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
  void* args[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mc), const_cast<Fp4Params*>(&p)};
  TDSV_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), args, S::kBytes,
                                   stream()));
}

}  // namespace

// out [R, N] bf16 = a [R, K] bf16 times the packed weight of each row's expert group.
//   b_mn = false: codes [G, N, K/2], scales [G, N, K/32]  (out = a W^T, the forward)
//   b_mn = true:  codes [G, K, N/2], scales [G, K, N/32]  (out = a W, the input gradient)
// Group rows are multiples of 128 (the permuted layout's padding); K is a multiple of 64 and N of
// 32. max_rows bounds the tile count when the routed row count lives only on the device.
void fp4_grouped_gemm(const at::Tensor& a, const at::Tensor& codes, const at::Tensor& scales,
                      const at::Tensor& group_off, const at::Tensor& group_rows, at::Tensor& out, bool b_mn,
                      int64_t max_rows) {
  check_cuda_tensor(a, "a");
  check_cuda_tensor(codes, "codes");
  check_cuda_tensor(scales, "scales");
  check_cuda_tensor(out, "out");
  TDSV_CHECK(codes.scalar_type() == at::kByte && scales.scalar_type() == at::kByte, "fp4 gemm: uint8 codes/scales");
  TDSV_CHECK(a.dim() == 2 && codes.dim() == 3 && scales.dim() == 3 && out.dim() == 2, "fp4 gemm: shapes");
  TDSV_CHECK(out.scalar_type() == at::kBFloat16, "fp4 gemm: bf16 output");
  const int G = static_cast<int>(codes.size(0));
  TDSV_CHECK(G <= kMaxGroups, "fp4 gemm: too many groups");
  TDSV_CHECK(group_off.numel() == G && group_rows.numel() == G, "fp4 gemm: group metadata size");
  TDSV_CHECK(group_off.scalar_type() == at::kInt && group_rows.scalar_type() == at::kInt, "int32 group metadata");
  const int K = static_cast<int>(a.size(1));
  const int N = static_cast<int>(out.size(1));
  TDSV_CHECK(out.size(0) == a.size(0), "fp4 gemm: output rows");
  TDSV_CHECK(K % 64 == 0 && N % 32 == 0, "fp4 gemm: K must be a multiple of 64 and N of 32");
  if (!b_mn) {
    TDSV_CHECK(codes.size(1) == N && codes.size(2) * 2 == K, "fp4 gemm: codes must be [G, N, K/2]");
    TDSV_CHECK(scales.size(1) == N && scales.size(2) * 32 == K, "fp4 gemm: scales must be [G, N, K/32]");
  } else {
    TDSV_CHECK(codes.size(1) == K && codes.size(2) * 2 == N, "fp4 gemm: codes must be [G, K, N/2]");
    TDSV_CHECK(scales.size(1) == K && scales.size(2) * 32 == N, "fp4 gemm: scales must be [G, K, N/32]");
  }
  TDSV_CHECK(reinterpret_cast<uintptr_t>(codes.data_ptr()) % 16 == 0, "fp4 gemm: codes must be 16-byte aligned");
  // scales are copied as the aligned 4-byte words that hold them (never past the word of the last
  // scale, which the allocator's 512-byte granularity keeps inside the allocation)
  TDSV_CHECK(reinterpret_cast<uintptr_t>(scales.data_ptr()) % 4 == 0, "fp4 gemm: scales must be 4-byte aligned");
  if (a.size(0) == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  constexpr int bn = 128;
  const CUtensorMap ma = bf16_map(a, BMT);
  const CUtensorMap mc = bf16_map(out, 32);
  Fp4Params p{};
  p.N = N;
  p.K = K;
  p.num_groups = G;
  p.group_off = group_off.data_ptr<int>();
  p.group_rows = group_rows.data_ptr<int>();
  p.codes = codes.data_ptr<uint8_t>();
  p.scales = scales.data_ptr<uint8_t>();
  p.status = status_word_ptr();
  const int64_t rows = max_rows > 0 ? max_rows : a.size(0);
  // each group's rows round up to whole 256-row tiles, at most one partial tile per group
  const int max_tiles = static_cast<int>(((rows + BMT - 1) / BMT + G) * ((N + bn - 1) / bn));
  if (!b_mn) launch_fp4<false, bn>(ma, mc, p, max_tiles);
  else launch_fp4<true, bn>(ma, mc, p, max_tiles);
}

}  // namespace tdsv
