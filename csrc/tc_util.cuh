// Small tcgen05 / TMA helpers shared by the attention and indexer kernels (sm_100a).
#pragma once

#include "common.cuh"

namespace tdsv {

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
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16. A (M rows x 16 K values per instruction) is
// read from tensor memory: row m in lane m, K values packed two per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Plain bulk copy global -> this CTA's shared memory, completion on an mbarrier. 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// K-major operand stored as 64-column (128-byte) swizzled atoms `atom_bytes` apart along K:
// descriptor of MMA k-step kk (16 columns).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk, uint32_t atom_bytes) {
  return make_smem_desc_sw128(base + (kk >> 2) * atom_bytes + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (K rows x MN columns, MN split into 64-column atoms `atom_bytes` apart):
// k-step kk covers rows 16kk .. 16kk+15.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk, uint32_t atom_bytes) {
  return make_smem_desc_sw128(base + kk * 2048, atom_bytes, 1024);
}

// Bounded wait with mbarrier.try_wait and a suspend-time hint: the thread sleeps in hardware until
// the phase completes instead of polling and taking issue slots from the warps on its scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_sleep_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait_sleep(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) break;
  }
  report_status(status, code);
  return false;
}

// Bounded wait taken by a whole warp: every lane reaches the vote, so the warp leaves converged
// (tcgen05.ld / st are warp-collective) and takes a timeout branch together.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xffffffffu, mbar_sleep_wait(bar, parity, status, code));
}

// 2^x by the special-function unit (PTX ex2.approx.ftz.f32; denormal results flush to zero and
// ex2(-inf) = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled atom.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

}  // namespace tdsv
