// 5th-generation tensor core (tcgen05) helpers for sm_100a kernels: tensor
// memory (TMEM) allocation, UMMA shared-memory and instruction descriptors, the
// kind::tf32 MMA, its commit to an mbarrier and the TMEM -> register load.
// Layouts follow the PTX ISA's tcgen05 chapter; field positions match the
// UMMA descriptors of CUTLASS's cute/arch/mma_sm100_desc.hpp.
#pragma once
#include <cstdint>

#include "mbarrier.cuh"

namespace yuf {

// ---- tensor memory ---------------------------------------------------------
// One full warp allocates `cols` columns (a power of two >= 32) for all 128
// lanes and writes the TMEM address into shared memory at `slot`.
YUF_DEVICE void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(cols)
               : "memory");
}
// Let other CTAs on this SM allocate (same warp as the allocation).
YUF_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
YUF_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// Order tcgen05 operations around a CTA barrier (before: issue side, after: wait side).
YUF_DEVICE void tc_fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
YUF_DEVICE void tc_fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- descriptors -----------------------------------------------------------
// Shared-memory matrix descriptor, K-major operand without swizzle: the tile is
// made of core matrices of 8 rows x 16 bytes (128 contiguous bytes); `lbo` is
// the byte distance between core matrices adjacent in K, `sbo` between core
// matrices adjacent in M/N (the next 8 rows).  Addresses and offsets are 16-byte
// multiples; bits 46-47 hold the descriptor version (1 on sm_100).
YUF_DEVICE uint64_t umma_desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle the
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 bytes (64 bf16), the
// 16-byte chunk c of row r stored at chunk c ^ (r % 8) of its 1024-byte group of
// eight rows; the next eight rows 1024 bytes on (SBO), LBO unused (one swizzle
// atom spans the MMA's K).  The tile must start on a 1024-byte boundary; a k
// step inside the row advances `saddr` by its byte offset (the swizzle is a
// function of the address bits, so the hardware finds the chunks the TMA
// placed).  Layout type 2 (bits 61-63) = SWIZZLE_128B.
YUF_DEVICE uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}
// Instruction descriptor of a dense kind::f16 MMA with bf16 A and B (bits 7-9 and
// 10-12 = 1), fp32 accumulators (bits 4-5 = 1), both operands K-major.
constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor of a dense kind::tf32 MMA with fp32 accumulators,
// both operands K-major: D format f32 (bits 4-5 = 1), A and B tf32 (bits 7-9 and
// 10-12 = 2), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t umma_idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- MMA -------------------------------------------------------------------
// D[tmem] (+)= A . B^T, issued by ONE thread; accumulate = 0 overwrites D.
YUF_DEVICE void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// D[tmem] (+)= A . B^T for bf16 operands (kind::f16), issued by ONE thread.
YUF_DEVICE void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
YUF_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---- CTA pairs (cta_group::2: one MMA over the tensor cores of two SMs) ----
// The pair is a cluster of two CTAs; the even rank (peer 0) issues the MMAs,
// whose A rows and B columns are split between the two CTAs' shared memory at
// the same offsets, and whose accumulator rows live in each CTA's own TMEM.
YUF_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `local` (a shared::cta address) in CTA `rank`
YUF_DEVICE uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// arrive on an mbarrier of another CTA of the cluster (address from mapa_shared)
YUF_DEVICE void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// four floats of another CTA's shared memory (address from mapa_shared)
YUF_DEVICE float4 ld_shared_cluster_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
// every thread of every CTA of the cluster
YUF_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMEM of the pair: one warp with the same warp index in each CTA
YUF_DEVICE void tmem_alloc_pair(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
}
YUF_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
YUF_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// D (M = 256 across the pair) (+)= A . B^T, bf16, issued by one thread of peer 0
YUF_DEVICE void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Arrive on the barrier at `bar`'s offset in every CTA of `cta_mask` once the
// pair MMAs issued so far have completed.
YUF_DEVICE void umma_commit_pair_multicast(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
YUF_DEVICE void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- TMEM -> registers -----------------------------------------------------
// The warp's 32 lanes starting at the lane field of `taddr` (a warp may only
// read its own quarter of the lanes: 32 * (warp % 4)), 8 consecutive 32-bit
// columns each: thread t of the warp receives lane (base + t).  The load and its
// completion wait (tcgen05.wait::ld) sit in one asm statement, so no instruction
// can touch the destination registers before they are valid.
YUF_DEVICE void tmem_ld_x8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive 32-bit columns of the warp's 32 TMEM lanes (thread t: lane
// base + t), with the completion wait in the same asm statement.
YUF_DEVICE void tmem_ld_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace yuf
