// Shared-memory mbarrier and bulk-copy (TMA) helpers for sm_100a kernels.
// Every wait is bounded: after WAIT_NS nanoseconds of the global timer the
// waiting thread gives up and the caller records a timeout and leaves.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace yuf {

constexpr unsigned long long WAIT_NS = 200ull * 1000 * 1000;  // 0.2 s

YUF_DEVICE uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
YUF_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
YUF_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
YUF_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
YUF_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
YUF_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
YUF_DEVICE unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// true when the barrier's phase `parity` completed within `limit_ns` (WAIT_NS
// unless a caller passes its own bound)
YUF_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns = WAIT_NS) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (unsigned int it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 63) == 0) {  // look at the clock every 64 polls
      const unsigned long long now = global_ns();
      if (it == 0) t0 = now;
      else if (now - t0 > limit_ns) return false;
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (both
// addresses and the size 16-byte multiples); this CTA only.
YUF_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// 1-D bulk copy shared -> global in the calling thread's bulk group.
YUF_DEVICE void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
YUF_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the source shared memory of all but the newest N committed groups has been read
template <int N>
YUF_DEVICE void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// all committed groups complete (their global writes done)
YUF_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace yuf
