// Tensor-memory-accelerator (TMA) helpers for sm_100a kernels: the driver's
// tensor-map encoder (host) and the 2-D tiled global -> shared copy onto an
// mbarrier (device).  Loads are per CTA only (no cluster multicast).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mbarrier.cuh"

namespace yuf {

// cuTensorMapEncodeTiled looked up once through the runtime (nullptr when the
// driver has none).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// One box of a 2-D tensor map at element coordinates (x = innermost, y) into
// this CTA's shared memory; completes `bytes` (the whole box, also where it
// reaches past the tensor and is zero-filled) on `bar`.  x times the element
// size must be a multiple of 16 bytes.
YUF_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// The same load issued by either CTA of a cta_group::2 pair: the box lands in
// the issuing CTA's shared memory and completes its bytes on the mbarrier at
// shared::cluster address `bar_cluster` (peer 0's, from mapa_shared).
YUF_DEVICE void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

}  // namespace yuf
