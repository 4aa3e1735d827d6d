// Shared helpers for the sm_100a kernels of the WKV-7 + ROSA hot path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/yufb200.h"

#define YUF_DEVICE __device__ __forceinline__

namespace yuf {

// log(retention) = W_SCALE * sigmoid(w_raw); the clamp of yufmusicgen/model.py:156
// and rwkv7_clampw.cu:16,42.
constexpr float W_SCALE = -0.6065306597f;

YUF_DEVICE float sigmoidf_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Packed fp32x2 arithmetic (one sm_100 instruction for two lanes of math).
YUF_DEVICE float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
YUF_DEVICE float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
YUF_DEVICE float2 f2(float x) { return make_float2(x, x); }

template <int WIDTH>
YUF_DEVICE float group_sum(float v) {
#pragma unroll
  for (int o = 1; o < WIDTH; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

YUF_DEVICE void cp_async_16(void* smem, const void* gmem) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
YUF_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
YUF_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

}  // namespace yuf

// Host-side error reporting shared by every C-ABI entry point.
namespace yuf {
void set_error(const char* fmt, ...);
yuf_status_t check_launch(const char* what);
// stream-ordered scratch for the raw ops (a per-device pool that keeps its pages)
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st);
void scratch_free(void* p, cudaStream_t st);
}  // namespace yuf

namespace yuf {
// Sum over aligned groups of G consecutive lanes (G need not be a power of 2).
template <int G>
YUF_DEVICE float lane_group_sum(float v, int lane) {
  if constexpr ((G & (G - 1)) == 0) {
#pragma unroll
    for (int o = 1; o < G; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  } else {
    const int base = lane - lane % G, gi = lane % G;
    float s = v;
#pragma unroll
    for (int o = 1; o < G; ++o) s += __shfl_sync(0xffffffffu, v, base + (gi + o) % G);
    return s;
  }
}
}  // namespace yuf

namespace yuf {
// Smallest lane stride >= C, a multiple of 4 floats (LDS.128), for which the G
// lanes' 16-byte windows at the same offset land on distinct banks.
constexpr int conflict_free_stride(int C, int G) {
  for (int cs = (C + 3) / 4 * 4;; cs += 4) {
    bool ok = true;
    for (int g1 = 0; g1 < G && ok; ++g1)
      for (int g2 = g1 + 1; g2 < G && ok; ++g2) {
        const int d = ((g2 - g1) * cs) % 32;
        ok = d >= 4 && d <= 28;
      }
    if (ok) return cs;
  }
}

}  // namespace yuf
