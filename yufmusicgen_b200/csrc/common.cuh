// Shared helpers for the sm_100a kernels of the WKV-7 + ROSA hot path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

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

// ---- programmatic dependent launch (PDL) ----------------------------------
// The engine's decode step is a chain of ~15 small kernels per layer whose cost
// is dominated by the gap between one kernel's end and the next one's start.
// Launched with programmatic stream serialization, a kernel may be scheduled
// while its predecessor still runs: it first waits for the predecessor grid to
// complete with all its memory visible (pdl_wait, before touching global memory
// the predecessor could write or read), then lets its own successor launch
// (pdl_trigger), so at most two kernels of the chain are resident and the
// successor's launch and set-up overlap this kernel's work.  Both are no-ops
// for a kernel launched the ordinary way.
namespace yuf {
YUF_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
YUF_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// the calling host thread's launches use PDL while a PdlScope(true) is alive
bool pdl_enabled();
struct PdlScope {
  explicit PdlScope(bool on);
  ~PdlScope();
  bool prev;
};
// kernel<<<grid, block, smem, s>>>(args...), with programmatic stream
// serialization when pdl_enabled(); errors surface through check_launch.
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace yuf

// The time-mix epilogue's per-channel parameters of one layer ([H * N] each),
// for the WKV kernels that fold it in: w = w0 + lw, kk = normalize(k * k_k),
// alpha = sigmoid(a0 + la), a = -kk, b = kk * alpha, k' = k * (1 + (alpha - 1) * k_a).
namespace yuf {
struct WkvTm {
  const float *w0, *a0, *k_k, *k_a;
};
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

namespace yuf {
// Tensor-core fp32 products with near-fp32 accuracy ("3xTF32"): each operand x
// is split into hi = x with its 13 low mantissa bits cleared (a tf32 value) and
// lo = x - hi (exact in fp32; the tensor core reads its top 19 bits), and
// a*b = ah*bh + ah*bl + al*bh, with al*bl (~2^-20 relative) dropped.  The split
// is one logic op and one subtraction, no conversion instruction.
YUF_DEVICE void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}
YUF_DEVICE void split4(const float4 x, uint4& hi, uint4& lo) {
  split_tf32(x.x, hi.x, lo.x);
  split_tf32(x.y, hi.y, lo.y);
  split_tf32(x.z, hi.z, lo.z);
  split_tf32(x.w, hi.w, lo.w);
}
// D += A B for one m16n8k8 tile (A row-major 16x8, B 8x8 given by columns).
YUF_DEVICE void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// Fragment values (lane = 4g + q): a = {A[g][q], A[g+8][q], A[g][q+4], A[g+8][q+4]},
// b = {B[q][g], B[q+4][g]}, d = {D[g][2q], D[g][2q+1], D[g+8][2q], D[g+8][2q+1]}.
// The three products go to three accumulators (main, and the two cross terms)
// so that consecutive k-steps form three short dependency chains; the caller
// sums them once at the end (small terms first).
struct Acc3 {
  float d[4], e1[4], e2[4];
};
YUF_DEVICE void acc3_init(Acc3& x, float v0, float v1, float v2, float v3) {
  x.d[0] = v0; x.d[1] = v1; x.d[2] = v2; x.d[3] = v3;
#pragma unroll
  for (int i = 0; i < 4; ++i) x.e1[i] = x.e2[i] = 0.f;
}
YUF_DEVICE void mma_3xtf32(Acc3& x, const float (&a)[4], const float (&b)[2]) {
  uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], ah[i], al[i]);
#pragma unroll
  for (int i = 0; i < 2; ++i) split_tf32(b[i], bh[i], bl[i]);
  mma_tf32(x.e1, al, bh);
  mma_tf32(x.e2, ah, bl);
  mma_tf32(x.d, ah, bh);
}
YUF_DEVICE float acc3_get(const Acc3& x, int i) { return x.d[i] + (x.e1[i] + x.e2[i]); }
YUF_DEVICE void acc_init(Acc3& x, float v0, float v1, float v2, float v3) { acc3_init(x, v0, v1, v2, v3); }
YUF_DEVICE void acc_init(float (&x)[4], float v0, float v1, float v2, float v3) {
  x[0] = v0; x[1] = v1; x[2] = v2; x[3] = v3;
}
YUF_DEVICE float acc_get(const Acc3& x, int i) { return acc3_get(x, i); }
YUF_DEVICE float acc_get(const float (&x)[4], int i) { return x[i]; }
// The same products into one accumulator (for register-tight callers).
YUF_DEVICE void mma_3xtf32(float (&d)[4], const float (&a)[4], const float (&b)[2]) {
  uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], ah[i], al[i]);
#pragma unroll
  for (int i = 0; i < 2; ++i) split_tf32(b[i], bh[i], bl[i]);
  mma_tf32(d, al, bh);
  mma_tf32(d, ah, bl);
  mma_tf32(d, ah, bh);
}

// Sum each of V per-thread values over the block; every thread receives all V
// sums in out[] (shared).  scratch holds nwarps * V floats.
template <int V>
YUF_DEVICE void block_sum_array(const float (&x)[V], float* scratch, float* out, int nwarps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    float s = x[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) scratch[warp * V + i] = s;
  }
  __syncthreads();
  if (threadIdx.x < V) {
    float s = 0.f;
    for (int wi = 0; wi < nwarps; ++wi) s += scratch[wi * V + threadIdx.x];
    out[threadIdx.x] = s;
  }
  __syncthreads();
}

}  // namespace yuf
