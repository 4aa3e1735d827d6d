// Single-token WKV-7 step (batched decode) for sm_100a.
//
// Same math as wkv7.cu for T = 1 (yufmusicgen/model.py:145-165 with one token,
// the stateful path the reference decode takes, model.py:193).  A decode step
// is a pure stream over the state: every (sequence, head) reads its N x N state
// once, updates it with one rank-2 correction and writes it back, so the
// kernel is built for bytes in flight rather than latency: small CTAs with few
// registers so many stay resident per SM, one resident wave of them looping over
// the (b, h) heads with the next head's state already loading while the current
// one is updated, state rows read and written as coalesced float2 runs (the 4
// lanes of a row cover it contiguously, a warp covers 8 consecutive rows), and
// the five shared per-token vectors (retention computed once per column) staged
// in double-buffered shared memory.

#include <algorithm>

#include "common.cuh"

namespace yuf {

template <int N>
__global__ void __launch_bounds__(N * 4)
    wkv7_decode_kernel(const float* __restrict__ r, const float* __restrict__ w,
                       const float* __restrict__ k, const float* __restrict__ v,
                       const float* __restrict__ a, const float* __restrict__ b, const float* s0,
                       float* __restrict__ y, float* s_out, int BH) {
  constexpr int G = 4, C = N / G, C2 = C / 2;
  __shared__ float vec[2][5 * N];  // ret, k, a, b, r of the current and the next head
  const int tid = threadIdx.x;
  const int row = tid / G, g = tid - row * G, j0 = g * C;
  int bh = blockIdx.x;
  if (bh >= BH) return;

  float2 S[C2];
  float vi, pre[5];
  // issue the loads of head h's state row slice and token vectors (registers only)
  auto fetch = [&](int h, float2 (&S_)[C2], float& vi_, float (&p_)[5]) {
    const size_t o = (size_t)h * N;
    const size_t srow = (size_t)h * N * N + (size_t)row * N + j0;
#pragma unroll
    for (int c = 0; c < C2; ++c)
      S_[c] = s0 ? *reinterpret_cast<const float2*>(s0 + srow + 2 * c) : make_float2(0.f, 0.f);
    vi_ = v[o + row];
    if (tid < N) {
      p_[0] = w[o + tid];
      p_[1] = k[o + tid];
      p_[2] = a[o + tid];
      p_[3] = b[o + tid];
      p_[4] = r[o + tid];
    }
  };
  auto stage = [&](float* vs, const float (&p_)[5]) {
    if (tid < N) {
      vs[tid] = __expf(W_SCALE * sigmoidf_fast(p_[0]));
#pragma unroll
      for (int q = 1; q < 5; ++q) vs[q * N + tid] = p_[q];
    }
  };
  fetch(bh, S, vi, pre);
  stage(vec[0], pre);
  for (int it = 0;; ++it) {
    __syncthreads();  // vec[it & 1] staged; every thread is done with vec[(it + 1) & 1]
    const int nb = bh + gridDim.x;
    float2 Sn[C2];
    float vin = 0.f, pn[5];
    if (nb < BH) fetch(nb, Sn, vin, pn);  // next head's loads in flight during this one
    const float* vs = vec[it & 1];
    const float* W_ = vs + j0;
    const float* K_ = vs + N + j0;
    const float* A_ = vs + 2 * N + j0;
    const float* B_ = vs + 3 * N + j0;
    const float* R_ = vs + 4 * N + j0;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) acc = ffma2(S[c], *reinterpret_cast<const float2*>(A_ + 2 * c), acc);
    const float sa = group_sum<G>(acc.x + acc.y);
    float2 yacc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const float2 upd = ffma2(f2(sa), *reinterpret_cast<const float2*>(B_ + 2 * c),
                               fmul2(f2(vi), *reinterpret_cast<const float2*>(K_ + 2 * c)));
      S[c] = ffma2(S[c], *reinterpret_cast<const float2*>(W_ + 2 * c), upd);
      yacc = ffma2(S[c], *reinterpret_cast<const float2*>(R_ + 2 * c), yacc);
    }
    const float yv = group_sum<G>(yacc.x + yacc.y);
    const size_t o = (size_t)bh * N;
    if (g == 0) y[o + row] = yv;
    if (s_out) {
      const size_t srow = (size_t)bh * N * N + (size_t)row * N + j0;
#pragma unroll
      for (int c = 0; c < C2; ++c) *reinterpret_cast<float2*>(s_out + srow + 2 * c) = S[c];
    }
    if (nb >= BH) break;
    stage(vec[(it + 1) & 1], pn);
#pragma unroll
    for (int c = 0; c < C2; ++c) S[c] = Sn[c];
    vi = vin;
    bh = nb;
  }
}

// Resident CTAs per SM of the decode kernel for head size N (cached).
template <int N>
static int decode_blocks_per_sm() {
  static int n = [] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, wkv7_decode_kernel<N>, N * 4, 0) !=
            cudaSuccess ||
        v < 1)
      v = 1;
    return v;
  }();
  return n;
}

static int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// Grid: one resident wave of CTAs, each looping over heads bh, bh + grid, ...
// with the next head's loads issued before the current head's arithmetic.
yuf_status_t wkv7_decode_dispatch(const float* r, const float* w, const float* k, const float* v,
                                  const float* a, const float* b, const float* s0, float* y,
                                  float* s_out, int BH, int N, cudaStream_t stream) {
  if (BH <= 0) return YUF_OK;
  switch (N) {
#define CASE(NN)                                                                                 \
  case NN: {                                                                                     \
    const int grid = std::min(BH, decode_blocks_per_sm<NN>() * sm_count());                     \
    wkv7_decode_kernel<NN><<<grid, NN * 4, 0, stream>>>(r, w, k, v, a, b, s0, y, s_out, BH);    \
    return check_launch("wkv7_decode_kernel");                                                   \
  }
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
