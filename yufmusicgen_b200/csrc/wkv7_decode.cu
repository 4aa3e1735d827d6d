// Single-token WKV-7 step (batched decode) for sm_100a.
//
// Same math as wkv7.cu for T = 1 (yufmusicgen/model.py:145-165 with one token,
// the stateful path the reference decode takes, model.py:193).  A decode step
// is a pure stream over the state: every (sequence, head) reads its N x N state
// once, updates it with one rank-2 correction and writes it back, so the
// kernel is built for bytes in flight rather than latency: one small CTA per
// (b, h) with few registers so many CTAs stay resident per SM, state rows read
// and written as coalesced float2 runs (the 4 lanes of a row cover it
// contiguously, a warp covers 8 consecutive rows), and the five shared per-token
// vectors (retention computed once per column) staged in shared memory while
// the state loads are in flight.

#include "common.cuh"

namespace yuf {

template <int N>
__global__ void __launch_bounds__(N * 4)
    wkv7_decode_kernel(const float* __restrict__ r, const float* __restrict__ w,
                       const float* __restrict__ k, const float* __restrict__ v,
                       const float* __restrict__ a, const float* __restrict__ b, const float* s0,
                       float* __restrict__ y, float* s_out) {
  constexpr int G = 4, C = N / G, C2 = C / 2;
  __shared__ float vec[5 * N];  // ret, k, a, b, r
  const size_t bh = blockIdx.x;
  const size_t o = bh * N;  // [B, 1, H, N]: token row of (b, h)
  const int tid = threadIdx.x;
  const int row = tid / G, g = tid - row * G, j0 = g * C;
  const size_t srow = bh * N * N + (size_t)row * N + j0;

  float2 S[C2];
#pragma unroll
  for (int c = 0; c < C2; ++c)
    S[c] = s0 ? *reinterpret_cast<const float2*>(s0 + srow + 2 * c) : make_float2(0.f, 0.f);
  const float vi = v[o + row];
  if (tid < N) {
    vec[tid] = __expf(W_SCALE * sigmoidf_fast(w[o + tid]));
    vec[N + tid] = k[o + tid];
    vec[2 * N + tid] = a[o + tid];
    vec[3 * N + tid] = b[o + tid];
    vec[4 * N + tid] = r[o + tid];
  }
  __syncthreads();
  const float* W_ = vec + j0;
  const float* K_ = vec + N + j0;
  const float* A_ = vec + 2 * N + j0;
  const float* B_ = vec + 3 * N + j0;
  const float* R_ = vec + 4 * N + j0;
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
  if (g == 0) y[o + row] = yv;
  if (s_out) {
#pragma unroll
    for (int c = 0; c < C2; ++c) *reinterpret_cast<float2*>(s_out + srow + 2 * c) = S[c];
  }
}

yuf_status_t wkv7_decode_dispatch(const float* r, const float* w, const float* k, const float* v,
                                  const float* a, const float* b, const float* s0, float* y,
                                  float* s_out, int BH, int N, cudaStream_t stream) {
  switch (N) {
#define CASE(NN)                                                                             \
  case NN:                                                                                   \
    wkv7_decode_kernel<NN><<<BH, NN * 4, 0, stream>>>(r, w, k, v, a, b, s0, y, s_out);       \
    return check_launch("wkv7_decode_kernel");
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
