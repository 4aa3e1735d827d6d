// Time-parallel WKV-7 prefill for sm_100a.
//
// The sequential scan (wkv7.cu) gives one CTA to each (sequence, head) and walks
// all T tokens; with few sequences (the 0.1B prefill: B = 2, H = 16, 32 CTAs for
// 148 SMs) most of the GPU idles.  The recurrence is linear in the state,
//   S_t = S_{t-1} G_t + v_t k_t^T,   G_t = diag(w_t) + a_t b_t^T,
// so over a chunk of K tokens  S_end = S_start P + U  with the chunk's
// transition P = G_1 ... G_K and its own contribution U (the end state from a
// zero start).  Three passes:
//   1. every (sequence, chunk, head) computes U and P (wkv7.cu MODE 1: N rows
//      from zero with the value input, N identity rows without it);
//   2. per (sequence, head) the chunk start states S_c = S_{c-1} P_c + U_c
//      (wkv7_carry_kernel, an N x N x N product per chunk, P_c/U_c prefetched
//      with cp.async while the previous product runs);
//   3. every (sequence, chunk, head) rescans its tokens from S_{c-1} and writes y
//      (wkv7.cu MODE 0 over the chunks as batch entries).
// Tokens past the last whole chunk are scanned from the carried state by the
// sequential kernel.  Exact in exact arithmetic; the fp32 rounding differs from
// the sequential order only by the product association of pass 2.

#include "common.cuh"

namespace yuf {

constexpr int WKV_PAR_K = 128;  // tokens per chunk

yuf_status_t wkv7_dispatch_strided(const float* r, const float* w, const float* k, const float* v,
                                   const float* a, const float* b, const float* s0, float* y,
                                   float* s_out, float* ckpt, float* sa, int B, int T, int H, int N,
                                   bool compat, int Tstride, int Cper, cudaStream_t stream);
yuf_status_t wkv7_summary_dispatch(const float* w, const float* k, const float* v, const float* a,
                                   const float* b, float* U, float* P, int B, int T, int H, int N,
                                   int Tstride, int Cper, cudaStream_t stream);

// One CTA per (sequence, head); thread (ib, jb) owns a RB x 4 block of S.
template <int N, int RB>
__global__ void __launch_bounds__(N * N / (RB * 4))
    wkv7_carry_kernel(const float* __restrict__ U, const float* __restrict__ P, const float* s0,
                      float* __restrict__ S_start, float* s_out, int C, int H) {
  constexpr int NT = N * N / (RB * 4);
  constexpr int NN = N * N;
  extern __shared__ float4 carry_sm[];
  float* Ss = reinterpret_cast<float*>(carry_sm);   // [N][N] running state
  float* Pb0 = Ss + NN;                              // [2][N][N] transitions, double buffered
  const int bh = blockIdx.x;
  const int s = bh / H, h = bh - s * H;
  const int tid = threadIdx.x;
  const int ib = tid / (N / 4), jb = tid - ib * (N / 4);
  const int i0 = ib * RB, j0 = jb * 4;
  const float* s0p = s0 ? s0 + (size_t)bh * NN : nullptr;
  for (int q = tid; q < NN; q += NT) Ss[q] = s0p ? s0p[q] : 0.f;
  auto fetch = [&](int c, int buf) {
    const size_t off = (((size_t)s * C + c) * H + h) * NN;
    for (int q = tid; q < NN / 4; q += NT) cp_async_16(Pb0 + buf * NN + 4 * q, P + off + 4 * q);
    cp_async_commit();
  };
  if (C > 0) fetch(0, 0);
  for (int c = 0; c < C; ++c) {
    const int buf = c & 1;
    __syncthreads();  // Ss final for this chunk; buffer buf^1 free
    {
      float* dst = S_start + (((size_t)s * C + c) * H + h) * NN;
      for (int q = tid; q < NN / 4; q += NT)
        reinterpret_cast<float4*>(dst)[q] = reinterpret_cast<const float4*>(Ss)[q];
    }
    if (c + 1 < C) {
      fetch(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float acc[RB][4];
    const float* Uc = U + (((size_t)s * C + c) * H + h) * NN;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const float4 u = *reinterpret_cast<const float4*>(Uc + (i0 + r) * N + j0);
      acc[r][0] = u.x; acc[r][1] = u.y; acc[r][2] = u.z; acc[r][3] = u.w;
    }
    const float* Pc = Pb0 + buf * NN;
#pragma unroll 4
    for (int l = 0; l < N; ++l) {
      const float4 p = *reinterpret_cast<const float4*>(Pc + l * N + j0);
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const float sv = Ss[(i0 + r) * N + l];
        acc[r][0] = fmaf(sv, p.x, acc[r][0]);
        acc[r][1] = fmaf(sv, p.y, acc[r][1]);
        acc[r][2] = fmaf(sv, p.z, acc[r][2]);
        acc[r][3] = fmaf(sv, p.w, acc[r][3]);
      }
    }
    __syncthreads();  // every read of Ss done
#pragma unroll
    for (int r = 0; r < RB; ++r)
      *reinterpret_cast<float4*>(&Ss[(i0 + r) * N + j0]) =
          make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
  }
  __syncthreads();
  if (s_out)
    for (int q = tid; q < NN; q += NT) s_out[(size_t)bh * NN + q] = Ss[q];
}

template <int N>
static yuf_status_t launch_carry(const float* U, const float* P, const float* s0, float* S_start,
                                 float* s_out, int B, int C, int H, cudaStream_t st) {
  constexpr int RB = N >= 96 ? 4 : 2;
  const size_t bytes = 3 * (size_t)N * N * sizeof(float);
  auto kern = wkv7_carry_kernel<N, RB>;
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) {
      set_error("wkv7 carry: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, N * N / (RB * 4), bytes, st>>>(U, P, s0, S_start, s_out, C, H);
  return check_launch("wkv7_carry_kernel");
}

// The parallel path does about 3x the sequential work (the N transition rows of
// pass 1 and the rescan); it wins when the sequential scan would leave SMs idle,
// i.e. when there are fewer (sequence, head) chains than about 2/3 of the 148 SMs
// (measured: B*H = 32 -> 6x faster per layer, B*H = 128 -> 1.3x slower).
bool wkv7_parallel_applies(int B, int T, int H) {
  return T >= 2 * WKV_PAR_K && (long long)B * H <= 96;
}

size_t wkv7_parallel_scratch_floats(int B, int T, int H, int N) {
  const size_t C = (size_t)T / WKV_PAR_K;
  return 3 * (size_t)B * C * H * N * N + (size_t)B * H * N * N;
}

yuf_status_t wkv7_parallel(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           int B, int T, int H, int N, float* scratch, cudaStream_t st) {
  constexpr int K = WKV_PAR_K;
  const int C = T / K, Tm = C * K;
  const size_t per = (size_t)B * C * H * N * N;
  float* U = scratch;
  float* P = U + per;
  float* S_start = P + per;
  float* S_mid = S_start + per;  // state after the whole chunks when a tail follows
  const bool tail = Tm < T;
  yuf_status_t rc = wkv7_summary_dispatch(w, k, v, a, b, U, P, B * C, K, H, N, T, C, st);
  if (rc != YUF_OK) return rc;
  switch (N) {
#define CASE(NN) \
  case NN: rc = launch_carry<NN>(U, P, s0, S_start, tail ? S_mid : s_out, B, C, H, st); break;
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
  if (rc != YUF_OK) return rc;
  rc = wkv7_dispatch_strided(r, w, k, v, a, b, S_start, y, nullptr, nullptr, nullptr, B * C, K, H, N,
                             false, T, C, st);
  if (rc != YUF_OK || !tail) return rc;
  const size_t off = (size_t)Tm * H * N;
  return wkv7_dispatch_strided(r + off, w + off, k + off, v + off, a + off, b + off, S_mid, y + off,
                               s_out, nullptr, nullptr, B, T - Tm, H, N, false, T, 1, st);
}

}  // namespace yuf
