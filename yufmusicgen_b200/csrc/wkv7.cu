// WKV-7 scan kernels for sm_100a.
//
// Math (yufmusicgen/model.py:145-165; rwkv7_clampw.cu:20-75), per (batch b,
// head h), state S in R^{N x N} (row i = value dim, column j = key dim):
//   ret_j  = exp(-0.6065306597 * sigmoid(w_j))
//   sa_i   = sum_j a_j S_ij
//   S_ij  <- S_ij ret_j + sa_i b_j + v_i k_j
//   y_i    = sum_j S_ij r_j
//
// Every state ROW is an independent recurrence: row i only needs v_i and the
// per-token vectors (ret, k, a, b, r) that all rows share.  The kernel gives
// one CTA to one (b, h); each row is split over G = 4 lanes of a warp (lane g
// owns columns [g*C, g*C + C), C = N/4), so the per-row dot products are a
// two-step xor-shuffle reduction and the state lives in registers as packed
// fp32x2 pairs updated with FFMA2.  The shared per-token vectors are staged
// into shared memory 16 tokens at a time with cp.async, double buffered so
// the next chunk streams in from HBM while the current one is scanned; the
// retention exp/sigmoid is applied once per element there instead of once per
// row.  y is staged in shared memory and written back as float4 rows.
//
// The same kernel is the batched decode step (T = 1, state read from and
// written back to HBM) and, with COMPAT, the reference op's output contract
// (sa and transposed 16-token checkpoints).

#include "common.cuh"

namespace yuf {

constexpr int WKV_G = 4;    // lanes per state row
constexpr int WKV_TS = 16;  // tokens per staged chunk (= the reference checkpoint interval)

template <int N>
constexpr size_t wkv_smem_bytes() {
  return (size_t)(2 * 6 * WKV_TS * N + WKV_TS * N) * sizeof(float);
}

template <int N, bool COMPAT>
__global__ void __launch_bounds__(N* WKV_G)
    wkv7_scan_kernel(const float* __restrict__ r, const float* __restrict__ w,
                     const float* __restrict__ k, const float* __restrict__ v,
                     const float* __restrict__ a, const float* __restrict__ b,
                     const float* s0, float* __restrict__ y, float* s_out,
                     float* __restrict__ ckpt, float* __restrict__ sa_out, int T, int H) {
  constexpr int G = WKV_G;
  constexpr int C = N / G;
  constexpr int C2 = C / 2;
  constexpr int NT = N * G;
  constexpr int TS = WKV_TS;
  static_assert(N % 8 == 0, "head size must be a multiple of 8");

  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* ys = sm + 2 * 6 * TS * N;

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int tid = threadIdx.x;
  const int row = tid / G, g = tid - row * G;
  const int j0 = g * C;

  float2 S[C2];
  const size_t srow = (size_t)bh * N * N + (size_t)row * N + j0;
  if (s0 != nullptr) {
#pragma unroll
    for (int c = 0; c < C2; ++c) S[c] = *reinterpret_cast<const float2*>(s0 + srow + 2 * c);
  } else {
#pragma unroll
    for (int c = 0; c < C2; ++c) S[c] = make_float2(0.f, 0.f);
  }

  const size_t tok_stride = (size_t)H * N;
  const size_t head_off = ((size_t)bb * T * H + hh) * N;
  const float* src[6] = {r + head_off, w + head_off, k + head_off,
                         v + head_off, a + head_off, b + head_off};

  auto stage = [&](int buf, int t0, int Tc) {
    constexpr int Q = N / 4;  // float4 per token vector
    const int per_arr = Tc * Q;
#pragma unroll
    for (int arr = 0; arr < 6; ++arr) {
      for (int idx = tid; idx < per_arr; idx += NT) {
        const int t = idx / Q, q = idx - t * Q;
        cp_async_16(sm + ((buf * 6 + arr) * TS + t) * N + 4 * q,
                    src[arr] + (size_t)(t0 + t) * tok_stride + 4 * q);
      }
    }
    cp_async_commit();
  };

  const int nchunks = (T + TS - 1) / TS;
  const int n_ckpt = T / TS;
  if (nchunks > 0) stage(0, 0, min(TS, T));
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    const int t0 = c * TS;
    const int Tc = min(TS, T - t0);
    if (c + 1 < nchunks) {
      stage(buf ^ 1, t0 + TS, min(TS, T - t0 - TS));
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float* wb = sm + (buf * 6 + 1) * TS * N;
    for (int idx = tid; idx < Tc * N; idx += NT) wb[idx] = __expf(W_SCALE * sigmoidf_fast(wb[idx]));
    __syncthreads();

    const float* R_ = sm + (buf * 6 + 0) * TS * N + j0;
    const float* W_ = sm + (buf * 6 + 1) * TS * N + j0;
    const float* K_ = sm + (buf * 6 + 2) * TS * N + j0;
    const float* V_ = sm + (buf * 6 + 3) * TS * N;
    const float* A_ = sm + (buf * 6 + 4) * TS * N + j0;
    const float* B_ = sm + (buf * 6 + 5) * TS * N + j0;
#pragma unroll 2
    for (int t = 0; t < Tc; ++t) {
      const int o = t * N;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2)
        acc = ffma2(S[c2], *reinterpret_cast<const float2*>(A_ + o + 2 * c2), acc);
      const float sa = group_sum<G>(acc.x + acc.y);
      const float vi = V_[o + row];
      float2 yacc = make_float2(0.f, 0.f);
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2) {
        const float2 kk = *reinterpret_cast<const float2*>(K_ + o + 2 * c2);
        const float2 bv = *reinterpret_cast<const float2*>(B_ + o + 2 * c2);
        const float2 wv = *reinterpret_cast<const float2*>(W_ + o + 2 * c2);
        const float2 rv = *reinterpret_cast<const float2*>(R_ + o + 2 * c2);
        const float2 upd = ffma2(f2(sa), bv, fmul2(f2(vi), kk));
        S[c2] = ffma2(S[c2], wv, upd);
        yacc = ffma2(S[c2], rv, yacc);
      }
      const float yv = group_sum<G>(yacc.x + yacc.y);
      if (g == 0) ys[o + row] = yv;
      if constexpr (COMPAT) {
        const int tt = t0 + t;
        if (g == 0) sa_out[((size_t)bb * T + tt) * tok_stride + (size_t)hh * N + row] = sa;
        if (((tt + 1) % TS) == 0) {
          float* cp = ckpt + ((size_t)bh * n_ckpt + tt / TS) * N * N + row;
#pragma unroll
          for (int c2 = 0; c2 < C2; ++c2) {
            cp[(size_t)(j0 + 2 * c2) * N] = S[c2].x;
            cp[(size_t)(j0 + 2 * c2 + 1) * N] = S[c2].y;
          }
        }
      }
    }
    __syncthreads();
    constexpr int Q = N / 4;
    for (int idx = tid; idx < Tc * Q; idx += NT) {
      const int t = idx / Q, q = idx - t * Q;
      *reinterpret_cast<float4*>(y + head_off + (size_t)(t0 + t) * tok_stride + 4 * q) =
          *reinterpret_cast<const float4*>(ys + t * N + 4 * q);
    }
  }
  if (s_out != nullptr) {
#pragma unroll
    for (int c = 0; c < C2; ++c) *reinterpret_cast<float2*>(s_out + srow + 2 * c) = S[c];
  }
}

template <int N, bool COMPAT>
static yuf_status_t launch_wkv7(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, const float* s0, float* y,
                                float* s_out, float* ckpt, float* sa, int B, int T, int H,
                                cudaStream_t stream) {
  constexpr size_t smem = wkv_smem_bytes<N>();
  auto kern = wkv7_scan_kernel<N, COMPAT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("wkv7: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, N * WKV_G, smem, stream>>>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, T, H);
  return check_launch("wkv7_scan_kernel");
}

#define YUF_WKV_SIZES(X) X(16) X(32) X(40) X(48) X(64) X(96) X(128)

yuf_status_t wkv7_dispatch(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           float* ckpt, float* sa, int B, int T, int H, int N, bool compat,
                           cudaStream_t stream) {
  switch (N) {
#define CASE(NN)                                                                              \
  case NN:                                                                                    \
    return compat ? launch_wkv7<NN, true>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, B, T, H,  \
                                          stream)                                             \
                  : launch_wkv7<NN, false>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, B, T, H, \
                                           stream);
    YUF_WKV_SIZES(CASE)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
