// Chunked WKV-7 prefill scan for sm_100a.
//
// Same math as wkv7.cu (yufmusicgen/model.py:145-165), reorganised so that the
// per-token cross-lane reduction chain of the sequential form disappears.
//
// Each state row s (row i of S, length N) evolves as
//   s_t = s_{t-1} * w_t + sa_t b_t + v_t k_t,   sa_t = s_{t-1} . a_t,   y_t = s_t . r_t
// For a chunk of L tokens starting from the true state s_0, let e_t be the plain
// per-column EMA  e_t = e_{t-1} * w_t + v_t k_t  (e_0 = s_0) and
// G_t = prod_{u<=t} w_u (cumulative retention, per column).  Then
//   s_t  = e_t + sum_{tau<=t} sa_tau (b_tau * G_t / G_tau)
//   sa_t = pa_t + sum_{tau<t} sa_tau M[tau][t],     pa_t = e_{t-1} . a_t
//   y_t  = pr_t + sum_{tau<=t} sa_tau Nn[tau][t],    pr_t = e_t . r_t
// with the per-HEAD matrices (shared by all N rows)
//   M[tau][t]  = (b_tau / G_tau) . (a_t G_{t-1})      (tau < t)
//   Nn[tau][t] = (b_tau / G_tau) . (r_t G_t)          (tau <= t)
// Row vectors: sa = pa X with X = (I - M)^{-1}, so
//   y   = pr + pa Q,           Q  = X Nn
//   s_L = e_L + pa F',         F' = X F,  F[tau] = b_tau G_L / G_tau.
// Per chunk the head-level work (retention, cumulative products, the L x L
// Gram matrices, X, Q, F') is done once by the whole CTA; the row-level work is
// an EMA with two dot products per token (no communication), ONE batched
// reduction of the 2L partial dots per row, and two small dense updates.  The
// retention bound w = exp(-0.6065 sigmoid(.)) >= 0.545 keeps 1/G_tau below
// 0.545^-16 ~ 1.6e4 for L = 16, well inside fp32.
//
// Layout: one CTA per (b, h).  A row is split over G lanes of one warp (lane g
// owns C consecutive columns; columns past N are zero padding), 32/G rows per
// warp.  For N = 40, G = 3: 4 warps of 10 rows, one warp per SM sub-partition.

#include "common.cuh"

namespace yuf {

constexpr int CK_L = 16;

template <int N>
struct ChunkCfg {
  static constexpr int G = (N == 40) ? 3 : (N == 16 ? 2 : 4);
  static constexpr int C0 = (N + G - 1) / G;
  static constexpr int C = (C0 + 1) / 2 * 2;   // columns per lane (even: float2 math)
  static constexpr int CS = conflict_free_stride(C, G);  // lane stride in shared memory
  static constexpr int VP = G * CS;            // padded vector length
  static constexpr int RPW = 32 / G;           // rows per warp
  static constexpr int NWARPS = (N + RPW - 1) / RPW;
  static constexpr int NT = 32 * NWARPS;
  // shared memory layout (floats)
  static constexpr int L = CK_L;
  static constexpr int RAW = 0;                       // [2][6][L][N]
  static constexpr int WP = RAW + 2 * 6 * L * N;      // [L][VP] retention
  static constexpr int KP = WP + L * VP;
  static constexpr int AP = KP + L * VP;
  static constexpr int RP = AP + L * VP;
  static constexpr int FP = RP + L * VP;              // F' = X F, padded
  static constexpr int AT = FP + L * VP;              // [L][N] a_t G_{t-1}
  static constexpr int RT = AT + L * N;               // r_t G_t
  static constexpr int BH = RT + L * N;               // b_t / G_t
  static constexpr int FR = BH + L * N;               // F (unpadded)
  static constexpr int MM = FR + L * N;               // [L][L] M[tau][t]
  static constexpr int NM = MM + L * L;               // Nn[tau][t]
  static constexpr int XM = NM + L * L;               // X[tau][t]
  static constexpr int QT = XM + L * L;               // Q^T: QT[t][sigma]
  static constexpr int YS = QT + L * L;               // [L][N] staged y
  static constexpr int TOTAL = YS + L * N;
  static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
};

// (tau, t) of the 120 strictly-upper M entries followed by the 136 Nn entries.
struct GramPairs {
  unsigned char tau[256], t[256];
  constexpr GramPairs() : tau(), t() {
    int e = 0;
    for (int tt = 0; tt < CK_L; ++tt)
      for (int ta = 0; ta < tt; ++ta) { tau[e] = (unsigned char)ta; t[e] = (unsigned char)tt; ++e; }
    for (int tt = 0; tt < CK_L; ++tt)
      for (int ta = 0; ta <= tt; ++ta) { tau[e] = (unsigned char)ta; t[e] = (unsigned char)tt; ++e; }
  }
};
__constant__ GramPairs c_gram = GramPairs();

template <int N>
__global__ void __launch_bounds__(ChunkCfg<N>::NT)
    wkv7_chunk_kernel(const float* __restrict__ r, const float* __restrict__ w,
                      const float* __restrict__ k, const float* __restrict__ v,
                      const float* __restrict__ a, const float* __restrict__ b, const float* s0,
                      float* __restrict__ y, float* s_out, int T, int H) {
  using K = ChunkCfg<N>;
  constexpr int L = K::L, G = K::G, C = K::C, C2 = C / 2, CS = K::CS, VP = K::VP;
  constexpr int NT = K::NT, RPW = K::RPW;

  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lrow = lane / G;
  const bool lane_ok = lrow < RPW;  // lanes past RPW*G idle (G = 3)
  const int row_raw = warp * RPW + (lane_ok ? lrow : 0);
  const bool row_ok = lane_ok && row_raw < N;
  const int row = row_ok ? row_raw : 0;
  const int g = lane_ok ? lane - lrow * G : 0;
  const int j0 = g * C;

  // Zero the padded vectors once: padding columns stay zero for the whole scan.
  for (int i = tid; i < 5 * L * VP; i += NT) sm[K::WP + i] = 0.f;

  // State row slice in registers (padding columns are zero).
  float2 e[C2];
  const size_t srow = (size_t)bh * N * N + (size_t)row * N;
#pragma unroll
  for (int c = 0; c < C2; ++c) {
    const int j = j0 + 2 * c;
    e[c] = (s0 != nullptr && row_ok && j < N) ? *reinterpret_cast<const float2*>(s0 + srow + j)
                                              : make_float2(0.f, 0.f);
  }

  const size_t tok_stride = (size_t)H * N;
  const size_t head_off = ((size_t)bb * T * H + hh) * N;
  const float* src[6] = {r + head_off, w + head_off, k + head_off,
                         v + head_off, a + head_off, b + head_off};
  auto stage = [&](int buf, int t0, int Tc) {
    constexpr int Q4 = N / 4;
    const int per_arr = Tc * Q4;
#pragma unroll
    for (int arr = 0; arr < 6; ++arr) {
      for (int idx = tid; idx < per_arr; idx += NT) {
        const int t = idx / Q4, q = idx - t * Q4;
        cp_async_16(sm + K::RAW + ((buf * 6 + arr) * L + t) * N + 4 * q,
                    src[arr] + (size_t)(t0 + t) * tok_stride + 4 * q);
      }
    }
    cp_async_commit();
  };
  auto pad = [](int j) { return (j / C) * CS + (j % C); };

  const int nchunks = (T + L - 1) / L;
  if (nchunks > 0) stage(0, 0, min(L, T));
  __syncthreads();  // zero-fill of the padded vectors is complete

  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    const int t0 = c * L;
    const int Tc = min(L, T - t0);
    if (c + 1 < nchunks) {
      stage(buf ^ 1, t0 + L, min(L, T - t0 - L));
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float* rawr = sm + K::RAW + (buf * 6 + 0) * L * N;
    float* raww = sm + K::RAW + (buf * 6 + 1) * L * N;
    float* rawk = sm + K::RAW + (buf * 6 + 2) * L * N;
    float* rawv = sm + K::RAW + (buf * 6 + 3) * L * N;
    float* rawa = sm + K::RAW + (buf * 6 + 4) * L * N;
    float* rawb = sm + K::RAW + (buf * 6 + 5) * L * N;

    // --- T1: retention and padded copies (parallel over (t, j)).  Tokens past
    // the end of T act as identity steps: w = 1, k = a = r = b = v = 0.
    for (int idx = tid; idx < L * N; idx += NT) {
      const int t = idx / N, j = idx - t * N;
      const int pj = t * VP + pad(j);
      if (t < Tc) {
        const float ret = __expf(W_SCALE * sigmoidf_fast(raww[idx]));
        raww[idx] = ret;  // raw w slot now holds the retention
        sm[K::WP + pj] = ret;
        sm[K::KP + pj] = rawk[idx];
        sm[K::AP + pj] = rawa[idx];
        sm[K::RP + pj] = rawr[idx];
      } else {
        raww[idx] = 1.f;
        rawv[idx] = 0.f;
        sm[K::WP + pj] = 1.f;
        sm[K::KP + pj] = 0.f;
        sm[K::AP + pj] = 0.f;
        sm[K::RP + pj] = 0.f;
      }
    }
    __syncthreads();
    // --- T2: cumulative retention per column (serial over the chunk).
    for (int j = tid; j < N; j += NT) {
      float gp = 1.f, gi = 1.f;
#pragma unroll
      for (int t = 0; t < L; ++t) {
        const int idx = t * N + j;
        const bool ok = t < Tc;
        const float ret = raww[idx];
        sm[K::AT + idx] = ok ? rawa[idx] * gp : 0.f;
        gp *= ret;
        gi = __fdividef(1.f, gp);
        sm[K::RT + idx] = ok ? rawr[idx] * gp : 0.f;
        sm[K::BH + idx] = ok ? rawb[idx] * gi : 0.f;
      }
#pragma unroll
      for (int t = 0; t < L; ++t) sm[K::FR + t * N + j] = sm[K::BH + t * N + j] * gp;
    }
    __syncthreads();
    // --- T3: Gram matrices M (tau < t) and Nn (tau <= t).
    for (int e2 = tid; e2 < 256; e2 += NT) {
      const int ta = c_gram.tau[e2], tt = c_gram.t[e2];
      const float4* bv = reinterpret_cast<const float4*>(sm + K::BH + ta * N);
      const float4* ov = reinterpret_cast<const float4*>(sm + (e2 < 120 ? K::AT : K::RT) + tt * N);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int q = 0; q < N / 4; ++q) {
        const float4 x = bv[q], z = ov[q];
        acc0 = fmaf(x.x, z.x, acc0);
        acc1 = fmaf(x.y, z.y, acc1);
        acc0 = fmaf(x.z, z.z, acc0);
        acc1 = fmaf(x.w, z.w, acc1);
      }
      sm[(e2 < 120 ? K::MM : K::NM) + ta * L + tt] = acc0 + acc1;
    }
    __syncthreads();
    // --- T4: X = (I - M)^{-1} (row-vector convention), one row per thread,
    // right-looking so the dependency chain is one FMA per step.
    if (tid < L) {
      const int ta = tid;
      float acc[L];
#pragma unroll
      for (int t = 0; t < L; ++t) acc[t] = 0.f;
#pragma unroll
      for (int s = 0; s < L; ++s) {
        if (s >= ta) {
          const float x = (s == ta) ? 1.f : acc[s];
          sm[K::XM + ta * L + s] = x;
#pragma unroll
          for (int t = s + 1; t < L; ++t) acc[t] = fmaf(x, sm[K::MM + s * L + t], acc[t]);
        } else {
          sm[K::XM + ta * L + s] = 0.f;
        }
      }
    }
    __syncthreads();
    // --- T5: Q = X Nn (stored transposed) and F' = X F (padded).
    for (int idx = tid; idx < L * L + L * N; idx += NT) {
      if (idx < L * L) {
        const int sg = idx / L, tt = idx - sg * L;
        float acc = 0.f;
        for (int ta = sg; ta <= tt; ++ta) acc = fmaf(sm[K::XM + sg * L + ta], sm[K::NM + ta * L + tt], acc);
        sm[K::QT + tt * L + sg] = (sg <= tt) ? acc : 0.f;
      } else {
        const int i2 = idx - L * L;
        const int sg = i2 / N, j = i2 - sg * N;
        float acc = 0.f;
        for (int ta = sg; ta < L; ++ta) acc = fmaf(sm[K::XM + sg * L + ta], sm[K::FR + ta * N + j], acc);
        sm[K::FP + sg * VP + pad(j)] = acc;
      }
    }
    __syncthreads();

    // --- R: row phase.  EMA with the two partial dots per token.
    float pa[L], pr[L];
    const float* Wl = sm + K::WP + g * CS;
    const float* Kl = sm + K::KP + g * CS;
    const float* Al = sm + K::AP + g * CS;
    const float* Rl = sm + K::RP + g * CS;
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const float vi = rawv[t * N + row];
      float2 da = make_float2(0.f, 0.f), dr = make_float2(0.f, 0.f);
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2) {
        const float2 av = *reinterpret_cast<const float2*>(Al + t * VP + 2 * c2);
        da = ffma2(e[c2], av, da);
      }
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2) {
        const float2 wv = *reinterpret_cast<const float2*>(Wl + t * VP + 2 * c2);
        const float2 kv = *reinterpret_cast<const float2*>(Kl + t * VP + 2 * c2);
        e[c2] = ffma2(e[c2], wv, fmul2(f2(vi), kv));
      }
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2) {
        const float2 rv = *reinterpret_cast<const float2*>(Rl + t * VP + 2 * c2);
        dr = ffma2(e[c2], rv, dr);
      }
      pa[t] = da.x + da.y;
      pr[t] = dr.x + dr.y;
    }
    // One batched all-reduce of the 2L partial dots over the row's lanes.
#pragma unroll
    for (int t = 0; t < L; ++t) {
      pa[t] = lane_group_sum<G>(pa[t], lane);
      pr[t] = lane_group_sum<G>(pr[t], lane);
    }
    // y_t = pr_t + sum_{sigma <= t} pa_sigma Q[sigma][t]
    float* ys = sm + K::YS;
#pragma unroll
    for (int t = 0; t < L; ++t) {
      float acc = pr[t];
      const float* qt = sm + K::QT + t * L;
#pragma unroll
      for (int s = 0; s <= t; ++s) acc = fmaf(pa[s], qt[s], acc);
      if (g == 0 && row_ok && t < Tc) ys[t * N + row] = acc;
    }
    // s_L = e_L + sum_sigma pa_sigma F'[sigma]
    const float* Fl = sm + K::FP + g * CS;
#pragma unroll
    for (int s = 0; s < L; ++s) {
      const float2 ps = f2(pa[s]);
#pragma unroll
      for (int c2 = 0; c2 < C2; ++c2)
        e[c2] = ffma2(ps, *reinterpret_cast<const float2*>(Fl + s * VP + 2 * c2), e[c2]);
    }
    __syncthreads();
    constexpr int Q4 = N / 4;
    for (int idx = tid; idx < Tc * Q4; idx += NT) {
      const int t = idx / Q4, q = idx - t * Q4;
      *reinterpret_cast<float4*>(y + head_off + (size_t)(t0 + t) * tok_stride + 4 * q) =
          *reinterpret_cast<const float4*>(ys + t * N + 4 * q);
    }
  }
  if (s_out != nullptr && row_ok) {
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c;
      if (j < N) *reinterpret_cast<float2*>(s_out + srow + j) = e[c];
    }
  }
}

template <int N>
static yuf_status_t launch_chunk(const float* r, const float* w, const float* k, const float* v,
                                 const float* a, const float* b, const float* s0, float* y,
                                 float* s_out, int B, int T, int H, cudaStream_t stream) {
  using K = ChunkCfg<N>;
  auto kern = wkv7_chunk_kernel<N>;
  if (K::BYTES > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::BYTES);
    if (e != cudaSuccess) {
      set_error("wkv7 chunk: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, K::NT, K::BYTES, stream>>>(r, w, k, v, a, b, s0, y, s_out, T, H);
  return check_launch("wkv7_chunk_kernel");
}

yuf_status_t wkv7_chunk_dispatch(const float* r, const float* w, const float* k, const float* v,
                                 const float* a, const float* b, const float* s0, float* y,
                                 float* s_out, int B, int T, int H, int N, cudaStream_t stream) {
  switch (N) {
#define CASE(NN) \
  case NN:       \
    return launch_chunk<NN>(r, w, k, v, a, b, s0, y, s_out, B, T, H, stream);
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
