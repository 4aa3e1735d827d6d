// WKV-7 scan kernels for sm_100a (sequential form).
//
// Math (yufmusicgen/model.py:145-165; rwkv7_clampw.cu:20-75), per (batch b,
// head h), state S in R^{N x N} (row i = value dim, column j = key dim):
//   ret_j  = exp(-0.6065306597 * sigmoid(w_j))
//   sa_i   = sum_j a_j S_ij
//   S_ij  <- S_ij ret_j + sa_i b_j + v_i k_j
//   y_i    = sum_j S_ij r_j
//
// Every state ROW is an independent recurrence: row i only needs v_i and the
// per-token vectors (ret, k, a, b, r) that all rows share.  One CTA owns one
// (b, h); each row is split over G lanes of a warp (lane g owns C consecutive
// columns, C even, columns past N are zero padding), 32/G rows per warp, and the
// state lives in registers as fp32x2 pairs updated with FFMA2.  The row's two
// dot products per token are a G-lane shuffle reduction.
//
// Shared per-token vectors are staged 16 tokens at a time: cp.async brings the
// raw rows from HBM (double buffered, the next chunk streams in while the
// current one is scanned), then one pass applies exp/sigmoid once per element
// and writes each vector into a padded layout whose lane stride CS keeps the G
// lanes of a row on distinct banks, so every read is a conflict-free LDS.128
// broadcast to the rows of the warp.
//
// Head size 40 uses G = 3 (C = 14, two padding columns): 10 rows per warp, 4
// warps, one per SM sub-partition.
//
// MODE 0 is the scan (prefill; with COMPAT also the reference op's sa and
// transposed 16-token checkpoints).  MODE 1 summarises a chunk of tokens for the
// time-parallel scan (wkv7_parallel.cu): it runs 2N rows -- rows 0..N-1 from a
// zero state with the value input (their end state is the chunk's own
// contribution U), rows N..2N-1 from the identity without value input (their end
// state is the chunk's transition P, S_end = S_start P + U) -- and writes U and P
// instead of y.  `Tstride` is the token count between consecutive sequences and
// `Cper` the number of T-token chunks per sequence (Tstride = T, Cper = 1 for a
// plain [B, T, H, N] tensor), so the chunks of every sequence can be processed as
// their own batch entries.

#include "common.cuh"

namespace yuf {

constexpr int WKV_TS = 16;  // tokens per staged chunk (= the reference checkpoint interval)

template <int N, int ROWS>
struct SeqCfg {
  static constexpr int G = (N == 40) ? 3 : (N == 16 ? 2 : 4);
  static constexpr int C0 = (N + G - 1) / G;
  static constexpr int C = (C0 + 1) / 2 * 2;
  static constexpr int CS = conflict_free_stride(C, G);
  static constexpr int VP = G * CS;
  static constexpr int RPW = 32 / G;
  static constexpr int NWARPS = (ROWS + RPW - 1) / RPW;
  static constexpr int NT = 32 * NWARPS;
  static constexpr int TS = WKV_TS;
  // shared memory (floats): raw[2][6][TS][N], then padded W,K,A,B,R [TS][VP]
  static constexpr int RAW = 0;
  static constexpr int PAD = RAW + 2 * 6 * TS * N;
  static constexpr int TOTAL = PAD + 5 * TS * VP;
  static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
};

template <int N, int MODE, bool COMPAT>
__global__ void __launch_bounds__(SeqCfg<N, (MODE == 1 ? 2 * N : N)>::NT, 1)
    wkv7_scan_kernel(const float* __restrict__ r, const float* __restrict__ w,
                     const float* __restrict__ k, const float* __restrict__ v,
                     const float* __restrict__ a, const float* __restrict__ b,
                     const float* s0, float* __restrict__ y, float* s_out,
                     float* __restrict__ ckpt, float* __restrict__ sa_out, int T, int H,
                     int Tstride, int Cper, float* __restrict__ U_out, float* __restrict__ P_out) {
  constexpr int ROWS = MODE == 1 ? 2 * N : N;
  using K = SeqCfg<N, ROWS>;
  constexpr int G = K::G, C = K::C, C2 = C / 2, CS = K::CS, VP = K::VP, NT = K::NT;
  constexpr int RPW = K::RPW, TS = K::TS;

  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lrow = lane / G;
  const bool lane_ok = lrow < RPW;
  const int vrow_raw = warp * RPW + (lane_ok ? lrow : 0);  // 0..ROWS-1
  const bool row_ok = lane_ok && vrow_raw < ROWS;
  const int vrow = row_ok ? vrow_raw : 0;
  const bool ident = MODE == 1 && vrow >= N;  // transition rows: identity start, no value input
  const int row = ident ? vrow - N : vrow;    // state row 0..N-1
  const int g = lane_ok ? lane - lrow * G : 0;
  const int j0 = g * C;

  // padding columns of the padded vectors stay zero for the whole scan
  const int t_used = min(TS, T);  // padded token rows ever read
  for (int i = tid; i < 5 * TS * VP; i += NT)
    if ((i / VP) % TS < t_used) sm[K::PAD + i] = 0.f;

  float2 S[C2];
  const size_t srow = (size_t)bh * N * N + (size_t)row * N;
#pragma unroll
  for (int c = 0; c < C2; ++c) {
    const int j = j0 + 2 * c;
    if (MODE == 1) {
      S[c] = make_float2(ident && j == row ? 1.f : 0.f, ident && j + 1 == row ? 1.f : 0.f);
    } else {
      S[c] = (s0 != nullptr && row_ok && j < N) ? *reinterpret_cast<const float2*>(s0 + srow + j)
                                                : make_float2(0.f, 0.f);
    }
  }

  const size_t tok_stride = (size_t)H * N;
  // batch entry bb covers tokens [c*T, c*T + T) of sequence s, bb = s*Cper + c
  const size_t head_off =
      (((size_t)(bb / Cper) * Tstride + (size_t)(bb % Cper) * T) * H + hh) * N;
  const float* src[6] = {r + head_off, w + head_off, k + head_off,
                         v + head_off, a + head_off, b + head_off};
  auto stage = [&](int buf, int t0, int Tc) {
    constexpr int Q4 = N / 4;
    const int per_arr = Tc * Q4;
#pragma unroll
    for (int arr = 0; arr < 6; ++arr) {
      if (MODE == 1 && arr == 0) continue;  // no y, no r
      for (int idx = tid; idx < per_arr; idx += NT) {
        const int t = idx / Q4, q = idx - t * Q4;
        cp_async_16(sm + K::RAW + ((buf * 6 + arr) * TS + t) * N + 4 * q,
                    src[arr] + (size_t)(t0 + t) * tok_stride + 4 * q);
      }
    }
    cp_async_commit();
  };

  const int nchunks = (T + TS - 1) / TS;
  const int n_ckpt = T / TS;
  if (nchunks > 0) stage(0, 0, min(TS, T));
  __syncthreads();

  // padded vectors: 0 = ret, 1 = k, 2 = a, 3 = b, 4 = r
  const float* Pw = sm + K::PAD + 0 * TS * VP + g * CS;
  const float* Pk = sm + K::PAD + 1 * TS * VP + g * CS;
  const float* Pa = sm + K::PAD + 2 * TS * VP + g * CS;
  const float* Pb = sm + K::PAD + 3 * TS * VP + g * CS;
  const float* Pr = sm + K::PAD + 4 * TS * VP + g * CS;

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
    const float* raw = sm + K::RAW + buf * 6 * TS * N;
    const float* rawv = raw + 3 * TS * N;
    // retention once per element
    for (int idx = tid; idx < Tc * N; idx += NT) {
      const int t = idx / N, j = idx - t * N;
      const int pj = K::PAD + t * VP + (j / C) * CS + (j % C);
      sm[pj + 0 * TS * VP] = __expf(W_SCALE * sigmoidf_fast(raw[1 * TS * N + idx]));
      sm[pj + 1 * TS * VP] = raw[2 * TS * N + idx];
      sm[pj + 2 * TS * VP] = raw[4 * TS * N + idx];
      sm[pj + 3 * TS * VP] = raw[5 * TS * N + idx];
      if (MODE == 0) sm[pj + 4 * TS * VP] = raw[0 * TS * N + idx];
    }
    __syncthreads();

    // The fully unrolled loop lets the compiler issue token t+1's loads during
    // token t's math; operands are read as float4 (CQ per vector and lane).
    constexpr int CQ = (C + 3) / 4;
#define YUF_H2(arr, c2) ((c2 & 1) ? make_float2(arr[c2 >> 1].z, arr[c2 >> 1].w) \
                                  : make_float2(arr[c2 >> 1].x, arr[c2 >> 1].y))
#pragma unroll
    for (int t = 0; t < TS; ++t) {
      if (t < Tc) {  // uniform across the CTA: short chunks (decode) skip the rest
        const int o = t * VP;
        float4 qA[CQ], qK[CQ], qB[CQ], qW[CQ], qR[CQ];
#pragma unroll
        for (int q = 0; q < CQ; ++q) {
          qA[q] = *reinterpret_cast<const float4*>(Pa + o + 4 * q);
          qK[q] = *reinterpret_cast<const float4*>(Pk + o + 4 * q);
          qB[q] = *reinterpret_cast<const float4*>(Pb + o + 4 * q);
          qW[q] = *reinterpret_cast<const float4*>(Pw + o + 4 * q);
          if (MODE == 0) qR[q] = *reinterpret_cast<const float4*>(Pr + o + 4 * q);
        }
        const float cv = ident ? 0.f : rawv[t * N + row];
        float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c2 = 0; c2 < C2; ++c2) {
          if (c2 & 1) a1 = ffma2(S[c2], YUF_H2(qA, c2), a1); else a0 = ffma2(S[c2], YUF_H2(qA, c2), a0);
        }
        const float sa = lane_group_sum<G>((a0.x + a1.x) + (a0.y + a1.y), lane);
        float2 y0 = make_float2(0.f, 0.f), y1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c2 = 0; c2 < C2; ++c2) {
          S[c2] = ffma2(S[c2], YUF_H2(qW, c2), ffma2(f2(sa), YUF_H2(qB, c2), fmul2(f2(cv), YUF_H2(qK, c2))));
          if (MODE == 0) {
            if (c2 & 1) y1 = ffma2(S[c2], YUF_H2(qR, c2), y1); else y0 = ffma2(S[c2], YUF_H2(qR, c2), y0);
          }
        }
        if (MODE == 0) {
          const float yv = lane_group_sum<G>((y0.x + y1.x) + (y0.y + y1.y), lane);
          if (g == 0 && row_ok) y[head_off + (size_t)(t0 + t) * tok_stride + row] = yv;
        }
        if constexpr (COMPAT) {
          const int tt = t0 + t;
          if (g == 0 && row_ok) sa_out[((size_t)bb * T + tt) * tok_stride + (size_t)hh * N + row] = sa;
          if (((tt + 1) % TS) == 0 && row_ok) {
            float* cp = ckpt + ((size_t)bh * n_ckpt + tt / TS) * N * N + row;
#pragma unroll
            for (int c2 = 0; c2 < C2; ++c2) {
              const int j = j0 + 2 * c2;
              if (j < N) {
                cp[(size_t)j * N] = S[c2].x;
                cp[(size_t)(j + 1) * N] = S[c2].y;
              }
            }
          }
        }
      }
    }
#undef YUF_H2
    __syncthreads();  // raw buffer `buf` and the padded vectors are reused next chunk
  }
  float* dst = MODE == 1 ? (ident ? P_out : U_out) : s_out;
  if (dst != nullptr && row_ok) {
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c;
      if (j < N) *reinterpret_cast<float2*>(dst + srow + j) = S[c];
    }
  }
}

template <int N, int MODE, bool COMPAT>
static yuf_status_t launch_wkv7(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, const float* s0, float* y,
                                float* s_out, float* ckpt, float* sa, int B, int T, int H,
                                int Tstride, int Cper, float* U, float* P, cudaStream_t stream) {
  using K = SeqCfg<N, (MODE == 1 ? 2 * N : N)>;
  auto kern = wkv7_scan_kernel<N, MODE, COMPAT>;
  if (K::BYTES > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::BYTES);
    if (e != cudaSuccess) {
      set_error("wkv7: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, K::NT, K::BYTES, stream>>>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, T, H, Tstride,
                                           Cper, U, P);
  return check_launch("wkv7_scan_kernel");
}

#define YUF_WKV_SIZES(X) X(16) X(32) X(40) X(48) X(64) X(96) X(128)

yuf_status_t wkv7_dispatch_strided(const float* r, const float* w, const float* k, const float* v,
                                   const float* a, const float* b, const float* s0, float* y,
                                   float* s_out, float* ckpt, float* sa, int B, int T, int H, int N,
                                   bool compat, int Tstride, int Cper, cudaStream_t stream) {
  switch (N) {
#define CASE(NN)                                                                              \
  case NN:                                                                                    \
    return compat ? launch_wkv7<NN, 0, true>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, B, T, H, \
                                             Tstride, Cper, nullptr, nullptr, stream)         \
                  : launch_wkv7<NN, 0, false>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, B, T, H, \
                                              Tstride, Cper, nullptr, nullptr, stream);
    YUF_WKV_SIZES(CASE)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

yuf_status_t wkv7_dispatch(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           float* ckpt, float* sa, int B, int T, int H, int N, bool compat,
                           cudaStream_t stream) {
  return wkv7_dispatch_strided(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, B, T, H, N, compat, T, 1,
                               stream);
}

// Chunk summaries (MODE 1): U, P [B, H, N, N] of T tokens per batch entry.
yuf_status_t wkv7_summary_dispatch(const float* w, const float* k, const float* v, const float* a,
                                   const float* b, float* U, float* P, int B, int T, int H, int N,
                                   int Tstride, int Cper, cudaStream_t stream) {
  switch (N) {
#define CASE(NN)                                                                                    \
  case NN:                                                                                          \
    return launch_wkv7<NN, 1, false>(w, w, k, v, a, b, nullptr, nullptr, nullptr, nullptr, nullptr, \
                                     B, T, H, Tstride, Cper, U, P, stream);
    YUF_WKV_SIZES(CASE)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
