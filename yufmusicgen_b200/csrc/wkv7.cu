// WKV-7 scan kernels for sm_100a (sequential form: prefill and decode).
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
// broadcast to the rows of the warp.  The 16-token loop is fully unrolled with
// y held in registers, so the loads of token t+1 overlap the math of token t.
//
// Head size 40 uses G = 3 (C = 14, two padding columns): 10 rows per warp, 4
// warps, one per SM sub-partition.
//
// The same kernel is the batched decode step (T = 1, state read from and
// written back to HBM) and, with COMPAT, the reference op's output contract
// (sa and transposed 16-token checkpoints).

#include "common.cuh"

namespace yuf {

constexpr int WKV_TS = 16;  // tokens per staged chunk (= the reference checkpoint interval)

template <int N>
struct SeqCfg {
  static constexpr int G = (N == 40) ? 3 : (N == 16 ? 2 : 4);
  static constexpr int C0 = (N + G - 1) / G;
  static constexpr int C = (C0 + 1) / 2 * 2;
  static constexpr int CS = conflict_free_stride(C, G);
  static constexpr int VP = G * CS;
  static constexpr int RPW = 32 / G;
  static constexpr int NWARPS = (N + RPW - 1) / RPW;
  static constexpr int NT = 32 * NWARPS;
  static constexpr int TS = WKV_TS;
  // shared memory (floats): raw[2][6][TS][N], then padded W,K,A,B,R [TS][VP]
  static constexpr int RAW = 0;
  static constexpr int PAD = RAW + 2 * 6 * TS * N;
  static constexpr int TOTAL = PAD + 5 * TS * VP;
  static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
};

template <int N, bool COMPAT>
__global__ void __launch_bounds__(SeqCfg<N>::NT, 1)
    wkv7_scan_kernel(const float* __restrict__ r, const float* __restrict__ w,
                     const float* __restrict__ k, const float* __restrict__ v,
                     const float* __restrict__ a, const float* __restrict__ b,
                     const float* s0, float* __restrict__ y, float* s_out,
                     float* __restrict__ ckpt, float* __restrict__ sa_out, int T, int H) {
  using K = SeqCfg<N>;
  constexpr int G = K::G, C = K::C, C2 = C / 2, CS = K::CS, VP = K::VP, NT = K::NT;
  constexpr int RPW = K::RPW, TS = K::TS;

  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lrow = lane / G;
  const bool lane_ok = lrow < RPW;
  const int row_raw = warp * RPW + (lane_ok ? lrow : 0);
  const bool row_ok = lane_ok && row_raw < N;
  const int row = row_ok ? row_raw : 0;
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
    S[c] = (s0 != nullptr && row_ok && j < N) ? *reinterpret_cast<const float2*>(s0 + srow + j)
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
    // retention once per element; tokens past T are identity steps
    for (int idx = tid; idx < Tc * N; idx += NT) {
      const int t = idx / N, j = idx - t * N;
      const int pj = K::PAD + t * VP + (j / C) * CS + (j % C);
      const bool ok = t < Tc;
      sm[pj + 0 * TS * VP] = ok ? __expf(W_SCALE * sigmoidf_fast(raw[1 * TS * N + idx])) : 1.f;
      sm[pj + 1 * TS * VP] = ok ? raw[2 * TS * N + idx] : 0.f;
      sm[pj + 2 * TS * VP] = ok ? raw[4 * TS * N + idx] : 0.f;
      sm[pj + 3 * TS * VP] = ok ? raw[5 * TS * N + idx] : 0.f;
      sm[pj + 4 * TS * VP] = ok ? raw[0 * TS * N + idx] : 0.f;
    }
    __syncthreads();

    // Register double buffer: the five vectors of token t+1 are loaded (as
    // float4) while token t is computed, so shared-memory latency overlaps math.
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
          qR[q] = *reinterpret_cast<const float4*>(Pr + o + 4 * q);
        }
        const float cv = rawv[t * N + row];
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
          if (c2 & 1) y1 = ffma2(S[c2], YUF_H2(qR, c2), y1); else y0 = ffma2(S[c2], YUF_H2(qR, c2), y0);
        }
        const float yv = lane_group_sum<G>((y0.x + y1.x) + (y0.y + y1.y), lane);
        if (g == 0 && row_ok) y[head_off + (size_t)(t0 + t) * tok_stride + row] = yv;
      if constexpr (COMPAT) {
        const int tt = t0 + t;
        {
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
    }
#undef YUF_H2
    __syncthreads();  // raw buffer `buf` and the padded vectors are reused next chunk
  }
  if (s_out != nullptr && row_ok) {
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c;
      if (j < N) *reinterpret_cast<float2*>(s_out + srow + j) = S[c];
    }
  }
}

template <int N, bool COMPAT>
static yuf_status_t launch_wkv7(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, const float* s0, float* y,
                                float* s_out, float* ckpt, float* sa, int B, int T, int H,
                                cudaStream_t stream) {
  using K = SeqCfg<N>;
  auto kern = wkv7_scan_kernel<N, COMPAT>;
  if (K::BYTES > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::BYTES);
    if (e != cudaSuccess) {
      set_error("wkv7: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, K::NT, K::BYTES, stream>>>(r, w, k, v, a, b, s0, y, s_out, ckpt, sa, T, H);
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
