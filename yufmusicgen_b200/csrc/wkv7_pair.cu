// Single-pass chunk summary and output correction for the time-parallel
// WKV-7 prefill (wkv7_parallel.cu).
//
// For a chunk of tokens with start state S_0:
//   S_t = S_0 P_t + U_t,   P_t = G_1 ... G_t,   U_t = scan from a zero state,
//   y_t = S_t r_t = (U_t r_t) + S_0 (P_t r_t) = yU_t + S_0 q_t.
// The pair kernels run, for every state row i, the zero-start row (U) and the
// identity-start row (P, no value input) in the SAME lane, so every per-token
// vector loaded from shared memory serves both rows, and write
//   yU_t (into y), q_t = P_t r_t (row t of Q, [K, N] per chunk and head,
//   token-major like y), U = U_end and P = P_end.
// After the carry (S_0 of every chunk), wkv7_correct_kernel adds S_0 q_t to y:
// a [len x N] x [N x N] product per (chunk, head) instead of a second scan.
//
// Work item bb = s * Cper + c is chunk c of sequence s: tokens
// [c*K, min(c*K + K, Tstride)) -- the last chunk of a sequence may be shorter.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "mbarrier.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace yuf {

// ---- TMA staging of the pair kernel ---------------------------------------
// Each input [B*T, H*N] fp32 tensor is described by a 2-D tensor map (box = N
// columns x 8 rows: one head's 8 tokens); one thread issues the six loads of an
// 8-token group onto an mbarrier with the expected byte count, every thread
// waits on the barrier's phase.  Waits are bounded: after WAIT_NS nanoseconds
// (global timer) a thread counts a timeout in g_pair_wait_timeouts and leaves
// the kernel.
struct PairTmaps {
  CUtensorMap m[6];  // r, w, k, v, a, b
};

__device__ unsigned int g_pair_wait_timeouts;

YUF_DEVICE size_t item_head_off(int bb, int hh, int K, int H, int N, int Tstride, int Cper) {
  return (((size_t)(bb / Cper) * Tstride + (size_t)(bb % Cper) * K) * H + hh) * N;
}
YUF_DEVICE int item_len(int bb, int K, int Tstride, int Cper) {
  return min(K, Tstride - (bb % Cper) * K);
}

constexpr int PAIR_TS = 16;

// Multi-warp form for N >= 48: G lanes per state row; RP row pairs per lane
// (each loaded column value then feeds 2*RP rows).
template <int N>
struct PairCfg {
  static constexpr int G = (N == 16) ? 2 : 4;
  static constexpr int C0 = (N + G - 1) / G;
  static constexpr int C = (C0 + 1) / 2 * 2;
  static constexpr int RP = C <= 12 ? 2 : 1;
  static constexpr int CS = conflict_free_stride(C, G);
  static constexpr int VP = G * CS;
  static constexpr int RPW = 32 / G;  // row groups per warp (RP pairs each)
  static constexpr int NWARPS = (N + RPW * RP - 1) / (RPW * RP);
  static constexpr int NT = 32 * NWARPS;
  static constexpr int TS = PAIR_TS;
  static constexpr int RAW = 0;
  static constexpr int PAD = RAW + 2 * 6 * TS * N;
  static constexpr int TOTAL = PAD + 5 * TS * VP;
  static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
};

template <int N>
__global__ void __launch_bounds__(PairCfg<N>::NT, 1)
    wkv7_pair_kernel(const float* __restrict__ r, const float* __restrict__ w,
                     const float* __restrict__ k, const float* __restrict__ v,
                     const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                     float* __restrict__ Q, float* __restrict__ U_out, float* __restrict__ P_out,
                     int K_, int H, int Tstride, int Cper) {
  using K = PairCfg<N>;
  constexpr int G = K::G, C = K::C, C2 = C / 2, CS = K::CS, VP = K::VP, NT = K::NT;
  constexpr int RPW = K::RPW, TS = K::TS, RP = K::RP;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int T = item_len(bb, K_, Tstride, Cper);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lrow = lane / G;
  const bool lane_ok = lrow < RPW;
  const int rgrp = warp * RPW + (lane_ok ? lrow : 0);
  const int g = lane_ok ? lane - lrow * G : 0;
  const int j0 = g * C;
  int row[RP];
  bool row_ok[RP];
#pragma unroll
  for (int p = 0; p < RP; ++p) {
    const int rr = rgrp * RP + p;
    row_ok[p] = lane_ok && rr < N;
    row[p] = row_ok[p] ? rr : 0;
  }

  const int t_used = min(TS, T);
  for (int i = tid; i < 5 * TS * VP; i += NT)
    if ((i / VP) % TS < t_used) sm[K::PAD + i] = 0.f;

  float2 SU[RP][C2], SP[RP][C2];
#pragma unroll
  for (int p = 0; p < RP; ++p)
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c;
      SU[p][c] = make_float2(0.f, 0.f);
      SP[p][c] = make_float2(j == row[p] ? 1.f : 0.f, j + 1 == row[p] ? 1.f : 0.f);
    }

  const size_t tok_stride = (size_t)H * N;
  const size_t head_off = item_head_off(bb, hh, K_, H, N, Tstride, Cper);
  float* Qh = Q + (size_t)bh * K_ * N;  // Q[bb][hh][t][row]
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
  if (nchunks > 0) stage(0, 0, min(TS, T));
  __syncthreads();
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
    for (int idx = tid; idx < Tc * N; idx += NT) {
      const int t = idx / N, j = idx - t * N;
      const int pj = K::PAD + t * VP + (j / C) * CS + (j % C);
      sm[pj + 0 * TS * VP] = __expf(W_SCALE * sigmoidf_fast(raw[1 * TS * N + idx]));
      sm[pj + 1 * TS * VP] = raw[2 * TS * N + idx];
      sm[pj + 2 * TS * VP] = raw[4 * TS * N + idx];
      sm[pj + 3 * TS * VP] = raw[5 * TS * N + idx];
      sm[pj + 4 * TS * VP] = raw[0 * TS * N + idx];
    }
    __syncthreads();
    constexpr int CQ = (C + 3) / 4;
#define YUF_H2(arr, c2) ((c2 & 1) ? make_float2(arr[c2 >> 1].z, arr[c2 >> 1].w) \
                                  : make_float2(arr[c2 >> 1].x, arr[c2 >> 1].y))
#pragma unroll
    for (int t = 0; t < TS; ++t) {
      if (t < Tc) {
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
#pragma unroll
        for (int p = 0; p < RP; ++p) {
          const float cv = rawv[t * N + row[p]];
          float2 u0 = make_float2(0.f, 0.f), u1 = u0, p0 = u0, p1 = u0;
#pragma unroll
          for (int c2 = 0; c2 < C2; ++c2) {
            const float2 av = YUF_H2(qA, c2);
            if (c2 & 1) { u1 = ffma2(SU[p][c2], av, u1); p1 = ffma2(SP[p][c2], av, p1); }
            else        { u0 = ffma2(SU[p][c2], av, u0); p0 = ffma2(SP[p][c2], av, p0); }
          }
          const float saU = lane_group_sum<G>((u0.x + u1.x) + (u0.y + u1.y), lane);
          const float saP = lane_group_sum<G>((p0.x + p1.x) + (p0.y + p1.y), lane);
          float2 yu0 = make_float2(0.f, 0.f), yu1 = yu0, yp0 = yu0, yp1 = yu0;
#pragma unroll
          for (int c2 = 0; c2 < C2; ++c2) {
            const float2 wv = YUF_H2(qW, c2), bv = YUF_H2(qB, c2), rv = YUF_H2(qR, c2);
            SU[p][c2] = ffma2(SU[p][c2], wv, ffma2(f2(saU), bv, fmul2(f2(cv), YUF_H2(qK, c2))));
            SP[p][c2] = ffma2(SP[p][c2], wv, fmul2(f2(saP), bv));
            if (c2 & 1) { yu1 = ffma2(SU[p][c2], rv, yu1); yp1 = ffma2(SP[p][c2], rv, yp1); }
            else        { yu0 = ffma2(SU[p][c2], rv, yu0); yp0 = ffma2(SP[p][c2], rv, yp0); }
          }
          const float yU = lane_group_sum<G>((yu0.x + yu1.x) + (yu0.y + yu1.y), lane);
          const float qv = lane_group_sum<G>((yp0.x + yp1.x) + (yp0.y + yp1.y), lane);
          if (g == 0 && row_ok[p]) {
            y[head_off + (size_t)(t0 + t) * tok_stride + row[p]] = yU;
            Qh[(size_t)(t0 + t) * N + row[p]] = qv;
          }
        }
      }
    }
#undef YUF_H2
    __syncthreads();
  }
#pragma unroll
  for (int p = 0; p < RP; ++p) {
    if (!row_ok[p]) continue;
    const size_t srow = (size_t)bh * N * N + (size_t)row[p] * N;
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c;
      if (j < N) {
        *reinterpret_cast<float2*>(U_out + srow + j) = SU[p][c];
        *reinterpret_cast<float2*>(P_out + srow + j) = SP[p][c];
      }
    }
  }
}

// One block per (chunk, head) for N <= 64: NW warps (1 for N <= 40, 2 for 48
// and 64), each of 8 row groups of 4 lanes.  Lane (rg, g) of warp wp,
// rg = lane / 4, g = lane % 4, owns the R state rows i0 .. i0+R-1,
// i0 = (8 wp + rg) R (R = 5 at N = 40, 4 at N = 64) -- each as a zero-start row
// and an identity-start row -- over the C = N / 4 columns g*C .. g*C+C-1.  Every per-token column value a lane reads from shared
// memory then feeds 2R rows, so the kernel is bound by the FMA pipe rather than
// by shared-memory delivery (the multi-warp kernel above feeds 4 rows per read).
//
// Decay-scaled state.  Inside a group of TS tokens the lanes carry
// S'_t = S_t / gamma_t (column-wise, gamma_t = w_1 ... w_t since the group
// started), for which the update loses its decay product:
//   S'_t = S'_{t-1} + sa_t (b_t / gamma_t)^T + v_t (k_t / gamma_t)^T,
//   sa_t = S'_{t-1} (gamma_{t-1} a_t),   y_t = S'_t (gamma_t r_t)
// -- two FMAs per zero-start element and one per identity-start element
// instead of three and two.  The scaled vectors are made once per token and
// column when the group is staged; at the group end S = S' gamma_end, so
// gamma stays >= 0.545^TS (no underflow, 1/gamma <= 128 for TS = 8).
//
// Per token: the two row dot products with a (all-reduced over the 4 lanes of a
// row group), the update, and the two dot products with r, reduce-scattered so
// that each lane finishes a few of the 2N outputs and stores them directly (a
// warp's stores of one token cover one contiguous row of y and of Q).
// Staging per group: cp.async brings the raw rows, one pass (a lane per column
// pair, sequential over the group's tokens) makes the scaled vectors in the
// lane layout, then the next group's copy starts while this group is scanned;
// single buffers keep the block small (15 KB at N = 40, 12 warps per SM).
#ifndef YUF_PAIRW_UNROLL
#define YUF_PAIRW_UNROLL 8
#endif
constexpr int PAIRW_UNROLL = YUF_PAIRW_UNROLL;  // token loop unroll: code size vs. scheduling

template <int N>
struct PairWCfg {
  static constexpr int G = 4;                                   // lanes per row group
  static constexpr int R = N == 48 ? 3 : (N == 64 ? 4 : N / 8);  // rows per lane
  static constexpr int NW = N / (8 * R);                        // warps (8 row groups each)
  static constexpr int NT = 32 * NW;
  static constexpr int C = N / G;                               // columns per lane
  static constexpr int C2 = C / 2;
  static constexpr int CS = conflict_free_stride(C, G);
  static constexpr int VP = G * CS;
  static constexpr int TS = 8;                    // tokens per staged group
  static constexpr int RAW = 0;                   // [6][TS][N] raw rows r, w, k, v, a, b
  static constexpr int PAD = RAW + 6 * TS * N;    // [4][TS][VP] scaled a, b, k, r in lane layout
  static constexpr int GEND = PAD + 4 * TS * VP;  // [VP] gamma at the group end
  static constexpr int VV = GEND + VP;            // [TS][N] values
  static constexpr int PRM = VV + TS * N;         // [4][N] the head's w0, a0, k_k, k_a (time-mix folded in)
  static constexpr int NRM = PRM + 4 * N;         // [TS] 1 / |k k_k| per token (time-mix folded in)
  static constexpr int MBAR = (NRM + TS + 1) / 2 * 2;  // one 8-byte mbarrier
  static constexpr int TOTAL = MBAR + 2;
  static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
  static constexpr uint32_t TX_BYTES = 6u * TS * N * sizeof(float);  // six full boxes per group
  static constexpr uint32_t TX_BYTES_TM = 5u * TS * N * sizeof(float);  // time-mix folded in: no b box
  static_assert(N % 8 == 0 && C % 2 == 0 && N <= 64 && NW * 8 * R == N,
                "warp pair kernel: N in {16, 32, 40, 48, 64}");
  static_assert((TS * N * sizeof(float)) % 128 == 0, "TMA boxes land on 128-byte boundaries");
};

// Barrier over the block's warps (a warp barrier when the block is one warp).
template <int NW>
YUF_DEVICE void block_sync() {
  if constexpr (NW == 1) __syncwarp();
  else __syncthreads();
}

// true on every thread when `p` holds on any thread of the block
template <int NW>
YUF_DEVICE bool block_any(bool p) {
  if constexpr (NW == 1) return __any_sync(0xffffffffu, p);
  else return __syncthreads_or(p) != 0;
}

// C floats of one padded vector as float2 pairs (C/4 LDS.128 and one LDS.64).
template <int C>
YUF_DEVICE void load_cols(float2 (&dst)[C / 2], const float* p) {
#pragma unroll
  for (int q = 0; q < C / 4; ++q) {
    const float4 x = *reinterpret_cast<const float4*>(p + 4 * q);
    dst[2 * q] = make_float2(x.x, x.y);
    dst[2 * q + 1] = make_float2(x.z, x.w);
  }
  if constexpr (C % 4 != 0) dst[C / 2 - 1] = *reinterpret_cast<const float2*>(p + C - 2);
}

#ifndef YUF_PAIRW_MINB
#define YUF_PAIRW_MINB 1  // minimum resident blocks per SM the register budget is set for
#endif
// TM: the time-mix epilogue folded in (WkvTm): the boxes are r, the w and a
// low-rank outputs, k and v as the projections left them, and the scaled
// vectors are formed from them (timemix_post_kernel's arithmetic) with the
// head's 1 / |k k_k| per token from a first pass over the group.
template <int N, bool TM = false>
__global__ void __launch_bounds__(PairWCfg<N>::NT, YUF_PAIRW_MINB)
    wkv7_pairw_kernel(const float* __restrict__ r, const float* __restrict__ w,
                      const float* __restrict__ k, const float* __restrict__ v,
                      const float* __restrict__ a, const float* __restrict__ b,
                      float* __restrict__ y, float* __restrict__ Q, float* __restrict__ U_out,
                      float* __restrict__ P_out, int K_, int H, int Tstride, int Cper,
                      const __grid_constant__ PairTmaps tm, const WkvTm prm) {
  using K = PairWCfg<N>;
  constexpr int R = K::R, C = K::C, C2 = K::C2, CS = K::CS, VP = K::VP, TS = K::TS;
  constexpr int RH = (R + 1) / 2;  // outputs kept by the even lane of a pair after reduce-scatter
  extern __shared__ __align__(128) float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + K::MBAR);

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int T = item_len(bb, K_, Tstride, Cper);
  constexpr int NT = K::NT;
  const int tid = threadIdx.x;
  const int lane = K::NW == 1 ? tid : (tid & 31), wp = K::NW == 1 ? 0 : tid >> 5;
  const int rg = lane >> 2, g = lane & 3;
  const int i0 = (wp * 8 + rg) * R, j0 = g * C;

  float2 SU[R][C2], SP[R][C2];
#pragma unroll
  for (int p = 0; p < R; ++p)
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const int j = j0 + 2 * c, i = i0 + p;
      SU[p][c] = make_float2(0.f, 0.f);
      SP[p][c] = make_float2(j == i ? 1.f : 0.f, j + 1 == i ? 1.f : 0.f);
    }

  const size_t tok_stride = (size_t)H * N;
  const size_t head_off = item_head_off(bb, hh, K_, H, N, Tstride, Cper);
  float* Qh = Q + (size_t)bh * K_ * N;  // Q[bb][hh][t][row]
  // TMA coordinates of this item's first token: column hh*N, row s*Tstride + c*K
  const int tx = hh * N;
  const int ty = (bb / Cper) * Tstride + (bb % Cper) * K_;
  auto stage = [&](int t0) {  // one thread: the six (TM: five) 8-token boxes of a group
    mbar_expect_tx(bar, TM ? K::TX_BYTES_TM : K::TX_BYTES);
#pragma unroll
    for (int arr = 0; arr < (TM ? 5 : 6); ++arr)
      tma_load_2d(sm + K::RAW + arr * TS * N, &tm.m[arr], bar, tx, ty + t0);
  };

  const int ngroups = (T + TS - 1) / TS;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if constexpr (TM) {  // the head's parameters (weights: no kernel of the chain writes them)
    for (int i = tid; i < 4 * N; i += NT) {
      const int which = i / N, jj = i - which * N;
      const float* src = which == 0 ? prm.w0 : (which == 1 ? prm.a0 : (which == 2 ? prm.k_k : prm.k_a));
      sm[K::PRM + i] = src[hh * N + jj];
    }
  }
  block_sync<K::NW>();
  if (tid == 0 && ngroups > 0) stage(0);
  const float* Pa = sm + K::PAD + 0 * TS * VP + g * CS;
  const float* Pb = sm + K::PAD + 1 * TS * VP + g * CS;
  const float* Pk = sm + K::PAD + 2 * TS * VP + g * CS;
  const float* Pr = sm + K::PAD + 3 * TS * VP + g * CS;
  const float* Pg = sm + K::GEND + g * CS;
  const float* vv = sm + K::VV;
  const int h = (lane >> 1) & 1, e = lane & 1;  // reduce-scatter roles inside the row group
  const int rbase = i0 + (e ? RH : 0);
  const int nk = e ? R - RH : RH;
  float* obase = h ? Qh + rbase : y + head_off + rbase;
  const size_t ostride = h ? (size_t)N : tok_stride;

  for (int gi = 0; gi < ngroups; ++gi) {
    const int t0 = gi * TS;
    const int Tc = min(TS, T - t0);
    // A group that never landed: the block votes, counts one timeout, lets the
    // staging copy still in flight into its shared memory land (bounded) and
    // leaves together; the outputs of the launch are void.
    if (block_any<K::NW>(!mbar_wait(bar, gi & 1))) {
      if (tid == 0) {
        atomicAdd(&g_pair_wait_timeouts, 1u);
        mbar_wait(bar, gi & 1);
      }
      return;
    }
    if constexpr (TM) {  // 1 / |k k_k| of each token: warp 0, four lanes a token
      if (wp == 0) {
        const int t = lane >> 2, q4 = lane & 3;
        float ss = 0.f;
        if (t < Tc) {
          for (int jj = q4 * (N / 4); jj < (q4 + 1) * (N / 4); ++jj) {
            const float kk = sm[K::RAW + 2 * TS * N + t * N + jj] * sm[K::PRM + 2 * N + jj];
            ss = fmaf(kk, kk, ss);
          }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if (q4 == 0) sm[K::NRM + t] = 1.f / fmaxf(sqrtf(ss), 1e-12f);  // F.normalize eps (model.py:116)
      }
      block_sync<K::NW>();
    }
    // scaled vectors: a thread per column pair, running gamma over the group's tokens
    if (tid < N / 2) {
      const int j = 2 * tid;
      const int pj = (j / C) * CS + (j % C);  // lane-layout offset of the pair
      float2 gam = make_float2(1.f, 1.f), ginv = gam;
      float2 pw0, pa0, pkk, pka;
      if constexpr (TM) {
        pw0 = *reinterpret_cast<const float2*>(sm + K::PRM + j);
        pa0 = *reinterpret_cast<const float2*>(sm + K::PRM + N + j);
        pkk = *reinterpret_cast<const float2*>(sm + K::PRM + 2 * N + j);
        pka = *reinterpret_cast<const float2*>(sm + K::PRM + 3 * N + j);
      }
      for (int t = 0; t < Tc; ++t) {
        const int rj = t * N + j;
        float2 wr = *reinterpret_cast<const float2*>(sm + K::RAW + 1 * TS * N + rj);
        if constexpr (TM) wr = make_float2(pw0.x + wr.x, pw0.y + wr.y);
        const float sx = W_SCALE * sigmoidf_fast(wr.x), sy = W_SCALE * sigmoidf_fast(wr.y);
        float2 av, bv, kv;
        if constexpr (TM) {
          const float2 kr = *reinterpret_cast<const float2*>(sm + K::RAW + 2 * TS * N + rj);
          const float2 la = *reinterpret_cast<const float2*>(sm + K::RAW + 4 * TS * N + rj);
          const float inv = sm[K::NRM + t];
          const float kkx = kr.x * pkk.x * inv, kky = kr.y * pkk.y * inv;
          const float alx = sigmoidf_fast(pa0.x + la.x), aly = sigmoidf_fast(pa0.y + la.y);
          av = make_float2(-kkx, -kky);
          bv = make_float2(kkx * alx, kky * aly);
          kv = make_float2(kr.x * (1.f + (alx - 1.f) * pka.x), kr.y * (1.f + (aly - 1.f) * pka.y));
        } else {
          av = *reinterpret_cast<const float2*>(sm + K::RAW + 4 * TS * N + rj);
          bv = *reinterpret_cast<const float2*>(sm + K::RAW + 5 * TS * N + rj);
          kv = *reinterpret_cast<const float2*>(sm + K::RAW + 2 * TS * N + rj);
        }
        const float2 rv = *reinterpret_cast<const float2*>(sm + K::RAW + 0 * TS * N + rj);
        float* d = sm + K::PAD + t * VP + pj;
        *reinterpret_cast<float2*>(d + 0 * TS * VP) = fmul2(av, gam);  // gamma_{t-1} a_t
        gam = fmul2(gam, make_float2(__expf(sx), __expf(sy)));
        ginv = fmul2(ginv, make_float2(__expf(-sx), __expf(-sy)));
        *reinterpret_cast<float2*>(d + 1 * TS * VP) = fmul2(bv, ginv);  // b_t / gamma_t
        *reinterpret_cast<float2*>(d + 2 * TS * VP) = fmul2(kv, ginv);  // k_t / gamma_t
        *reinterpret_cast<float2*>(d + 3 * TS * VP) = fmul2(rv, gam);   // gamma_t r_t
        *reinterpret_cast<float2*>(sm + K::VV + rj) =
            *reinterpret_cast<const float2*>(sm + K::RAW + 3 * TS * N + rj);
      }
      *reinterpret_cast<float2*>(sm + K::GEND + pj) = gam;
    }
    block_sync<K::NW>();
    if (tid == 0 && gi + 1 < ngroups) {  // raw boxes are free again (all reads done)
      fence_proxy_async();
      stage(t0 + TS);
    }

    // sa of the group's first token; every later token's sa comes out of the
    // previous token's pass over the state together with that token's outputs
    float sU[R], sP[R];
    {
      float2 av[C2];
      load_cols<C>(av, Pa);
#pragma unroll
      for (int p = 0; p < R; ++p) {
        float2 u = make_float2(0.f, 0.f), q = u;
#pragma unroll
        for (int c = 0; c < C2; ++c) {
          u = ffma2(SU[p][c], av[c], u);
          q = ffma2(SP[p][c], av[c], q);
        }
        sU[p] = u.x + u.y;
        sP[p] = q.x + q.y;
      }
#pragma unroll
      for (int p = 0; p < R; ++p) {
        sU[p] += __shfl_xor_sync(0xffffffffu, sU[p], 1);
        sP[p] += __shfl_xor_sync(0xffffffffu, sP[p], 1);
      }
#pragma unroll
      for (int p = 0; p < R; ++p) {
        sU[p] += __shfl_xor_sync(0xffffffffu, sU[p], 2);
        sP[p] += __shfl_xor_sync(0xffffffffu, sP[p], 2);
      }
    }
#pragma unroll PAIRW_UNROLL
    for (int t = 0; t < TS; ++t) {
      if (t < Tc) {
        const int o = t * VP;
        {
          float2 bv[C2], kv[C2];
          load_cols<C>(bv, Pb + o);
          load_cols<C>(kv, Pk + o);
          float vr[R];
#pragma unroll
          for (int p = 0; p < R; ++p) vr[p] = vv[t * N + i0 + p];
#pragma unroll
          for (int p = 0; p < R; ++p)
#pragma unroll
            for (int c = 0; c < C2; ++c) {
              SU[p][c] = ffma2(f2(sU[p]), bv[c], ffma2(f2(vr[p]), kv[c], SU[p][c]));
              SP[p][c] = ffma2(f2(sP[p]), bv[c], SP[p][c]);
            }
        }
        // one pass over the updated state: outputs of token t and sa of token
        // t + 1 (for the group's last token the a row read is not a token's and
        // its sa is dropped)
        float2 rv[C2], av[C2];
        load_cols<C>(rv, Pr + o);
        load_cols<C>(av, Pa + o + VP);
        float yo[2 * R];  // [0, R): zero-start outputs, [R, 2R): q
#pragma unroll
        for (int p = 0; p < R; ++p) {
          float2 u = make_float2(0.f, 0.f), q = u, ua = u, qa = u;
#pragma unroll
          for (int c = 0; c < C2; ++c) {
            u = ffma2(SU[p][c], rv[c], u);
            q = ffma2(SP[p][c], rv[c], q);
            ua = ffma2(SU[p][c], av[c], ua);
            qa = ffma2(SP[p][c], av[c], qa);
          }
          yo[p] = u.x + u.y;
          yo[R + p] = q.x + q.y;
          sU[p] = ua.x + ua.y;
          sP[p] = qa.x + qa.y;
        }
        // reduce-scatter of the outputs over the row group (lanes with h = 0 keep
        // the zero-start outputs, h = 1 the q values; then e = 0 keeps rows
        // [0, RH), e = 1 the rest), interleaved with the all-reduce of sa
        float kept[R];
#pragma unroll
        for (int p = 0; p < R; ++p) {
          const float send = h ? yo[p] : yo[R + p];
          kept[p] = (h ? yo[R + p] : yo[p]) + __shfl_xor_sync(0xffffffffu, send, 2);
          sU[p] += __shfl_xor_sync(0xffffffffu, sU[p], 1);
          sP[p] += __shfl_xor_sync(0xffffffffu, sP[p], 1);
        }
        float* orow = obase + (size_t)(t0 + t) * ostride;
#pragma unroll
        for (int p = 0; p < RH; ++p) {
          const float hi = (RH + p < R) ? kept[RH + p] : 0.f;
          const float send = e ? kept[p] : hi;
          const float fin = (e ? hi : kept[p]) + __shfl_xor_sync(0xffffffffu, send, 1);
          if (p < nk) orow[p] = fin;
        }
#pragma unroll
        for (int p = 0; p < R; ++p) {
          sU[p] += __shfl_xor_sync(0xffffffffu, sU[p], 2);
          sP[p] += __shfl_xor_sync(0xffffffffu, sP[p], 2);
        }
      }
    }
    // back to the unscaled state: S = S' gamma_end
    {
      float2 ge[C2];
      load_cols<C>(ge, Pg);
#pragma unroll
      for (int p = 0; p < R; ++p)
#pragma unroll
        for (int c = 0; c < C2; ++c) {
          SU[p][c] = fmul2(SU[p][c], ge[c]);
          SP[p][c] = fmul2(SP[p][c], ge[c]);
        }
    }
    block_sync<K::NW>();  // the next group's staging pass overwrites the lane layout
  }
#pragma unroll
  for (int p = 0; p < R; ++p) {
    const size_t srow = (size_t)bh * N * N + (size_t)(i0 + p) * N;
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      *reinterpret_cast<float2*>(U_out + srow + j0 + 2 * c) = SU[p][c];
      *reinterpret_cast<float2*>(P_out + srow + j0 + 2 * c) = SP[p][c];
    }
  }
}

// y[t][i] += sum_j S0[i][j] q_t[j] over one (chunk, head): a [len x N] x
// [N x N]^T product on the tensor cores (mma.sync m16n8k8, 3xTF32 for near-fp32
// accuracy).  cp.async stages the chunk's Q (rows padded to N + 4 floats, which
// makes the A-fragment loads bank-conflict free; rows past len zero-filled up
// to the 16-row tile); S0 is split once into its tf32 high and low parts in
// shared memory.  Each warp takes 16-token row tiles across all N/8 column
// tiles, so an A fragment is loaded and split once per k-step for N/8 products;
// the accumulators start from y (loaded before the staging completes).  A block
// covers TW = 80 tokens of a chunk (one tile per warp), so a chunk spreads over
// several blocks and each block waits on memory once.
template <int N>
struct CorrCfg {
  static constexpr int NP = N + 4;
  static constexpr int WARPS = 5;
  static constexpr int NT = 32 * WARPS;
  static constexpr int TW = 16 * WARPS;  // tokens per block: one 16-token tile per warp
};

template <int N>
__global__ void __launch_bounds__(256)
    wkv7_correct_kernel(const float* __restrict__ S0, const float* __restrict__ Q,
                        float* __restrict__ y, int K_, int H, int Tstride, int Cper, int skip_first,
                        int parts) {
  constexpr int NP = CorrCfg<N>::NP, NT = CorrCfg<N>::NT, WARPS = CorrCfg<N>::WARPS, Q4 = N / 4;
  constexpr int NTL = N / 8, TW = CorrCfg<N>::TW;
  extern __shared__ float4 corr_sm[];
  uint32_t* Sh = reinterpret_cast<uint32_t*>(corr_sm);  // [N][NP] tf32 high parts of S0
  uint32_t* Sl = Sh + N * NP;                            // [N][NP] low parts
  float* Qs = reinterpret_cast<float*>(Sl + N * NP);     // [TW][NP]
  const int bh = blockIdx.x / parts, part = blockIdx.x - bh * parts;
  const int bb = bh / H, hh = bh - bb * H;
  if (skip_first && bb % Cper == 0) return;  // chunk 0 starts from the zero state
  const int tb = part * TW;                  // first token of this block in the chunk
  const int T = min(TW, item_len(bb, K_, Tstride, Cper) - tb);
  if (T <= 0) return;
  const int T16 = (T + 15) / 16 * 16;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const float* S0h = S0 + (size_t)bh * N * N;
  const float* Qg = Q + ((size_t)bh * K_ + tb) * N;
  for (int x = tid; x < T * Q4; x += NT) {
    const int t = x / Q4, c = x - t * Q4;
    cp_async_16(Qs + t * NP + 4 * c, Qg + t * N + 4 * c);
  }
  for (int x = tid; x < N * Q4; x += NT) {  // S0 rows, split in place below
    const int i = x / Q4, c = x - i * Q4;
    cp_async_16(Sh + i * NP + 4 * c, S0h + i * N + 4 * c);
  }
  cp_async_commit();
  for (int x = T * NP + tid; x < T16 * NP; x += NT) Qs[x] = 0.f;
  const size_t tok_stride = (size_t)H * N;
  const size_t head_off = item_head_off(bb, hh, K_, H, N, Tstride, Cper) + (size_t)tb * tok_stride;
  const int mtiles = T16 / 16;
  float2 yv[NTL][2];
  auto load_y = [&](int mt) {
    const int t_lo = mt * 16 + g, t_hi = t_lo + 8;
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) {
      const int col = nt * 8 + 2 * q;
      yv[nt][0] = yv[nt][1] = make_float2(0.f, 0.f);
      if (t_lo < T) yv[nt][0] = *reinterpret_cast<const float2*>(y + head_off + (size_t)t_lo * tok_stride + col);
      if (t_hi < T) yv[nt][1] = *reinterpret_cast<const float2*>(y + head_off + (size_t)t_hi * tok_stride + col);
    }
  };
  if (warp < mtiles) load_y(warp);  // in flight while the staging completes
  cp_async_wait<0>();
  __syncthreads();
  for (int x = tid; x < N * N; x += NT) {
    const int o = (x / N) * NP + x % N;
    uint32_t hi, lo;
    split_tf32(__uint_as_float(Sh[o]), hi, lo);
    Sh[o] = hi;
    Sl[o] = lo;
  }
  __syncthreads();
  for (int mt = warp; mt < mtiles; mt += WARPS) {
    if (mt != warp) load_y(mt);
    const int t_lo = mt * 16 + g, t_hi = t_lo + 8;
    // an opaque zero keeps the S fragment loads inside the loop (hoisting all
    // of them would take N*N/8 registers per thread and cut the occupancy)
    int z;
    asm volatile("mov.u32 %0, 0;" : "=r"(z));
    const uint32_t* ShI = Sh + z;
    const uint32_t* SlI = Sl + z;
    float acc[NTL][4];
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) {
      acc[nt][0] = yv[nt][0].x; acc[nt][1] = yv[nt][0].y;
      acc[nt][2] = yv[nt][1].x; acc[nt][3] = yv[nt][1].y;
    }
#pragma unroll
    for (int k0 = 0; k0 < N; k0 += 8) {
      const float a[4] = {Qs[t_lo * NP + k0 + q], Qs[t_hi * NP + k0 + q],
                          Qs[t_lo * NP + k0 + q + 4], Qs[t_hi * NP + k0 + q + 4]};
      uint32_t ah[4], al[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) split_tf32(a[r], ah[r], al[r]);
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt) {
        const int srow = (nt * 8 + g) * NP + k0 + q;
        const uint32_t bh_[2] = {ShI[srow], ShI[srow + 4]};
        const uint32_t bl_[2] = {SlI[srow], SlI[srow + 4]};
        mma_tf32(acc[nt], al, bh_);
        mma_tf32(acc[nt], ah, bl_);
        mma_tf32(acc[nt], ah, bh_);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) {
      const int col = nt * 8 + 2 * q;
      if (t_lo < T)
        *reinterpret_cast<float2*>(y + head_off + (size_t)t_lo * tok_stride + col) =
            make_float2(acc[nt][0], acc[nt][1]);
      if (t_hi < T)
        *reinterpret_cast<float2*>(y + head_off + (size_t)t_hi * tok_stride + col) =
            make_float2(acc[nt][2], acc[nt][3]);
    }
  }
}

// The same correction on the 5th-generation tensor cores (N <= 64): per block a
// tile of up to 128 tokens of one (chunk, head) as one UMMA problem,
//   D[128 x NM] = A[128 x N] . B[NM x N]^T,   A = the tile's q rows,
//   B = S0 (rows past N zero; NM = N rounded up to 16),
// accumulated in tensor memory (TMEM lane = token row, column = output i).
// fp32 accuracy by 3xTF32: D = Alo Bhi + Ahi Blo + Ahi Bhi, three kind::tf32
// MMAs per 8-wide k-step into the one accumulator.  Operands sit in shared memory
// in the canonical K-major layout without swizzle (8-row x 16-byte core matrices;
// the K-adjacent core matrix 128 bytes on, the next 8 rows N/4 * 128 bytes on),
// written by the threads that load them (each thread one token row of A) after
// the tf32 split.  One thread issues the MMAs and commits them to an mbarrier;
// every warp then reads its 32 TMEM lanes and adds them to its tokens' y rows,
// which were loaded while the operands were staged.  The wait is bounded
// (WAIT_NS; an expiry is counted in g_pair_wait_timeouts, waited for once more
// and the block's outputs are void), and the TMEM columns are always freed.
// Measured on config 2 it is not yet faster than the mma.sync kernel (shared
// memory holds it to 4 blocks per SM and each block runs load, split, MMA and
// epilogue back to back), so it serves the explicit YUF_WKV_PARALLEL_TC choice.
template <int N>
struct CorrTcCfg {
  static constexpr int M = 128;                  // tokens per tile = TMEM lanes
  static constexpr int NM = (N + 15) / 16 * 16;  // MMA N: S0 rows, zero padded
  static constexpr int KC = N / 4;               // 16-byte chunks per operand row
  static constexpr uint32_t LBO = 128;           // next core matrix along K
  static constexpr uint32_t SBO = KC * 128;      // next 8 rows
  static constexpr int A_BYTES = M * N * 4;
  static constexpr int B_BYTES = NM * N * 4;
  static constexpr int OFF_AH = 0, OFF_AL = A_BYTES;
  static constexpr int OFF_BH = 2 * A_BYTES, OFF_BL = 2 * A_BYTES + B_BYTES;
  static constexpr int OFF_BAR = 2 * A_BYTES + 2 * B_BYTES;  // 16-byte multiple
  static constexpr int OFF_SLOT = OFF_BAR + 8;
  static constexpr size_t BYTES = OFF_SLOT + 8 + 128;        // + alignment slack of the base
  static constexpr uint32_t TMEM_COLS = NM <= 32 ? 32 : 64;
  static constexpr uint32_t IDESC = umma_idesc_tf32(M, NM);
  static_assert(N % 8 == 0 && N <= 64, "tcgen05 correction: N in {16, 32, 40, 48, 64}");
};

// byte offset of the 16-byte chunk c (elements 4c .. 4c+3) of operand row r
template <int N>
YUF_DEVICE uint32_t corr_tc_off(int r, int c) {
  return (uint32_t)((r & 7) * 16 + c * 128 + (r >> 3) * (int)CorrTcCfg<N>::SBO);
}


template <int N>
__global__ void __launch_bounds__(128)
    wkv7_correct_tc_kernel(const float* __restrict__ S0, const float* __restrict__ Q,
                           float* __restrict__ y, int K_, int H, int Tstride, int Cper, int skip_first,
                           int parts) {
  using Cf = CorrTcCfg<N>;
  constexpr int KC = Cf::KC;
  extern __shared__ __align__(128) unsigned char corr_tc_raw[];
  unsigned char* sm = corr_tc_raw + ((128u - (smem_u32(corr_tc_raw) & 127u)) & 127u);
  const int bh = blockIdx.x / parts, part = blockIdx.x - bh * parts;
  const int bb = bh / H, hh = bh - bb * H;
  if (skip_first && bb % Cper == 0) return;  // chunk 0 starts from the zero state
  const int tb = part * Cf::M;               // first token of this tile in the chunk
  const int T = min(Cf::M, item_len(bb, K_, Tstride, Cper) - tb);
  if (T <= 0) return;
  const int tid = threadIdx.x, warp = tid >> 5;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cf::OFF_BAR);
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + Cf::OFF_SLOT);

  if (warp == 0) {
    tmem_alloc(slot, Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  // this thread's token row: its y row is loaded now and added after the MMAs
  const int row = tid;
  const bool live = row < T;
  const size_t tok_stride = (size_t)H * N;
  float* yrow = y + item_head_off(bb, hh, K_, H, N, Tstride, Cper) + (size_t)(tb + (live ? row : 0)) * tok_stride;
  float4 yv[KC];
#pragma unroll
  for (int c = 0; c < KC; ++c)
    yv[c] = live ? reinterpret_cast<const float4*>(yrow)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  // A: the tile's q rows (rows past T zero), split into tf32 high and low parts
  const float4* qrow = reinterpret_cast<const float4*>(Q + ((size_t)bh * K_ + tb + (live ? row : 0)) * N);
#pragma unroll
  for (int c = 0; c < KC; ++c) {
    const float4 x = live ? qrow[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    uint4 hi, lo;
    split4(x, hi, lo);
    const uint32_t o = corr_tc_off<N>(row, c);
    *reinterpret_cast<uint4*>(sm + Cf::OFF_AH + o) = hi;
    *reinterpret_cast<uint4*>(sm + Cf::OFF_AL + o) = lo;
  }
  // B: S0 of this (chunk, head), rows N .. NM-1 zero
  const float4* s0 = reinterpret_cast<const float4*>(S0 + (size_t)bh * N * N);
  for (int x = tid; x < Cf::NM * KC; x += 128) {
    const int i = x / KC, c = x - i * KC;
    const float4 v = i < N ? s0[i * KC + c] : make_float4(0.f, 0.f, 0.f, 0.f);
    uint4 hi, lo;
    split4(v, hi, lo);
    const uint32_t o = corr_tc_off<N>(i, c);
    *reinterpret_cast<uint4*>(sm + Cf::OFF_BH + o) = hi;
    *reinterpret_cast<uint4*>(sm + Cf::OFF_BL + o) = lo;
  }
  fence_proxy_async();  // the operand stores become visible to the tensor core
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *slot;
  if (tid == 0) {
    const uint32_t ah = smem_u32(sm + Cf::OFF_AH), al = smem_u32(sm + Cf::OFF_AL);
    const uint32_t bh_ = smem_u32(sm + Cf::OFF_BH), bl = smem_u32(sm + Cf::OFF_BL);
#pragma unroll
    for (int s = 0; s < N / 8; ++s) {
      const uint32_t k = (uint32_t)s * 2 * Cf::LBO;  // two 16-byte chunks per k-step
      umma_tf32(tmem, umma_desc_kmajor(al + k, Cf::LBO, Cf::SBO), umma_desc_kmajor(bh_ + k, Cf::LBO, Cf::SBO),
                Cf::IDESC, s > 0 ? 1u : 0u);
      umma_tf32(tmem, umma_desc_kmajor(ah + k, Cf::LBO, Cf::SBO), umma_desc_kmajor(bl + k, Cf::LBO, Cf::SBO),
                Cf::IDESC, 1u);
      umma_tf32(tmem, umma_desc_kmajor(ah + k, Cf::LBO, Cf::SBO), umma_desc_kmajor(bh_ + k, Cf::LBO, Cf::SBO),
                Cf::IDESC, 1u);
    }
    umma_commit(bar);
  }
  __syncwarp();
  bool done = mbar_wait(bar, 0);
  done = __all_sync(0xffffffffu, done);
  if (!done) {
    if ((tid & 31) == 0) atomicAdd(&g_pair_wait_timeouts, 1u);
    mbar_wait(bar, 0);  // once more, bounded, before the columns are freed
  } else {
    tc_fence_after_sync();
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll
    for (int c8 = 0; c8 < N / 8; ++c8) {
      float d[8];
      tmem_ld_x8(lane_base + (uint32_t)(c8 * 8), d);
      float4& y0 = yv[2 * c8];
      float4& y1 = yv[2 * c8 + 1];
      y0.x += d[0]; y0.y += d[1]; y0.z += d[2]; y0.w += d[3];
      y1.x += d[4]; y1.y += d[5]; y1.z += d[6]; y1.w += d[7];
    }
    if (live) {
#pragma unroll
      for (int c = 0; c < KC; ++c) reinterpret_cast<float4*>(yrow)[c] = yv[c];
    }
  }
  tc_fence_before_sync();
  __syncthreads();  // every warp's TMEM reads are done
  if (warp == 0) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, Cf::TMEM_COLS);
  }
}

// Resident pair blocks per device for head size N (blocks per SM x SMs),
// queried once per (device, N).
int wkv7_pair_slots(int N) {
  static int cache[64][8] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  const int ni = N == 16 ? 0 : N == 32 ? 1 : N == 40 ? 2 : N == 48 ? 3 : N == 64 ? 4 : N == 96 ? 5 : 6;
  if (cache[dev][ni] > 0) return cache[dev][ni];
  int sms = 148, per_sm = 1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaSuccess;
  switch (N) {
#define SLOTW(NN)                                                                                \
  case NN: {                                                                                     \
    auto kern = wkv7_pairw_kernel<NN>;                                                           \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PairWCfg<NN>::BYTES); \
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PairWCfg<NN>::NT,           \
                                                      PairWCfg<NN>::BYTES);                        \
    break;                                                                                       \
  }
#define SLOT(NN)                                                                                 \
  case NN: {                                                                                     \
    auto kern = wkv7_pair_kernel<NN>;                                                            \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PairCfg<NN>::BYTES); \
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, PairCfg<NN>::NT, PairCfg<NN>::BYTES); \
    break;                                                                                       \
  }
    SLOTW(16) SLOTW(32) SLOTW(40) SLOTW(48) SLOTW(64) SLOT(96) SLOT(128)
#undef SLOTW
#undef SLOT
    default:
      break;
  }
  if (e != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  cache[dev][ni] = std::max(1, per_sm * sms);
  return cache[dev][ni];
}

// Largest chunk the correction kernel can stage for head size N (multiple of 8).
int wkv7_correct_max_chunk(int N) {
  (void)N;  // the correction walks a chunk 80 tokens per block: no staging limit
  return 1 << 20;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// Tensor maps of the six [rows, H*N] inputs, box = N columns x 8 rows.
static yuf_status_t make_pair_tmaps(const float* const (&src)[6], long long rows, int H, int N,
                                    PairTmaps* out) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    set_error("wkv7 pair: cuTensorMapEncodeTiled is unavailable");
    return YUF_ERR_CUDA;
  }
  const cuuint64_t gdim[2] = {(cuuint64_t)H * N, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)H * N * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)N, 8u};
  const cuuint32_t estride[2] = {1u, 1u};
  for (int i = 0; i < 6; ++i) {
    const CUresult rc = enc(&out->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(src[i]),
                            gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
      set_error("wkv7 pair: cuTensorMapEncodeTiled failed (%d) for input %d", (int)rc, i);
      return YUF_ERR_CUDA;
    }
  }
  return YUF_OK;
}

// Self-test of the bounded-wait path: one warp waits on an mbarrier that nothing
// ever arrives on, with the given bound, and records the expiry exactly as a
// scan kernel does (the timeout count the host reads through yuf_wait_timeouts /
// yuf_sync_check).  No copy is in flight, nothing faults, the context stays usable.
__global__ void wait_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar, 0, limit_ns));
  if (!ok && threadIdx.x == 0) atomicAdd(&g_pair_wait_timeouts, 1u);
}

yuf_status_t wait_selftest(unsigned long long limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns);
  return check_launch("wait_selftest_kernel");
}

// Timeouts of the pair kernel's bounded barrier waits on the current device
// since the last call (0 in a healthy run); clears the count.
unsigned int wkv7_pair_wait_timeouts() {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g_pair_wait_timeouts, sizeof(n)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_pair_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return ~0u;
  }
  return n;
}

// prm (nullable): the time-mix epilogue folded in (r, lw, k, v, la as the
// projections left them in place of r, w, k, v, a; b unused); head sizes up to
// 64 only -- YUF_ERR_UNSUPPORTED above.
yuf_status_t wkv7_pair_dispatch(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, float* y, float* Q, float* U, float* P,
                                int items, int K, int H, int N, int Tstride, int Cper, cudaStream_t st,
                                const WkvTm* prm) {
  if (prm && N > 64) return YUF_ERR_UNSUPPORTED;
  PairTmaps tm;
  if (N <= 64) {
    const float* const src[6] = {r, w, k, v, a, b};
    const yuf_status_t rc = make_pair_tmaps(src, (long long)(items / Cper) * Tstride, H, N, &tm);
    if (rc != YUF_OK) return rc;
  }
  switch (N) {
#define CASEW(NN)                                                                                \
  case NN: {                                                                                     \
    using Kc = PairWCfg<NN>;                                                                     \
    auto kern = prm ? wkv7_pairw_kernel<NN, true> : wkv7_pairw_kernel<NN, false>;               \
    if (Kc::BYTES > 48 * 1024 &&                                                                 \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Kc::BYTES) != \
            cudaSuccess) {                                                                       \
      set_error("wkv7 pair: cudaFuncSetAttribute failed");                                      \
      return YUF_ERR_CUDA;                                                                       \
    }                                                                                            \
    kern<<<items * H, Kc::NT, Kc::BYTES, st>>>(r, w, k, v, a, b, y, Q, U, P, K, H, Tstride, Cper, \
                                                tm, prm ? *prm : WkvTm{});                       \
    return check_launch("wkv7_pairw_kernel");                                                    \
  }
#define CASE(NN)                                                                                 \
  case NN: {                                                                                     \
    using Kc = PairCfg<NN>;                                                                      \
    auto kern = wkv7_pair_kernel<NN>;                                                            \
    if (Kc::BYTES > 48 * 1024 &&                                                                 \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Kc::BYTES) != \
            cudaSuccess) {                                                                       \
      set_error("wkv7 pair: cudaFuncSetAttribute failed");                                      \
      return YUF_ERR_CUDA;                                                                       \
    }                                                                                            \
    kern<<<items * H, Kc::NT, Kc::BYTES, st>>>(r, w, k, v, a, b, y, Q, U, P, K, H, Tstride, Cper); \
    return check_launch("wkv7_pair_kernel");                                                     \
  }
    CASEW(16) CASEW(32) CASEW(40) CASEW(48) CASEW(64) CASE(96) CASE(128)
#undef CASEW
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

yuf_status_t wkv7_correct_dispatch(const float* S0, const float* Q, float* y, int items, int K, int H,
                                   int N, int Tstride, int Cper, bool skip_first, bool tc, cudaStream_t st) {
  if (tc) switch (N) {  // head sizes up to 64 on request: the tcgen05 kernel
#define CASE_TC(NN)                                                                                \
  case NN: {                                                                                       \
    auto kern = wkv7_correct_tc_kernel<NN>;                                                        \
    const size_t tb = CorrTcCfg<NN>::BYTES;                                                        \
    if (tb > 48 * 1024 &&                                                                          \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tb) !=        \
            cudaSuccess) {                                                                         \
      set_error("wkv7 correct: cudaFuncSetAttribute failed");                                     \
      return YUF_ERR_CUDA;                                                                         \
    }                                                                                              \
    const int parts = (K + CorrTcCfg<NN>::M - 1) / CorrTcCfg<NN>::M;                               \
    kern<<<items * H * parts, 128, tb, st>>>(S0, Q, y, K, H, Tstride, Cper, skip_first ? 1 : 0,    \
                                             parts);                                               \
    return check_launch("wkv7_correct_tc_kernel");                                                 \
  }
    CASE_TC(16) CASE_TC(32) CASE_TC(40) CASE_TC(48) CASE_TC(64)
#undef CASE_TC
    default:
      break;
  }
  const size_t bytes = ((size_t)2 * N + 80) * (N + 4) * sizeof(float);
  switch (N) {
#define CASE(NN)                                                                                   \
  case NN: {                                                                                       \
    auto kern = wkv7_correct_kernel<NN>;                                                           \
    if (bytes > 48 * 1024 &&                                                                       \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=     \
            cudaSuccess) {                                                                         \
      set_error("wkv7 correct: cudaFuncSetAttribute failed");                                     \
      return YUF_ERR_CUDA;                                                                         \
    }                                                                                              \
    const int parts = (K + CorrCfg<NN>::TW - 1) / CorrCfg<NN>::TW;                                 \
    kern<<<items * H * parts, CorrCfg<NN>::NT, bytes, st>>>(S0, Q, y, K, H, Tstride, Cper,          \
                                                            skip_first ? 1 : 0, parts);            \
    return check_launch("wkv7_correct_kernel");                                                    \
  }
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
