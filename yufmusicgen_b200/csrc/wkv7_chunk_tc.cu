// Chunked WKV-7 prefill with the state contractions on the tensor cores (sm_100a).
//
// One CTA per (sequence, head) walks the sequence in chunks of L = 16 tokens;
// the N x N state stays in mma accumulator registers for the whole sequence.
// Per token the recurrence is (yufmusicgen/model.py:145-165, rwkv7_clampw.cu)
//   sa = S a,   S <- S diag(d) + sa b^T + v k^T,   y = S r,   d = exp(W_SCALE sigmoid(w)).
// Per chunk, with gamma_t = d_0 ... d_t (per column, gamma_{-1} = 1) and the
// scaled vectors
//   a~_t = gamma_{t-1} a_t,  b~_t = b_t / gamma_t,  k~_t = k_t / gamma_t,  r~_t = gamma_t r_t,
// the column-scaled state S'_t = S_t diag(1 / gamma_t) obeys
//   S'_t = S'_{t-1} + sa_t b~_t^T + v_t k~_t^T,   sa_t = S'_{t-1} a~_t,   y_t = S'_t r~_t
// (S'_{-1} = S, the chunk's start state).  With the chunk's Gram matrices
//   Lab[t][s] = a~_t . b~_s,  Lak[t][s] = a~_t . k~_s   (s < t),
//   Mrb[t][s] = r~_t . b~_s,  Mrk[t][s] = r~_t . k~_s   (s <= t),
// forward substitution over t gives sa_t = S w_t + u_t with
//   w_t = a~_t + sum_{s<t} Lab[t][s] w_s,      u_t = sum_{s<t} Lab[t][s] u_s + Lak[t][s] v_s,
// and then
//   y_t = S q_t + yu_t,   q_t = r~_t + sum_{s<=t} Mrb[t][s] w_s,
//                         yu_t = sum_{s<=t} Mrb[t][s] u_s + Mrk[t][s] v_s,
//   S_next = (S + sum_t sa_t b~_t^T + v_t k~_t^T) diag(gamma_15).
// Only the three products with S depend on the previous chunk:
//   SA^T = W S^T + U,   Y^T = Q S^T + YU   ([16 x N] x [N x N]),
//   dS = SA^T^T B~ + V^T K~                 ([N x 16] x [16 x N]),
// and they run on the tensor cores (mma.sync m16n8k8 tf32, 3xTF32: each fp32
// operand split into a tf32 high part and the remainder, three products, fp32
// accumulation -- fp32-class accuracy).  The retention bound d >= 0.545 keeps
// 1 / gamma below 0.545^-16 ~ 1.6e4 inside a chunk, far inside fp32, and every
// term a~_t . b~_s (s < t) carries the ratio gamma_{t-1} / gamma_s <= 1.
//
// Warp roles (per CTA):
//   * NS scan warps, warp w owning state rows 16w .. 16w+15 (all N columns):
//     per chunk SA^T and Y^T for its rows (S as the mma B operand straight from
//     the accumulator registers, the k index permuted so that a thread's two
//     accumulator columns are its two k slots), y stored to global, SA staged
//     through a warp-private scratch as the A operand of dS, S updated in fp32;
//   * NP prep warps, each preparing a whole chunk (chunks round-robin): the
//     scaled vectors in place of the staged inputs, the four Gram matrices and
//     the products W, U (and Q, YU for N <= 40; for wider heads the scan warps
//     add Y^T's in-chunk terms Mrb SA^T + Mrk V themselves) on mma.sync
//     (3xTF32), T by forward substitution;
//   * one loader warp: six TMA boxes (LD columns x 16 tokens, one per input) per
//     chunk straight into the chunk's slot.
// One ring of NB chunk slots: tma_full (the boxes' bytes), prep_full (the prep
// warp's 32 lanes), slot_empty (every scan lane).  A slot is loaded, prepared
// in place and scanned, so one chunk in flight costs one slot.
// Every wait is bounded; a timed-out wait counts in g_ctc_wait_timeouts and the
// CTA leaves after its TMA copies in flight have landed.
// Inputs are read once, y written once, the state read and written once.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "mbarrier.cuh"
#include "tma.cuh"

namespace yuf {

__device__ unsigned int g_ctc_wait_timeouts;

constexpr int CTC_L = 16;

// row stride (floats) of the prepared vectors: >= n and = 8 (mod 32), which
// makes the mma fragment loads bank-conflict free
constexpr int ctc_ld(int n) { return n + ((8 - n % 32) + 32) % 32; }

template <int N>
struct CtcCfg {
  static constexpr int L = CTC_L;
  static constexpr int LD = ctc_ld(N);
  static constexpr int NS = (N + 15) / 16;     // scan warps
  static constexpr int NJ = N / 8;             // 8-column tiles
  static constexpr int GL = L + 4;             // Gram row stride (= 20 mod 32: conflict-free fragments)
  static constexpr int SLD = 24;               // SA scratch row stride (= 24 mod 32: conflict free)
  // Where Y^T's in-chunk terms are formed.  YS: the scan warps form
  // Y^T = R~ S^T + Mrb SA^T + Mrk V themselves (wide heads, where the prep is
  // the longer side: N = 64 prep 1270 us against scan 755 us per B*H = 128
  // step when the prep made Q and YU); otherwise the prep makes
  // Q = R~ + Mrb W and YU = (Mrb T Lak + Mrk) V and the scan forms
  // Y^T = Q S^T + YU (N = 40: the other way round the scan became the longer
  // side, 185 against 124 us).
  static constexpr bool YS = LD > 40;
  static constexpr int NP = YS ? 4 : 5;        // prep warps
  static constexpr int NB = YS ? NP + 1 : NP + 2;  // chunk slots: NP in prep, one scanned (+ one loading)
  static constexpr int NT = 32 * (NS + NP + 1);
  // A chunk slot, rows of LD floats: the six TMA boxes (LD columns x L tokens:
  // r, w, k, v, a, b), transformed in place into r~, the log-decay running sums,
  // k~, v, a~, b~; then W, U, gamma_15 and either Mrb and Mrk ([L][GL] each,
  // YS) or Q and YU.
  static constexpr int S_R = 0, S_W = L * LD, S_K = 2 * L * LD, S_V = 3 * L * LD, S_A = 4 * L * LD,
                       S_B = 5 * L * LD, P_W = 6 * L * LD, P_U = 7 * L * LD, P_M = 8 * L * LD,
                       P_Q = 8 * L * LD, P_YU = 9 * L * LD, P_G = (YS ? 9 : 10) * L * LD;
  static constexpr int SLOT = (P_G + LD + 31) / 32 * 32;
  // prep warp scratch as [L][GL]: Lab (then T), Lak, T Lak; without YS also
  // Mrb, Mrk and Mrb T Lak + Mrk
  static constexpr int X_G = 0, X_T = 2 * L * GL, X_RB = 3 * L * GL, X_M2 = 5 * L * GL;
  static constexpr int XS = ((YS ? 3 : 6) * L * GL + 31) / 32 * 32;
  static constexpr int OFF_X = NB * SLOT;
  static constexpr int OFF_SA = OFF_X + NP * XS;
  static constexpr int OFF_PRM = OFF_SA + NS * L * SLD;  // the head's w0, a0, k_k, k_a ([4][LD], TM)
  static constexpr int OFF_BAR = OFF_PRM + 4 * LD;
  static constexpr int NBAR = 3 * NB;
  static constexpr size_t BYTES = (size_t)OFF_BAR * 4 + NBAR * 8;
  static constexpr uint32_t TX = 6u * L * LD * 4;
  static constexpr uint32_t TX_TM = 5u * L * LD * 4;  // TM: no b box
  static_assert(N % 8 == 0 && N <= 64, "chunked tensor-core scan: N a multiple of 8, at most 64");
  static_assert((L * LD * 4) % 128 == 0 && SLOT % 32 == 0, "TMA boxes on 128-byte boundaries");
  static_assert(LD <= 256 && (LD * 4) % 16 == 0, "TMA box width");
  static_assert(OFF_BAR % 2 == 0, "mbarriers 8-byte aligned");
  static_assert(2 * L * GL <= L * LD, "Mrb and Mrk fit their slot region");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

struct CtcTmaps {
  CUtensorMap m[6];  // r, w, k, v, a, b as [B*T, H*N] fp32
};

// The time-mix epilogue folded into the prep (TM): the boxes are then r, the w
// and a low-rank outputs, k and v as the projections left them, and the prep
// forms (yufmusicgen/model.py:113-125), per token and column,
//   w = w0 + lw,  kk = normalize(k * k_k) over the head,  alpha = sigmoid(a0 + la),
//   a = -kk,  b = kk * alpha,  k' = k * (1 + (alpha - 1) * k_a)
// -- the arithmetic of timemix_post_kernel -- before it scales them.
struct CtcTm {
  const float *w0, *a0, *k_k, *k_a;  // [H * N] per-channel parameters of the layer
};

YUF_DEVICE void split_a(const float (&x)[4], uint32_t (&h)[4], uint32_t (&l)[4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) split_tf32(x[e], h[e], l[e]);
}
YUF_DEVICE void split_b(float x0, float x1, uint32_t (&h)[2], uint32_t (&l)[2]) {
  split_tf32(x0, h[0], l[0]);
  split_tf32(x1, h[1], l[1]);
}

// Prep products on the tensor cores (mma.sync m16n8k8, 3xTF32), one warp:
//   out_p = C_p + A_p B_p  for p < NPR independent products,
//   A_p: [16][GL] row-major (t, s);  B_p, C_p, out_p: [16][LD] (16 x 16 by 16 x N,
//   C_p may be null).  The products' fragments are all loaded before the first
//   mma and the outputs stored after the last; the mma instructions of the
//   products and column tiles are interleaved term by term, so that consecutive
//   ones feed different accumulators.  Not inlined: the calls of a chunk share
//   the code.
struct PrepProd {
  const float* A;
  const float* B;
  const float* C;
  float* out;
};
template <int N, int LD, int GL, int NPR>
__device__ __noinline__ void prep_mma(PrepProd p0, PrepProd p1) {
  constexpr int NJ = N / 8;
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const PrepProd pr[2] = {p0, p1};
  uint32_t ah[NPR][2][4], al[NPR][2][4];
  uint32_t bh[NPR][2][NJ][2], bl[NPR][2][NJ][2];
  float d[NPR][NJ][4];
#pragma unroll
  for (int o = 0; o < NPR; ++o) {
    const float* A = pr[o].A;
    const float* B = pr[o].B;
    const float* C = pr[o].C;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const float x[4] = {A[g * GL + 8 * kk + q], A[(g + 8) * GL + 8 * kk + q], A[g * GL + 8 * kk + q + 4],
                          A[(g + 8) * GL + 8 * kk + q + 4]};
#pragma unroll
      for (int e = 0; e < 4; ++e) split_tf32(x[e], ah[o][kk][e], al[o][kk][e]);
#pragma unroll
      for (int nt = 0; nt < NJ; ++nt) {
        split_tf32(B[(8 * kk + q) * LD + 8 * nt + g], bh[o][kk][nt][0], bl[o][kk][nt][0]);
        split_tf32(B[(8 * kk + q + 4) * LD + 8 * nt + g], bh[o][kk][nt][1], bl[o][kk][nt][1]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NJ; ++nt) {
      if (C) {
        const float2 c0 = *reinterpret_cast<const float2*>(C + g * LD + 8 * nt + 2 * q);
        const float2 c1 = *reinterpret_cast<const float2*>(C + (g + 8) * LD + 8 * nt + 2 * q);
        d[o][nt][0] = c0.x; d[o][nt][1] = c0.y; d[o][nt][2] = c1.x; d[o][nt][3] = c1.y;
      } else {
        d[o][nt][0] = d[o][nt][1] = d[o][nt][2] = d[o][nt][3] = 0.f;
      }
    }
  }
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
    for (int o = 0; o < NPR; ++o)
#pragma unroll
      for (int nt = 0; nt < NJ; ++nt) mma_tf32(d[o][nt], al[o][kk], bh[o][kk][nt]);
#pragma unroll
    for (int o = 0; o < NPR; ++o)
#pragma unroll
      for (int nt = 0; nt < NJ; ++nt) mma_tf32(d[o][nt], ah[o][kk], bl[o][kk][nt]);
#pragma unroll
    for (int o = 0; o < NPR; ++o)
#pragma unroll
      for (int nt = 0; nt < NJ; ++nt) mma_tf32(d[o][nt], ah[o][kk], bh[o][kk][nt]);
  }
#pragma unroll
  for (int o = 0; o < NPR; ++o)
#pragma unroll
    for (int nt = 0; nt < NJ; ++nt) {
      *reinterpret_cast<float2*>(pr[o].out + g * LD + 8 * nt + 2 * q) = make_float2(d[o][nt][0], d[o][nt][1]);
      *reinterpret_cast<float2*>(pr[o].out + (g + 8) * LD + 8 * nt + 2 * q) = make_float2(d[o][nt][2], d[o][nt][3]);
    }
}

// The chunk's Gram matrices on the tensor cores, one warp:
//   [a~; r~] [b~; k~]^T  (32 x N by N x 32, 3xTF32), masked to
//   Lab, Lak (s < t), stored row-major [t][GL] at Gab and Gab + 16 GL, and
//   Mrb, Mrk (s <= t) at Grb and Grb + 16 GL.
template <int N, int LD, int GL>
__device__ __noinline__ void prep_gram(const float* At, const float* Rt, const float* Bt, const float* Kt, float* Gab,
                                       float* Grb) {
  constexpr int NJ = N / 8;
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  float d[2][4][4];  // [a~ | r~][b~ s0-7 | b~ s8-15 | k~ s0-7 | k~ s8-15]
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) d[mt][nt][e] = 0.f;
#pragma unroll 1
  for (int kc = 0; kc < NJ; ++kc) {
    // k slots q / q+4 <-> columns 8kc + 2q / 8kc + 2q + 1 (float2 loads)
    uint32_t ah[2][4], al[2][4], bh[4][2], bl[4][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const float* M = mt ? Rt : At;
      const float2 x0 = *reinterpret_cast<const float2*>(M + g * LD + 8 * kc + 2 * q);
      const float2 x1 = *reinterpret_cast<const float2*>(M + (g + 8) * LD + 8 * kc + 2 * q);
      split_tf32(x0.x, ah[mt][0], al[mt][0]);
      split_tf32(x1.x, ah[mt][1], al[mt][1]);
      split_tf32(x0.y, ah[mt][2], al[mt][2]);
      split_tf32(x1.y, ah[mt][3], al[mt][3]);
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const float* M = (nt < 2 ? Bt : Kt) + (8 * (nt & 1) + g) * LD + 8 * kc + 2 * q;
      const float2 x = *reinterpret_cast<const float2*>(M);
      split_tf32(x.x, bh[nt][0], bl[nt][0]);
      split_tf32(x.y, bh[nt][1], bl[nt][1]);
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma_tf32(d[mt][nt], al[mt], bh[nt]);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma_tf32(d[mt][nt], ah[mt], bl[nt]);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma_tf32(d[mt][nt], ah[mt], bh[nt]);
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      float* M = (mt ? Grb : Gab) + (nt >> 1) * 16 * GL;  // Lab, Lak / Mrb, Mrk
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = g + 8 * (e >> 1), sidx = 8 * (nt & 1) + 2 * q + (e & 1);
        const bool keep = mt ? sidx <= t : sidx < t;
        M[t * GL + sidx] = keep ? d[mt][nt][e] : 0.f;
      }
    }
}

// p ? a : b as one select instruction: both operands are computed first, so
// the items of an unrolled loop keep their independent dependency chains (a
// conditional around each item's loads or math would serialise them), and a
// non-finite value in a masked slot cannot leak through a multiply.
YUF_DEVICE float sel(bool p, float a, float b) {
  float r;
  asm("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\tselp.f32 %0, %1, %2, q;\n\t}"
      : "=f"(r)
      : "f"(a), "f"(b), "r"((int)p));
  return r;
}

// true once; the caller that flips the flag counts the timeout
YUF_DEVICE void ctc_abort(int* flag) {
  if (atomicExch(flag, 1) == 0) atomicAdd(&g_ctc_wait_timeouts, 1u);
}

template <int N, bool TM>
__global__ void __launch_bounds__(CtcCfg<N>::NT, 1)
    wkv7_chunk_tc_kernel(const float* __restrict__ s0, float* __restrict__ y, float* __restrict__ s_out, int T,
                         int H, const __grid_constant__ CtcTmaps tm, const CtcTm prm) {
  using K = CtcCfg<N>;
  constexpr int L = K::L, LD = K::LD, NS = K::NS, NP = K::NP, NB = K::NB, NJ = K::NJ;
  constexpr int GL = K::GL, SLD = K::SLD;
  extern __shared__ __align__(128) float ctc_smem[];
  float* sm = ctc_smem;
  uint64_t* tma_full = reinterpret_cast<uint64_t*>(sm + K::OFF_BAR);  // [NB] the slot's boxes landed
  uint64_t* prep_full = tma_full + NB;                                 // [NB] the slot is prepared
  uint64_t* slot_empty = prep_full + NB;                               // [NB] the scan is done with it
  __shared__ int abort_flag;

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = (T + L - 1) / L;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NB; ++s) {
      mbar_init(&tma_full[s], 1);
      mbar_init(&prep_full[s], 32);
      mbar_init(&slot_empty[s], 32 * NS);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (TM) {  // the head's time-mix parameters (weights: no kernel of the chain writes them)
    float* pr = sm + K::OFF_PRM;
    for (int i = threadIdx.x; i < 4 * N; i += blockDim.x) {
      const int which = i / N, j = i - which * N;
      const float* src = which == 0 ? prm.w0 : (which == 1 ? prm.a0 : (which == 2 ? prm.k_k : prm.k_a));
      pr[which * LD + j] = src[hh * N + j];
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  volatile int* abort_v = &abort_flag;

  if (warp < NS) {  // ------------------------------------------------------ scan warps
    const int g = lane >> 2, q = lane & 3;
    const int i0 = warp * 16;
    const bool h1 = i0 + 16 <= N;  // the tile's second 8 rows are state rows
    const size_t sbase = (size_t)bh * N * N;
    float S[NJ][4];
#pragma unroll
    for (int c = 0; c < NJ; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = i0 + g + (e >> 1) * 8, col = 8 * c + 2 * q + (e & 1);
        S[c][e] = (s0 && row < N) ? s0[sbase + (size_t)row * N + col] : 0.f;
      }
    float* SA = sm + K::OFF_SA + warp * L * SLD;
    const size_t ystride = (size_t)H * N;
    float* ybase = y + ((size_t)bb * T * H + hh) * N + i0;
    for (int c = 0; c < nchunks; ++c) {
      const int slot = c % NB;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&prep_full[slot], (uint32_t)(c / NB) & 1u));
      if (!ok || *abort_v) {
        if (lane == 0) ctc_abort(&abort_flag);
        break;
      }
      const float* P = sm + slot * K::SLOT;
      // SA^T = W S^T + U and Y^T = Q S^T + YU (or, YS, its first term R~ S^T)
      // for this warp's rows: M = token, N = state row, K = column
      float sa[2][4], yy[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = i0 + 8 * h + 2 * q;
        const float2 u0 = *reinterpret_cast<const float2*>(P + K::P_U + g * LD + col);
        const float2 u1 = *reinterpret_cast<const float2*>(P + K::P_U + (g + 8) * LD + col);
        sa[h][0] = u0.x; sa[h][1] = u0.y; sa[h][2] = u1.x; sa[h][3] = u1.y;
        if constexpr (K::YS) {
          yy[h][0] = yy[h][1] = yy[h][2] = yy[h][3] = 0.f;
        } else {
          const float2 y0 = *reinterpret_cast<const float2*>(P + K::P_YU + g * LD + col);
          const float2 y1 = *reinterpret_cast<const float2*>(P + K::P_YU + (g + 8) * LD + col);
          yy[h][0] = y0.x; yy[h][1] = y0.y; yy[h][2] = y1.x; yy[h][3] = y1.y;
        }
      }
      const float* QA = P + (K::YS ? K::S_R : K::P_Q);
#pragma unroll
      for (int kc = 0; kc < NJ; ++kc) {
        // A: rows g, g+8 of W (and Q or R~), k slots q / q+4 <-> columns 8kc+2q / 8kc+2q+1
        const float2 w0 = *reinterpret_cast<const float2*>(P + K::P_W + g * LD + 8 * kc + 2 * q);
        const float2 w1 = *reinterpret_cast<const float2*>(P + K::P_W + (g + 8) * LD + 8 * kc + 2 * q);
        const float2 q0 = *reinterpret_cast<const float2*>(QA + g * LD + 8 * kc + 2 * q);
        const float2 q1 = *reinterpret_cast<const float2*>(QA + (g + 8) * LD + 8 * kc + 2 * q);
        uint32_t wh[4], wl[4], qh[4], ql[4];
        split_a({w0.x, w1.x, w0.y, w1.y}, wh, wl);
        split_a({q0.x, q1.x, q0.y, q1.y}, qh, ql);
        // B: S[i0 + 8h + g][8kc + 2q (+1)], the accumulator pair of tile kc
        uint32_t bhi[2][2], blo[2][2];
        split_b(S[kc][0], S[kc][1], bhi[0], blo[0]);
        split_b(S[kc][2], S[kc][3], bhi[1], blo[1]);
        // the three terms of the four products in turn, so that consecutive
        // mma instructions feed different accumulators
        mma_tf32(sa[0], wl, bhi[0]);
        mma_tf32(yy[0], ql, bhi[0]);
        if (h1) {
          mma_tf32(sa[1], wl, bhi[1]);
          mma_tf32(yy[1], ql, bhi[1]);
        }
        mma_tf32(sa[0], wh, blo[0]);
        mma_tf32(yy[0], qh, blo[0]);
        if (h1) {
          mma_tf32(sa[1], wh, blo[1]);
          mma_tf32(yy[1], qh, blo[1]);
        }
        mma_tf32(sa[0], wh, bhi[0]);
        mma_tf32(yy[0], qh, bhi[0]);
        if (h1) {
          mma_tf32(sa[1], wh, bhi[1]);
          mma_tf32(yy[1], qh, bhi[1]);
        }
      }
      // SA into the warp's scratch as [token][row]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = 8 * h + 2 * q;
        const bool real = h == 0 || h1;
        *reinterpret_cast<float2*>(SA + g * SLD + col) =
            real ? make_float2(sa[h][0], sa[h][1]) : make_float2(0.f, 0.f);
        *reinterpret_cast<float2*>(SA + (g + 8) * SLD + col) =
            real ? make_float2(sa[h][2], sa[h][3]) : make_float2(0.f, 0.f);
      }
      __syncwarp();
      // YS: Y^T += Mrb SA^T + Mrk V: M = token, N = state row, K = token
      if constexpr (K::YS) {
        const float* Mb = P + K::P_M;
        const float* Mk = Mb + L * GL;
        const float* V = P + K::S_V + i0 + g;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int sa0 = 8 * kk + q, sb0 = sa0 + 4;
          uint32_t mbh[4], mbl[4], mkh[4], mkl[4];
          split_a({Mb[g * GL + sa0], Mb[(g + 8) * GL + sa0], Mb[g * GL + sb0], Mb[(g + 8) * GL + sb0]}, mbh, mbl);
          split_a({Mk[g * GL + sa0], Mk[(g + 8) * GL + sa0], Mk[g * GL + sb0], Mk[(g + 8) * GL + sb0]}, mkh, mkl);
          uint32_t bsh[2][2], bsl[2][2], bvh[2][2], bvl[2][2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            split_b(SA[sa0 * SLD + 8 * h + g], SA[sb0 * SLD + 8 * h + g], bsh[h], bsl[h]);
            split_b(h == 0 || h1 ? V[sa0 * LD + 8 * h] : 0.f, h == 0 || h1 ? V[sb0 * LD + 8 * h] : 0.f, bvh[h],
                    bvl[h]);
          }
          mma_tf32(yy[0], mbl, bsh[0]);
          mma_tf32(yy[0], mkl, bvh[0]);
          if (h1) {
            mma_tf32(yy[1], mbl, bsh[1]);
            mma_tf32(yy[1], mkl, bvh[1]);
          }
          mma_tf32(yy[0], mbh, bsl[0]);
          mma_tf32(yy[0], mkh, bvl[0]);
          if (h1) {
            mma_tf32(yy[1], mbh, bsl[1]);
            mma_tf32(yy[1], mkh, bvl[1]);
          }
          mma_tf32(yy[0], mbh, bsh[0]);
          mma_tf32(yy[0], mkh, bvh[0]);
          if (h1) {
            mma_tf32(yy[1], mbh, bsh[1]);
            mma_tf32(yy[1], mkh, bvh[1]);
          }
        }
      }
      // y rows of this chunk
      const int t0 = c * L + g;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = 8 * h + 2 * q;
        if (h == 0 || h1) {
          if (t0 < T) *reinterpret_cast<float2*>(ybase + (size_t)t0 * ystride + col) = make_float2(yy[h][0], yy[h][1]);
          if (t0 + 8 < T)
            *reinterpret_cast<float2*>(ybase + (size_t)(t0 + 8) * ystride + col) = make_float2(yy[h][2], yy[h][3]);
        }
      }
      // dS = SA^T^T B~ + V^T K~: M = state row, N = column, K = token
      float dS[NJ][4];
#pragma unroll
      for (int c2 = 0; c2 < NJ; ++c2)
#pragma unroll
        for (int e = 0; e < 4; ++e) dS[c2][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int ta = 8 * kk + q, tb = ta + 4;
        uint32_t sah[4], sal[4], vh[4], val[4];
        split_a({SA[ta * SLD + g], SA[ta * SLD + g + 8], SA[tb * SLD + g], SA[tb * SLD + g + 8]}, sah, sal);
        const float* V = P + K::S_V + i0 + g;
        split_a({V[ta * LD], h1 ? V[ta * LD + 8] : 0.f, V[tb * LD], h1 ? V[tb * LD + 8] : 0.f}, vh, val);
        uint32_t bbh[NJ][2], bbl[NJ][2], kh[NJ][2], kl[NJ][2];
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) {
          split_b(P[K::S_B + ta * LD + 8 * c2 + g], P[K::S_B + tb * LD + 8 * c2 + g], bbh[c2], bbl[c2]);
          split_b(P[K::S_K + ta * LD + 8 * c2 + g], P[K::S_K + tb * LD + 8 * c2 + g], kh[c2], kl[c2]);
        }
        // term by term across the column tiles (independent accumulators back to back)
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], sal, bbh[c2]);
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], val, kh[c2]);
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], sah, bbl[c2]);
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], vh, kl[c2]);
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], sah, bbh[c2]);
#pragma unroll
        for (int c2 = 0; c2 < NJ; ++c2) mma_tf32(dS[c2], vh, kh[c2]);
      }
#pragma unroll
      for (int c2 = 0; c2 < NJ; ++c2) {
        const float2 gm = *reinterpret_cast<const float2*>(P + K::P_G + 8 * c2 + 2 * q);
        S[c2][0] = (S[c2][0] + dS[c2][0]) * gm.x;
        S[c2][1] = (S[c2][1] + dS[c2][1]) * gm.y;
        S[c2][2] = (S[c2][2] + dS[c2][2]) * gm.x;
        S[c2][3] = (S[c2][3] + dS[c2][3]) * gm.y;
      }
      __syncwarp();
      mbar_arrive(&slot_empty[slot]);
    }
    if (s_out && !*abort_v) {
#pragma unroll
      for (int c = 0; c < NJ; ++c)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int row = i0 + g + 8 * hr;
          if (row < N)
            *reinterpret_cast<float2*>(s_out + sbase + (size_t)row * N + 8 * c + 2 * q) =
                make_float2(S[c][2 * hr], S[c][2 * hr + 1]);
        }
    }
  } else if (warp < NS + NP) {  // ------------------------------------------- prep warps
    const int p = warp - NS;
    float* X = sm + K::OFF_X + p * K::XS;
    for (int c = p; c < nchunks; c += NP) {
      const int ps = c % NB;
      // The slot's previous chunk is scanned first (its slot_empty phase), so
      // that this warp never waits on tma_full two phases ahead: the loads of
      // chunks c - NB and c may complete out of order, and a parity wait that
      // far ahead would see chunk c - 2 NB's completed phase.
      bool ok = mbar_wait(&slot_empty[ps], ((uint32_t)(c / NB) & 1u) ^ 1u) &&
                mbar_wait(&tma_full[ps], (uint32_t)(c / NB) & 1u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || *abort_v) {
        if (lane == 0) ctc_abort(&abort_flag);
        break;
      }
      float* P = sm + ps * K::SLOT;  // the boxes r, w, k, v, a, b as [L][LD], transformed in place
      const int Tc = min(L, T - c * L);
      // Loads are grouped ahead of the stores of each step below: the slot and
      // the scratch live in one shared array, so the compiler could not move a
      // load above a preceding store.  Loops are kept rolled where that costs
      // no parallelism, so that the scan and prep code together stay small in
      // the instruction caches.  Every step below touches item (t, j) of the
      // slot from the same lane that reads it, so the in-place transforms are
      // race free.
      const float* pw0 = sm + K::OFF_PRM;  // TM: w0, a0, k_k, k_a, LD apart
      // (0) TM: 1 / |k * k_k| per token, lanes 2t and 2t+1 summing half the
      //     columns each (F.normalize eps, model.py:116)
      float inv_n = 0.f;
      if constexpr (TM) {
        const int t = lane >> 1, j0 = (lane & 1) * (N / 2);
        float ss = 0.f;
#pragma unroll 4
        for (int j = j0; j < j0 + N / 2; ++j) {
          const float kk = P[K::S_K + t * LD + j] * pw0[2 * LD + j];
          ss = fmaf(kk, kk, ss);
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        inv_n = 1.f / fmaxf(sqrtf(ss), 1e-12f);
      }
      // (1) log retentions ls = W_SCALE sigmoid(w), an item (t, j) per lane,
      //     in place of w (TM: w = w0 + lw)
      float* Gs = P + K::S_W;
      constexpr int ITEMS = L * N / 32;  // a multiple of 4
#pragma unroll 1
      for (int i0 = 0; i0 < ITEMS; i0 += 4) {
        float lw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = lane + 32 * (i0 + u), t = e / N;
          lw[u] = Gs[t * LD + (e - t * N)];
          if constexpr (TM) lw[u] += pw0[e - t * N];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = lane + 32 * (i0 + u), t = e / N;
          Gs[t * LD + (e - t * N)] = sel(t < Tc, W_SCALE * sigmoidf_fast(lw[u]), 0.f);
        }
      }
      __syncwarp();
      // (2) running sums G_t = ls_0 + ... + ls_t (gamma_t = exp(G_t)), a lane per column
#pragma unroll 1
      for (int j = lane; j < N; j += 32) {
        float x[L];
#pragma unroll
        for (int t = 0; t < L; ++t) x[t] = Gs[t * LD + j];
#pragma unroll
        for (int t = 1; t < L; ++t) x[t] += x[t - 1];
#pragma unroll
        for (int t = 0; t < L; ++t) Gs[t * LD + j] = x[t];
        P[K::P_G + j] = __expf(x[L - 1]);
      }
      __syncwarp();
      // (3) scaled vectors in place, four items per lane and step (tokens past
      //     the sequence's end become zeros)
#pragma unroll 1
      for (int i0 = 0; i0 < ITEMS; i0 += 4) {
        float G[4], Gp[4], ra[4], rb[4], rk[4], rr[4], rv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = lane + 32 * (i0 + u), t = e / N, j = e - t * N, o = t * LD + j;
          const bool live = t < Tc;
          G[u] = Gs[o];
          Gp[u] = sel(t > 0, Gs[o - (t > 0 ? LD : 0)], 0.f);
          rr[u] = sel(live, P[K::S_R + o], 0.f);
          rk[u] = sel(live, P[K::S_K + o], 0.f);
          rv[u] = sel(live, P[K::S_V + o], 0.f);
          if constexpr (TM) {
            // a = -kk, b = kk alpha, k' = k (1 + (alpha - 1) k_a) from the raw k and la
            const float inv = __shfl_sync(0xffffffffu, inv_n, 2 * t);
            const float kk = rk[u] * pw0[2 * LD + j] * inv;
            const float alpha = sigmoidf_fast(pw0[LD + j] + sel(live, P[K::S_A + o], 0.f));
            ra[u] = -kk;
            rb[u] = kk * alpha;
            rk[u] = rk[u] * (1.f + (alpha - 1.f) * pw0[3 * LD + j]);
          } else {
            ra[u] = sel(live, P[K::S_A + o], 0.f);
            rb[u] = sel(live, P[K::S_B + o], 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = lane + 32 * (i0 + u), t = e / N, o = t * LD + (e - t * N);
          const float gam = __expf(G[u]), ginv = __expf(-G[u]), gprev = __expf(Gp[u]);
          P[K::S_A + o] = ra[u] * gprev;  // gamma_{t-1} a_t
          P[K::S_B + o] = rb[u] * ginv;   // b_t / gamma_t
          P[K::S_K + o] = rk[u] * ginv;   // k_t / gamma_t
          P[K::S_R + o] = rr[u] * gam;    // gamma_t r_t
          P[K::S_V + o] = rv[u];
        }
      }
      __syncwarp();
      // (4) Gram matrices Lab, Lak, Mrb, Mrk (row-major [t][GL])
      prep_gram<N, LD, GL>(P + K::S_A, P + K::S_R, P + K::S_B, P + K::S_K, X + K::X_G,
                           K::YS ? P + K::P_M : X + K::X_RB);
      __syncwarp();
      // (5) T = (I - Lab)^-1 (unit lower triangular), lane c < 16 solving for
      //     column c; T replaces Lab once every lane has read it
      {
        float* Lab = X + K::X_G;
        const int cidx = lane & 15;
        float x[L];
#pragma unroll
        for (int t = 0; t < L; ++t) {
          float acc = t == cidx ? 1.f : 0.f;
#pragma unroll
          for (int s2 = 0; s2 < t; ++s2) acc = fmaf(Lab[t * GL + s2], x[s2], acc);
          x[t] = acc;
        }
        __syncwarp();
        if (lane < 16) {
#pragma unroll
          for (int t = 0; t < L; ++t) Lab[t * GL + cidx] = x[t];
        }
      }
      __syncwarp();
      // (6) TLak = T Lak (16 x 16), then W = T A~ and U = TLak V (U = T Lak V
      //     regrouped); without YS also M2 = Mrb TLak + Mrk, Q = R~ + Mrb W and
      //     YU = M2 V (YU = Mrb U + Mrk V regrouped).
      {
        const float* Tm = X + K::X_G;
        const float* Lak = Tm + L * GL;
        float* TLak = X + K::X_T;
        const PrepProd none{nullptr, nullptr, nullptr, nullptr};
        prep_mma<16, GL, GL, 1>({Tm, Lak, nullptr, TLak}, none);
        prep_mma<N, LD, GL, 1>({Tm, P + K::S_A, nullptr, P + K::P_W}, none);
        __syncwarp();
        if constexpr (!K::YS) {
          const float* Mrb = X + K::X_RB;
          const float* Mrk = Mrb + L * GL;
          float* M2 = X + K::X_M2;
          prep_mma<16, GL, GL, 1>({Mrb, TLak, Mrk, M2}, none);
          prep_mma<N, LD, GL, 1>({Mrb, P + K::P_W, P + K::S_R, P + K::P_Q}, none);
          prep_mma<N, LD, GL, 1>({TLak, P + K::S_V, nullptr, P + K::P_U}, none);
          __syncwarp();
          prep_mma<N, LD, GL, 1>({M2, P + K::S_V, nullptr, P + K::P_YU}, none);
        } else {
          prep_mma<N, LD, GL, 1>({TLak, P + K::S_V, nullptr, P + K::P_U}, none);
        }
      }
      __syncwarp();
      mbar_arrive(&prep_full[ps]);
    }
  } else if (lane == 0) {  // ------------------------------------------------- loader
    const int tx = hh * N, ty = bb * T;
    int c = 0;
    for (; c < nchunks; ++c) {
      const int ps = c % NB;
      if (!mbar_wait(&slot_empty[ps], ((uint32_t)(c / NB) & 1u) ^ 1u) || *abort_v) {
        ctc_abort(&abort_flag);
        break;
      }
      float* dst = sm + ps * K::SLOT;
      mbar_expect_tx(&tma_full[ps], TM ? K::TX_TM : K::TX);
#pragma unroll
      for (int arr = 0; arr < (TM ? 5 : 6); ++arr)
        tma_load_2d(dst + arr * L * LD, &tm.m[arr], &tma_full[ps], tx, ty + c * L);
    }
    // the copies still in flight land before the CTA may leave
    for (int c2 = max(0, c - NB); c2 < c; ++c2) mbar_wait(&tma_full[c2 % NB], (uint32_t)(c2 / NB) & 1u);
  }
}

// Tensor maps of the six [B*T, H*N] inputs, box = `width` columns x 16 tokens
// (the slot's row stride: columns past the head's N are the next head's, or
// zero fill past the last head, and are never used).
static yuf_status_t make_ctc_tmaps(const float* const (&src)[6], long long rows, int H, int N, int width,
                                   CtcTmaps* out) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    set_error("wkv7 chunked-tc: cuTensorMapEncodeTiled is unavailable");
    return YUF_ERR_CUDA;
  }
  const cuuint64_t gdim[2] = {(cuuint64_t)H * N, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)H * N * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)width, (cuuint32_t)CTC_L};
  const cuuint32_t estride[2] = {1u, 1u};
  for (int i = 0; i < 6; ++i) {
    const CUresult rc = enc(&out->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(src[i]), gdim,
                            gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
      set_error("wkv7 chunked-tc: cuTensorMapEncodeTiled failed (%d) for input %d", (int)rc, i);
      return YUF_ERR_CUDA;
    }
  }
  return YUF_OK;
}

template <int N, bool TM>
static yuf_status_t launch_ctc(const float* const (&src)[6], const float* s0, float* y, float* s_out, int B, int T,
                               int H, const CtcTm& prm, cudaStream_t st) {
  using K = CtcCfg<N>;
  static std::once_flag once[128];
  static cudaError_t attr[128];
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  std::call_once(once[dev], [&] {
    attr[dev] =
        cudaFuncSetAttribute(wkv7_chunk_tc_kernel<N, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::BYTES);
  });
  if (attr[dev] != cudaSuccess) {
    set_error("wkv7 chunked-tc: cannot set %zu bytes of shared memory: %s", K::BYTES,
              cudaGetErrorString(attr[dev]));
    return YUF_ERR_CUDA;
  }
  CtcTmaps tm;
  const yuf_status_t rc = make_ctc_tmaps(src, (long long)B * T, H, N, K::LD, &tm);
  if (rc != YUF_OK) return rc;
  launch_k(wkv7_chunk_tc_kernel<N, TM>, dim3(B * H), dim3(K::NT), K::BYTES, st, s0, y, s_out, T, H, tm, prm);
  return check_launch(TM ? "wkv7_chunk_tc_kernel (time-mix)" : "wkv7_chunk_tc_kernel");
}

bool wkv7_chunk_tc_supports(int N) { return N == 16 || N == 32 || N == 40 || N == 48 || N == 64; }

// One CTA per (sequence, head) walks the whole sequence, so this kernel wins
// once the chains fill the SMs: measured on B200 at T = 2048, N = 40 it takes
// 0.86x the time-parallel scan's time at B*H = 128 (one 86 %-full wave) and
// 0.81x at B*H = 1024, but 1.9x at B*H = 32; at T = 8192, N = 64, B*H = 128
// 0.57x.  Taken for T >= 256 when the waves of CTAs are at least 85 % full.
bool wkv7_chunk_tc_applies(int B, int T, int H, int N) {
  if (T < 256 || !wkv7_chunk_tc_supports(N)) return false;
  static int sms[128];
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return false;
    }
    sms[dev] = n;
  }
  const long long bh = (long long)B * H, waves = (bh + sms[dev] - 1) / sms[dev];
  return bh * 100 >= 85 * waves * sms[dev];
}

// Chunked tensor-core scan of [B, T, H, N] inputs from s0 (nullable), writing y
// and the final state (nullable).  Inputs 16-byte aligned.
yuf_status_t wkv7_chunk_tc(const float* r, const float* w, const float* k, const float* v, const float* a,
                           const float* b, const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                           cudaStream_t st) {
  if (T == 0) {  // no tokens: the final state is the initial one
    if (!s_out || s_out == s0) return YUF_OK;
    const size_t bytes = (size_t)B * H * N * N * sizeof(float);
    const cudaError_t e = s0 ? cudaMemcpyAsync(s_out, s0, bytes, cudaMemcpyDeviceToDevice, st)
                             : cudaMemsetAsync(s_out, 0, bytes, st);
    if (e != cudaSuccess) {
      set_error("wkv7 chunked-tc: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
    return YUF_OK;
  }
  const float* const src[6] = {r, w, k, v, a, b};
  const CtcTm none{nullptr, nullptr, nullptr, nullptr};
  switch (N) {
    case 16: return launch_ctc<16, false>(src, s0, y, s_out, B, T, H, none, st);
    case 32: return launch_ctc<32, false>(src, s0, y, s_out, B, T, H, none, st);
    case 40: return launch_ctc<40, false>(src, s0, y, s_out, B, T, H, none, st);
    case 48: return launch_ctc<48, false>(src, s0, y, s_out, B, T, H, none, st);
    case 64: return launch_ctc<64, false>(src, s0, y, s_out, B, T, H, none, st);
    default:
      set_error("wkv7 chunked-tc: head size N=%d has no kernel (N in {16, 32, 40, 48, 64})", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

// The same scan from the projections' raw outputs with the time-mix epilogue
// folded into its prep (CtcTm): r, k, v and the w / a low-rank outputs lw, la
// as [B, T, H, N]; w0, a0, k_k, k_a the layer's [H * N] parameters.  T >= 1.
yuf_status_t wkv7_chunk_tc_tm(const float* r, const float* k, const float* v, const float* lw, const float* la,
                              const float* w0, const float* a0, const float* k_k, const float* k_a,
                              const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                              cudaStream_t st) {
  if (T <= 0) {
    set_error("wkv7 chunked-tc (time-mix): T = %d", T);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  // the sixth tensor map is never loaded from in this mode (any valid tensor)
  const float* const src[6] = {r, lw, k, v, la, la};
  const CtcTm prm{w0, a0, k_k, k_a};
  switch (N) {
    case 16: return launch_ctc<16, true>(src, s0, y, s_out, B, T, H, prm, st);
    case 32: return launch_ctc<32, true>(src, s0, y, s_out, B, T, H, prm, st);
    case 40: return launch_ctc<40, true>(src, s0, y, s_out, B, T, H, prm, st);
    case 48: return launch_ctc<48, true>(src, s0, y, s_out, B, T, H, prm, st);
    case 64: return launch_ctc<64, true>(src, s0, y, s_out, B, T, H, prm, st);
    default:
      set_error("wkv7 chunked-tc (time-mix): head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

unsigned int wkv7_chunk_tc_wait_timeouts() {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g_ctc_wait_timeouts, sizeof(n)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_ctc_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return ~0u;
  }
  return n;
}

}  // namespace yuf
