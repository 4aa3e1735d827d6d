// Time-parallel WKV-7 prefill for sm_100a.
//
// The sequential scan (wkv7.cu) gives one CTA to each (sequence, head) and walks
// all T tokens; with few sequences (the 0.1B prefill: B = 2, H = 16, 32 CTAs for
// 148 SMs) most of the GPU idles, and even at B*H = 128 one chain per SM is bound
// by that SM's shared-memory delivery.  The recurrence is linear in the state,
//   S_t = S_{t-1} G_t + v_t k_t^T,   G_t = diag(w_t) + a_t b_t^T,
// so over a chunk of tokens  S_end = S_start P + U  with the chunk's transition
// P = G_1 ... G_K and its own contribution U (the end state from a zero start).
// Three passes:
//   1. every (sequence, chunk, head) scans its tokens once with, per state row,
//      the zero-start row and the identity-start row in the same lane
//      (wkv7_pair.cu): y from a zero start, q_t = P_t r_t, U and P;
//   2. per (sequence, head) the chunk start states S_c = S_{c-1} P_c + U_c
//      (wkv7_carry_kernel, an N x N x N product per chunk on the tensor cores,
//      P_c and U_c streamed in ahead through a cp.async ring);
//   3. every (sequence, chunk, head) adds S_{c-1} q_t to its y
//      (wkv7_correct_kernel, since y_t = yU_t + S_{c-1} q_t).
// The chunk count is chosen so that pass 1 fills the GPU in one wave: about
// (resident pair blocks) / (B*H) chunks per sequence, chunk length a multiple
// of 8, the last chunk of a sequence possibly shorter.  Exact in exact
// arithmetic; the fp32 rounding differs from the sequential order only by the
// product association of passes 2 and 3.

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace yuf {

#ifndef YUF_WKV_PAR_CMAX
#define YUF_WKV_PAR_CMAX 32
#endif
constexpr int WKV_PAR_CMAX = YUF_WKV_PAR_CMAX;  // the carry is sequential over chunks

yuf_status_t wkv7_pair_dispatch(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, float* y, float* Q, float* U, float* P,
                                int items, int K, int H, int N, int Tstride, int Cper, cudaStream_t st,
                                const WkvTm* prm = nullptr);
yuf_status_t wkv7_correct_dispatch(const float* S0, const float* Q, float* y, int items, int K, int H,
                                   int N, int Tstride, int Cper, bool skip_first, bool tc, cudaStream_t st);
int wkv7_pair_slots(int N);
int wkv7_correct_max_chunk(int N);

// Pass 2: per (sequence, head) the chunk start states S_c = S_{c-1} P_c + U_c,
// one CTA per (sequence, head) walking its chunks.  The N x N x N product runs
// on the tensor cores (mma.sync m16n8k8, 3xTF32 for fp32-level accuracy): one
// warp per 16 x 8 output tile (up to 32 warps), A = rows of S from shared memory
// (rows past N read as zero), B = P_c, accumulators initialised with U_c.  P_c
// and U_c come in through a cp.async ring: every chunk's inputs are in memory
// when the kernel starts, so the chain of chunks waits on memory only once.
// Row strides: S and U pad to N + 4 floats and P to the next width = 8 mod 32,
// which makes the A and B fragment loads bank-conflict free.
template <int N>
struct CarryCfg {
  static constexpr int MT = (N + 15) / 16;               // 16-row tiles (rows >= N are zero)
  static constexpr int NTL = N / 8;                      // 8-column tiles
  static constexpr int TILES = MT * NTL;
  static constexpr int WARPS = TILES < 32 ? TILES : 32;
  static constexpr int TPW = (TILES + WARPS - 1) / WARPS;  // tiles per warp
  static constexpr int NT = 32 * WARPS;
  static constexpr int NP = N + 4;
  static constexpr int PP = N + (40 - N % 32) % 32;
  static constexpr bool UIN = N <= 96;                   // U staged in the ring
  static constexpr int STAGE = N * PP + (UIN ? N * NP : 0);
  static constexpr int SROWS = MT * 16;
  static constexpr int FIT = (200 * 1024 / 4 - SROWS * NP) / STAGE;
  static constexpr int DEPTH = FIT < 2 ? 2 : (FIT > 4 ? 4 : FIT);
  static constexpr int FLOATS = SROWS * NP + DEPTH * STAGE;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <int N>
__global__ void __launch_bounds__(CarryCfg<N>::NT)
    wkv7_carry_kernel(const float* __restrict__ U, const float* __restrict__ P, const float* s0,
                      float* __restrict__ S_start, float* s_out, int C, int H) {
  using Cf = CarryCfg<N>;
  constexpr int NT = Cf::NT, NP = Cf::NP, PP = Cf::PP, NTL = Cf::NTL, TILES = Cf::TILES;
  constexpr int WARPS = Cf::WARPS, TPW = Cf::TPW, STAGE = Cf::STAGE, D = Cf::DEPTH, NN = N * N;
  constexpr int Q4 = N / 4;
  extern __shared__ float4 carry_sm[];
  float* Ss = reinterpret_cast<float*>(carry_sm);  // [SROWS][NP] running state
  float* ring = Ss + Cf::SROWS * NP;                // [D][N*PP (+ N*NP)]: P_c, U_c
  const int bh = blockIdx.x;
  const int s = bh / H, h = bh - s * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const float* s0p = s0 ? s0 + (size_t)bh * NN : nullptr;
  for (int x = tid; x < Cf::SROWS * NP; x += NT) {  // zero padding, and all of S without s0
    const int i = x / NP, j = x - i * NP;
    if (!s0p || i >= N || j >= N) Ss[x] = 0.f;
  }
  if (s0p) {  // s0 rows arrive with the first ring stage's group
    for (int x = tid; x < N * Q4; x += NT) {
      const int i = x / Q4, j4 = x - i * Q4;
      cp_async_16(Ss + i * NP + 4 * j4, s0p + (size_t)i * N + 4 * j4);
    }
  }
  auto fetch = [&](int c) {  // always commits a group (empty past the last chunk)
    if (c < C) {
      float* dst = ring + (c % D) * STAGE;
      const size_t off = (((size_t)s * C + c) * H + h) * NN;
      for (int x = tid; x < N * Q4; x += NT) {
        const int i = x / Q4, j4 = x - i * Q4;
        cp_async_16(dst + i * PP + 4 * j4, P + off + (size_t)i * N + 4 * j4);
        if (Cf::UIN) cp_async_16(dst + N * PP + i * NP + 4 * j4, U + off + (size_t)i * N + 4 * j4);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int c = 0; c < D - 1; ++c) fetch(c);
  for (int c = 0; c < C; ++c) {
    __syncthreads();  // Ss = S_{c-1}; stage (c - 1) % D free
    fetch(c + D - 1);
    cp_async_wait<D - 1>();  // chunk c's group landed (and, at c = 0, the s0 rows)
    __syncthreads();
    {
      float* dst = S_start + (((size_t)s * C + c) * H + h) * NN;
      for (int x = tid; x < N * Q4; x += NT) {
        const int i = x / Q4, j4 = x - i * Q4;
        *reinterpret_cast<float4*>(dst + i * N + 4 * j4) =
            *reinterpret_cast<const float4*>(Ss + i * NP + 4 * j4);
      }
    }
    const float* Pc = ring + (c % D) * STAGE;
    const float* Uc = Pc + N * PP;
    const float* Ug = U + (((size_t)s * C + c) * H + h) * NN;
    // three accumulator chains per tile while registers allow (N <= 64), one beyond
    using AccT = typename std::conditional<(TPW <= 1), Acc3, float[4]>::type;
    AccT acc[TPW];
#pragma unroll
    for (int tp = 0; tp < TPW; ++tp) {
      const int tile = warp + tp * WARPS;
      if (tile < TILES) {
        const int m0 = (tile / NTL) * 16, n0 = (tile % NTL) * 8;
        const int r_lo = m0 + g, r_hi = m0 + g + 8, col = n0 + 2 * q;
        float2 u_lo = make_float2(0.f, 0.f), u_hi = u_lo;
        if (Cf::UIN) {
          if (r_lo < N) u_lo = *reinterpret_cast<const float2*>(Uc + r_lo * NP + col);
          if (r_hi < N) u_hi = *reinterpret_cast<const float2*>(Uc + r_hi * NP + col);
        } else {
          if (r_lo < N) u_lo = *reinterpret_cast<const float2*>(Ug + (size_t)r_lo * N + col);
          if (r_hi < N) u_hi = *reinterpret_cast<const float2*>(Ug + (size_t)r_hi * N + col);
        }
        acc_init(acc[tp], u_lo.x, u_lo.y, u_hi.x, u_hi.y);
#pragma unroll
        for (int k0 = 0; k0 < N; k0 += 8) {
          const float a[4] = {Ss[r_lo * NP + k0 + q], Ss[r_hi * NP + k0 + q],
                              Ss[r_lo * NP + k0 + q + 4], Ss[r_hi * NP + k0 + q + 4]};
          const float b[2] = {Pc[(k0 + q) * PP + n0 + g], Pc[(k0 + q + 4) * PP + n0 + g]};
          mma_3xtf32(acc[tp], a, b);
        }
      }
    }
    __syncthreads();  // every read of Ss done
#pragma unroll
    for (int tp = 0; tp < TPW; ++tp) {
      const int tile = warp + tp * WARPS;
      if (tile < TILES) {
        const int m0 = (tile / NTL) * 16, n0 = (tile % NTL) * 8;
        const int r_lo = m0 + g, r_hi = m0 + g + 8, col = n0 + 2 * q;
        if (r_lo < N)
          *reinterpret_cast<float2*>(Ss + r_lo * NP + col) =
              make_float2(acc_get(acc[tp], 0), acc_get(acc[tp], 1));
        if (r_hi < N)
          *reinterpret_cast<float2*>(Ss + r_hi * NP + col) =
              make_float2(acc_get(acc[tp], 2), acc_get(acc[tp], 3));
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  if (s_out)
    for (int x = tid; x < NN; x += NT) s_out[(size_t)bh * NN + x] = Ss[(x / N) * NP + x % N];
}

template <int N>
static yuf_status_t launch_carry(const float* U, const float* P, const float* s0, float* S_start,
                                 float* s_out, int B, int C, int H, cudaStream_t st) {
  using Cf = CarryCfg<N>;
  auto kern = wkv7_carry_kernel<N>;
  if (Cf::BYTES > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::BYTES);
    if (e != cudaSuccess) {
      set_error("wkv7 carry: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H, Cf::NT, Cf::BYTES, st>>>(U, P, s0, S_start, s_out, C, H);
  return check_launch("wkv7_carry_kernel");
}

// Chunks per sequence and chunk length for B sequences of T tokens.
void wkv7_parallel_plan(int B, int T, int H, int N, int* C_out, int* K_out) {
  const long long BH = std::max(1LL, (long long)B * H);
  long long C = wkv7_pair_slots(N) / BH;
  C = std::max(2LL, std::min<long long>(C, WKV_PAR_CMAX));
  C = std::min<long long>(C, std::max(1, T / 16));
  int K = (int)((T + C - 1) / C);
  K = (K + 7) / 8 * 8;
  K = std::min(K, wkv7_correct_max_chunk(N));
  *K_out = K;
  *C_out = (T + K - 1) / K;
}

// The parallel path does about twice the sequential work (the N transition rows
// of pass 1); it wins while the sequential scan, one chain per CTA, would leave
// SMs idle or be bound by one SM's shared-memory delivery.  Measured on B200,
// T = 2048: N = 40 3.8x faster at B*H = 32, 2.4x at 128, 1.2x at 512; N = 64
// 4.9x at 32, 1.7x at 128, 1.4x at 256 (1.8x at 128 for T = 8192).  Taken while
// B*H is at most half the resident pair blocks (888 at N = 40, 370 at N = 64 on
// a 148-SM B200); head sizes above 64 use the multi-warp pair kernel, which
// wins only for few chains.
bool wkv7_parallel_applies(int B, int T, int H, int N) {
  const long long BH = (long long)B * H;
  if (T < 256) return false;
  return N <= 64 ? 2 * BH <= wkv7_pair_slots(N) : BH <= 64;
}

size_t wkv7_parallel_scratch_floats(int B, int T, int H, int N) {
  int C = 0, K = 0;
  wkv7_parallel_plan(B, T, H, N, &C, &K);
  // U, P and the chunk start states; Q ([K, N] per chunk and head)
  return 3 * (size_t)B * C * H * N * N + (size_t)B * C * H * K * N;
}

// Scratch for any B, T with B*T <= rows and T >= 256 (the engine's workspace):
// B*C*H <= max(slots, 2*B*H) + B*H*ceil(T / Kmax) and B*C*H*K <= 2*B*H*T.
size_t wkv7_parallel_scratch_bound(size_t rows, int H, int N) {
  if (rows < 256) return 0;  // no sequence of 256 tokens fits
  const size_t bh = (rows / 256) * (size_t)H;
  const size_t items = std::max<size_t>((size_t)wkv7_pair_slots(N), 2 * bh) +
                       (size_t)H * (rows / (size_t)wkv7_correct_max_chunk(N) + rows / 256 + 1);
  return 3 * items * N * N + 2 * rows * (size_t)H * N + 16;
}

yuf_status_t wkv7_parallel(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           int B, int T, int H, int N, float* scratch, cudaStream_t st, bool tc_correct,
                           const WkvTm* tm) {
  int C = 0, K = 0;
  wkv7_parallel_plan(B, T, H, N, &C, &K);
  const size_t per = (size_t)B * C * H * N * N;
  float* U = scratch;
  float* P = U + per;
  float* S_start = P + per;
  float* Qm = S_start + per;  // [B*C, H, K, N]
  // 1. one pass: y from a zero start (into y), Q, U, P
  yuf_status_t rc = wkv7_pair_dispatch(r, w, k, v, a, b, y, Qm, U, P, B * C, K, H, N, T, C, st, tm);
  if (rc != YUF_OK) return rc;
  // 2. chunk start states and the final state
  switch (N) {
#define CASE(NN) \
  case NN: rc = launch_carry<NN>(U, P, s0, S_start, s_out, B, C, H, st); break;
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
  if (rc != YUF_OK) return rc;
  // 3. y += S_start q_t per (chunk, head); chunk 0 of a zero start needs none
  return wkv7_correct_dispatch(S_start, Qm, y, B * C, K, H, N, T, C, s0 == nullptr, tc_correct, st);
}

}  // namespace yuf
