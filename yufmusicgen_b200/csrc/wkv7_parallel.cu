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
//      (wkv7_carry_kernel, an N x N x N product per chunk, P_c and U_c
//      prefetched with cp.async while the previous product runs);
//   3. every (sequence, chunk, head) adds S_{c-1} q_t to its y
//      (wkv7_correct_kernel, since y_t = yU_t + S_{c-1} q_t).
// The chunk count is chosen so that pass 1 fills the GPU in one wave: about
// (resident pair blocks) / (B*H) chunks per sequence, chunk length a multiple
// of 8, the last chunk of a sequence possibly shorter.  Exact in exact
// arithmetic; the fp32 rounding differs from the sequential order only by the
// product association of passes 2 and 3.

#include <algorithm>

#include "common.cuh"

namespace yuf {

constexpr int WKV_PAR_CMAX = 32;  // the carry is sequential over chunks

yuf_status_t wkv7_pair_dispatch(const float* r, const float* w, const float* k, const float* v,
                                const float* a, const float* b, float* y, float* Q, float* U, float* P,
                                int items, int K, int H, int N, int Tstride, int Cper, cudaStream_t st);
yuf_status_t wkv7_correct_dispatch(const float* S0, const float* Q, float* y, int items, int K, int H,
                                   int N, int Tstride, int Cper, bool skip_first, cudaStream_t st);
int wkv7_pair_slots(int N);
int wkv7_correct_max_chunk(int N);

// Pass 2: per (sequence, head) the chunk start states S_c = S_{c-1} P_c + U_c.
// State rows are independent recurrences, so each (sequence, head) is split
// into RS row blocks of NR = N/RS rows, one CTA each (RS = 4, 2 or 1: the most
// that fit in one wave of resident blocks, since a CTA walks every chunk of its
// sequence).  Thread = 1 row x 4 columns of the block.  P_c and the block's rows
// of U_c come in through a cp.async ring of up to 4 stages: every chunk's inputs are
// already in memory when the kernel starts, so the chain of chunks waits on the
// memory latency only once.
template <int N, int RS>
struct CarryCfg {
  static constexpr int NR = N / RS;
  static constexpr int NT = NR * N / 4;
  static constexpr int STAGE = N * N + NR * N;  // P_c and the block's rows of U_c
  static constexpr int FIT = (200 * 1024 / 4 - NR * N) / STAGE;
  static constexpr int DEPTH = FIT < 2 ? 2 : (FIT > 4 ? 4 : FIT);  // ring stages
  static constexpr int FLOATS = NR * N + DEPTH * STAGE;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <int N, int RS>
__global__ void __launch_bounds__(CarryCfg<N, RS>::NT)
    wkv7_carry_kernel(const float* __restrict__ U, const float* __restrict__ P, const float* s0,
                      float* __restrict__ S_start, float* s_out, int C, int H) {
  constexpr int NR = CarryCfg<N, RS>::NR, NT = CarryCfg<N, RS>::NT, NN = N * N;
  constexpr int STAGE = CarryCfg<N, RS>::STAGE, D = CarryCfg<N, RS>::DEPTH;
  extern __shared__ float4 carry_sm[];
  float* Ss = reinterpret_cast<float*>(carry_sm);  // [NR][N] rows of the running state
  float* ring = Ss + NR * N;                        // [D][N*N + NR*N]: P_c, then rows of U_c
  const int bh = blockIdx.x / RS, rb = blockIdx.x - bh * RS;
  const int r0 = rb * NR;
  const int s = bh / H, h = bh - s * H;
  const int tid = threadIdx.x;
  const int i = tid / (N / 4), j0 = (tid % (N / 4)) * 4;
  const size_t row_off = (size_t)r0 * N;
  const float* s0p = s0 ? s0 + (size_t)bh * NN + row_off : nullptr;
  for (int q = tid; q < NR * N; q += NT) Ss[q] = s0p ? s0p[q] : 0.f;
  auto fetch = [&](int c) {  // always commits a group (empty past the last chunk)
    if (c < C) {
      float* dst = ring + (c % D) * STAGE;
      const size_t off = (((size_t)s * C + c) * H + h) * NN;
      for (int q = tid; q < NN / 4; q += NT) cp_async_16(dst + 4 * q, P + off + 4 * q);
      for (int q = tid; q < NR * N / 4; q += NT)
        cp_async_16(dst + NN + 4 * q, U + off + row_off + 4 * q);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int c = 0; c < D - 1; ++c) fetch(c);
  for (int c = 0; c < C; ++c) {
    __syncthreads();  // Ss final for this chunk; stage (c - 1) % D free
    fetch(c + D - 1);
    {
      float* dst = S_start + (((size_t)s * C + c) * H + h) * NN + row_off;
      for (int q = tid; q < NR * N / 4; q += NT)
        reinterpret_cast<float4*>(dst)[q] = reinterpret_cast<const float4*>(Ss)[q];
    }
    cp_async_wait<D - 1>();  // chunk c's group landed
    __syncthreads();
    const float* Pc = ring + (c % D) * STAGE;
    float4 acc = *reinterpret_cast<const float4*>(Pc + NN + i * N + j0);
    float4 acc2 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int l = 0; l < N; l += 2) {
      const float4 p0 = *reinterpret_cast<const float4*>(Pc + l * N + j0);
      const float4 p1 = *reinterpret_cast<const float4*>(Pc + (l + 1) * N + j0);
      const float2 sv = *reinterpret_cast<const float2*>(Ss + i * N + l);
      acc.x = fmaf(sv.x, p0.x, acc.x); acc.y = fmaf(sv.x, p0.y, acc.y);
      acc.z = fmaf(sv.x, p0.z, acc.z); acc.w = fmaf(sv.x, p0.w, acc.w);
      acc2.x = fmaf(sv.y, p1.x, acc2.x); acc2.y = fmaf(sv.y, p1.y, acc2.y);
      acc2.z = fmaf(sv.y, p1.z, acc2.z); acc2.w = fmaf(sv.y, p1.w, acc2.w);
    }
    __syncthreads();  // every read of Ss done
    *reinterpret_cast<float4*>(Ss + i * N + j0) =
        make_float4(acc.x + acc2.x, acc.y + acc2.y, acc.z + acc2.z, acc.w + acc2.w);
  }
  cp_async_wait<0>();
  __syncthreads();
  if (s_out)
    for (int q = tid; q < NR * N; q += NT) s_out[(size_t)bh * NN + row_off + q] = Ss[q];
}

template <int N, int RS>
static yuf_status_t launch_carry_rs(const float* U, const float* P, const float* s0, float* S_start,
                                    float* s_out, int B, int C, int H, cudaStream_t st) {
  using Cf = CarryCfg<N, RS>;
  auto kern = wkv7_carry_kernel<N, RS>;
  if (Cf::BYTES > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::BYTES);
    if (e != cudaSuccess) {
      set_error("wkv7 carry: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  kern<<<B * H * RS, Cf::NT, Cf::BYTES, st>>>(U, P, s0, S_start, s_out, C, H);
  return check_launch("wkv7_carry_kernel");
}

// Resident blocks of a kernel per device (blocks per SM x SMs), 1 when unknown.
template <typename Kern>
static long long resident_blocks(Kern kern, int threads, size_t bytes) {
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (bytes > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, bytes) != cudaSuccess) {
    cudaGetLastError();
    per_sm = 1;
  }
  return (long long)std::max(1, per_sm) * sms;
}

template <int N>
static yuf_status_t launch_carry(const float* U, const float* P, const float* s0, float* S_start,
                                 float* s_out, int B, int C, int H, cudaStream_t st) {
  // RS = 4 always has a legal block size; 2 and 1 only while N*N/8 resp. N*N/4
  // threads fit in a block
  const long long BH = (long long)B * H;
  if (4 * BH <= resident_blocks(wkv7_carry_kernel<N, 4>, CarryCfg<N, 4>::NT, CarryCfg<N, 4>::BYTES))
    return launch_carry_rs<N, 4>(U, P, s0, S_start, s_out, B, C, H, st);
  if constexpr (CarryCfg<N, 2>::NT <= 1024) {
    if (2 * BH <= resident_blocks(wkv7_carry_kernel<N, 2>, CarryCfg<N, 2>::NT, CarryCfg<N, 2>::BYTES))
      return launch_carry_rs<N, 2>(U, P, s0, S_start, s_out, B, C, H, st);
    if constexpr (CarryCfg<N, 1>::NT <= 1024)
      return launch_carry_rs<N, 1>(U, P, s0, S_start, s_out, B, C, H, st);
  }
  return launch_carry_rs<N, 4>(U, P, s0, S_start, s_out, B, C, H, st);  // more than one wave
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
// SMs idle or be bound by one SM's shared-memory delivery.  Measured on B200 at
// T = 2048, N = 40: 3.8x faster at B*H = 32, 2.0x at 128, 1.2x at 512 (a third
// of the 1776 resident pair blocks).  Head sizes above 40 use the multi-warp
// pair kernel: 3.6x at B*H = 32 for N = 64, slower than sequential at 128.
bool wkv7_parallel_applies(int B, int T, int H, int N) {
  const long long BH = (long long)B * H;
  if (T < 256) return false;
  return N <= 40 ? 3 * BH <= wkv7_pair_slots(N) : BH <= 64;
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
                           int B, int T, int H, int N, float* scratch, cudaStream_t st) {
  int C = 0, K = 0;
  wkv7_parallel_plan(B, T, H, N, &C, &K);
  const size_t per = (size_t)B * C * H * N * N;
  float* U = scratch;
  float* P = U + per;
  float* S_start = P + per;
  float* Qm = S_start + per;  // [B*C, H, K, N]
  // 1. one pass: y from a zero start (into y), Q, U, P
  yuf_status_t rc = wkv7_pair_dispatch(r, w, k, v, a, b, y, Qm, U, P, B * C, K, H, N, T, C, st);
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
  return wkv7_correct_dispatch(S_start, Qm, y, B * C, K, H, N, T, C, s0 == nullptr, st);
}

}  // namespace yuf
