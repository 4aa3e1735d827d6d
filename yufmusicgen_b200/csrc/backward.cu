// Training backward of the two scans on sm_100a: the reference's torch ops
// yufmusicgen_rwkv7::backward (rwkv7_clampw.cpp:40-63, kernel rwkv7_clampw.cu:83-176)
// and yufmusicgen_rosa::backward (rosa_householder.cpp:52-83, kernel
// rosa_householder.cu:103-285), with the same buffers.  Both return the exact
// gradient of the forward recurrences; where the reference kernels differ from
// it (below) the result follows the mathematics, which is what torch autograd
// gives through the reference's own CPU recurrences.
//
// WKV-7 (yufmusicgen/model.py:156-164), per (sequence, head) chain, state S [N, N]
// (row i = value, column j = key):
//   sa = S a,  S' = S diag(ret) + sa b^T + v k^T,  y = S' r,  ret = exp(W_SCALE sigmoid(w)).
// Reverse mode with G = dL/dS' (zero after the last token; the final state
// carries no gradient):
//   G += dy r^T;  dr = S'^T dy;  dv = G k;  dk = G^T v;  db = G^T sa;  dsa = G b;
//   dret_j = sum_i G_ij S_ij;  da = S^T dsa;  G <- G diag(ret) + dsa a^T.
// The states before and after every token are recomputed, one 16-token chunk at
// a time, from the forward's chunk checkpoints and its saved sa: column j of S'
// is column j of S times ret_j plus sa b_j + v k_j, so a thread per column
// replays the chunk without any reduction and writes the 16 states (transposed)
// to a per-chain scratch.  The reference instead undoes each update by dividing
// by ret, which loses accuracy over a chunk.  G lives in shared memory; eight
// lanes serve row i for the row reductions (dv, dsa) and
// column i for the column reductions and the update, each over a slice of the
// other index, and combine their partial sums with shuffles.  A chunk's token
// vectors are staged in shared memory in one pass and the state slices are
// loaded one token ahead, so no global load sits on the per-token chain.
//
// ROSA (yufmusicgen/model.py:280-287, the CUDA op's ungated read,
// rosa_householder.cu:89-91), per sequence, memory m [R], unit direction d:
//   h = m - 2 (d.m) d,  m' = D h + sigmoid(write) tanh(cand),  read = m' - 2 (d.m') d.
// Reverse mode with P = dL/dm' (zero after the last token):
//   P += H dq;  d_cand, d_write from P;  d_decay_t = P h;  e = D P;  P <- e - 2 (d.e) d;
//   d_direction -= 2 [(d.dq) m' + (d.m') dq] + 2 [(d.e) m + (d.m) e].
// H = I - 2 d d^T is symmetric.  One CTA per sequence, a thread per channel,
// one block reduction of six dot products per token.  Differences from the
// reference kernel: it propagates D H P where the chain rule gives H D P, it
// contracts the direction term with P instead of D P and skips it at t = 0,
// and it fills d_read_raw from a shared array read before it is written;
// d_read_raw is zero here because the ungated read does not depend on read_raw.

#include "common.cuh"

namespace yuf {

constexpr int BWD_CHUNK = 16;

template <int N>
struct WkvBwd {
  static constexpr int L = 8;                      // lanes per row / column
  static constexpr int C = N / L;                  // elements per lane
  static constexpr int THREADS = N * L;
  static constexpr int GP = N + 1;                 // padded row of G
  static constexpr int NV = 9;                     // per token: r, ret, sig, k, v, a, b, dy, sa
  static constexpr int SMEM = (N * GP + BWD_CHUNK * NV * N + N) * 4;  // G, chunk vectors, dsa
  // load the state slices one token ahead (a third register slice; not at N = 128,
  // whose 1024 threads have 64 registers each)
  static constexpr bool PREFETCH = N < 128;
  static_assert(N % L == 0, "lane slices");
};
enum { VR = 0, VRET, VSIG, VK, VV, VA, VB, VDY, VSA };

// sum over the L lanes of a row group (consecutive lanes)
template <int L>
YUF_DEVICE float lane_sum(float x) {
#pragma unroll
  for (int o = 1; o < L; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int N>
__global__ void __launch_bounds__(WkvBwd<N>::THREADS)
    wkv7_backward_kernel(const float* __restrict__ r, const float* __restrict__ w,
                         const float* __restrict__ k, const float* __restrict__ v,
                         const float* __restrict__ a, const float* __restrict__ b,
                         const float* __restrict__ dy, const float* __restrict__ ck,
                         const float* __restrict__ sa, float* __restrict__ dr, float* __restrict__ dw,
                         float* __restrict__ dk, float* __restrict__ dv, float* __restrict__ da,
                         float* __restrict__ db, float* __restrict__ scratch, int T, int H) {
  using K = WkvBwd<N>;
  constexpr int L = K::L, C = K::C, NV = K::NV;
  extern __shared__ __align__(16) float sm[];
  float* G = sm;
  float* VS = sm + N * K::GP;            // [16][NV][N]: the chunk's token vectors
  float* DSA = VS + BWD_CHUNK * NV * N;  // [N]
  const int tid = threadIdx.x;
  const int x = tid / L, g = tid - x * L, i0 = g * C;  // x: the row / column this lane serves
  const int bh = blockIdx.x, bb = bh / H, hh = bh - bb * H;
  const int nc = T / BWD_CHUNK;
  const size_t NN = (size_t)N * N;
  float* scr = scratch + (size_t)bh * BWD_CHUNK * NN;  // [16][N][N]: S_t^T of the chunk's tokens
  const float* ckc = ck + (size_t)bh * nc * NN;        // [nc][N][N]: S^T after each chunk
  for (int q = tid; q < N * K::GP; q += K::THREADS) G[q] = 0.f;
  auto slice = [&](const float* base, float (&o)[C]) {  // this lane's part of row x of S^T
    if (base == nullptr) {
#pragma unroll
      for (int e = 0; e < C; ++e) o[e] = 0.f;
    } else if constexpr (C % 2 == 0) {
      const float2* p2 = reinterpret_cast<const float2*>(base + (size_t)x * N + i0);
#pragma unroll
      for (int e = 0; e < C / 2; ++e) {
        const float2 q = p2[e];
        o[2 * e] = q.x;
        o[2 * e + 1] = q.y;
      }
    } else {
      const float* p1 = base + (size_t)x * N + i0;
#pragma unroll
      for (int e = 0; e < C; ++e) o[e] = p1[e];
    }
  };

  for (int c = nc - 1; c >= 0; --c) {
    const float* start = c > 0 ? ckc + (size_t)(c - 1) * NN : nullptr;  // S^T before the chunk
    // ---- stage the chunk's vectors (one latency per chunk, not per token)
    __syncthreads();  // the previous chunk is done with VS
    for (int q = tid; q < BWD_CHUNK * NV * N; q += K::THREADS) {
      const int tau = q / (NV * N), rem = q - tau * NV * N, vi = rem / N, e = rem - vi * N;
      const size_t off = (((size_t)bb * T + c * BWD_CHUNK + tau) * H + hh) * N + e;
      const float* sp = vi == VR ? r : vi <= VSIG ? w : vi == VK ? k : vi == VV ? v
                      : vi == VA ? a : vi == VB ? b : vi == VDY ? dy : sa;
      float val = sp[off];
      if (vi == VSIG) val = sigmoidf_fast(val);
      else if (vi == VRET) val = __expf(W_SCALE * sigmoidf_fast(val));
      VS[q] = val;
    }
    __syncthreads();
    // ---- replay: lane (x, g) carries rows i0 .. i0+C-1 of column x of S
    {
      float col[C];
      slice(start, col);
      for (int tau = 0; tau < BWD_CHUNK; ++tau) {
        const float* vt = VS + tau * NV * N;
        const float retx = vt[VRET * N + x], kx = vt[VK * N + x], bx = vt[VB * N + x];
        float* o1 = scr + (size_t)tau * NN + (size_t)x * N + i0;
#pragma unroll
        for (int e = 0; e < C; ++e)
          col[e] = fmaf(col[e], retx, fmaf(vt[VSA * N + i0 + e], bx, vt[VV * N + i0 + e] * kx));
        if constexpr (C % 2 == 0) {
#pragma unroll
          for (int e = 0; e < C / 2; ++e)
            reinterpret_cast<float2*>(o1)[e] = make_float2(col[2 * e], col[2 * e + 1]);
        } else {
#pragma unroll
          for (int e = 0; e < C; ++e) o1[e] = col[e];
        }
      }
    }
    // ---- reverse over the chunk's tokens; the state slices of the next token
    // back are loaded one token ahead
    float sn[C], so[C], nx[C];
    slice(scr + (size_t)(BWD_CHUNK - 1) * NN, sn);
    if constexpr (K::PREFETCH) slice(scr + (size_t)(BWD_CHUNK - 2) * NN, so);
    // unrolled, so the slice rotation below is register renaming and the
    // one-token-ahead loads are not waited for early
#pragma unroll
    for (int tau = BWD_CHUNK - 1; tau >= 0; --tau) {
      // so = S before token tau (the previous chunk's end, or zero, at tau = 0)
      const float* prev = tau > 0 ? scr + (size_t)(tau - 1) * NN : start;
      if constexpr (K::PREFETCH) {
        if (tau >= 2) slice(scr + (size_t)(tau - 2) * NN, nx);
        else if (tau == 1) slice(start, nx);
      } else {
        slice(prev, so);
      }
      const size_t off = (((size_t)bb * T + c * BWD_CHUNK + tau) * H + hh) * N;
      const float* vt = VS + tau * NV * N;
      __syncthreads();  // the previous token's column pass is done with G and DSA
      {  // row pass, lane (x = row i, g): G += dy r^T, dv = G k, dsa = G b over its columns
        float* Gr = G + (size_t)x * K::GP + i0;
        const float dyi = vt[VDY * N + x];
        float dvi = 0.f, dsai = 0.f;
#pragma unroll
        for (int q = 0; q < C; ++q) {
          const float gv = fmaf(dyi, vt[VR * N + i0 + q], Gr[q]);
          Gr[q] = gv;
          dvi = fmaf(gv, vt[VK * N + i0 + q], dvi);
          dsai = fmaf(gv, vt[VB * N + i0 + q], dsai);
        }
        dvi = lane_sum<L>(dvi);
        dsai = lane_sum<L>(dsai);
        if (g == 0) {
          dv[off + x] = dvi;
          DSA[x] = dsai;
        }
      }
      __syncthreads();
      {  // column pass, lane (x = column j, g) over rows i0 .. i0+C-1
        const float retj = vt[VRET * N + x], aj = vt[VA * N + x];
        float drj = 0.f, dkj = 0.f, dbj = 0.f, dretj = 0.f, daj = 0.f;
#pragma unroll
        for (int e = 0; e < C; ++e) {
          const int i = i0 + e;
          float* gp = G + (size_t)i * K::GP + x;
          const float gv = *gp;
          drj = fmaf(sn[e], vt[VDY * N + i], drj);
          dkj = fmaf(gv, vt[VV * N + i], dkj);
          dbj = fmaf(gv, vt[VSA * N + i], dbj);
          dretj = fmaf(gv, so[e], dretj);
          daj = fmaf(so[e], DSA[i], daj);
          *gp = fmaf(gv, retj, DSA[i] * aj);
        }
        drj = lane_sum<L>(drj);
        dkj = lane_sum<L>(dkj);
        dbj = lane_sum<L>(dbj);
        dretj = lane_sum<L>(dretj);
        daj = lane_sum<L>(daj);
        if (g == 0) {
          const float sg = vt[VSIG * N + x];
          dr[off + x] = drj;
          dk[off + x] = dkj;
          db[off + x] = dbj;
          da[off + x] = daj;
          dw[off + x] = dretj * retj * W_SCALE * sg * (1.f - sg);
        }
      }
#pragma unroll
      for (int e = 0; e < C; ++e) {
        sn[e] = so[e];
        if constexpr (K::PREFETCH) so[e] = nx[e];
      }
    }
  }
}

// floats of scratch the WKV-7 backward needs
size_t wkv7_backward_scratch_floats(int B, int H, int N) {
  return (size_t)B * H * BWD_CHUNK * N * N;
}

yuf_status_t wkv7_backward_dispatch(const float* r, const float* w, const float* k, const float* v,
                                    const float* a, const float* b, const float* dy,
                                    const float* states, const float* sa, float* dr, float* dw,
                                    float* dk, float* dv, float* da, float* db, float* scratch,
                                    int B, int T, int H, int N, cudaStream_t st) {
  switch (N) {
#define CASE(NN)                                                                                 \
  case NN: {                                                                                     \
    auto kern = wkv7_backward_kernel<NN>;                                                        \
    if (WkvBwd<NN>::SMEM > 48 * 1024 &&                                                          \
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                  \
                             WkvBwd<NN>::SMEM) != cudaSuccess) {                                 \
      set_error("wkv7 backward: cudaFuncSetAttribute failed");                                  \
      return YUF_ERR_CUDA;                                                                       \
    }                                                                                            \
    kern<<<B * H, WkvBwd<NN>::THREADS, WkvBwd<NN>::SMEM, st>>>(                                \
        r, w, k, v, a, b, dy, states, sa, dr, dw, dk, dv, da, db, scratch, T, H);                \
    return check_launch("wkv7_backward_kernel");                                                 \
  }
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7 backward: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

// ---------------------------------------------------------------------------
// ROSA backward: one CTA per sequence, thread k = channel k.
__global__ void __launch_bounds__(1024)
    rosa_backward_kernel(const float* __restrict__ cand_s, const float* __restrict__ write_s,
                         const float* __restrict__ decay_s, const float* __restrict__ mem_s,
                         const float* __restrict__ direction, const float* __restrict__ d_read,
                         float* __restrict__ d_cand, float* __restrict__ d_write,
                         float* __restrict__ d_read_raw, float* __restrict__ d_decay,
                         float* __restrict__ d_dir, float* __restrict__ d_mem, int T, int R) {
  __shared__ float scratch[32 * 6];
  __shared__ float red[6];
  const int bb = blockIdx.x, kk = threadIdx.x, nwarps = blockDim.x >> 5;
  const bool act = kk < R;
  const float dk_ = act ? direction[kk] : 0.f;
  float P = 0.f, ddir = 0.f;
  for (int t = T - 1; t >= 0; --t) {
    const size_t o = ((size_t)bb * T + t) * R + kk;
    const size_t mo = ((size_t)bb * (T + 1) + t) * R + kk;
    const float q = act ? d_read[o] : 0.f;
    const float m_old = act ? mem_s[mo] : 0.f, m_new = act ? mem_s[mo + R] : 0.f;
    const float D = act ? decay_s[o] : 0.f;
    const float wg = act ? write_s[o] : 0.f, cg = act ? cand_s[o] : 0.f;
    // d.dq, d.m, d.m', d.(D P_old), d.(D dq), d.(D d)
    float x[6] = {dk_ * q, dk_ * m_old, dk_ * m_new, dk_ * D * P, dk_ * D * q, dk_ * D * dk_};
    block_sum_array<6>(x, scratch, red, nwarps);
    const float dq_d = red[0], mo_d = red[1], mn_d = red[2];
    P = P + fmaf(-2.f * dq_d, dk_, q);  // P += H dq
    // d.(D P) after the update, from the reduced pieces
    const float e_d = red[3] + red[4] - 2.f * dq_d * red[5];
    const float e = D * P;
    ddir -= 2.f * (dq_d * m_new + mn_d * q) + 2.f * (e_d * m_old + mo_d * e);
    if (act) {
      d_cand[o] = P * wg * (1.f - cg * cg);
      d_write[o] = P * cg * wg * (1.f - wg);
      d_read_raw[o] = 0.f;
      d_decay[o] = P * fmaf(-2.f * mo_d, dk_, m_old);
    }
    P = fmaf(-2.f * e_d, dk_, e);
  }
  if (act) {
    d_dir[(size_t)bb * R + kk] = ddir;
    d_mem[(size_t)bb * R + kk] = P;
  }
}

yuf_status_t rosa_backward_dispatch(const float* cand_s, const float* write_s, const float* decay_s,
                                    const float* mem_s, const float* direction, const float* d_read,
                                    float* d_cand, float* d_write, float* d_read_raw, float* d_decay,
                                    float* d_dir, float* d_mem, int B, int T, int R,
                                    cudaStream_t st) {
  const int threads = ((R + 31) / 32) * 32;
  rosa_backward_kernel<<<B, threads, 0, st>>>(cand_s, write_s, decay_s, mem_s, direction, d_read,
                                              d_cand, d_write, d_read_raw, d_decay, d_dir, d_mem,
                                              T, R);
  return check_launch("rosa_backward_kernel");
}

}  // namespace yuf
