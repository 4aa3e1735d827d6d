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
// by ret, which loses accuracy over a chunk.  G lives in shared memory; thread
// i owns row i for the row reductions (dv, dsa) and column i for the column
// reductions and the update.
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
  static constexpr int GP = N + 1;                 // padded row of G (conflict-free rows and columns)
  static constexpr int NV = 10;                    // r, ret, sig, k, v, a, b, dy, sa, dsa
  static constexpr int SMEM = (N * GP + NV * N) * 4;
};

template <int N>
__global__ void __launch_bounds__(N)
    wkv7_backward_kernel(const float* __restrict__ r, const float* __restrict__ w,
                         const float* __restrict__ k, const float* __restrict__ v,
                         const float* __restrict__ a, const float* __restrict__ b,
                         const float* __restrict__ dy, const float* __restrict__ ck,
                         const float* __restrict__ sa, float* __restrict__ dr, float* __restrict__ dw,
                         float* __restrict__ dk, float* __restrict__ dv, float* __restrict__ da,
                         float* __restrict__ db, float* __restrict__ scratch, int T, int H) {
  using K = WkvBwd<N>;
  extern __shared__ __align__(16) float sm[];
  float* G = sm;
  float* vr = sm + N * K::GP;
  float *R_ = vr, *RET = vr + N, *SIG = vr + 2 * N, *K_ = vr + 3 * N, *V_ = vr + 4 * N,
        *A_ = vr + 5 * N, *B_ = vr + 6 * N, *DY = vr + 7 * N, *SA = vr + 8 * N, *DSA = vr + 9 * N;
  const int j = threadIdx.x;
  const int bh = blockIdx.x, bb = bh / H, hh = bh - bb * H;
  const int nc = T / BWD_CHUNK;
  const size_t NN = (size_t)N * N;
  float* scr = scratch + (size_t)bh * BWD_CHUNK * NN;  // [16][N][N]: S_t^T of the chunk's tokens
  const float* ckc = ck + (size_t)bh * nc * NN;        // [nc][N][N]: S^T after each chunk
  for (int q = j; q < N * K::GP; q += N) G[q] = 0.f;

  for (int c = nc - 1; c >= 0; --c) {
    // ---- replay the chunk: thread j carries column j of S
    float col[N];
    if (c == 0) {
#pragma unroll
      for (int i = 0; i < N; ++i) col[i] = 0.f;
    } else {
      const float4* s4 = reinterpret_cast<const float4*>(ckc + (size_t)(c - 1) * NN + (size_t)j * N);
#pragma unroll
      for (int i4 = 0; i4 < N / 4; ++i4) {
        const float4 q = s4[i4];
        col[4 * i4] = q.x; col[4 * i4 + 1] = q.y; col[4 * i4 + 2] = q.z; col[4 * i4 + 3] = q.w;
      }
    }
    for (int tau = 0; tau < BWD_CHUNK; ++tau) {
      const size_t off = (((size_t)bb * T + c * BWD_CHUNK + tau) * H + hh) * N;
      __syncthreads();  // previous users of V_ / SA are done
      V_[j] = v[off + j];
      SA[j] = sa[off + j];
      __syncthreads();
      const float retj = __expf(W_SCALE * sigmoidf_fast(w[off + j]));
      const float kj = k[off + j], bj = b[off + j];
#pragma unroll
      for (int i = 0; i < N; ++i) col[i] = fmaf(col[i], retj, fmaf(SA[i], bj, V_[i] * kj));
      float4* o4 = reinterpret_cast<float4*>(scr + (size_t)tau * NN + (size_t)j * N);
#pragma unroll
      for (int i4 = 0; i4 < N / 4; ++i4)
        o4[i4] = make_float4(col[4 * i4], col[4 * i4 + 1], col[4 * i4 + 2], col[4 * i4 + 3]);
    }
    // ---- reverse over the chunk's tokens
    for (int tau = BWD_CHUNK - 1; tau >= 0; --tau) {
      const size_t off = (((size_t)bb * T + c * BWD_CHUNK + tau) * H + hh) * N;
      __syncthreads();  // the previous token's column pass is done with G and the vectors
      R_[j] = r[off + j];
      const float sg = sigmoidf_fast(w[off + j]);
      SIG[j] = sg;
      RET[j] = __expf(W_SCALE * sg);
      K_[j] = k[off + j];
      V_[j] = v[off + j];
      A_[j] = a[off + j];
      B_[j] = b[off + j];
      DY[j] = dy[off + j];
      SA[j] = sa[off + j];
      __syncthreads();
      {  // row pass, thread j = row i: G += dy r^T, dv = G k, dsa = G b
        float* Gr = G + (size_t)j * K::GP;
        const float dyi = DY[j];
        float dvi = 0.f, dsai = 0.f;
#pragma unroll 8
        for (int q = 0; q < N; ++q) {
          const float g = fmaf(dyi, R_[q], Gr[q]);
          Gr[q] = g;
          dvi = fmaf(g, K_[q], dvi);
          dsai = fmaf(g, B_[q], dsai);
        }
        dv[off + j] = dvi;
        DSA[j] = dsai;
      }
      __syncthreads();
      {  // column pass, thread j = column j
        const float* Snew = scr + (size_t)tau * NN + (size_t)j * N;
        const float* Sold = tau > 0 ? scr + (size_t)(tau - 1) * NN + (size_t)j * N
                                    : (c > 0 ? ckc + (size_t)(c - 1) * NN + (size_t)j * N : nullptr);
        const float retj = RET[j], aj = A_[j];
        float drj = 0.f, dkj = 0.f, dbj = 0.f, dretj = 0.f, daj = 0.f;
#pragma unroll 2
        for (int i4 = 0; i4 < N / 4; ++i4) {
          const float4 sn = reinterpret_cast<const float4*>(Snew)[i4];
          const float4 so = Sold ? reinterpret_cast<const float4*>(Sold)[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float snv[4] = {sn.x, sn.y, sn.z, sn.w}, sov[4] = {so.x, so.y, so.z, so.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 4 * i4 + e;
            float* gp = G + (size_t)i * K::GP + j;
            const float g = *gp;
            drj = fmaf(snv[e], DY[i], drj);
            dkj = fmaf(g, V_[i], dkj);
            dbj = fmaf(g, SA[i], dbj);
            dretj = fmaf(g, sov[e], dretj);
            daj = fmaf(sov[e], DSA[i], daj);
            *gp = fmaf(g, retj, DSA[i] * aj);
          }
        }
        const float sg = SIG[j];
        dr[off + j] = drj;
        dk[off + j] = dkj;
        db[off + j] = dbj;
        da[off + j] = daj;
        dw[off + j] = dretj * retj * W_SCALE * sg * (1.f - sg);
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
    kern<<<B * H, NN, WkvBwd<NN>::SMEM, st>>>(r, w, k, v, a, b, dy, states, sa, dr, dw, dk, dv,  \
                                             da, db, scratch, T, H);                             \
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
