// ROSA Householder-memory scan for sm_100a.
//
// Math (yufmusicgen/model.py:260-288; rosa_householder.cu:30-101), per batch
// row, memory m in R^R, unit direction d, post-sigmoid decay D = diag(decay):
//   p_t    = d . m_{t-1}
//   m_t    = D (m_{t-1} - 2 p_t d) + u_t,        u_t = sigmoid(write_t) * tanh(cand_t)
//   read_t = m_t - 2 (d . m_t) d  (= m_t - 2 p_{t+1} d), optionally * sigmoid(gate_t)
//
// The only coupling between channels is the scalar p_t.  Split m_t = e_t - 2 g_t
// with the plain per-channel EMA e_t = D e_{t-1} + u_t (e_0 = m_0) and the
// correction g_t = D (g_{t-1} + p_t d) (g_0 = 0).  Then
//   p_t = d . e_{t-1} - 2 sum_{tau<t} c_{t-tau} p_tau,   c_k = sum_j d_j^2 decay_j^k,
// a lower-triangular Toeplitz system whose matrix (I + 2C) is the same for every
// chunk of L tokens, because D and d do not depend on the token.  Its inverse is
// lower-triangular Toeplitz too (coefficients q_n, computed once per launch), so
// within a chunk:
//   1. each thread (one channel) runs its EMA over the chunk: no communication;
//   2. ONE block reduction yields all L+1 dot products s_t = d . e_t at once;
//   3. p_{t+1} = sum_tau q_{t-tau} s_tau (every thread, from shared memory);
//   4. each thread forms g_t, m_t and read_t.
// That replaces the reference's two block-wide O(R) dot products per token with
// one batched reduction per 16 tokens.  One CTA per batch row, one thread per
// channel; the next chunk's inputs are loaded into registers while the current
// one is processed.

#include "common.cuh"
#include "model_kernels.cuh"

namespace yuf {

constexpr int ROSA_L = 16;

bool rosa_parallel_applies(int B, int T, int R);
yuf_status_t rosa_parallel(const float* cand, const float* write, const float* gate,
                           const float* bias_c, const float* bias_w, const float* bias_g, int ld,
                           const float* decay, const float* dir, int raw, const float* m0,
                           float* read, float* m_out, int B, int T, int R, bool gated,
                           float* scratch, cudaStream_t s, const float* factors = nullptr);

// Per-layer constants of the scan for channel j of a block of `nwarps` warps:
// the unit direction d_j and post-sigmoid decay dec_j (from the raw parameters
// when raw != 0: decay = sigmoid(decay_param), d = normalize(householder),
// yufmusicgen/model.py:300-301) and the L+1 coefficients q_n of the inverse
// Toeplitz matrix (I + 2C)^{-1}, c_k = sum_j d_j^2 dec_j^k:
//   q_0 = 1,  q_n = -2 sum_{k=1..n} c_k q_{n-k}.
// Every thread of the block calls it (it holds block reductions and barriers).
constexpr int ROSA_COEF_D = 32;  // coefficient block: q [L+1] (padded to 32), d [R], dec [R]
YUF_DEVICE void rosa_setup(int j, int R, int nwarps, const float* __restrict__ decay,
                           const float* __restrict__ dir, int raw, float* scratch, float* c_sum,
                           float* q, float& d, float& dec, float (&qr)[ROSA_L + 1]) {
  constexpr int L = ROSA_L;
  const bool act = j < R;
  d = act ? dir[j] : 0.f;
  dec = act ? decay[j] : 0.f;
  if (raw) {
    dec = act ? 1.f / (1.f + expf(-dec)) : 0.f;
    float x1[1] = {d * d};
    block_sum_array<1>(x1, scratch, c_sum, nwarps);
    d = d / fmaxf(sqrtf(c_sum[0]), 1e-12f);
  }
  {  // c_k, k = 1..L (index 0 unused)
    float x[L + 1];
    float pw = d * d;
    x[0] = 0.f;
#pragma unroll
    for (int kk = 1; kk <= L; ++kk) {
      pw *= dec;
      x[kk] = pw;
    }
    block_sum_array<L + 1>(x, scratch, c_sum, nwarps);
  }
  if (j == 0) {
    q[0] = 1.f;
    for (int n = 1; n <= L; ++n) {
      float acc = 0.f;
      for (int kk = 1; kk <= n; ++kk) acc += c_sum[kk] * q[n - kk];
      q[n] = -2.f * acc;
    }
  }
  __syncthreads();
#pragma unroll
  for (int n = 0; n <= L; ++n) qr[n] = q[n];
}

// The setup once per launch of the time-parallel scan (one block of the scan
// kernels' width, so the reductions add in the same order): coef = [q (padded
// to ROSA_COEF_D), d (R), dec (R)], read by every chunk's block instead of
// repeating two block reductions and the serial solve.
__global__ void __launch_bounds__(1024)
    rosa_coef_kernel(const float* __restrict__ decay, const float* __restrict__ dir, int raw, int R,
                     float* __restrict__ coef) {
  __shared__ float scratch[32 * (ROSA_L + 1)];
  __shared__ float c_sum[ROSA_L + 1];
  __shared__ float q[ROSA_L + 1];
  const int j = threadIdx.x;
  float d, dec, qr[ROSA_L + 1];
  rosa_setup(j, R, blockDim.x >> 5, decay, dir, raw, scratch, c_sum, q, d, dec, qr);
  if (j <= ROSA_L) coef[j] = qr[j];
  if (j < R) {
    coef[ROSA_COEF_D + j] = d;
    coef[ROSA_COEF_D + R + j] = dec;
  }
}

// MODE 0: the scan.  MODE 1: end state only, from a zero initial state (no read
// output).  MODE 2: transition -- batch row bb starts from the unit vector e_bb
// with zero input for T steps, so m_out row bb = A^T e_bb, i.e. column bb of
// A^T (A the one-step transition, A^T its T-th power).
// LEAN: the register-light form for launches of many more blocks than the SMs
// hold at once (the chunk passes of a long time-parallel scan): p_t formed once
// per block in shared memory instead of by every thread, u_t formed inside the
// EMA, the next gate requested after the read stage, three 256-thread blocks
// per SM.  The default form keeps all of that in registers, which is faster
// where each block's chain of chunks is the critical path.
template <bool GATED, bool COMPAT, int MAXT, int MODE = 0, bool LEAN = false>
__global__ void __launch_bounds__(MAXT, LEAN ? 3 : 1)
    rosa_scan_kernel(const float* __restrict__ cand, const float* __restrict__ write,
                     const float* __restrict__ gate, const float* __restrict__ decay,
                     const float* __restrict__ dir, const float* m0, float* __restrict__ read,
                     float* m_out, float* __restrict__ cand_saved, float* __restrict__ write_saved,
                     float* __restrict__ read_saved, float* __restrict__ gate_saved,
                     float* __restrict__ decay_saved, float* __restrict__ mem_saved, int T, int R,
                     int ld, const float* __restrict__ bias_c, const float* __restrict__ bias_w,
                     const float* __restrict__ bias_g, int raw_params,
                     const float* __restrict__ coef = nullptr) {
  constexpr int L = ROSA_L;
  __shared__ float scratch[32 * (L + 1)];
  __shared__ float s_sum[L + 1];
  __shared__ float q[L + 1];
  __shared__ float c_sum[L + 1];
  __shared__ float p_sm[L + 1];

  const int bb = blockIdx.x;
  const int j = threadIdx.x;
  const int nwarps = blockDim.x >> 5;
  const bool act = j < R;
  // direction, decay and the Toeplitz inverse: precomputed for the launch
  // (rosa_coef_kernel, the time-parallel scan) or set up here
  float d, dec, qr[L + 1];
  if (coef != nullptr) {
    d = act ? coef[ROSA_COEF_D + j] : 0.f;
    dec = act ? coef[ROSA_COEF_D + R + j] : 0.f;
    if (j <= L) q[j] = coef[j];  // read after the first block reduction's barriers
    if constexpr (!LEAN) {
#pragma unroll
      for (int n = 0; n <= L; ++n) qr[n] = coef[n];
    }
  } else {
    rosa_setup(j, R, nwarps, decay, dir, raw_params, scratch, c_sum, q, d, dec, qr);
  }
  const float bc = (act && bias_c) ? bias_c[j] : 0.f;
  const float bw = (act && bias_w) ? bias_w[j] : 0.f;
  const float bg = (act && bias_g) ? bias_g[j] : 0.f;

  float m = (MODE == 2) ? ((act && j == bb) ? 1.f : 0.f)
                        : ((MODE == 1 || !act) ? 0.f : m0[(size_t)bb * R + j]);
  const size_t base = (size_t)bb * T * R + j;            // output [B, T, R]
  const size_t base_in = (size_t)bb * T * ld + j;        // inputs: row stride ld
  if (COMPAT && act) mem_saved[(size_t)bb * (T + 1) * R + j] = m;

  float cc[L], ww[L], gg[L];
  auto load_cw = [&](int t0) {
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const bool ok = act && (t0 + t < T) && MODE != 2;
      const size_t o = base_in + (size_t)(t0 + t) * ld;
      cc[t] = ok ? cand[o] + bc : 0.f;
      ww[t] = ok ? write[o] + bw : 0.f;
    }
  };
  auto load_g = [&](int t0) {
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const bool ok = act && (t0 + t < T) && MODE != 2;
      gg[t] = (ok && (GATED || COMPAT)) ? gate[base_in + (size_t)(t0 + t) * ld] + bg : 0.f;
    }
  };
  if (T > 0) {
    load_cw(0);
    load_g(0);
  }

  for (int t0 = 0; t0 < T; t0 += L) {
    const int Lc = min(L, T - t0);
    // LEAN: the gate is only read in step 4, so the next chunk's gate is
    // requested after it; otherwise (and for COMPAT's saved tensors) the
    // chunk's raw inputs are copied before the next chunk's are requested
    float gcur[(COMPAT || !LEAN) ? L : 1], ccur[COMPAT ? L : 1], wcur[COMPAT ? L : 1];
    float u[LEAN ? 1 : L];
    if constexpr (COMPAT) {
#pragma unroll
      for (int t = 0; t < L; ++t) {
        ccur[t] = cc[t];
        wcur[t] = ww[t];
      }
    }
    if constexpr (COMPAT || !LEAN) {
#pragma unroll
      for (int t = 0; t < L; ++t) gcur[t] = gg[t];
    }
    if constexpr (!LEAN) {
#pragma unroll
      for (int t = 0; t < L; ++t) u[t] = sigmoidf_fast(ww[t]) * tanhf(cc[t]);
      if (t0 + L < T) {  // prefetch the next chunk
        load_cw(t0 + L);
        load_g(t0 + L);
      }
    }

    // 1. per-channel EMA from the true chunk-start memory.
    float e[L + 1];
    e[0] = m;
#pragma unroll
    for (int t = 0; t < L; ++t) {
      float ut;
      if constexpr (LEAN) ut = sigmoidf_fast(ww[t]) * tanhf(cc[t]);
      else ut = u[t];
      e[t + 1] = (t < Lc) ? fmaf(dec, e[t], ut) : e[t];
    }
    if constexpr (LEAN) {
      if (t0 + L < T) {  // prefetch the next chunk
        load_cw(t0 + L);
        if constexpr (COMPAT) load_g(t0 + L);
      }
    }
    // 2. all L+1 projections s_t = d . e_t in one block reduction (the steps of
    //    block_sum_array, with d e_t formed in place).
    {
      const int lane = j & 31, warp = j >> 5;
#pragma unroll
      for (int i = 0; i <= L; ++i) {
        float sv = d * e[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, o);
        if (lane == 0) scratch[warp * (L + 1) + i] = sv;
      }
      __syncthreads();
      if (j <= L) {
        float sv = 0.f;
        for (int wi = 0; wi < nwarps; ++wi) sv += scratch[wi * (L + 1) + j];
        s_sum[j] = sv;
      }
      __syncthreads();
    }
    // 3. p_{t+1} = sum_{tau <= t} q_{t-tau} s_tau  (p index shifted by one): by
    //    every thread into registers, or (LEAN) once per block, thread t forming
    //    p_t into shared memory.
    float p[LEAN ? 1 : L + 1];
    if constexpr (LEAN) {
      if (j <= L) {
        float acc = 0.f;
        for (int tau = 0; tau <= j; ++tau) acc = fmaf(q[j - tau], s_sum[tau], acc);
        p_sm[j] = acc;
      }
      __syncthreads();
    } else {
      float sv[L + 1];
#pragma unroll
      for (int t = 0; t <= L; ++t) sv[t] = s_sum[t];
#pragma unroll
      for (int t = 0; t <= L; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int tau = 0; tau <= t; ++tau) acc = fmaf(qr[t - tau], sv[tau], acc);
        p[t] = acc;
      }
    }
    auto P = [&](int t) -> float {
      if constexpr (LEAN) return p_sm[t];
      else return p[t];
    };
    // 4. correction, memory and read.
    float gc = 0.f;
#pragma unroll
    for (int t = 0; t < L; ++t) {
      if (t < Lc) {
        gc = dec * fmaf(P(t), d, gc);
        const float mt = fmaf(-2.f, gc, e[t + 1]);
        const float rd = fmaf(-2.f * P(t + 1), d, mt);
        if (act && MODE == 0) {
          const size_t o = base + (size_t)(t0 + t) * R;
          if constexpr (COMPAT) {
            read[o] = rd;
            read_saved[o] = rd;
            cand_saved[o] = tanhf(ccur[t]);
            write_saved[o] = sigmoidf_fast(wcur[t]);
            gate_saved[o] = sigmoidf_fast(gcur[t]);
            decay_saved[o] = dec;
            mem_saved[(size_t)bb * (T + 1) * R + (size_t)(t0 + t + 1) * R + j] = mt;
          } else if constexpr (GATED) {
            float gv;
            if constexpr (LEAN) gv = gg[t];
            else gv = gcur[t];
            read[o] = rd * sigmoidf_fast(gv);
          } else {
            read[o] = rd;
          }
        }
        if (t == Lc - 1) m = mt;
      }
    }
    if constexpr (LEAN && !COMPAT)
      if (t0 + L < T) load_g(t0 + L);
    __syncthreads();  // s_sum / scratch / p_sm are rewritten by the next chunk
  }
  if (act && m_out != nullptr) m_out[(size_t)bb * R + j] = m;
}

// One token (decode): per sequence two block reductions instead of the chunk
// machinery (16 Toeplitz lags, their inverse and a 17-wide reduction):
//   p = d . m,  m' = D (m - 2 p d) + u,  read = (m' - 2 (d . m') d) [* sigmoid(gate)].
// With raw parameters (engine) d = householder / ||householder|| and the norm
// is folded into the first reduction.  read_bf (optional) receives a bf16 copy
// of read, the next projection's GEMM operand.
template <bool GATED>
__global__ void __launch_bounds__(1024)
    rosa_step_kernel(const float* __restrict__ cand, const float* __restrict__ write,
                     const float* __restrict__ gate, const float* __restrict__ decay,
                     const float* __restrict__ dir, const float* m0, float* __restrict__ read,
                     float* m_out, int R, int ld, const float* __restrict__ bias_c,
                     const float* __restrict__ bias_w, const float* __restrict__ bias_g,
                     int raw_params, __nv_bfloat16* __restrict__ read_bf) {
  pdl_wait();
  pdl_trigger();
  __shared__ float scratch[32 * 2];
  __shared__ float red[2];
  const int bb = blockIdx.x, j = threadIdx.x, nwarps = blockDim.x >> 5;
  const bool act = j < R;
  float d = act ? dir[j] : 0.f;
  float dec = act ? decay[j] : 0.f;
  if (raw_params) dec = act ? 1.f / (1.f + expf(-dec)) : 0.f;
  const float m = act ? (m0 ? m0[(size_t)bb * R + j] : 0.f) : 0.f;
  {
    float x2[2] = {d * d, d * m};
    block_sum_array<2>(x2, scratch, red, nwarps);
  }
  float p = red[1];
  if (raw_params) {
    const float inv = 1.f / fmaxf(sqrtf(red[0]), 1e-12f);
    d *= inv;
    p *= inv;
  }
  const size_t io = (size_t)bb * ld + j;
  const float bc = (act && bias_c) ? bias_c[j] : 0.f;
  const float bw = (act && bias_w) ? bias_w[j] : 0.f;
  const float u = act ? sigmoidf_fast(write[io] + bw) * tanhf(cand[io] + bc) : 0.f;
  const float mn = act ? fmaf(dec, fmaf(-2.f * p, d, m), u) : 0.f;
  __syncthreads();  // red / scratch are reused
  {
    float x1[1] = {d * mn};
    block_sum_array<1>(x1, scratch, red, nwarps);
  }
  if (act) {
    float rd = fmaf(-2.f * red[0], d, mn);
    if (GATED) rd *= sigmoidf_fast(gate[io] + ((bias_g) ? bias_g[j] : 0.f));
    read[(size_t)bb * R + j] = rd;
    if (read_bf) read_bf[(size_t)bb * R + j] = __float2bfloat16_rn(rd);
    if (m_out) m_out[(size_t)bb * R + j] = mn;
  }
}

template <bool GATED, bool COMPAT>
static yuf_status_t launch_rosa(const float* cand, const float* write, const float* gate,
                                const float* decay, const float* dir, const float* m0, float* read,
                                float* m_out, float* cs, float* ws, float* rs, float* gs, float* ds,
                                float* ms, int B, int T, int R, cudaStream_t stream) {
  const int threads = ((R + 31) / 32) * 32;
  if (threads <= 256)
    rosa_scan_kernel<GATED, COMPAT, 256><<<B, threads, 0, stream>>>(
        cand, write, gate, decay, dir, m0, read, m_out, cs, ws, rs, gs, ds, ms, T, R, R, nullptr,
        nullptr, nullptr, 0);
  else
    rosa_scan_kernel<GATED, COMPAT, 1024><<<B, threads, 0, stream>>>(
        cand, write, gate, decay, dir, m0, read, m_out, cs, ws, rs, gs, ds, ms, T, R, R, nullptr,
        nullptr, nullptr, 0);
  return check_launch("rosa_scan_kernel");
}

size_t rosa_parallel_scratch_floats(int B, int T, int R);

yuf_status_t rosa_dispatch(const float* cand, const float* write, const float* gate,
                           const float* decay, const float* dir, const float* m0, float* read,
                           float* m_out, int B, int T, int R, bool gated, cudaStream_t stream) {
  if (rosa_parallel_applies(B, T, R)) {
    // stream-ordered scratch: freed on the stream right after use
    float* scratch = nullptr;
    const size_t bytes = rosa_parallel_scratch_floats(B, T, R) * sizeof(float);
    cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&scratch), bytes, stream);
    if (e != cudaSuccess) {
      set_error("rosa: scratch allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
      return YUF_ERR_OUT_OF_MEMORY;
    }
    yuf_status_t st = rosa_parallel(cand, write, gate, nullptr, nullptr, nullptr, R, decay, dir, 0, m0,
                                    read, m_out, B, T, R, gated, scratch, stream);
    scratch_free(scratch, stream);
    return st;
  }
  if (gated)
    return launch_rosa<true, false>(cand, write, gate, decay, dir, m0, read, m_out, nullptr, nullptr,
                                    nullptr, nullptr, nullptr, nullptr, B, T, R, stream);
  return launch_rosa<false, false>(cand, write, gate, decay, dir, m0, read, m_out, nullptr, nullptr,
                                   nullptr, nullptr, nullptr, nullptr, B, T, R, stream);
}

yuf_status_t rosa_compat_dispatch(const float* cand, const float* write, const float* gate,
                                  const float* decay, const float* dir, const float* m0, float* read,
                                  float* m_out, float* cs, float* ws, float* rs, float* gs, float* ds,
                                  float* ms, int B, int T, int R, cudaStream_t stream) {
  return launch_rosa<false, true>(cand, write, gate, decay, dir, m0, read, m_out, cs, ws, rs, gs, ds,
                                  ms, B, T, R, stream);
}

static yuf_status_t rosa_engine_scan(const float* cand, const float* write, const float* gate,
                                     const float* bias_c, const float* bias_w, const float* bias_g,
                                     int ld, const float* decay_raw, const float* dir_raw,
                                     const float* m0, float* read, float* m_out, int B, int T, int R,
                                     float* scratch, const float* factors, cudaStream_t stream);

yuf_status_t rosa_engine_dispatch(const float* cand, const float* write, const float* gate,
                                  const float* bias_c, const float* bias_w, const float* bias_g,
                                  int ld, const float* decay_raw, const float* dir_raw,
                                  const float* m0, float* read, float* m_out, int B, int T, int R,
                                  float* scratch, __nv_bfloat16* read_bf, cudaStream_t stream,
                                  const float* factors) {
  if (T == 1 && R <= 1024) {
    launch_k(rosa_step_kernel<true>, dim3(B), dim3(((R + 31) / 32) * 32), 0, stream, 
        cand, write, gate, decay_raw, dir_raw, m0, read, m_out, R, ld, bias_c, bias_w, bias_g, 1,
        read_bf);
    return check_launch("rosa_step_kernel");
  }
  yuf_status_t st = rosa_engine_scan(cand, write, gate, bias_c, bias_w, bias_g, ld, decay_raw, dir_raw,
                                     m0, read, m_out, B, T, R, scratch, factors, stream);
  if (st == YUF_OK && read_bf) {
    launch_to_bf16(read, read_bf, (size_t)B * T * R, stream);
    return check_launch("to_bf16_kernel");
  }
  return st;
}

// The engine's multi-token scan: time-parallel when it applies, else one CTA
// per sequence.
static yuf_status_t rosa_engine_scan(const float* cand, const float* write, const float* gate,
                                     const float* bias_c, const float* bias_w, const float* bias_g,
                                     int ld, const float* decay_raw, const float* dir_raw,
                                     const float* m0, float* read, float* m_out, int B, int T, int R,
                                     float* scratch, const float* factors, cudaStream_t stream) {
  if (scratch && rosa_parallel_applies(B, T, R))
    return rosa_parallel(cand, write, gate, bias_c, bias_w, bias_g, ld, decay_raw, dir_raw, 1, m0,
                         read, m_out, B, T, R, true, scratch, stream, factors);
  const int threads = ((R + 31) / 32) * 32;
  if (threads <= 256)
    rosa_scan_kernel<true, false, 256><<<B, threads, 0, stream>>>(
        cand, write, gate, decay_raw, dir_raw, m0, read, m_out, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, T, R, ld, bias_c, bias_w, bias_g, 1);
  else
    rosa_scan_kernel<true, false, 1024><<<B, threads, 0, stream>>>(
        cand, write, gate, decay_raw, dir_raw, m0, read, m_out, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, T, R, ld, bias_c, bias_w, bias_g, 1);
  return check_launch("rosa_scan_kernel");
}

// ---------------------------------------------------------------------------
// Time-parallel ROSA scan.  With few sequences (the 0.1B prefill has B = 2) the
// one-CTA-per-sequence scan leaves the GPU idle, so the T axis is cut into
// chunks of K tokens.  The transition A = diag(decay)(I - 2 d d^T) does not
// depend on the token, hence:
//   1. A^K: scan R unit vectors for K steps with zero input (MODE 2);
//   2. every chunk, as its own "sequence", is scanned from a zero state (MODE 1)
//      giving its end state z_c -- chunks of one sequence are contiguous in
//      [B, T, R], so the chunk batch is the same tensor viewed as [B*T/K, K, R];
//   3. per sequence, m_c = A^K m_{c-1} + z_c over the chunks (rosa_carry_kernel);
//   4. every chunk is scanned again from its true start state (MODE 0).
// Exact in exact arithmetic (linearity of the recurrence in m).  K = 32 for
// R <= 128 (A^K in shared memory); K = 64 above, where the carry applies A^K in
// its diagonal-plus-rank-K form (rosa_lowrank_kernel).
static int rosa_par_k(int R) { return R <= 128 ? 32 : 64; }

// One CTA per sequence; A^K (stored transposed: AKt[j][i] = (A^K)[i][j]) in
// shared memory.
__global__ void __launch_bounds__(128)
    rosa_carry_kernel(const float* __restrict__ AKt, const float* __restrict__ z,
                      const float* m0, float* __restrict__ m_start, float* m_out, int C, int R) {
  extern __shared__ float4 sh4[];
  float* A = reinterpret_cast<float*>(sh4);  // [R][R]
  float* mv = A + R * R;                     // [R]
  const int b = blockIdx.x, i = threadIdx.x;
  // A^K staged asynchronously (R*R is a multiple of 4: R % 4 == 0 here, or the
  // scalar tail below)
  for (int q = i; q < R * R / 4; q += blockDim.x) cp_async_16(A + 4 * q, AKt + 4 * q);
  cp_async_commit();
  for (int q = (R * R / 4) * 4 + i; q < R * R; q += blockDim.x) A[q] = AKt[q];
  float m = (i < R && m0) ? m0[(size_t)b * R + i] : 0.f;
  float zc = (i < R && C > 0) ? z[(size_t)b * C * R + i] : 0.f;  // z of the current chunk
  cp_async_wait<0>();
  for (int c = 0; c < C; ++c) {
    const size_t row = ((size_t)b * C + c) * R;
    // next chunk's z is loaded now, so its latency hides behind this step
    const float zn = (i < R && c + 1 < C) ? z[row + R + i] : 0.f;
    if (i < R) {
      m_start[row + i] = m;
      mv[i] = m;
    }
    __syncthreads();
    if (i < R) {
      float a0 = zc, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int j = 0;
      for (; j + 4 <= R; j += 4) {
        a0 = fmaf(A[(j + 0) * R + i], mv[j + 0], a0);
        a1 = fmaf(A[(j + 1) * R + i], mv[j + 1], a1);
        a2 = fmaf(A[(j + 2) * R + i], mv[j + 2], a2);
        a3 = fmaf(A[(j + 3) * R + i], mv[j + 3], a3);
      }
      for (; j < R; ++j) a0 = fmaf(A[j * R + i], mv[j], a0);
      m = (a0 + a1) + (a2 + a3);
    }
    zc = zn;
    __syncthreads();
  }
  if (i < R && m_out) m_out[(size_t)b * R + i] = m;
}

// The same carry with A^K held in registers, for R in {32, 64, 128}: the thread
// pair (2i, 2i + 1) owns row i of A^K, each thread half of its columns (R/2
// registers), so a chunk step reads only m from shared memory (R/8 LDS.128 per
// thread, every lane of a warp at the same address), sums its half row in eight
// chains and combines the pair with one shuffle.  m is double buffered, so a
// step needs one barrier: a buffer is written again only two steps later, after
// every thread has passed the barrier that follows its reads.  The chunk end
// states z arrive by cp.async in blocks of ZB chunks, double buffered, so the
// chain of steps never waits on a global load.
template <int R>
__global__ void __launch_bounds__(2 * R)
    rosa_carry_reg_kernel(const float* __restrict__ AKt, const float* __restrict__ z,
                          const float* m0, float* __restrict__ m_start, float* m_out, int C) {
  constexpr int HALF = R / 2, ZB = 16, NT = 2 * R;
  static_assert(R % 32 == 0 && R <= 128, "register carry: R in {32, 64, 128}");
  __shared__ __align__(16) float mv[2][R];
  __shared__ __align__(16) float zs[2][ZB * R];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int i = tid >> 1, half = tid & 1, j0 = half * HALF;
  const int nblk = (C + ZB - 1) / ZB;
  auto fetch = [&](int blk) {  // chunks [blk*ZB, blk*ZB + ZB) of this sequence; always commits
    if (blk < nblk) {
      const int c0 = blk * ZB, n4 = min(ZB, C - c0) * R / 4;
      const float* src = z + ((size_t)b * C + c0) * R;
      for (int x = tid; x < n4; x += NT) cp_async_16(&zs[blk & 1][4 * x], src + 4 * x);
    }
    cp_async_commit();
  };
  fetch(0);
  float arow[HALF];
#pragma unroll
  for (int c = 0; c < HALF; ++c) arow[c] = AKt[(size_t)(j0 + c) * R + i];  // (A^K)[i][j0 + c]
  float mi = m0 ? m0[(size_t)b * R + i] : 0.f;
  for (int c = 0; c < C; ++c) {
    const size_t row = ((size_t)b * C + c) * R;
    const int blk = c / ZB, cc = c - blk * ZB;
    if (cc == 0) {
      __syncthreads();  // every read of the buffer refilled below is done
      fetch(blk + 1);
      cp_async_wait<1>();  // this block's chunks landed
      __syncthreads();
    }
    const float zc = zs[blk & 1][cc * R + i];
    float* mb = mv[c & 1];
    if (half == 0) {
      m_start[row + i] = mi;
      mb[i] = mi;
    }
    __syncthreads();
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll
    for (int q = 0; q < HALF / 4; ++q) {
      const float4 mm = *reinterpret_cast<const float4*>(mb + j0 + 4 * q);
      const int a = (2 * q) & 7;
      acc[a] = fmaf(arow[4 * q + 0], mm.x, acc[a]);
      acc[a + 1] = fmaf(arow[4 * q + 1], mm.y, acc[a + 1]);
      acc[a] = fmaf(arow[4 * q + 2], mm.z, acc[a]);
      acc[a + 1] = fmaf(arow[4 * q + 3], mm.w, acc[a + 1]);
    }
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    mi = s + zc;
  }
  cp_async_wait<0>();
  if (half == 0 && m_out) m_out[(size_t)b * R + i] = mi;
}

// R > 128: A^K (R x R) does not fit in shared memory, but it is a diagonal plus
// a rank-K matrix.  With A = D (I - 2 d d^T):
//   A^K x = D^K x - 2 sum_{s=1..K} p_s D^{K-s+1} d,   p_s = d^T A^{s-1} x,
// i.e. A^K = D^K - 2 W M with W[:, s] = D^{K-s+1} d and M[s, :] = d^T A^{s-1}.
// rosa_lowrank_kernel (one CTA) builds W (as Wt[s][i]), M (as Mt[j][s]) and D^K
// once per launch; the carry then costs 2 K R products per chunk instead of R^2.
__global__ void __launch_bounds__(256)
    rosa_lowrank_kernel(const float* __restrict__ decay, const float* __restrict__ dir, int raw,
                        float* __restrict__ Wt, float* __restrict__ Mt, float* __restrict__ DK, int K,
                        int R) {
  __shared__ float scratch[32];
  __shared__ float red[1];
  const int j = threadIdx.x, nwarps = blockDim.x >> 5;
  const bool act = j < R;
  float d = act ? dir[j] : 0.f;
  float dec = act ? decay[j] : 0.f;
  if (raw) {  // as in rosa_scan_kernel: decay = sigmoid(param), d = normalize(householder)
    dec = act ? 1.f / (1.f + expf(-dec)) : 0.f;
    float x1[1] = {d * d};
    block_sum_array<1>(x1, scratch, red, nwarps);
    d = d / fmaxf(sqrtf(red[0]), 1e-12f);
  }
  // W columns: D^{K-s+1} d, s = 1..K  (Wt[s-1][j])
  {
    float pw = dec;  // dec^1 for s = K
    for (int s = K; s >= 1; --s) {
      if (act) Wt[(size_t)(s - 1) * R + j] = pw * d;
      pw *= dec;
    }
  }
  {
    float pk = 1.f;
    for (int s = 0; s < K; ++s) pk *= dec;
    if (act) DK[j] = pk;
  }
  // M rows: x_1 = d, x_{s+1} = x_s A = (x_s D) - 2 ((x_s D) . d) d   (Mt[j][s-1])
  float x = d;
  for (int s = 1; s <= K; ++s) {
    if (act) Mt[(size_t)j * K + (s - 1)] = x;
    const float xd = x * dec;
    float x1[1] = {xd * d};
    block_sum_array<1>(x1, scratch, red, nwarps);
    x = xd - 2.f * red[0] * d;
  }
}

// One CTA per sequence; Wt [K][R] and Mt [R][K] in shared memory.
__global__ void __launch_bounds__(256)
    rosa_carry_lowrank_kernel(const float* __restrict__ Wt, const float* __restrict__ Mt,
                              const float* __restrict__ DK, const float* __restrict__ z,
                              const float* m0, float* __restrict__ m_start, float* m_out, int C, int K,
                              int R) {
  extern __shared__ float4 sh4[];
  const int KP = K;           // Ms rows are read across the threads s: conflict-free unpadded
  float* Ws = reinterpret_cast<float*>(sh4);  // [K][R]
  float* Ms = Ws + K * R;     // [R][K]
  float* mv = Ms + R * KP;    // [R]
  float* pv = mv + R;         // [K]
  const int b = blockIdx.x, i = threadIdx.x;
  const bool on = i < R;
  // factors staged asynchronously (K*R is a multiple of 4: K = 64)
  for (int q = i; q < K * R / 4; q += blockDim.x) {
    cp_async_16(Ws + 4 * q, Wt + 4 * q);
    cp_async_16(Ms + 4 * q, Mt + 4 * q);
  }
  cp_async_commit();
  const float dk = on ? DK[i] : 0.f;
  float m = (on && m0) ? m0[(size_t)b * R + i] : 0.f;
  float zc = (on && C > 0) ? z[(size_t)b * C * R + i] : 0.f;  // z of the current chunk
  cp_async_wait<0>();
  for (int c = 0; c < C; ++c) {
    const size_t row = ((size_t)b * C + c) * R;
    const float zn = (on && c + 1 < C) ? z[row + R + i] : 0.f;  // next chunk's z, in flight
    if (on) {
      m_start[row + i] = m;
      mv[i] = m;
    }
    __syncthreads();
    if (i < K) {  // p_s = M[s, :] . m
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int jj = 0;
      for (; jj + 4 <= R; jj += 4) {
        a0 = fmaf(Ms[(jj + 0) * KP + i], mv[jj + 0], a0);
        a1 = fmaf(Ms[(jj + 1) * KP + i], mv[jj + 1], a1);
        a2 = fmaf(Ms[(jj + 2) * KP + i], mv[jj + 2], a2);
        a3 = fmaf(Ms[(jj + 3) * KP + i], mv[jj + 3], a3);
      }
      for (; jj < R; ++jj) a0 = fmaf(Ms[jj * KP + i], mv[jj], a0);
      pv[i] = (a0 + a1) + (a2 + a3);
    }
    __syncthreads();
    if (on) {  // A^K m + z = D^K m - 2 W p + z
      float a0 = 0.f, a1 = 0.f;
      int s = 0;
      for (; s + 2 <= K; s += 2) {
        a0 = fmaf(Ws[s * R + i], pv[s], a0);
        a1 = fmaf(Ws[(s + 1) * R + i], pv[s + 1], a1);
      }
      for (; s < K; ++s) a0 = fmaf(Ws[s * R + i], pv[s], a0);
      m = fmaf(dk, m, zc) - 2.f * (a0 + a1);
    }
    zc = zn;
    __syncthreads();
  }
  if (on && m_out) m_out[(size_t)b * R + i] = m;
}

// The low-rank carry for R = 256, K = 64 with both factors in registers: the
// thread (s, q) = (tid / 4, tid % 4) holds M[s, j] for the channels j = q (mod 4)
// (64 values) and forms p_s with its three partners by two shuffles; the thread
// i holds row i of W (64 values) and applies D^K m - 2 W p + z for channel i.
// Each step reads m and p from shared memory (p as broadcast float4s) and
// needs two barriers.  Every thread copies its own channel's chunk end state z
// into an 8-deep shared ring by cp.async, seven chunks ahead, and waits only
// for its own copies.
__global__ void __launch_bounds__(256)
    rosa_carry_lowrank_reg_kernel(const float* __restrict__ Wt, const float* __restrict__ Mt,
                                  const float* __restrict__ DK, const float* __restrict__ z,
                                  const float* m0, float* __restrict__ m_start, float* m_out, int C) {
  constexpr int R = 256, K = 64, ZR = 8;
  __shared__ __align__(16) float mv[R];
  __shared__ __align__(16) float pv[K];
  __shared__ float zs[ZR][R];
  const int b = blockIdx.x, i = threadIdx.x;
  const int s = i >> 2, q = i & 3;
  float Mr[R / 4], Wc[K];
#pragma unroll
  for (int jj = 0; jj < R / 4; ++jj) Mr[jj] = Mt[(size_t)(4 * jj + q) * K + s];
#pragma unroll
  for (int ss = 0; ss < K; ++ss) Wc[ss] = Wt[(size_t)ss * R + i];
  const float dk = DK[i];
  float m = m0 ? m0[(size_t)b * R + i] : 0.f;
  const float* zb = z + (size_t)b * C * R + i;
  auto fetch = [&](int c) {  // this thread's z of chunk c into its ring slot; always commits
    if (c < C) {
      const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(&zs[c % ZR][i]));
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(zb + (size_t)c * R));
    }
    cp_async_commit();
  };
  for (int c = 0; c < ZR - 1; ++c) fetch(c);
  for (int c = 0; c < C; ++c) {
    fetch(c + ZR - 1);
    m_start[((size_t)b * C + c) * R + i] = m;
    mv[i] = m;
    __syncthreads();
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int jj = 0; jj < R / 4; jj += 4) {
      a0 = fmaf(Mr[jj + 0], mv[4 * (jj + 0) + q], a0);
      a1 = fmaf(Mr[jj + 1], mv[4 * (jj + 1) + q], a1);
      a2 = fmaf(Mr[jj + 2], mv[4 * (jj + 2) + q], a2);
      a3 = fmaf(Mr[jj + 3], mv[4 * (jj + 3) + q], a3);
    }
    float p = (a0 + a1) + (a2 + a3);
    p += __shfl_xor_sync(0xffffffffu, p, 1);
    p += __shfl_xor_sync(0xffffffffu, p, 2);
    if (q == 0) pv[s] = p;
    __syncthreads();
    float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f;
#pragma unroll
    for (int ss = 0; ss < K; ss += 4) {
      const float4 pp = *reinterpret_cast<const float4*>(pv + ss);
      w0 = fmaf(Wc[ss + 0], pp.x, w0);
      w1 = fmaf(Wc[ss + 1], pp.y, w1);
      w2 = fmaf(Wc[ss + 2], pp.z, w2);
      w3 = fmaf(Wc[ss + 3], pp.w, w3);
    }
    cp_async_wait<ZR - 1>();  // this thread's copy of chunk c has landed
    m = fmaf(dk, m, zs[c % ZR][i]) - 2.f * ((w0 + w1) + (w2 + w3));
  }
  cp_async_wait<0>();
  if (m_out) m_out[(size_t)b * R + i] = m;
}

static int sm_count_rosa() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      cudaGetLastError();
    return v > 0 ? v : 148;
  }();
  return n;
}

template <bool GATED, int MODE>
static void launch_mode(const float* cand, const float* write, const float* gate,
                        const float* bias_c, const float* bias_w, const float* bias_g, int ld,
                        const float* decay, const float* dir, int raw, const float* m0, float* read,
                        float* m_out, int B, int T, int R, const float* coef, cudaStream_t s) {
  const int threads = ((R + 31) / 32) * 32;
  // more blocks than two per SM: the register-light form, three blocks per SM
  if (B > 2 * sm_count_rosa())
    rosa_scan_kernel<GATED, false, 256, MODE, true><<<B, threads, 0, s>>>(
        cand, write, gate, decay, dir, m0, read, m_out, nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, T, R, ld, bias_c, bias_w, bias_g, raw, coef);
  else
    rosa_scan_kernel<GATED, false, 256, MODE><<<B, threads, 0, s>>>(
        cand, write, gate, decay, dir, m0, read, m_out, nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, T, R, ld, bias_c, bias_w, bias_g, raw, coef);
}

size_t rosa_parallel_scratch_floats(int B, int T, int R) {
  // A^K (R <= 128) or its low-rank factors W, M and D^K (2 K R + R <= R^2 for
  // R > 128, K = 64), then chunk end states and chunk start states
  const size_t C = (size_t)T / rosa_par_k(R);
  return (size_t)R * R + 2 * (size_t)B * C * R + ROSA_COEF_D + 2 * (size_t)R;
}

bool rosa_parallel_applies(int B, int T, int R) {
  // R within the 256-thread scan kernel, whole chunks, and enough of them to be
  // worth the extra passes
  const int K = rosa_par_k(R);
  return R <= 256 && T % K == 0 && T >= 4 * K && (long long)B * (T / K) >= 16;
}

// chunks per group of the two-level carry (R <= 128)
constexpr int ROSA_CARRY_G = 8;

size_t rosa_factor_floats(int R) {
  const size_t K = rosa_par_k(R);
  // R <= 128: A^K and A^(K G), both transposed
  return ROSA_COEF_D + 2 * (size_t)R + (R <= 128 ? 2 * (size_t)R * R : 2 * K * R + R);
}

// The layer constants of the time-parallel scan, from the raw parameters
// (raw != 0: decay = sigmoid(param), direction = normalize(householder)) or
// the post-activation ones: the coefficient block [q | d | decay]
// (ROSA_COEF_D + 2R floats), then A^K and A^(K G) transposed (R <= 128; the
// second for the two-level carry) or the factors W^T [K][R], M^T [R][K] and
// D^K [R] of A^K's low-rank form.  They depend on the layer's parameters only,
// so the engine builds them once per layer.
yuf_status_t rosa_prepare_factors(const float* decay, const float* dir, int raw, int R, float* out,
                                  cudaStream_t s) {
  if (R < 1 || R > 256) {
    set_error("rosa: time-parallel factors need 1 <= R <= 256 (R = %d)", R);
    return YUF_ERR_UNSUPPORTED;
  }
  const int K = rosa_par_k(R);
  float* coef = out;
  float* ak = out + ROSA_COEF_D + 2 * R;
  const int threads = ((R + 31) / 32) * 32;
  rosa_coef_kernel<<<1, threads, 0, s>>>(decay, dir, raw, R, coef);
  if (R <= 128) {
    // A^K and A^(K G) from R unit vectors (inputs unused in MODE 2)
    launch_mode<false, 2>(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, R, decay, dir, raw, nullptr,
                          nullptr, ak, R, K, R, coef, s);
    launch_mode<false, 2>(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, R, decay, dir, raw, nullptr,
                          nullptr, ak + (size_t)R * R, R, K * ROSA_CARRY_G, R, coef, s);
  } else {
    rosa_lowrank_kernel<<<1, threads, 0, s>>>(decay, dir, raw, ak, ak + (size_t)K * R, ak + 2 * (size_t)K * R, K,
                                              R);
  }
  return check_launch("rosa factors");
}

// The caller guarantees rosa_parallel_applies(); scratch holds
// rosa_parallel_scratch_floats() floats.  factors (nullable): the layer's
// rosa_prepare_factors() output for these parameters, which then are not
// rebuilt here.
yuf_status_t rosa_parallel(const float* cand, const float* write, const float* gate,
                           const float* bias_c, const float* bias_w, const float* bias_g, int ld,
                           const float* decay, const float* dir, int raw, const float* m0,
                           float* read, float* m_out, int B, int T, int R, bool gated,
                           float* scratch, cudaStream_t s, const float* factors) {
  const int K = rosa_par_k(R);
  const int C = T / K;
  float* AKt_s = scratch;
  float* z = AKt_s + (size_t)R * R;
  float* m_start = z + (size_t)B * C * R;
  float* coef_s = m_start + (size_t)B * C * R;  // q, d, dec of this layer
  if (!factors) {
    // build the layer constants into the scratch: coefficient block, then A^K
    // (or its low-rank factors) where the scratch keeps A^K
    const int threads = ((R + 31) / 32) * 32;
    rosa_coef_kernel<<<1, threads, 0, s>>>(decay, dir, raw, R, coef_s);
    if (R <= 128)
      launch_mode<false, 2>(cand, write, gate, nullptr, nullptr, nullptr, ld, decay, dir, raw, nullptr,
                            nullptr, AKt_s, R, K, R, coef_s, s);
    else
      rosa_lowrank_kernel<<<1, threads, 0, s>>>(decay, dir, raw, AKt_s, AKt_s + (size_t)K * R,
                                                AKt_s + 2 * (size_t)K * R, K, R);
  }
  const float* coef = factors ? factors : coef_s;
  const float* AKt = factors ? factors + ROSA_COEF_D + 2 * R : AKt_s;
  const int threads = ((R + 31) / 32) * 32;
  // 2. chunk end states from zero: chunks are the batch, K tokens each
  launch_mode<false, 1>(cand, write, gate, bias_c, bias_w, bias_g, ld, decay, dir, raw, nullptr,
                        nullptr, z, B * C, K, R, coef, s);
  // 3. carry across chunks
  constexpr int G = ROSA_CARRY_G;
  const int NG = C / G;
  if ((R == 32 || R == 64 || R == 128) && factors && C % G == 0 && NG >= 4 &&
      2LL * B * NG <= (long long)R) {
    // Two levels, depth 2 G + C / G instead of C: (a) every group of G chunks
    // from a zero state (its end state Zg), (b) per sequence the group start
    // states M_g+1 = A^(K G) M_g + Zg, (c) every group again from its true start,
    // writing the chunk start states.  Zg and M_g use the scratch's A^K area.
    const float* AKGt = AKt + (size_t)R * R;
    float* Zg = AKt_s;
    float* Mg = Zg + (size_t)B * NG * R;
    auto carry = [&](const float* A, const float* zz, const float* start, float* starts, float* end, int blocks,
                     int steps) {
      if (R == 32) rosa_carry_reg_kernel<32><<<blocks, 64, 0, s>>>(A, zz, start, starts, end, steps);
      else if (R == 64) rosa_carry_reg_kernel<64><<<blocks, 128, 0, s>>>(A, zz, start, starts, end, steps);
      else rosa_carry_reg_kernel<128><<<blocks, 256, 0, s>>>(A, zz, start, starts, end, steps);
    };
    carry(AKt, z, nullptr, m_start, Zg, B * NG, G);  // (a): the chunk starts written here are replaced in (c)
    carry(AKGt, Zg, m0, Mg, m_out, B, NG);           // (b)
    carry(AKt, z, Mg, m_start, nullptr, B * NG, G);  // (c)
  } else if (R == 32 || R == 64 || R == 128) {
    if (R == 32) rosa_carry_reg_kernel<32><<<B, 64, 0, s>>>(AKt, z, m0, m_start, m_out, C);
    else if (R == 64) rosa_carry_reg_kernel<64><<<B, 128, 0, s>>>(AKt, z, m0, m_start, m_out, C);
    else rosa_carry_reg_kernel<128><<<B, 256, 0, s>>>(AKt, z, m0, m_start, m_out, C);
  } else if (R <= 128) {
    const size_t sm = ((size_t)R * R + R) * sizeof(float);
    if (sm > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(rosa_carry_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e != cudaSuccess) {
        set_error("rosa: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        return YUF_ERR_CUDA;
      }
    }
    rosa_carry_kernel<<<B, threads, sm, s>>>(AKt, z, m0, m_start, m_out, C, R);
  } else {
    const float* Wt = AKt;                   // [K][R]
    const float* Mt = Wt + (size_t)K * R;    // [R][K]
    const float* DK = Mt + (size_t)R * K;    // [R]
    if (R == 256 && K == 64) {
      rosa_carry_lowrank_reg_kernel<<<B, 256, 0, s>>>(Wt, Mt, DK, z, m0, m_start, m_out, C);
    } else {
      const size_t sm = ((size_t)K * R + (size_t)R * K + R + K) * sizeof(float);
      cudaError_t e = cudaFuncSetAttribute(rosa_carry_lowrank_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      if (e != cudaSuccess) {
        set_error("rosa: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        return YUF_ERR_CUDA;
      }
      rosa_carry_lowrank_kernel<<<B, threads, sm, s>>>(Wt, Mt, DK, z, m0, m_start, m_out, C, K, R);
    }
  }
  // 4. rescan every chunk from its true start state
  if (gated)
    launch_mode<true, 0>(cand, write, gate, bias_c, bias_w, bias_g, ld, decay, dir, raw, m_start, read,
                         nullptr, B * C, K, R, coef, s);
  else
    launch_mode<false, 0>(cand, write, gate, bias_c, bias_w, bias_g, ld, decay, dir, raw, m_start, read,
                          nullptr, B * C, K, R, coef, s);
  return check_launch("rosa parallel scan");
}

}  // namespace yuf
