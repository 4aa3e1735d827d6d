// Single-token WKV-7 step (batched decode) for sm_100a.
//
// Same math as wkv7.cu for T = 1 (yufmusicgen/model.py:145-165 with one token,
// the stateful path the reference decode takes, model.py:193).  A decode step
// is a pure stream over the state: every (sequence, head) reads its N x N state
// once, updates it with one rank-2 correction and writes it back, so the
// kernel is built for bytes in flight rather than latency: small CTAs with few
// registers so many stay resident per SM, one resident wave of them looping over
// the (b, h) heads with the next head's state already loading while the current
// one is updated, state rows read and written as coalesced float2 runs (the 4
// lanes of a row cover it contiguously, a warp covers 8 consecutive rows), and
// the five shared per-token vectors (retention computed once per column) staged
// in double-buffered shared memory.

#include <algorithm>

#include "common.cuh"
#include "mbarrier.cuh"

namespace yuf {

template <int N>
__global__ void __launch_bounds__(N * 4)
    wkv7_decode_kernel(const float* __restrict__ r, const float* __restrict__ w,
                       const float* __restrict__ k, const float* __restrict__ v,
                       const float* __restrict__ a, const float* __restrict__ b, const float* s0,
                       float* __restrict__ y, float* s_out, int BH) {
  pdl_wait();
  pdl_trigger();
  constexpr int G = 4, C = N / G, C2 = C / 2;
  __shared__ float vec[2][5 * N];  // ret, k, a, b, r of the current and the next head
  const int tid = threadIdx.x;
  const int row = tid / G, g = tid - row * G, j0 = g * C;
  int bh = blockIdx.x;
  if (bh >= BH) return;

  float2 S[C2];
  float vi, pre[5];
  // issue the loads of head h's state row slice and token vectors (registers only)
  auto fetch = [&](int h, float2 (&S_)[C2], float& vi_, float (&p_)[5]) {
    const size_t o = (size_t)h * N;
    const size_t srow = (size_t)h * N * N + (size_t)row * N + j0;
#pragma unroll
    for (int c = 0; c < C2; ++c)
      S_[c] = s0 ? *reinterpret_cast<const float2*>(s0 + srow + 2 * c) : make_float2(0.f, 0.f);
    vi_ = v[o + row];
    if (tid < N) {
      p_[0] = w[o + tid];
      p_[1] = k[o + tid];
      p_[2] = a[o + tid];
      p_[3] = b[o + tid];
      p_[4] = r[o + tid];
    }
  };
  auto stage = [&](float* vs, const float (&p_)[5]) {
    if (tid < N) {
      vs[tid] = __expf(W_SCALE * sigmoidf_fast(p_[0]));
#pragma unroll
      for (int q = 1; q < 5; ++q) vs[q * N + tid] = p_[q];
    }
  };
  fetch(bh, S, vi, pre);
  stage(vec[0], pre);
  for (int it = 0;; ++it) {
    __syncthreads();  // vec[it & 1] staged; every thread is done with vec[(it + 1) & 1]
    const int nb = bh + gridDim.x;
    float2 Sn[C2];
    float vin = 0.f, pn[5];
    if (nb < BH) fetch(nb, Sn, vin, pn);  // next head's loads in flight during this one
    const float* vs = vec[it & 1];
    const float* W_ = vs + j0;
    const float* K_ = vs + N + j0;
    const float* A_ = vs + 2 * N + j0;
    const float* B_ = vs + 3 * N + j0;
    const float* R_ = vs + 4 * N + j0;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) acc = ffma2(S[c], *reinterpret_cast<const float2*>(A_ + 2 * c), acc);
    const float sa = group_sum<G>(acc.x + acc.y);
    float2 yacc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const float2 upd = ffma2(f2(sa), *reinterpret_cast<const float2*>(B_ + 2 * c),
                               fmul2(f2(vi), *reinterpret_cast<const float2*>(K_ + 2 * c)));
      S[c] = ffma2(S[c], *reinterpret_cast<const float2*>(W_ + 2 * c), upd);
      yacc = ffma2(S[c], *reinterpret_cast<const float2*>(R_ + 2 * c), yacc);
    }
    const float yv = group_sum<G>(yacc.x + yacc.y);
    const size_t o = (size_t)bh * N;
    if (g == 0) y[o + row] = yv;
    if (s_out) {
      const size_t srow = (size_t)bh * N * N + (size_t)row * N + j0;
#pragma unroll
      for (int c = 0; c < C2; ++c) *reinterpret_cast<float2*>(s_out + srow + 2 * c) = S[c];
    }
    if (nb >= BH) break;
    stage(vec[(it + 1) & 1], pn);
#pragma unroll
    for (int c = 0; c < C2; ++c) S[c] = Sn[c];
    vi = vin;
    bh = nb;
  }
}

// ---- bulk-copy (TMA) ring variant --------------------------------------------
// Each CTA owns a ring of STAGES shared-memory slots, one head per slot: the
// head's N x N state (N*N*4 contiguous bytes) and its six token vectors
// (r, w, k, v, a, b: N*4 bytes each) arrive by 1-D bulk copies on the slot's
// mbarrier; the CTA updates the state in shared memory and one thread writes it
// back with a bulk store.  STAGES-1 heads are in flight while one is computed,
// and the copies move whole contiguous blocks, so the kernel streams at close
// to copy bandwidth instead of waiting on per-thread load latency.
template <int N, bool TM = false>
struct DecRing {
  static constexpr int STATE_BYTES = N * N * 4;
  static constexpr int VEC_BYTES = N * 4;
  // state, r, w, k, v, a, b; TM: state, r, lw, k, v, la, lg, then the head's
  // w0, a0, k_k, k_a
  static constexpr int NVEC = TM ? 10 : 6;
  static constexpr int SLOT = STATE_BYTES + NVEC * VEC_BYTES;
  static constexpr int STAGES = SLOT * 4 <= 96 * 1024 ? 4 : (SLOT * 3 <= 128 * 1024 ? 3 : 2);
  static constexpr int EXTRA = (TM ? 6 * N + 16 : N) * 4;  // retention; the time-mix scratch
  static constexpr int SMEM = STAGES * SLOT + EXTRA + STAGES * 8;  // slots, scratch, barriers
  static_assert(SLOT % 16 == 0 && VEC_BYTES % 16 == 0, "bulk copies need 16-byte multiples");
  static_assert(N % 8 == 0, "N * 4 threads in whole warps");
};

__device__ unsigned int g_decode_wait_timeouts;

// The time-mix epilogue of the head, folded in (TM): the slot's vectors are
// then r, the w / a / g low-rank outputs, k and v as the projections left them,
// and each head first forms (yufmusicgen/model.py:113-125)
//   w = w0 + lw,  kk = normalize(k * k_k),  alpha = sigmoid(a0 + la),
//   a = -kk,  b = kk * alpha,  k' = k * (1 + (alpha - 1) * k_a),  g = sigmoid(lg)
// (g to global for the output gate), the arithmetic of timemix_post_kernel.
struct DecTm {
  const float *w0, *a0, *k_k, *k_a;  // [H * N] per-channel parameters
  float* g;                          // [BH * N] output gate
  int H;
};

template <int N, bool TM>
__global__ void __launch_bounds__(N * 4)
    wkv7_decode_ring_kernel(const float* __restrict__ r, const float* __restrict__ w,
                            const float* __restrict__ k, const float* __restrict__ v,
                            const float* __restrict__ a, const float* __restrict__ b,
                            const float* s0, float* __restrict__ y, float* s_out, int BH, const DecTm tm) {
  pdl_wait();
  pdl_trigger();
  using K = DecRing<N, TM>;
  constexpr int G = 4, C = N / G, C2 = C / 2;
  extern __shared__ __align__(128) unsigned char dsm[];
  float* ret = reinterpret_cast<float*>(dsm + K::STAGES * K::SLOT);
  float* tmv = ret + N;                 // TM: a, b, k', kk, alpha (N each), the warps' partial norms
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + K::STAGES * K::SLOT + K::EXTRA);
  const int tid = threadIdx.x;
  const int row = tid / G, g = tid - row * G, j0 = g * C;
  const int first = blockIdx.x, stride = gridDim.x;
  const int nheads = first < BH ? (BH - 1 - first) / stride + 1 : 0;
  if (nheads == 0) return;

  const float* vsrc[6] = {r, w, k, v, a, b};
  auto issue = [&](int j) {  // thread 0: head j of this CTA into slot j % STAGES
    const int sl = j % K::STAGES;
    const size_t bh = (size_t)first + (size_t)j * stride;
    unsigned char* slot = dsm + sl * K::SLOT;
    mbar_expect_tx(&full[sl], K::SLOT);
    bulk_load(slot, s0 + bh * N * N, K::STATE_BYTES, &full[sl]);
#pragma unroll
    for (int q = 0; q < 6; ++q)
      bulk_load(slot + K::STATE_BYTES + q * K::VEC_BYTES, vsrc[q] + bh * N, K::VEC_BYTES, &full[sl]);
    if constexpr (TM) {
      const size_t c0 = (size_t)((int)bh % tm.H) * N;
      const float* psrc[4] = {tm.w0, tm.a0, tm.k_k, tm.k_a};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        bulk_load(slot + K::STATE_BYTES + (6 + q) * K::VEC_BYTES, psrc[q] + c0, K::VEC_BYTES, &full[sl]);
    }
  };
  if (tid == 0) {
    for (int sl = 0; sl < K::STAGES; ++sl) mbar_init(&full[sl], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // thread 0: heads whose copies were started
  if (tid == 0)
    for (; issued < min(nheads, K::STAGES); ++issued) issue(issued);

  for (int j = 0; j < nheads; ++j) {
    const int sl = j % K::STAGES;
    const bool ok = mbar_wait(&full[sl], (uint32_t)(j / K::STAGES) & 1u);
    if (__syncthreads_or(!ok)) {  // a copy never landed: record it, leave together
      if (tid == 0) {
        atomicAdd(&g_decode_wait_timeouts, 1u);
        bulk_wait_all();
        // give the loads still in flight into this CTA's slots a bounded chance to land
        for (int h = j; h < issued; ++h) mbar_wait(&full[h % K::STAGES], (uint32_t)(h / K::STAGES) & 1u);
      }
      return;
    }
    float* St = reinterpret_cast<float*>(dsm + sl * K::SLOT);
    const float* vec = St + N * N;  // r, w, k, v, a, b (TM: r, lw, k, v, la, lg)
    const float* K_ = vec + 2 * N + j0;
    const float* A_ = vec + 4 * N + j0;
    const float* B_ = vec + 5 * N + j0;
    if constexpr (TM) {
      const int bh = first + j * stride;
      const float* prm = vec + 6 * N;  // the head's w0, a0, k_k, k_a
      float kk2 = 0.f;  // this column's |kk|^2 term; 0 past the N columns
      if (tid < N) {
        const float kv = vec[2 * N + tid];
        const float kk = kv * prm[2 * N + tid];
        const float alpha = sigmoidf_fast(prm[N + tid] + vec[4 * N + tid]);
        ret[tid] = __expf(W_SCALE * sigmoidf_fast(prm[tid] + vec[N + tid]));
        tmv[2 * N + tid] = kv * (1.f + (alpha - 1.f) * prm[3 * N + tid]);  // k'
        tmv[3 * N + tid] = kk;                                      // kk before the norm
        tmv[4 * N + tid] = alpha;
        tm.g[(size_t)bh * N + tid] = sigmoidf_fast(vec[5 * N + tid]);
        kk2 = kk * kk;
      }
      // every thread of the CTA in the butterfly (no branch around it), one
      // partial per warp
      kk2 = group_sum<32>(kk2);
      if ((tid & 31) == 0) tmv[5 * N + (tid >> 5)] = kk2;
      __syncthreads();
      if (tid < N) {
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < N / 8; ++q) sum += tmv[5 * N + q];  // the N * 4 / 32 warps' partials
        const float inv = 1.f / fmaxf(sqrtf(sum), 1e-12f);  // F.normalize eps (model.py:116)
        const float kk = tmv[3 * N + tid] * inv;
        tmv[tid] = -kk;                         // a
        tmv[N + tid] = kk * tmv[4 * N + tid];  // b
      }
      __syncthreads();
      K_ = tmv + 2 * N + j0;
      A_ = tmv + j0;
      B_ = tmv + N + j0;
    } else {
      if (tid < N) ret[tid] = __expf(W_SCALE * sigmoidf_fast(vec[N + tid]));
      __syncthreads();
    }
    const float* W_ = ret + j0;
    const float* R_ = vec + j0;
    const float vi = vec[3 * N + row];
    float* Srow = St + row * N + j0;
    float2 S[C2];
#pragma unroll
    for (int c = 0; c < C2; ++c) S[c] = *reinterpret_cast<const float2*>(Srow + 2 * c);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) acc = ffma2(S[c], *reinterpret_cast<const float2*>(A_ + 2 * c), acc);
    const float sa = group_sum<G>(acc.x + acc.y);
    float2 yacc = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < C2; ++c) {
      const float2 upd = ffma2(f2(sa), *reinterpret_cast<const float2*>(B_ + 2 * c),
                               fmul2(f2(vi), *reinterpret_cast<const float2*>(K_ + 2 * c)));
      S[c] = ffma2(S[c], *reinterpret_cast<const float2*>(W_ + 2 * c), upd);
      yacc = ffma2(S[c], *reinterpret_cast<const float2*>(R_ + 2 * c), yacc);
      *reinterpret_cast<float2*>(Srow + 2 * c) = S[c];
    }
    const float yv = group_sum<G>(yacc.x + yacc.y);
    const size_t bh = (size_t)first + (size_t)j * stride;
    if (g == 0) y[bh * N + row] = yv;
    fence_proxy_async();  // the state writes above feed the bulk store below
    __syncthreads();
    if (tid == 0) {
      bulk_store(s_out + bh * N * N, St, K::STATE_BYTES);
      bulk_commit();
      // refill the previous head's slot once its store has read it
      if (j >= 1 && j - 1 + K::STAGES < nheads) {
        bulk_wait_read<1>();
        issue(issued++);
      }
    }
  }
  if (tid == 0) bulk_wait_all();
}

// Timeouts of the ring kernel's bounded waits since the last call; clears them.
unsigned int wkv7_decode_wait_timeouts() {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g_decode_wait_timeouts, sizeof(n)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_decode_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return ~0u;
  }
  return n;
}

// Resident ring CTAs per SM for head size N on the current device (0: the ring
// cannot run); sets the kernel's shared-memory limit on first use per device.
template <int N, bool TM>
static int ring_blocks_per_sm() {
  static int cache[64];  // per device: blocks + 1, 0 = not yet known
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 0;
  }
  if (cache[dev]) return cache[dev] - 1;
  int v = 0;
  if (cudaFuncSetAttribute(wkv7_decode_ring_kernel<N, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DecRing<N, TM>::SMEM) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, wkv7_decode_ring_kernel<N, TM>, N * 4,
                                                    DecRing<N, TM>::SMEM) != cudaSuccess) {
    cudaGetLastError();
    v = 0;
  }
  cache[dev] = v + 1;
  return v;
}

// Resident CTAs per SM of the decode kernel for head size N (cached).
template <int N>
static int decode_blocks_per_sm() {
  static int n = [] {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, wkv7_decode_kernel<N>, N * 4, 0) !=
            cudaSuccess ||
        v < 1)
      v = 1;
    return v;
  }();
  return n;
}

static int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// Set the ring kernel's shared-memory limit and cache its occupancy for head
// size N; the engine calls this before capturing decode graphs.
void wkv7_decode_prepare(int N) {
  switch (N) {
    case 16: ring_blocks_per_sm<16, false>(); ring_blocks_per_sm<16, true>(); break;
    case 32: ring_blocks_per_sm<32, false>(); ring_blocks_per_sm<32, true>(); break;
    case 40: ring_blocks_per_sm<40, false>(); ring_blocks_per_sm<40, true>(); break;
    case 48: ring_blocks_per_sm<48, false>(); ring_blocks_per_sm<48, true>(); break;
    case 64: ring_blocks_per_sm<64, false>(); ring_blocks_per_sm<64, true>(); break;
    case 96: ring_blocks_per_sm<96, false>(); ring_blocks_per_sm<96, true>(); break;
    case 128: ring_blocks_per_sm<128, false>(); ring_blocks_per_sm<128, true>(); break;
    default: break;
  }
  sm_count();
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid: one resident wave of CTAs, each looping over heads bh, bh + grid, ...
// The bulk-copy ring when the buffers allow it, else the register-prefetch loop.
yuf_status_t wkv7_decode_dispatch(const float* r, const float* w, const float* k, const float* v,
                                  const float* a, const float* b, const float* s0, float* y,
                                  float* s_out, int BH, int N, cudaStream_t stream) {
  if (BH <= 0) return YUF_OK;
  // the ring needs a state to read and write, all on 16-byte boundaries
  const bool ring = s0 && s_out && aligned16(s0) && aligned16(s_out) && aligned16(r) &&
                    aligned16(w) && aligned16(k) && aligned16(v) && aligned16(a) && aligned16(b);
  switch (N) {
#define CASE(NN)                                                                                 \
  case NN: {                                                                                     \
    const int per_sm = ring ? ring_blocks_per_sm<NN, false>() : 0;                               \
    if (per_sm > 0) {                                                                            \
      const int grid = std::min(BH, per_sm * sm_count());                                        \
      launch_k(wkv7_decode_ring_kernel<NN, false>, dim3(grid), dim3(NN * 4), DecRing<NN>::SMEM, stream,            \
          r, w, k, v, a, b, s0, y, s_out, BH, DecTm{});                                          \
      return check_launch("wkv7_decode_ring_kernel");                                            \
    }                                                                                            \
    const int grid = std::min(BH, decode_blocks_per_sm<NN>() * sm_count());                     \
    launch_k(wkv7_decode_kernel<NN>, dim3(grid), dim3(NN * 4), 0, stream, r, w, k, v, a, b, s0, y, s_out, BH);    \
    return check_launch("wkv7_decode_kernel");                                                   \
  }
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      set_error("wkv7: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

// The decode step with the time-mix epilogue folded in: r, k, v and the w / a /
// g low-rank outputs as the projections left them ([BH, N] rows), the layer's
// per-channel w0, a0, k_k, k_a ([H * N]); writes y, the state and the output
// gate g.  YUF_ERR_UNSUPPORTED when the bulk-copy ring cannot run (a buffer off
// a 16-byte boundary, no state, no occupancy): the caller then takes the
// separate epilogue kernel and wkv7_decode_dispatch.
yuf_status_t wkv7_decode_tm_dispatch(const float* r, const float* k, const float* v, const float* lw,
                                     const float* la, const float* lg, const float* w0, const float* a0,
                                     const float* k_k, const float* k_a, float* g, const float* s0, float* y,
                                     float* s_out, int BH, int H, int N, cudaStream_t stream) {
  if (BH <= 0) return YUF_OK;
  const bool ring = s0 && s_out && H > 0 && BH % H == 0 && aligned16(s0) && aligned16(s_out) && aligned16(r) &&
                    aligned16(k) && aligned16(v) && aligned16(lw) && aligned16(la) && aligned16(lg) &&
                    aligned16(w0) && aligned16(a0) && aligned16(k_k) && aligned16(k_a);
  if (!ring) return YUF_ERR_UNSUPPORTED;
  const DecTm tm{w0, a0, k_k, k_a, g, H};
  switch (N) {
#define CASE(NN)                                                                                 \
  case NN: {                                                                                     \
    const int per_sm = ring_blocks_per_sm<NN, true>();                                           \
    if (per_sm <= 0) return YUF_ERR_UNSUPPORTED;                                                 \
    const int grid = std::min(BH, per_sm * sm_count());                                          \
    launch_k(wkv7_decode_ring_kernel<NN, true>, dim3(grid), dim3(NN * 4), DecRing<NN, true>::SMEM, stream, r, lw, k, v, \
             la, lg, s0, y, s_out, BH, tm);                                                      \
    return check_launch("wkv7_decode_ring_kernel (time-mix)");                                   \
  }
    CASE(16) CASE(32) CASE(40) CASE(48) CASE(64) CASE(96) CASE(128)
#undef CASE
    default:
      return YUF_ERR_UNSUPPORTED;
  }
}

}  // namespace yuf
