// Row-split sequential WKV-7 scan (prefill) for sm_100a.
//
// Every state row is an independent recurrence (yufmusicgen/model.py:158-164):
//   sa_i = sum_j a_j S_ij,   S_ij <- S_ij w_j + sa_i b_j + v_i k_j,   y_i = sum_j S_ij r_j,
// so a (sequence, head) chain is a bundle of N recurrences that share their
// per-token column vectors.  One CTA per chain: N / (8 R) scan warps, each row
// held by a group of 4 lanes (N / 4 columns each, R rows per lane group, the
// state in registers as fp32x2 pairs), plus one producer warp.  The time axis
// is walked token by token; what bounds a token is the dependency chain
//   sa_t (a 4-lane dot product) -> S' += sa_t b'_t -> sa_{t+1} ...,
// not arithmetic or bytes, so the chain is kept short:
//   * decay-scaled state: inside a group of TS = 8 tokens the lanes carry
//     S'_t = S_t / gamma_t (gamma_t = w_1 ... w_t since the group began), so the
//     update has no decay product, S'_t = S'_{t-1} + sa_t b'_t + v_t k'_t with
//     b' = b / gamma_t, k' = k / gamma_t, sa_t = S'_{t-1} (gamma_{t-1} a_t),
//     y_t = S'_t (gamma_t r_t); the value term does not wait for sa; at the
//     group end S = S' gamma_end (gamma >= 0.545^8, 1 / gamma <= 128);
//   * the producer warp stages each group with six TMA boxes (one per input,
//     the head's N columns x 8 tokens) into a ring of slots and turns the raw
//     rows into the scaled vectors, in the lanes' padded layout, ahead of the
//     scan warps (full / ready / empty mbarriers per slot; every wait bounded).
// Inputs are read once, y written once, the state in and out once: the bytes of
// the op and nothing more (no chunk summaries, no second pass over y).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "mbarrier.cuh"
#include "tma.cuh"

namespace yuf {

__device__ unsigned int g_rows_wait_timeouts;

template <int N>
struct RowsCfg {
  static constexpr int G = 4;                          // lanes per row
  static constexpr int C = N / G;                      // columns per lane
  static constexpr int C2 = C / 2;
  static constexpr int R = N >= 96 ? 2 : 1;            // rows per lane group
  static constexpr int NWS = N / (8 * R);              // scan warps
  static constexpr int NT = 32 * (NWS + 1);            // + the producer warp
  static constexpr int TS = 8;                         // tokens per staged group
  static constexpr int NR = N >= 96 ? 3 : (N >= 64 ? 4 : 6);  // raw slots: groups loaded ahead
  static constexpr int NB = 4;                         // scaled slots
  static constexpr int CS = conflict_free_stride(C, G);
  static constexpr int VP = G * CS;                    // padded vector length
  // raw slot (floats): [6][TS][N], the TMA destination
  static constexpr int RAW_SLOT = 6 * TS * N;
  // scaled slot (floats): a', b', k', r' [4][TS][VP], v [TS][N], gamma_end [VP]
  static constexpr int SV = 4 * TS * VP;
  static constexpr int SGEND = SV + TS * N;
  static constexpr int SC_SLOT = (SGEND + VP + 31) / 32 * 32;  // 128-byte multiple
  static constexpr int SCALED = NR * RAW_SLOT;
  static constexpr int BAR = SCALED + NB * SC_SLOT;            // NR + 2 NB mbarriers
  static constexpr size_t BYTES = (size_t)BAR * 4 + (NR + 2 * NB) * 8 + 128;
  static constexpr uint32_t TX = 6u * TS * N * 4;
  static_assert(N % 8 == 0 && C % 2 == 0 && NWS * 8 * R == N, "rows kernel: N in {16, 32, 40, 48, 64, 96, 128}");
  static_assert((TS * N * 4) % 128 == 0, "TMA boxes land on 128-byte boundaries");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

struct RowsTmaps {
  CUtensorMap m[6];  // r, w, k, v, a, b
};

template <int N>
__global__ void __launch_bounds__(RowsCfg<N>::NT, 1)
    wkv7_rows_kernel(const float* __restrict__ s0, float* __restrict__ y, float* __restrict__ s_out, int T,
                     int H, const __grid_constant__ RowsTmaps tm) {
  using K = RowsCfg<N>;
  constexpr int C = K::C, C2 = K::C2, R = K::R, TS = K::TS, NB = K::NB, NR = K::NR, CS = K::CS, VP = K::VP;
  extern __shared__ __align__(128) float rows_smem[];
  float* sm = rows_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + K::BAR);  // [NR] raw boxes landed
  uint64_t* ready = full + NR;                                // [NB] scaled slot filled
  uint64_t* empty = ready + NB;                               // [NB] scaled slot consumed
  __shared__ int abort_flag;

  const int bh = blockIdx.x;
  const int bb = bh / H, hh = bh - bb * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = (T + TS - 1) / TS;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NR; ++s) mbar_init(&full[s], 1);
    for (int s = 0; s < NB; ++s) {
      mbar_init(&ready[s], 1);
      mbar_init(&empty[s], K::NWS);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  if (warp == K::NWS) {  // ------------------------------------------------- producer
    const int tx = hh * N, ty = bb * T;
    auto issue = [&](int gi) {  // lane 0: the six boxes of group gi into raw slot gi % NR
      float* Rw = sm + (gi % NR) * K::RAW_SLOT;
      uint64_t* bar = &full[gi % NR];
      mbar_expect_tx(bar, K::TX);
#pragma unroll
      for (int arr = 0; arr < 6; ++arr) tma_load_2d(Rw + arr * TS * N, &tm.m[arr], bar, tx, ty + gi * TS);
    };
    int issued = 0;
    if (lane == 0)
      for (; issued < min(NR, ngroups); ++issued) issue(issued);
    issued = __shfl_sync(0xffffffffu, issued, 0);
    for (int gi = 0; gi < ngroups; ++gi) {
      const int rs = gi % NR, ss = gi % NB;
      bool ok = mbar_wait(&full[rs], (uint32_t)(gi / NR) & 1u) && mbar_wait(&empty[ss], ((uint32_t)(gi / NB) & 1u) ^ 1u);
      ok = __all_sync(0xffffffffu, ok) && !*(volatile int*)&abort_flag;
      if (!ok) { abort_flag = 1; break; }
      const float* Rw = sm + rs * K::RAW_SLOT;
      float* Sc = sm + K::SCALED + ss * K::SC_SLOT;
      const int Tc = min(TS, T - gi * TS);
      // scaled vectors, a lane per column pair, gamma running over the group; v copied
      for (int jp = lane; jp < N / 2; jp += 32) {
        const int j = 2 * jp;
        const int pj = (j / C) * CS + (j % C);
        float2 gam = make_float2(1.f, 1.f), ginv = gam;
        for (int t = 0; t < Tc; ++t) {
          const int rj = t * N + j;
          const float2 wr = *reinterpret_cast<const float2*>(Rw + 1 * TS * N + rj);
          const float sx = W_SCALE * sigmoidf_fast(wr.x), sy = W_SCALE * sigmoidf_fast(wr.y);
          const float2 av = *reinterpret_cast<const float2*>(Rw + 4 * TS * N + rj);
          const float2 bv = *reinterpret_cast<const float2*>(Rw + 5 * TS * N + rj);
          const float2 kv = *reinterpret_cast<const float2*>(Rw + 2 * TS * N + rj);
          const float2 rv = *reinterpret_cast<const float2*>(Rw + 0 * TS * N + rj);
          float* d = Sc + t * VP + pj;
          *reinterpret_cast<float2*>(d + 0 * TS * VP) = fmul2(av, gam);  // gamma_{t-1} a_t
          gam = fmul2(gam, make_float2(__expf(sx), __expf(sy)));
          ginv = fmul2(ginv, make_float2(__expf(-sx), __expf(-sy)));
          *reinterpret_cast<float2*>(d + 1 * TS * VP) = fmul2(bv, ginv);  // b_t / gamma_t
          *reinterpret_cast<float2*>(d + 2 * TS * VP) = fmul2(kv, ginv);  // k_t / gamma_t
          *reinterpret_cast<float2*>(d + 3 * TS * VP) = fmul2(rv, gam);   // gamma_t r_t
          *reinterpret_cast<float2*>(Sc + K::SV + rj) = *reinterpret_cast<const float2*>(Rw + 3 * TS * N + rj);
        }
        *reinterpret_cast<float2*>(Sc + K::SGEND + pj) = gam;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ready[ss]);
        if (issued < ngroups) {  // the raw slot is free again: load the group NR ahead into it
          fence_proxy_async();
          issue(issued);
        }
      }
      issued = min(issued + 1, max(issued, ngroups));
      issued = __shfl_sync(0xffffffffu, issued, 0);
    }
    if (lane == 0 && *(volatile int*)&abort_flag)  // let boxes still in flight land before leaving
      for (int g2 = 0; g2 < NR; ++g2) {
        const int gl = issued - 1 - g2;  // the last NR groups issued
        if (gl < 0) break;
        mbar_wait(&full[gl % NR], (uint32_t)(gl / NR) & 1u);
      }
  } else {  // ---------------------------------------------------------- scan warps
    const int rg = lane >> 2, g = lane & 3;
    const int i0 = (warp * 8 + rg) * R, j0 = g * C;
    const size_t srow0 = (size_t)bh * N * N;
    float2 Sx[R][C2];
#pragma unroll
    for (int p = 0; p < R; ++p)
#pragma unroll
      for (int c = 0; c < C2; ++c)
        Sx[p][c] = s0 ? *reinterpret_cast<const float2*>(s0 + srow0 + (size_t)(i0 + p) * N + j0 + 2 * c)
                      : make_float2(0.f, 0.f);
    const size_t tok_stride = (size_t)H * N;
    float* ybase = y + ((size_t)bb * T * H + hh) * N + i0;
    for (int gi = 0; gi < ngroups; ++gi) {
      const int ss = gi % NB;
      bool ok = __all_sync(0xffffffffu, mbar_wait(&ready[ss], (uint32_t)(gi / NB) & 1u));
      if (!ok || *(volatile int*)&abort_flag) { abort_flag = 1; break; }
      const float* Sc = sm + K::SCALED + ss * K::SC_SLOT;
      const float* Pa = Sc + 0 * TS * VP + g * CS;
      const float* Pb = Sc + 1 * TS * VP + g * CS;
      const float* Pk = Sc + 2 * TS * VP + g * CS;
      const float* Pr = Sc + 3 * TS * VP + g * CS;
      const float* Pv = Sc + K::SV + i0;
      const int Tc = min(TS, T - gi * TS);
      // sa of the group's first token (the state enters the group unscaled)
      float sa[R];
      {
        float2 av[C2];
#pragma unroll
        for (int c = 0; c < C2; ++c) av[c] = *reinterpret_cast<const float2*>(Pa + 2 * c);
#pragma unroll
        for (int p = 0; p < R; ++p) {
          float2 u0 = make_float2(0.f, 0.f), u1 = u0;
#pragma unroll
          for (int c = 0; c < C2; ++c) {
            if (c & 1) u1 = ffma2(Sx[p][c], av[c], u1);
            else u0 = ffma2(Sx[p][c], av[c], u0);
          }
          sa[p] = (u0.x + u1.x) + (u0.y + u1.y);
        }
#pragma unroll
        for (int p = 0; p < R; ++p) {
          sa[p] += __shfl_xor_sync(0xffffffffu, sa[p], 1);
          sa[p] += __shfl_xor_sync(0xffffffffu, sa[p], 2);
        }
      }
#pragma unroll
      for (int t = 0; t < TS; ++t) {
        if (t < Tc) {
          const int o = t * VP;
          float2 bv[C2], kv[C2], rv[C2], an[C2];
#pragma unroll
          for (int c = 0; c < C2; ++c) {
            bv[c] = *reinterpret_cast<const float2*>(Pb + o + 2 * c);
            kv[c] = *reinterpret_cast<const float2*>(Pk + o + 2 * c);
            rv[c] = *reinterpret_cast<const float2*>(Pr + o + 2 * c);
            an[c] = *reinterpret_cast<const float2*>(Pa + o + VP + 2 * c);  // a' of token t + 1
          }
          float vr[R];
#pragma unroll
          for (int p = 0; p < R; ++p) vr[p] = Pv[t * N + p];
          float yo[R];
#pragma unroll
          for (int p = 0; p < R; ++p) {
            float2 y0 = make_float2(0.f, 0.f), y1 = y0, u0 = y0, u1 = y0;
#pragma unroll
            for (int c = 0; c < C2; ++c) {
              Sx[p][c] = ffma2(f2(sa[p]), bv[c], ffma2(f2(vr[p]), kv[c], Sx[p][c]));
              if (c & 1) {
                y1 = ffma2(Sx[p][c], rv[c], y1);
                u1 = ffma2(Sx[p][c], an[c], u1);
              } else {
                y0 = ffma2(Sx[p][c], rv[c], y0);
                u0 = ffma2(Sx[p][c], an[c], u0);
              }
            }
            yo[p] = (y0.x + y1.x) + (y0.y + y1.y);
            sa[p] = (u0.x + u1.x) + (u0.y + u1.y);
          }
#pragma unroll
          for (int p = 0; p < R; ++p) {
            sa[p] += __shfl_xor_sync(0xffffffffu, sa[p], 1);
            yo[p] += __shfl_xor_sync(0xffffffffu, yo[p], 1);
            sa[p] += __shfl_xor_sync(0xffffffffu, sa[p], 2);
            yo[p] += __shfl_xor_sync(0xffffffffu, yo[p], 2);
          }
          if (g < R) {
            float v = yo[0];
#pragma unroll
            for (int p = 1; p < R; ++p)
              if (g == p) v = yo[p];
            ybase[(size_t)(gi * TS + t) * tok_stride + g] = v;
          }
        }
      }
      // back to the unscaled state: S = S' gamma_end
      {
        float2 ge[C2];
#pragma unroll
        for (int c = 0; c < C2; ++c) ge[c] = *reinterpret_cast<const float2*>(Sc + K::SGEND + g * CS + 2 * c);
#pragma unroll
        for (int p = 0; p < R; ++p)
#pragma unroll
          for (int c = 0; c < C2; ++c) Sx[p][c] = fmul2(Sx[p][c], ge[c]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[ss]);
    }
    if (s_out && !*(volatile int*)&abort_flag) {
#pragma unroll
      for (int p = 0; p < R; ++p)
#pragma unroll
        for (int c = 0; c < C2; ++c)
          *reinterpret_cast<float2*>(s_out + srow0 + (size_t)(i0 + p) * N + j0 + 2 * c) = Sx[p][c];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicAdd(&g_rows_wait_timeouts, 1u);
}

// Tensor maps of the six [B*T, H*N] inputs, box = N columns x TS rows.
static yuf_status_t make_rows_tmaps(const float* const (&src)[6], long long rows, int H, int N, RowsTmaps* out) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    set_error("wkv7 rows: cuTensorMapEncodeTiled is unavailable");
    return YUF_ERR_CUDA;
  }
  const cuuint64_t gdim[2] = {(cuuint64_t)H * N, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)H * N * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)N, 8u};
  const cuuint32_t estride[2] = {1u, 1u};
  for (int i = 0; i < 6; ++i) {
    const CUresult rc = enc(&out->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(src[i]), gdim,
                            gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
      set_error("wkv7 rows: cuTensorMapEncodeTiled failed (%d) for input %d", (int)rc, i);
      return YUF_ERR_CUDA;
    }
  }
  return YUF_OK;
}

template <int N>
static yuf_status_t launch_rows(const float* const (&src)[6], const float* s0, float* y, float* s_out, int B,
                                int T, int H, cudaStream_t st) {
  using K = RowsCfg<N>;
  static std::once_flag once[128];
  static cudaError_t attr[128];
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  std::call_once(once[dev], [&] {
    attr[dev] = cudaFuncSetAttribute(wkv7_rows_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::BYTES);
  });
  if (attr[dev] != cudaSuccess) {
    set_error("wkv7 rows: cannot set %zu bytes of shared memory: %s", K::BYTES, cudaGetErrorString(attr[dev]));
    return YUF_ERR_CUDA;
  }
  RowsTmaps tm;
  const yuf_status_t rc = make_rows_tmaps(src, (long long)B * T, H, N, &tm);
  if (rc != YUF_OK) return rc;
  launch_k(wkv7_rows_kernel<N>, dim3(B * H), dim3(K::NT), K::BYTES, st, s0, y, s_out, T, H, tm);
  return check_launch("wkv7_rows_kernel");
}

// Row-split sequential scan of [B, T, H, N] inputs from s0 (nullable), writing
// y and the final state (nullable).  Inputs 16-byte aligned.
yuf_status_t wkv7_rows(const float* r, const float* w, const float* k, const float* v, const float* a,
                       const float* b, const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                       cudaStream_t st) {
  if (T == 0) {  // no tokens: the final state is the initial one
    if (!s_out || s_out == s0) return YUF_OK;
    const size_t bytes = (size_t)B * H * N * N * sizeof(float);
    const cudaError_t e = s0 ? cudaMemcpyAsync(s_out, s0, bytes, cudaMemcpyDeviceToDevice, st)
                             : cudaMemsetAsync(s_out, 0, bytes, st);
    if (e != cudaSuccess) {
      set_error("wkv7 rows: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
    return YUF_OK;
  }
  const float* const src[6] = {r, w, k, v, a, b};
  switch (N) {
    case 16: return launch_rows<16>(src, s0, y, s_out, B, T, H, st);
    case 32: return launch_rows<32>(src, s0, y, s_out, B, T, H, st);
    case 40: return launch_rows<40>(src, s0, y, s_out, B, T, H, st);
    case 48: return launch_rows<48>(src, s0, y, s_out, B, T, H, st);
    case 64: return launch_rows<64>(src, s0, y, s_out, B, T, H, st);
    case 96: return launch_rows<96>(src, s0, y, s_out, B, T, H, st);
    case 128: return launch_rows<128>(src, s0, y, s_out, B, T, H, st);
    default:
      set_error("wkv7 rows: head size N=%d has no kernel", N);
      return YUF_ERR_UNSUPPORTED;
  }
}

unsigned int wkv7_rows_wait_timeouts() {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g_rows_wait_timeouts, sizeof(n)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_rows_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return ~0u;
  }
  return n;
}

}  // namespace yuf
