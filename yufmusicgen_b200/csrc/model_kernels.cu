// Elementwise / row kernels of the YufMusicGen block on sm_100a.
//
// Every kernel follows one formula of the reference block
// (yufmusicgen/model.py:97-131, 195-197, 290-342, 365-422) and fuses what the
// reference runs as separate ATen passes: the six token-shift mixes in one
// pass over the LayerNorm output (model.py:98-105), the w/a/g activations with
// the per-head kk normalisation and the key adjustment (model.py:108-122), the
// output LayerNorm with the gate multiply (model.py:196), SiLU(in)*gate
// (model.py:377).  Rows are tokens; one warp per row for the d-wide reductions.

#include "model_kernels.cuh"

namespace yuf {

YUF_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

YUF_DEVICE void store_out(float* p, size_t i, float v) { p[i] = v; }
YUF_DEVICE void store_out(__nv_bfloat16* p, size_t i, float v) { p[i] = __float2bfloat16_rn(v); }
// four consecutive elements, i a multiple of 4 (one 16- or 8-byte store)
YUF_DEVICE void store4(float* p, size_t i, float4 v) { *reinterpret_cast<float4*>(p + i) = v; }
YUF_DEVICE void store4(__nv_bfloat16* p, size_t i, float4 v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&lo);
  u.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p + i) = u;
}
YUF_DEVICE float4 f4_lerp(float4 x, float4 delta, float4 m) {
  return make_float4(fmaf(delta.x, m.x, x.x), fmaf(delta.y, m.y, x.y), fmaf(delta.z, m.z, x.z),
                     fmaf(delta.w, m.w, x.w));
}

// Sum over the block; every thread gets the total.  red: 32 floats of shared
// memory, reusable by the next call.
YUF_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();  // the previous call's readers are done with red
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int q = 0; q < nw; ++q) t += red[q];
  return t;
}

// x[row, :] = E[ids[row], :]  (nn.Embedding, model.py:411)
__global__ void embed_kernel(const int32_t* __restrict__ ids, const float* __restrict__ E,
                             float* __restrict__ x, int rows, int d, int vocab, int* __restrict__ err) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  if (row >= rows) return;
  int id = ids[row];
  if (id < 0 || id >= vocab) {  // out-of-range ids are reported, never read
    if (threadIdx.x == 0) atomicExch(err, 1);
    id = 0;
  }
  const float4* src = reinterpret_cast<const float4*>(E + (size_t)id * d);
  float4* dst = reinterpret_cast<float4*>(x + (size_t)row * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = src[i];
}

// LayerNorm over d (eps 1e-5, biased variance: nn.LayerNorm).  One warp per row.
// Optionally multiplies by gate[row, :] after the affine (out_norm(y) * g), or
// by sigmoid(gate[row, :]) when gate_sig (the gate's pre-activation, as the
// low-rank projection left it).
template <typename OUT>
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                 const float* __restrict__ b, const float* __restrict__ gate,
                                 OUT* __restrict__ out, int rows, int d, int gate_sig) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * d;
  float s = 0.f;
  for (int i = lane; i < d; i += 32) s += xr[i];
  const float mean = warp_sum(s) / d;
  float q = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float c = xr[i] - mean;
    q = fmaf(c, c, q);
  }
  const float rstd = rsqrtf(warp_sum(q) / d + 1e-5f);
  for (int i = lane; i < d; i += 32) {
    float v = (xr[i] - mean) * rstd * w[i] + b[i];
    if (gate) {
      const float gv = gate[(size_t)row * d + i];
      v *= gate_sig ? sigmoidf_fast(gv) : gv;
    }
    store_out(out, (size_t)row * d + i, v);
  }
}

// The same, with the row held in registers: VPL float4 per lane (d <= 128 VPL),
// one read of x (and of gate), two-pass mean/variance from registers.
template <typename OUT, int VPL>
__global__ void __launch_bounds__(128)
    layernorm_reg_kernel(const float* __restrict__ x, const float* __restrict__ w,
                         const float* __restrict__ b, const float* __restrict__ gate,
                         OUT* __restrict__ out, int rows, int d, int gate_sig) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int d4 = d >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * d);
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    v[u] = i < d4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
  }
  const float mean = warp_sum(s) / d;
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    if (lane + 32 * u < d4) {
      const float cx = v[u].x - mean, cy = v[u].y - mean, cz = v[u].z - mean, cw = v[u].w - mean;
      q = fmaf(cx, cx, fmaf(cy, cy, fmaf(cz, cz, fmaf(cw, cw, q))));
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / d + 1e-5f);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const float4* g4 = gate ? reinterpret_cast<const float4*>(gate + (size_t)row * d) : nullptr;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    if (i < d4) {
      const float4 ww = w4[i], bb = b4[i];
      float4 o = make_float4((v[u].x - mean) * rstd * ww.x + bb.x, (v[u].y - mean) * rstd * ww.y + bb.y,
                             (v[u].z - mean) * rstd * ww.z + bb.z, (v[u].w - mean) * rstd * ww.w + bb.w);
      if (g4) {
        float4 gg = g4[i];
        if (gate_sig) gg = make_float4(sigmoidf_fast(gg.x), sigmoidf_fast(gg.y), sigmoidf_fast(gg.z), sigmoidf_fast(gg.w));
        o.x *= gg.x; o.y *= gg.y; o.z *= gg.z; o.w *= gg.w;
      }
      store4(out, (size_t)row * d + 4 * i, o);
    }
  }
}

// Token shift + the six lerps (model.py:98-105):
//   delta = xt - shifted, x_c = xt + delta * mix_c, shifted = [prev, xt[:-1]]
// out layout [6][rows][d] in the order r, k, v, w, a, g (the order the batched
// projections consume).  The caller copies the new `prev` (xt of each
// sequence's last token, model.py:197) after this kernel, so `prev` is only read.
// Small row counts (decode batches): one CTA per row, one float4 per thread
// (d <= 4096), so a batch of a few hundred rows covers every SM and each thread
// has a single load in its dependency chain.  MIX: the TimeMix variant of
// ln_mix_step_kernel (xt written, prev read then replaced by xt, six lerps to
// out [6][rows][d]); otherwise LayerNorm, optional gate multiply, out [rows][d].
template <typename OUT, bool MIX>
__global__ void __launch_bounds__(1024)
    ln_row_kernel(const float* __restrict__ x, const float* __restrict__ w,
                  const float* __restrict__ b, const float* __restrict__ gate, OUT* __restrict__ out,
                  int rows, int d, float* __restrict__ xt, float* prev, const float* __restrict__ mix,
                  int gate_sig) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x, i = threadIdx.x, d4 = d >> 2;
  const bool act = i < d4;
  const size_t base = (size_t)row * d + 4 * (size_t)i;
  const float4 v = act ? *reinterpret_cast<const float4*>(x + base) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 pv = make_float4(0.f, 0.f, 0.f, 0.f), gv = make_float4(1.f, 1.f, 1.f, 1.f);
  if (act && MIX) pv = *reinterpret_cast<const float4*>(prev + base);
  if (act && !MIX && gate) {
    gv = *reinterpret_cast<const float4*>(gate + base);
    if (gate_sig) gv = make_float4(sigmoidf_fast(gv.x), sigmoidf_fast(gv.y), sigmoidf_fast(gv.z), sigmoidf_fast(gv.w));
  }
  const float mean = block_sum((v.x + v.y) + (v.z + v.w), red) / d;
  const float cx = v.x - mean, cy = v.y - mean, cz = v.z - mean, cw = v.w - mean;
  const float q = act ? fmaf(cx, cx, fmaf(cy, cy, fmaf(cz, cz, cw * cw))) : 0.f;
  const float rstd = rsqrtf(block_sum(q, red) / d + 1e-5f);
  if (!act) return;
  const float4 ww = reinterpret_cast<const float4*>(w)[i], bb = reinterpret_cast<const float4*>(b)[i];
  float4 o = make_float4(cx * rstd * ww.x + bb.x, cy * rstd * ww.y + bb.y, cz * rstd * ww.z + bb.z,
                         cw * rstd * ww.w + bb.w);
  if constexpr (MIX) {
    *reinterpret_cast<float4*>(xt + base) = o;
    *reinterpret_cast<float4*>(prev + base) = o;
    const float4 delta = make_float4(o.x - pv.x, o.y - pv.y, o.z - pv.z, o.w - pv.w);
    const size_t total = (size_t)rows * d;
    const float4* m4 = reinterpret_cast<const float4*>(mix);
    // mix rows in the reference order r, w, k, v, a, g; outputs in r, k, v, w, a, g
    store4(out, 0 * total + base, f4_lerp(o, delta, m4[0 * d4 + i]));
    store4(out, 3 * total + base, f4_lerp(o, delta, m4[1 * d4 + i]));
    store4(out, 1 * total + base, f4_lerp(o, delta, m4[2 * d4 + i]));
    store4(out, 2 * total + base, f4_lerp(o, delta, m4[3 * d4 + i]));
    store4(out, 4 * total + base, f4_lerp(o, delta, m4[4 * d4 + i]));
    store4(out, 5 * total + base, f4_lerp(o, delta, m4[5 * d4 + i]));
  } else {
    o = make_float4(o.x * gv.x, o.y * gv.y, o.z * gv.z, o.w * gv.w);
    store4(out, base, o);
  }
}

// One token per sequence (decode): the TimeMix layer norm, the six lerps and the
// token-shift update fused.  One warp per row, the row in registers (VPL float4
// per lane): xt = LN(x) is written for the caller, prev is read and then
// overwritten with xt by the same lane, the six mixes go to out [6][B][d].
template <typename OUT, int VPL>
__global__ void __launch_bounds__(128)
    ln_mix_step_kernel(const float* __restrict__ x, const float* __restrict__ w,
                       const float* __restrict__ b, float* __restrict__ xt, float* prev,
                       const float* __restrict__ mix, OUT* __restrict__ out, int B, int d) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= B) return;
  const int d4 = d >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * d);
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    v[u] = i < d4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
  }
  const float mean = warp_sum(s) / d;
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    if (lane + 32 * u < d4) {
      const float cx = v[u].x - mean, cy = v[u].y - mean, cz = v[u].z - mean, cw = v[u].w - mean;
      q = fmaf(cx, cx, fmaf(cy, cy, fmaf(cz, cz, fmaf(cw, cw, q))));
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / d + 1e-5f);
  const size_t total = (size_t)B * d;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4* p4 = reinterpret_cast<float4*>(prev + (size_t)row * d);
  float4* t4 = reinterpret_cast<float4*>(xt + (size_t)row * d);
  const float4* m4 = reinterpret_cast<const float4*>(mix);
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    if (i < d4) {
      const float4 ww = w4[i], bb = b4[i], pv = p4[i];
      const float4 o = make_float4(
          (v[u].x - mean) * rstd * ww.x + bb.x, (v[u].y - mean) * rstd * ww.y + bb.y,
          (v[u].z - mean) * rstd * ww.z + bb.z, (v[u].w - mean) * rstd * ww.w + bb.w);
      t4[i] = o;
      p4[i] = o;
      const float4 delta = make_float4(o.x - pv.x, o.y - pv.y, o.z - pv.z, o.w - pv.w);
      const size_t oi = (size_t)row * d + 4 * i;
      // mix rows in the reference order r, w, k, v, a, g; outputs in r, k, v, w, a, g
      store4(out, 0 * total + oi, f4_lerp(o, delta, m4[0 * d4 + i]));
      store4(out, 3 * total + oi, f4_lerp(o, delta, m4[1 * d4 + i]));
      store4(out, 1 * total + oi, f4_lerp(o, delta, m4[2 * d4 + i]));
      store4(out, 2 * total + oi, f4_lerp(o, delta, m4[3 * d4 + i]));
      store4(out, 4 * total + oi, f4_lerp(o, delta, m4[4 * d4 + i]));
      store4(out, 5 * total + oi, f4_lerp(o, delta, m4[5 * d4 + i]));
    }
  }
}

// The TimeMix layer norm of one row into registers (VPL float4 per lane, the
// arithmetic of layernorm_reg_kernel): two-pass mean and variance, then the affine.
template <int VPL>
YUF_DEVICE void ln_row_regs(const float* __restrict__ xrow, const float4* __restrict__ w4,
                            const float4* __restrict__ b4, int d, int lane, float4 (&o)[VPL]) {
  const int d4 = d >> 2;
  const float4* xr = reinterpret_cast<const float4*>(xrow);
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    v[u] = i < d4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
  }
  const float mean = warp_sum(s) / d;
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    if (lane + 32 * u < d4) {
      const float cx = v[u].x - mean, cy = v[u].y - mean, cz = v[u].z - mean, cw = v[u].w - mean;
      q = fmaf(cx, cx, fmaf(cy, cy, fmaf(cz, cz, fmaf(cw, cw, q))));
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / d + 1e-5f);
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    if (i < d4) {
      const float4 ww = w4[i], bb = b4[i];
      o[u] = make_float4((v[u].x - mean) * rstd * ww.x + bb.x, (v[u].y - mean) * rstd * ww.y + bb.y,
                         (v[u].z - mean) * rstd * ww.z + bb.z, (v[u].w - mean) * rstd * ww.w + bb.w);
    } else {
      o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// Prefill: the TimeMix layer norm, the token shift and the six lerps in one
// pass (model.py:98-105).  One warp per row (b, t): the row's norm and, for
// t > 0, the previous row's norm recomputed (its x is read again, mostly from
// L2) -- for t = 0 the shift source is prev[b], the previous call's last norm.
// xt receives only each sequence's last row (the caller copies it into prev
// after this kernel, so prev is only read here); out [6][rows][d] in the order
// r, k, v, w, a, g.
template <typename OUT, int VPL>
__global__ void __launch_bounds__(128)
    ln_mix_rows_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                       float* __restrict__ xt, const float* __restrict__ prev, const float* __restrict__ mix,
                       OUT* __restrict__ out, int B, int T, int d) {
  pdl_wait();
  pdl_trigger();
  const int rows = B * T;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int bb = row / T, t = row - bb * T;
  const int d4 = d >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4 o[VPL], sh[VPL];
  ln_row_regs<VPL>(x + (size_t)row * d, w4, b4, d, lane, o);
  if (t > 0) {
    ln_row_regs<VPL>(x + (size_t)(row - 1) * d, w4, b4, d, lane, sh);
  } else {
    const float4* p4 = reinterpret_cast<const float4*>(prev + (size_t)bb * d);
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      const int i = lane + 32 * u;
      sh[u] = i < d4 ? p4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const size_t total = (size_t)rows * d;
  const float4* m4 = reinterpret_cast<const float4*>(mix);
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int i = lane + 32 * u;
    if (i < d4) {
      const size_t oi = (size_t)row * d + 4 * i;
      if (t == T - 1) *reinterpret_cast<float4*>(xt + oi) = o[u];
      const float4 delta = make_float4(o[u].x - sh[u].x, o[u].y - sh[u].y, o[u].z - sh[u].z, o[u].w - sh[u].w);
      // mix rows in the reference order r, w, k, v, a, g; outputs in r, k, v, w, a, g
      store4(out, 0 * total + oi, f4_lerp(o[u], delta, m4[0 * d4 + i]));
      store4(out, 3 * total + oi, f4_lerp(o[u], delta, m4[1 * d4 + i]));
      store4(out, 1 * total + oi, f4_lerp(o[u], delta, m4[2 * d4 + i]));
      store4(out, 2 * total + oi, f4_lerp(o[u], delta, m4[3 * d4 + i]));
      store4(out, 4 * total + oi, f4_lerp(o[u], delta, m4[4 * d4 + i]));
      store4(out, 5 * total + oi, f4_lerp(o[u], delta, m4[5 * d4 + i]));
    }
  }
}

template <typename OUT>
__global__ void mix_kernel(const float* __restrict__ xt, const float* __restrict__ prev,
                           const float* __restrict__ mix, OUT* __restrict__ out, int B, int T, int d) {
  pdl_wait();
  pdl_trigger();
  const size_t rows = (size_t)B * T;
  const size_t total = rows * d;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / d;
    const int c = (int)(i - row * d);
    const int t = (int)(row % T);
    const int bb = (int)(row / T);
    const float x = xt[i];
    const float sh = t == 0 ? prev[(size_t)bb * d + c] : xt[i - d];
    const float delta = x - sh;
    // mix rows in the reference order r, w, k, v, a, g; outputs in r, k, v, w, a, g
    store_out(out, 0 * total + i, x + delta * mix[0 * d + c]);
    store_out(out, 3 * total + i, x + delta * mix[1 * d + c]);
    store_out(out, 1 * total + i, x + delta * mix[2 * d + c]);
    store_out(out, 2 * total + i, x + delta * mix[3 * d + c]);
    store_out(out, 4 * total + i, x + delta * mix[4 * d + c]);
    store_out(out, 5 * total + i, x + delta * mix[5 * d + c]);
  }
}

// out[i] = tanh(x[i]) for i < n_tanh, x[i] for n_tanh <= i < n (the tail is
// only a copy: the bf16 path converts the other low-rank branches in the same pass).
template <typename OUT>
__global__ void tanh_kernel(const float* __restrict__ x, OUT* __restrict__ out, size_t n_tanh,
                            size_t n) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    store_out(out, i, i < n_tanh ? tanhf(x[i]) : x[i]);
}

// w/a/g activations, kk normalisation and key adjustment (model.py:108-122).
// Inputs (row-major [rows, d]): k (key proj), lw = tanh(xw W1) W2, la = (xa A1) A2,
// lg = (xg G1) G2.  Outputs: w_raw = w0 + lw, a_op = -kk, b_op = kk * a,
// k_adj = k * (1 + (a - 1) * k_a), g = sigmoid(lg).  One warp per (row, head).
__global__ void timemix_post_kernel(const float* __restrict__ k, const float* __restrict__ lw,
                                    const float* __restrict__ la, const float* __restrict__ lg,
                                    const float* __restrict__ w0, const float* __restrict__ a0,
                                    const float* __restrict__ k_k, const float* __restrict__ k_a,
                                    float* __restrict__ w_raw, float* __restrict__ k_adj,
                                    float* __restrict__ a_op, float* __restrict__ b_op,
                                    float* __restrict__ g_out, int rows, int H, int N) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x >> 5;
  const size_t item = (size_t)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (size_t)rows * H) return;
  const size_t row = item / H;
  const int h = (int)(item - row * H);
  const int d = H * N;
  const size_t base = row * d + (size_t)h * N;
  // two columns per lane (N is even): 8-byte loads and stores
  float ss = 0.f;
  for (int j = 2 * lane; j < N; j += 64) {
    const float2 kv = *reinterpret_cast<const float2*>(k + base + j);
    const float2 kk = *reinterpret_cast<const float2*>(k_k + h * N + j);
    ss = fmaf(kv.x * kk.x, kv.x * kk.x, ss);
    ss = fmaf(kv.y * kk.y, kv.y * kk.y, ss);
  }
  const float nrm = sqrtf(warp_sum(ss));
  const float inv = 1.f / fmaxf(nrm, 1e-12f);  // F.normalize eps (model.py:116)
  for (int j = 2 * lane; j < N; j += 64) {
    const int c = h * N + j;
    const size_t i = base + j;
    const float2 kv = *reinterpret_cast<const float2*>(k + i);
    const float2 kkp = *reinterpret_cast<const float2*>(k_k + c);
    const float2 kap = *reinterpret_cast<const float2*>(k_a + c);
    const float2 a0p = *reinterpret_cast<const float2*>(a0 + c);
    const float2 w0p = *reinterpret_cast<const float2*>(w0 + c);
    const float2 lwv = *reinterpret_cast<const float2*>(lw + i);
    const float2 lav = *reinterpret_cast<const float2*>(la + i);
    const float2 lgv = *reinterpret_cast<const float2*>(lg + i);
    const float ax = sigmoidf_fast(a0p.x + lav.x), ay = sigmoidf_fast(a0p.y + lav.y);
    const float kkx = kv.x * kkp.x * inv, kky = kv.y * kkp.y * inv;
    *reinterpret_cast<float2*>(w_raw + i) = make_float2(w0p.x + lwv.x, w0p.y + lwv.y);
    *reinterpret_cast<float2*>(a_op + i) = make_float2(-kkx, -kky);
    *reinterpret_cast<float2*>(b_op + i) = make_float2(kkx * ax, kky * ay);
    *reinterpret_cast<float2*>(k_adj + i) =
        make_float2(kv.x * (1.f + (ax - 1.f) * kap.x), kv.y * (1.f + (ay - 1.f) * kap.y));
    *reinterpret_cast<float2*>(g_out + i) =
        make_float2(sigmoidf_fast(lgv.x), sigmoidf_fast(lgv.y));
  }
}

// SiLU(in) * gate over the fused [rows, 2F] projection (in | gate halves).
// One block per row (grid-strided over rows), four columns per thread (F % 4 == 0).
template <typename OUT>
__global__ void silu_mul_kernel(const float* __restrict__ ig, OUT* __restrict__ out, int rows,
                                int F) {
  pdl_wait();
  pdl_trigger();
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* in = ig + (size_t)row * 2 * F;
    const size_t o = (size_t)row * F;
    for (int c = 4 * threadIdx.x; c < F; c += 4 * blockDim.x) {
      const float4 h = *reinterpret_cast<const float4*>(in + c);
      const float4 gv = *reinterpret_cast<const float4*>(in + F + c);
      store_out(out, o + c + 0, h.x / (1.f + expf(-h.x)) * gv.x);
      store_out(out, o + c + 1, h.y / (1.f + expf(-h.y)) * gv.y);
      store_out(out, o + c + 2, h.z / (1.f + expf(-h.z)) * gv.z);
      store_out(out, o + c + 3, h.w / (1.f + expf(-h.w)) * gv.w);
    }
  }
}

// float -> bfloat16 copy (activations feeding a bf16-weight GEMM)
__global__ void to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, size_t n) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

// ---- host launchers ----
static int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  return (int)(g > 148 * 32 ? 148 * 32 : (g == 0 ? 1 : g));
}

void launch_embed(const int32_t* ids, const float* E, float* x, int rows, int d, int vocab, int* err,
                  cudaStream_t s) {
  launch_k(embed_kernel, dim3(rows), dim3(128), 0, s, ids, E, x, rows, d, vocab, err);
}
template <typename OUT>
void launch_layernorm(const float* x, const float* w, const float* b, const float* gate, OUT* out,
                      int rows, int d, cudaStream_t s, bool gate_sigmoid) {
  const int gs = gate_sigmoid ? 1 : 0;
  if (rows < 4 * 148 && d % 4 == 0 && d <= 4096) {  // small batch: one CTA per row
    launch_k(ln_row_kernel<OUT, false>, dim3(rows), dim3(((d / 4 + 31) / 32) * 32), 0, s, x, w, b, gate, out, rows, d,
                                                                         nullptr, nullptr, nullptr, gs);
    return;
  }
  // one row per warp, four warps per block
  const int wpb = 4;
  const int blocks = (rows + wpb - 1) / wpb;
  if (d % 4 == 0 && d <= 8 * 128) {  // row in registers (d <= 1024)
    const int vpl = (d / 4 + 31) / 32;
    switch (vpl) {
#define CASE(V)                                                                                  \
  case V:                                                                                        \
    launch_k(layernorm_reg_kernel<OUT, V>, dim3(blocks), dim3(32 * wpb), 0, s, x, w, b, gate, out, rows, d, gs); \
    return;
      CASE(1) CASE(2) CASE(3) CASE(4) CASE(5) CASE(6) CASE(7) CASE(8)
#undef CASE
      default: break;
    }
  }
  const int warps = 8;
  launch_k(layernorm_kernel<OUT>, dim3((rows + warps - 1) / warps), dim3(32 * warps), 0, s, x, w, b, gate, out, rows, d,
           gs);
}
template <typename OUT>
bool launch_ln_mix_step(const float* x, const float* w, const float* b, float* xt, float* prev,
                        const float* mix, OUT* out, int B, int d, cudaStream_t s) {
  if (d % 4 != 0) return false;
  if (B < 4 * 148 && d <= 4096) {
    launch_k(ln_row_kernel<OUT, true>, dim3(B), dim3(((d / 4 + 31) / 32) * 32), 0, s, x, w, b, nullptr, out, B, d, xt,
                                                                     prev, mix, 0);
    return true;
  }
  if (d > 8 * 128) return false;
  const int wpb = 4;
  const int blocks = (B + wpb - 1) / wpb;
  switch ((d / 4 + 31) / 32) {
#define CASE(V)                                                                                 \
  case V:                                                                                       \
    launch_k(ln_mix_step_kernel<OUT, V>, dim3(blocks), dim3(32 * wpb), 0, s, x, w, b, xt, prev, mix, out, B, d); \
    return true;
    CASE(1) CASE(2) CASE(3) CASE(4) CASE(5) CASE(6) CASE(7) CASE(8)
#undef CASE
    default: return false;
  }
}
template <typename OUT>
bool launch_ln_mix_rows(const float* x, const float* w, const float* b, float* xt, const float* prev,
                        const float* mix, OUT* out, int B, int T, int d, cudaStream_t s) {
  if (d % 4 != 0 || d > 8 * 128 || (long long)B * T > 0x7fffffffLL) return false;
  const int wpb = 4;
  const int blocks = (int)(((long long)B * T + wpb - 1) / wpb);
  switch ((d / 4 + 31) / 32) {
#define CASE(V)                                                                                 \
  case V:                                                                                       \
    launch_k(ln_mix_rows_kernel<OUT, V>, dim3(blocks), dim3(32 * wpb), 0, s, x, w, b, xt, prev, mix, out, B, T, d); \
    return true;
    CASE(1) CASE(2) CASE(3) CASE(4) CASE(5) CASE(6) CASE(7) CASE(8)
#undef CASE
    default: return false;
  }
}
template <typename OUT>
void launch_mix(const float* xt, const float* prev, const float* mix, OUT* out, int B, int T, int d,
                cudaStream_t s) {
  launch_k(mix_kernel<OUT>, dim3(grid_for((size_t)B * T * d, 256)), dim3(256), 0, s, xt, prev, mix, out, B, T, d);
}
template <typename OUT>
void launch_tanh(const float* x, OUT* out, size_t n_tanh, size_t n, cudaStream_t s) {
  launch_k(tanh_kernel<OUT>, dim3(grid_for(n, 256)), dim3(256), 0, s, x, out, n_tanh, n);
}
void launch_timemix_post(const float* k, const float* lw, const float* la, const float* lg,
                         const float* w0, const float* a0, const float* k_k, const float* k_a,
                         float* w_raw, float* k_adj, float* a_op, float* b_op, float* g, int rows,
                         int H, int N, cudaStream_t s) {
  const int warps = 8;
  const size_t items = (size_t)rows * H;
  launch_k(timemix_post_kernel, dim3((unsigned)((items + warps - 1) / warps)), dim3(32 * warps), 0, s, 
      k, lw, la, lg, w0, a0, k_k, k_a, w_raw, k_adj, a_op, b_op, g, rows, H, N);
}
template <typename OUT>
void launch_silu_mul(const float* ig, OUT* out, int rows, int F, cudaStream_t s) {
  launch_k(silu_mul_kernel<OUT>, dim3(rows < 148 * 64 ? rows : 148 * 64), dim3(256), 0, s, ig, out, rows, F);
}
void launch_to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s) {
  launch_k(to_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, x, y, n);
}

template void launch_layernorm<float>(const float*, const float*, const float*, const float*, float*,
                                      int, int, cudaStream_t, bool);
template void launch_layernorm<__nv_bfloat16>(const float*, const float*, const float*, const float*,
                                              __nv_bfloat16*, int, int, cudaStream_t, bool);
template bool launch_ln_mix_step<float>(const float*, const float*, const float*, float*, float*,
                                         const float*, float*, int, int, cudaStream_t);
template bool launch_ln_mix_step<__nv_bfloat16>(const float*, const float*, const float*, float*,
                                                float*, const float*, __nv_bfloat16*, int, int,
                                                cudaStream_t);
template bool launch_ln_mix_rows<float>(const float*, const float*, const float*, float*, const float*,
                                         const float*, float*, int, int, int, cudaStream_t);
template bool launch_ln_mix_rows<__nv_bfloat16>(const float*, const float*, const float*, float*, const float*,
                                                 const float*, __nv_bfloat16*, int, int, int, cudaStream_t);
template void launch_mix<float>(const float*, const float*, const float*, float*, int, int, int,
                                cudaStream_t);
template void launch_mix<__nv_bfloat16>(const float*, const float*, const float*, __nv_bfloat16*,
                                        int, int, int, cudaStream_t);
template void launch_tanh<float>(const float*, float*, size_t, size_t, cudaStream_t);
template void launch_tanh<__nv_bfloat16>(const float*, __nv_bfloat16*, size_t, size_t, cudaStream_t);
template void launch_silu_mul<float>(const float*, float*, int, int, cudaStream_t);
template void launch_silu_mul<__nv_bfloat16>(const float*, __nv_bfloat16*, int, int, cudaStream_t);

}  // namespace yuf
