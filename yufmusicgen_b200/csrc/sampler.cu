// On-device token sampler for batched decode.
//
// The reference samples on the host after every step (yufmusicgen/cli/generate.py:45-56,
// 139-154): mask the logits (only MIDI ids, plus EOS after 16 generated tokens),
// divide by the temperature, keep the smallest prefix of the sorted distribution
// whose mass reaches top_p, and draw with torch.multinomial -- one device->host
// sync per token.  Here one CTA per sequence does the same on the GPU:
//   1. masked, temperature-scaled logits of the row go to shared memory;
//   2. the top_k largest, in descending order with ties to the smaller id (a
//      radix select for the k-th largest, then a rank sort of the k);
//   3. softmax over those k, then the top-p cut inside them (a token is dropped
//      when the mass before it already exceeds top_p, generate.py:52), then an
//      inverse-CDF draw with a uniform from Philox4x32-10.
// The uniform for (seed, sequence, step) is the first output word of
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
// as 1, 2, 3", SC'11) with key (seed_lo, seed_hi) and counter
// (step_lo, step_hi, sequence, 0), mapped to [0, 1) as (x >> 8) * 2^-24, so a
// run is reproducible and independent of the batch layout.  temperature <= 0
// selects the argmax (greedy).

#include <cfloat>

#include "common.cuh"

namespace yuf {

struct U4 {
  uint32_t x, y, z, w;
};

// Philox4x32-10 as published (round multipliers and Weyl key increments).
YUF_DEVICE U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}

YUF_DEVICE float philox_uniform(uint64_t seed, uint64_t step, uint32_t seq) {
  const U4 out = philox4x32_10(U4{(uint32_t)step, (uint32_t)(step >> 32), seq, 0u}, (uint32_t)seed,
                               (uint32_t)(seed >> 32));
  return (float)(out.x >> 8) * (1.0f / 16777216.0f);
}

constexpr int SAMPLER_THREADS = 512;
constexpr int SAMPLER_MAX_K = 1024;

// Order-preserving map float -> uint32 (larger float, larger key); -0 is
// canonicalised to +0 by the caller so equal floats have equal keys.
YUF_DEVICE uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Step 2 above as a radix select instead of top_k argmax rounds: four 8-bit
// histogram passes (most significant digit first) find the key of the k-th
// largest logit; every logit above it is a candidate, and of those equal to it
// the smallest ids fill the remaining places (the same set, and after the rank
// sort the same order, as descending extraction with ties to the smaller id).
__global__ void __launch_bounds__(SAMPLER_THREADS)
    sample_kernel(const float* __restrict__ logits, int V, float inv_temp, int top_k, float top_p,
                  uint64_t seed, uint64_t step, int seq0, int mask_below, int eos_id, int allow_eos,
                  int32_t* __restrict__ out_ids, float* __restrict__ out_u) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float srow[];                 // [V] masked scaled logits
  __shared__ float top_v[SAMPLER_MAX_K];
  __shared__ int top_i[SAMPLER_MAX_K];
  __shared__ float cand_v[SAMPLER_MAX_K];
  __shared__ int cand_i[SAMPLER_MAX_K];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[3];
  __shared__ int wsum[SAMPLER_THREADS / 32];
  __shared__ int n_above;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const float* row = logits + (size_t)b * V;
  for (int i = tid; i < V; i += SAMPLER_THREADS) {
    const bool allowed = i >= mask_below || (allow_eos && i == eos_id);
    srow[i] = allowed ? row[i] * inv_temp + 0.f : -FLT_MAX;
  }
  if (tid == 0) n_above = 0;
  if (top_k == 1) {
    // greedy: one block-wide argmax (ties -> the smaller id)
    __syncthreads();
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += SAMPLER_THREADS) {
      const float x = srow[i];
      if (x > bv || (x == bv && i < bi)) { bv = x; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { cand_v[wid] = bv; cand_i[wid] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int q = 1; q < SAMPLER_THREADS / 32; ++q)
        if (cand_v[q] > bv || (cand_v[q] == bv && cand_i[q] < bi)) { bv = cand_v[q]; bi = cand_i[q]; }
      out_ids[b] = bi;
      if (out_u) out_u[b] = philox_uniform(seed, step, (uint32_t)(seq0 + b));
    }
    return;
  }
  // radix select: after the passes, `prefix` is the k-th largest key and `need`
  // the number of logits equal to it that belong to the top k
  uint32_t prefix = 0, pmask = 0, need = (uint32_t)top_k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += SAMPLER_THREADS) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += SAMPLER_THREADS) {
      const uint32_t key = order_key(srow[i]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (wid == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending); find the bin where the
      // count from the top reaches `need`
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        tot += c[j];
      }
      uint32_t inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      uint32_t acc = inc - tot;
      if (acc < need && need <= inc) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc < need && need <= acc + c[j]) {
            sel[0] = prefix | ((uint32_t)(255 - 8 * lane - j) << shift);
            sel[1] = need - acc;
            sel[2] = c[j];  // logits in the chosen bin
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    prefix = sel[0];
    need = sel[1];
    pmask |= 255u << shift;
  }
  const uint32_t thr = prefix;
  const int n_gt = top_k - (int)need;
  // all logits equal to the threshold are taken (the usual case): they are
  // gathered with those above it, the rank sort orders them by id
  const bool take_all_eq = sel[2] == need;
  // candidates above the threshold (any order; ranked below)
  for (int i = tid; i < V; i += SAMPLER_THREADS) {
    const float x = srow[i];
    const uint32_t key = order_key(x);
    if (key > thr || (take_all_eq && key == thr)) {
      const int slot = atomicAdd(&n_above, 1);
      cand_v[slot] = x;
      cand_i[slot] = i;
    }
  }
  // otherwise the logits equal to the threshold, smallest ids first: contiguous
  // id ranges per thread and a block-wide exclusive scan of their counts
  if (!take_all_eq) {
    const int per = (V + SAMPLER_THREADS - 1) / SAMPLER_THREADS;
    const int lo = min(V, tid * per), hi = min(V, lo + per);
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += order_key(srow[i]) == thr;
    int inc = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    if (lane == 31) wsum[wid] = inc;
    __syncthreads();
    int rank = inc - cnt;
    for (int q = 0; q < wid; ++q) rank += wsum[q];
    for (int i = lo; i < hi && rank < (int)need; ++i) {
      if (order_key(srow[i]) == thr) {
        cand_v[n_gt + rank] = srow[i];
        cand_i[n_gt + rank] = i;
        ++rank;
      }
    }
  }
  __syncthreads();
  // rank sort: value descending, ties by the smaller id
  for (int t = tid; t < top_k; t += SAMPLER_THREADS) {
    const float v = cand_v[t];
    const int id = cand_i[t];
    int r = 0;
    for (int q = 0; q < top_k; ++q) {
      const float w = cand_v[q];
      r += (w > v) || (w == v && cand_i[q] < id);
    }
    top_v[r] = v;
    top_i[r] = id;
  }
  __syncthreads();
  if (tid == 0) {
    const float u = philox_uniform(seed, step, (uint32_t)(seq0 + b));
    int pick = top_i[0];
    if (inv_temp > 0.f && top_k > 1) {
      // softmax over the k candidates (descending), top-p cut, inverse CDF
      const float mx = top_v[0];
      float tot = 0.f;
      int kk = 0;
      for (; kk < top_k; ++kk) {
        if (top_v[kk] == -FLT_MAX || top_v[kk] == -INFINITY) break;  // masked
        tot += __expf(top_v[kk] - mx);
      }
      float cum = 0.f, kept = 0.f;
      int keep = 0;
      for (; keep < kk; ++keep) {
        const float p = __expf(top_v[keep] - mx) / tot;
        if (cum > top_p) break;  // mass before this token already exceeds top_p
        cum += p;
        kept += p;
      }
      if (keep == 0) keep = 1;
      const float target = u * kept;
      float acc = 0.f;
      pick = top_i[keep - 1];
      for (int q = 0; q < keep; ++q) {
        acc += __expf(top_v[q] - mx) / tot;
        if (target < acc) { pick = top_i[q]; break; }
      }
    }
    out_ids[b] = pick;
    if (out_u) out_u[b] = u;
  }
}

// Philox uniforms only (for checking the generator against a host restatement).
__global__ void philox_kernel(uint64_t seed, uint64_t step, int seq0, int n, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = philox_uniform(seed, step, (uint32_t)(seq0 + i));
}

}  // namespace yuf

using namespace yuf;

extern "C" yuf_status_t yuf_sample(const float* logits, int B, int V, float temperature, int top_k,
                                   float top_p, uint64_t seed, uint64_t step, int seq0,
                                   int mask_below, int eos_id, int allow_eos, int32_t* out_ids,
                                   float* out_uniform, void* stream) {
  if (B < 0 || V < 1 || !logits || !out_ids) {
    set_error("sample: need B >= 0, V >= 1, logits and out_ids");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (top_k < 1 || top_k > SAMPLER_MAX_K || top_k > V) {
    set_error("sample: top_k=%d must be in [1, min(%d, V)]", top_k, SAMPLER_MAX_K);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (!(top_p > 0.f) || top_p > 1.f) {
    set_error("sample: top_p=%g must be in (0, 1]", (double)top_p);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  const size_t smem = (size_t)V * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("sample: vocabulary of %d does not fit the sampler's shared-memory row", V);
    return YUF_ERR_UNSUPPORTED;
  }
  if (B == 0) return YUF_OK;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("sample: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return YUF_ERR_CUDA;
    }
  }
  const float inv_temp = temperature > 0.f ? 1.f / temperature : 0.f;
  const int k = temperature > 0.f ? top_k : 1;
  launch_k(sample_kernel, dim3(B), dim3(SAMPLER_THREADS), smem, static_cast<cudaStream_t>(stream), 
      logits, V, temperature > 0.f ? inv_temp : 1.f, k, top_p, seed, step, seq0, mask_below, eos_id,
      allow_eos, out_ids, out_uniform);
  return check_launch("sample_kernel");
}

extern "C" yuf_status_t yuf_philox_uniform(uint64_t seed, uint64_t step, int seq0, int n, float* out,
                                           void* stream) {
  if (n < 0 || (n > 0 && !out)) {
    set_error("philox: need n >= 0 and an output buffer");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (n == 0) return YUF_OK;
  philox_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(seed, step, seq0, n, out);
  return check_launch("philox_kernel");
}
