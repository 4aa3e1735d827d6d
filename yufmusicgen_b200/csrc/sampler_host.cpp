// Host-side sampling that draws the same tokens as the reference's CPU loop:
// sample_token (yufmusicgen/cli/generate.py:45-56) after torch.manual_seed
// (training.py:23-28), i.e. temperature, a descending sort, softmax, the top-p
// cut `cumulative - p > top_p`, a second softmax and torch.multinomial(p, 1) on
// the CPU generator.  (The bit-level reading of that path is the one the
// reference's own Rust client restates, vulkan/src/sampler.rs:1-270.)
//
// * Generator: MT19937 (Matsumoto & Nishimura 1998) with the 2002 seeding
//   recurrence s[j] = 1812433253 (s[j-1] ^ (s[j-1] >> 30)) + j from the low 32
//   bits of the seed -- torch's CPU generator.
// * A single-sample multinomial on the CPU keys every element with an Exp(1)
//   draw q = -log1p(-u) (u: two 32-bit words, the low 53 bits of hi:lo, times
//   2^-53; computed in double, rounded to float) and returns argmax(p / q) --
//   the exponential-race form of a categorical draw.  Every element of the
//   probability row consumes one draw, in the row's (sorted) order.
// * The sort is std::sort of (value, index) pairs with torch's descending
//   comparator, which orders equal values as torch's CPU sort does.
// * Sums follow torch's CPU kernels: the softmax sum in float over 8-lane
//   partial sums, the cumulative sum accumulated in double and stored as float.
// The per-element exp is the C library's expf, so a probability may differ
// from torch's vectorised exp in the last bit; a token can only differ where
// two keys p/q tie to that precision.
//
// Host code only (no GPU); the generator is not thread-safe per instance.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <numeric>
#include <vector>

#include "../../include/yufb200.h"

namespace yuf {
void set_error(const char* fmt, ...);
}

struct yuf_mt19937 {
  uint32_t s[624];
  int idx;
};

namespace {

void mt_seed(yuf_mt19937* g, uint64_t seed) {
  g->s[0] = (uint32_t)(seed & 0xffffffffu);
  for (int j = 1; j < 624; ++j) g->s[j] = 1812433253u * (g->s[j - 1] ^ (g->s[j - 1] >> 30)) + (uint32_t)j;
  g->idx = 624;
}

void mt_twist(yuf_mt19937* g) {
  for (int j = 0; j < 624; ++j) {
    const uint32_t y = (g->s[j] & 0x80000000u) | (g->s[(j + 1) % 624] & 0x7fffffffu);
    g->s[j] = g->s[(j + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
  }
  g->idx = 0;
}

uint32_t mt_next(yuf_mt19937* g) {
  if (g->idx >= 624) mt_twist(g);
  uint32_t y = g->s[g->idx++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

double mt_uniform53(yuf_mt19937* g) {
  const uint64_t hi = mt_next(g), lo = mt_next(g);
  return (double)(((hi << 32) | lo) & ((1ull << 53) - 1)) * (1.0 / 9007199254740992.0);
}

float mt_exponential(yuf_mt19937* g) { return (float)(-std::log1p(-mt_uniform53(g))); }

// float sum over 8 interleaved lanes (element i into lane i % 8), lanes folded
// pairwise; the elements past the last full group of eight are added last.
float lane_sum8(const float* x, size_t n) {
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int l = 0; l < 8; ++l) lanes[l] += x[i + l];
  float tail = 0.f;
  for (; i < n; ++i) tail += x[i];
  const float a = lanes[0] + lanes[1], b = lanes[2] + lanes[3], c = lanes[4] + lanes[5], d = lanes[6] + lanes[7];
  return (a + b) + (c + d) + tail;
}

// softmax of x[0..n) in place (max-shifted expf, one reciprocal, a multiply)
void softmax_inplace(float* x, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::max(mx, x[i]);
  for (size_t i = 0; i < n; ++i) x[i] = std::exp(x[i] - mx);
  const float inv = 1.f / lane_sum8(x, n);
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

int32_t argmax_first(const float* x, int V) {
  int32_t best = 0;
  for (int i = 1; i < V; ++i)
    if (x[i] > x[best]) best = i;
  return best;
}

int32_t sample_row(const float* logits, int V, float temperature, float top_p, yuf_mt19937* g,
                   std::vector<int32_t>& order) {
  if (temperature <= 0.f) return argmax_first(logits, V);
  // descending sort of (value, index) pairs with std::sort and torch's
  // descending comparator (NaN first, then larger values): the same
  // introsort on the same sequence, so equal logits land in the same order as
  // in torch.sort(descending=True) on the CPU
  std::vector<std::pair<float, int32_t>> kv(V);
  for (int i = 0; i < V; ++i) kv[i] = {logits[i] / temperature, i};
  std::sort(kv.begin(), kv.end(), [](const std::pair<float, int32_t>& l, const std::pair<float, int32_t>& r) {
    return (std::isnan(l.first) && !std::isnan(r.first)) || l.first > r.first;
  });
  order.resize(V);
  std::vector<float> p(V), s(V);
  for (int i = 0; i < V; ++i) {
    order[i] = kv[i].second;
    s[i] = p[i] = kv[i].first;
  }
  softmax_inplace(p.data(), V);
  // top-p: drop an entry when the mass before it exceeds top_p
  double cum = 0.0;
  for (int i = 0; i < V; ++i) {
    cum += p[i];
    if ((float)cum - p[i] > top_p) s[i] = -INFINITY;
  }
  softmax_inplace(s.data(), V);
  // multinomial(s, 1): argmax of s / Exp(1) keys, one key per element in order
  int best = 0;
  float best_key = -INFINITY;
  for (int i = 0; i < V; ++i) {
    const float q = mt_exponential(g);
    const float key = s[i] / q;
    if (key > best_key) {
      best_key = key;
      best = i;
    }
  }
  return order[best];
}

}  // namespace

extern "C" {

yuf_status_t yuf_mt19937_create(uint64_t seed, yuf_mt19937** out) {
  if (!out) {
    yuf::set_error("mt19937: null output");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  yuf_mt19937* g = new (std::nothrow) yuf_mt19937;
  if (!g) {
    yuf::set_error("mt19937: out of host memory");
    return YUF_ERR_OUT_OF_MEMORY;
  }
  mt_seed(g, seed);
  *out = g;
  return YUF_OK;
}

yuf_status_t yuf_mt19937_destroy(yuf_mt19937* g) {
  delete g;
  return YUF_OK;
}

yuf_status_t yuf_mt19937_next(yuf_mt19937* g, uint32_t* out, int64_t n) {
  if (!g || (n > 0 && !out) || n < 0) {
    yuf::set_error("mt19937: null generator or output, or n < 0");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  for (int64_t i = 0; i < n; ++i) out[i] = mt_next(g);
  return YUF_OK;
}

yuf_status_t yuf_mt19937_exponential(yuf_mt19937* g, float* out, int64_t n) {
  if (!g || (n > 0 && !out) || n < 0) {
    yuf::set_error("mt19937: null generator or output, or n < 0");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  for (int64_t i = 0; i < n; ++i) out[i] = mt_exponential(g);
  return YUF_OK;
}

yuf_status_t yuf_sample_host(const float* logits, int B, int V, float temperature, float top_p,
                             yuf_mt19937* g, int32_t* out_ids) {
  if (!logits || !g || !out_ids || B < 0 || V < 1) {
    yuf::set_error("sample_host: null logits, generator or output, or bad sizes (B=%d V=%d)", B, V);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (!std::isfinite(temperature) || !std::isfinite(top_p)) {
    yuf::set_error("sample_host: temperature and top_p must be finite");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  std::vector<int32_t> order;
  for (int b = 0; b < B; ++b) {
    const float* row = logits + (size_t)b * V;
    if (temperature > 0.f) {
      bool any = false;
      for (int i = 0; i < V && !any; ++i) any = row[i] > -INFINITY;
      if (!any) {
        yuf::set_error("sample_host: row %d has no selectable token (all -inf)", b);
        return YUF_ERR_INVALID_ARGUMENT;
      }
    }
    out_ids[b] = sample_row(row, V, temperature, top_p, g, order);
  }
  return YUF_OK;
}

}  // extern "C"
