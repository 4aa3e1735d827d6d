// Model engine: the YufMusicGen block stack on one B200 with device-resident
// recurrent state slots (C ABI in include/yufb200.h).
//
// Forward of one block (yufmusicgen/model.py:365-378), rows = tokens:
//   xt  = LN_time(x)                                   layernorm_kernel
//   6 token-shift mixes of xt (prev = state)           mix_kernel
//   r,k,v = x_{r,k,v} W^T                              one batched GEMM
//   lr1 = x_{w,a,g} L1 (tanh on the w part in the epilogue) ; lr2 = lr1 L2   two batched GEMMs
//   w_raw, k_adj, a_op, b_op, g                        timemix_post_kernel
//   y, S  = WKV-7 scan (state slot in/out)             wkv7 kernels
//   x    += W_o (LN_out(y) * g)                        layernorm(+gate) + GEMM accumulating into x
//   [cand|write|gate] = LN_rosa(x) W^T                 one GEMM ([3R, d] weight)
//   read, m = ROSA scan (+ bias, gated, state slot)    rosa scan kernel
//   x    += read W_out^T                               GEMM accumulating into x
//   x    += W_out(silu(x_f W_in^T) * (x_f W_g^T))      GEMM [8d, d] with a SiLU-gate epilogue,
//                                                      GEMM accumulating into x
// then logits = LN_final(x) E^T (tied head, model.py:389-391, 421).
//
// Every projection is the library's tcgen05 GEMM (gemm.cu), with the work
// around it folded into the epilogues: tanh of the w branch (lr1), the residual
// adds of W_o / ROSA out / FFN out (accumulate into x), and SiLU(in) * gate of
// the FFN (its weight packed in 64-row in/gate groups), so no [rows, 8d]
// intermediate exists.  bf16-weight mode: bf16 weights and bf16 activations
// with fp32 accumulation.  fp32 mode: fp32 weights (stored as their tf32 high
// part and remainder) and fp32 activations at fp32 accuracy (3xTF32).
// Everything else (scans, norms, activations, state) stays fp32.

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "gemm.cuh"
#include "model_kernels.cuh"

namespace yuf {

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~DevBuf() { if (p) cudaFree(p); }
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
};

static int reference_low_rank(int d) {
  // max(32, int(round(2.5 * sqrt(d) / 32) * 32)), Python round-half-even (model.py:59)
  const double x = 2.5 * std::sqrt((double)d) / 32.0;
  double r = std::nearbyint(x);  // default rounding mode: half to even
  return std::max(32, (int)r * 32);
}

}  // namespace yuf

using namespace yuf;

// A projection weight [rows, K]: bf16 in bf16-weight mode (lo unused); in fp32
// mode its tf32 high part and the fp32 remainder, two planes of rows * K.
struct Wt {
  void* hi = nullptr;
  void* lo = nullptr;
};

struct LayerW {
  float *ln_t_w, *ln_t_b, *mix, *w0, *a0, *k_k, *k_a;
  Wt W_rkv, W_lr1, W_lr2, W_o;
  float *ln_o_w, *ln_o_b, *ln_r_w, *ln_r_b, *householder, *decay, *b_rosa;
  float* rosa_factors = nullptr;  // the time-parallel ROSA scan's layer constants, built at load
  Wt W_rosa_in, W_rosa_out;
  float *ln_f_w, *ln_f_b;
  Wt W_ffn_in, W_ffn_out;
};

struct yuf_model {
  yuf_model_config cfg{};
  int precision = 0;
  int device = 0;
  std::vector<std::unique_ptr<DevBuf>> owned;
  float* emb = nullptr;        // [V, d] fp32
  Wt emb_gemm;                 // LM head operand (the tied embedding as a projection weight)
  float *fin_w = nullptr, *fin_b = nullptr;
  std::vector<LayerW> L;
  // state slots
  int n_slots = 0;
  float *st_prev = nullptr, *st_S = nullptr, *st_m = nullptr;
  // workspace
  size_t ws_rows = 0;
  std::unique_ptr<DevBuf> ws;
  int* d_err = nullptr;
  // decode-step CUDA graphs, keyed by (B, slot0, ids, logits); a workspace
  // reallocation bumps ws_gen and invalidates them
  struct DecodeGraph {
    int B, slot0;
    const void* ids;
    const void* logits;
    size_t ws_gen;
    cudaGraphExec_t exec;
  };
  bool decode_graphs = false;
  // a decode step runs the low-rank projections (x_{w,a,g} L1, then L2) on a
  // second stream beside the r/k/v projection: both read the mixes, and the
  // time-mix epilogue joins them
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  ~yuf_model() {
    if (ev_join) cudaEventDestroy(ev_join);
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (side) cudaStreamDestroy(side);
  }
  size_t ws_gen = 0;
  std::vector<DecodeGraph> graphs;
  void drop_graphs() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.exec);
    graphs.clear();
  }
  // yuf_generate's working buffers: the last logits [B, V] and the sampled ids
  // [B], grown on demand (stable pointers, so its decode graphs replay)
  std::unique_ptr<DevBuf> gen;
  // debug dumps: region -> per layer host copies of the last call
  bool debug = false;
  std::map<std::string, std::vector<std::vector<float>>> dumps;
  std::vector<std::string> debug_regions;  // empty: every region
  std::vector<char> debug_layers;          // empty: every layer

  void* alloc(size_t bytes) {
    auto b = std::make_unique<DevBuf>();
    if (cudaMalloc(&b->p, bytes) != cudaSuccess) return nullptr;
    b->bytes = bytes;
    void* p = b->p;
    owned.push_back(std::move(b));
    return p;
  }
  int d() const { return cfg.d_model; }
  int H() const { return cfg.n_heads; }
  int N() const { return cfg.head_size; }
  int R() const { return cfg.rosa_size; }
  int lr() const { return cfg.low_rank; }
  int V() const { return cfg.vocab_size; }
  size_t wsz() const { return precision == YUF_PRECISION_BF16_WEIGHTS ? 2 : 4; }
  size_t slot_prev() const { return (size_t)d(); }
  size_t slot_S() const { return (size_t)H() * N() * N(); }
  size_t slot_m() const { return (size_t)R(); }
};

namespace yuf {
#define Y_REQUIRE(cond, ...)                 \
  do {                                       \
    if (!(cond)) {                           \
      set_error(__VA_ARGS__);                \
      return YUF_ERR_INVALID_ARGUMENT;       \
    }                                        \
  } while (0)
#define Y_CUDA(call)                                                          \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      set_error("%s failed: %s", #call, cudaGetErrorString(e_));              \
      return e_ == cudaErrorMemoryAllocation ? YUF_ERR_OUT_OF_MEMORY : YUF_ERR_CUDA; \
    }                                                                         \
  } while (0)
#define Y_TRY(call)                    \
  do {                                 \
    yuf_status_t st_ = (call);         \
    if (st_ != YUF_OK) return st_;     \
  } while (0)

// C[z] = A[z] . W[z]^T on the tcgen05 GEMM (gemm.cu) in the model's precision:
// bf16 operands (bf16-weight mode) or fp32 operands at fp32 accuracy (3xTF32).
// a_brows / w_brows: rows between batches in A / W; c_bstride: elements
// between batches in C.  `epi` names the bf16-mode epilogue; fp32 mode writes
// the same results in fp32 (GEMM_EPI_BF16 -> fp32 with the same tanh,
// GEMM_EPI_SWIGLU -> GEMM_EPI_SWIGLU_F32).
static yuf_status_t proj(const yuf_model* m, const void* A, long long lda, long long a_brows, const Wt& W,
                         long long w_brows, void* C, long long ldc, long long c_bstride, int M, int N, int K,
                         int batch, int epi, bool accumulate, cudaStream_t s, int n_out = 0,
                         bool tanh_batch0 = false) {
  GemmArgs g{};
  g.A = A;
  g.lda = lda;
  g.a_brows = a_brows;
  g.a_rows = (long long)(batch - 1) * a_brows + M;
  g.W = W.hi;
  g.w_brows = w_brows;
  g.w_rows = (long long)(batch - 1) * w_brows + N;
  g.C = C;
  g.ldc = ldc;
  g.c_bstride = c_bstride;
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = batch;
  g.epi = epi;
  g.beta = accumulate ? 1.f : 0.f;
  g.tanh_batch0 = tanh_batch0 ? 1 : 0;
  g.n_out = n_out;
  if (m->precision == YUF_PRECISION_BF16_WEIGHTS) return gemm_bf16(g, s);
  g.epi = epi == GEMM_EPI_SWIGLU ? GEMM_EPI_SWIGLU_F32 : GEMM_EPI_F32;
  return gemm_tf32x3(g, W.lo, s);
}

// Rows of the packed FFN in/gate weight: 64-row groups of ffn_in.weight and
// ffn_gate.weight alternating, the hidden width padded to 64.
static int ffn_pad(int d) { return (4 * d + 63) / 64 * 64; }

// Workspace for `rows` token rows (grown on demand; never shrinks).
struct WS {
  float *x, *xt, *mixed, *rkv, *lr1, *lr2, *w_raw, *k_adj, *a_op, *b_op, *g, *y, *tmp, *rosa, *read,
      *h, *scan;  // scan: scratch of the time-parallel scans
  __nv_bfloat16* bf;  // bf16 staging of a GEMM input (largest: [rows, 4d] or [6][rows][d])
};

static size_t ws_floats_per_row(const yuf_model* m) {
  const size_t d = m->d(), lr = m->lr(), R = m->R();
  return d /*x*/ + d /*xt*/ + 6 * d /*mixed*/ + 3 * d /*rkv*/ + 3 * lr /*lr1*/ + 3 * d /*lr2*/ +
         5 * d /*w_raw,k_adj,a_op,b_op,g*/ + d /*y*/ + d /*tmp*/ + 3 * R /*rosa*/ + R /*read*/ +
         4 * d /*h*/;
}

// Scratch of the time-parallel scans for a forward over `rows` token rows.
static size_t scan_rosa_floats(const yuf_model* m, size_t rows) {
  const size_t R = m->R();
  // A^K, chunk end and start states, the layer's coefficient block (32 + 2R);
  // rounded so the WKV part stays 16-byte aligned
  return (R * R + 2 * (rows / 32 + 1) * R + 32 + 2 * R + 3) / 4 * 4;
}

static size_t scan_scratch_floats(const yuf_model* m, size_t rows) {
  // ROSA: A^K + chunk end/start states (32-token chunks); WKV: the time-parallel
  // scan's bound for any batch of at most `rows` tokens
  return scan_rosa_floats(m, rows) + wkv7_parallel_scratch_bound(rows, m->H(), m->N());
}

// bf16 staging elements per token row: the largest GEMM input written in bf16
// (the six mixes [6][rows][d], the three low-rank activations [3][rows][lr], the
// FFN hidden [rows][4d], the ROSA read [rows][R]).
static size_t bf_elems_per_row(const yuf_model* m) {
  return (size_t)std::max({6 * m->d(), 3 * m->lr(), m->R()});
}

// decode_only: a T = 1 step, which never touches the time-parallel scans' scratch
static size_t ws_bytes(const yuf_model* m, size_t rows, bool decode_only = false) {
  const size_t per = ws_floats_per_row(m);
  const size_t scan = decode_only ? 0 : scan_scratch_floats(m, rows);
  return (rows * per + scan) * sizeof(float) + rows * bf_elems_per_row(m) * sizeof(__nv_bfloat16) +
         512;
}

static yuf_status_t ensure_ws(yuf_model* m, size_t rows) {
  if (rows <= m->ws_rows) return YUF_OK;
  auto b = std::make_unique<DevBuf>();
  const size_t bytes = ws_bytes(m, rows);
  Y_CUDA(cudaMalloc(&b->p, bytes));
  b->bytes = bytes;
  m->ws = std::move(b);
  m->ws_rows = rows;
  ++m->ws_gen;
  m->drop_graphs();  // captured graphs point into the old workspace
  return YUF_OK;
}

static WS carve(yuf_model* m, size_t rows, void* base, bool decode_only = false) {
  float* p = static_cast<float*>(base);
  const size_t d = m->d(), lr = m->lr(), R = m->R();
  WS w;
  auto take = [&](size_t n) { float* q = p; p += n; return q; };
  w.x = take(rows * d);
  w.xt = take(rows * d);
  w.mixed = take(6 * rows * d);
  w.rkv = take(3 * rows * d);
  w.lr1 = take(3 * rows * lr);
  w.lr2 = take(3 * rows * d);
  w.w_raw = take(rows * d);
  w.k_adj = take(rows * d);
  w.a_op = take(rows * d);
  w.b_op = take(rows * d);
  w.g = take(rows * d);
  w.y = take(rows * d);
  w.tmp = take(rows * d);
  w.rosa = take(rows * 3 * R);
  w.read = take(rows * R);
  w.h = take(rows * 4 * d);
  {  // 16-byte alignment for the scans' cp.async / float4 accesses
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    p = reinterpret_cast<float*>((a + 15) & ~uintptr_t(15));
  }
  w.scan = decode_only ? nullptr : take(scan_scratch_floats(m, rows));
  uintptr_t u = reinterpret_cast<uintptr_t>(p);
  u = (u + 255) & ~uintptr_t(255);
  w.bf = reinterpret_cast<__nv_bfloat16*>(u);
  return w;
}

static void dump(yuf_model* m, const char* region, int layer, const float* dev, size_t n,
                 cudaStream_t s) {
  if (!m->debug) return;
  if (!m->debug_regions.empty() &&
      std::find(m->debug_regions.begin(), m->debug_regions.end(), region) == m->debug_regions.end())
    return;
  if (layer >= 0 && !m->debug_layers.empty() &&
      (layer >= (int)m->debug_layers.size() || !m->debug_layers[layer]))
    return;
  auto& v = m->dumps[region];
  if ((int)v.size() <= layer + 1) v.resize(layer + 2);
  auto& h = v[layer + 1];
  h.resize(n);
  cudaMemcpyAsync(h.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost, s);
  cudaStreamSynchronize(s);
}

// One forward over B sequences x T tokens (rows = B*T), state slots [slot0, slot0+B).
// ws_base: workspace to carve the row buffers from; nullptr = the model's own
// (grown on demand).
static yuf_status_t forward(yuf_model* m, const int32_t* ids, int B, int T, int slot0,
                            float* logits_last, float* logits_all, cudaStream_t s,
                            void* ws_base = nullptr) {
  const size_t rows = (size_t)B * T;
  const int d = m->d(), H = m->H(), N = m->N(), R = m->R(), lr = m->lr(), V = m->V();
  // a decode step is a chain of small dependent kernels: launch them with
  // programmatic dependent launch (each kernel's start overlaps its predecessor)
  PdlScope pdl(T == 1 && !m->debug);
  // a caller-supplied workspace serves a decode step only (sized by ws_bytes(.., true))
  const bool caller_ws = ws_base != nullptr;
  if (!caller_ws) {
    Y_TRY(ensure_ws(m, rows));
    ws_base = m->ws->p;
  }
  WS w = carve(m, rows, ws_base, caller_ws);
  launch_embed(ids, m->emb, w.x, (int)rows, d, V, m->d_err, s);
  const size_t RD = rows * d;
  // bf16-weight mode: the producers of GEMM inputs (mixes, layer norms, the FFN
  // gate) write bf16 straight into the staging buffer instead of fp32 plus a copy
  const bool bf = m->precision == YUF_PRECISION_BF16_WEIGHTS;
  auto ln_in = [&](const float* x, const float* lw, const float* lb, const float* gate,
                   bool gate_sig = false) -> const void* {
    if (bf) {
      launch_layernorm<__nv_bfloat16>(x, lw, lb, gate, w.bf, (int)rows, d, s, gate_sig);
      return w.bf;
    }
    launch_layernorm<float>(x, lw, lb, gate, w.tmp, (int)rows, d, s, gate_sig);
    return w.tmp;
  };
  for (int li = 0; li < m->cfg.n_layers; ++li) {
    const LayerW& Lw = m->L[li];
    float* prev = m->st_prev + ((size_t)li * m->n_slots + slot0) * m->slot_prev();
    float* S = m->st_S + ((size_t)li * m->n_slots + slot0) * m->slot_S();
    float* mem = m->st_m + ((size_t)li * m->n_slots + slot0) * m->slot_m();
    // --- TimeMix
    const void* mixed = bf ? static_cast<const void*>(w.bf) : w.mixed;
    const bool fused_mix =
        T == 1 && (bf ? launch_ln_mix_step<__nv_bfloat16>(w.x, Lw.ln_t_w, Lw.ln_t_b, w.xt, prev,
                                                           Lw.mix, w.bf, B, d, s)
                      : launch_ln_mix_step<float>(w.x, Lw.ln_t_w, Lw.ln_t_b, w.xt, prev, Lw.mix,
                                                  w.mixed, B, d, s));
    if (!fused_mix) {
      // one pass for the norm, the shift and the lerps; debug runs keep the
      // separate norm so that every row's xt can be dumped
      const bool fused_rows =
          !m->debug && (bf ? launch_ln_mix_rows<__nv_bfloat16>(w.x, Lw.ln_t_w, Lw.ln_t_b, w.xt, prev, Lw.mix,
                                                               w.bf, B, T, d, s)
                           : launch_ln_mix_rows<float>(w.x, Lw.ln_t_w, Lw.ln_t_b, w.xt, prev, Lw.mix, w.mixed,
                                                       B, T, d, s));
      if (!fused_rows) {
        launch_layernorm<float>(w.x, Lw.ln_t_w, Lw.ln_t_b, nullptr, w.xt, (int)rows, d, s);
        if (bf)
          launch_mix<__nv_bfloat16>(w.xt, prev, Lw.mix, w.bf, B, T, d, s);
        else
          launch_mix<float>(w.xt, prev, Lw.mix, w.mixed, B, T, d, s);
      }
      Y_CUDA(cudaMemcpy2DAsync(prev, d * sizeof(float), w.xt + (size_t)(T - 1) * d,
                               (size_t)T * d * sizeof(float), d * sizeof(float), B,
                               cudaMemcpyDeviceToDevice, s));
    }
    const size_t esz = m->precision == YUF_PRECISION_BF16_WEIGHTS ? 2 : 4;
    const char* mixed_hi = static_cast<const char*>(mixed) + 3 * RD * esz;  // w, a, g mixes
    // r, k, v; then x_{w,a,g} L1 with tanh on the w branch (bf16 in bf16 mode),
    // written into the lr1 buffer, which feeds L2.  A decode step runs the two
    // low-rank projections on the side stream, concurrently with r, k, v.
    const bool fork = T == 1 && m->side != nullptr;
    cudaStream_t s_lr = fork ? m->side : s;
    if (fork) {
      Y_CUDA(cudaEventRecord(m->ev_fork, s));
      Y_CUDA(cudaStreamWaitEvent(m->side, m->ev_fork, 0));
    }
    Y_TRY(proj(m, mixed_hi, d, (long long)rows, Lw.W_lr1, lr, w.lr1, lr, (long long)rows * lr, (int)rows, lr,
               d, 3, GEMM_EPI_BF16, false, s_lr, 0, true));
    Y_TRY(proj(m, w.lr1, lr, (long long)rows, Lw.W_lr2, d, w.lr2, d, RD, (int)rows, d, lr, 3, GEMM_EPI_F32,
               false, s_lr));
    Y_TRY(proj(m, mixed, d, (long long)rows, Lw.W_rkv, d, w.rkv, d, RD, (int)rows, d, d, 3, GEMM_EPI_F32,
               false, s));
    if (fork) {
      Y_CUDA(cudaEventRecord(m->ev_join, m->side));
      Y_CUDA(cudaStreamWaitEvent(s, m->ev_join, 0));
    }
    // The decode step and the prefill scans (chunked tensor-core, and the first
    // pass of the time-parallel one) fold the time-mix epilogue into the WKV
    // kernel (no separate pass over the projections' outputs); a prefill leaves
    // the output gate to the output norm, which takes sigmoid(lg) itself.  Debug runs keep the epilogue separate, so
    // that its outputs can be dumped.
    yuf_status_t tm_st = YUF_ERR_UNSUPPORTED;
    const float* out_gate = w.g;
    bool out_gate_sig = false;
    if (!m->debug) {
      if (T == 1) {
        tm_st = wkv7_decode_tm_dispatch(w.rkv, w.rkv + RD, w.rkv + 2 * RD, w.lr2, w.lr2 + RD, w.lr2 + 2 * RD,
                                        Lw.w0, Lw.a0, Lw.k_k, Lw.k_a, w.g, S, w.y, S, B * H, H, N, s);
      } else if (wkv7_chunk_tc_applies(B, T, H, N)) {
        tm_st = wkv7_chunk_tc_tm(w.rkv, w.rkv + RD, w.rkv + 2 * RD, w.lr2, w.lr2 + RD, Lw.w0, Lw.a0, Lw.k_k,
                                 Lw.k_a, S, w.y, S, B, T, H, N, s);
      } else if (wkv7_parallel_applies(B, T, H, N)) {
        const WkvTm prm{Lw.w0, Lw.a0, Lw.k_k, Lw.k_a};
        tm_st = wkv7_parallel(w.rkv, w.lr2, w.rkv + RD, w.rkv + 2 * RD, w.lr2 + RD, w.lr2 + RD, S, w.y, S, B, T,
                              H, N, w.scan + scan_rosa_floats(m, rows), s, false, &prm);
      }
      if (T > 1 && tm_st != YUF_ERR_UNSUPPORTED) {
        out_gate = w.lr2 + 2 * RD;
        out_gate_sig = true;
      }
    }
    if (tm_st != YUF_ERR_UNSUPPORTED) {
      Y_TRY(tm_st);
    } else {
      launch_timemix_post(w.rkv + RD, w.lr2, w.lr2 + RD, w.lr2 + 2 * RD, Lw.w0, Lw.a0, Lw.k_k, Lw.k_a,
                          w.w_raw, w.k_adj, w.a_op, w.b_op, w.g, (int)rows, H, N, s);
      if (T == 1)
        Y_TRY(wkv7_decode_dispatch(w.rkv, w.w_raw, w.k_adj, w.rkv + 2 * RD, w.a_op, w.b_op, S, w.y, S,
                                   B * H, N, s));
      else if (wkv7_chunk_tc_applies(B, T, H, N))
        Y_TRY(wkv7_chunk_tc(w.rkv, w.w_raw, w.k_adj, w.rkv + 2 * RD, w.a_op, w.b_op, S, w.y, S, B, T, H, N,
                            s));
      else if (wkv7_parallel_applies(B, T, H, N))
        Y_TRY(wkv7_parallel(w.rkv, w.w_raw, w.k_adj, w.rkv + 2 * RD, w.a_op, w.b_op, S, w.y, S, B, T, H,
                            N, w.scan + scan_rosa_floats(m, rows), s));
      else
        Y_TRY(wkv7_dispatch(w.rkv, w.w_raw, w.k_adj, w.rkv + 2 * RD, w.a_op, w.b_op, S, w.y, S, nullptr,
                            nullptr, B, T, H, N, false, s));
    }
    const void* att = ln_in(w.y, Lw.ln_o_w, Lw.ln_o_b, out_gate, out_gate_sig);
    if (m->debug) {
      dump(m, "ln0", li, w.xt, RD, s);
      dump(m, "r", li, w.rkv, RD, s);
      dump(m, "w", li, w.w_raw, RD, s);
      dump(m, "k", li, w.k_adj, RD, s);
      dump(m, "v", li, w.rkv + 2 * RD, RD, s);
      dump(m, "a", li, w.a_op, RD, s);
      dump(m, "b", li, w.b_op, RD, s);
      dump(m, "g", li, w.g, RD, s);
      dump(m, "y", li, w.y, RD, s);
    }
    // x += W_o (LN_out(y) * g)
    Y_TRY(proj(m, att, d, 0, Lw.W_o, 0, w.x, d, 0, (int)rows, d, d, 1, GEMM_EPI_F32, true, s));
    if (m->debug) dump(m, "h1", li, w.x, RD, s);
    // --- ROSA: [cand | write | gate] = LN_rosa(x) W^T, scan, x += read W_out^T
    const void* xr = ln_in(w.x, Lw.ln_r_w, Lw.ln_r_b, nullptr);
    Y_TRY(proj(m, xr, d, 0, Lw.W_rosa_in, 0, w.rosa, 3 * R, 0, (int)rows, 3 * R, d, 1, GEMM_EPI_F32, false, s));
    Y_TRY(rosa_engine_dispatch(w.rosa, w.rosa + R, w.rosa + 2 * R, Lw.b_rosa, Lw.b_rosa + R,
                               Lw.b_rosa + 2 * R, 3 * R, Lw.decay, Lw.householder, mem, w.read, mem, B,
                               T, R, w.scan, bf ? w.bf : nullptr, s, Lw.rosa_factors));
    if (m->debug) dump(m, "read", li, w.read, rows * R, s);
    Y_TRY(proj(m, bf ? static_cast<const void*>(w.bf) : w.read, R, 0, Lw.W_rosa_out, 0, w.x, d, 0, (int)rows,
               d, R, 1, GEMM_EPI_F32, true, s));
    if (m->debug) dump(m, "h2", li, w.x, RD, s);
    // --- FFN: x += W_out(SiLU(x_f W_in^T) * (x_f W_g^T))
    const void* xf = ln_in(w.x, Lw.ln_f_w, Lw.ln_f_b, nullptr);
    // the hidden leaves the GEMM through the SiLU-gate epilogue into the h buffer
    Y_TRY(proj(m, xf, d, 0, Lw.W_ffn_in, 0, w.h, 4 * d, 0, (int)rows, 2 * ffn_pad(d), d, 1, GEMM_EPI_SWIGLU,
               false, s, 4 * d));
    Y_TRY(proj(m, w.h, 4 * d, 0, Lw.W_ffn_out, 0, w.x, d, 0, (int)rows, d, 4 * d, 1, GEMM_EPI_F32, true, s));
    if (m->debug) dump(m, "h3", li, w.x, RD, s);
  }
  // final norm + tied LM head
  const void* hn = ln_in(w.x, m->fin_w, m->fin_b, nullptr);
  const size_t esz = bf ? 2 : 4;
  if (logits_all)
    Y_TRY(proj(m, hn, d, 0, m->emb_gemm, 0, logits_all, V, 0, (int)rows, V, d, 1, GEMM_EPI_F32, false, s));
  if (logits_last) {
    const void* last = static_cast<const char*>(hn) + (size_t)(T - 1) * d * esz;
    Y_TRY(proj(m, last, (long long)T * d, 0, m->emb_gemm, 0, logits_last, V, 0, B, V, d, 1, GEMM_EPI_F32, false,
               s));
    if (m->debug) dump(m, "logits", -1, logits_last, (size_t)B * V, s);
  }
  return check_launch("model forward");
}

// ---------------------------------------------------------------- loading
struct HostTensor {
  const float* p;
  int64_t n;
};

static yuf_status_t upload(yuf_model* m, const std::unordered_map<std::string, HostTensor>& t,
                           const std::string& name, int64_t n, float** out) {
  auto it = t.find(name);
  Y_REQUIRE(it != t.end(), "model: missing tensor %s", name.c_str());
  Y_REQUIRE(it->second.n == n, "model: tensor %s has %lld elements, expected %lld", name.c_str(),
            (long long)it->second.n, (long long)n);
  float* d = static_cast<float*>(m->alloc(n * sizeof(float)));
  if (!d) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
  Y_CUDA(cudaMemcpy(d, it->second.p, n * sizeof(float), cudaMemcpyHostToDevice));
  *out = d;
  return YUF_OK;
}

// A packed host fp32 weight to the device in the model precision: bf16, or
// the tf32 high part and the remainder (two planes) for fp32 mode.
static yuf_status_t upload_weight(yuf_model* m, const std::vector<float>& host, Wt* out) {
  const size_t total = host.size();
  if (m->precision == YUF_PRECISION_BF16_WEIGHTS) {
    std::vector<__nv_bfloat16> hb(total);
    for (size_t i = 0; i < total; ++i) hb[i] = __float2bfloat16_rn(host[i]);
    void* d = m->alloc(total * 2);
    if (!d) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
    Y_CUDA(cudaMemcpy(d, hb.data(), total * 2, cudaMemcpyHostToDevice));
    out->hi = d;
    out->lo = nullptr;
  } else {
    std::vector<float> hl(2 * total);
    split_tf32_host(host.data(), total, hl.data(), hl.data() + total);
    float* d = static_cast<float*>(m->alloc(2 * total * 4));
    if (!d) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
    Y_CUDA(cudaMemcpy(d, hl.data(), 2 * total * 4, cudaMemcpyHostToDevice));
    out->hi = d;
    out->lo = d + total;
  }
  return YUF_OK;
}

// Pack host fp32 matrices (each [rows_i, K], row-major) into one GEMM weight in
// the model precision.  transpose: the source is [K, rows] (a Parameter used as
// x @ P, model.py:108-112) and is transposed to [rows, K].
static yuf_status_t pack_weight(yuf_model* m, const std::unordered_map<std::string, HostTensor>& t,
                                const std::vector<std::string>& names, const std::vector<int>& rows,
                                int K, bool transpose, Wt* out) {
  size_t total = 0;
  for (int r : rows) total += (size_t)r * K;
  std::vector<float> host(total);
  size_t off = 0;
  for (size_t i = 0; i < names.size(); ++i) {
    auto it = t.find(names[i]);
    Y_REQUIRE(it != t.end(), "model: missing tensor %s", names[i].c_str());
    Y_REQUIRE(it->second.n == (int64_t)rows[i] * K, "model: tensor %s has %lld elements, expected %lld",
              names[i].c_str(), (long long)it->second.n, (long long)rows[i] * K);
    const float* src = it->second.p;
    if (!transpose) {
      std::memcpy(host.data() + off, src, (size_t)rows[i] * K * sizeof(float));
    } else {
      for (int r = 0; r < rows[i]; ++r)
        for (int k = 0; k < K; ++k) host[off + (size_t)r * K + k] = src[(size_t)k * rows[i] + r];
    }
    off += (size_t)rows[i] * K;
  }
  return upload_weight(m, host, out);
}

// ffn_in.weight and ffn_gate.weight ([F, d] each) interleaved in 64-row groups
// -- rows 128g .. 128g+63 = ffn_in rows 64g .., rows 128g+64 .. 128g+127 = the
// same ffn_gate rows -- with F padded to a multiple of 64 by zero rows, the
// layout the GEMM's SiLU-gate epilogue pairs columns in.
static yuf_status_t pack_ffn_in(yuf_model* m, const std::unordered_map<std::string, HostTensor>& t,
                                const std::string& in_name, const std::string& gate_name, Wt* out) {
  const int d = m->d(), F = 4 * d, Fp = ffn_pad(d);
  auto in = t.find(in_name), gate = t.find(gate_name);
  Y_REQUIRE(in != t.end() && gate != t.end(), "model: missing tensor %s or %s", in_name.c_str(),
            gate_name.c_str());
  Y_REQUIRE(in->second.n == (int64_t)F * d && gate->second.n == (int64_t)F * d,
            "model: %s / %s must hold %lld elements", in_name.c_str(), gate_name.c_str(), (long long)F * d);
  std::vector<float> host((size_t)2 * Fp * d, 0.f);
  for (int r = 0; r < F; ++r) {
    const size_t dst_in = ((size_t)(r / 64) * 128 + r % 64) * d, dst_gate = dst_in + (size_t)64 * d;
    std::memcpy(host.data() + dst_in, in->second.p + (size_t)r * d, (size_t)d * 4);
    std::memcpy(host.data() + dst_gate, gate->second.p + (size_t)r * d, (size_t)d * 4);
  }
  return upload_weight(m, host, out);
}

static yuf_status_t load_weights(yuf_model* m, const std::unordered_map<std::string, HostTensor>& t) {
  const int d = m->d(), R = m->R(), lr = m->lr(), V = m->V(), F = 4 * d;
  Y_TRY(upload(m, t, "token_embedding.weight", (int64_t)V * d, &m->emb));
  Y_TRY(upload(m, t, "final_norm.weight", d, &m->fin_w));
  Y_TRY(upload(m, t, "final_norm.bias", d, &m->fin_b));
  auto lm = t.find("lm_head.weight");
  if (lm != t.end() && lm->second.p != t.at("token_embedding.weight").p) {
    // A separate head is only meaningful untied; the reference ties them.
    Y_REQUIRE(std::memcmp(lm->second.p, t.at("token_embedding.weight").p, (size_t)V * d * 4) == 0,
              "model: lm_head.weight differs from token_embedding.weight (untied heads unsupported)");
  }
  Y_TRY(pack_weight(m, t, {"token_embedding.weight"}, {V}, d, false, &m->emb_gemm));
  m->L.resize(m->cfg.n_layers);
  for (int i = 0; i < m->cfg.n_layers; ++i) {
    LayerW& Lw = m->L[i];
    const std::string p = "blocks." + std::to_string(i) + ".";
    const std::string tm = p + "time_mix.", ro = p + "rosa.";
    Y_TRY(upload(m, t, p + "norm_time.weight", d, &Lw.ln_t_w));
    Y_TRY(upload(m, t, p + "norm_time.bias", d, &Lw.ln_t_b));
    {  // mix rows in the reference order r, w, k, v, a, g
      std::vector<float> mix(6 * (size_t)d);
      const char* names[6] = {"mix_r", "mix_w", "mix_k", "mix_v", "mix_a", "mix_g"};
      for (int c = 0; c < 6; ++c) {
        auto it = t.find(tm + names[c]);
        Y_REQUIRE(it != t.end() && it->second.n == d, "model: bad tensor %s%s", tm.c_str(), names[c]);
        std::memcpy(mix.data() + (size_t)c * d, it->second.p, d * 4);
      }
      Lw.mix = static_cast<float*>(m->alloc(mix.size() * 4));
      if (!Lw.mix) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
      Y_CUDA(cudaMemcpy(Lw.mix, mix.data(), mix.size() * 4, cudaMemcpyHostToDevice));
    }
    Y_TRY(upload(m, t, tm + "w0", d, &Lw.w0));
    Y_TRY(upload(m, t, tm + "a0", d, &Lw.a0));
    Y_TRY(upload(m, t, tm + "k_k", d, &Lw.k_k));
    Y_TRY(upload(m, t, tm + "k_a", d, &Lw.k_a));
    Y_TRY(pack_weight(m, t, {tm + "receptance.weight", tm + "key.weight", tm + "value.weight"},
                      {d, d, d}, d, false, &Lw.W_rkv));
    Y_TRY(pack_weight(m, t, {tm + "w1", tm + "a1", tm + "g1"}, {lr, lr, lr}, d, true, &Lw.W_lr1));
    Y_TRY(pack_weight(m, t, {tm + "w2", tm + "a2", tm + "g2"}, {d, d, d}, lr, true, &Lw.W_lr2));
    Y_TRY(pack_weight(m, t, {tm + "output.weight"}, {d}, d, false, &Lw.W_o));
    Y_TRY(upload(m, t, tm + "out_norm.weight", d, &Lw.ln_o_w));
    Y_TRY(upload(m, t, tm + "out_norm.bias", d, &Lw.ln_o_b));
    Y_TRY(upload(m, t, p + "norm_rosa.weight", d, &Lw.ln_r_w));
    Y_TRY(upload(m, t, p + "norm_rosa.bias", d, &Lw.ln_r_b));
    Y_TRY(upload(m, t, ro + "householder", R, &Lw.householder));
    Y_TRY(upload(m, t, ro + "decay", R, &Lw.decay));
    if (R <= 256) {  // the time-parallel scan's constants depend on these two parameters only
      Lw.rosa_factors = static_cast<float*>(m->alloc(rosa_factor_floats(R) * sizeof(float)));
      if (!Lw.rosa_factors) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
      Y_TRY(rosa_prepare_factors(Lw.decay, Lw.householder, 1, R, Lw.rosa_factors, nullptr));
      Y_CUDA(cudaStreamSynchronize(nullptr));
    }
    Y_TRY(pack_weight(m, t, {ro + "input.weight", ro + "write_gate.weight", ro + "read_gate.weight"},
                      {R, R, R}, d, false, &Lw.W_rosa_in));
    {
      std::vector<float> bias(3 * (size_t)R);
      const char* names[3] = {"input.bias", "write_gate.bias", "read_gate.bias"};
      for (int c = 0; c < 3; ++c) {
        auto it = t.find(ro + names[c]);
        Y_REQUIRE(it != t.end() && it->second.n == R, "model: bad tensor %s%s", ro.c_str(), names[c]);
        std::memcpy(bias.data() + (size_t)c * R, it->second.p, R * 4);
      }
      Lw.b_rosa = static_cast<float*>(m->alloc(bias.size() * 4));
      if (!Lw.b_rosa) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
      Y_CUDA(cudaMemcpy(Lw.b_rosa, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice));
    }
    Y_TRY(pack_weight(m, t, {ro + "output.weight"}, {d}, R, false, &Lw.W_rosa_out));
    Y_TRY(upload(m, t, p + "norm_ffn.weight", d, &Lw.ln_f_w));
    Y_TRY(upload(m, t, p + "norm_ffn.bias", d, &Lw.ln_f_b));
    Y_TRY(pack_ffn_in(m, t, p + "ffn_in.weight", p + "ffn_gate.weight", &Lw.W_ffn_in));
    Y_TRY(pack_weight(m, t, {p + "ffn_out.weight"}, {d}, F, false, &Lw.W_ffn_out));
  }
  return YUF_OK;
}

static yuf_status_t validate_cfg(yuf_model_config* c) {
  Y_REQUIRE(c->d_model == c->n_heads * c->head_size, "model: d_model must equal n_heads * head_size");
  Y_REQUIRE(c->d_model >= 32 && c->n_layers >= 1, "model: model is too small to be useful");
  Y_REQUIRE(c->d_model % 8 == 0, "model: d_model must be a multiple of 8");
  Y_REQUIRE(c->vocab_size > 0 && c->rosa_size >= 1 && c->rosa_size <= 1024, "model: bad vocab/rosa size");
  if (c->low_rank <= 0) c->low_rank = reference_low_rank(c->d_model);
  Y_REQUIRE(c->low_rank <= 4 * c->d_model && c->low_rank % 8 == 0,
            "model: low_rank %d must be a multiple of 8 and at most 4 * d_model", c->low_rank);
  return YUF_OK;
}

yuf_status_t model_create_from_map(const yuf_model_config* cfg, int precision, int device,
                                   const std::unordered_map<std::string, HostTensor>& t,
                                   yuf_model** out) {
  Y_REQUIRE(cfg && out, "model: null argument");
  Y_REQUIRE(precision == YUF_PRECISION_FP32 || precision == YUF_PRECISION_BF16_WEIGHTS,
            "model: unknown precision %d", precision);
  yuf_model_config c = *cfg;
  Y_TRY(validate_cfg(&c));
  if (c.rosa_size % (precision == YUF_PRECISION_BF16_WEIGHTS ? 8 : 4) != 0) {
    set_error("model: rosa_size %d must be a multiple of %d in this precision (16-byte rows for the "
              "tensor-core GEMM)", c.rosa_size, precision == YUF_PRECISION_BF16_WEIGHTS ? 8 : 4);
    return YUF_ERR_UNSUPPORTED;
  }
  switch (c.head_size) {
    case 16: case 32: case 40: case 48: case 64: case 96: case 128: break;
    default: set_error("model: head_size %d has no kernel", c.head_size); return YUF_ERR_UNSUPPORTED;
  }
  Y_CUDA(cudaSetDevice(device));
  auto m = std::make_unique<yuf_model>();
  m->cfg = c;
  m->precision = precision;
  m->device = device;
  m->d_err = static_cast<int*>(m->alloc(sizeof(int)));
  if (!m->d_err) { set_error("model: out of device memory"); return YUF_ERR_OUT_OF_MEMORY; }
  Y_CUDA(cudaMemset(m->d_err, 0, sizeof(int)));
  Y_CUDA(cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking));
  Y_CUDA(cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming));
  Y_CUDA(cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming));
  Y_TRY(load_weights(m.get(), t));
  *out = m.release();
  return YUF_OK;
}

}  // namespace yuf

extern "C" {

yuf_status_t yuf_model_create(const yuf_model_config* cfg, int precision, int device, int n_tensors,
                              const char* const* names, const float* const* host_data,
                              const int64_t* numels, yuf_model** out) {
  Y_REQUIRE(n_tensors >= 0 && (n_tensors == 0 || (names && host_data && numels)), "model: bad tensor list");
  std::unordered_map<std::string, HostTensor> t;
  for (int i = 0; i < n_tensors; ++i) {
    Y_REQUIRE(names[i] && host_data[i], "model: tensor %d has a null name or pointer", i);
    t[names[i]] = HostTensor{host_data[i], numels[i]};
  }
  return model_create_from_map(cfg, precision, device, t, out);
}

yuf_status_t yuf_model_destroy(yuf_model* m) {
  if (!m) return YUF_OK;
  cudaSetDevice(m->device);
  m->drop_graphs();
  delete m;
  return YUF_OK;
}

yuf_status_t yuf_model_get_config(const yuf_model* m, yuf_model_config* out) {
  Y_REQUIRE(m && out, "model: null argument");
  *out = m->cfg;
  return YUF_OK;
}

yuf_status_t yuf_state_alloc(yuf_model* m, int n_slots) {
  Y_REQUIRE(m && n_slots >= 1, "state: need at least one slot");
  Y_CUDA(cudaSetDevice(m->device));
  const size_t Lr = m->cfg.n_layers, n = n_slots;
  float* p = static_cast<float*>(m->alloc(Lr * n * m->slot_prev() * 4));
  float* S = static_cast<float*>(m->alloc(Lr * n * m->slot_S() * 4));
  float* mm = static_cast<float*>(m->alloc(Lr * n * m->slot_m() * 4));
  if (!p || !S || !mm) { set_error("state: out of device memory for %d slots", n_slots); return YUF_ERR_OUT_OF_MEMORY; }
  Y_CUDA(cudaMemset(p, 0, Lr * n * m->slot_prev() * 4));
  Y_CUDA(cudaMemset(S, 0, Lr * n * m->slot_S() * 4));
  Y_CUDA(cudaMemset(mm, 0, Lr * n * m->slot_m() * 4));
  m->st_prev = p;
  m->st_S = S;
  m->st_m = mm;
  m->n_slots = n_slots;
  return YUF_OK;
}

yuf_status_t yuf_state_reset(yuf_model* m, int slot0, int n, void* stream) {
  Y_REQUIRE(m && m->n_slots > 0, "state: no slots allocated");
  Y_REQUIRE(slot0 >= 0 && n >= 0 && slot0 + n <= m->n_slots, "state: slots [%d, %d) out of range", slot0, slot0 + n);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int li = 0; li < m->cfg.n_layers; ++li) {
    const size_t base = (size_t)li * m->n_slots + slot0;
    Y_CUDA(cudaMemsetAsync(m->st_prev + base * m->slot_prev(), 0, n * m->slot_prev() * 4, s));
    Y_CUDA(cudaMemsetAsync(m->st_S + base * m->slot_S(), 0, n * m->slot_S() * 4, s));
    Y_CUDA(cudaMemsetAsync(m->st_m + base * m->slot_m(), 0, n * m->slot_m() * 4, s));
  }
  return YUF_OK;
}

static yuf_status_t state_copy(yuf_model* m, int layer, int slot0, int n, float* prev, float* S,
                               float* mm, bool to_model, cudaStream_t s) {
  Y_REQUIRE(m && m->n_slots > 0, "state: no slots allocated");
  Y_REQUIRE(layer >= 0 && layer < m->cfg.n_layers, "state: layer %d out of range", layer);
  Y_REQUIRE(slot0 >= 0 && n >= 0 && slot0 + n <= m->n_slots, "state: slots out of range");
  const size_t base = (size_t)layer * m->n_slots + slot0;
  struct { float* mine; float* theirs; size_t per; } parts[3] = {
      {m->st_prev + base * m->slot_prev(), prev, m->slot_prev()},
      {m->st_S + base * m->slot_S(), S, m->slot_S()},
      {m->st_m + base * m->slot_m(), mm, m->slot_m()}};
  for (auto& pt : parts) {
    if (!pt.theirs) continue;
    if (to_model)
      Y_CUDA(cudaMemcpyAsync(pt.mine, pt.theirs, n * pt.per * 4, cudaMemcpyDeviceToDevice, s));
    else
      Y_CUDA(cudaMemcpyAsync(pt.theirs, pt.mine, n * pt.per * 4, cudaMemcpyDeviceToDevice, s));
  }
  return YUF_OK;
}

yuf_status_t yuf_state_export(yuf_model* m, int layer, int slot0, int n, float* prev, float* S,
                              float* mm, void* stream) {
  return state_copy(m, layer, slot0, n, prev, S, mm, false, static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_state_import(yuf_model* m, int layer, int slot0, int n, const float* prev,
                              const float* S, const float* mm, void* stream) {
  return state_copy(m, layer, slot0, n, const_cast<float*>(prev), const_cast<float*>(S),
                    const_cast<float*>(mm), true, static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_prefill(yuf_model* m, const int32_t* ids, int B, int T, int slot0,
                         float* logits_last, float* logits_all, void* stream) {
  Y_REQUIRE(m, "prefill: null model");
  Y_REQUIRE(m->n_slots > 0, "prefill: call yuf_state_alloc first");
  Y_REQUIRE(B >= 1 && T >= 1 && ids, "prefill: need B >= 1, T >= 1 and ids");
  Y_REQUIRE(slot0 >= 0 && slot0 + B <= m->n_slots, "prefill: slots [%d, %d) out of range (%d slots)",
            slot0, slot0 + B, m->n_slots);
  Y_CUDA(cudaSetDevice(m->device));
  return forward(m, ids, B, T, slot0, logits_last, logits_all, static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_step(yuf_model* m, const int32_t* ids, int B, int slot0, float* logits, void* stream) {
  Y_REQUIRE(m, "step: null model");
  Y_REQUIRE(m->n_slots > 0, "step: call yuf_state_alloc first");
  Y_REQUIRE(B >= 1 && ids && logits, "step: need B >= 1, ids and logits");
  Y_REQUIRE(slot0 >= 0 && slot0 + B <= m->n_slots, "step: slots [%d, %d) out of range (%d slots)",
            slot0, slot0 + B, m->n_slots);
  Y_CUDA(cudaSetDevice(m->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!m->decode_graphs || s == nullptr || m->debug) return forward(m, ids, B, 1, slot0, logits, nullptr, s);
  // Replay a captured graph of this exact step (same batch, slots and buffers).
  Y_TRY(ensure_ws(m, (size_t)B));
  for (auto& g : m->graphs)
    if (g.B == B && g.slot0 == slot0 && g.ids == ids && g.logits == logits && g.ws_gen == m->ws_gen) {
      Y_CUDA(cudaGraphLaunch(g.exec, s));
      return YUF_OK;
    }
  cudaGraph_t graph = nullptr;
  Y_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  yuf_status_t st = forward(m, ids, B, 1, slot0, logits, nullptr, s);
  cudaError_t e = cudaStreamEndCapture(s, &graph);
  if (st != YUF_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (e != cudaSuccess) {
    set_error("step: graph capture failed: %s", cudaGetErrorString(e));
    return YUF_ERR_CUDA;
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    set_error("step: graph instantiation failed: %s", cudaGetErrorString(e));
    return YUF_ERR_CUDA;
  }
  if (m->graphs.size() >= 64) m->drop_graphs();
  m->graphs.push_back({B, slot0, ids, logits, m->ws_gen, exec});
  Y_CUDA(cudaGraphLaunch(exec, s));
  return YUF_OK;
}

}  // extern "C"

namespace yuf {
// Step s of yuf_generate: record the sampled ids and end a sequence at its first
// EOS.  lengths[b] == n_steps means "still running" (set at step 0); an ended
// sequence records eos_id and is fed eos_id from then on.
__global__ void gen_record_kernel(int32_t* __restrict__ ids, int32_t* __restrict__ tokens,
                                  int32_t* __restrict__ lengths, int B, int n_steps, int s,
                                  int eos_id) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int len = s == 0 ? n_steps : lengths[b];
  int tok = ids[b];
  if (len != n_steps) tok = eos_id;                      // ended at an earlier step
  else if (eos_id >= 0 && tok == eos_id) len = s;        // ends now
  tokens[(size_t)b * n_steps + s] = len != n_steps ? eos_id : tok;
  ids[b] = tok;
  lengths[b] = len;
}
}  // namespace yuf

extern "C" {

yuf_status_t yuf_generate(yuf_model* m, const int32_t* prompt_ids, int B, int T, int slot0,
                          int n_steps, const yuf_generate_params* p, int32_t* tokens,
                          int32_t* lengths, void* stream) {
  Y_REQUIRE(m && p, "generate: null model or params");
  Y_REQUIRE(m->n_slots > 0, "generate: call yuf_state_alloc first");
  Y_REQUIRE(B >= 1 && T >= 1 && n_steps >= 1, "generate: need B, T and n_steps >= 1 (got %d, %d, %d)",
            B, T, n_steps);
  Y_REQUIRE(prompt_ids && tokens && lengths, "generate: prompt_ids, tokens and lengths must be non-NULL");
  Y_REQUIRE(slot0 >= 0 && slot0 + B <= m->n_slots, "generate: slots [%d, %d) out of range (%d slots)",
            slot0, slot0 + B, m->n_slots);
  Y_REQUIRE(p->top_k >= 1 && p->top_k <= 1024, "generate: top_k must be in [1, 1024] (got %d)", p->top_k);
  Y_REQUIRE(std::isfinite(p->temperature) && std::isfinite(p->top_p) && p->top_p > 0.f,
            "generate: temperature must be finite and top_p finite and > 0");
  Y_REQUIRE(p->seq0 >= 0, "generate: seq0 must be >= 0");
  Y_REQUIRE(p->mask_below >= 0 && p->mask_below < m->V(), "generate: mask_below must be in [0, %d)", m->V());
  Y_REQUIRE(p->eos_id >= -1 && p->eos_id < m->V(), "generate: eos_id must be -1 or in [0, %d)", m->V());
  Y_REQUIRE(p->min_tokens_before_eos >= 0, "generate: min_tokens_before_eos must be >= 0");
  Y_CUDA(cudaSetDevice(m->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t V = m->V();
  const size_t logit_bytes = ((size_t)B * V * 4 + 255) / 256 * 256;
  const size_t need = logit_bytes + (size_t)B * 4;
  if (!m->gen || m->gen->bytes < need) {
    if (m->gen) Y_CUDA(cudaStreamSynchronize(s));  // queued work may still read the old buffers
    auto buf = std::make_unique<DevBuf>();
    if (cudaMalloc(&buf->p, need) != cudaSuccess) {
      cudaGetLastError();
      set_error("generate: out of device memory for %zu bytes of working buffers", need);
      return YUF_ERR_OUT_OF_MEMORY;
    }
    buf->bytes = need;
    m->gen = std::move(buf);
  }
  float* logits = static_cast<float*>(m->gen->p);
  int32_t* ids = reinterpret_cast<int32_t*>(static_cast<char*>(m->gen->p) + logit_bytes);
  Y_TRY(yuf_prefill(m, prompt_ids, B, T, slot0, logits, nullptr, stream));
  const int eos_for_mask = p->eos_id >= 0 ? p->eos_id : 0;
  const float top_p = std::min(p->top_p, 1.f);  // >= 1 keeps the whole top-k
  PdlScope pdl(true);  // sampling and recording join the decode steps' launch chain
  for (int st = 0; st < n_steps; ++st) {
    const int allow_eos = p->eos_id >= 0 && st >= p->min_tokens_before_eos;
    Y_TRY(yuf_sample(logits, B, (int)V, p->temperature, p->top_k, top_p, p->seed, (uint64_t)st,
                     p->seq0, p->mask_below, eos_for_mask, allow_eos, ids, nullptr, stream));
    launch_k(gen_record_kernel, dim3((B + 127) / 128), dim3(128), 0, s, ids, tokens, lengths, B, n_steps, st, p->eos_id);
    Y_CUDA(cudaGetLastError());
    Y_TRY(yuf_step(m, ids, B, slot0, logits, stream));
  }
  return YUF_OK;
}

yuf_status_t yuf_model_set_decode_graphs(yuf_model* m, int enabled) {
  Y_REQUIRE(m, "null model");
  m->decode_graphs = enabled != 0;
  if (!m->decode_graphs) m->drop_graphs();
  if (m->decode_graphs) {
    Y_CUDA(cudaSetDevice(m->device));
    wkv7_decode_prepare(m->N());
  }
  return YUF_OK;
}

yuf_status_t yuf_model_sync_check(yuf_model* m, void* stream) {
  Y_REQUIRE(m, "null model");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Y_CUDA(cudaStreamSynchronize(s));
  int err = 0;
  Y_CUDA(cudaMemcpy(&err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    Y_CUDA(cudaMemset(m->d_err, 0, sizeof(int)));
    set_error("model: a token id was outside [0, %d)", m->cfg.vocab_size);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  // bounded device waits of the scan kernels (a nonzero count voids the outputs)
  return yuf_sync_check(stream);
}

yuf_status_t yuf_model_set_debug(yuf_model* m, int enabled) {
  Y_REQUIRE(m, "null model");
  m->debug = enabled != 0;
  if (!m->debug) m->dumps.clear();
  return YUF_OK;
}

yuf_status_t yuf_model_set_debug_filter(yuf_model* m, const char* regions, const int* layers,
                                        int n_layers) {
  Y_REQUIRE(m, "null model");
  Y_REQUIRE(n_layers >= 0 && (n_layers == 0 || layers), "debug: bad layer list");
  std::vector<std::string> names;
  if (regions) {
    std::string cur;
    for (const char* c = regions;; ++c) {
      if (*c == ',' || *c == 0) {
        if (!cur.empty()) names.push_back(cur);
        cur.clear();
        if (*c == 0) break;
      } else if (*c != ' ') {
        cur.push_back(*c);
      }
    }
  }
  std::vector<char> mask;
  if (n_layers > 0) {
    mask.assign(m->cfg.n_layers, 0);
    for (int i = 0; i < n_layers; ++i) {
      Y_REQUIRE(layers[i] >= 0 && layers[i] < m->cfg.n_layers, "debug: layer %d out of range", layers[i]);
      mask[layers[i]] = 1;
    }
  }
  m->debug_regions = std::move(names);
  m->debug_layers = std::move(mask);
  return YUF_OK;
}

yuf_status_t yuf_debug_dump(yuf_model* m, const char* region, int layer, float* host_out,
                            size_t capacity, size_t* n_written) {
  Y_REQUIRE(m && region, "null argument");
  auto it = m->dumps.find(region);
  Y_REQUIRE(it != m->dumps.end(), "debug: region %s was not recorded (enable debug first)", region);
  Y_REQUIRE(layer + 1 >= 0 && layer + 1 < (int)it->second.size() && !it->second[layer + 1].empty(),
            "debug: region %s has no layer %d", region, layer);
  const auto& v = it->second[layer + 1];
  if (n_written) *n_written = v.size();
  if (host_out) {
    Y_REQUIRE(capacity >= v.size(), "debug: buffer holds %zu floats, region needs %zu", capacity, v.size());
    std::memcpy(host_out, v.data(), v.size() * 4);
  }
  return YUF_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode step (yuf_step_static).
//
// Some callers may not allocate device memory at all: code running in a host
// application's real-time callback (an audio plug-in rendering the next notes,
// where cudaMalloc's implicit device synchronisation and unbounded latency are
// not allowed), or code living inside a process that hands it a fixed device
// memory budget up front.  yuf_step_static serves them: its per-call working
// memory comes from the fixed array below instead of the model's grow-on-demand
// workspace, so a call allocates nothing (the model, its weights and its state
// slots were all allocated when the model was built).
//
// The array is a file-scope __device__ object: every GPU that loads this library
// holds it (YUF_STATIC_SCRATCH_BYTES) until the process exits.  Host code cannot
// use its name as a device address, so every call looks the address up with
// cudaGetSymbolAddress, with the model's device current (a lookup allocates
// nothing; the first one on a device may load the library's device code, so
// that first call belongs before any stream capture).  The step's scratch is
// sized for one token per sequence (no time-parallel scan scratch).
namespace yuf {
constexpr size_t YUF_STATIC_SCRATCH_BYTES = 8u << 20;  // 8 MiB
}  // namespace yuf
static __device__ __align__(256) unsigned char g_step_scratch[yuf::YUF_STATIC_SCRATCH_BYTES];

extern "C" yuf_status_t yuf_step_static(yuf_model* m, const int32_t* ids, int B, int slot0,
                                        float* logits, void* stream) {
  Y_REQUIRE(m, "step_static: null model");
  Y_REQUIRE(B >= 1 && ids && logits, "step_static: need B >= 1, ids and logits");
  const size_t need = ws_bytes(m, (size_t)B, true);
  if (need > YUF_STATIC_SCRATCH_BYTES) {
    size_t max_b = 0;
    while (ws_bytes(m, max_b + 1, true) <= YUF_STATIC_SCRATCH_BYTES) ++max_b;
    set_error("step_static: %d sequences need %zu bytes of scratch; the fixed scratch holds %zu "
              "bytes (at most %zu sequences for this model)",
              B, need, (size_t)YUF_STATIC_SCRATCH_BYTES, max_b);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  Y_REQUIRE(!m->debug, "step_static: parity dumps copy to host buffers; disable debug first");
  Y_REQUIRE(m->n_slots > 0, "step_static: call yuf_state_alloc first");
  Y_REQUIRE(slot0 >= 0 && slot0 + B <= m->n_slots, "step_static: slots [%d, %d) out of range (%d slots)",
            slot0, slot0 + B, m->n_slots);
  Y_CUDA(cudaSetDevice(m->device));
  void* base = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&base, g_step_scratch);
  if (e != cudaSuccess || base == nullptr) {
    set_error("step_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    return YUF_ERR_CUDA;
  }
  // Every scratch region is written before it is read within the step, so
  // nothing has to be cleared between calls.
  return forward(m, ids, B, 1, slot0, logits, nullptr, static_cast<cudaStream_t>(stream), base);
}
