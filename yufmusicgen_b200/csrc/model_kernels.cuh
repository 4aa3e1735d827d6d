// Declarations of the block kernels (model_kernels.cu) and the scan
// dispatchers used by the model engine.
#pragma once
#include <cuda_bf16.h>

#include "common.cuh"

namespace yuf {

void launch_embed(const int32_t* ids, const float* E, float* x, int rows, int d, int vocab, int* err,
                  cudaStream_t s);
// gate (nullable) multiplies the normalised row; gate_sigmoid: sigmoid(gate) does
template <typename OUT>
void launch_layernorm(const float* x, const float* w, const float* b, const float* gate, OUT* out,
                      int rows, int d, cudaStream_t s, bool gate_sigmoid = false);
template <typename OUT>
void launch_mix(const float* xt, const float* prev, const float* mix, OUT* out, int B, int T, int d,
                cudaStream_t s);
// one token per sequence: layer norm + six lerps + prev := xt in one launch;
// false (nothing launched) when d is not a multiple of 4 or above 1024
template <typename OUT>
bool launch_ln_mix_step(const float* x, const float* w, const float* b, float* xt, float* prev,
                        const float* mix, OUT* out, int B, int d, cudaStream_t s);
// B sequences x T tokens (prefill): layer norm + token shift + six lerps in one
// launch, xt written for each sequence's last row only; false (nothing
// launched) when d is not a multiple of 4 or above 1024
template <typename OUT>
bool launch_ln_mix_rows(const float* x, const float* w, const float* b, float* xt, const float* prev,
                        const float* mix, OUT* out, int B, int T, int d, cudaStream_t s);
// tanh of the first n_tanh elements, plain copy (conversion) of the rest up to n
template <typename OUT>
void launch_tanh(const float* x, OUT* out, size_t n_tanh, size_t n, cudaStream_t s);
void launch_timemix_post(const float* k, const float* lw, const float* la, const float* lg,
                         const float* w0, const float* a0, const float* k_k, const float* k_a,
                         float* w_raw, float* k_adj, float* a_op, float* b_op, float* g, int rows,
                         int H, int N, cudaStream_t s);
template <typename OUT>
void launch_silu_mul(const float* ig, OUT* out, int rows, int F, cudaStream_t s);
void launch_to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s);

yuf_status_t wkv7_dispatch(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           float* ckpt, float* sa, int B, int T, int H, int N, bool compat,
                           cudaStream_t stream);
// one-time setup of the decode kernels for head size N (outside graph capture)
void wkv7_decode_prepare(int N);
yuf_status_t wkv7_decode_tm_dispatch(const float* r, const float* k, const float* v, const float* lw,
                                     const float* la, const float* lg, const float* w0, const float* a0,
                                     const float* k_k, const float* k_a, float* g, const float* s0, float* y,
                                     float* s_out, int BH, int H, int N, cudaStream_t stream);
yuf_status_t wkv7_decode_dispatch(const float* r, const float* w, const float* k, const float* v,
                                  const float* a, const float* b, const float* s0, float* y,
                                  float* s_out, int BH, int N, cudaStream_t stream);
// ROSA scan over inputs with row stride `ld` (elements between tokens) and
// optional per-channel biases added to cand/write/gate before the activations.
yuf_status_t rosa_engine_dispatch(const float* cand, const float* write, const float* gate,
                                  const float* bias_c, const float* bias_w, const float* bias_g,
                                  int ld, const float* decay_raw, const float* dir_raw,
                                  const float* m0, float* read, float* m_out, int B, int T, int R,
                                  float* scratch, __nv_bfloat16* read_bf, cudaStream_t stream,
                                  const float* factors = nullptr);
// floats of scratch the time-parallel ROSA scan needs (0 if it does not apply)
size_t rosa_parallel_scratch_floats(int B, int T, int R);
// a layer's time-parallel ROSA constants (coefficients, A^K or its low-rank
// factors): floats, and the launches that build them from the raw parameters
size_t rosa_factor_floats(int R);
yuf_status_t rosa_prepare_factors(const float* decay, const float* dir, int raw, int R, float* out,
                                  cudaStream_t s);
bool rosa_parallel_applies(int B, int T, int R);

}  // namespace yuf

namespace yuf {
// Time-parallel WKV-7 prefill (wkv7_parallel.cu): runs for T >= 256; scratch
// holds wkv7_parallel_scratch_floats() floats, 16-byte aligned.
// wkv7_parallel_scratch_bound(rows, H, N) covers every B, T with B*T <= rows.
bool wkv7_parallel_applies(int B, int T, int H, int N);
size_t wkv7_parallel_scratch_floats(int B, int T, int H, int N);
size_t wkv7_parallel_scratch_bound(size_t rows, int H, int N);
// tm (nullable): the time-mix epilogue folded into the first pass -- r, lw, k,
// v, la as the projections left them in place of r, w, k, v, a (b unused);
// YUF_ERR_UNSUPPORTED (nothing launched) for head sizes above 64.
yuf_status_t wkv7_parallel(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           int B, int T, int H, int N, float* scratch, cudaStream_t st,
                           bool tc_correct = false, const WkvTm* tm = nullptr);
// Chunked WKV-7 prefill on the tensor cores (wkv7_chunk_tc.cu): one CTA per
// (sequence, head), no scratch; N in {16, 32, 40, 48, 64}.
bool wkv7_chunk_tc_supports(int N);
bool wkv7_chunk_tc_applies(int B, int T, int H, int N);
yuf_status_t wkv7_chunk_tc(const float* r, const float* w, const float* k, const float* v, const float* a,
                           const float* b, const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                           cudaStream_t st);
// the same with the time-mix epilogue folded in: r, k, v, lw, la as the projections
// left them, the layer's w0, a0, k_k, k_a
yuf_status_t wkv7_chunk_tc_tm(const float* r, const float* k, const float* v, const float* lw, const float* la,
                              const float* w0, const float* a0, const float* k_k, const float* k_a,
                              const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                              cudaStream_t st);
}  // namespace yuf
