/* yufb200 -- C ABI of the B200-native WKV-7 + ROSA hot path of YufMusicGen.
 *
 * Every entry point:
 *   - takes plain device pointers and sizes (no framework types),
 *   - launches on the CUDA stream given as `stream` (a cudaStream_t; NULL is
 *     the legacy default stream, as the reference kernels use),
 *   - returns a yuf_status_t and never throws; on failure the thread-local
 *     message of yuf_last_error() says why,
 *   - validates shapes and pointers on the host before any launch.
 * The caller owns every buffer.  All tensors are fp32, row-major, contiguous.
 *
 * Layouts (the reference's, yufmusicgen/model.py:97-165, 260-288):
 *   r, w, k, v, a, b, y : [B, T, H, N]   (w is the RAW decay; the kernel applies
 *                                         exp(-0.6065306597 * sigmoid(w)))
 *   state s             : [B, H, N, N]   row i = value dim, column j = key dim
 *   cand, write, gate   : [B, T, R]; memory m : [B, R]; decay (post-sigmoid) and
 *                         direction (unit) : [R]
 */
#ifndef YUFB200_H
#define YUFB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum yuf_status {
  YUF_OK = 0,
  YUF_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer, misaligned buffer */
  YUF_ERR_UNSUPPORTED = 2,      /* size this build has no kernel for        */
  YUF_ERR_CUDA = 3,             /* a CUDA runtime or launch error           */
  YUF_ERR_OUT_OF_MEMORY = 4,
  YUF_ERR_IO = 5,
  YUF_ERR_TIMEOUT = 6
} yuf_status_t;

/* Name of a status code. */
const char* yuf_status_string(yuf_status_t status);
/* Message of the last failing call on this host thread ("" if none). */
const char* yuf_last_error(void);
/* ABI version of this library (bumped on any incompatible change). */
int yuf_abi_version(void);
/* Number of bounded device-side waits (the time-parallel scan's staging barrier) that
   expired on the current device since the previous call; the count is cleared.  0 in
   a healthy run; a nonzero count means the outputs of the affected launches are void.
   Synchronous (reads a device counter).  No reference counterpart: the reference
   kernels have no bounded waits. */
unsigned int yuf_wait_timeouts(void);
/* Synchronise `stream`, then report the bounded device waits that expired since the
   last check (clearing the count): YUF_ERR_TIMEOUT when any did -- the outputs of the
   launches involved are void -- else YUF_OK.  No reference counterpart (the reference
   kernels have no bounded waits). */
yuf_status_t yuf_sync_check(void* stream);
/* Test hook of the bounded-wait path (no reference counterpart): launches one warp
   that waits, with a bound of `limit_ns` nanoseconds (<= 2 s), on a barrier nothing
   arrives at, and records the expiry as a scan kernel would; the next yuf_sync_check
   then returns YUF_ERR_TIMEOUT.  Faults nothing; the context stays usable. */
yuf_status_t yuf_debug_wait_selftest(unsigned long long limit_ns, void* stream);

/* WKV-7 forward scan with an optional initial state.
 * Replaces the forward launch behind torch.ops.yufmusicgen_rwkv7.forward
 * (reference yufmusicgen/cuda/rwkv7_clampw.cpp:18-33 -> rwkv7_clampw.cu:76-79)
 * and the stateful PyTorch recurrence the reference falls back to for decode
 * (yufmusicgen/model.py:145-165, 193).
 *   s0    : [B,H,N,N] initial state, or NULL for zeros (the reference op has no
 *           initial state at all, yufmusicgen/cuda/rwkv7_clampw.cu:25-29).
 *   s_out : [B,H,N,N] final state, canonical layout, or NULL.  May alias s0.
 * Any T >= 0 (no padding to 16 needed).  N in {16, 32, 40, 48, 64, 96, 128}. */
yuf_status_t yuf_wkv7_forward(const float* r, const float* w, const float* k, const float* v,
                              const float* a, const float* b, const float* s0, float* y,
                              float* s_out, int B, int T, int H, int N, void* stream);

/* Algorithm choice for yuf_wkv7_forward_ex. */
enum {
  YUF_WKV_AUTO = 0,       /* T == 1: single-token kernel; T >= 256 and few (sequence, head)
                             chains (N <= 64: B*H <= half the resident pair blocks, 888 at
                             N = 40 and 370 at N = 64 on a 148-SM B200; larger N:
                             B*H <= 64): time-parallel;
                             else sequential                                                    */
  YUF_WKV_SEQUENTIAL = 1, /* token by token, one CTA per (sequence, head)                         */
  YUF_WKV_CHUNKED = 2,    /* 16-token chunks, no per-token reduction chain                        */
  YUF_WKV_PARALLEL = 3,   /* chunks scanned in parallel (about one wave of blocks), states
                             carried between them; takes stream-ordered scratch for the chunk
                             transitions from a library-owned pool that keeps its pages; T >= 256 */
  YUF_WKV_PARALLEL_TC = 4, /* YUF_WKV_PARALLEL with the output correction y += S0 q_t on the
                             tcgen05 tensor cores (TMEM accumulators, 3xTF32) for N <= 64;
                             today slower than the default mma.sync correction            */
  YUF_WKV_ROWS = 5,        /* token by token, one CTA per (sequence, head) with the state rows
                             split over warps (4 lanes per row, decay-scaled state inside
                             8-token groups staged by a producer warp with TMA); reads the
                             inputs and writes y once                                     */
  YUF_WKV_CHUNKED_TC = 6   /* 16-token chunks, one CTA per (sequence, head), the state in
                             tensor-core accumulators: per chunk the state products
                             (W S^T, Q S^T, SA^T B~ + V^T K~) on mma.sync 3xTF32, the
                             chunk-local Gram matrices and substitution on the FMA pipe by
                             prep warps, inputs staged by TMA; N in {16, 32, 40, 48, 64}  */
};
/* yuf_wkv7_forward with an explicit algorithm (same results to fp32 rounding). */
yuf_status_t yuf_wkv7_forward_ex(const float* r, const float* w, const float* k, const float* v,
                                 const float* a, const float* b, const float* s0, float* y,
                                 float* s_out, int B, int T, int H, int N, int algo,
                                 void* stream);

/* The reference op's exact output contract (rwkv7_clampw.cu:20-75, used by
 * yufmusicgen/cuda_ops.py:189-233): zero initial state, T % 16 == 0, and besides
 * y it fills
 *   states [B,H,T/16,N,N] : the state after every 16th token, TRANSPOSED
 *                           (states[b,h,c,j,i] = S_ij), the layout the reference
 *                           backward kernel reads;
 *   sa     [B,T,H,N]      : sa_i = sum_j a_j S_ij before each update. */
yuf_status_t yuf_wkv7_forward_compat(const float* r, const float* w, const float* k,
                                     const float* v, const float* a, const float* b, float* y,
                                     float* states, float* sa, int B, int T, int H, int N,
                                     void* stream);

/* ROSA Householder scan (yufmusicgen/model.py:260-288):
 *   m_t    = decay * (m - 2 (m.d) d) + sigmoid(write_t) * tanh(cand_t)
 *   read_t = (m_t - 2 (m_t.d) d) * (gated ? sigmoid(gate_t) : 1)
 * gated = 1 gives ROSAMemory._reference_recurrence's output; gated = 0 gives the
 * reference CUDA op's ungated read (rosa_householder.cu:89-91, the caller gates,
 * yufmusicgen/model.py:311).  `gate` may be NULL when gated = 0.
 * m_out may alias m0.  Any T >= 0; 1 <= R <= 1024. */
yuf_status_t yuf_rosa_forward(const float* cand, const float* write, const float* gate,
                              const float* decay, const float* direction, const float* m0,
                              float* read, float* m_out, int B, int T, int R, int gated,
                              void* stream);

/* The reference ROSA op's exact output contract
 * (torch.ops.yufmusicgen_rosa.forward, rosa_householder.cpp:24-50 ->
 * rosa_householder.cu:30-101): ungated read_out [B,T,R], memory_out [B,R] and the
 * saved tensors cand_saved = tanh(cand), write_saved = sigmoid(write),
 * read_saved = read_out, gate_saved = sigmoid(read_raw), decay_saved [B,T,R]
 * (decay broadcast) and mem_saved [B,T+1,R] (m_0 .. m_T).
 * D (= R) in {16, 32, 64, 128, 256}, the reference's supported sizes. */
yuf_status_t yuf_rosa_forward_compat(const float* cand, const float* write, const float* read_raw,
                                     const float* decay, const float* direction,
                                     const float* memory, float* read_out, float* memory_out,
                                     float* cand_saved, float* write_saved, float* read_saved,
                                     float* gate_saved, float* decay_saved, float* mem_saved,
                                     int B, int T, int R, void* stream);

/* Training backward of the WKV-7 op: the reference's
 * torch.ops.yufmusicgen_rwkv7.backward (rwkv7_clampw.cpp:40-63 ->
 * rwkv7_clampw.cu:83-176), same buffers.  Inputs r..b [B,T,H,N] as given to
 * yuf_wkv7_forward_compat, dy [B,T,H,N] = dL/dy, and that call's `states`
 * [B,H,T/16,N,N] (transposed checkpoints) and `sa` [B,T,H,N].  Writes the
 * gradients dr, dw (w.r.t. the raw w, through the retention clamp), dk, dv,
 * da, db, each [B,T,H,N], for a zero initial state with no gradient on the
 * final state.  T % 16 == 0; every pointer 16-byte aligned.  Scratch of
 * 16*N*N floats per (b,h) comes from the library's stream-ordered pool.  The
 * result is the exact gradient (fp32): the states are replayed from the
 * checkpoints, where the reference divides by the retention to step back. */
yuf_status_t yuf_wkv7_backward(const float* r, const float* w, const float* k, const float* v,
                               const float* a, const float* b, const float* dy,
                               const float* states, const float* sa, float* dr, float* dw,
                               float* dk, float* dv, float* da, float* db, int B, int T, int H,
                               int N, void* stream);

/* Training backward of the ROSA op: the reference's
 * torch.ops.yufmusicgen_rosa.backward (rosa_householder.cpp:52-83 ->
 * rosa_householder.cu:103-285), same buffers.  Reads the saved tensors of
 * yuf_rosa_forward_compat (cand_saved, write_saved, decay_saved, mem_saved;
 * read_saved, gate_saved, final_memory and workspace are accepted and unused),
 * direction [R] and d_read [B,T,R] = dL/d(ungated read).  Writes d_cand,
 * d_write (w.r.t. the raw pre-activations), d_read_raw (zero: the ungated read
 * does not depend on it), d_decay [B,T,R] (per step; the caller sums over B,T),
 * d_direction_partial [B,R] (per sequence; the caller sums over B) and
 * d_memory_out [B,R] = dL/dm_0.  The final memory carries no gradient.
 * 1 <= R <= 1024. */
yuf_status_t yuf_rosa_backward(const float* cand_saved, const float* write_saved,
                               const float* read_saved, const float* gate_saved,
                               const float* decay_saved, const float* mem_saved,
                               const float* direction, const float* final_memory,
                               const float* d_read, float* d_cand, float* d_write,
                               float* d_read_raw, float* d_decay, float* d_direction_partial,
                               float* d_memory_out, float* workspace, int B, int T, int R,
                               void* stream);

/* Projection GEMM of the engine (bf16 operands, fp32 accumulation, tcgen05
 * tensor cores), the nn.Linear products of yufmusicgen/model.py:107-112,
 * 195-197, 297-311, 376-377, 421 for a host that drives the block itself:
 *   C[z] = A[z] . W[z]^T  for z < batch,
 * A [M, K] bf16 with row stride lda (batch z starts a_batch_rows rows on), W
 * [N, K] bf16 contiguous (batch z starts w_batch_rows rows on), C with row
 * stride ldc (batch z starts c_batch_stride elements on).  A and W rows
 * 16-byte aligned (lda and K multiples of 8).  Epilogues:
 *   YUF_GEMM_F32         C fp32 = acc, or C += acc with accumulate != 0
 *                        (the block's residual adds);
 *   YUF_GEMM_BF16        C bf16 = acc;
 *   YUF_GEMM_BF16_TANH0  C bf16 = tanh(acc) for batch 0, acc for the others
 *                        (the w branch of the low-rank projections);
 *   YUF_GEMM_SILU_GATE   C bf16 [M, n_out] = SiLU(in) * gate, where W's rows
 *                        come in groups of 128: 64 rows of ffn_in.weight, then
 *                        the same 64 rows of ffn_gate.weight (model.py:376-377);
 *                        output column 64g + j pairs W rows 128g + j and
 *                        128g + 64 + j.  N % 128 == 0, n_out <= N / 2. */
enum {
  YUF_GEMM_F32 = 0,
  YUF_GEMM_BF16 = 1,
  YUF_GEMM_BF16_TANH0 = 2,
  YUF_GEMM_SILU_GATE = 3,
  YUF_GEMM_F32_TANH0 = 4,     /* yuf_gemm_tf32x3 only: fp32 tanh(acc) for batch 0 */
  YUF_GEMM_SILU_GATE_F32 = 5  /* yuf_gemm_tf32x3 only: the SiLU-gate epilogue, fp32 out */
};
yuf_status_t yuf_gemm_bf16(const void* A, long long lda, long long a_batch_rows, const void* W,
                           long long w_batch_rows, void* C, long long ldc, long long c_batch_stride,
                           int M, int N, int K, int batch, int epilogue, int accumulate, int n_out,
                           void* stream);
/* The same projections with fp32 operands at fp32 accuracy (the engine's fp32
 * mode): A fp32 (row stride lda), W as two fp32 parts [N, K] each, W_hi = W
 * with its 13 low mantissa bits cleared and W_lo = W - W_hi (yuf_tf32_split);
 * the kernel splits A the same way and sums A_lo W_hi + A_hi W_lo + A_hi W_hi
 * on the tensor cores (kind::tf32, "3xTF32", ~2^-20 relative per product).
 * Epilogues YUF_GEMM_F32 (accumulate allowed), YUF_GEMM_F32_TANH0,
 * YUF_GEMM_SILU_GATE_F32.  lda and K multiples of 4. */
yuf_status_t yuf_gemm_tf32x3(const float* A, long long lda, long long a_batch_rows, const float* W_hi,
                             const float* W_lo, long long w_batch_rows, float* C, long long ldc,
                             long long c_batch_stride, int M, int N, int K, int batch, int epilogue,
                             int accumulate, int n_out, void* stream);
/* Host: split n fp32 weights into the two parts yuf_gemm_tf32x3 takes. */
yuf_status_t yuf_tf32_split(const float* w, size_t n, float* hi, float* lo);

/* ------------------------------------------------------------------------ *
 * Model engine: the YufMusicGen block stack (yufmusicgen/model.py:345-445) on
 * the GPU with device-resident recurrent state, the batched counterpart of the
 * Vulkan engine's Model::new / Model::step / Model::reset_state
 * (vulkan/src/compute/model.rs:24-65).
 * ------------------------------------------------------------------------ */

typedef struct yuf_model yuf_model; /* opaque */

typedef struct yuf_model_config {
  int vocab_size, d_model, n_layers, n_heads, head_size, rosa_size;
  int low_rank; /* 0 = the reference rule max(32, round(2.5 sqrt(d) / 32) * 32), model.py:59 */
} yuf_model_config;

enum {
  YUF_PRECISION_FP32 = 0,        /* fp32 weights; GEMMs with fp32 accuracy (3xTF32 tensor cores) */
  YUF_PRECISION_BF16_WEIGHTS = 1 /* bf16 weights and GEMM inputs, fp32 accumulate and state */
};

/* Build a model on `device` from host fp32 tensors named as in the reference
 * state_dict (e.g. "blocks.3.time_mix.key.weight"); `lm_head.weight` may be
 * absent (tied to token_embedding.weight, model.py:389-391).  Every tensor the
 * architecture needs must be present with its exact element count. */
yuf_status_t yuf_model_create(const yuf_model_config* cfg, int precision, int device, int n_tensors,
                              const char* const* names, const float* const* host_data,
                              const int64_t* numels, yuf_model** out);
/* Build a model from a .yuf checkpoint (vulkan/scripts/export_checkpoint.py). */
yuf_status_t yuf_model_create_from_yuf(const char* path, int precision, int device, yuf_model** out);
yuf_status_t yuf_model_destroy(yuf_model* model);
yuf_status_t yuf_model_get_config(const yuf_model* model, yuf_model_config* out);

/* Allocate `n_slots` recurrent-state slots (per layer: prev [d], S [H,N,N],
 * m [R]) and zero them.  Replaces any previous slots. */
yuf_status_t yuf_state_alloc(yuf_model* model, int n_slots);
/* Zero slots [slot0, slot0 + n) on `stream` (Model::reset_state, model.rs:62-65). */
yuf_status_t yuf_state_reset(yuf_model* model, int slot0, int n, void* stream);
/* Copy slots [slot0, slot0 + n) of one layer to/from caller device buffers in
 * the reference layout: prev [n,d], S [n,H,N,N] (row = value, col = key), m [n,R]. */
yuf_status_t yuf_state_export(yuf_model* model, int layer, int slot0, int n, float* prev, float* S,
                              float* m, void* stream);
yuf_status_t yuf_state_import(yuf_model* model, int layer, int slot0, int n, const float* prev,
                              const float* S, const float* m, void* stream);

/* Prefill: run B sequences of T tokens (device int32 ids [B,T]) through the model
 * starting from the state in slots [slot0, slot0 + B) and leave the final
 * state there (YufMusicGen.forward(ids, state), model.py:406-422).
 * logits_last [B,V] and/or logits_all [B,T,V] (device, either may be NULL). */
yuf_status_t yuf_prefill(yuf_model* model, const int32_t* ids, int B, int T, int slot0,
                         float* logits_last, float* logits_all, void* stream);
/* Decode step: one token per sequence (device int32 ids [B]), slots
 * [slot0, slot0 + B), logits [B,V] (YufMusicGen.step, model.py:424-431). */
yuf_status_t yuf_step(yuf_model* model, const int32_t* ids, int B, int slot0, float* logits,
                      void* stream);
/* Decode step that allocates nothing (no counterpart in the reference).
 * Same inputs, outputs and results as yuf_step, for callers that may not
 * allocate device memory at call time -- e.g. a real-time audio callback in a
 * host application, where cudaMalloc's implicit synchronisation and latency
 * are not allowed, or a component handed a fixed device-memory budget.  Its
 * working memory is a fixed 8 MiB array compiled into this library (held on
 * every GPU that loads the library until exit) instead of the model's
 * grow-on-demand workspace; B larger than that array allows is rejected with
 * YUF_ERR_INVALID_ARGUMENT and a message giving the largest B for the model.
 * Every call looks up the array's device address (allocating nothing); the
 * first call on a device may load the library's device code, so make that
 * first call before any stream capture.  All calls share the one array:
 * calls whose work overlaps on the GPU (other streams, other threads) race and
 * must be serialised by the caller.  Nothing in the array needs clearing
 * between calls.  Parity dumps (yuf_model_set_debug) must be off. */
yuf_status_t yuf_step_static(yuf_model* model, const int32_t* ids, int B, int slot0, float* logits,
                             void* stream);
/* On-device sampling of one token per sequence from logits [B,V] (device) into
 * out_ids [B] (device int32), replacing the host-side sample_token of
 * yufmusicgen/cli/generate.py:45-56 and its masking (generate.py:142-149):
 * ids below `mask_below` are excluded except `eos_id` when allow_eos != 0;
 * logits are divided by `temperature` (<= 0: greedy argmax); the `top_k`
 * (1..1024) most likely tokens are kept, then the top-p cut inside them (a token
 * is dropped when the mass before it exceeds top_p), then one draw with the
 * uniform Philox4x32-10(key = seed, counter = (step, seq0 + b, 0)), so results
 * do not depend on batch layout.  out_uniform [B] (nullable) receives the
 * uniforms used.  V <= 51200. */
yuf_status_t yuf_sample(const float* logits, int B, int V, float temperature, int top_k,
                        float top_p, uint64_t seed, uint64_t step, int seq0, int mask_below,
                        int eos_id, int allow_eos, int32_t* out_ids, float* out_uniform,
                        void* stream);
/* The sampler's uniforms for sequences seq0 .. seq0 + n - 1 at (seed, step). */
yuf_status_t yuf_philox_uniform(uint64_t seed, uint64_t step, int seq0, int n, float* out,
                                void* stream);

/* Host-side sampling with the reference's own random stream (no GPU): the
 * sample_token rule of yufmusicgen/cli/generate.py:45-56 -- logits / temperature
 * (<= 0: argmax), descending sort, softmax, drop an entry when the mass before
 * it exceeds top_p, softmax again, torch.multinomial(p, 1) -- on a generator
 * equal to torch's CPU generator after torch.manual_seed(seed) (MT19937; the
 * bit-level reading of vulkan/src/sampler.rs:1-270).  A draw consumes one Exp(1)
 * key per vocabulary entry, in sorted order, and takes argmax(p / key), as the
 * CPU multinomial does for one sample; rows of a batch draw one after another
 * (the order torch fills a [B, V] batch in).  Probabilities use the C library's
 * expf, so a token can differ from torch's only where two keys tie to the last
 * bit.  Not thread-safe per generator. */
typedef struct yuf_mt19937 yuf_mt19937; /* opaque */
yuf_status_t yuf_mt19937_create(uint64_t seed, yuf_mt19937** out);
yuf_status_t yuf_mt19937_destroy(yuf_mt19937* rng);
/* The next n raw 32-bit words of the generator. */
yuf_status_t yuf_mt19937_next(yuf_mt19937* rng, uint32_t* out, int64_t n);
/* The next n Exp(1) draws as torch's CPU Tensor.exponential_() makes them. */
yuf_status_t yuf_mt19937_exponential(yuf_mt19937* rng, float* out, int64_t n);
/* One token per row of host logits [B, V] (masked entries -inf) into host
 * out_ids [B]. */
yuf_status_t yuf_sample_host(const float* logits, int B, int V, float temperature, float top_p,
                             yuf_mt19937* rng, int32_t* out_ids);

/* Sampling rule of yuf_generate (the reference loop's knobs, cli/generate.py:34-56,
 * 142-149, plus the top-k / Philox stream of benchmark config 4). */
typedef struct yuf_generate_params {
  float temperature;         /* <= 0: greedy argmax                                          */
  int top_k;                 /* 1..1024                                                      */
  float top_p;               /* nucleus cut inside the top-k (>= 1: off)                     */
  uint64_t seed;             /* Philox4x32-10 key                                            */
  int seq0;                  /* global index of the batch's first sequence (Philox counter)  */
  int mask_below;            /* ids below are excluded, except EOS once allowed (reference:  */
                             /* MIDI_OFFSET = 260; 0 = no mask)                              */
  int eos_id;                /* end-of-sequence id (reference: EOS = 2), -1 = never end      */
  int min_tokens_before_eos; /* EOS selectable once this many tokens were generated (16)     */
} yuf_generate_params;

/* Batched autoregressive generation on the device: the decode loop of the
 * reference's run_generation (yufmusicgen/cli/generate.py:130-154; the Vulkan
 * client's vulkan/src/generation.rs:176-214) for B sequences at once, with no
 * host synchronisation per token.  Prefills prompt_ids [B,T] (device int32) from
 * the state in slots [slot0, slot0 + B) -- zero them first (yuf_state_reset) for
 * fresh sequences, as run_generation starts from no state -- then n_steps times:
 * sample one token per sequence from the last logits (yuf_sample's rule with
 * step = the step index and allow_eos = step >= min_tokens_before_eos), record
 * it, and run one decode step with it (yuf_step; CUDA-graph replay when
 * yuf_model_set_decode_graphs is on).  A sequence ends at its first EOS, which
 * the reference does not emit (it breaks, generate.py:150-152):
 *   tokens  [B, n_steps] (device int32): the generated ids; from a sequence's
 *           end on, eos_id;
 *   lengths [B]          (device int32): tokens generated before EOS (n_steps if
 *           the sequence never ended).
 * Ended sequences keep stepping (with EOS as input) until the batch finishes, so
 * their slots' final state is not the reference's; the tokens are unaffected.
 * Working buffers (the last logits, the sampled ids) are kept by the model and
 * grow on demand. */
yuf_status_t yuf_generate(yuf_model* model, const int32_t* prompt_ids, int B, int T, int slot0,
                          int n_steps, const yuf_generate_params* params, int32_t* tokens,
                          int32_t* lengths, void* stream);

/* Replay yuf_step as a CUDA graph: the first call for a given (B, slot0, ids,
 * logits) captures the whole step on the caller's stream, later calls with the
 * same arguments launch the graph (one launch instead of ~25 per layer).  Only
 * on a non-NULL stream and with debug dumps off; growing the workspace (a
 * bigger prefill) drops the captured graphs.  Off by default. */
yuf_status_t yuf_model_set_decode_graphs(yuf_model* model, int enabled);
/* Synchronise `stream` and report device-side input errors of earlier calls
 * (token id outside [0, vocab): YUF_ERR_INVALID_ARGUMENT) and expired bounded
 * waits (YUF_ERR_TIMEOUT, as yuf_sync_check). */
yuf_status_t yuf_model_sync_check(yuf_model* model, void* stream);

/* ------------------------------------------------------------------------ *
 * REMI token codec and Standard MIDI File I/O (host only, no GPU): the
 * generated token stream <-> notes <-> .mid bytes, the counterpart of the
 * Vulkan client's RemiCodec (vulkan/src/remi.rs:26-312) and MIDI reader /
 * writer (vulkan/src/midi.rs:58-434), i.e. MidiTok 3.0 REMI as YufMusicGen
 * configures it: 8 ticks per quarter, 4/4 bars of 32 positions, a Program
 * token before every note, velocities 3..127 in steps of 4, the vocabulary's
 * Duration_<beat>.<position>.<resolution> values.
 * Two-call convention for outputs of unknown size: pass NULL buffers to get
 * the counts, then buffers of at least that size.
 * ------------------------------------------------------------------------ */

typedef struct yuf_note {
  int32_t start, duration; /* ticks of the score's division */
  int32_t pitch, velocity;
} yuf_note;

typedef struct yuf_track_desc {
  int32_t program;       /* 0..127; -1 for the drum track of a decoded token stream */
  int32_t is_drum;
  const char* name;      /* may be NULL or "" */
  const yuf_note* notes;
  int64_t n_notes;
} yuf_track_desc;

typedef struct yuf_remi yuf_remi; /* opaque codec */

/* Codec over a vocabulary (token id -> name, e.g. "Pitch_60", "Duration_0.2.8")
 * (RemiCodec::new, remi.rs:35-62). */
yuf_status_t yuf_remi_create(const char* const* vocab, int n_vocab, yuf_remi** out);
yuf_status_t yuf_remi_destroy(yuf_remi* codec);
/* Id of a token name, -1 when the vocabulary has none. */
int32_t yuf_remi_token_id(const yuf_remi* codec, const char* name);
/* Notes -> token ids (RemiCodec::encode, remi.rs:199-306): times scaled to 8 ticks
 * per quarter (round half up, durations >= 1), tracks with the same (program,
 * drum) merged, pitches outside 21..109 (drums 27..88) dropped, velocity and
 * duration snapped to the nearest vocabulary value (ties to the larger).
 * Fails when a token the score needs is not in the vocabulary. */
yuf_status_t yuf_remi_encode(const yuf_remi* codec, int ticks_per_quarter,
                             const yuf_track_desc* tracks, int n_tracks, int32_t* ids,
                             int64_t capacity, int64_t* n_ids);
/* Token ids -> notes at 8 ticks per quarter (RemiCodec::decode, remi.rs:74-180):
 * one track per program in order of appearance (track_programs [n_tracks]);
 * notes [n_notes] with their track index in note_track.  Malformed or unknown
 * tokens are skipped, as the reference does. */
yuf_status_t yuf_remi_decode(const yuf_remi* codec, const int32_t* ids, int64_t n_ids,
                             int32_t* track_programs, int max_tracks, int* n_tracks,
                             yuf_note* notes, int32_t* note_track, int64_t max_notes,
                             int64_t* n_notes);
/* Notes -> a format-1 Standard MIDI File (render_midi, midi.rs:351-402): per
 * track a name, a program change (channel 9 for drums, else program % 16) and
 * its notes as time-ordered note-on / note-off events.  Unlike the reference
 * writer, which serialises a track's notes one after another, overlapping notes
 * keep their times. */
yuf_status_t yuf_midi_render(int ticks_per_quarter, const yuf_track_desc* tracks, int n_tracks,
                             uint8_t* out, int64_t capacity, int64_t* n_bytes);
/* Standard MIDI File -> notes (parse_midi, midi.rs:64-281): one track per
 * (file track, channel) that has notes, channel 9 = drums, the channel's last
 * program change, note-offs matched to the latest open note of that pitch. */
yuf_status_t yuf_midi_parse(const uint8_t* bytes, int64_t n_bytes, int* ticks_per_quarter,
                            int32_t* track_programs, int32_t* track_is_drum, int max_tracks,
                            int* n_tracks, yuf_note* notes, int32_t* note_track,
                            int64_t max_notes, int64_t* n_notes);

/* Parity dumps (the regions of vulkan/scripts/dump_reference_step.py:186-322).
 * When enabled, every prefill/step keeps per-layer copies of: ln0, r, w, k, v,
 * a, b, g, y, h1, read, h2, h3 and (layer -1) logits of the last call. */
yuf_status_t yuf_model_set_debug(yuf_model* model, int enabled);
/* Restrict the parity dumps to some regions and layers, as the Vulkan engine's
 * debug_dump(&[&str]) names the regions it wants (vulkan/src/compute/model.rs):
 * `regions` comma-separated (NULL or "" = all), `layers` [n_layers] (0 = all;
 * the logits, layer -1, are kept whenever their region is). */
yuf_status_t yuf_model_set_debug_filter(yuf_model* model, const char* regions, const int* layers,
                                        int n_layers);
yuf_status_t yuf_debug_dump(yuf_model* model, const char* region, int layer, float* host_out,
                            size_t capacity, size_t* n_written);

#ifdef __cplusplus
}
#endif

#endif /* YUFB200_H */
