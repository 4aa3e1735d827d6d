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
  YUF_WKV_AUTO = 0,       /* chunked for T >= 16, sequential below          */
  YUF_WKV_SEQUENTIAL = 1, /* token-by-token (the decode step)                */
  YUF_WKV_CHUNKED = 2     /* 16-token chunks, no per-token reduction chain   */
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

#ifdef __cplusplus
}
#endif

#endif /* YUFB200_H */
