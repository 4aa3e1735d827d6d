// C ABI of the scan kernels: host-side validation, then dispatch on the
// caller's stream.  No entry point throws; failures return a status and leave
// a message for yuf_last_error().

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "model_kernels.cuh"

namespace yuf {

static thread_local char g_err[1024] = "";

static thread_local bool g_pdl = false;
bool pdl_enabled() { return g_pdl; }
PdlScope::PdlScope(bool on) : prev(g_pdl) { g_pdl = on; }
PdlScope::~PdlScope() { g_pdl = prev; }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

yuf_status_t check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return YUF_ERR_CUDA;
  }
  return YUF_OK;
}

// Scratch of the raw ops comes from a memory pool of this library's own, one
// per device, that keeps freed blocks (release threshold = max): a call that
// needs the same size as the previous one reuses its pages instead of mapping
// new ones, and the process's default pool keeps its own settings.
static std::mutex g_pool_mu;
static cudaMemPool_t g_pools[64] = {};

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pools[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      e = cudaMemPoolCreate(&g_pools[dev], &props);
      if (e != cudaSuccess) return e;
      uint64_t keep = ~0ull;
      e = cudaMemPoolSetAttribute(g_pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
      if (e != cudaSuccess) return e;
    }
    pool = g_pools[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

void scratch_free(void* p, cudaStream_t st) {
  if (p) cudaFreeAsync(p, st);
}

unsigned int wkv7_pair_wait_timeouts();
unsigned int wkv7_decode_wait_timeouts();
unsigned int gemm_wait_timeouts();
unsigned int wkv7_rows_wait_timeouts();
unsigned int wkv7_chunk_tc_wait_timeouts();
yuf_status_t wkv7_rows(const float* r, const float* w, const float* k, const float* v, const float* a,
                       const float* b, const float* s0, float* y, float* s_out, int B, int T, int H, int N,
                       cudaStream_t st);
yuf_status_t wait_selftest(unsigned long long limit_ns, cudaStream_t st);
yuf_status_t wkv7_dispatch(const float* r, const float* w, const float* k, const float* v,
                           const float* a, const float* b, const float* s0, float* y, float* s_out,
                           float* ckpt, float* sa, int B, int T, int H, int N, bool compat,
                           cudaStream_t stream);
yuf_status_t wkv7_chunk_dispatch(const float* r, const float* w, const float* k, const float* v,
                                 const float* a, const float* b, const float* s0, float* y,
                                 float* s_out, int B, int T, int H, int N, cudaStream_t stream);
yuf_status_t wkv7_decode_dispatch(const float* r, const float* w, const float* k, const float* v,
                                  const float* a, const float* b, const float* s0, float* y,
                                  float* s_out, int BH, int N, cudaStream_t stream);
yuf_status_t rosa_dispatch(const float* cand, const float* write, const float* gate,
                           const float* decay, const float* dir, const float* m0, float* read,
                           float* m_out, int B, int T, int R, bool gated, cudaStream_t stream);
yuf_status_t rosa_compat_dispatch(const float* cand, const float* write, const float* gate,
                                  const float* decay, const float* dir, const float* m0, float* read,
                                  float* m_out, float* cs, float* ws, float* rs, float* gs, float* ds,
                                  float* ms, int B, int T, int R, cudaStream_t stream);

yuf_status_t wkv7_backward_dispatch(const float* r, const float* w, const float* k, const float* v,
                                    const float* a, const float* b, const float* dy,
                                    const float* states, const float* sa, float* dr, float* dw,
                                    float* dk, float* dv, float* da, float* db, float* scratch,
                                    int B, int T, int H, int N, cudaStream_t st);
size_t wkv7_backward_scratch_floats(int B, int H, int N);
yuf_status_t rosa_backward_dispatch(const float* cand_s, const float* write_s, const float* decay_s,
                                    const float* mem_s, const float* direction, const float* d_read,
                                    float* d_cand, float* d_write, float* d_read_raw, float* d_decay,
                                    float* d_dir, float* d_mem, int B, int T, int R,
                                    cudaStream_t st);

static bool aligned(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

#define REQUIRE(cond, ...)                  \
  do {                                      \
    if (!(cond)) {                          \
      set_error(__VA_ARGS__);               \
      return YUF_ERR_INVALID_ARGUMENT;      \
    }                                       \
  } while (0)

static yuf_status_t check_wkv_args(const float* const* in, int n_in, int B, int T, int H, int N) {
  REQUIRE(B >= 0 && T >= 0 && H >= 0 && N > 0, "wkv7: negative or zero size (B=%d T=%d H=%d N=%d)",
          B, T, H, N);
  const long long elems = (long long)B * T * H * N;
  REQUIRE(elems < (1LL << 40), "wkv7: tensor too large");
  for (int i = 0; i < n_in; ++i) {
    REQUIRE(elems == 0 || in[i] != nullptr, "wkv7: input %d is NULL", i);
    REQUIRE(aligned(in[i], 16), "wkv7: input %d is not 16-byte aligned", i);
  }
  return YUF_OK;
}

}  // namespace yuf

using namespace yuf;

extern "C" {

unsigned int yuf_wait_timeouts(void) {
  const unsigned int p = yuf::wkv7_pair_wait_timeouts(), d = yuf::wkv7_decode_wait_timeouts(),
                     g = yuf::gemm_wait_timeouts(), r = yuf::wkv7_rows_wait_timeouts(),
                     c = yuf::wkv7_chunk_tc_wait_timeouts();
  return (p == ~0u || d == ~0u || g == ~0u || r == ~0u || c == ~0u) ? ~0u : p + d + g + r + c;
}

yuf_status_t yuf_sync_check(void* stream) {
  g_err[0] = 0;
  const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("sync_check: %s", cudaGetErrorString(e));
    return YUF_ERR_CUDA;
  }
  const unsigned int n = yuf_wait_timeouts();
  if (n == ~0u) {
    set_error("sync_check: the wait-timeout counters could not be read");
    return YUF_ERR_CUDA;
  }
  if (n != 0) {
    set_error("%u bounded device wait(s) expired: the outputs of the affected launches are void", n);
    return YUF_ERR_TIMEOUT;
  }
  return YUF_OK;
}

yuf_status_t yuf_debug_wait_selftest(unsigned long long limit_ns, void* stream) {
  g_err[0] = 0;
  REQUIRE(limit_ns <= 2000ull * 1000 * 1000, "wait selftest: limit %llu ns is above 2 s", limit_ns);
  return wait_selftest(limit_ns, static_cast<cudaStream_t>(stream));
}

const char* yuf_status_string(yuf_status_t s) {
  switch (s) {
    case YUF_OK: return "YUF_OK";
    case YUF_ERR_INVALID_ARGUMENT: return "YUF_ERR_INVALID_ARGUMENT";
    case YUF_ERR_UNSUPPORTED: return "YUF_ERR_UNSUPPORTED";
    case YUF_ERR_CUDA: return "YUF_ERR_CUDA";
    case YUF_ERR_OUT_OF_MEMORY: return "YUF_ERR_OUT_OF_MEMORY";
    case YUF_ERR_IO: return "YUF_ERR_IO";
    case YUF_ERR_TIMEOUT: return "YUF_ERR_TIMEOUT";
  }
  return "YUF_ERR_UNKNOWN";
}

const char* yuf_last_error(void) { return g_err; }

int yuf_abi_version(void) { return 1; }

yuf_status_t yuf_wkv7_forward_ex(const float* r, const float* w, const float* k, const float* v,
                                 const float* a, const float* b, const float* s0, float* y,
                                 float* s_out, int B, int T, int H, int N, int algo,
                                 void* stream) {
  g_err[0] = 0;
  const float* in[7] = {r, w, k, v, a, b, y};
  yuf_status_t st = check_wkv_args(in, 7, B, T, H, N);
  if (st != YUF_OK) return st;
  REQUIRE(aligned(s0, 8) && aligned(s_out, 8), "wkv7: state buffers must be 8-byte aligned");
  REQUIRE(algo >= YUF_WKV_AUTO && algo <= YUF_WKV_CHUNKED_TC, "wkv7: unknown algorithm %d", algo);
  REQUIRE((algo != YUF_WKV_PARALLEL && algo != YUF_WKV_PARALLEL_TC) || T >= 256,
          "wkv7: the time-parallel scan needs T >= 256 (T=%d)", T);
  if (B == 0 || H == 0) return YUF_OK;
  cudaStream_t st_ = static_cast<cudaStream_t>(stream);
  if (T == 1 && algo != YUF_WKV_CHUNKED)
    return wkv7_decode_dispatch(r, w, k, v, a, b, s0, y, s_out, B * H, N, st_);
  if (algo == YUF_WKV_CHUNKED) return wkv7_chunk_dispatch(r, w, k, v, a, b, s0, y, s_out, B, T, H, N, st_);
  if (algo == YUF_WKV_ROWS) return wkv7_rows(r, w, k, v, a, b, s0, y, s_out, B, T, H, N, st_);
  if (algo == YUF_WKV_CHUNKED_TC || (algo == YUF_WKV_AUTO && wkv7_chunk_tc_applies(B, T, H, N)))
    return wkv7_chunk_tc(r, w, k, v, a, b, s0, y, s_out, B, T, H, N, st_);
  if (algo == YUF_WKV_PARALLEL || algo == YUF_WKV_PARALLEL_TC ||
      (algo == YUF_WKV_AUTO && wkv7_parallel_applies(B, T, H, N))) {
    // stream-ordered scratch for the chunk transitions, released right after use
    const size_t bytes = wkv7_parallel_scratch_floats(B, T, H, N) * sizeof(float);
    void* scratch = nullptr;
    cudaError_t e = scratch_alloc(&scratch, bytes, st_);
    if (e != cudaSuccess) {
      set_error("wkv7: scratch allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
      return YUF_ERR_OUT_OF_MEMORY;
    }
    yuf_status_t rc = wkv7_parallel(r, w, k, v, a, b, s0, y, s_out, B, T, H, N,
                                    static_cast<float*>(scratch), st_, algo == YUF_WKV_PARALLEL_TC);
    scratch_free(scratch, st_);
    return rc;
  }
  return wkv7_dispatch(r, w, k, v, a, b, s0, y, s_out, nullptr, nullptr, B, T, H, N, false,
                       static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_wkv7_forward(const float* r, const float* w, const float* k, const float* v,
                              const float* a, const float* b, const float* s0, float* y,
                              float* s_out, int B, int T, int H, int N, void* stream) {
  return yuf_wkv7_forward_ex(r, w, k, v, a, b, s0, y, s_out, B, T, H, N, YUF_WKV_AUTO, stream);
}

yuf_status_t yuf_wkv7_forward_compat(const float* r, const float* w, const float* k,
                                     const float* v, const float* a, const float* b, float* y,
                                     float* states, float* sa, int B, int T, int H, int N,
                                     void* stream) {
  g_err[0] = 0;
  const float* in[7] = {r, w, k, v, a, b, y};
  yuf_status_t st = check_wkv_args(in, 7, B, T, H, N);
  if (st != YUF_OK) return st;
  REQUIRE(T % 16 == 0, "wkv7 compat: T=%d must be a multiple of 16 (pad as cuda_ops.py does)", T);
  REQUIRE(((long long)B * T * H * N == 0) || (states != nullptr && sa != nullptr),
          "wkv7 compat: states and sa are required");
  if (B == 0 || H == 0) return YUF_OK;
  return wkv7_dispatch(r, w, k, v, a, b, nullptr, y, nullptr, states, sa, B, T, H, N, true,
                       static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_rosa_forward(const float* cand, const float* write, const float* gate,
                              const float* decay, const float* direction, const float* m0,
                              float* read, float* m_out, int B, int T, int R, int gated,
                              void* stream) {
  g_err[0] = 0;
  REQUIRE(B >= 0 && T >= 0, "rosa: negative size (B=%d T=%d)", B, T);
  REQUIRE(R >= 1 && R <= 1024, "rosa: R=%d outside 1..1024", R);
  REQUIRE(decay && direction && m0, "rosa: decay, direction and m0 are required");
  REQUIRE((long long)B * T == 0 || (cand && write && read), "rosa: cand, write, read are required");
  REQUIRE(!gated || (long long)B * T == 0 || gate, "rosa: gate is required when gated");
  if (B == 0) return YUF_OK;
  return rosa_dispatch(cand, write, gate, decay, direction, m0, read, m_out, B, T, R, gated != 0,
                       static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_rosa_forward_compat(const float* cand, const float* write, const float* read_raw,
                                     const float* decay, const float* direction,
                                     const float* memory, float* read_out, float* memory_out,
                                     float* cand_saved, float* write_saved, float* read_saved,
                                     float* gate_saved, float* decay_saved, float* mem_saved,
                                     int B, int T, int R, void* stream) {
  g_err[0] = 0;
  REQUIRE(B >= 0 && T >= 0, "rosa compat: negative size (B=%d T=%d)", B, T);
  REQUIRE(R == 16 || R == 32 || R == 64 || R == 128 || R == 256,
          "ROSA CUDA kernel supports D in {16, 32, 64, 128, 256}");
  REQUIRE(decay && direction && memory && memory_out && mem_saved,
          "rosa compat: decay, direction, memory, memory_out, mem_saved are required");
  REQUIRE((long long)B * T == 0 || (cand && write && read_raw && read_out && cand_saved &&
                                    write_saved && read_saved && gate_saved && decay_saved),
          "rosa compat: a per-step tensor is NULL");
  if (B == 0) return YUF_OK;
  return rosa_compat_dispatch(cand, write, read_raw, decay, direction, memory, read_out, memory_out,
                              cand_saved, write_saved, read_saved, gate_saved, decay_saved,
                              mem_saved, B, T, R, static_cast<cudaStream_t>(stream));
}

yuf_status_t yuf_wkv7_backward(const float* r, const float* w, const float* k, const float* v,
                               const float* a, const float* b, const float* dy,
                               const float* states, const float* sa, float* dr, float* dw,
                               float* dk, float* dv, float* da, float* db, int B, int T, int H,
                               int N, void* stream) {
  g_err[0] = 0;
  const float* in[13] = {r, w, k, v, a, b, dy, sa, dr, dw, dk, dv, da};
  yuf_status_t st = check_wkv_args(in, 13, B, T, H, N);
  if (st != YUF_OK) return st;
  REQUIRE(T % 16 == 0, "wkv7 backward: T=%d must be a multiple of 16 (pad as cuda_ops.py does)", T);
  REQUIRE((long long)B * T * H == 0 || (db && aligned(db, 16) && states && aligned(states, 16)),
          "wkv7 backward: db and states must be non-NULL and 16-byte aligned");
  if (!(N == 16 || N == 32 || N == 40 || N == 48 || N == 64 || N == 96 || N == 128)) {
    set_error("wkv7 backward: head size N=%d has no kernel (supported: 16, 32, 40, 48, 64, 96, 128)",
              N);
    return YUF_ERR_UNSUPPORTED;
  }
  if ((long long)B * T * H == 0) return YUF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* scratch = nullptr;
  const size_t bytes = wkv7_backward_scratch_floats(B, H, N) * sizeof(float);
  cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&scratch), bytes, s);
  if (e != cudaSuccess) {
    set_error("wkv7 backward: scratch allocation of %zu bytes failed: %s", bytes,
              cudaGetErrorString(e));
    return YUF_ERR_OUT_OF_MEMORY;
  }
  st = wkv7_backward_dispatch(r, w, k, v, a, b, dy, states, sa, dr, dw, dk, dv, da, db, scratch, B,
                              T, H, N, s);
  scratch_free(scratch, s);
  return st;
}

yuf_status_t yuf_rosa_backward(const float* cand_saved, const float* write_saved,
                               const float* read_saved, const float* gate_saved,
                               const float* decay_saved, const float* mem_saved,
                               const float* direction, const float* final_memory,
                               const float* d_read, float* d_cand, float* d_write,
                               float* d_read_raw, float* d_decay, float* d_direction_partial,
                               float* d_memory_out, float* workspace, int B, int T, int R,
                               void* stream) {
  (void)read_saved;
  (void)gate_saved;
  (void)final_memory;
  (void)workspace;
  g_err[0] = 0;
  REQUIRE(B >= 0 && T >= 0, "rosa backward: negative size (B=%d T=%d)", B, T);
  REQUIRE(R >= 1 && R <= 1024, "rosa backward: R=%d outside 1..1024", R);
  REQUIRE(B == 0 || (direction && mem_saved && d_direction_partial && d_memory_out),
          "rosa backward: direction, mem_saved, d_direction_partial, d_memory_out are required");
  REQUIRE((long long)B * T == 0 || (cand_saved && write_saved && decay_saved && d_read && d_cand &&
                                    d_write && d_read_raw && d_decay),
          "rosa backward: a per-step tensor is NULL");
  if (B == 0) return YUF_OK;
  return rosa_backward_dispatch(cand_saved, write_saved, decay_saved, mem_saved, direction, d_read,
                                d_cand, d_write, d_read_raw, d_decay, d_direction_partial,
                                d_memory_out, B, T, R, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
