/* Plain-C restatement of the two hot-path recurrences -- TEST INFRASTRUCTURE.
 *
 * Used as the timed CPU baseline (bench.py's cpu_baseline leg and
 * `bench.py --impl reference`) and as a second oracle in tests.  It follows
 * the reference's PyTorch fp32 loops:
 *   WKV-7: RWKV7TimeMix._torch_recurrence   yufmusicgen/model.py:145-165
 *   ROSA : ROSAMemory._reference_recurrence yufmusicgen/model.py:260-288
 * Each (batch, head) chain of the WKV scan and each batch row of the ROSA
 * scan is independent, so OpenMP spreads them over the host cores.
 * Layouts: r,w,k,v,a,b,y [B,T,H,N]; S [B,H,N,N] row i = value, col j = key.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

void oracle_wkv7_scan(const float* r, const float* w, const float* k, const float* v,
                      const float* a, const float* b, const float* s0, float* y, float* sT,
                      int B, int T, int H, int N, int n_threads) {
#pragma omp parallel for collapse(2) schedule(static) num_threads(n_threads)
  for (int bb = 0; bb < B; ++bb) {
    for (int hh = 0; hh < H; ++hh) {
      float* S = (float*)malloc(sizeof(float) * N * N);
      float* ret = (float*)malloc(sizeof(float) * N);
      float* sa = (float*)malloc(sizeof(float) * N);
      const size_t sbase = ((size_t)bb * H + hh) * N * N;
      if (s0) memcpy(S, s0 + sbase, sizeof(float) * N * N);
      else memset(S, 0, sizeof(float) * N * N);
      for (int t = 0; t < T; ++t) {
        const size_t o = (((size_t)bb * T + t) * H + hh) * N;
        for (int j = 0; j < N; ++j) ret[j] = expf(-0.6065306597f * sigm(w[o + j]));
        for (int i = 0; i < N; ++i) {        /* sa_i = sum_j a_j S_ij */
          float acc = 0.f;
          for (int j = 0; j < N; ++j) acc += a[o + j] * S[i * N + j];
          sa[i] = acc;
        }
        for (int i = 0; i < N; ++i) {        /* S_ij = S_ij ret_j + sa_i b_j + v_i k_j ; y_i = sum_j S_ij r_j */
          float acc = 0.f;
          const float vi = v[o + i], sai = sa[i];
          for (int j = 0; j < N; ++j) {
            float s = S[i * N + j] * ret[j] + sai * b[o + j] + vi * k[o + j];
            S[i * N + j] = s;
            acc += s * r[o + j];
          }
          y[o + i] = acc;
        }
      }
      if (sT) memcpy(sT + sbase, S, sizeof(float) * N * N);
      free(S); free(ret); free(sa);
    }
  }
}

/* read (gated) [B,T,R]; m0,mT [B,R]; decay post-sigmoid [R]; dir unit [R]. */
void oracle_rosa_scan(const float* cand, const float* write, const float* read_gate,
                      const float* decay, const float* dir, const float* m0, float* read,
                      float* mT, int B, int T, int R, int gated, int n_threads) {
#pragma omp parallel for schedule(static) num_threads(n_threads)
  for (int bb = 0; bb < B; ++bb) {
    float* m = (float*)malloc(sizeof(float) * R);
    memcpy(m, m0 + (size_t)bb * R, sizeof(float) * R);
    for (int t = 0; t < T; ++t) {
      const size_t o = ((size_t)bb * T + t) * R;
      float p = 0.f;
      for (int j = 0; j < R; ++j) p += m[j] * dir[j];
      for (int j = 0; j < R; ++j)
        m[j] = decay[j] * (m[j] - 2.f * p * dir[j]) + sigm(write[o + j]) * tanhf(cand[o + j]);
      float q = 0.f;
      for (int j = 0; j < R; ++j) q += m[j] * dir[j];
      for (int j = 0; j < R; ++j) {
        float rv = m[j] - 2.f * q * dir[j];
        read[o + j] = gated ? rv * sigm(read_gate[o + j]) : rv;
      }
    }
    memcpy(mT + (size_t)bb * R, m, sizeof(float) * R);
    free(m);
  }
}
