/*
 * cc1d_oracle.c -- plain C (OpenMP) restatement of the reference causal_conv1d
 * forward and backward, TEST INFRASTRUCTURE ONLY.
 *
 * Used as the timed CPU baseline (bench.py's cpu_baseline and --impl reference legs)
 * and cross-checked against the numpy restatement (oracle/numpy_oracle.py) by the CPU
 * test suite.  Never linked into the product library.
 *
 * Semantics restated (paths relative to the reference project root):
 *   forward   causal_conv1d/causal_conv1d_interface.py:135-174 (causal_conv1d_ref) and
 *             causal_conv1d/cpp_functions.py:21-54 (seq_idx masks, initial states),
 *             final states cpp_functions.py:57-61,82-88;
 *   backward  autograd through the above (cpp_functions.py:115-166).
 * Arithmetic: fp32 accumulation, one rounding to the output dtype.
 * Element types: 0 = float32, 1 = float16, 2 = bfloat16 (storage bits).
 * Strides are in elements; tensors are logical (batch, dim, seqlen).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BLK 64 /* channels per work item */

static inline float ld(const void* p, int dt, int64_t i) {
  if (dt == 0) return ((const float*)p)[i];
  if (dt == 1) return (float)((const _Float16*)p)[i];
  uint32_t u = ((uint32_t)((const uint16_t*)p)[i]) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline void st(void* p, int dt, int64_t i, float v) {
  if (dt == 0) {
    ((float*)p)[i] = v;
  } else if (dt == 1) {
    ((_Float16*)p)[i] = (_Float16)v;
  } else {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      ((uint16_t*)p)[i] = (uint16_t)((u >> 16) | 0x40u);
    } else {
      u += 0x7fffu + ((u >> 16) & 1u);
      ((uint16_t*)p)[i] = (uint16_t)(u >> 16);
    }
  }
}

static inline float silu(float p) { return p / (1.0f + expf(-p)); }

static inline float silu_grad(float p) {
  float s = 1.0f / (1.0f + expf(-p));
  return s * (1.0f + p * (1.0f - s));
}

/* x at position l (l may be negative: initial states or zero). */
static inline float x_at(const void* x, int xdt, const int64_t* xs, const void* init, int idt,
                         const int64_t* is, int64_t b, int64_t d, int64_t l, int W) {
  if (l >= 0) return ld(x, xdt, b * xs[0] + d * xs[1] + l * xs[2]);
  if (!init) return 0.0f;
  return ld(init, idt, b * is[0] + d * is[1] + (W - 1 + l) * is[2]);
}

int cc1d_oracle_fwd(int64_t B, int64_t D, int64_t L, int W, int xdt, const void* x, const int64_t* xs,
                    const float* weight, const float* bias, const int32_t* seq, int idt, const void* init,
                    const int64_t* is, int act, void* out, const int64_t* os, int fdt, void* fin,
                    const int64_t* fs) {
  const int64_t nblk = (D + BLK - 1) / BLK;
#pragma omp parallel for schedule(static)
  for (int64_t item = 0; item < B * nblk; ++item) {
    const int64_t b = item / nblk;
    const int64_t d0 = (item % nblk) * BLK;
    const int64_t d1 = d0 + BLK < D ? d0 + BLK : D;
    for (int64_t l = 0; l < L; ++l) {
      const int32_t s_cur = seq ? seq[b * L + l] : 0;
      for (int64_t d = d0; d < d1; ++d) {
        float acc = bias ? bias[d] : 0.0f;
        for (int w = 0; w < W; ++w) {
          const int64_t pos = l - (W - 1) + w;
          if (seq && (pos < 0 || seq[b * L + pos] != s_cur)) continue;
          acc += weight[d * W + w] * x_at(x, xdt, xs, init, idt, is, b, d, pos, W);
        }
        if (seq && s_cur < 0) acc = 0.0f;
        if (act) acc = silu(acc);
        st(out, xdt, b * os[0] + d * os[1] + l * os[2], acc);
      }
    }
    if (fin) {
      for (int64_t d = d0; d < d1; ++d)
        for (int k = 0; k < W - 1; ++k) {
          const int64_t pos = L - (W - 1) + k;
          st(fin, fdt, b * fs[0] + d * fs[1] + k * fs[2], x_at(x, xdt, xs, init, idt, is, b, d, pos, W));
        }
    }
  }
  return 0;
}

/* dweight (D, W) and dbias (D,) are fp32 outputs; dinit/dfinal optional. */
int cc1d_oracle_bwd(int64_t B, int64_t D, int64_t L, int W, int xdt, const void* x, const int64_t* xs,
                    const float* weight, const float* bias, const int32_t* seq, int idt, const void* init,
                    const int64_t* is, const void* dout, const int64_t* gs, int dfdt, const void* dfinal,
                    const int64_t* dfs, int act, void* dx, const int64_t* dxs, void* dinit,
                    const int64_t* dis, float* dweight, float* dbias) {
  const int64_t nblk = (D + BLK - 1) / BLK;
  float* part = (float*)calloc((size_t)(B * D * (W + 1)), sizeof(float));
  if (!part) return 1;
#pragma omp parallel for schedule(static)
  for (int64_t item = 0; item < B * nblk; ++item) {
    const int64_t b = item / nblk;
    const int64_t d0 = (item % nblk) * BLK;
    const int64_t d1 = d0 + BLK < D ? d0 + BLK : D;
    float* g = (float*)malloc((size_t)(L + W) * sizeof(float));
    for (int64_t d = d0; d < d1; ++d) {
      /* g[l] = dout * silu'(p) (masked) */
      for (int64_t l = 0; l < L; ++l) {
        const int32_t s_cur = seq ? seq[b * L + l] : 0;
        float gv = ld(dout, xdt, b * gs[0] + d * gs[1] + l * gs[2]);
        if (act) {
          float p = bias ? bias[d] : 0.0f;
          for (int w = 0; w < W; ++w) {
            const int64_t pos = l - (W - 1) + w;
            if (seq && (pos < 0 || seq[b * L + pos] != s_cur)) continue;
            p += weight[d * W + w] * x_at(x, xdt, xs, init, idt, is, b, d, pos, W);
          }
          if (seq && s_cur < 0) p = 0.0f;
          gv *= silu_grad(p);
        }
        if (seq && s_cur < 0) gv = 0.0f;
        g[l] = gv;
      }
      float* pd = part + (b * D + d) * (W + 1);
      for (int64_t l = 0; l < L; ++l) {
        const int32_t s_cur = seq ? seq[b * L + l] : 0;
        pd[W] += g[l];
        for (int w = 0; w < W; ++w) {
          const int64_t pos = l - (W - 1) + w;
          if (seq && (pos < 0 || seq[b * L + pos] != s_cur)) continue;
          pd[w] += g[l] * x_at(x, xdt, xs, init, idt, is, b, d, pos, W);
        }
      }
      /* dx[j] = sum_k w[W-1-k] g[j+k]; positions j < 0 are dinitial */
      const int64_t jlo = dinit ? -(int64_t)(W - 1) : 0;
      for (int64_t j = jlo; j < L; ++j) {
        const int32_t s_j = (seq && j >= 0) ? seq[b * L + j] : -1;
        float s = 0.0f;
        for (int k = 0; k < W; ++k) {
          const int64_t q = j + k;
          if (q < 0 || q >= L) continue;
          if (seq && seq[b * L + q] != s_j) continue;
          s += weight[d * W + (W - 1 - k)] * g[q];
        }
        const int64_t tail0 = L - (W - 1);
        if (dfinal && j >= tail0) s += ld(dfinal, dfdt, b * dfs[0] + d * dfs[1] + (j - tail0) * dfs[2]);
        if (j >= 0) st(dx, xdt, b * dxs[0] + d * dxs[1] + j * dxs[2], s);
        else st(dinit, idt, b * dis[0] + d * dis[1] + (j + W - 1) * dis[2], s);
      }
    }
    free(g);
  }
  /* fixed-order reduction over the batch */
  for (int64_t d = 0; d < D; ++d) {
    for (int w = 0; w <= W; ++w) {
      float s = 0.0f;
      for (int64_t b = 0; b < B; ++b) s += part[(b * D + d) * (W + 1) + w];
      if (w < W) dweight[d * W + w] = s;
      else if (dbias) dbias[d] = s;
    }
  }
  free(part);
  return 0;
}

int cc1d_oracle_max_threads(void) {
#ifdef _OPENMP
  extern int omp_get_max_threads(void);
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Sets the OpenMP thread count of the calls above (launchers such as torchrun set
 * OMP_NUM_THREADS=1 for every process; the CPU baseline wants every host core). */
void cc1d_oracle_set_threads(int n) {
#ifdef _OPENMP
  extern void omp_set_num_threads(int);
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
