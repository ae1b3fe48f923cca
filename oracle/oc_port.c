/*
 * CPU port of the reference's decode path — TEST / BASELINE INFRASTRUCTURE.
 *
 * Only bench.py's cpu_baseline leg and its `--impl reference` arm, and the
 * tests, call this library.  The product (orthocache_b200) never links it.
 *
 * It restates, in C with OpenMP over all host cores, what the reference's
 * CPU (JAX/XLA) path computes for one decode step of
 * pipeline.orthocache_forward(mode='compact') with a given tau:
 *
 *   1. compute_multiband_mask (spectral_energy.py:199-234):
 *      gate 1 = compute_query_aware_mask -> compute_query_aware_bounds, which
 *      runs the 512-point FWHT of every key block (spectral_energy.py:156);
 *      gate 2 = compute_spectral_decay_ratio -> compute_spectral_bands, which
 *      runs the FWHT of every key block again (spectral_energy.py:90).  The
 *      port keeps both transforms, as the reference does.
 *   2. stream compaction (compaction.py:56-98): union over heads, stable
 *      active-first order, copy of the retained K/V blocks into compact
 *      buffers with a zero tail.
 *   3. attention over the num_active compacted blocks with the online
 *      softmax of adaptive_attention._multihead_loop (adaptive_attention.py:90-120):
 *      fp32 logits q.k / sqrt(d), running max / sum / output, o / l.
 *
 * FWHT: stages h = 1..256, a+b / a-b, then / 22.627416997969522 (fwht.py:25-61).
 * Keys / values / queries are bfloat16 (uint16 bit patterns), as in the
 * benchmark configuration; arithmetic is float32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define BLK 512

static inline float bf(uint16_t x) {
  union { uint32_t u; float f; } c;
  c.u = ((uint32_t)x) << 16;
  return c.f;
}

/* FWHT of a 512 x D tile (row-major, rows = tokens) in place. */
static void fwht_tile(float* t, int D) {
  for (int h = 1; h < BLK; h <<= 1)
    for (int i = 0; i < BLK; i += 2 * h)
      for (int j = i; j < i + h; ++j) {
        float* a = t + (size_t)j * D;
        float* b = t + (size_t)(j + h) * D;
        for (int c = 0; c < D; ++c) {
          const float x = a[c], y = b[c];
          a[c] = x + y;
          b[c] = x - y;
        }
      }
  const float norm = 22.627416997969522f;
  for (size_t e = 0; e < (size_t)BLK * D; ++e) t[e] = t[e] / norm;
}

static void load_tile(float* t, const uint16_t* k, int j, int h, int H, int D) {
  for (int r = 0; r < BLK; ++r) {
    const uint16_t* src = k + (((size_t)j * BLK + r) * H + h) * D;
    for (int c = 0; c < D; ++c) t[(size_t)r * D + c] = bf(src[c]);
  }
}

/* The two gates' scores of the first nb blocks: bmax (nb, Hkv) = max over the
 * Sq*G query rows of the query-aware bound (FWHT pass 1), zeta (nb, Hkv) =
 * E_high / (E_low + 1e-6) (FWHT pass 2), as compute_multiband_mask computes
 * them (spectral_energy.py:141-234). */
static void port_scores(const uint16_t* k, const uint16_t* q, int nb, int Hkv, int Hq, int D, int Sq, float* bmax,
                        float* zeta) {
  const int G = Hq / Hkv;
  const float sqrt_d = sqrtf((float)D);
  /* Gate 1: query-aware bounds (FWHT pass 1). */
#pragma omp parallel
  {
    float* t = (float*)malloc(sizeof(float) * BLK * D);
#pragma omp for schedule(dynamic)
    for (int cell = 0; cell < nb * Hkv; ++cell) {
      const int j = cell / Hkv, h = cell % Hkv;
      load_tile(t, k, j, h, Hkv, D);
      fwht_tile(t, D);
      double ac = 0.0;
      for (size_t e = D; e < (size_t)BLK * D; ++e) ac += (double)t[e] * t[e];
      const float sac = sqrtf((float)ac);
      float m = -INFINITY;
      for (int s = 0; s < Sq; ++s)
        for (int g = 0; g < G; ++g) {
          const uint16_t* qr = q + ((size_t)s * Hq + h * G + g) * D;
          float dot = 0.f, nrm = 0.f;
          for (int c = 0; c < D; ++c) {
            const float qv = bf(qr[c]);
            dot += qv * (t[c] / 22.627416997969522f);
            nrm += qv * qv;
          }
          const float b = dot / sqrt_d + sqrtf(nrm) * sac / sqrt_d;
          if (b > m) m = b;
        }
      bmax[cell] = m;
    }
    free(t);
  }
  /* Gate 2: spectral decay ratio (FWHT pass 2). */
#pragma omp parallel
  {
    float* t = (float*)malloc(sizeof(float) * BLK * D);
#pragma omp for schedule(dynamic)
    for (int cell = 0; cell < nb * Hkv; ++cell) {
      const int j = cell / Hkv, h = cell % Hkv;
      load_tile(t, k, j, h, Hkv, D);
      fwht_tile(t, D);
      double lo = 0.0, hi = 0.0;
      for (int r = 1; r < 64; ++r)
        for (int c = 0; c < D; ++c) lo += (double)t[(size_t)r * D + c] * t[(size_t)r * D + c];
      for (int r = 256; r < BLK; ++r)
        for (int c = 0; c < D; ++c) hi += (double)t[(size_t)r * D + c] * t[(size_t)r * D + c];
      zeta[cell] = (float)hi / ((float)lo + 1e-6f);
    }
    free(t);
  }
}

int oc_port_scores(const uint16_t* k, const uint16_t* q, int S, int Hkv, int Hq, int D, int Sq, float* bmax,
                   float* zeta) {
  port_scores(k, q, S / BLK, Hkv, Hq, D, Sq, bmax, zeta);
  return 0;
}

int oc_port_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/*
 * One decode step.  k, v: (S, Hkv, D) bf16; q: (Sq, Hq, D) bf16.
 * Outputs: keep (nb, Hkv) uint8; perm (nb) int32; *count; out (Sq, Hq, D) f32.
 * blocks_limit > 0 restricts scoring to the first blocks_limit blocks (a
 * bounded sample for timing); attention still covers the retained ones.
 * Scratch: compact_k / compact_v, each nb*512*Hkv*D uint16 (caller-owned).
 */
int oc_port_decode(const uint16_t* k, const uint16_t* v, const uint16_t* q, int S, int Hkv, int Hq, int D,
                   int Sq, float tau, float zeta_max, int blocks_limit, uint8_t* keep, int32_t* perm,
                   int32_t* count, float* out, uint16_t* compact_k, uint16_t* compact_v) {
  const int nb_all = S / BLK;
  const int nb = blocks_limit > 0 && blocks_limit < nb_all ? blocks_limit : nb_all;
  const int G = Hq / Hkv;
  const float sqrt_d = sqrtf((float)D);
  float* bmax = (float*)malloc(sizeof(float) * nb * Hkv);
  float* zeta = (float*)malloc(sizeof(float) * nb * Hkv);

  port_scores(k, q, nb, Hkv, Hq, D, Sq, bmax, zeta);
  /* Two gates, union over heads, stable compaction. */
  int n = 0;
  for (int j = 0; j < nb_all; ++j) {
    int any = 0;
    for (int h = 0; h < Hkv; ++h) {
      uint8_t kp = 0;
      if (j < nb) kp = (bmax[j * Hkv + h] >= tau) && (zeta[j * Hkv + h] <= zeta_max);
      keep[j * Hkv + h] = kp;
      any |= kp;
    }
    if (any) perm[n++] = j;
  }
  int m_i = n;
  for (int j = 0; j < nb_all; ++j) {
    int any = 0;
    for (int h = 0; h < Hkv; ++h) any |= keep[j * Hkv + h];
    if (!any) perm[m_i++] = j;
  }
  *count = n;
  /* Copy retained blocks into the compact buffers, zero tail (compaction.py:85-98). */
  const size_t blk_elems = (size_t)BLK * Hkv * D;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < nb_all; ++i) {
    if (i < n) {
      memcpy(compact_k + i * blk_elems, k + (size_t)perm[i] * blk_elems, blk_elems * 2);
      memcpy(compact_v + i * blk_elems, v + (size_t)perm[i] * blk_elems, blk_elems * 2);
    } else {
      memset(compact_k + i * blk_elems, 0, blk_elems * 2);
      memset(compact_v + i * blk_elems, 0, blk_elems * 2);
    }
  }
  /* Online-softmax attention over the n compacted blocks, per (row, query head). */
#pragma omp parallel
  {
    float* lg = (float*)malloc(sizeof(float) * BLK);
    float* o = (float*)malloc(sizeof(float) * D);
#pragma omp for schedule(dynamic)
    for (int row = 0; row < Sq * Hq; ++row) {
      const int s = row / Hq, hq = row % Hq, h = hq / G;
      const uint16_t* qr = q + ((size_t)s * Hq + hq) * D;
      float qf[512];
      for (int c = 0; c < D; ++c) qf[c] = bf(qr[c]);
      float mrun = -1e30f, l = 0.f;
      for (int c = 0; c < D; ++c) o[c] = 0.f;
      for (int i = 0; i < n; ++i) {
        float mb = -INFINITY;
        for (int t = 0; t < BLK; ++t) {
          const uint16_t* kr = compact_k + i * blk_elems + ((size_t)t * Hkv + h) * D;
          float dot = 0.f;
          for (int c = 0; c < D; ++c) dot += qf[c] * bf(kr[c]);
          lg[t] = dot / sqrt_d;
          if (lg[t] > mb) mb = lg[t];
        }
        const float mn = mb > mrun ? mb : mrun;
        const float sc = expf(mrun - mn);
        l *= sc;
        for (int c = 0; c < D; ++c) o[c] *= sc;
        for (int t = 0; t < BLK; ++t) {
          const float p = expf(lg[t] - mn);
          l += p;
          const uint16_t* vr = compact_v + i * blk_elems + ((size_t)t * Hkv + h) * D;
          for (int c = 0; c < D; ++c) o[c] += p * bf(vr[c]);
        }
        mrun = mn;
      }
      for (int c = 0; c < D; ++c) out[(size_t)row * D + c] = n ? o[c] / l : 0.f;
    }
    free(lg);
    free(o);
  }
  free(bmax);
  free(zeta);
  return 0;
}
