/*
 * C restatement of the PagedKV-Fusion reference arithmetic
 * (TEST INFRASTRUCTURE ONLY -- never linked into the product library).
 *
 * It spells out, operation by operation, the float32 evaluation order that
 * NumPy uses inside pagedkv_fusion/reference.py, so the bit-exact contract
 * of the CUDA kernels is written down in plain C and can be checked against
 * both NumPy and the golden vectors:
 *
 *   eviction score      reference.py:38-71   (pairwise masked sum, IEEE
 *                                              divide, unfused blend)
 *   eviction selection  reference.py:74-81   (ascending (score, id))
 *   quantization        reference.py:88-105  (IEEE divide, half-even)
 *   paged attention     reference.py:140-173 (evaluated in double here, a
 *                                              higher-precision yardstick)
 *
 * Built with -ffp-contract=off so no multiply-add is fused.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* NumPy's float32 pairwise sum over n contiguous values
 * (8 interleaved accumulators, fixed tree, sequential tail, halving above
 * 128 terms).  Restated from the behaviour of np.add.reduce on float32. */
static float pairwise_sum_f32(const float *a, int64_t n) {
  if (n < 8) {
    float r = 0.0f;
    for (int64_t i = 0; i < n; ++i) r = r + a[i];
    return r;
  }
  if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int64_t i = 8;
    const int64_t stop = n - (n % 8);
    for (; i < stop; i += 8)
      for (int j = 0; j < 8; ++j) r[j] = r[j] + a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res = res + a[i];
    return res;
  }
  int64_t half = n / 2;
  half -= half % 8;
  return pairwise_sum_f32(a, half) + pairwise_sum_f32(a + half, n - half);
}

void pkv_oracle_eviction_scores(const float *recency, const float *frequency,
                                const float *attn, const uint8_t *valid,
                                float *scores, int64_t num_blocks,
                                int64_t block_size, float w_r, float w_f,
                                float w_a) {
  float *row = (float *)malloc(sizeof(float) * (size_t)(block_size > 0 ? block_size : 1));
  for (int64_t b = 0; b < num_blocks; ++b) {
    int64_t n_valid = 0;
    for (int64_t t = 0; t < block_size; ++t) {
      const int ok = valid[b * block_size + t] != 0;
      row[t] = ok ? attn[b * block_size + t] : 0.0f;
      n_valid += ok;
    }
    const float total = 0.0f + pairwise_sum_f32(row, block_size); /* output starts at +0.0 */
    const float mean = n_valid > 0 ? (float)((double)total / (double)n_valid) : 0.0f;
    const float a = w_r * recency[b];
    const float f = w_f * frequency[b];
    const float m = w_a * mean;
    scores[b] = (a + f) + m;
  }
  free(row);
}

static uint32_t orderable_key(float s) {
  uint32_t u;
  memcpy(&u, &s, 4);
  if (isnan(s)) return 0xFFFFFFFFu;
  if (u == 0x80000000u) u = 0;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static int cmp_u64(const void *x, const void *y) {
  const uint64_t a = *(const uint64_t *)x, b = *(const uint64_t *)y;
  return (a > b) - (a < b);
}

/* out must hold min(k, n) entries; returns that count. */
int64_t pkv_oracle_select(const float *scores, int64_t n, int64_t k, int64_t *out) {
  if (k > n) k = n;
  if (k <= 0) return 0;
  uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)n);
  for (int64_t i = 0; i < n; ++i)
    keys[i] = ((uint64_t)orderable_key(scores[i]) << 32) | (uint64_t)i;
  qsort(keys, (size_t)n, sizeof(uint64_t), cmp_u64);
  for (int64_t i = 0; i < k; ++i) out[i] = (int64_t)(keys[i] & 0xFFFFFFFFu);
  free(keys);
  return k;
}

void pkv_oracle_quantize(const float *kv, int8_t *q, float *scale,
                         int64_t num_blocks, int64_t block_size,
                         int64_t num_kv_heads, int64_t head_dim) {
  for (int64_t b = 0; b < num_blocks; ++b) {
    for (int64_t h = 0; h < num_kv_heads; ++h) {
      float amax = 0.0f;
      for (int64_t t = 0; t < block_size; ++t)
        for (int64_t d = 0; d < head_dim; ++d) {
          const float x = fabsf(kv[((b * block_size + t) * num_kv_heads + h) * head_dim + d]);
          if (x > amax || isnan(x)) amax = x;
        }
      const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
      scale[b * num_kv_heads + h] = s;
      for (int64_t t = 0; t < block_size; ++t)
        for (int64_t d = 0; d < head_dim; ++d) {
          const int64_t i = ((b * block_size + t) * num_kv_heads + h) * head_dim + d;
          float r = rintf(kv[i] / s); /* default rounding: to nearest even */
          if (r > 127.0f) r = 127.0f;
          if (r < -127.0f) r = -127.0f;
          q[i] = (int8_t)r;
        }
    }
  }
}

/* Decode attention in double precision.  Returns 0, or -(s+1) when
 * sequence s references an out-of-range block. */
int64_t pkv_oracle_paged_attention(const float *q, const int8_t *kq, const float *ks,
                                   const int8_t *vq, const float *vs,
                                   const int32_t *block_tables, const int32_t *seq_lens,
                                   float *out, int64_t num_seqs, int64_t num_heads,
                                   int64_t num_kv_heads, int64_t head_dim,
                                   int64_t block_size, int64_t num_blocks,
                                   int64_t max_blocks, double sm_scale) {
  const int64_t group = num_heads / num_kv_heads;
  for (int64_t s = 0; s < num_seqs; ++s) {
    /* tokens beyond the block-table width are not attended (the CUDA path
     * clamps the same way and records PKV_DEVERR_SEQ_TOO_LONG) */
    int64_t L = seq_lens[s] > 0 ? seq_lens[s] : 0;
    if (L > max_blocks * block_size) L = max_blocks * block_size;
    double *logit = (double *)malloc(sizeof(double) * (size_t)(L > 0 ? L : 1));
    for (int64_t h = 0; h < num_heads; ++h) {
      const int64_t kvh = h / group;
      const float *qh = q + (s * num_heads + h) * head_dim;
      double *acc = (double *)calloc((size_t)head_dim, sizeof(double));
      double mx = -INFINITY, l = 0.0;
      for (int64_t t = 0; t < L; ++t) {
        const int64_t b = block_tables[s * max_blocks + t / block_size];
        if (b < 0 || b >= num_blocks) { free(acc); free(logit); return -(s + 1); }
        const int8_t *kr = kq + ((b * block_size + t % block_size) * num_kv_heads + kvh) * head_dim;
        const double sc = ks[b * num_kv_heads + kvh];
        double dot = 0.0;
        for (int64_t d = 0; d < head_dim; ++d) dot += (double)kr[d] * sc * (double)qh[d];
        logit[t] = dot * sm_scale;
        if (logit[t] > mx) mx = logit[t];
      }
      for (int64_t t = 0; t < L; ++t) {
        const int64_t b = block_tables[s * max_blocks + t / block_size];
        const int8_t *vr = vq + ((b * block_size + t % block_size) * num_kv_heads + kvh) * head_dim;
        const double p = exp(logit[t] - mx);
        const double sc = vs[b * num_kv_heads + kvh];
        l += p;
        for (int64_t d = 0; d < head_dim; ++d) acc[d] += p * (double)vr[d] * sc;
      }
      float *oh = out + (s * num_heads + h) * head_dim;
      for (int64_t d = 0; d < head_dim; ++d) oh[d] = L > 0 ? (float)(acc[d] / l) : 0.0f;
      free(acc);
    }
    free(logit);
  }
  return 0;
}
