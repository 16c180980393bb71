/*
 * CPU oracle for the Qwen3 attention hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's semantics, used (a) by the tests
 * as the checker of the CUDA path and (b) by bench.py as the timed CPU
 * baseline.  Nothing in the product path links or calls this file.
 *
 * What it restates (reference = aeilot/roofline-inference):
 *   - qk-norm + RoPE: agent-test/v2/kernels.py:116-146 (one token) and
 *     :169-204 (L tokens), as pinned by the reference test
 *     agent-test/v2/test_engine.py:52-59 (mx.fast.rms_norm eps 1e-6,
 *     mx.fast.rope(dims 128, traditional=False, base, scale 1.0, offset)).
 *     RMSNorm rounding points n = bf16(w * bf16(x * inv)) (kernels.py:131-133).
 *     The RoPE angle is the reference's FP32 value (kernels.py:134-138, 152):
 *     theta = float(pos) * exp2(-(d/64) * float(log2(base))), each product
 *     rounded to FP32 and exp2 rounded once to FP32 (mx.fast.rope forms it
 *     the same way).  Its cosine/sine are then evaluated in FP64, the value
 *     the Metal fast::cos / fast::sin approximate.  With angle_f64 set the
 *     angle itself is formed in FP64 instead (the idealised rope), to count
 *     how far the reference's FP32 angle moves the BF16 outputs.
 *   - decode attention: the MLX call at agent-test/v2/engine.py:154-155,
 *     softmax(scale * q K^T) V over n keys, GQA head h -> KV head h / 2,
 *     no mask (engine.py:148-155).  FP32 arithmetic, exact max, one rounding
 *     of the output.
 *   - causal prefill attention: agent-test/v2/attention.py:1-11, 24, 111
 *     (bottom-right aligned mask: query i sees keys <= kL - qL + i), FP32.
 * Outputs are returned unrounded (FP32) and/or rounded once to BF16 (round to
 * nearest even), so tests can measure error both ways.
 *
 * Parity status: no golden vector of the reference survives without MLX
 * (its tests draw inputs from mx.random), so this oracle is pinned against an
 * independent FP64 numpy restatement (oracle/reference_np.py) and committed
 * fixtures (tests/golden/), not against MLX itself.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define D 128

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* round to nearest even; inputs here are finite */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* dot product of two 128-vectors, 8 independent partial sums (vectorises) */
static inline float dot128(const float *a, const float *b) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int d = 0; d < D; d += 8)
    for (int u = 0; u < 8; ++u) acc[u] += a[d + u] * b[d + u];
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

int oracle_version(void) { return 1; }

/* ---------------------------------------------------------------- rope
 * qkv [L][(nq+2nkv)*128] -> q_out [nq][Lp][128] (rows >= L zero),
 * kv_out [2][nkv][kv_rows][128] written at rows kv_row0 + t. */
void oracle_qk_norm_rope(const uint16_t *qkv, int L, const uint16_t *qw, const uint16_t *kw,
                         int offset, int nq, int nkv, double base, int Lp, uint16_t *q_out,
                         uint16_t *kv_out, int kv_rows, int kv_row0, int angle_f64) {
  const int items = nq + 2 * nkv;
  float inv_freq[64];
  double inv_freq64[64];
  const float lb = (float)log2(base); /* the f-string literal, read as FP32 */
  for (int d = 0; d < 64; ++d) {
    volatile float x = -((float)d / 64.0f) * lb; /* one FP32 rounding */
    inv_freq[d] = (float)exp2((double)x);
    inv_freq64[d] = pow(base, -(double)d / 64.0);
  }
  memset(q_out, 0, sizeof(uint16_t) * (size_t)nq * Lp * D);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < L; ++t) {
    double cs[64], sn[64];
    for (int d = 0; d < 64; ++d) {
      volatile float th32 = (float)(offset + t) * inv_freq[d]; /* FP32 product */
      const double th = angle_f64 ? (double)(offset + t) * inv_freq64[d] : (double)th32;
      cs[d] = cos(th);
      sn[d] = sin(th);
    }
    for (int item = 0; item < items; ++item) {
      const uint16_t *src = qkv + ((size_t)t * items + item) * D;
      if (item >= nq + nkv) { /* V: copy */
        const int hv = item - nq - nkv;
        memcpy(kv_out + ((size_t)(nkv + hv) * kv_rows + kv_row0 + t) * D, src, D * sizeof(uint16_t));
        continue;
      }
      const uint16_t *w = item < nq ? qw : kw;
      float x[D];
      double ss = 0.0;
      for (int d = 0; d < D; ++d) {
        x[d] = bf16_to_f32(src[d]);
        ss += (double)x[d] * x[d];
      }
      const float inv = (float)(1.0 / sqrt(ss / 128.0 + 1e-6));
      double nv[D];
      for (int d = 0; d < D; ++d) nv[d] = round_bf16(bf16_to_f32(w[d]) * round_bf16(x[d] * inv));
      uint16_t *dst = item < nq ? q_out + ((size_t)item * Lp + t) * D
                                : kv_out + ((size_t)(item - nq) * kv_rows + kv_row0 + t) * D;
      for (int d = 0; d < 64; ++d) {
        const double x1 = nv[d], x2 = nv[d + 64];
        dst[d] = f32_to_bf16((float)(x1 * cs[d] - x2 * sn[d]));
        dst[d + 64] = f32_to_bf16((float)(x1 * sn[d] + x2 * cs[d]));
      }
    }
  }
}

/* ---------------------------------------------------------------- decode
 * One KV head `h` of one sequence: q heads 2h, 2h+1.  K, V: [n][128] rows of
 * this head.  Writes out_f32[2][128]. */
static void decode_head(const uint16_t *q2, const uint16_t *K, const uint16_t *V, int n,
                        float scale, float *out_f32, float *scratch /* [2][n] */) {
  float qf[2][D];
  for (int hh = 0; hh < 2; ++hh)
    for (int d = 0; d < D; ++d) qf[hh][d] = bf16_to_f32(q2[hh * D + d]);
  float *s0 = scratch, *s1 = scratch + n;
  float m0 = -INFINITY, m1 = -INFINITY;
  float kf[D];
  for (int i = 0; i < n; ++i) {
    const uint16_t *kr = K + (size_t)i * D;
    for (int d = 0; d < D; ++d) kf[d] = bf16_to_f32(kr[d]);
    s0[i] = dot128(qf[0], kf) * scale;
    s1[i] = dot128(qf[1], kf) * scale;
    if (s0[i] > m0) m0 = s0[i];
    if (s1[i] > m1) m1 = s1[i];
  }
  float o0[D], o1[D];
  for (int d = 0; d < D; ++d) o0[d] = o1[d] = 0.f;
  double l0 = 0.0, l1 = 0.0;
  for (int i = 0; i < n; ++i) {
    const float p0 = expf(s0[i] - m0), p1 = expf(s1[i] - m1);
    l0 += p0;
    l1 += p1;
    const uint16_t *vr = V + (size_t)i * D;
    for (int d = 0; d < D; ++d) {
      const float v = bf16_to_f32(vr[d]);
      o0[d] += p0 * v;
      o1[d] += p1 * v;
    }
  }
  for (int d = 0; d < D; ++d) {
    out_f32[d] = (float)(o0[d] / l0);
    out_f32[D + d] = (float)(o1[d] / l1);
  }
}

/* B sequences; caches[b] -> [2][nkv][cap][128]; lens[b] keys; q [B][nq][128];
 * out_f32 [B][nq][128] (may be NULL), out_bf16 [B][nq][128] (may be NULL).
 * scratch: [threads][2][max_n] floats supplied by the caller via a
 * per-thread allocation inside (variable-length arrays on the heap). */
#include <stdlib.h>
void oracle_decode_attention_batched(const uint16_t *q, const uint16_t *const *caches,
                                     const int32_t *lens, int B, int cap, int nq, int nkv,
                                     float scale, float *out_f32, uint16_t *out_bf16) {
  int max_n = 1;
  for (int b = 0; b < B; ++b)
    if (lens[b] > max_n) max_n = lens[b];
#pragma omp parallel
  {
    float *scratch = (float *)malloc(sizeof(float) * 2 * (size_t)max_n);
#pragma omp for collapse(2) schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
      for (int h = 0; h < nkv; ++h) {
        const uint16_t *cache = caches[b];
        const uint16_t *K = cache + (size_t)h * cap * D;
        const uint16_t *V = cache + (size_t)(nkv + h) * cap * D;
        float o[2 * D];
        decode_head(q + ((size_t)b * nq + 2 * h) * D, K, V, lens[b], scale, o, scratch);
        for (int hh = 0; hh < 2; ++hh)
          for (int d = 0; d < D; ++d) {
            const size_t idx = ((size_t)b * nq + 2 * h + hh) * D + d;
            if (out_f32) out_f32[idx] = o[hh * D + d];
            if (out_bf16) out_bf16[idx] = f32_to_bf16(o[hh * D + d]);
          }
      }
    }
    free(scratch);
  }
}

void oracle_decode_attention(const uint16_t *q, const uint16_t *cache, int cap, int n, int nq,
                             int nkv, float scale, float *out_f32, uint16_t *out_bf16) {
  const uint16_t *caches[1] = {cache};
  const int32_t lens[1] = {n};
  oracle_decode_attention_batched(q, caches, lens, 1, cap, nq, nkv, scale, out_f32, out_bf16);
}

/* ---------------------------------------------------------------- prefill
 * Q [H][qLp][128]; K, V [nkv][cap][128]; query rows [row_begin, row_end) of
 * every head; out_f32 [qL][H*128] (only the selected rows are written). */
void oracle_prefill_attention(const uint16_t *Q, const uint16_t *K, const uint16_t *V, int qL,
                              int kL, int qLp, int cap, int H, int nkv, float scale,
                              int row_begin, int row_end, float *out_f32) {
  const int off = kL - qL;
  const int group = H / nkv;
#pragma omp parallel
  {
    float *s = (float *)malloc(sizeof(float) * (size_t)kL);
    float *kf = (float *)malloc(sizeof(float) * (size_t)D);
#pragma omp for collapse(2) schedule(dynamic, 4)
    for (int h = 0; h < H; ++h) {
      for (int i = row_begin; i < row_end; ++i) {
        const int g = h / group;
        const uint16_t *Kg = K + (size_t)g * cap * D;
        const uint16_t *Vg = V + (size_t)g * cap * D;
        float qf[D];
        for (int d = 0; d < D; ++d) qf[d] = bf16_to_f32(Q[((size_t)h * qLp + i) * D + d]);
        const int last = off + i; /* inclusive */
        float m = -INFINITY;
        for (int j = 0; j <= last; ++j) {
          for (int d = 0; d < D; ++d) kf[d] = bf16_to_f32(Kg[(size_t)j * D + d]);
          s[j] = dot128(qf, kf) * scale;
          if (s[j] > m) m = s[j];
        }
        float o[D];
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        double l = 0.0;
        for (int j = 0; j <= last; ++j) {
          const float p = expf(s[j] - m);
          l += p;
          const uint16_t *vr = Vg + (size_t)j * D;
          for (int d = 0; d < D; ++d) o[d] += p * bf16_to_f32(vr[d]);
        }
        float *dst = out_f32 + (size_t)i * H * D + (size_t)h * D;
        for (int d = 0; d < D; ++d) dst[d] = (float)(o[d] / l);
      }
    }
    free(s);
    free(kf);
  }
}
