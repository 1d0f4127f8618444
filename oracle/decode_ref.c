/* CPU restatement of the reference's decoder_forward step (test infrastructure: the timed
 * CPU baseline and a checker, never part of the product path).
 *
 * Follows crates/qwen-asr/src/decoder.rs:550-645 with the kernels it calls:
 *   rms_norm                      kernels/mod.rs:1191-1212
 *   quantize_f32_to_int8          kernels/mod.rs:1795-1802 (round half away from zero)
 *   int8 matvecs q/k/v, SwiGLU,   kernels/mod.rs:884-1034, leaf kernels/neon.rs:716-800:
 *     out-proj/down + residual      y = (float)(int32 sum) * x_scale * w_scale
 *   bf16 matvecs                  kernels/generic.rs:10-21 (f32 accumulation)
 *   per-head RMSNorm + NeoX RoPE  kernels/mod.rs:1214-1240, 1780-1788
 *   single-token attention        kernels/mod.rs:1492-1534 (online softmax, one pass)
 *   SwiGLU                        kernels/mod.rs:1291-1340 (g / (1 + exp(-g)) * u)
 *   final norm + argmax           kernels/mod.rs:1832-1939 (first maximum wins)
 * The KV cache is f32 [layer][kv_head][max_seq][128] (decoder.rs:185-197), filled by the
 * caller's prefill. Weights arrive exactly as the reference holds them: int8 rows with f32
 * row scales (quantised at load) or bf16 bits. Matvec rows are spread over OpenMP threads,
 * as the reference spreads them over its thread pool (kernels/mod.rs:839-881). */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  int hidden, q_heads, kv_heads, inter, layers, vocab, max_seq, int8;
  float eps;
  /* per layer (arrays of `layers` pointers); q/k/v rows concatenated, gate/up interleaved */
  const int8_t* const* q_qkv;
  const float* const* s_qkv;
  const int8_t* const* q_o;
  const float* const* s_o;
  const int8_t* const* q_gu;
  const float* const* s_gu;
  const int8_t* const* q_down;
  const float* const* s_down;
  const uint16_t* const* b_qkv;
  const uint16_t* const* b_o;
  const uint16_t* const* b_gu;
  const uint16_t* const* b_down;
  const float* const* n1;
  const float* const* n2;
  const float* const* qn;
  const float* const* kn;
  const float* final_norm;
  const int8_t* lm_q;
  const float* lm_s;
  const uint16_t* lm_b;
  const uint16_t* embed; /* [vocab][hidden] bf16 */
  const float* inv_freq; /* [64] */
  float* k_cache;
  float* v_cache;
} RefModel;

static inline float bf16f(uint16_t b) {
  union {
    uint32_t u;
    float f;
  } v;
  v.u = (uint32_t)b << 16;
  return v.f;
}

static void rms_norm(const float* x, const float* w, float* y, int n, float eps) {
  float ss = 0.f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}

static float round_half_away(float v) { return v >= 0.f ? floorf(v + 0.5f) : -floorf(-v + 0.5f); }

static float quantize(const float* x, int n, int8_t* q) {
  float amax = 0.f;
  for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
  const float scale = amax > 0.f ? amax / 127.0f : 1.0f;
  const float inv = 127.0f / fmaxf(amax, 1e-10f);
  for (int i = 0; i < n; ++i) {
    float r = round_half_away(x[i] * inv);
    r = r > 127.f ? 127.f : (r < -127.f ? -127.f : r);
    q[i] = (int8_t)r;
  }
  return scale;
}

/* y[o] (+)= W[o] . x for rows [0, rows) */
static void mv_int8(const int8_t* w, const float* ws, const int8_t* xq, float xs, int rows, int cols, float* y,
                    const float* resid) {
#pragma omp parallel for schedule(static)
  for (int o = 0; o < rows; ++o) {
    const int8_t* r = w + (size_t)o * cols;
    int32_t acc = 0;
    for (int i = 0; i < cols; ++i) acc += (int32_t)r[i] * (int32_t)xq[i];
    float v = (float)acc * xs * ws[o];
    y[o] = resid ? resid[o] + v : v;
  }
}

static void mv_bf16(const uint16_t* w, const float* x, int rows, int cols, float* y, const float* resid) {
#pragma omp parallel for schedule(static)
  for (int o = 0; o < rows; ++o) {
    const uint16_t* r = w + (size_t)o * cols;
    float acc = 0.f;
    for (int i = 0; i < cols; ++i) acc += bf16f(r[i]) * x[i];
    y[o] = resid ? resid[o] + acc : acc;
  }
}

static void head_norm_rope(float* v, const float* w, float eps, const float* c, const float* s) {
  float t[128];
  rms_norm(v, w, t, 128, eps);
  for (int d = 0; d < 64; ++d) {
    v[d] = t[d] * c[d] + (-t[d + 64]) * s[d];
    v[d + 64] = t[d + 64] * c[d] + t[d] * s[d];
  }
}

/* Runs n_steps decoder_forward steps from position pos0. Step 0 consumes x0 (a prompt row),
 * step i > 0 the embedding of forced[i-1] (teacher forcing) or of the previous argmax.
 * out_ids[i] = step i's argmax; logits (optional) = the last step's logits. Returns 0. */
int qasr_ref_decode(const RefModel* m, const float* x0, int pos0, int n_steps, const int* forced, int* out_ids,
                    float* logits) {
  const int h = m->hidden, qd = m->q_heads * 128, kvd = m->kv_heads * 128, inter = m->inter;
  const int G = m->q_heads / m->kv_heads, nqkv = qd + 2 * kvd;
  int big = nqkv > 2 * inter ? nqkv : 2 * inter;
  if (m->vocab > big) big = m->vocab;
  if (h > big) big = h;
  int widest = qd > inter ? qd : inter;
  if (h > widest) widest = h;
  float* x = malloc(sizeof(float) * h);
  float* xn = malloc(sizeof(float) * widest);
  float* buf = malloc(sizeof(float) * big);
  float* att = malloc(sizeof(float) * qd);
  float* mid = malloc(sizeof(float) * inter);
  int8_t* xq = malloc((size_t)widest);
  if (!x || !xn || !buf || !att || !mid || !xq) return -1;
  const float scale = 1.0f / sqrtf(128.0f);
  memcpy(x, x0, sizeof(float) * h);
  for (int step = 0; step < n_steps; ++step) {
    const int pos = pos0 + step;
    if (step > 0) {
      const int tok = forced ? forced[step - 1] : out_ids[step - 1];
      for (int i = 0; i < h; ++i) x[i] = bf16f(m->embed[(size_t)tok * h + i]);
    }
    float c[64], s[64];
    for (int d = 0; d < 64; ++d) {
      const float ang = (float)pos * m->inv_freq[d];
      c[d] = cosf(ang);
      s[d] = sinf(ang);
    }
    for (int l = 0; l < m->layers; ++l) {
      rms_norm(x, m->n1[l], xn, h, m->eps);
      if (m->int8) {
        const float xs = quantize(xn, h, xq);
        mv_int8(m->q_qkv[l], m->s_qkv[l], xq, xs, nqkv, h, buf, NULL);
      } else {
        mv_bf16(m->b_qkv[l], xn, nqkv, h, buf, NULL);
      }
      float* q = buf;
      float* k = buf + qd;
      float* v = buf + qd + kvd;
      for (int hh = 0; hh < m->q_heads; ++hh) head_norm_rope(q + hh * 128, m->qn[l], m->eps, c, s);
      for (int hh = 0; hh < m->kv_heads; ++hh) head_norm_rope(k + hh * 128, m->kn[l], m->eps, c, s);
      for (int hh = 0; hh < m->kv_heads; ++hh) {
        const size_t off = (((size_t)l * m->kv_heads + hh) * m->max_seq + pos) * 128;
        memcpy(m->k_cache + off, k + hh * 128, 512);
        memcpy(m->v_cache + off, v + hh * 128, 512);
      }
#pragma omp parallel for schedule(static)
      for (int hh = 0; hh < m->q_heads; ++hh) {
        const int kvh = hh / G;
        const float* qr = q + hh * 128;
        const float* kb = m->k_cache + ((size_t)l * m->kv_heads + kvh) * m->max_seq * 128;
        const float* vb = m->v_cache + ((size_t)l * m->kv_heads + kvh) * m->max_seq * 128;
        float* o = att + hh * 128;
        float mx = -1e30f, se = 0.f;
        for (int d = 0; d < 128; ++d) o[d] = 0.f;
        for (int j = 0; j <= pos; ++j) {
          float dot = 0.f;
          for (int d = 0; d < 128; ++d) dot += qr[d] * kb[(size_t)j * 128 + d];
          const float sc = dot * scale;
          if (sc > mx) {
            const float corr = expf(mx - sc);
            se = se * corr + 1.0f;
            for (int d = 0; d < 128; ++d) o[d] = o[d] * corr + vb[(size_t)j * 128 + d];
            mx = sc;
          } else {
            const float wt = expf(sc - mx);
            se += wt;
            for (int d = 0; d < 128; ++d) o[d] += wt * vb[(size_t)j * 128 + d];
          }
        }
        if (se > 0.f) {
          const float inv = 1.0f / se;
          for (int d = 0; d < 128; ++d) o[d] *= inv;
        }
      }
      if (m->int8) {
        const float xs = quantize(att, qd, xq);
        mv_int8(m->q_o[l], m->s_o[l], xq, xs, h, qd, buf, x);
      } else {
        mv_bf16(m->b_o[l], att, h, qd, buf, x);
      }
      memcpy(x, buf, sizeof(float) * h);
      rms_norm(x, m->n2[l], xn, h, m->eps);
      if (m->int8) {
        const float xs = quantize(xn, h, xq);
        mv_int8(m->q_gu[l], m->s_gu[l], xq, xs, 2 * inter, h, buf, NULL);
      } else {
        mv_bf16(m->b_gu[l], xn, 2 * inter, h, buf, NULL);
      }
      for (int j = 0; j < inter; ++j) {
        const float g = buf[2 * j], u = buf[2 * j + 1];
        mid[j] = g / (1.0f + expf(-g)) * u;
      }
      if (m->int8) {
        const float xs = quantize(mid, inter, xq);
        mv_int8(m->q_down[l], m->s_down[l], xq, xs, h, inter, buf, x);
      } else {
        mv_bf16(m->b_down[l], mid, h, inter, buf, x);
      }
      memcpy(x, buf, sizeof(float) * h);
    }
    rms_norm(x, m->final_norm, xn, h, m->eps);
    if (m->int8) {
      const float xs = quantize(xn, h, xq);
      mv_int8(m->lm_q, m->lm_s, xq, xs, m->vocab, h, buf, NULL);
    } else {
      mv_bf16(m->lm_b, xn, m->vocab, h, buf, NULL);
    }
    int best = 0;
    for (int i = 1; i < m->vocab; ++i)
      if (buf[i] > buf[best]) best = i;
    out_ids[step] = best;
    if (logits && step == n_steps - 1) memcpy(logits, buf, sizeof(float) * m->vocab);
  }
  free(x);
  free(xn);
  free(buf);
  free(att);
  free(mid);
  free(xq);
  return 0;
}

/* Threads the matvecs use (the reference's -t; <= 0 keeps the OpenMP default). */
void qasr_ref_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
