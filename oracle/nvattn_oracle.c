/*
 * nvattn_oracle.c -- CPU oracle for the paged-attention hot path.
 * TEST INFRASTRUCTURE ONLY (see nvattn_oracle.h).  Parity against the
 * reference is unpinned: the reference has no tests and ggml is not vendored.
 * Compile with -ffp-contract=off.
 */
#define _GNU_SOURCE
#include "nvattn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------------ */
/* conversions                                                               */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ggml_compute_fp32_to_bf16 (ggml-impl.h): round to nearest even on the
 * upper 16 bits; NaN keeps its sign and top payload bits and is forced
 * quiet.  Subnormals are rounded like any other value. */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = f32_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 64u);
  return (uint16_t)((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

float orc_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* IEEE binary16, round to nearest even, gradual underflow (what the F16C
 * conversion ggml uses on x86 computes). */
uint16_t orc_f32_to_f16(float f) {
  uint32_t u = f32_bits(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
  if (a >= 0x47800000u) return (uint16_t)(sign | 0x7c00u); /* >= 2^16, inf */
  if (a < 0x38800000u) {
    /* below 2^-14: the f16 value is an integer multiple of 2^-24. */
    float m = bits_f32(a) * 16777216.0f; /* exact scaling by 2^24 */
    return (uint16_t)(sign | (uint16_t)rintf(m));
  }
  uint32_t h = (a >> 13) - ((127u - 15u) << 10);
  uint32_t rem = a & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
  uint32_t m = (uint32_t)h & 0x3ffu;
  if (e == 0) {
    float v = (float)m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
    return sign ? -v : v;
  }
  if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
  return bits_f32(sign | ((e + 127u - 15u) << 23) | (m << 13));
}

void orc_f32_to_bf16_row(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_f32_to_bf16(x[i]);
}

void orc_bf16_to_f32_row(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_bf16_to_f32(x[i]);
}

/* ---- f16 rounding of float vectors (values kept as f16-exact floats) ----
 * The x86 path uses the F16C instructions, which round exactly like
 * orc_f32_to_f16 (round to nearest even, gradual underflow, quiet NaN). */

static inline float f16r(float x) { return orc_f16_to_f32(orc_f32_to_f16(x)); }

static void round_f16_sw(float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = f16r(x[i]);
}

/* y[i] = f16(fma(x[i], v, y[i]))  -- ggml_vec_mad_f16 */
static void mad_f16_sw(float* y, const float* x, float v, int n) {
  for (int i = 0; i < n; ++i) y[i] = f16r(fmaf(x[i], v, y[i]));
}

/* y[i] = f16(y[i] * v)  -- ggml_vec_scale_f16 */
static void scale_f16_sw(float* y, float v, int n) {
  for (int i = 0; i < n; ++i) y[i] = f16r(y[i] * v);
}

#if defined(__x86_64__)
__attribute__((target("avx,f16c"))) static void round_f16_hw(float* x, int64_t n) {
  int64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    __m256 v = _mm256_loadu_ps(x + i);
    _mm256_storeu_ps(x + i, _mm256_cvtph_ps(_mm256_cvtps_ph(v, _MM_FROUND_TO_NEAREST_INT)));
  }
  for (; i < n; ++i) x[i] = f16r(x[i]);
}

__attribute__((target("avx,f16c,fma"))) static void mad_f16_hw(float* y, const float* x,
                                                                 float v, int n) {
  const __m256 vv = _mm256_set1_ps(v);
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    __m256 r = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), vv, _mm256_loadu_ps(y + i));
    _mm256_storeu_ps(y + i, _mm256_cvtph_ps(_mm256_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT)));
  }
  for (; i < n; ++i) y[i] = f16r(fmaf(x[i], v, y[i]));
}

__attribute__((target("avx,f16c"))) static void scale_f16_hw(float* y, float v, int n) {
  const __m256 vv = _mm256_set1_ps(v);
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    __m256 r = _mm256_mul_ps(_mm256_loadu_ps(y + i), vv);
    _mm256_storeu_ps(y + i, _mm256_cvtph_ps(_mm256_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT)));
  }
  for (; i < n; ++i) y[i] = f16r(y[i] * v);
}

static int have_f16c(void) {
  static int cached = -1;
  if (cached < 0) {
    __builtin_cpu_init();
    cached = __builtin_cpu_supports("avx") && __builtin_cpu_supports("f16c") &&
             __builtin_cpu_supports("fma");
  }
  return cached;
}
#define ROUND_F16(x, n) (have_f16c() ? round_f16_hw(x, n) : round_f16_sw(x, n))
#define MAD_F16(y, x, v, n) (have_f16c() ? mad_f16_hw(y, x, v, n) : mad_f16_sw(y, x, v, n))
#define SCALE_F16(y, v, n) (have_f16c() ? scale_f16_hw(y, v, n) : scale_f16_sw(y, v, n))
#else
#define ROUND_F16(x, n) round_f16_sw(x, n)
#define MAD_F16(y, x, v, n) mad_f16_sw(y, x, v, n)
#define SCALE_F16(y, v, n) scale_f16_sw(y, v, n)
#endif

int orc_f16_hw_path(void) {
#if defined(__x86_64__)
  return have_f16c();
#else
  return 0;
#endif
}

void orc_round_f16_row(float* x, int64_t n, int use_hw) {
#if defined(__x86_64__)
  if (use_hw && have_f16c()) {
    round_f16_hw(x, n);
    return;
  }
#endif
  (void)use_hw;
  round_f16_sw(x, n);
}

/* ------------------------------------------------------------------------ */
/* RoPE (ggml rope cache, NEOX pairing)                                      */
/* ------------------------------------------------------------------------ */

static float corr_dim(int n_dims, int n_ctx_orig, float n_rot, float base) {
  return n_dims * logf(n_ctx_orig / (n_rot * 2 * (float)M_PI)) / (2 * logf(base));
}

void orc_rope_corr_dims(int n_dims, int n_ctx_orig, float freq_base,
                        float beta_fast, float beta_slow, float dims[2]) {
  float start = floorf(corr_dim(n_dims, n_ctx_orig, beta_fast, freq_base));
  float end = ceilf(corr_dim(n_dims, n_ctx_orig, beta_slow, freq_base));
  dims[0] = start > 0 ? start : 0;
  dims[1] = end < (float)(n_dims - 1) ? end : (float)(n_dims - 1);
}

static float yarn_ramp(float low, float high, int i0) {
  float den = high - low;
  if (den < 0.001f) den = 0.001f;
  float y = (i0 / 2 - low) / den;
  if (y < 0) y = 0;
  if (y > 1) y = 1;
  return 1 - y;
}

void orc_rope_cache(int pos, const orc_params* p, float* cache) {
  const int n_dims = p->head_dim;
  float corr[2];
  orc_rope_corr_dims(n_dims, p->rope_n_ctx_orig, p->rope_theta,
                     p->rope_beta_fast, p->rope_beta_slow, corr);
  const float theta_scale = powf(p->rope_theta, -2.0f / n_dims);
  float theta_extrap = (float)pos;
  for (int i0 = 0; i0 < n_dims; i0 += 2) {
    float theta_interp = p->rope_freq_scale * theta_extrap;
    float theta = theta_interp;
    float mscale = p->rope_attn_factor;
    if (p->rope_ext_factor != 0.0f) {
      float ramp_mix = yarn_ramp(corr[0], corr[1], i0) * p->rope_ext_factor;
      theta = theta_interp * (1 - ramp_mix) + theta_extrap * ramp_mix;
      mscale *= 1.0f + 0.1f * logf(1.0f / p->rope_freq_scale);
    }
    cache[i0 + 0] = cosf(theta) * mscale;
    cache[i0 + 1] = sinf(theta) * mscale;
    theta_extrap *= theta_scale;
  }
}

void orc_rope_table(int n_pos, const orc_params* p, float* table) {
  for (int pos = 0; pos < n_pos; ++pos)
    orc_rope_cache(pos, p, table + (int64_t)pos * p->head_dim);
}

/* ggml_compute_forward_rms_norm_f32: double accumulation of float squares,
 * in index order; mean rounded to float; scale = 1/sqrtf(mean+eps);
 * y = x*scale, then ggml_mul by the (bf16->f32) weight. */
static void rms_norm_mul(const float* x, const uint16_t* w, int n, float eps,
                         float* y) {
  double sum = 0.0;
  for (int i = 0; i < n; ++i) {
    float sq = x[i] * x[i];
    sum += (double)sq;
  }
  const float mean = (float)(sum / n);
  const float scale = 1.0f / sqrtf(mean + eps);
  for (int i = 0; i < n; ++i) {
    float t = x[i] * scale;
    y[i] = t * orc_bf16_to_f32(w[i]);
  }
}

/* NEOX rotation: pairs (i, i + n/2) rotated by theta_i. */
static void rope_neox(const float* x, const float* cache, int n, float* y) {
  const int half = n / 2;
  for (int i0 = 0; i0 < n; i0 += 2) {
    const int ic = i0 / 2;
    const float c = cache[i0], s = cache[i0 + 1];
    const float x0 = x[ic], x1 = x[ic + half];
    const float a = x0 * c, b = x1 * s;
    const float e = x0 * s, f = x1 * c;
    y[ic] = a - b;
    y[ic + half] = e + f;
  }
}

/* ------------------------------------------------------------------------ */
/* tiny parallel-for                                                         */
/* ------------------------------------------------------------------------ */

typedef void (*work_fn)(void* ctx, int64_t item);
typedef struct {
  work_fn fn;
  void* ctx;
  int64_t n;
  atomic_llong next;
} pf_state;

static void* pf_worker(void* arg) {
  pf_state* st = (pf_state*)arg;
  for (;;) {
    long long i = atomic_fetch_add(&st->next, 1);
    if (i >= st->n) break;
    st->fn(st->ctx, (int64_t)i);
  }
  return NULL;
}

static void parallel_for(int n_threads, int64_t n, work_fn fn, void* ctx) {
  if (n_threads <= 0) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  if ((int64_t)n_threads > n) n_threads = (int)(n > 0 ? n : 1);
  pf_state st;
  st.fn = fn;
  st.ctx = ctx;
  st.n = n;
  atomic_init(&st.next, 0);
  if (n_threads == 1) {
    pf_worker(&st);
    return;
  }
  pthread_t th[256];
  int started = 0;
  for (int t = 1; t < n_threads; ++t)
    if (pthread_create(&th[started], NULL, pf_worker, &st) == 0) started++;
  pf_worker(&st);
  for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* fused q/k norm + rope + store                                             */
/* ------------------------------------------------------------------------ */

static inline int64_t cache_row(const orc_params* p, int layer, int64_t slot,
                                int kvh) {
  return (((int64_t)layer * p->n_slots + slot) * p->n_kv_heads + kvh) *
         (int64_t)p->head_dim;
}

void orc_qk_norm_rope_store(const orc_params* p, int layer, int n_tokens,
                            const float* q, const float* k, const float* v,
                            const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                            const int32_t* positions, const int32_t* slots,
                            float* q_out, float* k_out, uint16_t* k_cache,
                            uint16_t* v_cache) {
  const int d = p->head_dim, Hq = p->n_q_heads, Hkv = p->n_kv_heads;
  float* cache = (float*)malloc(sizeof(float) * d);
  float* tmp = (float*)malloc(sizeof(float) * d);
  float* kr = (float*)malloc(sizeof(float) * d);
  for (int t = 0; t < n_tokens; ++t) {
    orc_rope_cache(positions[t], p, cache);
    for (int h = 0; h < Hq; ++h) {
      const float* x = q + ((int64_t)t * Hq + h) * d;
      rms_norm_mul(x, q_norm_w, d, p->rms_eps, tmp);
      rope_neox(tmp, cache, d, q_out + ((int64_t)t * Hq + h) * d);
    }
    for (int h = 0; h < Hkv; ++h) {
      const float* x = k + ((int64_t)t * Hkv + h) * d;
      rms_norm_mul(x, k_norm_w, d, p->rms_eps, tmp);
      rope_neox(tmp, cache, d, kr);
      if (k_out) memcpy(k_out + ((int64_t)t * Hkv + h) * d, kr, sizeof(float) * d);
      if (slots[t] >= 0) {
        const int64_t row = cache_row(p, layer, slots[t], h);
        orc_f32_to_bf16_row(kr, k_cache + row, d);
        orc_f32_to_bf16_row(v + ((int64_t)t * Hkv + h) * d, v_cache + row, d);
      }
    }
  }
  free(cache);
  free(tmp);
  free(kr);
}

/* ------------------------------------------------------------------------ */
/* attention                                                                 */
/* ------------------------------------------------------------------------ */

/* The keys of one (sequence, kv head), gathered once and shared by the GQA
 * group's query heads: K[j][d], V[j][d] as floats holding exactly the
 * values attention consumes -- bf16 cache rows or f32 rows, and in GGML mode
 * rounded to f16 (the reference's ggml_cast F32->F16, qwen3.cpp:388-393). */
typedef struct {
  float* k;
  float* v;
  int64_t n;
} key_set;

static void key_set_free(key_set* ks) {
  free(ks->k);
  free(ks->v);
}

/* Keys [0, n_keys) of block-table row `bt_row`; keys j >= new_from come from
 * the f32 rows new_k/new_v (stride between consecutive keys: new_stride
 * floats) when new_k is non-NULL. */
static int gather_keys(const orc_params* p, int mode, int layer,
                       const uint16_t* kc, const uint16_t* vc,
                       const int32_t* bt_row, int64_t n_keys, int kvh,
                       const float* new_k, const float* new_v, int64_t new_from,
                       int64_t new_stride, key_set* ks) {
  const int d = p->head_dim;
  ks->n = n_keys;
  ks->k = (float*)malloc(sizeof(float) * (size_t)(n_keys > 0 ? n_keys : 1) * d);
  ks->v = (float*)malloc(sizeof(float) * (size_t)(n_keys > 0 ? n_keys : 1) * d);
  if (!ks->k || !ks->v) return -1;
  for (int64_t t = 0; t < n_keys; ++t) {
    float* kd = ks->k + t * d;
    float* vd = ks->v + t * d;
    if (new_k && t >= new_from) {
      memcpy(kd, new_k + (t - new_from) * new_stride, sizeof(float) * d);
      memcpy(vd, new_v + (t - new_from) * new_stride, sizeof(float) * d);
    } else {
      const int64_t blk = bt_row[t / p->block_size];
      const int64_t slot = blk * p->block_size + t % p->block_size;
      const int64_t row = cache_row(p, layer, slot, kvh);
      orc_bf16_to_f32_row(kc + row, kd, d);
      orc_bf16_to_f32_row(vc + row, vd, d);
    }
  }
  if (mode == ORC_MODE_GGML) {
    ROUND_F16(ks->k, n_keys * d);
    ROUND_F16(ks->v, n_keys * d);
  }
  return 0;
}

/* One query row against keys idx[0..n) (or 0..n when idx is NULL), in order.
 * GGML: ggml_compute_forward_flash_attn_ext_f16_one_chunk with F16 K/V, mask
 * value 0 on visited keys: Q rounded to f16; score = double sum of float
 * products (ggml_vec_dot_f16, scalar path) rounded to float, times scale;
 * online softmax in float with expf; f16 V accumulator (ggml_vec_scale_f16 /
 * ggml_vec_mad_f16); out = VKQ / S.
 * TRUTH: fp64 online softmax and accumulation. */
static void attend_row(int mode, int d, float scale, const float* q,
                       const key_set* ks, const int64_t* idx, int64_t n,
                       float* out) {
  if (mode == ORC_MODE_GGML) {
    float qf[512], vkq[512];
    memcpy(qf, q, sizeof(float) * d);
    ROUND_F16(qf, d);
    memset(vkq, 0, sizeof(float) * d);
    float M = -INFINITY, S = 0.0f;
    for (int64_t jj = 0; jj < n; ++jj) {
      const int64_t j = idx ? idx[jj] : jj;
      const float* kj = ks->k + j * d;
      double sumd = 0.0;
      for (int i = 0; i < d; ++i) {
        const float prod = qf[i] * kj[i];
        sumd += (double)prod;
      }
      float s = (float)sumd;
      s = s * scale;
      s = s + 0.0f; /* additive mask value 0 */
      const float Mold = M;
      float ms = 1.0f, vs = 1.0f;
      if (s > M) {
        M = s;
        ms = expf(Mold - M);
        SCALE_F16(vkq, ms, d);
      } else {
        vs = expf(s - M);
      }
      MAD_F16(vkq, ks->v + j * d, vs, d);
      const float t = S * ms;
      S = t + vs;
    }
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
    for (int i = 0; i < d; ++i) out[i] = vkq[i] * S_inv;
  } else {
    double qd[512], acc[512];
    for (int i = 0; i < d; ++i) {
      qd[i] = (double)q[i];
      acc[i] = 0.0;
    }
    double m = -INFINITY, l = 0.0;
    for (int64_t jj = 0; jj < n; ++jj) {
      const int64_t j = idx ? idx[jj] : jj;
      const float* kj = ks->k + j * d;
      const float* vj = ks->v + j * d;
      double s = 0.0;
      for (int i = 0; i < d; ++i) s += qd[i] * (double)kj[i];
      s *= (double)scale;
      const double m_new = s > m ? s : m;
      const double alpha = exp(m - m_new);
      const double pw = exp(s - m_new);
      l = l * alpha + pw;
      for (int i = 0; i < d; ++i) acc[i] = acc[i] * alpha + pw * (double)vj[i];
      m = m_new;
    }
    for (int i = 0; i < d; ++i) out[i] = l > 0.0 ? (float)(acc[i] / l) : 0.0f;
  }
}

typedef struct {
  const orc_params* p;
  int mode, layer, max_blocks, n_seqs;
  const float* q;
  const uint16_t *kc, *vc;
  const int32_t *bt, *cl, *cu_q, *q_start;
  const float *nk, *nv;
  float* out;
  int64_t chunk_rows;        /* prefill: query rows per work item */
  const int64_t* item_base;  /* prefill: first item index of each sequence */
} attn_ctx;

/* ---- paged decode: one item = (sequence, kv head) ---- */
static void decode_item(void* vctx, int64_t item) {
  attn_ctx* c = (attn_ctx*)vctx;
  const orc_params* p = c->p;
  const int Hq = p->n_q_heads, Hkv = p->n_kv_heads, d = p->head_dim;
  const int G = Hq / Hkv;
  const int s = (int)(item / Hkv), kvh = (int)(item % Hkv);
  const int64_t L = c->cl[s];
  key_set ks;
  const int use_new = c->nk != NULL;
  if (gather_keys(p, c->mode, c->layer, c->kc, c->vc, c->bt + (int64_t)s * c->max_blocks, L,
                  kvh, use_new ? c->nk + ((int64_t)s * Hkv + kvh) * d : NULL,
                  use_new ? c->nv + ((int64_t)s * Hkv + kvh) * d : NULL, L - 1, 0, &ks) == 0) {
    for (int g = 0; g < G; ++g) {
      const int64_t row = (int64_t)s * Hq + kvh * G + g;
      attend_row(c->mode, d, p->scale, c->q + row * d, &ks, NULL, L, c->out + row * d);
    }
  }
  key_set_free(&ks);
}

void orc_paged_decode(const orc_params* p, int mode, int layer, int n_seqs,
                      const float* q, const uint16_t* k_cache,
                      const uint16_t* v_cache, const int32_t* block_tables,
                      int max_blocks, const int32_t* context_lens,
                      const float* new_k, const float* new_v, float* out) {
  attn_ctx c;
  memset(&c, 0, sizeof(c));
  c.p = p;
  c.mode = mode;
  c.layer = layer;
  c.max_blocks = max_blocks;
  c.n_seqs = n_seqs;
  c.q = q;
  c.kc = k_cache;
  c.vc = v_cache;
  c.bt = block_tables;
  c.cl = context_lens;
  c.nk = new_k;
  c.nv = new_v;
  c.out = out;
  parallel_for(p->n_threads, (int64_t)n_seqs * p->n_kv_heads, decode_item, &c);
}

/* ---- paged prefill: one item = (sequence, kv head, chunk of query rows) ---- */
static void prefill_item(void* vctx, int64_t item) {
  attn_ctx* c = (attn_ctx*)vctx;
  const orc_params* p = c->p;
  const int Hq = p->n_q_heads, Hkv = p->n_kv_heads, d = p->head_dim;
  const int G = Hq / Hkv;
  int s = 0;
  while (s + 1 < c->n_seqs && c->item_base[s + 1] <= item) ++s;
  const int64_t local = item - c->item_base[s];
  const int kvh = (int)(local % Hkv);
  const int64_t chunk = local / Hkv;
  const int64_t r0 = c->cu_q[s] + chunk * c->chunk_rows;
  int64_t r1 = r0 + c->chunk_rows;
  if (r1 > c->cu_q[s + 1]) r1 = c->cu_q[s + 1];
  if (r0 >= r1) return;
  const int64_t P_last = c->q_start[s] + (r1 - 1 - c->cu_q[s]);
  const int use_new = c->nk != NULL;
  key_set ks;
  if (gather_keys(p, c->mode, c->layer, c->kc, c->vc, c->bt + (int64_t)s * c->max_blocks,
                  P_last + 1, kvh,
                  use_new ? c->nk + ((int64_t)c->cu_q[s] * Hkv + kvh) * d : NULL,
                  use_new ? c->nv + ((int64_t)c->cu_q[s] * Hkv + kvh) * d : NULL,
                  c->q_start[s], (int64_t)Hkv * d, &ks) == 0) {
    for (int64_t r = r0; r < r1; ++r) {
      const int64_t P = c->q_start[s] + (r - c->cu_q[s]);
      for (int g = 0; g < G; ++g) {
        const int64_t row = r * Hq + kvh * G + g;
        attend_row(c->mode, d, p->scale, c->q + row * d, &ks, NULL, P + 1, c->out + row * d);
      }
    }
  }
  key_set_free(&ks);
}

void orc_paged_prefill(const orc_params* p, int mode, int layer, int n_seqs,
                       const float* q, const int32_t* cu_q,
                       const int32_t* q_start, const int32_t* context_lens,
                       const int32_t* block_tables, int max_blocks,
                       const uint16_t* k_cache, const uint16_t* v_cache,
                       const float* new_k, const float* new_v, float* out) {
  attn_ctx c;
  memset(&c, 0, sizeof(c));
  c.p = p;
  c.mode = mode;
  c.layer = layer;
  c.max_blocks = max_blocks;
  c.n_seqs = n_seqs;
  c.q = q;
  c.kc = k_cache;
  c.vc = v_cache;
  c.bt = block_tables;
  c.cl = context_lens;
  c.cu_q = cu_q;
  c.q_start = q_start;
  c.nk = new_k;
  c.nv = new_v;
  c.out = out;
  c.chunk_rows = 64;
  int64_t* base = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n_seqs + 1));
  base[0] = 0;
  for (int s = 0; s < n_seqs; ++s) {
    const int64_t rows = cu_q[s + 1] - cu_q[s];
    base[s + 1] = base[s] + ((rows + c.chunk_rows - 1) / c.chunk_rows) * p->n_kv_heads;
  }
  c.item_base = base;
  parallel_for(p->n_threads, base[n_seqs], prefill_item, &c);
  free(base);
}

/* ------------------------------------------------------------------------ */
/* the reference's concat-all decode (GGML mode)                             */
/* ------------------------------------------------------------------------ */

void orc_concat_decode_ggml(const orc_params* p, int layer, int n_seqs,
                            const float* q, const uint16_t* k_cache,
                            const uint16_t* v_cache,
                            const int32_t* block_tables, int max_blocks,
                            const int32_t* context_lens, const float* new_k,
                            const float* new_v, float* out) {
  const int Hq = p->n_q_heads, Hkv = p->n_kv_heads, d = p->head_dim;
  const int64_t row_elems = (int64_t)Hkv * d;
  int64_t total_hist = 0;
  for (int s = 0; s < n_seqs; ++s) total_hist += context_lens[s] - 1;
  const int64_t total_kv = total_hist + n_seqs;
  const int64_t total_kv_pad = (total_kv + 255) / 256 * 256;

  /* LoadHistoryKV: gather bf16 rows, convert bf16->f32 (model_runner.cpp
   * :327-354); graph concat with the new f32 rows and zero pad
   * (qwen3.cpp:653-658); ggml_cast to F16 of the whole buffer (:388-393). */
  float* kf = (float*)calloc((size_t)(total_kv_pad * row_elems), sizeof(float));
  float* vf = (float*)calloc((size_t)(total_kv_pad * row_elems), sizeof(float));
  int64_t off = 0;
  for (int s = 0; s < n_seqs; ++s) {
    const int ctx = context_lens[s] - 1;
    for (int t = 0; t < ctx; ++t) {
      const int64_t blk = block_tables[(int64_t)s * max_blocks + t / p->block_size];
      const int64_t slot = blk * p->block_size + t % p->block_size;
      const int64_t row = cache_row(p, layer, slot, 0);
      orc_bf16_to_f32_row(k_cache + row, kf + (off + t) * row_elems, row_elems);
      orc_bf16_to_f32_row(v_cache + row, vf + (off + t) * row_elems, row_elems);
    }
    off += ctx;
  }
  memcpy(kf + total_hist * row_elems, new_k, sizeof(float) * n_seqs * row_elems);
  memcpy(vf + total_hist * row_elems, new_v, sizeof(float) * n_seqs * row_elems);
  ROUND_F16(kf, total_kv_pad * row_elems);
  ROUND_F16(vf, total_kv_pad * row_elems);

  /* Per kv head, a key_set view with stride d (row j of head h lives at
   * (j*Hkv + h)*d); FillVarlenMask (model_runner.cpp:219-243) leaves row s
   * its own history [hist_off_s, hist_off_s + ctx_s) and column total_hist+s,
   * visited in increasing column order. */
  int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)(total_kv_pad + 1));
  float* kh = (float*)malloc(sizeof(float) * (size_t)total_kv_pad * d);
  float* vh = (float*)malloc(sizeof(float) * (size_t)total_kv_pad * d);
  for (int kvh = 0; kvh < Hkv; ++kvh) {
    for (int64_t j = 0; j < total_kv_pad; ++j) {
      memcpy(kh + j * d, kf + j * row_elems + (int64_t)kvh * d, sizeof(float) * d);
      memcpy(vh + j * d, vf + j * row_elems + (int64_t)kvh * d, sizeof(float) * d);
    }
    key_set ks = {kh, vh, total_kv_pad};
    int64_t hoff = 0;
    for (int s = 0; s < n_seqs; ++s) {
      int64_t n = 0;
      for (int64_t j = 0; j < total_kv_pad; ++j) {
        const int visible = (j >= hoff && j < hoff + context_lens[s] - 1) || j == total_hist + s;
        if (visible) idx[n++] = j; /* masked columns (-inf) are skipped */
      }
      for (int h = kvh * (Hq / Hkv); h < (kvh + 1) * (Hq / Hkv); ++h)
        attend_row(ORC_MODE_GGML, d, p->scale, q + ((int64_t)s * Hq + h) * d, &ks, idx, n,
                   out + ((int64_t)s * Hq + h) * d);
      hoff += context_lens[s] - 1;
    }
  }
  free(idx);
  free(kh);
  free(vh);
  free(kf);
  free(vf);
}

/* ------------------------------------------------------------------------ */
/* the reference's prefill attention (GGML mode)                             */
/* ------------------------------------------------------------------------ */

typedef struct {
  const orc_params* p;
  int n_seqs;
  int64_t n_tokens, n_kv_pad, rows_per_item;
  const int32_t* cu_q;
  const float *q, *kh, *vh; /* kh/vh: [Hkv][n_kv_pad][d], f16-rounded */
  float* out;
} concat_prefill_ctx;

/* one item = (kv head, block of query rows); each row scans its whole mask
 * row, as the masked attention over the padded buffer does */
static void concat_prefill_item(void* vctx, int64_t item) {
  concat_prefill_ctx* c = (concat_prefill_ctx*)vctx;
  const orc_params* p = c->p;
  const int Hq = p->n_q_heads, Hkv = p->n_kv_heads, d = p->head_dim;
  const int G = Hq / Hkv;
  const int kvh = (int)(item % Hkv);
  const int64_t r0 = (item / Hkv) * c->rows_per_item;
  int64_t r1 = r0 + c->rows_per_item;
  if (r1 > c->n_tokens) r1 = c->n_tokens;
  key_set ks = {(float*)c->kh + (int64_t)kvh * c->n_kv_pad * d,
                (float*)c->vh + (int64_t)kvh * c->n_kv_pad * d, c->n_kv_pad};
  int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)(c->n_kv_pad + 1));
  int s = 0;
  for (int64_t r = r0; r < r1; ++r) {
    while (s + 1 < c->n_seqs && c->cu_q[s + 1] <= r) ++s;
    /* FillCausalMask: column j is 0 (attend) for cu_q[s] <= j <= r, -inf
     * elsewhere, padded columns included; -inf columns are skipped */
    int64_t n = 0;
    for (int64_t j = 0; j < c->n_kv_pad; ++j)
      if (j >= c->cu_q[s] && j <= r) idx[n++] = j;
    for (int g = 0; g < G; ++g) {
      const int64_t row = r * Hq + (int64_t)kvh * G + g;
      attend_row(ORC_MODE_GGML, d, p->scale, c->q + row * d, &ks, idx, n, c->out + row * d);
    }
  }
  free(idx);
}

void orc_concat_prefill_ggml(const orc_params* p, int n_seqs, const int32_t* cu_q,
                             const float* q, const float* new_k, const float* new_v,
                             float* out) {
  const int Hkv = p->n_kv_heads, d = p->head_dim;
  const int64_t T = cu_q[n_seqs];
  const int64_t T_pad = (T + 255) / 256 * 256; /* qwen3.cpp:461 */
  /* ggml_pad with zeros (qwen3.cpp:524-527), then ggml_cast to F16
   * (:388-393); one contiguous [n_kv_pad][d] plane per kv head */
  float* kh = (float*)calloc((size_t)(Hkv * T_pad * d), sizeof(float));
  float* vh = (float*)calloc((size_t)(Hkv * T_pad * d), sizeof(float));
  for (int h = 0; h < Hkv; ++h)
    for (int64_t j = 0; j < T; ++j) {
      memcpy(kh + ((int64_t)h * T_pad + j) * d, new_k + (j * Hkv + h) * d, sizeof(float) * d);
      memcpy(vh + ((int64_t)h * T_pad + j) * d, new_v + (j * Hkv + h) * d, sizeof(float) * d);
    }
  ROUND_F16(kh, (int64_t)Hkv * T_pad * d);
  ROUND_F16(vh, (int64_t)Hkv * T_pad * d);
  concat_prefill_ctx c = {p, n_seqs, T, T_pad, 16, cu_q, q, kh, vh, out};
  parallel_for(p->n_threads, ((T + c.rows_per_item - 1) / c.rows_per_item) * Hkv,
               concat_prefill_item, &c);
  free(kh);
  free(vh);
}

/* ------------------------------------------------------------------------ */
/* token sampling (model_runner.cpp:417-489)                                */
/* ------------------------------------------------------------------------ */

static void penalize_row(int n_vocab, float* row, float penalty, const int32_t* hist,
                         int64_t n_hist) {
  for (int64_t j = 0; j < n_hist; ++j) {
    const int32_t tok = hist[j];
    if (tok < 0 || tok >= n_vocab) continue; /* size_t id >= n_vocab is skipped */
    float* v = &row[tok];
    *v = *v < 0.0f ? *v * penalty : *v / penalty;
  }
}

void orc_penalize_rows(int n_seqs, int n_vocab, const float* logits, int64_t row_stride,
                       const float* penalties, const int32_t* history,
                       const int64_t* history_offsets, float* out) {
  for (int s = 0; s < n_seqs; ++s) {
    float* row = out + (int64_t)s * n_vocab;
    memcpy(row, logits + (int64_t)s * row_stride, sizeof(float) * (size_t)n_vocab);
    if (penalties[s] > 1.0f && history != NULL && history_offsets != NULL)
      penalize_row(n_vocab, row, penalties[s], history + history_offsets[s],
                   history_offsets[s + 1] - history_offsets[s]);
  }
}

void orc_sample(int n_seqs, int n_vocab, const float* logits, int64_t row_stride,
                const float* temperatures, const float* penalties, const int32_t* history,
                const int64_t* history_offsets, const float* uniforms, int32_t* tokens) {
  float* row = (float*)malloc(sizeof(float) * (size_t)n_vocab);
  float* probs = (float*)malloc(sizeof(float) * (size_t)n_vocab);
  for (int s = 0; s < n_seqs; ++s) {
    /* one row: offsets shifted so that [0], [1] bound sequence s's ids */
    orc_penalize_rows(1, n_vocab, logits + (int64_t)s * row_stride, row_stride, penalties + s,
                      history, history_offsets ? history_offsets + s : NULL, row);
    const float temp = temperatures[s];
    if (temp < 1e-6f) {
      int best = 0;
      float best_val = row[0];
      for (int i = 1; i < n_vocab; ++i)
        if (row[i] > best_val) {
          best_val = row[i];
          best = i;
        }
      tokens[s] = best;
      continue;
    }
    float max_logit = row[0];
    for (int i = 1; i < n_vocab; ++i)
      if (row[i] > max_logit) max_logit = row[i];
    float sum = 0.0f;
    for (int i = 0; i < n_vocab; ++i) {
      probs[i] = expf((row[i] - max_logit) / temp);
      sum += probs[i];
    }
    const float r = uniforms[s] * (sum - 0.0f) + 0.0f;
    float cumulative = 0.0f;
    int idx = n_vocab - 1;
    for (int i = 0; i < n_vocab; ++i) {
      cumulative += probs[i];
      if (cumulative >= r) {
        idx = i;
        break;
      }
    }
    tokens[s] = idx;
  }
  free(row);
  free(probs);
}

float orc_canonical_float(uint32_t x) {
  const float u = (float)x / 4294967296.0f;
  return u >= 1.0f ? nextafterf(1.0f, 0.0f) : u;
}
