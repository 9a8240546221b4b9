/*
 * rxla_oracle.c — CPU restatement of rxla's W8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see rxla_oracle.h): the checker for the CUDA
 * library and the timed CPU baseline.  Nothing in the product links it.
 *
 * Build: oracle/build_oracle.sh (gcc -O3 -fopenmp -ffp-contract=off; no FMA
 * contraction, so f32 expressions round exactly where the reference's
 * StableHLO ops round).
 */
#include "rxla_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */

uint16_t oracle_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

float oracle_bf16_round(float x) { return oracle_bf16_to_f32(oracle_f32_to_bf16(x)); }

/* ------------------------------------------------------------------- RNG */

uint64_t oracle_splitmix64(uint64_t x) {
  uint64_t z = x + 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

static inline uint64_t stream_word(uint64_t seed, uint64_t i) {
  return oracle_splitmix64(oracle_splitmix64(seed) + i);
}

static inline double unit_open(uint64_t r) { /* (0, 1] */
  return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}
static inline double unit_closed_open(uint64_t r) { /* [0, 1) */
  return (double)(r >> 11) * (1.0 / 9007199254740992.0);
}

void oracle_fill_normal(float* out, int64_t n, uint64_t seed, float mean, float std) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double u1 = unit_open(stream_word(seed, 2 * (uint64_t)i));
    double u2 = unit_closed_open(stream_word(seed, 2 * (uint64_t)i + 1));
    double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    out[i] = (float)(mean + std * z);
  }
}

void oracle_fill_uniform(float* out, int64_t n, uint64_t seed, float lo, float hi) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double u = unit_closed_open(stream_word(seed, (uint64_t)i));
    out[i] = (float)(lo + (hi - lo) * u);
  }
}

void oracle_fill_randint(int32_t* out, int64_t n, uint64_t seed, int32_t lo, int32_t hi) {
  uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    uint64_t r = stream_word(seed, (uint64_t)i);
    out[i] = (int32_t)((int64_t)lo + (int64_t)(r % span));
  }
}

/* ------------------------------------------------------------ W8 storage */

void oracle_quantize_w8(const float* w, int64_t n, int64_t k, int64_t group, uint8_t* q,
                        float* scale) {
  /* benchmarks/quantize_qwen3_5_w8.py:33-44, f32 tensor arithmetic */
  int64_t groups = k / group;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t g = 0; g < groups; ++g) {
      const float* src = w + r * k + g * group;
      float amax = 0.0f;
      for (int64_t j = 0; j < group; ++j) {
        float a = fabsf(src[j]);
        if (a > amax) amax = a;
      }
      if (amax < 1e-12f) amax = 1e-12f;
      float s = amax / 127.0f;
      scale[r * groups + g] = s;
      for (int64_t j = 0; j < group; ++j) {
        float v = rintf(src[j] / s); /* torch.round: half to even */
        if (v > 127.0f) v = 127.0f;
        if (v < -127.0f) v = -127.0f;
        q[r * k + g * group + j] = (uint8_t)((int32_t)v + 128);
      }
    }
  }
}

/* -------------------------------------------------------- QuantizedLinear */

void oracle_w8_linear(const float* x, int64_t m, int64_t k, const uint8_t* w,
                      const float* scale, int64_t n, int64_t group, int32_t mode, float* y) {
  int64_t groups = k / group;
  float* xr = (float*)malloc(sizeof(float) * (size_t)(m * k));
  for (int64_t i = 0; i < m * k; ++i) xr[i] = (mode == 0) ? x[i] : oracle_bf16_round(x[i]);
#pragma omp parallel
  {
    float* wrow = (float*)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
      if (mode == 2 || mode == 3) {
        /* four tokens at a time: four independent sums, each in the same
         * sequential order as a token alone (identical results, less time
         * waiting on one dependent add chain) */
        for (int64_t m0 = 0; m0 < m; m0 += 4) {
          const int64_t nt = m - m0 < 4 ? m - m0 : 4;
          double acc[4] = {0.0, 0.0, 0.0, 0.0};
          for (int64_t g = 0; g < groups; ++g) {
            double part[4] = {0.0, 0.0, 0.0, 0.0};
            for (int64_t j = 0; j < group; ++j) {
              int64_t c = g * group + j;
              const double wq = (double)((int32_t)w[r * k + c] - 128);
              for (int64_t u = 0; u < nt; ++u) part[u] += (double)xr[(m0 + u) * k + c] * wq;
            }
            for (int64_t u = 0; u < nt; ++u) acc[u] += part[u] * (double)scale[r * groups + g];
          }
          for (int64_t u = 0; u < nt; ++u)
            y[(m0 + u) * n + r] = mode == 3 ? oracle_bf16_round((float)acc[u]) : (float)acc[u];
        }
        continue;
      }
      /* layers.rs:277-288: cast(F32) -> add(-128) -> mul(scale) in f32 */
      for (int64_t c = 0; c < k; ++c) {
        float wd = (float)((int32_t)w[r * k + c] - 128) * scale[r * groups + c / group];
        wrow[c] = (mode == 1 || mode == 4 || mode == 5) ? oracle_bf16_round(wd) : wd;
      }
      int64_t mm = 0;
      if (mode != 4 && mode != 5) {
        /* four tokens at a time, each its own sequential f64 sum (identical
         * results to one token at a time) */
        for (; mm + 4 <= m; mm += 4) {
          double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
          const float* x0 = xr + mm * k;
          for (int64_t c = 0; c < k; ++c) {
            const double wv = (double)wrow[c];
            a0 += (double)x0[c] * wv;
            a1 += (double)x0[k + c] * wv;
            a2 += (double)x0[2 * k + c] * wv;
            a3 += (double)x0[3 * k + c] * wv;
          }
          const double a[4] = {a0, a1, a2, a3};
          for (int u = 0; u < 4; ++u)
            y[(mm + u) * n + r] = mode == 1 ? oracle_bf16_round((float)a[u]) : (float)a[u];
        }
      }
      for (; mm < m; ++mm) {
        float out;
        if (mode == 4 || mode == 5) { /* mode 1 with an fp32 running sum (noise-floor
                                         * probe); mode 5 leaves the sum unrounded */
          float facc = 0.0f;
          for (int64_t c = 0; c < k; ++c) facc += xr[mm * k + c] * wrow[c];
          out = facc;
        } else {
          double acc = 0.0;
          for (int64_t c = 0; c < k; ++c) acc += (double)xr[mm * k + c] * (double)wrow[c];
          out = (float)acc;
        }
        y[mm * n + r] = (mode == 1 || mode == 4) ? oracle_bf16_round(out) : out;
      }
    }
    free(wrow);
  }
  free(xr);
}

void oracle_linear(const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                   int32_t bf16, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t mm = 0; mm < m; ++mm) {
      double acc = 0.0;
      for (int64_t c = 0; c < k; ++c) {
        float xv = bf16 ? oracle_bf16_round(x[mm * k + c]) : x[mm * k + c];
        acc += (double)xv * (double)w[r * k + c];
      }
      y[mm * n + r] = bf16 ? oracle_bf16_round((float)acc) : (float)acc;
    }
  }
}

/* ---------------------------------------------------------------- RMSNorm */

void oracle_rms_norm(const float* x, int64_t rows, int64_t width, const float* w, float eps,
                     float* y) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * width;
    double ss = 0.0;
    for (int64_t c = 0; c < width; ++c) ss += (double)xr[c] * (double)xr[c];
    float mean = (float)(ss / (double)width);
    float rs = (float)(1.0 / sqrt((double)(mean + eps)));
    for (int64_t c = 0; c < width; ++c) {
      float t = xr[c] * rs;
      y[r * width + c] = t * w[c];
    }
  }
}

/* ------------------------------------------------------------------- RoPE */

void oracle_rope_inv_freq(float theta, int32_t rotary_dim, float* inv_freq) {
  for (int32_t i = 0; i < rotary_dim / 2; ++i)
    inv_freq[i] = powf(theta, (-2.0f * (float)i) / (float)rotary_dim);
}

void oracle_rope_split_half(float* x, int64_t rows, int64_t width, int32_t rotary_dim,
                            const int32_t* positions, const float* inv_freq) {
  int32_t half = rotary_dim / 2;
  for (int64_t r = 0; r < rows; ++r) {
    float* v = x + r * width;
    float pos = (float)positions[r];
    for (int32_t i = 0; i < half; ++i) {
      float angle = pos * inv_freq[i];
      float c = (float)cos((double)angle);
      float s = (float)sin((double)angle);
      float a = v[i], b = v[i + half];
      float ac = a * c, bs = b * s, bc = b * c, as = a * s;
      v[i] = ac - bs;
      v[i + half] = bc + as;
    }
  }
}

void oracle_rope_cos_sin(const float* x, int64_t rows, int64_t width, const float* cos_t,
                         const float* sin_t, int32_t layout, float* y) {
  int64_t half = width / 2;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t i = 0; i < half; ++i) {
      int64_t ia = layout == 0 ? i : 2 * i;
      int64_t ib = layout == 0 ? i + half : 2 * i + 1;
      float a = x[r * width + ia], b = x[r * width + ib];
      float c = cos_t[r * half + i], s = sin_t[r * half + i];
      float ac = a * c, bs = b * s, bc = b * c, as = a * s;
      y[r * width + ia] = ac - bs;
      y[r * width + ib] = bc + as;
    }
  }
}

/* -------------------------------------------------------------- attention */

void oracle_causal_mask(const int32_t* qpos, int64_t nq, const int32_t* kpos, int64_t nk,
                        float* mask) {
  for (int64_t i = 0; i < nq; ++i)
    for (int64_t j = 0; j < nk; ++j) mask[i * nk + j] = (kpos[j] <= qpos[i]) ? 0.0f : -INFINITY;
}

void oracle_gqa_attention(const float* q, const float* k, const float* v, const float* mask,
                          int64_t mask_b_stride, int64_t mask_h_stride, int64_t B, int64_t hq,
                          int64_t hkv, int64_t T, int64_t S, int64_t D, int64_t Dv, float scale,
                          float* out) {
  int64_t group = hq / hkv;
#pragma omp parallel
  {
    double* logits = (double*)malloc(sizeof(double) * (size_t)(S > 0 ? S : 1));
#pragma omp for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; ++b) {
      for (int64_t h = 0; h < hq; ++h) {
        int64_t kvh = h / group;
        const float* kb = k + (b * hkv + kvh) * S * D;
        const float* vb = v + (b * hkv + kvh) * S * Dv;
        for (int64_t t = 0; t < T; ++t) {
          const float* qr = q + ((b * hq + h) * T + t) * D;
          double mx = -INFINITY;
          for (int64_t s = 0; s < S; ++s) {
            double dot = 0.0;
            for (int64_t d = 0; d < D; ++d) dot += (double)qr[d] * (double)kb[s * D + d];
            double l = dot * (double)scale;
            if (mask) l += (double)mask[b * mask_b_stride + h * mask_h_stride + t * S + s];
            logits[s] = l;
            if (l > mx) mx = l;
          }
          double sum = 0.0;
          for (int64_t s = 0; s < S; ++s) {
            logits[s] = exp(logits[s] - mx);
            sum += logits[s];
          }
          float* o = out + ((b * hq + h) * T + t) * Dv;
          for (int64_t d = 0; d < Dv; ++d) {
            double acc = 0.0;
            for (int64_t s = 0; s < S; ++s) acc += logits[s] * (double)vb[s * Dv + d];
            o[d] = (float)(acc / sum);
          }
        }
      }
    }
    free(logits);
  }
}

/* --------------------------------------------------------------- KV cache */

int32_t oracle_kv_update(float* k_cache, float* v_cache, const int64_t* cache_shape,
                         const float* k_upd, const float* v_upd, const int64_t* upd_shape,
                         int32_t rank, const int32_t* starts, int32_t checked) {
  int64_t eff[8];
  for (int32_t a = 0; a < rank; ++a) {
    int64_t limit = cache_shape[a] - upd_shape[a];
    int64_t s = starts[a];
    if (checked) {
      if (s < 0 || s > limit) return 0; /* kv_cache.rs:100-104: both caches kept */
    } else {
      if (s < 0) s = 0; /* dynamic_update_slice clamps (kv_cache.rs:43-47) */
      if (s > limit) s = limit;
    }
    eff[a] = s;
  }
  int64_t total = 1;
  for (int32_t a = 0; a < rank; ++a) total *= upd_shape[a];
  for (int64_t i = 0; i < total; ++i) {
    int64_t rem = i, off = 0, stride = 1;
    int64_t idx[8];
    for (int32_t a = rank - 1; a >= 0; --a) {
      idx[a] = rem % upd_shape[a];
      rem /= upd_shape[a];
    }
    for (int32_t a = rank - 1; a >= 0; --a) {
      off += (idx[a] + eff[a]) * stride;
      stride *= cache_shape[a];
    }
    k_cache[off] = k_upd[i];
    v_cache[off] = v_upd[i];
  }
  return 1;
}

/* ----------------------------------------------------- paged decode oracle */

static void head_rms_norm(float* v, int32_t d, const float* w, float eps) {
  oracle_rms_norm(v, 1, d, w, eps, v);
}

void oracle_paged_decode_attention(
    int32_t batch, int32_t hq, int32_t hkv, int32_t d, const float* q, const float* k_new,
    const float* v_new, int64_t q_row_stride, int64_t kv_row_stride, const float* q_norm_w,
    const float* k_norm_w, float eps, const float* inv_freq, int32_t rotary_dim, float scale,
    uint16_t* k_pages, uint16_t* v_pages, int32_t page_size, int32_t max_pages_per_seq,
    const int32_t* page_table, const int32_t* pages_per_seq, int32_t* ctx_lens,
    int32_t kv_update, int32_t advance_ctx, int32_t* accepted, float* out) {
  int32_t group = hq / hkv;
  if (scale == 0.0f) scale = 1.0f / sqrtf((float)d);
  float* qh = (float*)malloc(sizeof(float) * (size_t)d);
  float* kh = (float*)malloc(sizeof(float) * (size_t)d);
  for (int32_t b = 0; b < batch; ++b) {
    int32_t pos = ctx_lens[b];
    int32_t cap = (pages_per_seq ? pages_per_seq[b] : max_pages_per_seq) * page_size;
    /* update_at clamps the start into the cache (kv_cache.rs:43-47); the checked
     * form writes nothing for an out-of-range start (kv_cache.rs:70-112) */
    int32_t in_range = pos >= 0 && pos < cap;
    int32_t ok = cap > 0 && (in_range || kv_update == 0);
    int32_t slot = pos < 0 ? 0 : (pos >= cap ? cap - 1 : pos);
    if (accepted) accepted[b] = ok;
    /* keys are visible iff slot index <= query position (attention.rs:14-32) */
    int32_t n_keys = pos < 0 ? 0 : (pos + 1 < cap ? pos + 1 : cap);
    for (int32_t kv = 0; kv < hkv; ++kv) {
      if (ok) {
        memcpy(kh, k_new + (int64_t)b * kv_row_stride + (int64_t)kv * d, sizeof(float) * d);
        if (k_norm_w) head_rms_norm(kh, d, k_norm_w, eps);
        if (inv_freq && rotary_dim > 0) oracle_rope_split_half(kh, 1, d, rotary_dim, &pos, inv_freq);
        int32_t page = page_table[(int64_t)b * max_pages_per_seq + slot / page_size];
        int64_t base = (((int64_t)page * hkv + kv) * page_size + slot % page_size) * d;
        for (int32_t i = 0; i < d; ++i) {
          k_pages[base + i] = oracle_f32_to_bf16(kh[i]);
          v_pages[base + i] =
              oracle_f32_to_bf16(v_new[(int64_t)b * kv_row_stride + (int64_t)kv * d + i]);
        }
      }
      for (int32_t g = 0; g < group; ++g) {
        int32_t h = kv * group + g;
        memcpy(qh, q + (int64_t)b * q_row_stride + (int64_t)h * d, sizeof(float) * d);
        if (q_norm_w) head_rms_norm(qh, d, q_norm_w, eps);
        if (inv_freq && rotary_dim > 0) oracle_rope_split_half(qh, 1, d, rotary_dim, &pos, inv_freq);
        double* lg = (double*)malloc(sizeof(double) * (size_t)(n_keys > 0 ? n_keys : 1));
        double mx = -INFINITY;
        for (int32_t s = 0; s < n_keys; ++s) {
          int32_t page = page_table[(int64_t)b * max_pages_per_seq + s / page_size];
          int64_t base = (((int64_t)page * hkv + kv) * page_size + s % page_size) * d;
          double dot = 0.0;
          for (int32_t i = 0; i < d; ++i) dot += (double)qh[i] * (double)oracle_bf16_to_f32(k_pages[base + i]);
          lg[s] = dot * (double)scale;
          if (lg[s] > mx) mx = lg[s];
        }
        double sum = 0.0;
        for (int32_t s = 0; s < n_keys; ++s) {
          lg[s] = exp(lg[s] - mx);
          sum += lg[s];
        }
        for (int32_t i = 0; i < d; ++i) {
          double acc = 0.0;
          for (int32_t s = 0; s < n_keys; ++s) {
            int32_t page = page_table[(int64_t)b * max_pages_per_seq + s / page_size];
            int64_t base = (((int64_t)page * hkv + kv) * page_size + s % page_size) * d;
            acc += lg[s] * (double)oracle_bf16_to_f32(v_pages[base + i]);
          }
          float o = n_keys > 0 ? (float)(acc / sum) : 0.0f;
          out[(int64_t)b * hq * d + (int64_t)h * d + i] = oracle_bf16_round(o);
        }
        free(lg);
      }
    }
    if (advance_ctx) ctx_lens[b] = pos + ok;
  }
  free(qh);
  free(kh);
}

/* ---------------------------------------------------------------- decoder */

typedef struct oracle_param {
  char name[96];
  int32_t dtype; /* 0 f32, 1 bf16, 2 u8 */
  int64_t elems, rows, cols;
  void* data;
} oracle_param;

struct oracle_decoder {
  oracle_decoder_config cfg;
  int32_t nparams;
  oracle_param* params;
  uint16_t* k_cache; /* [layers][batch][hkv][max_ctx][d] bf16 */
  uint16_t* v_cache;
  int32_t* ctx;
  float* inv_freq;
};

static int32_t dec_groups(const oracle_decoder_config* c, int64_t k) {
  return c->group_size > 0 ? (int32_t)(k / c->group_size) : 1;
}

static void add_param2(oracle_decoder* dec, const char* name, int32_t dtype, int64_t rows,
                       int64_t cols) {
  int64_t elems = rows * cols;
  oracle_param* p = &dec->params[dec->nparams++];
  snprintf(p->name, sizeof(p->name), "%s", name);
  p->dtype = dtype;
  p->elems = elems;
  p->rows = rows;
  p->cols = cols;
  size_t esz = dtype == 0 ? 4 : (dtype == 1 ? 2 : 1);
  p->data = calloc((size_t)elems, esz);
}

static void add_param(oracle_decoder* dec, const char* name, int32_t dtype, int64_t elems) {
  add_param2(dec, name, dtype, 1, elems);
}

static void add_w8(oracle_decoder* dec, const char* prefix, int64_t n, int64_t k) {
  char nm[96];
  snprintf(nm, sizeof(nm), "%s.weight", prefix);
  add_param2(dec, nm, 2, n, k);
  snprintf(nm, sizeof(nm), "%s.scale", prefix);
  add_param2(dec, nm, 0, n, dec_groups(&dec->cfg, k));
}

static oracle_param* find_param(oracle_decoder* dec, const char* name) {
  for (int32_t i = 0; i < dec->nparams; ++i)
    if (strcmp(dec->params[i].name, name) == 0) return &dec->params[i];
  return NULL;
}

oracle_decoder* oracle_decoder_create(const oracle_decoder_config* cfg) {
  oracle_decoder* dec = (oracle_decoder*)calloc(1, sizeof(oracle_decoder));
  dec->cfg = *cfg;
  const oracle_decoder_config* c = cfg;
  int64_t H = c->hidden, D = c->head_dim, I = c->intermediate;
  dec->params = (oracle_param*)calloc((size_t)(16 * c->layers + 8), sizeof(oracle_param));
  if (c->embedding_bf16) {
    add_param2(dec, "embed_tokens.weight", 1, c->vocab, H);
  } else {
    add_w8(dec, "embed_tokens", c->vocab, H);
  }
  char pre[96];
  for (int32_t l = 0; l < c->layers; ++l) {
    snprintf(pre, sizeof(pre), "layers.%d.input_layernorm.weight", l);
    add_param(dec, pre, 0, H);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_proj", l);
    add_w8(dec, pre, c->q_heads * D, H);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_proj", l);
    add_w8(dec, pre, c->kv_heads * D, H);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.v_proj", l);
    add_w8(dec, pre, c->kv_heads * D, H);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_norm.weight", l);
    add_param(dec, pre, 0, D);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_norm.weight", l);
    add_param(dec, pre, 0, D);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.o_proj", l);
    add_w8(dec, pre, H, c->q_heads * D);
    snprintf(pre, sizeof(pre), "layers.%d.post_attention_layernorm.weight", l);
    add_param(dec, pre, 0, H);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.gate_proj", l);
    add_w8(dec, pre, I, H);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.up_proj", l);
    add_w8(dec, pre, I, H);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.down_proj", l);
    add_w8(dec, pre, H, I);
  }
  add_param(dec, "norm.weight", 0, H);
  size_t cache = (size_t)c->layers * c->max_batch * c->kv_heads * c->max_context * D;
  dec->k_cache = (uint16_t*)calloc(cache, 2);
  dec->v_cache = (uint16_t*)calloc(cache, 2);
  dec->ctx = (int32_t*)calloc((size_t)c->max_batch, 4);
  dec->inv_freq = (float*)calloc((size_t)D, 4);
  oracle_rope_inv_freq(c->rope_theta, (int32_t)D, dec->inv_freq);
  return dec;
}

void oracle_decoder_destroy(oracle_decoder* dec) {
  if (!dec) return;
  for (int32_t i = 0; i < dec->nparams; ++i) free(dec->params[i].data);
  free(dec->params);
  free(dec->k_cache);
  free(dec->v_cache);
  free(dec->ctx);
  free(dec->inv_freq);
  free(dec);
}

int64_t oracle_decoder_parameter(oracle_decoder* dec, const char* name, void** ptr,
                                 int32_t* dtype) {
  oracle_param* p = find_param(dec, name);
  if (!p) return -1;
  *ptr = p->data;
  /* report rxla_b200_dtype codes: F32 0, BF16 1, U8 2 */
  *dtype = p->dtype;
  size_t esz = p->dtype == 0 ? 4 : (p->dtype == 1 ? 2 : 1);
  return p->elems * (int64_t)esz;
}

void oracle_decoder_init_synthetic(oracle_decoder* dec, uint64_t seed) {
  for (int32_t i = 0; i < dec->nparams; ++i) {
    oracle_param* p = &dec->params[i];
    uint64_t s = seed * 1000003ull + (uint64_t)i;
    const char* nm = p->name;
    size_t len = strlen(nm);
    int is_scale = len > 6 && strcmp(nm + len - 6, ".scale") == 0;
    if (is_scale) continue; /* written with its weight */
    if (p->dtype == 0) { /* norm weights: 1 + N(0, 0.02), bf16-valued */
      float* f = (float*)p->data;
      oracle_fill_normal(f, p->elems, s, 1.0f, 0.02f);
      for (int64_t j = 0; j < p->elems; ++j) f[j] = oracle_bf16_round(f[j]);
    } else if (p->dtype == 1) { /* bf16 embedding N(0, 0.02) */
      float* tmp = (float*)malloc(sizeof(float) * (size_t)p->elems);
      oracle_fill_normal(tmp, p->elems, s, 0.0f, 0.02f);
      uint16_t* b = (uint16_t*)p->data;
      for (int64_t j = 0; j < p->elems; ++j) b[j] = oracle_f32_to_bf16(tmp[j]);
      free(tmp);
    } else { /* W8: N(0, 0.02) quantized with its scale (next parameter) */
      oracle_param* sc = &dec->params[i + 1];
      int64_t rows = p->rows, k = p->cols;
      int64_t group = k / sc->cols;
      float* tmp = (float*)malloc(sizeof(float) * (size_t)p->elems);
      oracle_fill_normal(tmp, p->elems, s, 0.0f, 0.02f);
      oracle_quantize_w8(tmp, rows, k, group, (uint8_t*)p->data, (float*)sc->data);
      free(tmp);
    }
  }
}

void oracle_decoder_reset(oracle_decoder* dec) {
  memset(dec->ctx, 0, sizeof(int32_t) * (size_t)dec->cfg.max_batch);
}

int32_t oracle_decoder_context(oracle_decoder* dec, int32_t b) { return dec->ctx[b]; }

void oracle_decoder_kv(oracle_decoder* dec, int32_t layer, uint16_t** k, uint16_t** v) {
  size_t per = (size_t)dec->cfg.max_batch * dec->cfg.kv_heads * dec->cfg.max_context *
               dec->cfg.head_dim;
  *k = dec->k_cache + (size_t)layer * per;
  *v = dec->v_cache + (size_t)layer * per;
}

static float silu_f32(float g) {
  /* crates/rxla-core/src/ops.rs:336-341: x * sigmoid(x), sigmoid with a
   * nonpositive exponent argument */
  float sig;
  if (g >= 0.0f) {
    float e = (float)exp(-(double)g);
    sig = 1.0f / (1.0f + e);
  } else {
    float e = (float)exp((double)g);
    sig = e / (1.0f + e);
  }
  return g * sig;
}

/* y[m, n] = bf16-compute W8 linear (layers.rs:289-297) */
static void dec_w8(oracle_decoder* dec, const char* prefix, const float* x, int64_t m,
                   int64_t k, int64_t n, float* y) {
  char nm[96];
  snprintf(nm, sizeof(nm), "%s.weight", prefix);
  oracle_param* w = find_param(dec, nm);
  snprintf(nm, sizeof(nm), "%s.scale", prefix);
  oracle_param* s = find_param(dec, nm);
  int64_t group = dec->cfg.group_size > 0 ? dec->cfg.group_size : k;
  oracle_w8_linear(x, m, k, (const uint8_t*)w->data, (const float*)s->data, n, group,
                   dec->cfg.linear_mode == 3 || dec->cfg.linear_mode == 4 ? dec->cfg.linear_mode : 1,
                   y);
}

/* Tied LM head: logits [M, V] of the final-norm output xn [M, H].
 * The reference (crates/rxla-models/src/qwen3_5/mod.rs:157-173) is an F32
 * linear: hidden(f32) · ((q - 128) · s in f32)ᵀ with no bf16 cast of either
 * operand — restated with an f64 sum (mode 0).  linear_mode 4 (the
 * noise-floor model of a bf16-activation, fp32-accumulation implementation)
 * rounds both operands to bf16 and sums in fp32 instead (mode 5). */
static void dec_head(oracle_decoder* dec, const float* xn, int64_t M, float* logits) {
  const oracle_decoder_config* c = &dec->cfg;
  int64_t H = c->hidden, V = c->vocab;
  oracle_param* emb = find_param(dec, "embed_tokens.weight");
  oracle_param* embs = find_param(dec, "embed_tokens.scale");
  const int bf16_model = c->linear_mode == 4;
  if (c->embedding_bf16) {
    uint16_t* e = (uint16_t*)emb->data;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < V; ++r) {
      for (int64_t b = 0; b < M; ++b) {
        if (bf16_model) {
          float acc = 0.0f;
          for (int64_t j = 0; j < H; ++j)
            acc += oracle_bf16_round(xn[b * H + j]) * oracle_bf16_to_f32(e[r * H + j]);
          logits[b * V + r] = acc;
        } else {
          double acc = 0.0;
          for (int64_t j = 0; j < H; ++j)
            acc += (double)xn[b * H + j] * (double)oracle_bf16_to_f32(e[r * H + j]);
          logits[b * V + r] = (float)acc;
        }
      }
    }
  } else {
    int64_t group = c->group_size > 0 ? c->group_size : H;
    oracle_w8_linear(xn, M, H, (const uint8_t*)emb->data, (const float*)embs->data, V, group,
                     bf16_model ? 5 : 0, logits);
  }
}

void oracle_decoder_step(oracle_decoder* dec, const int32_t* tokens, int32_t batch,
                         float* logits, int32_t* next_tokens) {
  const oracle_decoder_config* c = &dec->cfg;
  int64_t H = c->hidden, D = c->head_dim, I = c->intermediate, V = c->vocab;
  int64_t HQ = c->q_heads, HKV = c->kv_heads, G = HQ / HKV;
  int64_t M = batch;
  float* h = (float*)calloc((size_t)(M * H), 4);
  float* xn = (float*)calloc((size_t)(M * H), 4);
  float* q = (float*)calloc((size_t)(M * HQ * D), 4);
  float* kk = (float*)calloc((size_t)(M * HKV * D), 4);
  float* vv = (float*)calloc((size_t)(M * HKV * D), 4);
  float* att = (float*)calloc((size_t)(M * HQ * D), 4);
  float* o = (float*)calloc((size_t)(M * H), 4);
  float* gate = (float*)calloc((size_t)(M * I), 4);
  float* up = (float*)calloc((size_t)(M * I), 4);
  char pre[96];

  /* embedding (qwen3_5/mod.rs:134-155 for W8; a bf16 table widened to f32) */
  oracle_param* emb = find_param(dec, "embed_tokens.weight");
  oracle_param* embs = find_param(dec, "embed_tokens.scale");
  for (int64_t b = 0; b < M; ++b) {
    int64_t t = tokens[b];
    for (int64_t j = 0; j < H; ++j) {
      if (c->embedding_bf16) {
        h[b * H + j] = oracle_bf16_to_f32(((uint16_t*)emb->data)[t * H + j]);
      } else {
        int64_t groups = embs->elems / V;
        int64_t grp = c->group_size > 0 ? j / c->group_size : 0;
        h[b * H + j] = (float)((int32_t)((uint8_t*)emb->data)[t * H + j] - 128) *
                       ((float*)embs->data)[t * groups + grp];
      }
    }
  }
  for (int32_t l = 0; l < c->layers; ++l) {
    snprintf(pre, sizeof(pre), "layers.%d.input_layernorm.weight", l);
    oracle_rms_norm(h, M, H, (float*)find_param(dec, pre)->data, c->rms_eps, xn);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_proj", l);
    dec_w8(dec, pre, xn, M, H, HQ * D, q);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_proj", l);
    dec_w8(dec, pre, xn, M, H, HKV * D, kk);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.v_proj", l);
    dec_w8(dec, pre, xn, M, H, HKV * D, vv);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_norm.weight", l);
    float* qn = (float*)find_param(dec, pre)->data;
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_norm.weight", l);
    float* kn = (float*)find_param(dec, pre)->data;
    for (int64_t b = 0; b < M; ++b) {
      int32_t pos = dec->ctx[b];
      for (int64_t hh = 0; hh < HQ; ++hh) {
        float* v = q + b * HQ * D + hh * D;
        head_rms_norm(v, (int32_t)D, qn, c->rms_eps);
        oracle_rope_split_half(v, 1, D, (int32_t)D, &pos, dec->inv_freq);
      }
      for (int64_t hh = 0; hh < HKV; ++hh) {
        float* v = kk + b * HKV * D + hh * D;
        head_rms_norm(v, (int32_t)D, kn, c->rms_eps);
        oracle_rope_split_half(v, 1, D, (int32_t)D, &pos, dec->inv_freq);
        size_t base = ((((size_t)l * c->max_batch + b) * HKV + hh) * c->max_context + pos) * D;
        for (int64_t i = 0; i < D; ++i) {
          dec->k_cache[base + i] = oracle_f32_to_bf16(v[i]);
          dec->v_cache[base + i] = oracle_f32_to_bf16(vv[b * HKV * D + hh * D + i]);
        }
      }
      /* attention over positions [0, pos] of the bf16 cache, f64 softmax */
      int32_t n_keys = pos + 1;
      double scale = (double)(1.0f / sqrtf((float)D));
#pragma omp parallel for schedule(static)
      for (int64_t hh = 0; hh < HQ; ++hh) {
        int64_t kv = hh / G;
        size_t base = (((size_t)l * c->max_batch + b) * HKV + kv) * c->max_context * D;
        const float* qr = q + b * HQ * D + hh * D;
        double* lg = (double*)malloc(sizeof(double) * (size_t)n_keys);
        double mx = -INFINITY;
        for (int32_t s = 0; s < n_keys; ++s) {
          double dot = 0.0;
          for (int64_t i = 0; i < D; ++i)
            dot += (double)qr[i] * (double)oracle_bf16_to_f32(dec->k_cache[base + s * D + i]);
          lg[s] = dot * scale;
          if (lg[s] > mx) mx = lg[s];
        }
        double sum = 0.0;
        for (int32_t s = 0; s < n_keys; ++s) {
          lg[s] = exp(lg[s] - mx);
          sum += lg[s];
        }
        for (int64_t i = 0; i < D; ++i) {
          double acc = 0.0;
          for (int32_t s = 0; s < n_keys; ++s)
            acc += lg[s] * (double)oracle_bf16_to_f32(dec->v_cache[base + s * D + i]);
          att[b * HQ * D + hh * D + i] = (float)(acc / sum);
        }
        free(lg);
      }
    }
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.o_proj", l);
    dec_w8(dec, pre, att, M, HQ * D, H, o);
    for (int64_t i = 0; i < M * H; ++i) h[i] = h[i] + o[i];
    snprintf(pre, sizeof(pre), "layers.%d.post_attention_layernorm.weight", l);
    oracle_rms_norm(h, M, H, (float*)find_param(dec, pre)->data, c->rms_eps, xn);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.gate_proj", l);
    dec_w8(dec, pre, xn, M, H, I, gate);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.up_proj", l);
    dec_w8(dec, pre, xn, M, H, I, up);
    for (int64_t i = 0; i < M * I; ++i) gate[i] = silu_f32(gate[i]) * up[i];
    snprintf(pre, sizeof(pre), "layers.%d.mlp.down_proj", l);
    dec_w8(dec, pre, gate, M, I, H, o);
    for (int64_t i = 0; i < M * H; ++i) h[i] = h[i] + o[i];
  }
  oracle_rms_norm(h, M, H, (float*)find_param(dec, "norm.weight")->data, c->rms_eps, xn);
  dec_head(dec, xn, M, logits);
  for (int64_t b = 0; b < M; ++b) {
    int32_t best = 0;
    float bv = logits[b * V];
    for (int64_t r = 1; r < V; ++r)
      if (logits[b * V + r] > bv) {
        bv = logits[b * V + r];
        best = (int32_t)r;
      }
    next_tokens[b] = best;
    dec->ctx[b] += 1;
  }
  free(h);
  free(xn);
  free(q);
  free(kk);
  free(vv);
  free(att);
  free(o);
  free(gate);
  free(up);
}

/* Full-sequence forward of one prompt (positions 0 .. T-1) with the causal
 * mask, the way the reference runs a prompt (crates/rxla-models/src/qwen3_5/
 * mod.rs:199-260: causal_attention_mask at :229, SDPA of
 * crates/rxla-core/src/attention.rs:83-252): every linear over all T rows,
 * attention of the whole [T, T] score matrix under the additive mask.  K and V
 * are rounded to bf16 as the paged cache stores them.  Writes the last row's
 * logits [V] and its greedy token; the decoder's state is not touched. */
static void decoder_forward_impl(oracle_decoder* dec, int32_t seq, const int32_t* tokens,
                                 int32_t T, float* logits, int32_t* next_token) {
  const oracle_decoder_config* c = &dec->cfg;
  int64_t H = c->hidden, D = c->head_dim, I = c->intermediate, V = c->vocab;
  int64_t HQ = c->q_heads, HKV = c->kv_heads;
  int64_t M = T;
  float* h = (float*)calloc((size_t)(M * H), 4);
  float* xn = (float*)calloc((size_t)(M * H), 4);
  float* q = (float*)calloc((size_t)(M * HQ * D), 4);
  float* kk = (float*)calloc((size_t)(M * HKV * D), 4);
  float* vv = (float*)calloc((size_t)(M * HKV * D), 4);
  float* qh = (float*)calloc((size_t)(M * HQ * D), 4);  /* [HQ, T, D] */
  float* kh = (float*)calloc((size_t)(M * HKV * D), 4); /* [HKV, T, D] */
  float* vh = (float*)calloc((size_t)(M * HKV * D), 4);
  float* oh = (float*)calloc((size_t)(M * HQ * D), 4);
  float* att = (float*)calloc((size_t)(M * HQ * D), 4);
  float* o = (float*)calloc((size_t)(M * H), 4);
  float* gate = (float*)calloc((size_t)(M * I), 4);
  float* up = (float*)calloc((size_t)(M * I), 4);
  float* mask = (float*)calloc((size_t)(M * M), 4);
  int32_t* pos = (int32_t*)calloc((size_t)M, 4);
  char pre[96];
  for (int64_t t = 0; t < M; ++t) pos[t] = (int32_t)t;
  oracle_causal_mask(pos, M, pos, M, mask);

  oracle_param* emb = find_param(dec, "embed_tokens.weight");
  oracle_param* embs = find_param(dec, "embed_tokens.scale");
  for (int64_t b = 0; b < M; ++b) {
    int64_t t = tokens[b];
    for (int64_t j = 0; j < H; ++j) {
      if (c->embedding_bf16) {
        h[b * H + j] = oracle_bf16_to_f32(((uint16_t*)emb->data)[t * H + j]);
      } else {
        int64_t groups = embs->elems / V;
        int64_t grp = c->group_size > 0 ? j / c->group_size : 0;
        h[b * H + j] = (float)((int32_t)((uint8_t*)emb->data)[t * H + j] - 128) *
                       ((float*)embs->data)[t * groups + grp];
      }
    }
  }
  for (int32_t l = 0; l < c->layers; ++l) {
    snprintf(pre, sizeof(pre), "layers.%d.input_layernorm.weight", l);
    oracle_rms_norm(h, M, H, (float*)find_param(dec, pre)->data, c->rms_eps, xn);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_proj", l);
    dec_w8(dec, pre, xn, M, H, HQ * D, q);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_proj", l);
    dec_w8(dec, pre, xn, M, H, HKV * D, kk);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.v_proj", l);
    dec_w8(dec, pre, xn, M, H, HKV * D, vv);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.q_norm.weight", l);
    float* qn = (float*)find_param(dec, pre)->data;
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.k_norm.weight", l);
    float* kn = (float*)find_param(dec, pre)->data;
    for (int64_t t = 0; t < M; ++t) {
      for (int64_t hh = 0; hh < HQ; ++hh) {
        float* v = q + t * HQ * D + hh * D;
        head_rms_norm(v, (int32_t)D, qn, c->rms_eps);
        oracle_rope_split_half(v, 1, D, (int32_t)D, &pos[t], dec->inv_freq);
        memcpy(qh + (hh * M + t) * D, v, (size_t)D * 4);
      }
      for (int64_t hh = 0; hh < HKV; ++hh) {
        float* v = kk + t * HKV * D + hh * D;
        head_rms_norm(v, (int32_t)D, kn, c->rms_eps);
        oracle_rope_split_half(v, 1, D, (int32_t)D, &pos[t], dec->inv_freq);
        for (int64_t i = 0; i < D; ++i) {
          kh[(hh * M + t) * D + i] = oracle_bf16_round(v[i]);
          vh[(hh * M + t) * D + i] = oracle_bf16_round(vv[t * HKV * D + hh * D + i]);
        }
        if (seq >= 0) { /* prefill: the row's K/V into the sequence's cache slot t */
          size_t base = ((((size_t)l * c->max_batch + seq) * HKV + hh) * c->max_context + t) * D;
          for (int64_t i = 0; i < D; ++i) {
            dec->k_cache[base + i] = oracle_f32_to_bf16(kh[(hh * M + t) * D + i]);
            dec->v_cache[base + i] = oracle_f32_to_bf16(vh[(hh * M + t) * D + i]);
          }
        }
      }
    }
    oracle_gqa_attention(qh, kh, vh, mask, 0, 0, 1, HQ, HKV, M, M, D, D,
                         1.0f / sqrtf((float)D), oh);
    for (int64_t t = 0; t < M; ++t)
      for (int64_t hh = 0; hh < HQ; ++hh)
        memcpy(att + t * HQ * D + hh * D, oh + (hh * M + t) * D, (size_t)D * 4);
    snprintf(pre, sizeof(pre), "layers.%d.self_attn.o_proj", l);
    dec_w8(dec, pre, att, M, HQ * D, H, o);
    for (int64_t i = 0; i < M * H; ++i) h[i] = h[i] + o[i];
    snprintf(pre, sizeof(pre), "layers.%d.post_attention_layernorm.weight", l);
    oracle_rms_norm(h, M, H, (float*)find_param(dec, pre)->data, c->rms_eps, xn);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.gate_proj", l);
    dec_w8(dec, pre, xn, M, H, I, gate);
    snprintf(pre, sizeof(pre), "layers.%d.mlp.up_proj", l);
    dec_w8(dec, pre, xn, M, H, I, up);
    for (int64_t i = 0; i < M * I; ++i) gate[i] = silu_f32(gate[i]) * up[i];
    snprintf(pre, sizeof(pre), "layers.%d.mlp.down_proj", l);
    dec_w8(dec, pre, gate, M, I, H, o);
    for (int64_t i = 0; i < M * H; ++i) h[i] = h[i] + o[i];
  }
  /* the head on the last row */
  const float* hl = h + (M - 1) * H;
  oracle_rms_norm(hl, 1, H, (float*)find_param(dec, "norm.weight")->data, c->rms_eps, xn);
  dec_head(dec, xn, 1, logits);
  int32_t best = 0;
  for (int64_t r = 1; r < V; ++r)
    if (logits[r] > logits[best]) best = (int32_t)r;
  *next_token = best;
  free(h);
  free(xn);
  free(q);
  free(kk);
  free(vv);
  free(qh);
  free(kh);
  free(vh);
  free(oh);
  free(att);
  free(o);
  free(gate);
  free(up);
  free(mask);
  free(pos);
}

void oracle_decoder_forward(oracle_decoder* dec, const int32_t* tokens, int32_t T, float* logits,
                            int32_t* next_token) {
  decoder_forward_impl(dec, -1, tokens, T, logits, next_token);
}

/* The same full-sequence forward for sequence `seq` of the decoder's state,
 * which must be empty (context 0): the prompt rows' K/V (bf16, as a
 * token-by-token decode writes them) land in the sequence's cache and its
 * context becomes T, so decode steps continue after the prompt.  Returns 0,
 * or -1 (nothing done) when the sequence is not empty or T does not fit. */
int32_t oracle_decoder_prefill(oracle_decoder* dec, int32_t seq, const int32_t* tokens, int32_t T,
                               float* logits, int32_t* next_token) {
  if (seq < 0 || seq >= dec->cfg.max_batch || dec->ctx[seq] != 0 || T <= 0 ||
      T > dec->cfg.max_context)
    return -1;
  decoder_forward_impl(dec, seq, tokens, T, logits, next_token);
  dec->ctx[seq] = T;
  return 0;
}

/* Context length of sequence `seq` set directly (the cached K/V values at
 * positions below it are whatever the cache holds): for timing a decode step
 * at a long context without decoding the prompt. */
int32_t oracle_decoder_set_context(oracle_decoder* dec, int32_t seq, int32_t ctx) {
  if (seq < 0 || seq >= dec->cfg.max_batch || ctx < 0 || ctx >= dec->cfg.max_context) return -1;
  dec->ctx[seq] = ctx;
  return 0;
}

void oracle_set_num_threads(int32_t n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int32_t oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
