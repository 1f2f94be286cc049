/*
 * npu_oracle.c -- TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline).
 *
 * A plain-C restatement of the RustGears Npu(Int8) inference path.  Build with
 * `-O2 -ffp-contract=off -fno-fast-math` (oracle/Makefile): Rust never contracts
 * a*b+c into an FMA, and Rust's f32::{tanh,exp,ln,cos} call glibc's
 * tanhf/expf/logf/cosf on linux-gnu, which this file calls too.
 *
 * Threading mirrors the reference's rayon decomposition so that the timed CPU
 * baseline does the same work split: rows for Linear when m*k*n >= 32768
 * (quantize.rs:104), images for Conv2d when n >= 2 (npu.rs:331), planes for
 * MaxPool2d when total >= 8192 (kernels.rs:201).  Integer accumulation and
 * per-element f32 epilogues make every result independent of the thread count.
 */
#include "npu_oracle.h"

#define OG_MAX_RESIDUAL 8

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* ------------------------------------------------------------------------ */
/* parallel-for over [0, n) with static contiguous chunks                    */
/* ------------------------------------------------------------------------ */
typedef void (*og_body)(void* ctx, int64_t begin, int64_t end);
typedef struct { og_body fn; void* ctx; int64_t b, e; } og_chunk;

static void* og_chunk_run(void* p) {
  og_chunk* c = (og_chunk*)p;
  c->fn(c->ctx, c->b, c->e);
  return NULL;
}

static void og_parallel_for(int64_t n, int32_t nthreads, og_body fn, void* ctx) {
  if (n <= 0) return;
  if (nthreads <= 1 || n == 1) { fn(ctx, 0, n); return; }
  if (nthreads > n) nthreads = (int32_t)n;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  og_chunk ch[256];
  int64_t per = n / nthreads, rem = n % nthreads, at = 0;
  for (int32_t t = 0; t < nthreads; ++t) {
    int64_t len = per + (t < rem ? 1 : 0);
    ch[t].fn = fn; ch[t].ctx = ctx; ch[t].b = at; ch[t].e = at + len; at += len;
  }
  for (int32_t t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, og_chunk_run, &ch[t]);
  og_chunk_run(&ch[0]);
  for (int32_t t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* RNG: src/rng.rs                                                           */
/* ------------------------------------------------------------------------ */
#define OG_GOLDEN 0x9E3779B97F4A7C15ull

void og_rng_seed(og_rng* r, uint64_t seed) { r->state = seed ^ OG_GOLDEN; } /* rng.rs:16-18 */

uint64_t og_rng_next_u64(og_rng* r) { /* rng.rs:21-27 */
  r->state += OG_GOLDEN;
  uint64_t z = r->state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

float og_rng_uniform(og_rng* r) { /* rng.rs:30-32: 24 random bits / 2^24 (exact in f32) */
  return (float)(og_rng_next_u64(r) >> 40) / 16777216.0f;
}

float og_rng_uniform_range(og_rng* r, float lo, float hi) { /* rng.rs:35-37 */
  float u = og_rng_uniform(r);
  float span = hi - lo;
  float t = span * u;
  return lo + t;
}

float og_rng_normal(og_rng* r) { /* rng.rs:40-44: Box-Muller, cosine branch only */
  float u1 = fmaxf(og_rng_uniform(r), 1e-7f);
  float u2 = og_rng_uniform(r);
  const float two_pi = 2.0f * 3.14159265358979323846f; /* 2.0 * f32::consts::PI */
  float a = sqrtf(-2.0f * logf(u1));
  float b = cosf(two_pi * u2);
  return a * b;
}

void og_fill_uniform_range(og_rng* r, float* out, int64_t n, float lo, float hi) {
  for (int64_t i = 0; i < n; ++i) out[i] = og_rng_uniform_range(r, lo, hi);
}
void og_fill_normal(og_rng* r, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = og_rng_normal(r);
}
void og_fill_normal_scaled(og_rng* r, float* out, int64_t n, float std) {
  /* init::normal = randn(shape) then detach_scaled(std): v * s (nn/init.rs:18-20, 30-32) */
  for (int64_t i = 0; i < n; ++i) { float v = og_rng_normal(r); out[i] = v * std; }
}
void og_fill_below(og_rng* r, int64_t* out, int64_t n, uint64_t bound) {
  for (int64_t i = 0; i < n; ++i) out[i] = (int64_t)(og_rng_next_u64(r) % bound);
}
float og_kaiming_bound(int64_t fan_in) { /* init.rs:7 */
  float f = (float)(fan_in > 1 ? fan_in : 1);
  return sqrtf(6.0f / f);
}
float og_bias_bound(int64_t fan_in) { /* init.rs:24 */
  float f = (float)(fan_in > 1 ? fan_in : 1);
  return 1.0f / sqrtf(f);
}

/* ------------------------------------------------------------------------ */
/* activations: inference/mod.rs:38-53 -> device/backend.rs:61-78            */
/* ------------------------------------------------------------------------ */
float og_act_apply(int32_t act, float param, float x) {
  switch (act) {
    case OG_ACT_NONE: return x;
    case OG_ACT_RELU: return fmaxf(x, 0.0f);               /* x.max(0.0): NaN -> 0 */
    case OG_ACT_SIGMOID: { float e = expf(-x); float d = 1.0f + e; return 1.0f / d; }
    case OG_ACT_TANH: return tanhf(x);
    case OG_ACT_GELU: {
      /* 0.5 * x * (1.0 + (GELU_C * (x + 0.044715 * x * x * x)).tanh()), left to right */
      const float gelu_c = 0.7978846f;
      float c = 0.044715f * x; c = c * x; c = c * x;
      float inner = x + c;
      float t = tanhf(gelu_c * inner);
      float h = 0.5f * x;
      float s = 1.0f + t;
      return h * s;
    }
    case OG_ACT_LEAKY_RELU: return x > 0.0f ? x : param * x;
    /* extension: nn::Silu (nn/layers.rs:337-346) = x.mul(x.sigmoid()), the sigmoid of
     * UnaryOp::apply (device/backend.rs:72) */
    case OG_ACT_SILU: { float sg = 1.0f / (1.0f + expf(-x)); return x * sg; }
    default: return x;
  }
}

/* ------------------------------------------------------------------------ */
/* symmetric per-tensor quantization: inference/quantize.rs:18-35            */
/* ------------------------------------------------------------------------ */
float og_quant_scale(const float* v, int64_t n) {
  float m = 0.0f;
  for (int64_t i = 0; i < n; ++i) m = fmaxf(m, fabsf(v[i])); /* fold(0, max(|v|)): NaN ignored */
  return m < 1e-12f ? 1.0f : m / 127.0f;
}

static inline int8_t og_q1(float v, float inv) {
  float t = roundf(v * inv);                 /* round half away from zero */
  if (isnan(t)) return 0;                    /* `as i8` maps NaN to 0 */
  if (t < -127.0f) t = -127.0f;
  if (t > 127.0f) t = 127.0f;
  return (int8_t)t;
}

float og_quantize_into(const float* v, int64_t n, int8_t* out) {
  float scale = og_quant_scale(v, n);
  float inv = 1.0f / scale;
  for (int64_t i = 0; i < n; ++i) out[i] = og_q1(v[i], inv);
  return scale;
}

/* dot_i8: quantize.rs:68-88 (integer-exact; the unroll order cannot change the sum) */
static inline int32_t og_dot_i8(const int8_t* a, const int8_t* b, int64_t len) {
  int32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  int64_t i = 0;
  for (; i + 4 <= len; i += 4) {
    a0 += (int32_t)a[i] * b[i];
    a1 += (int32_t)a[i + 1] * b[i + 1];
    a2 += (int32_t)a[i + 2] * b[i + 2];
    a3 += (int32_t)a[i + 3] * b[i + 3];
  }
  int32_t t = (a0 + a1) + (a2 + a3);
  for (; i < len; ++i) t += (int32_t)a[i] * b[i];
  return t;
}

/* int8_gemm_fused body for rows [b,e): quantize.rs:93-144 */
typedef struct {
  const int8_t* a; const int8_t* w; const float* bias; float cs;
  int64_t k, n; int32_t act; float param; float* out; int32_t* acc;
  int64_t row0;  /* row offset of out/acc relative to a */
  const float* wsc; float sa;  /* per-channel weights: column j's scale is sa * wsc[j] */
} og_gemm_ctx;

static void og_gemm_rows(void* p, int64_t b, int64_t e) {
  og_gemm_ctx* c = (og_gemm_ctx*)p;
  for (int64_t r = b; r < e; ++r) {
    const int8_t* arow = c->a + r * c->k;
    float* orow = c->out + (r - c->row0) * c->n;
    for (int64_t j = 0; j < c->n; ++j) {
      int32_t acc = og_dot_i8(arow, c->w + j * c->k, c->k);
      if (c->acc) c->acc[(r - c->row0) * c->n + j] = acc;
      const float cs = c->wsc ? c->sa * c->wsc[j] : c->cs;
      float v = (float)acc * cs;          /* (acc as f32) * combined_scale */
      v = v + c->bias[j];                 /* + bias[c] */
      orow[j] = og_act_apply(c->act, c->param, v);
    }
  }
}

/* round_fp16 (quantize.rs:50-64): exponent below -14 -> +0, above 15 -> +-65504
 * (inf and NaN included), else keep 10 mantissa bits, the 13th bit rounding up. */
float og_round_fp16(float x) {
  uint32_t bits; memcpy(&bits, &x, 4);
  uint32_t sign = bits & 0x80000000u;
  int32_t e = (int32_t)((bits >> 23) & 0xffu) - 127;
  if (e < -14) return 0.0f;
  uint32_t r = e > 15 ? (sign | 0x477fe000u) : ((bits + (1u << 12)) & ~0x1fffu);
  float y; memcpy(&y, &r, 4);
  return y;
}

/* fp16_gemm_fused_into (npu.rs:431-445) for rows [b,e): a [m,k] f32, w [n,k]:
 * acc = 0; acc += round_fp16(a) * w in k order; out = act(round_fp16(acc + bias)). */
typedef struct {
  const float* a; const float* w; const float* bias;
  int64_t k, n; int32_t act; float param; float* out;
} og_fp16_ctx;

static void og_fp16_rows(void* p, int64_t b, int64_t e) {
  og_fp16_ctx* c = (og_fp16_ctx*)p;
  for (int64_t r = b; r < e; ++r) {
    const float* arow = c->a + r * c->k;
    for (int64_t j = 0; j < c->n; ++j) {
      const float* brow = c->w + j * c->k;
      float acc = 0.0f;
      for (int64_t i = 0; i < c->k; ++i) {
        float t = og_round_fp16(arow[i]) * brow[i];
        acc = acc + t;
      }
      c->out[r * c->n + j] = og_act_apply(c->act, c->param, og_round_fp16(acc + c->bias[j]));
    }
  }
}

/* ------------------------------------------------------------------------ */
/* kernels.rs / shape.rs helpers                                             */
/* ------------------------------------------------------------------------ */
int64_t og_out_size(int64_t input, int64_t k, int64_t stride, int64_t pad) { /* kernels.rs:10-15 */
  int64_t padded = input + 2 * pad;
  if (k <= 0 || stride <= 0 || padded < k) return -1;
  return (padded - k) / stride + 1;
}

void og_im2col(const float* x, int32_t c, int32_t h, int32_t w, int32_t k, int32_t stride,
               int32_t pad, int32_t oh, int32_t ow, float* cols) { /* kernels.rs:28-96 */
  int64_t l = (int64_t)oh * ow;
  if (pad > 0) memset(cols, 0, sizeof(float) * (size_t)(c * k * k) * (size_t)l);
  if (stride == 1) {
    for (int32_t ch = 0; ch < c; ++ch) {
      int64_t ch_off = (int64_t)ch * h * w;
      for (int32_t ki = 0; ki < k; ++ki) {
        int32_t dy = ki - pad;
        int32_t oy_start = -dy > 0 ? -dy : 0;
        int32_t oy_end = (h - dy) < oh ? (h - dy) : oh; if (oy_end < 0) oy_end = 0;
        for (int32_t kj = 0; kj < k; ++kj) {
          int32_t dx = kj - pad;
          int32_t ox_start = -dx > 0 ? -dx : 0;
          int32_t ox_end = (w - dx) < ow ? (w - dx) : ow; if (ox_end < 0) ox_end = 0;
          if (ox_start >= ox_end) continue;
          int32_t ix_start = ox_start + dx;
          int32_t len = ox_end - ox_start;
          int64_t base = ((int64_t)(ch * k + ki) * k + kj) * l;
          for (int32_t oy = oy_start; oy < oy_end; ++oy) {
            int32_t iy = oy + dy;
            memcpy(cols + base + (int64_t)oy * ow + ox_start, x + ch_off + (int64_t)iy * w + ix_start,
                   sizeof(float) * (size_t)len);
          }
        }
      }
    }
  } else {
    for (int32_t ch = 0; ch < c; ++ch)
      for (int32_t ki = 0; ki < k; ++ki)
        for (int32_t kj = 0; kj < k; ++kj) {
          int64_t base = ((int64_t)(ch * k + ki) * k + kj) * l;
          for (int32_t oy = 0; oy < oh; ++oy) {
            int32_t iy = oy * stride + ki - pad;
            if (iy < 0 || iy >= h) continue;
            for (int32_t ox = 0; ox < ow; ++ox) {
              int32_t ix = ox * stride + kj - pad;
              if (ix < 0 || ix >= w) continue;
              cols[base + (int64_t)oy * ow + ox] = x[((int64_t)ch * h + iy) * w + ix];
            }
          }
        }
  }
}

void og_transpose2d(const float* x, int64_t rows, int64_t cols, float* out) { /* shape.rs:105-123 */
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) out[c * rows + r] = x[r * cols + c];
}

/* max_pool2d: kernels.rs:165-213 (pad 0; strict > keeps the first of ties; NaN propagates) */
typedef struct { const float* x; float* y; int32_t h, w, k, s, oh, ow; } og_pool_ctx;
static void og_pool_planes(void* p, int64_t b, int64_t e) {
  og_pool_ctx* c = (og_pool_ctx*)p;
  for (int64_t plane = b; plane < e; ++plane) {
    const float* xp = c->x + plane * (int64_t)c->h * c->w;
    float* yp = c->y + plane * (int64_t)c->oh * c->ow;
    for (int32_t oy = 0; oy < c->oh; ++oy)
      for (int32_t ox = 0; ox < c->ow; ++ox) {
        float best = -INFINITY;
        for (int32_t ki = 0; ki < c->k; ++ki)
          for (int32_t kj = 0; kj < c->k; ++kj) {
            float v = xp[(int64_t)(oy * c->s + ki) * c->w + ox * c->s + kj];
            if (v > best || isnan(v)) best = v;
          }
        yp[oy * c->ow + ox] = best;
      }
  }
}
void og_maxpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t k,
                  int32_t stride, float* y, int32_t nthreads) {
  og_pool_ctx ctx = { x, y, h, w, k, stride, (int32_t)og_out_size(h, k, stride, 0),
                      (int32_t)og_out_size(w, k, stride, 0) };
  int64_t planes = n * c, total = planes * ctx.oh * ctx.ow;
  if (total <= 0) return;
  og_parallel_for(planes, total >= 8192 ? nthreads : 1, og_pool_planes, &ctx);
}

void og_activation(const float* x, int64_t n, int32_t act, float param, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = og_act_apply(act, param, x[i]);
}

/* Extension: adaptive_avg_pool2d (tensor/ops.rs:994-1014): region rows
 * [y*h/oh, ceil((y+1)*h/oh)), columns likewise; f32 sum in row-major order from 0,
 * then one division by the region's element count. */
void og_adaptive_avgpool2d(const float* x, int64_t n, int32_t c, int32_t h, int32_t w, int32_t oh,
                           int32_t ow, float* y) {
  for (int64_t plane = 0; plane < n * c; ++plane)
    for (int32_t oy = 0; oy < oh; ++oy)
      for (int32_t ox = 0; ox < ow; ++ox) {
        const int32_t y0 = oy * h / oh, y1 = ((oy + 1) * h + oh - 1) / oh;
        const int32_t x0 = ox * w / ow, x1 = ((ox + 1) * w + ow - 1) / ow;
        float sum = 0.0f;
        for (int32_t yy = y0; yy < y1; ++yy)
          for (int32_t xx = x0; xx < x1; ++xx) sum += x[(plane * h + yy) * w + xx];
        y[(plane * oh + oy) * ow + ox] = sum / (float)((y1 - y0) * (x1 - x0));
      }
}

/* Extension: residual add (tensor/ops.rs:67-76 binary Add, same shapes) followed by
 * the block's activation: y = act(x + s). */
void og_residual_add(const float* x, const float* sv, int64_t n, int32_t act, float param, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = og_act_apply(act, param, x[i] + sv[i]);
}

/* ---- transformer extensions ------------------------------------------------- */

/* Embedding::forward (nn/layers.rs:438-446): row ids[r] of the table; the id is the f32
 * value cast `as usize` (truncation, NaN and negatives saturate to 0); an id >= V is
 * the reference's assertion failure (-6 here). */
int32_t og_embedding(const og_op* op, const float* ids, int64_t n, float* y) {
  const int64_t v = op->in_features, d = op->out_features;
  for (int64_t r = 0; r < n; ++r) {
    const float f = ids[r];
    uint64_t idx = 0;
    if (f >= 18446744073709551616.0f) idx = UINT64_MAX;
    else if (f >= 1.0f) idx = (uint64_t)f;
    if (idx >= (uint64_t)v) return -6;
    memcpy(y + r * d, op->extra + (int64_t)idx * d, sizeof(float) * (size_t)d);
  }
  return 0;
}

/* RMSNorm::forward (nn/norm.rs:413-417): rms = sqrt(mean_dim(x*x, -1) + eps) with the
 * squares summed serially from 0 (sum_dim, tensor/ops.rs:715-727) and the mean as a
 * multiplication by 1/d (mean_dim, 755-758); y = (x / rms) * weight. */
void og_rmsnorm(const og_op* op, const float* x, int64_t rows, float* y) {
  const int64_t d = op->in_features;
  const float inv_d = 1.0f / (float)d;
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * d;
    float s = 0.0f;
    for (int64_t i = 0; i < d; ++i) { const float sq = xr[i] * xr[i]; s += sq; }
    const float rms = sqrtf(s * inv_d + op->act_param);
    for (int64_t i = 0; i < d; ++i) y[r * d + i] = (xr[i] / rms) * op->extra[i];
  }
}

/* cpu_matmul per batch (device/cpu.rs:43-64 with matmul_avx2 233-395): every output
 * starts at 0 and accumulates fma(a[i][p], b[p][j], c) for p = 0..k-1 in order;
 * columns past the last full 8-wide block accumulate unfused (c += a * b). */
void og_bmm_fma(const float* a, const float* bm, int64_t batch, int64_t m, int64_t k, int64_t n, float* c) {
  const int64_t nv = n / 8 * 8;
  for (int64_t b = 0; b < batch; ++b) {
    const float* ab = a + b * m * k;
    const float* bb = bm + b * k * n;
    float* cb = c + b * m * n;
    for (int64_t i = 0; i < m; ++i)
      for (int64_t j = 0; j < n; ++j) {
        float acc = 0.0f;
        if (j < nv) {
          for (int64_t p = 0; p < k; ++p) acc = fmaf(ab[i * k + p], bb[p * n + j], acc);
        } else {
          for (int64_t p = 0; p < k; ++p) { const float t = ab[i * k + p] * bb[p * n + j]; acc += t; }
        }
        cb[i * n + j] = acc;
      }
  }
}

/* MultiHeadAttention, non-causal (nn/attention.rs:162-196) with its q, k, v, o Linears
 * on the INT8 path: heads split [b, t, h, dh] -> [b*h, t, dh], scores = bmm(q, k^T) *
 * (1 / sqrt(dh)), softmax over keys, bmm(p, v), heads merged, o projection. */
void og_attention(const og_op* op, const float* x, int64_t b, int64_t t, float* y, int32_t nthreads) {
  const int64_t d = op->in_features, h = op->out_features, dh = d / h, rows = b * t;
  float* q = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  float* k = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  float* v = (float*)malloc(sizeof(float) * (size_t)(rows * d));
  og_op_linear(&op->sub[0], x, rows, q, NULL, NULL, NULL, nthreads);
  og_op_linear(&op->sub[1], x, rows, k, NULL, NULL, NULL, nthreads);
  og_op_linear(&op->sub[2], x, rows, v, NULL, NULL, NULL, nthreads);
  const int64_t bh = b * h;
  float* qs = (float*)malloc(sizeof(float) * (size_t)(bh * t * dh));
  float* kt = (float*)malloc(sizeof(float) * (size_t)(bh * dh * t));   /* k transposed: [bh, dh, t] */
  float* vs = (float*)malloc(sizeof(float) * (size_t)(bh * t * dh));
  for (int64_t bi = 0; bi < b; ++bi)
    for (int64_t ti = 0; ti < t; ++ti)
      for (int64_t hi = 0; hi < h; ++hi)
        for (int64_t e = 0; e < dh; ++e) {
          const int64_t src = (bi * t + ti) * d + hi * dh + e, g = bi * h + hi;
          qs[(g * t + ti) * dh + e] = q[src];
          kt[(g * dh + e) * t + ti] = k[src];
          vs[(g * t + ti) * dh + e] = v[src];
        }
  float* sc = (float*)malloc(sizeof(float) * (size_t)(bh * t * t));
  og_bmm_fma(qs, kt, bh, t, dh, t, sc);
  const float scale = 1.0f / sqrtf((float)dh);
  for (int64_t i = 0; i < bh * t * t; ++i) sc[i] = sc[i] * scale;
  og_softmax(sc, bh * t, t, sc);
  float* o = (float*)malloc(sizeof(float) * (size_t)(bh * t * dh));
  og_bmm_fma(sc, vs, bh, t, t, dh, o);
  float* merged = q;  /* reuse: [b, t, d] */
  for (int64_t g = 0; g < bh; ++g)
    for (int64_t ti = 0; ti < t; ++ti)
      for (int64_t e = 0; e < dh; ++e)
        merged[((g / h) * t + ti) * d + (g % h) * dh + e] = o[(g * t + ti) * dh + e];
  og_op_linear(&op->sub[3], merged, rows, y, NULL, NULL, NULL, nthreads);
  free(q); free(k); free(v); free(qs); free(kt); free(vs); free(sc); free(o);
}

/* SwiGLU::forward (nn/layers.rs:507-513) with bias-free INT8 Linears:
 * down((g * sigmoid(g)) * u), g = gate(x), u = up(x). */
void og_swiglu(const og_op* op, const float* x, int64_t rows, float* y, int32_t nthreads) {
  const int64_t hd = op->out_features;
  float* g = (float*)malloc(sizeof(float) * (size_t)(rows * hd));
  float* u = (float*)malloc(sizeof(float) * (size_t)(rows * hd));
  og_op_linear(&op->sub[0], x, rows, g, NULL, NULL, NULL, nthreads);
  og_op_linear(&op->sub[1], x, rows, u, NULL, NULL, NULL, nthreads);
  for (int64_t i = 0; i < rows * hd; ++i) {
    const float silu = g[i] * og_act_apply(OG_ACT_SIGMOID, 0.0f, g[i]);
    g[i] = silu * u[i];
  }
  og_op_linear(&op->sub[2], g, rows, y, NULL, NULL, NULL, nthreads);
  free(g); free(u);
}

void og_softmax(const float* x, int64_t outer, int64_t last, float* y) { /* ops.rs:1058-1076 */
  for (int64_t o = 0; o < outer; ++o) {
    const float* xr = x + o * last; float* yr = y + o * last;
    float mx = -INFINITY;
    for (int64_t j = 0; j < last; ++j) mx = fmaxf(mx, xr[j]);
    float s = 0.0f;
    for (int64_t j = 0; j < last; ++j) { float e = expf(xr[j] - mx); yr[j] = e; s += e; }
    for (int64_t j = 0; j < last; ++j) yr[j] = yr[j] / s;
  }
}

/* ------------------------------------------------------------------------ */
/* compile: inference/mod.rs:225-257 (fold) + npu.rs:188-276 (fuse+quantize) */
/* ------------------------------------------------------------------------ */
typedef struct {
  int32_t kind, in_f, out_f, in_c, out_c, k, stride, pad, act; float param;
  float* w; int64_t w_len; float* b; int64_t b_len;
} og_flayer;

static og_flayer* og_fold(const og_layer* L, int32_t n, int32_t* out_n) {
  og_flayer* out = (og_flayer*)calloc((size_t)(n > 0 ? n : 1), sizeof(og_flayer));
  int32_t m = 0;
  for (int32_t i = 0; i < n; ++i) {
    const og_layer* l = &L[i];
    if (l->kind == OG_LAYER_CHANNEL_AFFINE && m > 0) {
      og_flayer* p = &out[m - 1];
      int64_t c = l->weight_len;
      if (p->kind == OG_LAYER_LINEAR && p->out_f == c) {
        for (int64_t r = 0; r < p->in_f; ++r)
          for (int64_t j = 0; j < p->out_f; ++j) p->w[r * p->out_f + j] *= l->weight[j];
        for (int64_t j = 0; j < p->out_f; ++j) { float t = p->b[j] * l->weight[j]; p->b[j] = t + l->bias[j]; }
        continue;
      }
      if ((p->kind == OG_LAYER_CONV2D || p->kind == OG_LAYER_SHORTCUT_CONV2D) && p->out_c == c) {
        int64_t plane = (int64_t)p->in_c * p->k * p->k;
        for (int64_t o = 0; o < p->out_c; ++o) {
          for (int64_t j = 0; j < plane; ++j) p->w[o * plane + j] *= l->weight[o];
          float t = p->b[o] * l->weight[o]; p->b[o] = t + l->bias[o];
        }
        continue;
      }
    }
    og_flayer* f = &out[m++];
    f->kind = l->kind; f->in_f = l->in_features; f->out_f = l->out_features;
    f->in_c = l->in_channels; f->out_c = l->out_channels; f->k = l->kernel;
    f->stride = l->stride; f->pad = l->padding; f->act = l->act; f->param = l->act_param;
    f->w_len = l->weight_len; f->b_len = l->bias_len;
    if (l->weight_len) { f->w = (float*)malloc(sizeof(float) * (size_t)l->weight_len); memcpy(f->w, l->weight, sizeof(float) * (size_t)l->weight_len); }
    if (l->bias_len) { f->b = (float*)malloc(sizeof(float) * (size_t)l->bias_len); memcpy(f->b, l->bias, sizeof(float) * (size_t)l->bias_len); }
  }
  *out_n = m;
  return out;
}

void og_fold_batch_norm_count(const og_layer* layers, int32_t n, int32_t* out_count) {
  int32_t m = 0;
  og_flayer* f = og_fold(layers, n, &m);
  for (int32_t i = 0; i < m; ++i) { free(f[i].w); free(f[i].b); }
  free(f);
  *out_count = m;
}

/* An INT8 Linear as npu::compile builds one (npu.rs:207-216): W [in,out] transposed to
 * [out,in], per-tensor i8; a NULL bias is a bias-free Linear (zeros, no f32 bias bytes). */
static void og_make_linear(og_program* p, og_op* op, const float* w_in_out, int32_t in, int32_t out,
                           const float* b) {
  memset(op, 0, sizeof(*op));
  op->kind = OG_LAYER_LINEAR; op->in_features = in; op->out_features = out; op->act = OG_ACT_NONE;
  const int64_t wl = (int64_t)in * out;
  float* wt = (float*)malloc(sizeof(float) * (size_t)(wl > 0 ? wl : 1));
  og_transpose2d(w_in_out, in, out, wt);
  op->wq = (int8_t*)malloc((size_t)(wl > 0 ? wl : 1)); op->wq_len = wl;
  op->w_scale = og_quantize_into(wt, wl, op->wq);
  free(wt);
  op->bias = (float*)calloc((size_t)(out > 0 ? out : 1), sizeof(float)); op->bias_len = out;
  if (b) memcpy(op->bias, b, sizeof(float) * (size_t)out);
  p->fp32_bytes += (wl + (b ? out : 0)) * 4;
  p->npu_bytes += (wl + 4) + (b ? out : 0) * 4;
}

/* Per-output-channel weight quantization (extension): each of the `rows` rows of the
 * [rows, cols] matrix gets its own QuantTensor::from_f32 scale (quantize.rs:18-24). */
static void og_quantize_rows_per_channel(og_op* op, const float* w, int64_t rows, int64_t cols) {
  op->w_scale = 0.0f;
  op->w_scale_ch = (float*)malloc(sizeof(float) * (size_t)(rows > 0 ? rows : 1));
  for (int64_t r = 0; r < rows; ++r) op->w_scale_ch[r] = og_quantize_into(w + r * cols, cols, op->wq + r * cols);
}

og_program* og_compile(const og_layer* layers, int32_t n_layers, int32_t precision) {
  return og_compile_ex(layers, n_layers, precision, 0);
}

og_program* og_compile_ex(const og_layer* layers, int32_t n_layers, int32_t precision, int32_t weight_quant) {
  int32_t m = 0;
  og_flayer* f = og_fold(layers, n_layers, &m);
  og_program* p = (og_program*)calloc(1, sizeof(og_program));
  p->precision = precision; p->original_layers = n_layers;
  p->ops = (og_op*)calloc((size_t)(m > 0 ? m : 1), sizeof(og_op));
  int32_t nops = 0;
  for (int32_t i = 0; i < m; ++i) {
    og_flayer* l = &f[i];
    int32_t next_act = (i + 1 < m && f[i + 1].kind == OG_LAYER_ACTIVATION);
    og_op* op = &p->ops[nops];
    memset(op, 0, sizeof(*op));
    if (l->kind == OG_LAYER_LINEAR || l->kind == OG_LAYER_CONV2D || l->kind == OG_LAYER_SHORTCUT_CONV2D) {
      /* a shortcut conv works on the saved block input: an Activation after it belongs
       * to the main path, so it is not fused */
      if (l->kind == OG_LAYER_SHORTCUT_CONV2D) next_act = 0;
      op->kind = l->kind;
      op->act = next_act ? f[i + 1].act : OG_ACT_NONE;
      op->act_param = next_act ? f[i + 1].param : 0.0f;
      int64_t wl = l->w_len;
      op->wq = (int8_t*)malloc((size_t)(wl > 0 ? wl : 1)); op->wq_len = wl;
      if (l->kind == OG_LAYER_LINEAR) {
        op->in_features = l->in_f; op->out_features = l->out_f;
        float* wt = (float*)malloc(sizeof(float) * (size_t)(wl > 0 ? wl : 1));
        og_transpose2d(l->w, l->in_f, l->out_f, wt);       /* npu.rs:208: [in,out] -> [out,in] */
        if (weight_quant) og_quantize_rows_per_channel(op, wt, l->out_f, l->in_f);
        else op->w_scale = og_quantize_into(wt, wl, op->wq);  /* npu.rs:209: per-tensor */
        op->wh = wt; op->wh_len = wl;                      /* npu.rs:210: round_fp16 of w_t */
        for (int64_t j = 0; j < wl; ++j) op->wh[j] = og_round_fp16(op->wh[j]);
      } else {
        op->in_channels = l->in_c; op->out_channels = l->out_c; op->kernel = l->k;
        op->stride = l->stride; op->padding = l->pad;
        if (weight_quant) og_quantize_rows_per_channel(op, l->w, l->out_c, wl / (l->out_c > 0 ? l->out_c : 1));
        else op->w_scale = og_quantize_into(l->w, wl, op->wq);  /* npu.rs:231: [O, C*k*k] per-tensor */
        op->wh = (float*)malloc(sizeof(float) * (size_t)(wl > 0 ? wl : 1)); op->wh_len = wl;
        for (int64_t j = 0; j < wl; ++j) op->wh[j] = og_round_fp16(l->w[j]);  /* npu.rs:232 */
      }
      op->bias = (float*)malloc(sizeof(float) * (size_t)(l->b_len > 0 ? l->b_len : 1));
      memcpy(op->bias, l->b, sizeof(float) * (size_t)l->b_len); op->bias_len = l->b_len;
      p->fp32_bytes += (l->w_len + l->b_len) * 4;
      const int64_t n_scales = weight_quant ? (l->kind == OG_LAYER_LINEAR ? l->out_f : l->out_c) : 1;
      p->npu_bytes += precision == OG_PREC_INT8 ? (wl + 4 * n_scales) + l->b_len * 4 : l->w_len * 2 + l->b_len * 2;
      if (next_act) ++i;
    } else if (l->kind == OG_LAYER_CHANNEL_AFFINE) {
      /* standalone affine -> diagonal FusedLinear (npu.rs:254-270); no byte accounting */
      int64_t c = l->w_len;
      float* w = (float*)calloc((size_t)(c * c > 0 ? c * c : 1), sizeof(float));
      for (int64_t j = 0; j < c; ++j) w[j * c + j] = l->w[j];
      op->kind = OG_LAYER_LINEAR; op->in_features = (int32_t)c; op->out_features = (int32_t)c;
      op->wq = (int8_t*)malloc((size_t)(c * c > 0 ? c * c : 1)); op->wq_len = c * c;
      if (weight_quant) og_quantize_rows_per_channel(op, w, c, c);
      else op->w_scale = og_quantize_into(w, c * c, op->wq);
      op->wh = w; op->wh_len = c * c;                    /* npu.rs:266: the unrounded diagonal */
      op->bias = (float*)malloc(sizeof(float) * (size_t)(c > 0 ? c : 1));
      memcpy(op->bias, l->b, sizeof(float) * (size_t)c); op->bias_len = c;
      op->act = OG_ACT_NONE;
    } else if (l->kind == OG_LAYER_ATTENTION || l->kind == OG_LAYER_SWIGLU) {
      const int32_t d = l->in_f, hdim = l->out_f;
      op->kind = l->kind; op->in_features = d; op->out_features = hdim;
      if (l->kind == OG_LAYER_ATTENTION) {   /* out_features = heads */
        op->sub = (og_op*)calloc(4, sizeof(og_op)); op->n_sub = 4;
        for (int32_t j = 0; j < 4; ++j)
          og_make_linear(p, &op->sub[j], l->w + (int64_t)j * d * d, d, d, l->b + (int64_t)j * d);
      } else {                               /* out_features = hidden */
        op->sub = (og_op*)calloc(3, sizeof(og_op)); op->n_sub = 3;
        og_make_linear(p, &op->sub[0], l->w, d, hdim, NULL);
        og_make_linear(p, &op->sub[1], l->w + (int64_t)d * hdim, d, hdim, NULL);
        og_make_linear(p, &op->sub[2], l->w + 2 * (int64_t)d * hdim, hdim, d, NULL);
      }
    } else if (l->kind == OG_LAYER_EMBEDDING || l->kind == OG_LAYER_RMSNORM) {
      op->kind = l->kind; op->in_features = l->in_f; op->out_features = l->out_f;
      op->act_param = l->param;
      op->extra = (float*)malloc(sizeof(float) * (size_t)(l->w_len > 0 ? l->w_len : 1));
      memcpy(op->extra, l->w, sizeof(float) * (size_t)l->w_len); op->extra_len = l->w_len;
      p->fp32_bytes += l->w_len * 4;   /* kept in f32 on both paths */
      p->npu_bytes += l->w_len * 4;
    } else {
      op->kind = l->kind; op->kernel = l->k; op->stride = l->stride;
      op->act = l->act; op->act_param = l->param;
    }
    ++nops;
  }
  for (int32_t i = 0; i < m; ++i) { free(f[i].w); free(f[i].b); }
  free(f);
  p->n_ops = nops;
  return p;
}

void og_program_free(og_program* p) {
  if (!p) return;
  for (int32_t i = 0; i < p->n_ops; ++i) {
    for (int32_t j = 0; j < p->ops[i].n_sub; ++j) { free(p->ops[i].sub[j].wq); free(p->ops[i].sub[j].bias); }
    free(p->ops[i].sub); free(p->ops[i].extra); free(p->ops[i].wh);
    free(p->ops[i].wq); free(p->ops[i].bias); free(p->ops[i].w_scale_ch);
  }
  free(p->ops); free(p);
}

/* Rust `{}` Display of an f32 (shortest round-trip repr, no exponent) for LeakyReLU(s). */
static void og_fmt_f32(float v, char* buf, int cap) {
  for (int prec = 1; prec <= 60; ++prec) {
    snprintf(buf, (size_t)cap, "%.*f", prec, (double)v);
    if (strtof(buf, NULL) == v) break;
  }
  /* Rust prints integral floats without a fraction ("1"), others in shortest form */
  char* dot = strchr(buf, '.');
  if (dot) {
    char* end = buf + strlen(buf) - 1;
    while (end > dot && *end == '0') *end-- = 0;
    if (end == dot) *end = 0;
  }
}

static const char* og_act_name(int32_t act, float param, char* tmp, int cap) {
  switch (act) {
    case OG_ACT_NONE: return "none";
    case OG_ACT_RELU: return "ReLU";
    case OG_ACT_SIGMOID: return "Sigmoid";
    case OG_ACT_TANH: return "Tanh";
    case OG_ACT_GELU: return "GELU";
    case OG_ACT_LEAKY_RELU: { char f[64]; og_fmt_f32(param, f, 64); snprintf(tmp, (size_t)cap, "LeakyReLU(%s)", f); return tmp; }
    case OG_ACT_SILU: return "SiLU";
    default: return "?";
  }
}

int32_t og_op_label(const og_op* op, char* buf, int32_t cap) { /* npu.rs:83-104 */
  char t[96];
  const char* an = og_act_name(op->act, op->act_param, t, 96);
  switch (op->kind) {
    case OG_LAYER_LINEAR:
      if (op->act == OG_ACT_NONE) return snprintf(buf, (size_t)cap, "NPU::Gemm(%d->%d)", op->in_features, op->out_features);
      return snprintf(buf, (size_t)cap, "NPU::FusedGemmAct(%d->%d, %s)", op->in_features, op->out_features, an);
    case OG_LAYER_CONV2D:
      if (op->act == OG_ACT_NONE) return snprintf(buf, (size_t)cap, "NPU::Conv2d(%d->%d, k=%d)", op->in_channels, op->out_channels, op->kernel);
      return snprintf(buf, (size_t)cap, "NPU::FusedConv2dAct(%d->%d, k=%d, %s)", op->in_channels, op->out_channels, op->kernel, an);
    case OG_LAYER_MAXPOOL2D: return snprintf(buf, (size_t)cap, "NPU::MaxPool2d(k=%d)", op->kernel);
    case OG_LAYER_FLATTEN: return snprintf(buf, (size_t)cap, "NPU::Flatten");
    case OG_LAYER_ACTIVATION: return snprintf(buf, (size_t)cap, "NPU::Act(%s)", an);
    case OG_LAYER_SOFTMAX: return snprintf(buf, (size_t)cap, "NPU::Softmax");
    case OG_LAYER_RESIDUAL_BEGIN: return snprintf(buf, (size_t)cap, "NPU::ResidualBegin");
    case OG_LAYER_RESIDUAL_END:
      if (op->act == OG_ACT_NONE) return snprintf(buf, (size_t)cap, "NPU::ResidualAdd");
      return snprintf(buf, (size_t)cap, "NPU::ResidualAdd(%s)", an);
    case OG_LAYER_SHORTCUT_CONV2D:
      return snprintf(buf, (size_t)cap, "NPU::ShortcutConv2d(%d->%d, k=%d)", op->in_channels, op->out_channels, op->kernel);
    case OG_LAYER_ADAPTIVE_AVGPOOL2D: return snprintf(buf, (size_t)cap, "NPU::AdaptiveAvgPool2d(%dx%d)", op->kernel, op->stride);
    case OG_LAYER_EMBEDDING: return snprintf(buf, (size_t)cap, "NPU::Embedding(%d, %d)", op->in_features, op->out_features);
    case OG_LAYER_RMSNORM: return snprintf(buf, (size_t)cap, "NPU::RMSNorm(%d)", op->in_features);
    case OG_LAYER_ATTENTION: return snprintf(buf, (size_t)cap, "NPU::Attention(d=%d, heads=%d)", op->in_features, op->out_features);
    case OG_LAYER_SWIGLU: return snprintf(buf, (size_t)cap, "NPU::SwiGLU(%d->%d->%d)", op->in_features, op->out_features, op->in_features);
    default: return snprintf(buf, (size_t)cap, "NPU::?");
  }
}

int32_t og_program_summary(const og_program* p, int32_t raw_count, char* buf, int32_t cap) { /* npu.rs:280-293 */
  float ratio = p->npu_bytes == 0 ? 1.0f : (float)p->fp32_bytes / (float)p->npu_bytes;
  int32_t at = snprintf(buf, (size_t)cap,
      "InferenceSession [provider = NPU (%s), layers: %d -> %d fused ops, weights: %lld B -> %lld B (%.2fx compression)]\n  Pipeline: ",
      p->precision == OG_PREC_INT8 ? "INT8" : "FP16", raw_count, p->n_ops,
      (long long)p->fp32_bytes, (long long)p->npu_bytes, (double)ratio);
  for (int32_t i = 0; i < p->n_ops; ++i) {
    if (i && at < cap) at += snprintf(buf + at, (size_t)(cap - at), " -> ");
    if (at < cap) at += og_op_label(&p->ops[i], buf + at, cap - at);
  }
  return at;
}

/* ------------------------------------------------------------------------ */
/* per-op execution                                                          */
/* ------------------------------------------------------------------------ */
/* Quantization with a scale fixed in advance (the calibration extension): the
 * reference's rounding and clamp (quantize.rs:22) with inv = 1 / scale. */
static void og_quantize_with_scale(const float* v, int64_t n, float scale, int8_t* out) {
  float inv = 1.0f / scale;
  for (int64_t i = 0; i < n; ++i) out[i] = og_q1(v[i], inv);
}

void og_op_linear(const og_op* op, const float* x, int64_t rows, float* y,
                  float* a_scale, int8_t* aq, int32_t* acc, int32_t nthreads) {
  int64_t k = op->in_features, n = op->out_features;
  int8_t* q = aq ? aq : (int8_t*)malloc((size_t)(rows * k > 0 ? rows * k : 1));
  float sa;
  if (op->frozen) {
    sa = op->frozen_scale;
    og_quantize_with_scale(x, rows * k, sa, q);
  } else {
    sa = og_quantize_into(x, rows * k, q);                /* QuantTensor::from_f32 (serial) */
  }
  ((og_op*)op)->seen_scale = sa;
  if (a_scale) *a_scale = sa;
  og_gemm_ctx c = { q, op->wq, op->bias, sa * op->w_scale, k, n, op->act, op->act_param, y, acc, 0,
                    op->w_scale_ch, sa };
  int32_t par = rows * k * n >= 32 * 1024;                /* quantize.rs:104 */
  og_parallel_for(rows, par ? nthreads : 1, og_gemm_rows, &c);
  if (!aq) free(q);
}

void og_op_linear_with_amax(const og_op* op, const float* x, int64_t rows, float amax, float* y,
                            int32_t nthreads) {
  /* FusedLinear with the activation absmax supplied by the caller (a batch shard
   * quantizing with the max over every shard: the multi-device restatement). */
  int64_t k = op->in_features, n = op->out_features;
  float sa = op->frozen ? op->frozen_scale : (amax < 1e-12f ? 1.0f : amax / 127.0f);
  ((og_op*)op)->seen_scale = sa;
  float inv = 1.0f / sa;
  int8_t* q = (int8_t*)malloc((size_t)(rows * k > 0 ? rows * k : 1));
  for (int64_t i = 0; i < rows * k; ++i) q[i] = og_q1(x[i], inv);
  og_gemm_ctx c = { q, op->wq, op->bias, sa * op->w_scale, k, n, op->act, op->act_param, y, NULL, 0,
                    op->w_scale_ch, sa };
  og_parallel_for(rows, rows * k * n >= 32 * 1024 ? nthreads : 1, og_gemm_rows, &c);
  free(q);
}

void og_op_linear_rows(const og_op* op, const float* x, int64_t rows, int64_t r0, int64_t r1,
                       float* y, float* a_scale, int32_t* acc, int32_t nthreads) {
  int64_t k = op->in_features, n = op->out_features;
  float sa = op->frozen ? op->frozen_scale : og_quant_scale(x, rows * k);
  float inv = 1.0f / sa;
  int64_t sub = r1 - r0;
  int8_t* q = (int8_t*)malloc((size_t)(sub * k > 0 ? sub * k : 1));
  for (int64_t i = 0; i < sub * k; ++i) q[i] = og_q1(x[r0 * k + i], inv);
  if (a_scale) *a_scale = sa;
  og_gemm_ctx c = { q, op->wq, op->bias, sa * op->w_scale, k, n, op->act, op->act_param, y, acc, 0,
                    op->w_scale_ch, sa };
  og_parallel_for(sub, nthreads, og_gemm_rows, &c);
  free(q);
}

typedef struct {
  const og_op* op; const float* x; float* y; float* a_scales; int8_t* aq; int32_t* acc;
  int32_t c, h, w, oh, ow;
  int32_t fp16;  /* NpuPrecision::Fp16 arm (npu.rs:351-353) */
} og_conv_ctx;

static void og_conv_images(void* p, int64_t b, int64_t e) { /* npu.rs:331-359 per image */
  og_conv_ctx* c = (og_conv_ctx*)p;
  const og_op* op = c->op;
  int64_t l = (int64_t)c->oh * c->ow, ckk = (int64_t)c->c * op->kernel * op->kernel;
  int64_t O = op->out_channels;
  float* cols = (float*)malloc(sizeof(float) * (size_t)(ckk * l > 0 ? ckk * l : 1));
  float* cols_t = (float*)malloc(sizeof(float) * (size_t)(ckk * l > 0 ? ckk * l : 1));
  int8_t* q = (int8_t*)malloc((size_t)(ckk * l > 0 ? ckk * l : 1));
  float* ylo = (float*)malloc(sizeof(float) * (size_t)(l * O > 0 ? l * O : 1));
  int32_t* alo = c->acc ? (int32_t*)malloc(sizeof(int32_t) * (size_t)(l * O > 0 ? l * O : 1)) : NULL;
  int64_t img_stride = (int64_t)c->c * c->h * c->w;
  for (int64_t im = b; im < e; ++im) {
    const float* img = c->x + im * img_stride;
    og_im2col(img, c->c, c->h, c->w, op->kernel, op->stride, op->padding, c->oh, c->ow, cols);
    og_transpose2d(cols, ckk, l, cols_t);
    if (c->fp16) {                                       /* fp16_gemm_fused_into */
      og_fp16_ctx g = { cols_t, op->wh, op->bias, ckk, O, op->act, op->act_param, ylo };
      og_fp16_rows(&g, 0, l);
      og_transpose2d(ylo, l, O, c->y + im * O * l);
      continue;
    }
    float sa = og_quantize_into(cols_t, ckk * l, q);     /* per-image scale */
    if (c->a_scales) c->a_scales[im] = sa;
    if (c->aq) { float inv = 1.0f / sa; for (int64_t i = 0; i < img_stride; ++i) c->aq[im * img_stride + i] = og_q1(img[i], inv); }
    og_gemm_ctx g = { q, op->wq, op->bias, sa * op->w_scale, ckk, O, op->act, op->act_param, ylo, alo, 0,
                      op->w_scale_ch, sa };
    og_gemm_rows(&g, 0, l);                              /* int8_gemm_fused_serial */
    og_transpose2d(ylo, l, O, c->y + im * O * l);        /* [L,O] -> [O,L] */
    if (alo)
      for (int64_t r = 0; r < l; ++r)
        for (int64_t o = 0; o < O; ++o) c->acc[im * O * l + o * l + r] = alo[r * O + o];
  }
  free(cols); free(cols_t); free(q); free(ylo); free(alo);
}

void og_op_conv2d(const og_op* op, const float* x, int64_t n, int32_t h, int32_t w, float* y,
                  float* a_scales, int8_t* aq, int32_t* acc, int32_t nthreads) {
  og_conv_ctx c = { op, x, y, a_scales, aq, acc, op->in_channels, h, w,
                    (int32_t)og_out_size(h, op->kernel, op->stride, op->padding),
                    (int32_t)og_out_size(w, op->kernel, op->stride, op->padding), 0 };
  int64_t out_stride = (int64_t)op->out_channels * c.oh * c.ow;
  og_parallel_for(n, (n >= 2 && out_stride > 0) ? nthreads : 1, og_conv_images, &c);
}

/* The FP16 arms of FusedLinear (npu.rs:317) and FusedConv2d (npu.rs:351-353, 372-374). */
void og_op_linear_fp16(const og_op* op, const float* x, int64_t rows, float* y, int32_t nthreads) {
  og_fp16_ctx c = { x, op->wh, op->bias, op->in_features, op->out_features, op->act, op->act_param, y };
  og_parallel_for(rows, nthreads, og_fp16_rows, &c);     /* serial in the reference; rows are independent */
}

void og_op_conv2d_fp16(const og_op* op, const float* x, int64_t n, int32_t h, int32_t w, float* y,
                       int32_t nthreads) {
  og_conv_ctx c = { op, x, y, NULL, NULL, NULL, op->in_channels, h, w,
                    (int32_t)og_out_size(h, op->kernel, op->stride, op->padding),
                    (int32_t)og_out_size(w, op->kernel, op->stride, op->padding), 1 };
  int64_t out_stride = (int64_t)op->out_channels * c.oh * c.ow;
  og_parallel_for(n, (n >= 2 && out_stride > 0) ? nthreads : 1, og_conv_images, &c);
}

static int64_t og_now_ns(void) {
  struct timespec ts; clock_gettime(CLOCK_MONOTONIC, &ts);
  return (int64_t)ts.tv_sec * 1000000000ll + ts.tv_nsec;
}

int32_t og_execute(const og_program* p, const float* x, const int64_t* shape, int32_t ndim,
                   float* y, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim,
                   int32_t nthreads, int64_t* op_ns, int64_t* op_macs) {
  int64_t sh[8]; int32_t nd = ndim;
  if (ndim < 1 || ndim > 8) return -1;
  const int32_t fp16 = p->precision == OG_PREC_FP16;
  if (!fp16 && p->precision != OG_PREC_INT8) return -5;
  int64_t len = 1;
  for (int32_t i = 0; i < ndim; ++i) { sh[i] = shape[i]; len *= shape[i]; }
  float* data = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
  memcpy(data, x, sizeof(float) * (size_t)len);
  /* residual blocks (extension): a stack of saved block inputs */
  float* saved[OG_MAX_RESIDUAL]; int64_t saved_sh[OG_MAX_RESIDUAL][8], saved_len[OG_MAX_RESIDUAL];
  int32_t saved_nd[OG_MAX_RESIDUAL], depth = 0;
#define OG_EXEC_FAIL(rc) do { for (int32_t d_ = 0; d_ < depth; ++d_) free(saved[d_]); free(data); return (rc); } while (0)
  for (int32_t oi = 0; oi < p->n_ops; ++oi) {
    const og_op* op = &p->ops[oi];
    int64_t t0 = og_now_ns(), macs = 0;
    float* out = NULL;
    switch (op->kind) {
      case OG_LAYER_LINEAR: {
        int64_t rows = len / op->in_features;
        macs = rows * op->in_features * op->out_features;
        out = (float*)malloc(sizeof(float) * (size_t)(rows * op->out_features > 0 ? rows * op->out_features : 1));
        if (fp16) og_op_linear_fp16(op, data, rows, out, nthreads);
        else og_op_linear(op, data, rows, out, NULL, NULL, NULL, nthreads);
        sh[nd - 1] = op->out_features; len = rows * op->out_features;
        break;
      }
      case OG_LAYER_CONV2D: {
        if (nd != 4 || sh[1] != op->in_channels) OG_EXEC_FAIL(-2);
        int64_t n = sh[0], h = sh[2], w = sh[3];
        int64_t oh = og_out_size(h, op->kernel, op->stride, op->padding);
        int64_t ow = og_out_size(w, op->kernel, op->stride, op->padding);
        if (oh <= 0 || ow <= 0) OG_EXEC_FAIL(-2);
        macs = n * op->out_channels * (int64_t)op->in_channels * op->kernel * op->kernel * oh * ow;
        out = (float*)malloc(sizeof(float) * (size_t)(n * op->out_channels * oh * ow > 0 ? n * op->out_channels * oh * ow : 1));
        if (fp16) og_op_conv2d_fp16(op, data, n, (int32_t)h, (int32_t)w, out, nthreads);
        else og_op_conv2d(op, data, n, (int32_t)h, (int32_t)w, out, NULL, NULL, NULL, nthreads);
        sh[1] = op->out_channels; sh[2] = oh; sh[3] = ow; len = n * op->out_channels * oh * ow;
        break;
      }
      case OG_LAYER_MAXPOOL2D: {
        if (nd != 4) OG_EXEC_FAIL(-2);
        int64_t oh = og_out_size(sh[2], op->kernel, op->stride, 0), ow = og_out_size(sh[3], op->kernel, op->stride, 0);
        if (oh <= 0 || ow <= 0) OG_EXEC_FAIL(-2);
        out = (float*)malloc(sizeof(float) * (size_t)(sh[0] * sh[1] * oh * ow > 0 ? sh[0] * sh[1] * oh * ow : 1));
        og_maxpool2d(data, sh[0], (int32_t)sh[1], (int32_t)sh[2], (int32_t)sh[3], op->kernel, op->stride, out, nthreads);
        sh[2] = oh; sh[3] = ow; len = sh[0] * sh[1] * oh * ow;
        break;
      }
      case OG_LAYER_FLATTEN: {
        int64_t rest = 1;
        for (int32_t i = 1; i < nd; ++i) rest *= sh[i];
        sh[1] = rest; nd = 2;
        break;
      }
      case OG_LAYER_ACTIVATION:
        og_activation(data, len, op->act, op->act_param, data);
        break;
      case OG_LAYER_SOFTMAX: {
        int64_t last = sh[nd - 1];
        out = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        og_softmax(data, last ? len / last : 0, last, out);
        break;
      }
      case OG_LAYER_RESIDUAL_BEGIN: {
        if (depth >= OG_MAX_RESIDUAL) OG_EXEC_FAIL(-2);
        saved[depth] = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        memcpy(saved[depth], data, sizeof(float) * (size_t)len);
        for (int32_t d = 0; d < nd; ++d) saved_sh[depth][d] = sh[d];
        saved_nd[depth] = nd; saved_len[depth] = len;
        ++depth;
        break;
      }
      case OG_LAYER_SHORTCUT_CONV2D: {  /* the conv of the a-10 semantics, on the saved input */
        if (depth < 1) OG_EXEC_FAIL(-2);
        int64_t* ss = saved_sh[depth - 1];
        if (saved_nd[depth - 1] != 4 || ss[1] != op->in_channels) OG_EXEC_FAIL(-2);
        int64_t n = ss[0], h = ss[2], w = ss[3];
        int64_t oh = og_out_size(h, op->kernel, op->stride, op->padding);
        int64_t ow = og_out_size(w, op->kernel, op->stride, op->padding);
        if (oh <= 0 || ow <= 0) OG_EXEC_FAIL(-2);
        macs = n * op->out_channels * (int64_t)op->in_channels * op->kernel * op->kernel * oh * ow;
        int64_t olen = n * op->out_channels * oh * ow;
        float* so = (float*)malloc(sizeof(float) * (size_t)(olen > 0 ? olen : 1));
        if (fp16) og_op_conv2d_fp16(op, saved[depth - 1], n, (int32_t)h, (int32_t)w, so, nthreads);
        else og_op_conv2d(op, saved[depth - 1], n, (int32_t)h, (int32_t)w, so, NULL, NULL, NULL, nthreads);
        free(saved[depth - 1]);
        saved[depth - 1] = so;
        ss[1] = op->out_channels; ss[2] = oh; ss[3] = ow; saved_len[depth - 1] = olen;
        break;
      }
      case OG_LAYER_RESIDUAL_END: {
        if (depth < 1) OG_EXEC_FAIL(-2);
        if (saved_nd[depth - 1] != nd || saved_len[depth - 1] != len) OG_EXEC_FAIL(-2);
        for (int32_t d = 0; d < nd; ++d)
          if (saved_sh[depth - 1][d] != sh[d]) OG_EXEC_FAIL(-2);
        og_residual_add(data, saved[depth - 1], len, op->act, op->act_param, data);
        --depth;
        free(saved[depth]);
        break;
      }
      case OG_LAYER_ADAPTIVE_AVGPOOL2D: {
        if (nd != 4 || op->kernel <= 0 || op->stride <= 0 || sh[2] <= 0 || sh[3] <= 0) OG_EXEC_FAIL(-2);
        int64_t olen = sh[0] * sh[1] * op->kernel * op->stride;
        out = (float*)malloc(sizeof(float) * (size_t)(olen > 0 ? olen : 1));
        og_adaptive_avgpool2d(data, sh[0], (int32_t)sh[1], (int32_t)sh[2], (int32_t)sh[3], op->kernel, op->stride, out);
        sh[2] = op->kernel; sh[3] = op->stride; len = olen;
        break;
      }
      case OG_LAYER_EMBEDDING: {
        if (nd >= 8) OG_EXEC_FAIL(-2);
        int64_t olen = len * op->out_features;
        out = (float*)malloc(sizeof(float) * (size_t)(olen > 0 ? olen : 1));
        if (og_embedding(op, data, len, out) != 0) { free(out); OG_EXEC_FAIL(-6); }
        sh[nd++] = op->out_features; len = olen;
        break;
      }
      case OG_LAYER_RMSNORM: {
        if (sh[nd - 1] != op->in_features) OG_EXEC_FAIL(-2);
        out = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        og_rmsnorm(op, data, len / op->in_features, out);
        break;
      }
      case OG_LAYER_ATTENTION: {
        if (fp16) OG_EXEC_FAIL(-5);  /* extension blocks: INT8 Linears only */
        if (nd != 3 || sh[2] != op->in_features || op->out_features <= 0 || op->in_features % op->out_features)
          OG_EXEC_FAIL(-2);
        const int64_t t = sh[1], dh = op->in_features / op->out_features;
        macs = 4 * sh[0] * t * (int64_t)op->in_features * op->in_features;   /* INT8 projections */
        (void)dh;
        out = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        if (len) og_attention(op, data, sh[0], t, out, nthreads);
        break;
      }
      case OG_LAYER_SWIGLU: {
        if (fp16) OG_EXEC_FAIL(-5);  /* extension blocks: INT8 Linears only */
        if (sh[nd - 1] != op->in_features) OG_EXEC_FAIL(-2);
        const int64_t rows = len / op->in_features;
        macs = 3 * rows * (int64_t)op->in_features * op->out_features;
        out = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        if (len) og_swiglu(op, data, rows, out, nthreads);
        break;
      }
      default: OG_EXEC_FAIL(-3);
    }
    if (out) { free(data); data = out; }
    if (op_ns) op_ns[oi] = og_now_ns() - t0;
    if (op_macs) op_macs[oi] = macs;
  }
  if (depth != 0) OG_EXEC_FAIL(-2);  /* an unclosed residual block */
  if (len > y_cap) OG_EXEC_FAIL(-4);
  memcpy(y, data, sizeof(float) * (size_t)len);
  for (int32_t i = 0; i < nd; ++i) y_shape[i] = sh[i];
  *y_ndim = nd;
  free(data);
  return 0;
}
#undef OG_EXEC_FAIL

/* ------------------------------------------------------------------------ */
/* f32 ExecutionProvider::Cpu (run_standard, mod.rs:260-331)                */
/* ------------------------------------------------------------------------ */
int32_t og_run_standard(const og_layer* layers, int32_t n_layers, const float* x, const int64_t* shape,
                        int32_t ndim, float* y, int64_t y_cap, int64_t* y_shape, int32_t* y_ndim) {
  if (ndim < 1 || ndim > 8) return -1;
  int32_t m = 0;
  og_flayer* f = og_fold(layers, n_layers, &m);          /* from_layers folds for Cpu (mod.rs:163-166) */
  int64_t sh[8], len = 1; int32_t nd = ndim;
  for (int32_t i = 0; i < ndim; ++i) { sh[i] = shape[i]; len *= shape[i]; }
  float* data = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
  memcpy(data, x, sizeof(float) * (size_t)len);
  int32_t rc = 0;
  for (int32_t li = 0; li < m && rc == 0; ++li) {
    const og_flayer* l = &f[li];
    float* out = NULL;
    switch (l->kind) {
      case OG_LAYER_LINEAR: {                               /* be.matmul(data, W[in,out]) then += bias */
        if (sh[nd - 1] != l->in_f) { rc = -2; break; }
        const int64_t rows = len / l->in_f;
        out = (float*)malloc(sizeof(float) * (size_t)(rows * l->out_f > 0 ? rows * l->out_f : 1));
        og_bmm_fma(data, l->w, 1, rows, l->in_f, l->out_f, out);
        for (int64_t r = 0; r < rows; ++r)
          for (int64_t c = 0; c < l->out_f; ++c) out[r * l->out_f + c] += l->b[c];
        sh[nd - 1] = l->out_f; len = rows * l->out_f;
        break;
      }
      case OG_LAYER_CONV2D: {                               /* conv2d_forward (kernels.rs:218-263) + bias */
        if (nd != 4 || sh[1] != l->in_c) { rc = -2; break; }
        const int64_t n = sh[0], h = sh[2], w = sh[3];
        const int64_t oh = og_out_size(h, l->k, l->stride, l->pad), ow = og_out_size(w, l->k, l->stride, l->pad);
        if (oh <= 0 || ow <= 0) { rc = -2; break; }
        const int64_t L = oh * ow, ckk = (int64_t)l->in_c * l->k * l->k, O = l->out_c;
        out = (float*)malloc(sizeof(float) * (size_t)(n * O * L > 0 ? n * O * L : 1));
        float* cols = (float*)malloc(sizeof(float) * (size_t)(ckk * L > 0 ? ckk * L : 1));
        for (int64_t b = 0; b < n; ++b) {
          og_im2col(data + b * l->in_c * h * w, l->in_c, (int32_t)h, (int32_t)w, l->k, l->stride, l->pad,
                    (int32_t)oh, (int32_t)ow, cols);
          og_bmm_fma(l->w, cols, 1, O, ckk, L, out + b * O * L);   /* W[O, ckk] @ cols[ckk, L] */
          for (int64_t o = 0; o < O; ++o)
            for (int64_t p = 0; p < L; ++p) out[(b * O + o) * L + p] += l->b[o];
        }
        free(cols);
        sh[1] = O; sh[2] = oh; sh[3] = ow; len = n * O * L;
        break;
      }
      case OG_LAYER_CHANNEL_AFFINE: {                       /* v * scale + shift over dim 1 */
        const int64_t c = l->w_len;
        if (nd < 2 || sh[1] != c) { rc = -2; break; }
        int64_t inner = 1;
        for (int32_t d = 2; d < nd; ++d) inner *= sh[d];
        for (int64_t nn = 0; nn < sh[0]; ++nn)
          for (int64_t ch = 0; ch < c; ++ch)
            for (int64_t i = 0; i < inner; ++i) {
              float* v = &data[(nn * c + ch) * inner + i];
              const float t = *v * l->w[ch];
              *v = t + l->b[ch];
            }
        break;
      }
      case OG_LAYER_MAXPOOL2D: {
        if (nd != 4) { rc = -2; break; }
        const int64_t oh = og_out_size(sh[2], l->k, l->stride, 0), ow = og_out_size(sh[3], l->k, l->stride, 0);
        if (oh <= 0 || ow <= 0) { rc = -2; break; }
        out = (float*)malloc(sizeof(float) * (size_t)(sh[0] * sh[1] * oh * ow > 0 ? sh[0] * sh[1] * oh * ow : 1));
        og_maxpool2d(data, sh[0], (int32_t)sh[1], (int32_t)sh[2], (int32_t)sh[3], l->k, l->stride, out, 1);
        sh[2] = oh; sh[3] = ow; len = sh[0] * sh[1] * oh * ow;
        break;
      }
      case OG_LAYER_FLATTEN: {
        int64_t rest = 1;
        for (int32_t d = 1; d < nd; ++d) rest *= sh[d];
        sh[1] = rest; nd = 2;
        break;
      }
      case OG_LAYER_ACTIVATION:
        og_activation(data, len, l->act, l->param, data);
        break;
      case OG_LAYER_SOFTMAX: {
        const int64_t last = sh[nd - 1];
        out = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
        og_softmax(data, last ? len / last : 0, last, out);
        break;
      }
      default:
        rc = -5;
    }
    if (out) { free(data); data = out; }
  }
  if (rc == 0 && len > y_cap) rc = -3;
  if (rc == 0) {
    memcpy(y, data, sizeof(float) * (size_t)len);
    for (int32_t d = 0; d < nd; ++d) y_shape[d] = sh[d];
    *y_ndim = nd;
  }
  free(data);
  for (int32_t i = 0; i < m; ++i) { free(f[i].w); free(f[i].b); }
  free(f);
  return rc;
}
