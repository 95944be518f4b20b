/*
 * CPU oracle (float64) for the web-engine B200 hot path. TEST INFRASTRUCTURE ONLY:
 * linked by tests, the smoke check and the bench's CPU-baseline leg, never by the product.
 * Each function names the reference file:line it restates; see oracle.h.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------- decoders: src/weights/fp8.ts ---------------- */

/* src/weights/fp8.ts:4-11: bias 7, no infinity, 0x7f/0xff are NaN, max 448. */
double or_e4m3(uint8_t b) {
  double sign = (b & 0x80) ? -1.0 : 1.0;
  int exp = (b >> 3) & 0xf, man = b & 7;
  if (exp == 0xf && man == 7) return NAN;
  if (exp == 0) return sign * (man / 8.0) * ldexp(1.0, -6);
  return sign * (1.0 + man / 8.0) * ldexp(1.0, exp - 7);
}

/* src/weights/fp8.ts:14-21 */
double or_e5m2(uint8_t b) {
  double sign = (b & 0x80) ? -1.0 : 1.0;
  int exp = (b >> 2) & 0x1f, man = b & 3;
  if (exp == 0x1f) return man ? NAN : sign * INFINITY;
  if (exp == 0) return sign * (man / 4.0) * ldexp(1.0, -14);
  return sign * (1.0 + man / 4.0) * ldexp(1.0, exp - 15);
}

/* src/weights/fp8.ts:23-29 */
double or_f16(uint16_t bits) {
  double sign = (bits & 0x8000) ? -1.0 : 1.0;
  int exp = (bits >> 10) & 0x1f, man = bits & 0x3ff;
  if (exp == 0x1f) return man ? NAN : sign * INFINITY;
  if (exp == 0) return sign * (man / 1024.0) * ldexp(1.0, -14);
  return sign * (1.0 + man / 1024.0) * ldexp(1.0, exp - 15);
}

static float f32_from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t bits_from_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* src/weights/fp8.ts:43-44: bf16 is the top half of an f32 */
float or_bf16_to_f32(uint16_t bits) { return f32_from_bits((uint32_t)bits << 16); }

uint16_t or_f32_to_bf16(float v) {
  uint32_t u = bits_from_f32(v);
  if ((u & 0x7fffffff) > 0x7f800000) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
  uint32_t rounding = 0x7fff + ((u >> 16) & 1);
  return (uint16_t)((u + rounding) >> 16);
}

uint16_t or_f32_to_f16(float v) {
  /* exact double arithmetic: scale into the f16 grid and round half to even with rint() */
  double a = fabs((double)v);
  uint16_t sign = signbit(v) ? 0x8000 : 0;
  if (isnan(v)) return 0x7e00;
  if (a == 0) return sign;
  int e;
  frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) -> leading bit at 2^(e-1) */
  int E = e - 1;
  if (E < -14) { /* subnormal: spacing 2^-24 */
    double m = rint(a * ldexp(1.0, 24));
    if (m >= 1024) return sign | 0x0400; /* rounds up to the smallest normal */
    return sign | (uint16_t)m;
  }
  double m = rint(a * ldexp(1.0, 10 - E)); /* in [1024, 2048] */
  if (m >= 2048) {
    m /= 2;
    E += 1;
  }
  if (E > 15) return sign | 0x7c00; /* overflow -> inf */
  return sign | (uint16_t)((E + 15) << 10) | (uint16_t)((long)m - 1024);
}

uint8_t or_f32_to_e4m3(float v) {
  if (isnan(v)) return 0x7f;
  uint8_t sign = signbit(v) ? 0x80 : 0;
  double a = fabs((double)v);
  if (a == 0) return sign;
  if (a >= 448.0) return sign | 0x7e; /* saturate (e4m3fn has no infinity) */
  int e;
  frexp(a, &e);
  int E = e - 1;
  if (E < -6) { /* subnormal: m * 2^-9, m in 0..8 */
    double m = rint(a * ldexp(1.0, 9));
    if (m >= 8) return sign | 0x08;
    return sign | (uint8_t)m;
  }
  double m = rint(a * ldexp(1.0, 3 - E)); /* in [8, 16] */
  if (m >= 16) {
    m /= 2;
    E += 1;
  }
  if (E > 8 || (E == 8 && m > 14)) return sign | 0x7e; /* > 448 after rounding: saturate */
  return sign | (uint8_t)((E + 7) << 3) | (uint8_t)((long)m - 8);
}

/* src/weights/fp8.ts:37-53 */
long or_to_float32(int dtype, const uint8_t* bytes, size_t nbytes, float* out) {
  size_t i;
  switch (dtype) {
    case 0:
      memcpy(out, bytes, nbytes / 4 * 4);
      return (long)(nbytes / 4);
    case 1:
      for (i = 0; i < nbytes / 2; i++) out[i] = or_bf16_to_f32((uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8)));
      return (long)(nbytes / 2);
    case 2:
      for (i = 0; i < nbytes / 2; i++) out[i] = (float)or_f16((uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8)));
      return (long)(nbytes / 2);
    case 3:
      for (i = 0; i < nbytes; i++) out[i] = (float)or_e4m3(bytes[i]);
      return (long)nbytes;
    case 4:
      for (i = 0; i < nbytes; i++) out[i] = (float)or_e5m2(bytes[i]);
      return (long)nbytes;
    default:
      return -1;
  }
}

/* ---------------- noise: src/model/noise.ts ---------------- */

#define MT_N 624
/* src/model/noise.ts:16-21 (torch keeps the low 32 bits of the seed) */
void or_mt_seed(or_mt19937* mt, uint64_t seed) {
  mt->state[0] = (uint32_t)seed;
  for (int i = 1; i < MT_N; i++)
    mt->state[i] = 1812433253u * (mt->state[i - 1] ^ (mt->state[i - 1] >> 30)) + (uint32_t)i;
  mt->index = MT_N;
}

/* src/model/noise.ts:34-41 */
static void mt_twist(or_mt19937* mt) {
  uint32_t* s = mt->state;
  for (int i = 0; i < MT_N; i++) {
    uint32_t y = (s[i] & 0x80000000u) | (s[(i + 1) % MT_N] & 0x7fffffffu);
    s[i] = s[(i + 397) % MT_N] ^ (y >> 1) ^ ((y & 1) ? 0x9908b0dfu : 0u);
  }
  mt->index = 0;
}

/* src/model/noise.ts:24-32 */
uint32_t or_mt_next(or_mt19937* mt) {
  if (mt->index >= MT_N) mt_twist(mt);
  uint32_t y = mt->state[mt->index++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

/* src/model/noise.ts:48: low 24 bits of one draw */
static float uniform24(or_mt19937* mt) { return (float)((or_mt_next(mt) & 0xffffff) * ldexp(1.0, -24)); }
/* src/model/noise.ts:51: 53 bits of two draws */
static double uniform53(or_mt19937* mt) {
  double hi = (double)(or_mt_next(mt) & 0x1fffff);
  double lo = (double)or_mt_next(mt);
  return (hi * 4294967296.0 + lo) * ldexp(1.0, -53);
}

/* src/model/noise.ts:54-62: Box-Muller on 16 values, pairs (j, j+8), float math */
static void fill16(float* d) {
  const float two_pi = (float)(2 * M_PI);
  for (int j = 0; j < 8; j++) {
    float u1 = (float)(1.0 - (double)d[j]);
    float radius = (float)sqrt((double)(float)(-2.0 * (double)(float)log((double)u1)));
    float theta = (float)((double)two_pi * (double)d[j + 8]);
    d[j] = (float)((double)radius * (double)(float)cos((double)theta));
    d[j + 8] = (float)((double)radius * (double)(float)sin((double)theta));
  }
}

/* src/model/noise.ts:65-84 */
void or_torch_randn(size_t n, uint64_t seed, float* out) {
  or_mt19937 mt;
  or_mt_seed(&mt, seed);
  if (n < 16) {
    for (size_t i = 0; i < n; i += 2) {
      double u1 = uniform53(&mt), u2 = uniform53(&mt);
      double r = sqrt(-2 * log1p(-u2)), theta = 2 * M_PI * u1;
      out[i] = (float)(r * cos(theta));
      if (i + 1 < n) out[i + 1] = (float)(r * sin(theta));
    }
    return;
  }
  for (size_t i = 0; i < n; i++) out[i] = uniform24(&mt);
  for (size_t i = 0; i + 16 <= n; i += 16) fill16(out + i);
  if (n % 16) {
    for (size_t i = n - 16; i < n; i++) out[i] = uniform24(&mt);
    fill16(out + n - 16);
  }
}

/* tests/gpu/matmul.test.ts:10-12 */
double or_lcg_next(uint32_t* seed) {
  *seed = *seed * 1664525u + 1013904223u;
  return *seed / 4294967296.0;
}

/* ---------------- matmul: tests/gpu/matmul.test.ts:26-35, src/kernels/matmul.ts ---------------- */

static inline double w_value(int fmt, const void* w, const uint16_t* gscale, long k_total, long row, long idx,
                             long n_i, long k_i) {
  switch (fmt) {
    case OR_W_F32:
      return ((const float*)w)[idx];
    case OR_W_BF16:
      return or_bf16_to_f32(((const uint16_t*)w)[idx]);
    case OR_W_FP8:
      return or_e4m3(((const uint8_t*)w)[idx]);
    default:
      (void)row;
      return or_int4_operand((const uint8_t*)w, gscale, k_total, n_i, k_i);
  }
}

static void matmul_rows(const float* x, int fmt, const void* w, double scale, const float* chan_scale,
                        const uint16_t* gscale, const or_mm_shape* s, double* y, long r0, long r1) {
  long m = s->m, n = s->n, k = s->k;
  long xs = s->x_stride ? s->x_stride : k, ws = s->w_stride ? s->w_stride : k, ys = s->y_stride ? s->y_stride : n;
  long split = s->k_split > 1 ? s->k_split : 1;
  /* slice length: ceil(K / split) rounded up to the 16-wide K step (src/kernels/matmul.ts:155-159) */
  long kc = ((k + split - 1) / split + 15) / 16 * 16;
  for (long z = 0; z < split; z++) {
    long kb = split > 1 ? z * kc : 0, ke = split > 1 ? (kb + kc < k ? kb + kc : k) : k;
    for (long i = r0; i < r1; i++)
      for (long j = 0; j < n; j++) {
        double acc = 0;
        for (long t = kb; t < ke; t++) {
          double xv = x[s->x_offset + i * xs + t];
          double wv = w_value(fmt, w, gscale, k, j, s->w_offset + j * ws + t, j, t);
          acc += xv * wv;
        }
        double sc = chan_scale ? chan_scale[j] : scale;
        double* out = &y[s->y_offset + (z * m + i) * ys + j];
        *out = s->accumulate ? *out + acc * sc : acc * sc;
      }
  }
  (void)m;
}

void or_matmul(const float* x, int fmt, const void* w, double scale, const float* chan_scale, const uint16_t* gscale,
               const or_mm_shape* s, double* y) {
  matmul_rows(x, fmt, w, scale, chan_scale, gscale, s, y, 0, s->m);
}

void or_matmul_mt(const float* x, int fmt, const void* w, double scale, const float* chan_scale,
                  const uint16_t* gscale, const or_mm_shape* s, double* y, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
  for (long i = 0; i < s->m; i++) matmul_rows(x, fmt, w, scale, chan_scale, gscale, s, y, i, i + 1);
  (void)threads;
}

/* src/model/ops.ts:38-45 */
long or_ksplit_for(long m, long n, long k) {
  const long TILE = 128, BUSY = 256, MIN_SLICE = 256;
  long tiles = ((m + TILE - 1) / TILE) * ((n + TILE - 1) / TILE);
  long want = (BUSY + tiles - 1) / tiles, cap = k / MIN_SLICE;
  long v = want < cap ? want : cap;
  return v > 1 ? v : 1;
}

double or_rel_error(const float* a, const double* b, size_t n) {
  double err = 0, mx = 0;
  for (size_t i = 0; i < n; i++) {
    double d = fabs((double)a[i] - b[i]);
    if (d > err || isnan(d)) err = isnan(d) ? INFINITY : d;
    if (fabs(b[i]) > mx) mx = fabs(b[i]);
  }
  return err / mx;
}

void or_compare(const float* a, const double* b, size_t n, double* cosine, double* max_error,
                double* relative_error) {
  double dot = 0, a2 = 0, b2 = 0, mx = 0, e2 = 0;
  for (size_t i = 0; i < n; i++) {
    double x = a[i], r = b[i], d = x - r;
    dot += x * r;
    a2 += x * x;
    b2 += r * r;
    if (fabs(d) > mx || isnan(d)) mx = isnan(d) ? INFINITY : fabs(d);
    e2 += d * d;
  }
  *cosine = dot / sqrt(a2 * b2);
  *max_error = mx;
  *relative_error = sqrt(e2 / b2);
}

/* ---------------- quantisers (this build's conventions) ---------------- */

void or_quant_fp8_channel(const float* w, long n, long k, uint8_t* q, float* scales) {
  for (long j = 0; j < n; j++) {
    float amax = 0;
    for (long t = 0; t < k; t++) amax = fmaxf(amax, fabsf(w[j * k + t]));
    float s = amax > 0 ? amax / 448.0f : 1.0f;
    scales[j] = s;
    for (long t = 0; t < k; t++) q[j * k + t] = or_f32_to_e4m3(w[j * k + t] / s);
  }
}

float or_quant_fp8_tensor(const float* w, long n, long k, uint8_t* q) {
  float amax = 0;
  for (long i = 0; i < n * k; i++) amax = fmaxf(amax, fabsf(w[i]));
  float s = amax > 0 ? amax / 448.0f : 1.0f;
  for (long i = 0; i < n * k; i++) q[i] = or_f32_to_e4m3(w[i] / s);
  return s;
}

void or_quant_int4_g64(const float* w, long n, long k, uint8_t* packed, uint16_t* scales) {
  long groups = k / 64;
  memset(packed, 0, (size_t)(n * k / 2));
  for (long j = 0; j < n; j++)
    for (long g = 0; g < groups; g++) {
      float amax = 0;
      for (long t = 0; t < 64; t++) amax = fmaxf(amax, fabsf(w[j * k + g * 64 + t]));
      uint16_t sb = or_f32_to_f16(amax / 7.0f);
      float s = (float)or_f16(sb);
      scales[j * groups + g] = sb;
      for (long t = 0; t < 64; t++) {
        long kk = g * 64 + t;
        int q = 0;
        if (s != 0) {
          float r = rintf(w[j * k + kk] / s);
          q = r < -8 ? -8 : (r > 7 ? 7 : (int)r);
        }
        uint8_t nib = (uint8_t)(q & 0xf);
        packed[(j * k + kk) / 2] |= (kk & 1) ? (uint8_t)(nib << 4) : nib;
      }
    }
}

float or_int4_operand(const uint8_t* packed, const uint16_t* scales, long k, long n_i, long k_i) {
  uint8_t byte = packed[(n_i * k + k_i) / 2];
  int nib = (k_i & 1) ? (byte >> 4) : (byte & 0xf);
  int q = nib >= 8 ? nib - 16 : nib;
  float s = (float)or_f16(scales[n_i * (k / 64) + k_i / 64]);
  return or_bf16_to_f32(or_f32_to_bf16((float)q * s));
}

void or_act_split(const float* x, long k, int terms, uint8_t* hi, uint8_t* lo, int* e_out) {
  float amax = 0;
  for (long t = 0; t < k; t++) amax = fmaxf(amax, fabsf(x[t]));
  int e = 0;
  if (amax > 0) {
    /* smallest e with amax * 2^-e <= 448 */
    int fe;
    frexp((double)amax / 448.0, &fe); /* amax/448 = f 2^fe, f in [0.5,1) */
    e = fe;
    while (e > -200 && ldexp((double)amax, -(e - 1)) <= 448.0) e--;
    while (ldexp((double)amax, -e) > 448.0) e++;
  }
  *e_out = e;
  for (long t = 0; t < k; t++) {
    float v = (float)ldexp((double)x[t], -e);
    uint8_t h = or_f32_to_e4m3(v);
    hi[t] = h;
    if (terms > 1) lo[t] = or_f32_to_e4m3((float)((double)v - or_e4m3(h)));
  }
}

/* ---------------- RMSNorm: tests/gpu/rmsnorm.test.ts:10-20 ---------------- */
void or_rmsnorm(const float* x, const float* w, const float* scale, const float* shift, long rows, long d, float eps,
                float offset, double* out) {
  for (long r = 0; r < rows; r++) {
    double sum = 0;
    for (long i = 0; i < d; i++) sum += (double)x[r * d + i] * x[r * d + i];
    double inv = 1.0 / sqrt(sum / d + (double)eps);
    for (long i = 0; i < d; i++) {
      double sc = scale ? scale[i] : 0.0, sh = shift ? shift[i] : 0.0;
      out[r * d + i] = x[r * d + i] * inv * ((double)offset + w[i]) * (1.0 + sc) + sh;
    }
  }
}

/* ---------------- RoPE: src/kernels/rope.ts:14-57 ---------------- */
void or_positions(long text, long rows, long cols, long* pos) {
  long t = 0;
  for (long i = 0; i < text; i++, t++) pos[3 * t] = pos[3 * t + 1] = pos[3 * t + 2] = 0;
  for (long i = 0; i < rows * cols; i++, t++) {
    pos[3 * t] = 0;
    pos[3 * t + 1] = i / cols;
    pos[3 * t + 2] = i % cols;
  }
}

long or_rope_tables(const long* pos, long tokens, int naxes, const long* axes, double theta, float* cos_t,
                    float* sin_t) {
  long pairs = 0;
  for (int a = 0; a < naxes; a++) {
    if (axes[a] % 2) return -1;
    pairs += axes[a] / 2;
  }
  if (!cos_t) return pairs;
  for (long t = 0; t < tokens; t++) {
    long pair = 0;
    for (int a = 0; a < naxes; a++) {
      long dim = axes[a];
      for (long j = 0; j < dim / 2; j++, pair++) {
        double angle = (double)pos[t * naxes + a] * pow(theta, -(double)(2 * j) / (double)dim);
        cos_t[t * pairs + pair] = (float)cos(angle);
        sin_t[t * pairs + pair] = (float)sin(angle);
      }
    }
  }
  return pairs;
}

void or_rope(const float* x, long tokens, long heads, long pairs, const float* cos_t, const float* sin_t, int pairing,
             double* out) {
  for (long t = 0; t < tokens; t++)
    for (long h = 0; h < heads; h++)
      for (long j = 0; j < pairs; j++) {
        double c = cos_t[t * pairs + j], s = sin_t[t * pairs + j];
        long base = (t * heads + h) * pairs * 2;
        long ia = pairing ? base + j : base + 2 * j;
        long ib = pairing ? base + j + pairs : base + 2 * j + 1;
        double a = x[ia], b = x[ib];
        out[ia] = a * c - b * s;
        out[ib] = b * c + a * s;
      }
}

/* ---------------- attention: tests/gpu/attention.test.ts:9-31 ---------------- */
void or_attention(const float* q, const float* k, const float* v, long tokens, long heads, long kv_heads, long dim,
                  int causal, double* out) {
  long group = heads / kv_heads;
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
  for (long h = 0; h < heads; h++)
    for (long i = 0; i < tokens; i++) {
      long g = h / group, n = causal ? i + 1 : tokens;
      double* s = (double*)malloc(sizeof(double) * (size_t)n);
      double m = -INFINITY, sum = 0;
      for (long j = 0; j < n; j++) {
        double dot = 0;
        for (long d = 0; d < dim; d++) dot += (double)q[(i * heads + h) * dim + d] * k[(j * kv_heads + g) * dim + d];
        s[j] = dot / sqrt((double)dim);
        if (s[j] > m) m = s[j];
      }
      for (long j = 0; j < n; j++) {
        s[j] = exp(s[j] - m);
        sum += s[j];
      }
      for (long d = 0; d < dim; d++) {
        double o = 0;
        for (long j = 0; j < n; j++) o += (s[j] / sum) * v[(j * kv_heads + g) * dim + d];
        out[(i * heads + h) * dim + d] = o;
      }
      free(s);
    }
}
