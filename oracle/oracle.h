/*
 * CPU oracle for the web-engine B200 hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker: the tests, the smoke
 * check and the bench's CPU-baseline leg link it. The product path never calls it.
 *
 * It restates, in plain C with float64 arithmetic, the reference's own CPU math for the
 * path (dotstories/web-engine, TypeScript):
 *   - fp8/bf16/f16 decoders ............ src/weights/fp8.ts:4-53
 *   - the float64 matmul reference ..... tests/gpu/matmul.test.ts:26-46, src/kernels/matmul.ts:140-178
 *   - kSplitFor ........................ src/model/ops.ts:42-45
 *   - RMSNorm + modulation ............. tests/gpu/rmsnorm.test.ts:10-20, src/kernels/rmsnorm.ts:42-46
 *   - positions / ropeTables / rotate .. src/kernels/rope.ts:14-57
 *   - compare (cos, maxErr, relErr) .... src/model/compare.ts:2-17
 *   - MT19937 + torch randn ............ src/model/noise.ts:9-84
 * and the conventions this build adds where the reference has none (they have no
 * reference counterpart, so their parity is pinned only by the golden vectors made
 * with torch, see tests/golden/make_golden.py):
 *   - per-output-channel fp8 quantisation (absmax/448, RNE, saturating),
 *   - int4 group-64 quantisation (fp16 absmax/7 scale, RNE, low nibble = even k),
 *   - the two-term e4m3 split of bf16 activations under a power-of-two row scale.
 */
#ifndef WE_ORACLE_H
#define WE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar decoders / encoders ---- */
double or_e4m3(uint8_t b);            /* NaN for 0x7f/0xff (src/weights/fp8.ts:4-11) */
double or_e5m2(uint8_t b);            /* src/weights/fp8.ts:14-21 */
double or_f16(uint16_t bits);         /* src/weights/fp8.ts:23-29 */
float or_bf16_to_f32(uint16_t bits);  /* src/weights/fp8.ts:43-44 (w << 16) */
uint16_t or_f32_to_bf16(float v);     /* round to nearest even (NaN kept quiet) */
uint16_t or_f32_to_f16(float v);      /* round to nearest even, overflow -> inf */
uint8_t or_f32_to_e4m3(float v);      /* round to nearest even, saturate to +-448, NaN -> 0x7f */

/* toFloat32 (src/weights/fp8.ts:37-53): dtype 0=F32 1=BF16 2=F16 3=F8_E4M3 4=F8_E5M2.
   Returns number of values written, or -1 for an unknown dtype. */
long or_to_float32(int dtype, const uint8_t* bytes, size_t nbytes, float* out);

/* ---- noise (src/model/noise.ts) ---- */
typedef struct { uint32_t state[624]; int index; } or_mt19937;
void or_mt_seed(or_mt19937* mt, uint64_t seed);
uint32_t or_mt_next(or_mt19937* mt);
void or_torch_randn(size_t n, uint64_t seed, float* out);

/* ---- the reference tests' LCG: seed = seed*1664525 + 1013904223 (mod 2^32), r = seed / 2^32 ---- */
double or_lcg_next(uint32_t* seed);

/* ---- matmul (weight formats) ---- */
enum { OR_W_F32 = 0, OR_W_BF16 = 1, OR_W_FP8 = 2, OR_W_INT4G64 = 3 };
/*
 * y[m, n] = scale_n * sum_k x[m, k] * W[n, k] in float64, W stored like nn.Linear [N, K].
 * fmt OR_W_FP8: bytes, e4m3. OR_W_BF16: u16 bits. OR_W_F32: floats.
 * OR_W_INT4G64: packed 2 per byte (low nibble = even k, two's complement), group scales
 *   f16 [N, K/64] in `gscale`; the operand is bf16_rne(q * float(s)) (the build's convention).
 * scale_n = chan_scale ? chan_scale[n] : scale.
 * Strides/offsets are in values (like matmulParams, src/kernels/matmul.ts:198-212);
 * y_stride/y_offset index y. k_split > 1: slice z of K (ceil(K/k_split) rounded up to 16,
 * src/kernels/matmul.ts:155-159) goes to partial z of y, [k_split, m, y_stride].
 * accumulate: y += instead of y = (src/kernels/matmul.ts:145).
 */
typedef struct {
  long m, n, k;
  long x_stride, w_stride, y_stride, x_offset, w_offset, y_offset;  /* 0 stride = contiguous */
  long k_split;                                                    /* 0/1 = none */
  int accumulate;
} or_mm_shape;
void or_matmul(const float* x, int fmt, const void* w, double scale, const float* chan_scale,
               const uint16_t* gscale, const or_mm_shape* s, double* y);
/* Same product, OpenMP over rows with `threads` threads (0 = all). CPU baseline timing. */
void or_matmul_mt(const float* x, int fmt, const void* w, double scale, const float* chan_scale,
                  const uint16_t* gscale, const or_mm_shape* s, double* y, int threads);

/* kSplitFor (src/model/ops.ts:42-45), TILE 128, BUSY 256, MIN_SLICE 256 */
long or_ksplit_for(long m, long n, long k);

/* max|a-b| / max|b| (tests/gpu/matmul.test.ts:39-46) */
double or_rel_error(const float* a, const double* b, size_t n);
/* compare (src/model/compare.ts:2-17) */
void or_compare(const float* a, const double* b, size_t n, double* cosine, double* max_error,
                double* relative_error);

/* ---- quantisers (this build's conventions) ---- */
/* per-output-channel: s_n = max_k |W| / 448 (0 -> 1), q = e4m3_rne_sat(W / s_n) */
void or_quant_fp8_channel(const float* w, long n, long k, uint8_t* q, float* scales);
/* per-tensor: s = max |W| / 448 (0 -> 1) */
float or_quant_fp8_tensor(const float* w, long n, long k, uint8_t* q);
/* int4 group 64 along K: s = f16_rne(absmax_g / 7), q = clamp(rint(W / s), -8, 7) (s == 0 -> q = 0).
   packed [N, K/2] bytes (low nibble even k), scales [N, K/64] f16 bits. k % 64 == 0. */
void or_quant_int4_g64(const float* w, long n, long k, uint8_t* packed, uint16_t* scales);
/* bf16 operand of element (n, k) of an int4 g64 weight */
float or_int4_operand(const uint8_t* packed, const uint16_t* scales, long k, long n_i, long k_i);

/* Two-term e4m3 split of one activation row under a power-of-two scale 2^e:
   e = smallest integer with amax / 2^e <= 448 (amax 0 -> e 0); hi = e4m3(x 2^-e),
   lo = e4m3(x 2^-e - hi). Writes e and the bytes; terms = 1 skips lo. */
void or_act_split(const float* x, long k, int terms, uint8_t* hi, uint8_t* lo, int* e);

/* ---- RMSNorm (tests/gpu/rmsnorm.test.ts:10-20) ---- */
void or_rmsnorm(const float* x, const float* w, const float* scale, const float* shift, long rows,
                long d, float eps, float offset, double* out);

/* ---- RoPE (src/kernels/rope.ts) ---- */
/* positions(text, rows, cols) -> [tokens][3] */
void or_positions(long text, long rows, long cols, long* pos);
/* ropeTables: pos [tokens][naxes], axes dims (even) -> cos/sin [tokens, pairs] f32. Returns pairs, -1 if odd. */
long or_rope_tables(const long* pos, long tokens, int naxes, const long* axes, double theta, float* cos_t,
                    float* sin_t);
/* rotate x [tokens, heads, 2*pairs] by the tables. pairing 0 = interleaved, 1 = half. */
void or_rope(const float* x, long tokens, long heads, long pairs, const float* cos_t, const float* sin_t,
             int pairing, double* out);

/* ---- attention (tests/gpu/attention.test.ts:9-31): softmax(q k^T / sqrt(dim)) v per head, GQA kv head
   = floor(h / (heads / kv_heads)); causal: query i sees keys j <= i. q [tokens, heads, dim], k, v
   [tokens, kv_heads, dim] -> out [tokens, heads, dim]. */
void or_attention(const float* q, const float* k, const float* v, long tokens, long heads, long kv_heads, long dim,
                  int causal, double* out);

#ifdef __cplusplus
}
#endif
#endif
