// The per-value steps of a block (src/kernels/elementwise.ts:38-84) as standalone bandwidth kernels, and
// RMSNorm fused with the e4m3 activation split that feeds the fp8 tensor-core GEMM.
//
// Standalone ops keep the reference's exact formulas (sigmoid 1 / (1 + exp(-v)), tanh-form GELU written
// with exp and clamped): swiglu silu(a) b, sigmoidGate a sigmoid(b), gatedAdd a + g[i % d] b, addBias
// a + g[i % d], geluTanh, add a + b, silu. Inside a block they are usually fused into the epilogue of
// the matmul that produces one of their inputs instead (we_epilogue).
#include "common.cuh"
#include "kernels.h"

namespace we {

template <int OP>
__device__ __forceinline__ float ew_apply(float a, float b, float g) {
  if constexpr (OP == WE_EW_SWIGLU) return a * sigmoid_ref(a) * b;
  else if constexpr (OP == WE_EW_SIGMOID_GATE) return a * sigmoid_ref(b);
  else if constexpr (OP == WE_EW_GATED_ADD) return a + g * b;
  else if constexpr (OP == WE_EW_ADD_BIAS) return a + g;
  else if constexpr (OP == WE_EW_GELU_TANH) return gelu_tanh_ref(a);
  else if constexpr (OP == WE_EW_ADD) return a + b;
  else return a * sigmoid_ref(a);  // WE_EW_SILU
}

// grid-stride over n values; 8 per step when the pointers allow 16-byte (bf16) / 32-byte (f32) accesses
template <int OP, int DT, int OT>
__global__ void elementwise_kernel(const void* __restrict__ a, const void* __restrict__ b, const float* __restrict__ g,
                                   int64_t n, int64_t d, void* __restrict__ out, int64_t n8) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    float va[8], vb[8], o[8];
    load8<DT>(a, 8 * i, va);
    if (b) load8<DT>(b, 8 * i, vb);
    else
#pragma unroll
      for (int e = 0; e < 8; e++) vb[e] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = ew_apply<OP>(va[e], vb[e], g ? g[(8 * i + e) % d] : 0.f);
    store8<OT>(out, 8 * i, o);
  }
  for (int64_t i = 8 * n8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float vb = b ? load_act<DT>(b, i) : 0.f;
    store_out<OT>(out, i, ew_apply<OP>(load_act<DT>(a, i), vb, g ? g[i % d] : 0.f));
  }
}

template <int OP>
static void ew_dispatch(const void* a, const void* b, const float* g, int64_t n, int64_t d, int dt, void* out, int ot,
                        int sms, cudaStream_t st) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  const bool vec = al(a) && (!b || al(b)) && al(out);
  const int64_t n8 = vec ? n / 8 : 0;
  int64_t grid = (n8 + (n - 8 * n8) + 255) / 256;
  if (grid > (int64_t)sms * 16) grid = (int64_t)sms * 16;
  if (grid < 1) grid = 1;
  if (dt == WE_BF16 && ot == WE_BF16) elementwise_kernel<OP, WE_BF16, WE_BF16><<<(unsigned)grid, 256, 0, st>>>(a, b, g, n, d, out, n8);
  else if (dt == WE_BF16) elementwise_kernel<OP, WE_BF16, WE_F32><<<(unsigned)grid, 256, 0, st>>>(a, b, g, n, d, out, n8);
  else if (ot == WE_BF16) elementwise_kernel<OP, WE_F32, WE_BF16><<<(unsigned)grid, 256, 0, st>>>(a, b, g, n, d, out, n8);
  else elementwise_kernel<OP, WE_F32, WE_F32><<<(unsigned)grid, 256, 0, st>>>(a, b, g, n, d, out, n8);
}

cudaError_t launch_elementwise(int op, const void* a, const void* b, const float* g, int64_t n, int64_t d, int dt,
                               void* out, int ot, int sms, cudaStream_t st) {
  switch (op) {
    case WE_EW_SWIGLU: ew_dispatch<WE_EW_SWIGLU>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_SIGMOID_GATE: ew_dispatch<WE_EW_SIGMOID_GATE>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_GATED_ADD: ew_dispatch<WE_EW_GATED_ADD>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_ADD_BIAS: ew_dispatch<WE_EW_ADD_BIAS>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_GELU_TANH: ew_dispatch<WE_EW_GELU_TANH>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_ADD: ew_dispatch<WE_EW_ADD>(a, b, g, n, d, dt, out, ot, sms, st); break;
    case WE_EW_SILU: ew_dispatch<WE_EW_SILU>(a, b, g, n, d, dt, out, ot, sms, st); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------- RMSNorm + modulation fused with the e4m3 split ----------------
// 8 values (four pairs, already scaled by the row's 2^-e) -> their e4m3 hi (and lo = e4m3(s - hi)) terms, 8 bytes each
template <int TERMS>
__device__ __forceinline__ void split_store8(const float2 (&s)[4], uint8_t* hi, uint8_t* lo) {
  uint32_t h[2], l[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const uint16_t h0 = f32x2_to_e4m3x2(s[2 * j].x, s[2 * j].y), h1 = f32x2_to_e4m3x2(s[2 * j + 1].x, s[2 * j + 1].y);
    h[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
    if (TERMS > 1) {
      const float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
      const float2 r0 = __fadd2_rn(s[2 * j], make_float2(-d0.x, -d0.y));
      const float2 r1 = __fadd2_rn(s[2 * j + 1], make_float2(-d1.x, -d1.y));
      l[j] = (uint32_t)f32x2_to_e4m3x2(r0.x, r0.y) | ((uint32_t)f32x2_to_e4m3x2(r1.x, r1.y) << 16);
    }
  }
  *reinterpret_cast<uint2*>(hi) = make_uint2(h[0], h[1]);
  if (TERMS > 1) *reinterpret_cast<uint2*>(lo) = make_uint2(l[0], l[1]);
}

// CTA-per-row RMSNorm + modulation + bf16 rounding + e4m3 split for rows of 2048..8192 values (d % 8 == 0). NT
// threads; thread t owns the 8-value chunks t, t + NT, ... (CH of them) of every row and keeps its columns'
// modulation in registers for all the rows the CTA strides over, as two factors: (offset + w)(1 + scale), rounded
// once, and the shift, so y = fma(x inv, (offset + w)(1 + scale), shift) (one f32 rounding from the product order
// of rmsnorm.ts:42-46). The rows are staged through shared memory by cp.async, S - 1 rows ahead of the one being
// reduced: each thread copies exactly the chunks it later reads, so the ring needs no barrier, and the loads in
// flight hold no registers. Per row: sum of squares (warp shuffle, then the NT / 32 warps in a fixed order), y
// rounded to bf16, the row's |y| max (warp redux, then the warps), the power-of-two row scale, the e4m3 planes; the
// arithmetic runs two values at a time (packed f32x2). Many values per thread keep the per-row reductions a small
// share of the instructions.
// RES: the row is x + r (f32 residual plus f32 update), written to xo before it is normalised (the residual add of a
// block, fused with the next RMSNorm and split); both inputs are staged.
template <int DT, int TERMS, int NT, int CH, int S, bool RES = false>
__global__ void __launch_bounds__(NT, NT == 192 ? 4 : 512 / NT) norm_split_row_kernel(
    const void* __restrict__ x, const float* __restrict__ w, const float* __restrict__ sc,
    const float* __restrict__ sh, int64_t rows, int64_t d, float eps, float offset, uint8_t* __restrict__ hi,
    uint8_t* __restrict__ lo, float* __restrict__ row_scale, const float* __restrict__ r = nullptr,
    float* __restrict__ xo = nullptr) {
  constexpr int NW = NT / 32;
  constexpr int ES = DT == WE_F32 ? 4 : 2;  // bytes per value of x
  constexpr int XB = 8 * ES;                 // bytes of one 8-value chunk of x
  constexpr int XSTAGE = CH * NT * XB, RSTAGE = CH * NT * 32;
  extern __shared__ __align__(16) uint8_t ring[];  // [S][CH][NT] chunks of x, then (RES) [S][CH][NT] of r
  __shared__ __align__(16) float red[2][NW];
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs (x, r, the modulation) are complete
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int dd = (int)d;
  float2 mw[CH][4], sf[CH][4];  // (offset + w)(1 + scale) and shift of this thread's columns, once per CTA
#pragma unroll
  for (int c = 0; c < CH; c++) {
    const int i = (c * NT + tid) * 8;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const bool live = i < dd;
      const float4 ww = live ? *reinterpret_cast<const float4*>(w + i + 4 * h) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 s4 = live && sc ? *reinterpret_cast<const float4*>(sc + i + 4 * h) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 h4 = live && sh ? *reinterpret_cast<const float4*>(sh + i + 4 * h) : make_float4(0.f, 0.f, 0.f, 0.f);
      mw[c][2 * h] = make_float2((offset + ww.x) * (1.f + s4.x), (offset + ww.y) * (1.f + s4.y));
      mw[c][2 * h + 1] = make_float2((offset + ww.z) * (1.f + s4.z), (offset + ww.w) * (1.f + s4.w));
      sf[c][2 * h] = make_float2(h4.x, h4.y);
      sf[c][2 * h + 1] = make_float2(h4.z, h4.w);
    }
  }
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
  auto issue = [&](int64_t row, int s) {  // this thread's chunks of `row` into stage s (an empty group past the end)
    if (row < rows) {
      const uint8_t* xr = static_cast<const uint8_t*>(x) + row * d * ES;
      const float* rr = RES ? r + row * d : nullptr;
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int i = (c * NT + tid) * 8;
        if (i >= dd) continue;
        const uint32_t xa = ring_s + s * XSTAGE + (c * NT + tid) * XB;
#pragma unroll
        for (int q = 0; q < XB / 16; q++) cp_async16(xa + 16 * q, xr + i * ES + 16 * q);
        if constexpr (RES) {
          const uint32_t ra = ring_s + S * XSTAGE + s * RSTAGE + (c * NT + tid) * 32;
          cp_async16(ra, rr + i);
          cp_async16(ra + 16, rr + i + 4);
        }
      }
    }
    cp_async_commit();
  };
  const int64_t G = gridDim.x;
  int64_t row = blockIdx.x;
#pragma unroll
  for (int s = 0; s < S - 1; s++) issue(row + s * G, s);
  int s = 0, sn = S - 1;  // stage of this row, stage the next issue fills (the one read one row ago)
  for (; row < rows; row += G) {
    issue(row + (S - 1) * G, sn);
    cp_async_wait<S - 1>();  // this row's group has landed
    float2 v[CH][4];
    float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int i = (c * NT + tid) * 8;
#pragma unroll
      for (int j = 0; j < 4; j++) v[c][j] = make_float2(0.f, 0.f);
      if (i >= dd) continue;
      const uint8_t* xs = ring + s * XSTAGE + (c * NT + tid) * XB;
      if constexpr (DT == WE_F32) {
        const float4 a = *reinterpret_cast<const float4*>(xs), b = *reinterpret_cast<const float4*>(xs + 16);
        v[c][0] = make_float2(a.x, a.y); v[c][1] = make_float2(a.z, a.w);
        v[c][2] = make_float2(b.x, b.y); v[c][3] = make_float2(b.z, b.w);
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(xs);
        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; j++) v[c][j] = make_float2(__uint_as_float(u[j] << 16), __uint_as_float(u[j] & 0xffff0000u));
      }
      if constexpr (RES) {
        const uint8_t* rs = ring + S * XSTAGE + s * RSTAGE + (c * NT + tid) * 32;
        const float4 a = *reinterpret_cast<const float4*>(rs), b = *reinterpret_cast<const float4*>(rs + 16);
        v[c][0] = __fadd2_rn(v[c][0], make_float2(a.x, a.y)); v[c][1] = __fadd2_rn(v[c][1], make_float2(a.z, a.w));
        v[c][2] = __fadd2_rn(v[c][2], make_float2(b.x, b.y)); v[c][3] = __fadd2_rn(v[c][3], make_float2(b.z, b.w));
        float* xor_ = xo + row * d + i;
        *reinterpret_cast<float4*>(xor_) = make_float4(v[c][0].x, v[c][0].y, v[c][1].x, v[c][1].y);
        *reinterpret_cast<float4*>(xor_ + 4) = make_float4(v[c][2].x, v[c][2].y, v[c][3].x, v[c][3].y);
      }
#pragma unroll
      for (int j = 0; j < 4; j++) ss2 = __ffma2_rn(v[c][j], v[c][j], ss2);
    }
    s = s + 1 == S ? 0 : s + 1;
    sn = sn + 1 == S ? 0 : sn + 1;
    const float ss = warp_sum(ss2.x + ss2.y);
    if (lane == 0) red[0][wp] = ss;
    __syncthreads();
    float tot = red[0][0];
#pragma unroll
    for (int k = 1; k < NW; k++) tot += red[0][k];
    const float inv = rsqrtf(tot / (float)dd + eps);
    const float2 inv2 = make_float2(inv, inv);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < CH; c++) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 p = __ffma2_rn(__fmul2_rn(v[c][j], inv2), mw[c][j], sf[c][j]);
        const uint32_t b = pack_bf16x2(p.x, p.y);
        v[c][j] = make_float2(__uint_as_float(b << 16), __uint_as_float(b & 0xffff0000u));
        amax = fmaxf(amax, fmaxf(fabsf(v[c][j].x), fabsf(v[c][j].y)));  // chunks past d are 0
      }
    }
    amax = warp_max_abs(amax);
    if (lane == 0) red[1][wp] = amax;
    __syncthreads();
    amax = red[1][0];
#pragma unroll
    for (int k = 1; k < NW; k++) amax = fmaxf(amax, red[1][k]);
    const int e = split_exponent(amax);
    if (tid == 0) row_scale[row] = ldexpf(1.0f, e);
    uint8_t* const hr = hi + row * d;
    uint8_t* const lr = TERMS > 1 ? lo + row * d : nullptr;
    // 2^-e is uniform over the row: one branch per row; the usual case (2^-e a normal float) scales by packed
    // multiplies (exact, as ldexpf), ldexpf only for rows whose scale is outside that range
    const int b = 127 - e;
    if (b >= 1 && b <= 254) {
      const float2 mul2 = make_float2(__int_as_float(b << 23), __int_as_float(b << 23));
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int i = (c * NT + tid) * 8;
        if (i >= dd) continue;
        float2 t[4];
#pragma unroll
        for (int j = 0; j < 4; j++) t[j] = __fmul2_rn(v[c][j], mul2);
        split_store8<TERMS>(t, hr + i, lr + i);
      }
    } else {
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int i = (c * NT + tid) * 8;
        if (i >= dd) continue;
        float2 t[4];
#pragma unroll
        for (int j = 0; j < 4; j++) t[j] = make_float2(ldexpf(v[c][j].x, -e), ldexpf(v[c][j].y, -e));
        split_store8<TERMS>(t, hr + i, lr + i);
      }
    }
    // red[0] was read before the second barrier and red[1] is next written after the next row's first one
  }
  cp_async_wait<0>();  // nothing is left in flight (every row issued was consumed); kept as the exit rule
}

// Bytes of one stage of the row ring: a row of x (and of r).
template <int DT, bool RES, int NT, int CH>
constexpr size_t norm_ring_stage_bytes() {
  return (size_t)CH * NT * (8 * (DT == WE_F32 ? 4 : 2) + (RES ? 32 : 0));
}

// Ring depth and grid, measured at 4608 x 3072 on B200 over thread shapes, ring depths and CTAs per SM: two stages
// (one row ahead) beat three or four in every form; the plain form runs best with every resident CTA (192 threads:
// 17.5 us, 0.76 of measured HBM for f32 rows), the residual form with two CTAs per SM (36.5 us, 0.85; three or four
// per SM 39-45 us). The thread shape sets the order of the sum of squares, so both forms share it and stay
// bit-identical; the ring depth and grid do not change the arithmetic.
template <int DT, int TERMS, int NT, int CH, bool RES>
static cudaError_t launch_norm_split_row(const void* x, const float* w, const float* sc, const float* sh, int64_t rows,
                                         int64_t d, float eps, float offset, uint8_t* hi, uint8_t* lo, float* rs,
                                         const float* r, float* xo, int sms, cudaStream_t st) {
  constexpr int S = 2;
  constexpr size_t smem = S * norm_ring_stage_bytes<DT, RES, NT, CH>();
  auto k = norm_split_row_kernel<DT, TERMS, NT, CH, S, RES>;
  // the ring plus the kernel's static reductions can pass the 48 KB a launch gets without this opt-in
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  unsigned grid = resident_grid(k, NT, sms, rows, smem);
  if (RES && grid > 2u * (unsigned)sms) grid = 2u * (unsigned)sms;
  return launch_pdl(k, dim3(grid), NT, smem, st, x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo);
}

// d % 8 == 0, d <= 8192: 2 chunks of 8 a thread on 128 or 192 threads up to d = 3072 (six warps measured faster at
// d = 3072 than four warps with 3 chunks each, or twelve with one), else 256 threads x up to 4
template <int DT, int TERMS, bool RES>
static cudaError_t norm_split_row(const void* x, const float* w, const float* sc, const float* sh, int64_t rows,
                                  int64_t d, float eps, float offset, uint8_t* hi, uint8_t* lo, float* rs,
                                  const float* r, float* xo, int sms, cudaStream_t st) {
  const int64_t chunks = d / 8;
#define WE_NS(NT, CH) \
  return launch_norm_split_row<DT, TERMS, NT, CH, RES>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo, sms, st)
  if (chunks <= 128 * 2) WE_NS(128, 2);
  if (chunks <= 192 * 2) WE_NS(192, 2);
  if (chunks <= 256 * 3) WE_NS(256, 3);
  if (chunks <= 256 * 4) WE_NS(256, 4);
#undef WE_NS
  return cudaErrorNotSupported;
}

cudaError_t launch_add_norm_split(const float* x, const float* r, float* xo, const float* w, const float* sc,
                                  const float* sh, int64_t rows, int64_t d, float eps, float offset, int terms,
                                  uint8_t* hi, uint8_t* lo, float* rs, int sms, cudaStream_t st) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (d % 8 || d > 8192 || !al(x) || !al(r) || !al(xo) || !al(w) || (sc && !al(sc)) || (sh && !al(sh)) ||
      ((uintptr_t)hi & 7) || (lo && ((uintptr_t)lo & 7)))
    return cudaErrorNotSupported;
  const cudaError_t e = terms > 1 ? norm_split_row<WE_F32, 2, true>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo, sms, st)
                                  : norm_split_row<WE_F32, 1, true>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo, sms, st);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_norm_split(const void* x, int xdt, const float* w, const float* sc, const float* sh, int64_t rows,
                              int64_t d, float eps, float offset, int terms, uint8_t* hi, uint8_t* lo, float* rs,
                              int sms, cudaStream_t st) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (d % 8 || d > 8192 || !al(x) || !al(w) || (sc && !al(sc)) || (sh && !al(sh)) || ((uintptr_t)hi & 7) ||
      (lo && ((uintptr_t)lo & 7)))
    return cudaErrorNotSupported;
  // every width takes the CTA-per-row kernel, so norm + split of x equals the residual form's on x = x1 + dn bit
  // for bit
  cudaError_t e;
  if (xdt == WE_BF16)
    e = terms > 1 ? norm_split_row<WE_BF16, 2, false>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, nullptr, nullptr, sms, st)
                  : norm_split_row<WE_BF16, 1, false>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, nullptr, nullptr, sms, st);
  else
    e = terms > 1 ? norm_split_row<WE_F32, 2, false>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, nullptr, nullptr, sms, st)
                  : norm_split_row<WE_F32, 1, false>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, nullptr, nullptr, sms, st);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace we
