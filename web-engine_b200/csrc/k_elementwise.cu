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
// One warp per row: the normalised, modulated row is rounded to bf16 (the value the unfused path
// would store), then split into hi / lo e4m3 planes under the row's power-of-two scale, exactly as
// quant_act_kernel does on that bf16 row. So the planes equal norm(bf16 out) followed by the split.
template <int DT, int TERMS, int UMAX>
__global__ void __launch_bounds__(128) norm_split_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                         const float* __restrict__ sc, const float* __restrict__ sh,
                                                         int64_t rows, int64_t d, float eps, float offset,
                                                         uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                                         float* __restrict__ row_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 4;
  for (int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); row < rows; row += warps) {
    float v[UMAX][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t i = (int64_t)(c * 32 + lane) * 8;
      if (i < d) {
        load8<DT>(x, row * d + i, v[c]);
        // the summation order of rmsnorm_warp_kernel, so a bf16 row normalises to the same bits
#pragma unroll
        for (int j = 0; j < 4; j++) ss = fmaf(v[c][2 * j], v[c][2 * j], fmaf(v[c][2 * j + 1], v[c][2 * j + 1], ss));
      }
    }
    const float inv = rsqrtf(warp_sum(ss) / (float)d + eps);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t i = (int64_t)(c * 32 + lane) * 8;
      if (i >= d) continue;
      float ww[8], s8[8], h8[8];
      load8f(w, i, ww);
      if (sc) load8f(sc, i, s8); else for (int j = 0; j < 8; j++) s8[j] = 0.f;
      if (sh) load8f(sh, i, h8); else for (int j = 0; j < 8; j++) h8[j] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float y = v[c][j] * inv * (offset + ww[j]) * (1.f + s8[j]) + h8[j];
        v[c][j] = bf16_bits_to_f32(f32_to_bf16_bits(y));
        amax = fmaxf(amax, fabsf(v[c][j]));
      }
    }
    amax = warp_max(amax);
    int e = 0;
    if (amax > 0.f) {
      int E;
      const float f = frexpf(amax, &E);
      e = (2.f * f <= 1.75f) ? E - 9 : E - 8;
    }
    if (lane == 0) row_scale[row] = ldexpf(1.0f, e);
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t i = (int64_t)(c * 32 + lane) * 8;
      if (i >= d) continue;
      float s[8];
#pragma unroll
      for (int j = 0; j < 8; j++) s[j] = ldexpf(v[c][j], -e);
      uint32_t h2[2], l2[2];
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const uint16_t h0 = f32x2_to_e4m3x2(s[4 * j], s[4 * j + 1]);
        const uint16_t h1 = f32x2_to_e4m3x2(s[4 * j + 2], s[4 * j + 3]);
        h2[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        if (TERMS > 1) {
          const float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
          const uint16_t l0 = f32x2_to_e4m3x2(s[4 * j] - d0.x, s[4 * j + 1] - d0.y);
          const uint16_t l1 = f32x2_to_e4m3x2(s[4 * j + 2] - d1.x, s[4 * j + 3] - d1.y);
          l2[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
      }
      *reinterpret_cast<uint2*>(hi + row * d + i) = make_uint2(h2[0], h2[1]);
      if (TERMS > 1) *reinterpret_cast<uint2*>(lo + row * d + i) = make_uint2(l2[0], l2[1]);
    }
  }
}

// The same, one 256-thread CTA per row for rows of 2048+ values: thread t keeps the row's 4-value chunks t,
// t + 256, ... in registers (3 chunks at d = 3072: few registers, many rows in flight per SM, where the warp per
// row form holds a whole row per warp and is latency-bound); the sum of squares and the maximum go through a
// shared-memory reduction over the 8 warps in a fixed order.
template <int DT>
__device__ __forceinline__ void load4(const void* p, int64_t i, float v[4]) {
  if constexpr (DT == WE_F32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i);
    v[0] = __uint_as_float(a.x << 16); v[1] = __uint_as_float(a.x & 0xffff0000u);
    v[2] = __uint_as_float(a.y << 16); v[3] = __uint_as_float(a.y & 0xffff0000u);
  }
}

// RES: the row is x + r (f32 residual plus f32 update), written to xo before it is normalised (the residual add
// of a block, fused with the next RMSNorm and split)
template <int DT, int TERMS, int CH, bool RES = false>
__global__ void __launch_bounds__(256) norm_split_row_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                             const float* __restrict__ sc, const float* __restrict__ sh,
                                                             int64_t rows, int64_t d, float eps, float offset,
                                                             uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                                             float* __restrict__ row_scale,
                                                             const float* __restrict__ r = nullptr,
                                                             float* __restrict__ xo = nullptr) {
  __shared__ float red[2][8];
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  float wo[CH][4], g1[CH][4], sf[CH][4];  // offset + w, 1 + scale, shift of this thread's columns, once per CTA
#pragma unroll
  for (int c = 0; c < CH; c++) {
    const int64_t i = (int64_t)(c * 256 + tid) * 4;
    const bool live = i < d;
    const float4 ww = live ? *reinterpret_cast<const float4*>(w + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 s4 = live && sc ? *reinterpret_cast<const float4*>(sc + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 h4 = live && sh ? *reinterpret_cast<const float4*>(sh + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float wv[4] = {ww.x, ww.y, ww.z, ww.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w}, hv[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      wo[c][j] = offset + wv[j];
      g1[c][j] = 1.f + sv[j];
      sf[c][j] = hv[j];
    }
  }
  // software-pipelined over rows: the next row's loads are in flight while this row is reduced and stored
  float nx[CH][4], nr[CH][4];
  auto fetch = [&](int64_t row) {
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 256 + tid) * 4;
      if (i < d && row < rows) {
        load4<DT>(x, row * d + i, nx[c]);
        if (RES) {
          const float4 u = *reinterpret_cast<const float4*>(r + row * d + i);
          nr[c][0] = u.x; nr[c][1] = u.y; nr[c][2] = u.z; nr[c][3] = u.w;
        }
      }
    }
  };
  fetch(blockIdx.x);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[CH][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; c++) {
#pragma unroll
      for (int j = 0; j < 4; j++) v[c][j] = RES ? nx[c][j] + nr[c][j] : nx[c][j];
    }
    fetch(row + gridDim.x);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 256 + tid) * 4;
      if (i < d) {
        if (RES) *reinterpret_cast<float4*>(xo + row * d + i) = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        ss = fmaf(v[c][0], v[c][0], fmaf(v[c][1], v[c][1], ss));
        ss = fmaf(v[c][2], v[c][2], fmaf(v[c][3], v[c][3], ss));
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[0][wp] = ss;
    __syncthreads();
    const float tot = ((red[0][0] + red[0][1]) + (red[0][2] + red[0][3])) + ((red[0][4] + red[0][5]) + (red[0][6] + red[0][7]));
    const float inv = rsqrtf(tot / (float)d + eps);
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 256 + tid) * 4;
      if (i >= d) continue;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float y = v[c][j] * inv * wo[c][j] * g1[c][j] + sf[c][j];
        v[c][j] = bf16_bits_to_f32(f32_to_bf16_bits(y));
        amax = fmaxf(amax, fabsf(v[c][j]));
      }
    }
    amax = warp_max(amax);
    if (lane == 0) red[1][wp] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(fmaxf(red[1][0], red[1][1]), fmaxf(red[1][2], red[1][3])),
                 fmaxf(fmaxf(red[1][4], red[1][5]), fmaxf(red[1][6], red[1][7])));
    int e = 0;
    if (amax > 0.f) {
      int E;
      const float f = frexpf(amax, &E);
      e = (2.f * f <= 1.75f) ? E - 9 : E - 8;
    }
    if (tid == 0) row_scale[row] = ldexpf(1.0f, e);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 256 + tid) * 4;
      if (i >= d) continue;
      float s[4];
#pragma unroll
      for (int j = 0; j < 4; j++) s[j] = ldexpf(v[c][j], -e);
      const uint16_t h0 = f32x2_to_e4m3x2(s[0], s[1]), h1 = f32x2_to_e4m3x2(s[2], s[3]);
      *reinterpret_cast<uint32_t*>(hi + row * d + i) = (uint32_t)h0 | ((uint32_t)h1 << 16);
      if (TERMS > 1) {
        const float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
        const uint16_t l0 = f32x2_to_e4m3x2(s[0] - d0.x, s[1] - d0.y), l1 = f32x2_to_e4m3x2(s[2] - d1.x, s[3] - d1.y);
        *reinterpret_cast<uint32_t*>(lo + row * d + i) = (uint32_t)l0 | ((uint32_t)l1 << 16);
      }
    }
    // red[0] was read before the second barrier and red[1] is next written after the next row's first one
  }
}

template <int DT, int TERMS>
static bool norm_split_row(const void* x, const float* w, const float* sc, const float* sh, int64_t rows, int64_t d,
                           float eps, float offset, uint8_t* hi, uint8_t* lo, float* rs, int sms, cudaStream_t st) {
  const int64_t ch = (d / 4 + 255) / 256;
#define WE_NS(CH)                                                                                              \
  {                                                                                                            \
    auto k = norm_split_row_kernel<DT, TERMS, CH>;                                                             \
    k<<<resident_grid(k, 256, sms, rows), 256, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, nullptr, \
                                                         nullptr);                                             \
  }
  if (ch <= 2) WE_NS(2)
  else if (ch <= 3) WE_NS(3)
  else if (ch <= 4) WE_NS(4)
  else if (ch <= 6) WE_NS(6)
  else if (ch <= 8) WE_NS(8)
  else return false;
#undef WE_NS
  return true;
}

template <int DT, int TERMS>
static bool norm_split_dispatch(const void* x, const float* w, const float* sc, const float* sh, int64_t rows,
                                int64_t d, float eps, float offset, uint8_t* hi, uint8_t* lo, float* rs, int sms,
                                cudaStream_t st) {
  if (d >= 2048 && norm_split_row<DT, TERMS>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, sms, st)) return true;
  int64_t g = (rows + 3) / 4;
  if (g > (int64_t)sms * 16) g = (int64_t)sms * 16;
  if (d <= 256 * 4) norm_split_kernel<DT, TERMS, 4><<<(unsigned)g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs);
  else if (d <= 256 * 8) norm_split_kernel<DT, TERMS, 8><<<(unsigned)g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs);
  else if (d <= 256 * 12) norm_split_kernel<DT, TERMS, 12><<<(unsigned)g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs);
  else if (d <= 256 * 16) norm_split_kernel<DT, TERMS, 16><<<(unsigned)g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs);
  else if (d <= 256 * 24) norm_split_kernel<DT, TERMS, 24><<<(unsigned)g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs);
  else return false;
  return true;
}

cudaError_t launch_add_norm_split(const float* x, const float* r, float* xo, const float* w, const float* sc,
                                  const float* sh, int64_t rows, int64_t d, float eps, float offset, int terms,
                                  uint8_t* hi, uint8_t* lo, float* rs, int sms, cudaStream_t st) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (d % 8 || d > 8192 || !al(x) || !al(r) || !al(xo) || !al(w) || (sc && !al(sc)) || (sh && !al(sh)) ||
      ((uintptr_t)hi & 7) || (lo && ((uintptr_t)lo & 7)))
    return cudaErrorNotSupported;
  const int64_t ch = (d / 4 + 255) / 256;
#define WE_ANS(CH)                                                                                                  \
  {                                                                                                                 \
    if (terms > 1) {                                                                                                \
      auto k = norm_split_row_kernel<WE_F32, 2, CH, true>;                                                          \
      k<<<resident_grid(k, 256, sms, rows), 256, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo);   \
    } else {                                                                                                        \
      auto k = norm_split_row_kernel<WE_F32, 1, CH, true>;                                                          \
      k<<<resident_grid(k, 256, sms, rows), 256, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, r, xo);   \
    }                                                                                                               \
  }
  if (ch <= 2) WE_ANS(2)
  else if (ch <= 3) WE_ANS(3)
  else if (ch <= 4) WE_ANS(4)
  else if (ch <= 6) WE_ANS(6)
  else WE_ANS(8)
#undef WE_ANS
  return cudaGetLastError();
}

cudaError_t launch_norm_split(const void* x, int xdt, const float* w, const float* sc, const float* sh, int64_t rows,
                              int64_t d, float eps, float offset, int terms, uint8_t* hi, uint8_t* lo, float* rs,
                              int sms, cudaStream_t st) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (d % 8 || !al(x) || !al(w) || (sc && !al(sc)) || (sh && !al(sh)) || ((uintptr_t)hi & 7) ||
      (lo && ((uintptr_t)lo & 7)))
    return cudaErrorNotSupported;
  bool ok;
  if (xdt == WE_BF16) ok = terms > 1 ? norm_split_dispatch<WE_BF16, 2>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, sms, st)
                                     : norm_split_dispatch<WE_BF16, 1>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, sms, st);
  else ok = terms > 1 ? norm_split_dispatch<WE_F32, 2>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, sms, st)
                      : norm_split_dispatch<WE_F32, 1>(x, w, sc, sh, rows, d, eps, offset, hi, lo, rs, sms, st);
  if (!ok) return cudaErrorNotSupported;
  return cudaGetLastError();
}

}  // namespace we
