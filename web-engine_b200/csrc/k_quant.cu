// Decode / quantise kernels: fp8 and int4 unpack (src/kernels/fp8.ts:24-36 unpackFp8 and the int4
// group-64 operand), weight quantisers, and the activation split that feeds the fp8 tensor-core GEMM.
// All are HBM-bandwidth kernels: 16-byte vector accesses where the layout allows, grid-stride
// loops sized to a multiple of the SM count.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace we {

// ---------------- unpack ----------------
// n16: number of 16-value chunks done with vector accesses (0 when the pointers are not 16-byte aligned)
__global__ void unpack_fp8_f32_kernel(const uint8_t* __restrict__ in, int64_t n, int64_t n16, float scale,
                                      float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 v = reinterpret_cast<const uint4*>(in)[i];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float r[16];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int b = 0; b < 4; b++) r[4 * j + b] = e4m3_to_f32((w[j] >> (8 * b)) & 0xffu) * scale;
    float4* o = reinterpret_cast<float4*>(out + 16 * i);
#pragma unroll
    for (int j = 0; j < 4; j++) o[j] = make_float4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
  }
  // ragged tail (n not a multiple of 16): one thread per value
  for (int64_t i = n16 * 16 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = e4m3_to_f32(in[i]) * scale;
}

__global__ void unpack_fp8_bf16_kernel(const uint8_t* __restrict__ in, int64_t n, int64_t n8, uint16_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    uint2 v = reinterpret_cast<const uint2*>(in)[i];
    uint32_t w[2] = {v.x, v.y};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      float2 a = e4m3x2_to_f32x2((uint16_t)(w[j] & 0xffffu));
      float2 b = e4m3x2_to_f32x2((uint16_t)(w[j] >> 16));
      o[2 * j] = pack_bf16x2(a.x, a.y);
      o[2 * j + 1] = pack_bf16x2(b.x, b.y);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f32_to_bf16_bits(e4m3_to_f32(in[i]));
}

// int4 g64 -> bf16 operand. One thread per 8 values (one u32 of packed nibbles), k % 64 == 0.
__global__ void unpack_int4_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales, int64_t n,
                                   int64_t k, uint16_t* __restrict__ out) {
  int64_t words = n * k / 8;
  int64_t groups = k / 64;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t w = reinterpret_cast<const uint32_t*>(packed)[i];
    int64_t e0 = i * 8;  // first value
    int64_t row = e0 / k, col = e0 % k;
    float s = __half2float(__ushort_as_half(scales[row * groups + col / 64]));
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float lo = int4_operand((w >> (8 * j)) & 0xfu, s);
      float hi = int4_operand((w >> (8 * j + 4)) & 0xfu, s);
      o[j] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------- weight quantisers ----------------
template <int DT>
__device__ float block_absmax_row(const void* w, int64_t base, int64_t k) {
  float m = 0.f;
  for (int64_t t = threadIdx.x; t < k; t += blockDim.x) m = fmaxf(m, fabsf(load_act<DT>(w, base + t)));
  __shared__ float red[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

template <int DT>
__global__ void quant_fp8_rows_kernel(const void* __restrict__ w, int64_t n, int64_t k, const float* __restrict__ tensor_amax,
                                      uint8_t* __restrict__ q, float* __restrict__ scales) {
  for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
    float amax = tensor_amax ? *tensor_amax : block_absmax_row<DT>(w, row * k, k);
    float s = amax > 0.f ? __fdiv_rn(amax, 448.0f) : 1.0f;
    if (threadIdx.x == 0 && (!tensor_amax || row == 0)) scales[tensor_amax ? 0 : row] = s;
    for (int64_t t = threadIdx.x; t < k; t += blockDim.x) q[row * k + t] = f32_to_e4m3(__fdiv_rn(load_act<DT>(w, row * k + t), s));
  }
}

template <int DT>
__global__ void absmax_all_kernel(const void* __restrict__ w, int64_t total, unsigned int* __restrict__ out_bits) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(load_act<DT>(w, i)));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // non-negative floats order as ints
}

// one warp per (row, group of 64); lane l owns values 2l, 2l+1 (one packed byte)
template <int DT>
__global__ void quant_int4_kernel(const void* __restrict__ w, int64_t n, int64_t k, uint8_t* __restrict__ packed,
                                  uint16_t* __restrict__ scales) {
  int64_t groups = k / 64;
  int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int lane = threadIdx.x & 31;
  for (int64_t gi = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); gi < n * groups; gi += warps) {
    int64_t row = gi / groups, g = gi % groups;
    int64_t base = row * k + g * 64 + 2 * lane;
    float a = load_act<DT>(w, base), b = load_act<DT>(w, base + 1);
    float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
    __half s16 = __float2half_rn(__fdiv_rn(amax, 7.0f));
    float s = __half2float(s16);
    int qa = 0, qb = 0;
    if (s != 0.f) {
      qa = (int)fminf(fmaxf(rintf(__fdiv_rn(a, s)), -8.f), 7.f);
      qb = (int)fminf(fmaxf(rintf(__fdiv_rn(b, s)), -8.f), 7.f);
    }
    packed[base / 2] = (uint8_t)((qa & 0xf) | ((qb & 0xf) << 4));
    if (lane == 0) scales[gi] = __half_as_ushort(s16);
  }
}

// ---------------- activation split (fp8 tensor-core path) ----------------
// exponent e: smallest integer with amax * 2^-e <= 448 (amax = m 2^E, m in [1,2): e = E-8 if m <= 1.75 else E-7)
__device__ __forceinline__ int act_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  int E;
  float f = frexpf(amax, &E);  // amax = f 2^E, f in [0.5, 1)
  float m = 2.f * f;
  E -= 1;
  return m <= 1.75f ? E - 8 : E - 7;
}

// 2^-e as a float multiplier when it is a normal float (exact scaling), else 0 (callers use ldexpf)
__device__ __forceinline__ float pow2_neg(int e) {
  const int b = 127 - e;
  return (b >= 1 && b <= 254) ? __int_as_float(b << 23) : 0.f;
}

// one CTA per row (grid-stride); VEC = values per 16-byte load of x
template <int DT, int TERMS>
__global__ void quant_act_kernel(const void* __restrict__ x, int64_t m, int64_t k, int64_t stride, uint8_t* __restrict__ hi,
                                 uint8_t* __restrict__ lo, float* __restrict__ row_scale, int vec_ok) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    int64_t base = row * stride;
    float amax = 0.f;
    for (int64_t t = threadIdx.x; t < k; t += blockDim.x) amax = fmaxf(amax, fabsf(load_act<DT>(x, base + t)));
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_max(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    int e = act_exponent(red[0]);
    __syncthreads();
    if (threadIdx.x == 0) row_scale[row] = ldexpf(1.0f, e);
    if (vec_ok) {
      // 8 values per step: 16 B of bf16 / 32 B of f32 in, 8 B per term out
      for (int64_t t = 8 * threadIdx.x; t < k; t += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = ldexpf(load_act<DT>(x, base + t + j), -e);
        uint32_t h[2], l[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
          uint16_t h0 = f32x2_to_e4m3x2(v[4 * j], v[4 * j + 1]);
          uint16_t h1 = f32x2_to_e4m3x2(v[4 * j + 2], v[4 * j + 3]);
          h[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
          if (TERMS > 1) {
            float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
            uint16_t l0 = f32x2_to_e4m3x2(v[4 * j] - d0.x, v[4 * j + 1] - d0.y);
            uint16_t l1 = f32x2_to_e4m3x2(v[4 * j + 2] - d1.x, v[4 * j + 3] - d1.y);
            l[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
          }
        }
        *reinterpret_cast<uint2*>(hi + row * k + t) = make_uint2(h[0], h[1]);
        if (TERMS > 1) *reinterpret_cast<uint2*>(lo + row * k + t) = make_uint2(l[0], l[1]);
      }
    } else {
      for (int64_t t = threadIdx.x; t < k; t += blockDim.x) {
        float v = ldexpf(load_act<DT>(x, base + t), -e);
        uint8_t h = f32_to_e4m3(v);
        hi[row * k + t] = h;
        if (TERMS > 1) lo[row * k + t] = f32_to_e4m3(v - e4m3_to_f32(h));
      }
    }
  }
}

// Register-cached variant: one 128-thread CTA per row, each thread keeps its CH chunks of 8 values
// (16-byte loads) in registers, so x is read once. k % 8 == 0, k <= 1024 CH, 16-byte aligned rows.
template <int DT, int TERMS, int CH>
__global__ void __launch_bounds__(128) quant_act_cached_kernel(const void* __restrict__ x, int64_t m, int64_t k,
                                                               int64_t stride, uint8_t* __restrict__ hi,
                                                               uint8_t* __restrict__ lo, float* __restrict__ row_scale) {
  __shared__ float red[4];
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    const int64_t base = row * stride;
    float v[CH][8];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t t = (int64_t)(c * 128 + threadIdx.x) * 8;
      if (t < k) {
        load8<DT>(x, base + t, v[c]);
#pragma unroll
        for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[c][j]));
      }
    }
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    const int e = act_exponent(amax);
    if (threadIdx.x == 0) row_scale[row] = ldexpf(1.0f, e);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t t = (int64_t)(c * 128 + threadIdx.x) * 8;
      if (t >= k) continue;
      float s[8];
#pragma unroll
      for (int j = 0; j < 8; j++) s[j] = ldexpf(v[c][j], -e);
      uint32_t h[2], l[2];
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const uint16_t h0 = f32x2_to_e4m3x2(s[4 * j], s[4 * j + 1]);
        const uint16_t h1 = f32x2_to_e4m3x2(s[4 * j + 2], s[4 * j + 3]);
        h[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        if (TERMS > 1) {
          const float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
          const uint16_t l0 = f32x2_to_e4m3x2(s[4 * j] - d0.x, s[4 * j + 1] - d0.y);
          const uint16_t l1 = f32x2_to_e4m3x2(s[4 * j + 2] - d1.x, s[4 * j + 3] - d1.y);
          l[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
      }
      *reinterpret_cast<uint2*>(hi + row * k + t) = make_uint2(h[0], h[1]);
      if (TERMS > 1) *reinterpret_cast<uint2*>(lo + row * k + t) = make_uint2(l[0], l[1]);
    }
  }
}

// Warp-per-row split for bf16 rows (k % 8 == 0, k <= 256 UMAX, 16-byte aligned rows): lane l keeps
// the row's 16-byte chunks l, l + 32, ... packed in registers; the row max is a shuffle reduction.
template <int TERMS, int UMAX>
__global__ void __launch_bounds__(128, 6) quant_act_warp_kernel(const uint16_t* __restrict__ x, int64_t m, int64_t k,
                                                             int64_t stride, uint8_t* __restrict__ hi,
                                                             uint8_t* __restrict__ lo, float* __restrict__ row_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 4;
  for (int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); row < m; row += warps) {
    const uint16_t* xr = x + row * stride;
    uint4 v[UMAX];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t t = (int64_t)(c * 32 + lane) * 8;
      if (t < k) {
        v[c] = *reinterpret_cast<const uint4*>(xr + t);
        // |bf16| max on the bit patterns: clear the sign bits, compare as integers
        const uint32_t a = v[c].x & 0x7fff7fffu, b = v[c].y & 0x7fff7fffu, cc = v[c].z & 0x7fff7fffu,
                       dd = v[c].w & 0x7fff7fffu;
        const uint32_t m1 = __vmaxu2(__vmaxu2(a, b), __vmaxu2(cc, dd));
        amax = fmaxf(amax, fmaxf(__uint_as_float(m1 << 16), __uint_as_float(m1 & 0xffff0000u)));
      }
    }
    amax = warp_max(amax);
    const int e = act_exponent(amax);
    if (lane == 0) row_scale[row] = ldexpf(1.0f, e);
    const float mul = pow2_neg(e);  // exact: scaling by a power of two
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t t = (int64_t)(c * 32 + lane) * 8;
      if (t >= k) continue;
      const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
      float s[8];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
        s[2 * j] = mul != 0.f ? a * mul : ldexpf(a, -e);
        s[2 * j + 1] = mul != 0.f ? b * mul : ldexpf(b, -e);
      }
      uint32_t h[2], l[2];
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const uint16_t h0 = f32x2_to_e4m3x2(s[4 * j], s[4 * j + 1]);
        const uint16_t h1 = f32x2_to_e4m3x2(s[4 * j + 2], s[4 * j + 3]);
        h[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        if (TERMS > 1) {
          const float2 d0 = e4m3x2_to_f32x2(h0), d1 = e4m3x2_to_f32x2(h1);
          const uint16_t l0 = f32x2_to_e4m3x2(s[4 * j] - d0.x, s[4 * j + 1] - d0.y);
          const uint16_t l1 = f32x2_to_e4m3x2(s[4 * j + 2] - d1.x, s[4 * j + 3] - d1.y);
          l[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
      }
      *reinterpret_cast<uint2*>(hi + row * k + t) = make_uint2(h[0], h[1]);
      if (TERMS > 1) *reinterpret_cast<uint2*>(lo + row * k + t) = make_uint2(l[0], l[1]);
    }
  }
}

// CTA-per-row split for long bf16 rows (k % 8 == 0, k <= 2048 CH, 16-byte aligned rows): 256 threads, thread t
// keeps the row's 16-byte chunks t, t + 256, ... in registers (few registers: many rows in flight per SM); the
// row max is a warp shuffle then a shared-memory reduction over the 8 warps. PF: the next row's chunks are
// loaded while this row is split (pays for short rows; at 6+ chunks the doubled registers cost more than it gains).
// 8 scaled values -> their e4m3 hi (and lo = e4m3(s - hi)) terms, 8 bytes per term
template <int TERMS>
__device__ __forceinline__ void split_store8(const float2 (&s)[4], uint8_t* hi, uint8_t* lo) {
  uint32_t h[2], l[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const uint16_t h0 = f32x2_to_e4m3x2(s[2 * j].x, s[2 * j].y);
    const uint16_t h1 = f32x2_to_e4m3x2(s[2 * j + 1].x, s[2 * j + 1].y);
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

template <int TERMS, int CH, int NT = 256, bool PF = false>
__global__ void __launch_bounds__(NT) quant_act_row_kernel(const uint16_t* __restrict__ x, int64_t m, int64_t k,
                                                           int64_t stride, uint8_t* __restrict__ hi,
                                                           uint8_t* __restrict__ lo, float* __restrict__ row_scale) {
  constexpr int NW = NT / 32;
  __shared__ float red[8];
  pdl_wait();  // launched by launch_pdl: the previous kernel's output (x) is complete
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  uint4 nv[CH];
  auto fetch = [&](int64_t row) {
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t t = (int64_t)(c * NT + tid) * 8;
      if (t < k && row < m) nv[c] = *reinterpret_cast<const uint4*>(x + row * stride + t);
    }
  };
  if (PF) fetch(blockIdx.x);
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    uint4 v[CH];
    uint32_t mx = 0;
    if (!PF) fetch(row);
#pragma unroll
    for (int c = 0; c < CH; c++) v[c] = nv[c];
    if (PF) fetch(row + gridDim.x);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t t = (int64_t)(c * NT + tid) * 8;
      if (t < k) {
        // |bf16| max on the bit patterns: clear the sign bits, compare as integers
        mx = __vmaxu2(mx, __vmaxu2(__vmaxu2(v[c].x & 0x7fff7fffu, v[c].y & 0x7fff7fffu),
                                   __vmaxu2(v[c].z & 0x7fff7fffu, v[c].w & 0x7fff7fffu)));
      }
    }
    float amax = warp_max(fmaxf(__uint_as_float(mx << 16), __uint_as_float(mx & 0xffff0000u)));
    if (lane == 0) red[wp] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int i = 1; i < NW; i++) amax = fmaxf(amax, red[i]);
    __syncthreads();  // red is rewritten by the next row
    const int e = act_exponent(amax);
    if (tid == 0) row_scale[row] = ldexpf(1.0f, e);
    const float mul = pow2_neg(e);  // exact: scaling by a power of two
    // The multiplier is uniform over the row: one branch per row, and in the usual case (2^-e a normal float) the
    // values are scaled two at a time by packed multiplies; ldexpf only for rows whose scale is outside that range.
    if (mul != 0.f) {
      const float2 mul2 = make_float2(mul, mul);
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int64_t t = (int64_t)(c * NT + tid) * 8;
        if (t >= k) continue;
        const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        float2 s[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          s[j] = __fmul2_rn(make_float2(__uint_as_float(u[j] << 16), __uint_as_float(u[j] & 0xffff0000u)), mul2);
        split_store8<TERMS>(s, hi + row * k + t, lo + row * k + t);
      }
    } else {
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int64_t t = (int64_t)(c * NT + tid) * 8;
        if (t >= k) continue;
        const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
        float2 s[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          s[j] = make_float2(ldexpf(__uint_as_float(u[j] << 16), -e), ldexpf(__uint_as_float(u[j] & 0xffff0000u), -e));
        split_store8<TERMS>(s, hi + row * k + t, lo + row * k + t);
      }
    }
  }
}

template <int TERMS>
static bool quant_act_row(const uint16_t* x, int64_t m, int64_t k, int64_t stride, uint8_t* hi, uint8_t* lo, float* rs,
                          int sms, cudaStream_t st) {
  // short rows: next-row prefetch on a grid of every resident CTA; long rows: one row at a time on 8 CTAs per SM
#define WE_QAR(CH, NT)                                                                                   \
  {                                                                                                      \
    constexpr bool pf = NT == 128;                                                                       \
    auto kern = quant_act_row_kernel<TERMS, CH, NT, pf>;                                                 \
    const int g = pf ? resident_grid(kern, NT, sms, m) : (int)std::min<int64_t>(m, (int64_t)sms * 8);    \
    (void)launch_pdl(kern, g, NT, 0, st, x, m, k, stride, hi, lo, rs);                                   \
  }
  if (k <= 128 * 8 * 4) {  // up to 4096 values: 128 threads, every thread busy at k = 3072
    const int64_t ch = (k / 8 + 127) / 128;
    if (ch <= 2) WE_QAR(2, 128)
    else if (ch <= 3) WE_QAR(3, 128)
    else WE_QAR(4, 128)
    return true;
  }
  const int64_t ch = (k / 8 + 255) / 256;
  if (ch <= 2) WE_QAR(2, 256)
  else if (ch <= 3) WE_QAR(3, 256)
  else if (ch <= 4) WE_QAR(4, 256)
  else if (ch <= 6) WE_QAR(6, 256)
  else if (ch <= 8) WE_QAR(8, 256)
  else return false;
#undef WE_QAR
  return true;
}

template <int TERMS>
static bool quant_act_warp(const uint16_t* x, int64_t m, int64_t k, int64_t stride, uint8_t* hi, uint8_t* lo, float* rs,
                           int sms, cudaStream_t st) {
  const int g = (int)std::min<int64_t>((m + 3) / 4, (int64_t)sms * 16);
  if (k <= 256 * 4) quant_act_warp_kernel<TERMS, 4><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (k <= 256 * 8) quant_act_warp_kernel<TERMS, 8><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (k <= 256 * 12) quant_act_warp_kernel<TERMS, 12><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (k <= 256 * 16) quant_act_warp_kernel<TERMS, 16><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (k <= 256 * 24) quant_act_warp_kernel<TERMS, 24><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else return false;
  return true;
}

template <int DT, int TERMS>
static bool quant_act_cached(const void* x, int64_t m, int64_t k, int64_t stride, uint8_t* hi, uint8_t* lo,
                             float* rs, int sms, cudaStream_t st) {
  const int g = (int)((m < (int64_t)sms * 16) ? m : (int64_t)sms * 16);
  const int64_t chunks = (k / 8 + 127) / 128;
  if (chunks <= 1) quant_act_cached_kernel<DT, TERMS, 1><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (chunks <= 2) quant_act_cached_kernel<DT, TERMS, 2><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (chunks <= 3) quant_act_cached_kernel<DT, TERMS, 3><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (chunks <= 4) quant_act_cached_kernel<DT, TERMS, 4><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (chunks <= 6) quant_act_cached_kernel<DT, TERMS, 6><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else if (chunks <= 8) quant_act_cached_kernel<DT, TERMS, 8><<<g, 128, 0, st>>>(x, m, k, stride, hi, lo, rs);
  else return false;
  return true;
}

// ---------------- launchers ----------------
static int grid_for(int64_t work, int threads, int sms, int per_sm = 8) {
  int64_t g = (work + threads - 1) / threads;
  int64_t cap = (int64_t)sms * per_sm;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

cudaError_t launch_unpack_fp8_f32(const uint8_t* in, int64_t n, float scale, float* out, int sms, cudaStream_t st) {
  bool vec = ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
  int64_t n16 = vec ? n / 16 : 0;
  unpack_fp8_f32_kernel<<<grid_for(n16 + (n - 16 * n16), 256, sms), 256, 0, st>>>(in, n, n16, scale, out);
  return cudaGetLastError();
}

cudaError_t launch_unpack_fp8_bf16(const uint8_t* in, int64_t n, uint16_t* out, int sms, cudaStream_t st) {
  bool vec = ((uintptr_t)in % 8 == 0) && ((uintptr_t)out % 16 == 0);
  int64_t n8 = vec ? n / 8 : 0;
  unpack_fp8_bf16_kernel<<<grid_for(n8 + (n - 8 * n8), 256, sms), 256, 0, st>>>(in, n, n8, out);
  return cudaGetLastError();
}

cudaError_t launch_unpack_int4(const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k, uint16_t* out,
                               int sms, cudaStream_t st) {
  unpack_int4_kernel<<<grid_for(n * k / 8, 256, sms), 256, 0, st>>>(packed, scales, n, k, out);
  return cudaGetLastError();
}

cudaError_t launch_quant_fp8(const void* w, int dt, int64_t n, int64_t k, bool per_channel, uint8_t* q, float* scales,
                             unsigned int* amax_scratch, int sms, cudaStream_t st) {
  int g = (int)((n < (int64_t)sms * 8) ? n : (int64_t)sms * 8);
  if (g < 1) g = 1;
  if (per_channel) {
    if (dt == WE_F32) quant_fp8_rows_kernel<WE_F32><<<g, 256, 0, st>>>(w, n, k, nullptr, q, scales);
    else quant_fp8_rows_kernel<WE_BF16><<<g, 256, 0, st>>>(w, n, k, nullptr, q, scales);
  } else {
    cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int), st);
    if (dt == WE_F32) absmax_all_kernel<WE_F32><<<grid_for(n * k, 256, sms), 256, 0, st>>>(w, n * k, amax_scratch);
    else absmax_all_kernel<WE_BF16><<<grid_for(n * k, 256, sms), 256, 0, st>>>(w, n * k, amax_scratch);
    const float* am = reinterpret_cast<const float*>(amax_scratch);
    if (dt == WE_F32) quant_fp8_rows_kernel<WE_F32><<<g, 256, 0, st>>>(w, n, k, am, q, scales);
    else quant_fp8_rows_kernel<WE_BF16><<<g, 256, 0, st>>>(w, n, k, am, q, scales);
  }
  return cudaGetLastError();
}

cudaError_t launch_quant_int4(const void* w, int dt, int64_t n, int64_t k, uint8_t* packed, uint16_t* scales, int sms,
                              cudaStream_t st) {
  int64_t warps = n * (k / 64);
  int g = grid_for(warps * 32, 256, sms);
  if (dt == WE_F32) quant_int4_kernel<WE_F32><<<g, 256, 0, st>>>(w, n, k, packed, scales);
  else quant_int4_kernel<WE_BF16><<<g, 256, 0, st>>>(w, n, k, packed, scales);
  return cudaGetLastError();
}

cudaError_t launch_quant_act(const void* x, int dt, int64_t m, int64_t k, int64_t stride, int terms, uint8_t* hi,
                             uint8_t* lo, float* row_scale, int sms, cudaStream_t st) {
  int threads = 128;
  int g = (int)((m < (int64_t)sms * 16) ? m : (int64_t)sms * 16);
  if (g < 1) g = 1;
  int vec_ok = (k % 8 == 0) && ((uintptr_t)hi % 8 == 0) && (!lo || (uintptr_t)lo % 8 == 0);
  const int esz = dt == WE_F32 ? 4 : 2;
  if (vec_ok && (uintptr_t)x % 16 == 0 && (stride * esz) % 16 == 0) {
    if (dt == WE_BF16) {
      const uint16_t* xb = static_cast<const uint16_t*>(x);
      // rows of 2048+ values: a CTA per row; shorter rows: a warp per row
      if (k >= 2048 && (terms > 1 ? quant_act_row<2>(xb, m, k, stride, hi, lo, row_scale, sms, st)
                                  : quant_act_row<1>(xb, m, k, stride, hi, lo, row_scale, sms, st)))
        return cudaGetLastError();
      if (terms > 1 ? quant_act_warp<2>(xb, m, k, stride, hi, lo, row_scale, sms, st)
                    : quant_act_warp<1>(xb, m, k, stride, hi, lo, row_scale, sms, st))
        return cudaGetLastError();
    }
    bool done;
    if (dt == WE_F32) done = terms > 1 ? quant_act_cached<WE_F32, 2>(x, m, k, stride, hi, lo, row_scale, sms, st)
                                       : quant_act_cached<WE_F32, 1>(x, m, k, stride, hi, lo, row_scale, sms, st);
    else done = terms > 1 ? quant_act_cached<WE_BF16, 2>(x, m, k, stride, hi, lo, row_scale, sms, st)
                          : quant_act_cached<WE_BF16, 1>(x, m, k, stride, hi, lo, row_scale, sms, st);
    if (done) return cudaGetLastError();
  }
  if (dt == WE_F32) {
    if (terms > 1) quant_act_kernel<WE_F32, 2><<<g, threads, 0, st>>>(x, m, k, stride, hi, lo, row_scale, vec_ok);
    else quant_act_kernel<WE_F32, 1><<<g, threads, 0, st>>>(x, m, k, stride, hi, lo, row_scale, vec_ok);
  } else {
    if (terms > 1) quant_act_kernel<WE_BF16, 2><<<g, threads, 0, st>>>(x, m, k, stride, hi, lo, row_scale, vec_ok);
    else quant_act_kernel<WE_BF16, 1><<<g, threads, 0, st>>>(x, m, k, stride, hi, lo, row_scale, vec_ok);
  }
  return cudaGetLastError();
}

}  // namespace we
