// RMSNorm (+ Krea modulation), RoPE and the fused q/k-norm + RoPE.
//
// Reference: rmsnormWgsl (src/kernels/rmsnorm.ts:13-48), ropeKernel (src/kernels/rope.ts:59-77), and the
// q/k path of attend() (src/model/block.ts:53-56: linear -> norm(qNorm, rows*heads, 128) -> rotate).
// These are HBM-bandwidth kernels. Row sums of squares are accumulated in fp32 like the reference
// shader (tree order differs; the result stays within the reference test's 1e-5).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace we {

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// One CTA per row (grid-stride over rows). VEC: 8 values per access (d % 8 == 0, aligned); the row
// is read twice, the second time from L1/L2.
template <int DT, int OT, bool VEC>
__global__ void rmsnorm_kernel(const void* __restrict__ x, const float* __restrict__ w, const float* __restrict__ sc,
                               const float* __restrict__ sh, int64_t rows, int64_t d, float eps, float offset,
                               void* __restrict__ out) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    int64_t base = row * d;
    float ss = 0.f;
    if (VEC) {
      for (int64_t i = 8 * threadIdx.x; i < d; i += 8 * blockDim.x) {
        float v[8];
        load8<DT>(x, base + i, v);
#pragma unroll
        for (int j = 0; j < 8; j++) ss = fmaf(v[j], v[j], ss);
      }
    } else {
      for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float v = load_act<DT>(x, base + i);
        ss = fmaf(v, v, ss);
      }
    }
    float inv = rsqrtf(block_sum(ss, red) / (float)d + eps);
    if (VEC) {
      for (int64_t i = 8 * threadIdx.x; i < d; i += 8 * blockDim.x) {
        float v[8], ww[8], s[8], h[8];
        load8<DT>(x, base + i, v);
        load8f(w, i, ww);
        if (sc) load8f(sc, i, s); else for (int j = 0; j < 8; j++) s[j] = 0.f;
        if (sh) load8f(sh, i, h); else for (int j = 0; j < 8; j++) h[j] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = v[j] * inv * (offset + ww[j]) * (1.f + s[j]) + h[j];
        store8<OT>(out, base + i, v);
      }
    } else {
      for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float v = load_act<DT>(x, base + i);
        float s = sc ? sc[i] : 0.f, h = sh ? sh[i] : 0.f;
        store_out<OT>(out, base + i, v * inv * (offset + w[i]) * (1.f + s) + h);
      }
    }
  }
}

// Register-cached RMSNorm: one 128-thread CTA per row keeps its CH chunks of 8 values in registers,
// so x is read from HBM once (d % 8 == 0, d <= 1024 CH, 16-byte aligned rows and vectors).
template <int DT, int OT, int CH>
__global__ void __launch_bounds__(128) rmsnorm_cached_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                             const float* __restrict__ sc, const float* __restrict__ sh,
                                                             int64_t rows, int64_t d, float eps, float offset,
                                                             void* __restrict__ out) {
  __shared__ float red[4];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * d;
    float v[CH][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 128 + threadIdx.x) * 8;
      if (i < d) {
        load8<DT>(x, base + i, v[c]);
#pragma unroll
        for (int j = 0; j < 8; j++) ss = fmaf(v[c][j], v[c][j], ss);
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)d + eps);
    __syncthreads();
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int64_t i = (int64_t)(c * 128 + threadIdx.x) * 8;
      if (i >= d) continue;
      float ww[8], s[8], h[8];
      load8f(w, i, ww);
      if (sc) load8f(sc, i, s); else for (int j = 0; j < 8; j++) s[j] = 0.f;
      if (sh) load8f(sh, i, h); else for (int j = 0; j < 8; j++) h[j] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) v[c][j] = v[c][j] * inv * (offset + ww[j]) * (1.f + s[j]) + h[j];
      store8<OT>(out, base + i, v[c]);
    }
  }
}

// Warp-per-row RMSNorm for bf16 rows (d % 8 == 0, d <= 256 UMAX, 16-byte aligned): lane l holds the
// row's 16-byte chunks l, l + 32, ... packed as bf16 in registers (4 registers per 8 values), so each
// warp-wide load is 512 contiguous bytes, x is read once, and the reduction is shuffles only. With
// ~2 KB of row per warp in flight, a full SM keeps the whole 4608-row block in one wave.
template <int OT, int UMAX>
__global__ void __launch_bounds__(128) rmsnorm_warp_kernel(const uint16_t* __restrict__ x, const float* __restrict__ w,
                                                           const float* __restrict__ sc, const float* __restrict__ sh,
                                                           int64_t rows, int64_t d, float eps, float offset,
                                                           void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 4;
  for (int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); row < rows; row += warps) {
    const uint16_t* xr = x + row * d;
    uint4 v[UMAX];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t i = (int64_t)(c * 32 + lane) * 8;
      if (i < d) {
        v[c] = *reinterpret_cast<const uint4*>(xr + i);
        const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
          ss = fmaf(a, a, fmaf(b, b, ss));
        }
      }
    }
    const float inv = rsqrtf(warp_sum(ss) / (float)d + eps);
#pragma unroll
    for (int c = 0; c < UMAX; c++) {
      const int64_t i = (int64_t)(c * 32 + lane) * 8;
      if (i >= d) continue;
      float f[8], ww[8], s[8], h[8];
      const uint32_t u[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        f[2 * j] = __uint_as_float(u[j] << 16);
        f[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
      }
      load8f(w, i, ww);
      if (sc) load8f(sc, i, s); else for (int j = 0; j < 8; j++) s[j] = 0.f;
      if (sh) load8f(sh, i, h); else for (int j = 0; j < 8; j++) h[j] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] = f[j] * inv * (offset + ww[j]) * (1.f + s[j]) + h[j];
      store8<OT>(out, row * d + i, f);
    }
  }
}

// CTA-per-row RMSNorm for rows of 2048..8192 values (16-byte aligned, d % 8 == 0): NT threads, thread t owns the
// 8-value chunks t, t + NT, ... (CH of them) of every row and keeps its columns' modulation in registers across the
// rows the CTA strides over (a warp-per-row form reloads those f32 vectors, six times the row's own bytes, for every
// row), as two factors: (offset + w)(1 + scale), rounded once, and the shift, so y = fma(x inv, (offset + w)(1 +
// scale), shift) (one f32 rounding from the product order of rmsnorm.ts:42-46). The rows are staged through shared
// memory by cp.async, S - 1 rows ahead: each thread copies the chunks it later reads (no barrier on the ring) and the
// loads in flight hold no registers. Sum of squares: warp shuffle, then the warps in a fixed order; the per-value
// arithmetic runs two values at a time (packed f32x2); offsets within a row are 32-bit (d <= 8192).
template <int DT, int OT, int NT, int CH, int S>
__global__ void __launch_bounds__(NT, NT == 192 ? 4 : 512 / NT) rmsnorm_row_kernel(
    const void* __restrict__ x, const float* __restrict__ w, const float* __restrict__ sc,
    const float* __restrict__ sh, int64_t rows, int64_t d, float eps, float offset, void* __restrict__ out) {
  constexpr int NW = NT / 32;
  constexpr int ES = DT == WE_F32 ? 4 : 2;  // bytes per value of x
  constexpr int XB = 8 * ES;                 // bytes of one 8-value chunk
  constexpr int XSTAGE = CH * NT * XB;
  extern __shared__ __align__(16) uint8_t ring[];  // [S][CH][NT] chunks
  __shared__ __align__(16) float red[NW];
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs (x, the modulation) are complete
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int dd = (int)d;
  float2 mw[CH][4], sf[CH][4];  // (offset + w)(1 + scale) and shift of this thread's columns
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
#pragma unroll
      for (int c = 0; c < CH; c++) {
        const int i = (c * NT + tid) * 8;
        if (i >= dd) continue;
        const uint32_t xa = ring_s + s * XSTAGE + (c * NT + tid) * XB;
#pragma unroll
        for (int q = 0; q < XB / 16; q++) cp_async16(xa + 16 * q, xr + i * ES + 16 * q);
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
#pragma unroll
      for (int j = 0; j < 4; j++) ss2 = __ffma2_rn(v[c][j], v[c][j], ss2);
    }
    s = s + 1 == S ? 0 : s + 1;
    sn = sn + 1 == S ? 0 : sn + 1;
    const float ss = warp_sum(ss2.x + ss2.y);
    if (lane == 0) red[wp] = ss;
    __syncthreads();
    float tot = red[0];
#pragma unroll
    for (int k = 1; k < NW; k++) tot += red[k];
    const float inv = rsqrtf(tot / (float)dd + eps);
    __syncthreads();  // red is rewritten by the next row
    const float2 inv2 = make_float2(inv, inv);
    uint8_t* const orow = static_cast<uint8_t*>(out) + row * d * (OT == WE_F32 ? 4 : 2);
#pragma unroll
    for (int c = 0; c < CH; c++) {
      const int i = (c * NT + tid) * 8;
      if (i >= dd) continue;
      float2 y[4];
#pragma unroll
      for (int j = 0; j < 4; j++) y[j] = __ffma2_rn(__fmul2_rn(v[c][j], inv2), mw[c][j], sf[c][j]);
      if constexpr (OT == WE_F32) {
        *reinterpret_cast<float4*>(orow + i * 4) = make_float4(y[0].x, y[0].y, y[1].x, y[1].y);
        *reinterpret_cast<float4*>(orow + i * 4 + 16) = make_float4(y[2].x, y[2].y, y[3].x, y[3].y);
      } else {
        *reinterpret_cast<uint4*>(orow + i * 2) = make_uint4(pack_bf16x2(y[0].x, y[0].y), pack_bf16x2(y[1].x, y[1].y),
                                                             pack_bf16x2(y[2].x, y[2].y), pack_bf16x2(y[3].x, y[3].y));
      }
    }
  }
  cp_async_wait<0>();  // nothing is left in flight (every row issued was consumed); kept as the exit rule
}

// q/k norm + RoPE for 128-wide heads (NORM false: RoPE alone): 16 lanes per head row, 8 values (16 bytes of
// bf16) per lane; a warp takes 2 R rows per step (R per half-warp) and issues all their loads (rows and cos/sin)
// before any arithmetic, so each warp keeps R x 48 bytes per lane in flight. Interleaved pairs stay in a lane;
// half pairing exchanges with lane ^ 8. TOK (heads % 8 == 0): a step's 8 rows are 8 heads of one token, so the
// token's cos/sin values are loaded once per step instead of once per row (they are twice a row's own bytes).
// PEER: row (token t, head h) goes to rank o = h / hl's exchange region instead of out: to
// dst[o] + ((row0 + t) hl + h - o hl) 128 values, i.e. [every rank's tokens, rank o's hl heads, 128] with this rank's
// tokens from row0 (sequence parallelism: the head scatter done by the stores themselves, over NVLink).
struct PeerRows {
  void* dst[WE_PEER_MAX];
  int64_t row0, hl;
};

template <int DT, int OT, int PAIRING, bool NORM, bool TOK = false, bool PEER = false>
__global__ void __launch_bounds__(256, TOK ? 3 : 2) qknorm_rope128_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                             float eps, float offset, const float* __restrict__ cs,
                                                             const float* __restrict__ sn, int64_t tokens,
                                                             int64_t heads, void* __restrict__ out,
                                                             const PeerRows peer = PeerRows{}) {
  constexpr int D = 128, P = 64, R = 4;
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs (q or k) are complete
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, sub = lane & 15, half = lane >> 4;
  const int64_t rows = tokens * heads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float ww[8];
  if (NORM) {
    load8f(w, sub * 8, ww);
#pragma unroll
    for (int e = 0; e < 8; e++) ww[e] += offset;
  }
  // warp-uniform loop over groups of 2 R rows; a row past the end is computed on row rows - 1 and not stored,
  // so the shuffles stay full-warp
  for (int64_t gi = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gi * 2 * R < rows; gi += warps) {
    float v[R][8], c[R][8], sv[R][8];
    int64_t base[R];
    bool live[R];
    if constexpr (TOK) {  // rows t heads + [8 k, 8 k + 8) of token t = gi / (heads / 8): every row live
      const int64_t t = gi / (heads >> 3);
#pragma unroll
      for (int r = 0; r < R; r++) {
        base[r] = (gi * 2 * R + 2 * r + half) * D + sub * 8;
        live[r] = true;
        load8<DT>(x, base[r], v[r]);
      }
      if (PAIRING == WE_ROPE_INTERLEAVED) {
        const float4 cc = *reinterpret_cast<const float4*>(cs + t * P + sub * 4);
        const float4 ss4 = *reinterpret_cast<const float4*>(sn + t * P + sub * 4);
        c[0][0] = cc.x; c[0][1] = cc.y; c[0][2] = cc.z; c[0][3] = cc.w;
        sv[0][0] = ss4.x; sv[0][1] = ss4.y; sv[0][2] = ss4.z; sv[0][3] = ss4.w;
      } else {
        load8f(cs, t * P + (sub & 7) * 8, c[0]);
        load8f(sn, t * P + (sub & 7) * 8, sv[0]);
      }
#pragma unroll
      for (int r = 1; r < R; r++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
          c[r][e] = c[0][e];
          sv[r][e] = sv[0][e];
        }
    } else {
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int64_t row0 = gi * 2 * R + 2 * r + half;
      live[r] = row0 < rows;
      const int64_t row = live[r] ? row0 : rows - 1;
      const int64_t t = row / heads;
      base[r] = row * D + sub * 8;
      load8<DT>(x, base[r], v[r]);
      if (PAIRING == WE_ROPE_INTERLEAVED) {
        const float4 cc = *reinterpret_cast<const float4*>(cs + t * P + sub * 4);
        const float4 ss4 = *reinterpret_cast<const float4*>(sn + t * P + sub * 4);
        c[r][0] = cc.x; c[r][1] = cc.y; c[r][2] = cc.z; c[r][3] = cc.w;
        sv[r][0] = ss4.x; sv[r][1] = ss4.y; sv[r][2] = ss4.z; sv[r][3] = ss4.w;
      } else {
        load8f(cs, t * P + (sub & 7) * 8, c[r]);
        load8f(sn, t * P + (sub & 7) * 8, sv[r]);
      }
    }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      if (NORM) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss = fmaf(v[r][e], v[r][e], ss);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
        for (int e = 0; e < 8; e++) v[r][e] *= inv * ww[e];
      }
      float o8[8];
      if (PAIRING == WE_ROPE_INTERLEAVED) {
#pragma unroll
        for (int g = 0; g < 4; g++) {
          o8[2 * g] = v[r][2 * g] * c[r][g] - v[r][2 * g + 1] * sv[r][g];
          o8[2 * g + 1] = v[r][2 * g + 1] * c[r][g] + v[r][2 * g] * sv[r][g];
        }
      } else {
        const bool first = sub < 8;
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float partner = __shfl_xor_sync(0xffffffffu, v[r][e], 8);
          o8[e] = first ? v[r][e] * c[r][e] - partner * sv[r][e] : v[r][e] * c[r][e] + partner * sv[r][e];
        }
      }
      if (live[r]) {
        if constexpr (PEER) {
          const int64_t row = base[r] / D, t = row / heads, h = row - t * heads, o = h / peer.hl;
          store8<OT>(peer.dst[o], ((peer.row0 + t) * peer.hl + h - o * peer.hl) * D + sub * 8, o8);
        } else {
          store8<OT>(out, base[r], o8);
        }
      }
    }
  }
  // the stores to other GPUs' memory are visible system-wide before this thread ends, so the flag barrier that
  // follows on the stream (a later kernel) publishes them
  if constexpr (PEER) __threadfence_system();
}

// RoPE, interleaved pairs (2j, 2j+1) or half pairs (j, j+P). One thread per (token, group of G pairs),
// looping over heads so each cos/sin value is loaded once per token (like the reference kernel).
template <int DT, int OT, int G, int PAIRING>
__global__ void rope_kernel(const void* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
                            int64_t tokens, int64_t heads, int64_t pairs, void* __restrict__ out) {
  int64_t groups = pairs / G;
  int64_t total = tokens * groups;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < total; it += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = it / groups, j0 = (it % groups) * G;
    float c[G], s[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
      c[g] = cs[t * pairs + j0 + g];
      s[g] = sn[t * pairs + j0 + g];
    }
    for (int64_t h = 0; h < heads; h++) {
      int64_t base = (t * heads + h) * pairs * 2;
      if (PAIRING == WE_ROPE_INTERLEAVED) {
        float v[2 * G];
        if constexpr (2 * G == 8) load8<DT>(x, base + 2 * j0, v);
        else for (int e = 0; e < 2 * G; e++) v[e] = load_act<DT>(x, base + 2 * j0 + e);
        float o[2 * G];
#pragma unroll
        for (int g = 0; g < G; g++) {
          o[2 * g] = v[2 * g] * c[g] - v[2 * g + 1] * s[g];
          o[2 * g + 1] = v[2 * g + 1] * c[g] + v[2 * g] * s[g];
        }
        if constexpr (2 * G == 8) store8<OT>(out, base + 2 * j0, o);
        else for (int e = 0; e < 2 * G; e++) store_out<OT>(out, base + 2 * j0 + e, o[e]);
      } else {
#pragma unroll
        for (int g = 0; g < G; g++) {
          float a = load_act<DT>(x, base + j0 + g), b = load_act<DT>(x, base + j0 + g + pairs);
          store_out<OT>(out, base + j0 + g, a * c[g] - b * s[g]);
          store_out<OT>(out, base + j0 + g + pairs, b * c[g] + a * s[g]);
        }
      }
    }
  }
}

// Fused q/k norm + RoPE: one warp per (token, head) row of D = 2 * pairs values; lane l holds the
// contiguous values [l V, l V + V) with V = D / 32 (D = 64, 128 or 256). Interleaved pairs stay in a
// lane; half pairing exchanges with lane l ^ 16.
template <int DT, int OT, int V, int PAIRING>
__global__ void qknorm_rope_kernel(const void* __restrict__ x, const float* __restrict__ w, float eps, float offset,
                                   const float* __restrict__ cs, const float* __restrict__ sn, int64_t tokens,
                                   int64_t heads, void* __restrict__ out) {
  constexpr int D = 32 * V, P = D / 2;
  int lane = threadIdx.x & 31;
  int64_t rows = tokens * heads;
  int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  float ww[V];
#pragma unroll
  for (int e = 0; e < V; e++) ww[e] = offset + w[lane * V + e];
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    int64_t t = row / heads;
    int64_t base = row * D + lane * V;
    float v[V];
    if constexpr (V == 8) load8<DT>(x, base, v);
    else {
#pragma unroll
      for (int e = 0; e < V; e++) v[e] = load_act<DT>(x, base + e);
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < V; e++) ss = fmaf(v[e], v[e], ss);
    float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
    for (int e = 0; e < V; e++) v[e] = v[e] * inv * ww[e];
    float o[V];
    if (PAIRING == WE_ROPE_INTERLEAVED) {
#pragma unroll
      for (int g = 0; g < V / 2; g++) {
        int64_t j = lane * (V / 2) + g;
        float c = cs[t * P + j], s = sn[t * P + j];
        o[2 * g] = v[2 * g] * c - v[2 * g + 1] * s;
        o[2 * g + 1] = v[2 * g + 1] * c + v[2 * g] * s;
      }
    } else {
      bool first = lane < 16;
#pragma unroll
      for (int e = 0; e < V; e++) {
        float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        int64_t j = (int64_t)(lane & 15) * V + e;  // pair index of this value
        float c = cs[t * P + j], s = sn[t * P + j];
        // first half: a = v, b = partner -> a c - b s ; second half: b = v, a = partner -> b c + a s
        o[e] = first ? v[e] * c - partner * s : v[e] * c + partner * s;
      }
    }
    if constexpr (V == 8) store8<OT>(out, base, o);
    else {
#pragma unroll
      for (int e = 0; e < V; e++) store_out<OT>(out, base + e, o[e]);
    }
  }
}

static int capped(int64_t want, int sms, int per_sm) {
  int64_t cap = (int64_t)sms * per_sm;
  if (want > cap) want = cap;
  return want < 1 ? 1 : (int)want;
}

template <int DT, int OT>
static void rmsnorm_dispatch(const void* x, const float* w, const float* sc, const float* sh, int64_t rows, int64_t d,
                             float eps, float offset, void* out, bool vec, int sms, cudaStream_t st) {
  if (vec && d >= 2048 && d % 8 == 0 && d <= 8192) {  // CTA per row, modulation held across rows
    // 2 chunks of 8 a thread on 128 or 192 threads up to d = 3072 (six warps measured 7 % faster there than four
    // warps with 3 chunks each), else 256 threads x up to 4; a ring of as many stages (2..4) as fit in 36 KB
    // (deeper rings measured slower: the first row of every CTA waits behind all the others)
#define WE_RNR(NT, CH)                                                                                        \
  {                                                                                                           \
    constexpr size_t per = (size_t)CH * NT * 8 * (DT == WE_F32 ? 4 : 2);                                      \
    constexpr int S = 36 * 1024 / per < 2 ? 2 : 36 * 1024 / per > 4 ? 4 : (int)(36 * 1024 / per);            \
    auto kern = rmsnorm_row_kernel<DT, OT, NT, CH, S>;                                                        \
    /* the ring plus the static reduction can pass the 48 KB a launch gets without this opt-in */             \
    (void)cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(per * S));           \
    (void)launch_pdl(kern, resident_grid(kern, NT, sms, rows, per * S), NT, per * S, st, x, w, sc, sh, rows, d, eps, \
                     offset, out);                                                                            \
    return;                                                                                                   \
  }
    const int64_t chunks = d / 8;
    if (chunks <= 128 * 2) WE_RNR(128, 2)
    if (chunks <= 192 * 2) WE_RNR(192, 2)
    if (chunks <= 256 * 3) WE_RNR(256, 3)
    WE_RNR(256, 4)
#undef WE_RNR
  }
  if constexpr (DT == WE_BF16) {
    if (vec && d <= 256 * 24) {
      const int g = capped((rows + 3) / 4, sms, 16);
      const uint16_t* xb = static_cast<const uint16_t*>(x);
      if (d <= 256 * 4) rmsnorm_warp_kernel<OT, 4><<<g, 128, 0, st>>>(xb, w, sc, sh, rows, d, eps, offset, out);
      else if (d <= 256 * 8) rmsnorm_warp_kernel<OT, 8><<<g, 128, 0, st>>>(xb, w, sc, sh, rows, d, eps, offset, out);
      else if (d <= 256 * 12) rmsnorm_warp_kernel<OT, 12><<<g, 128, 0, st>>>(xb, w, sc, sh, rows, d, eps, offset, out);
      else if (d <= 256 * 16) rmsnorm_warp_kernel<OT, 16><<<g, 128, 0, st>>>(xb, w, sc, sh, rows, d, eps, offset, out);
      else rmsnorm_warp_kernel<OT, 24><<<g, 128, 0, st>>>(xb, w, sc, sh, rows, d, eps, offset, out);
      return;
    }
  }
  if (vec && d >= 512) {
    const int64_t chunks = (d / 8 + 127) / 128;
    const int g = capped(rows, sms, 16);
    if (chunks <= 4) { rmsnorm_cached_kernel<DT, OT, 4><<<g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, out); return; }
    if (chunks <= 6) { rmsnorm_cached_kernel<DT, OT, 6><<<g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, out); return; }
    if (chunks <= 8) { rmsnorm_cached_kernel<DT, OT, 8><<<g, 128, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, out); return; }
  }
  int threads = d >= 2048 ? 256 : 128;
  int g = capped(rows, sms, 2048 / threads * 2);
  if (vec) rmsnorm_kernel<DT, OT, true><<<g, threads, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, out);
  else rmsnorm_kernel<DT, OT, false><<<g, threads, 0, st>>>(x, w, sc, sh, rows, d, eps, offset, out);
}

static bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

cudaError_t launch_rmsnorm(const void* x, int xdt, const float* w, const float* sc, const float* sh, int64_t rows,
                           int64_t d, float eps, float offset, void* out, int odt, int sms, cudaStream_t st) {
  bool vec = d % 8 == 0 && al16(x) && al16(out) && al16(w) && (!sc || al16(sc)) && (!sh || al16(sh));
  if (xdt == WE_BF16 && odt == WE_BF16) rmsnorm_dispatch<WE_BF16, WE_BF16>(x, w, sc, sh, rows, d, eps, offset, out, vec, sms, st);
  else if (xdt == WE_BF16) rmsnorm_dispatch<WE_BF16, WE_F32>(x, w, sc, sh, rows, d, eps, offset, out, vec, sms, st);
  else if (odt == WE_BF16) rmsnorm_dispatch<WE_F32, WE_BF16>(x, w, sc, sh, rows, d, eps, offset, out, vec, sms, st);
  else rmsnorm_dispatch<WE_F32, WE_F32>(x, w, sc, sh, rows, d, eps, offset, out, vec, sms, st);
  return cudaGetLastError();
}

// the 128-wide head kernel: token-grouped rows when heads % 8 == 0 (WE_QK_TOK=0 turns that off for tests),
// on a grid of every resident CTA (each warp strides over groups of 8 rows)
template <int DT, int OT, bool NORM>
static void launch_qk128(const void* x, const float* w, float eps, float offset, const float* cs, const float* sn,
                         int64_t tokens, int64_t heads, int pairing, void* out, int sms, cudaStream_t st) {
  static const bool tok_ok = [] {
    const char* e = getenv("WE_QK_TOK");
    return !(e && atoi(e) == 0);
  }();
  const int64_t groups = (tokens * heads + 7) / 8;
#define WE_QK(PAIR, TOK)                                                                                       \
  {                                                                                                            \
    auto kern = qknorm_rope128_kernel<DT, OT, PAIR, NORM, TOK>;                                                \
    (void)launch_pdl(kern, resident_grid(kern, 256, sms, (groups + 7) / 8), 256, 0, st, x, w, eps, offset, cs, sn, \
                     tokens, heads, out, PeerRows{});                                                          \
  }
  const bool tok = tok_ok && heads % 8 == 0;
  if (pairing == WE_ROPE_INTERLEAVED) {
    if (tok) WE_QK(WE_ROPE_INTERLEAVED, true) else WE_QK(WE_ROPE_INTERLEAVED, false)
  } else {
    if (tok) WE_QK(WE_ROPE_HALF, true) else WE_QK(WE_ROPE_HALF, false)
  }
#undef WE_QK
}

template <int DT, int OT>
static void rope_dispatch(const void* x, const float* cs, const float* sn, int64_t tokens, int64_t heads, int64_t pairs,
                          int pairing, void* out, bool vec, int sms, cudaStream_t st) {
  if (pairs == 64 && vec && ((uintptr_t)cs & 15) == 0 && ((uintptr_t)sn & 15) == 0) {  // 128-wide heads: row layout
    launch_qk128<DT, OT, false>(x, nullptr, 0.f, 0.f, cs, sn, tokens, heads, pairing, out, sms, st);
    return;
  }
  int threads = 128;
  if (pairing == WE_ROPE_INTERLEAVED) {
    if (vec) {
      int g = capped((tokens * (pairs / 4) + threads - 1) / threads, sms, 16);
      rope_kernel<DT, OT, 4, WE_ROPE_INTERLEAVED><<<g, threads, 0, st>>>(x, cs, sn, tokens, heads, pairs, out);
    } else {
      int g = capped((tokens * pairs + threads - 1) / threads, sms, 16);
      rope_kernel<DT, OT, 1, WE_ROPE_INTERLEAVED><<<g, threads, 0, st>>>(x, cs, sn, tokens, heads, pairs, out);
    }
  } else {
    int g = capped((tokens * pairs + threads - 1) / threads, sms, 16);
    rope_kernel<DT, OT, 1, WE_ROPE_HALF><<<g, threads, 0, st>>>(x, cs, sn, tokens, heads, pairs, out);
  }
}

cudaError_t launch_rope(const void* x, int xdt, const float* cs, const float* sn, int64_t tokens, int64_t heads,
                        int64_t pairs, int pairing, void* out, int odt, int sms, cudaStream_t st) {
  bool vec = pairs % 4 == 0 && al16(x) && al16(out);
  if (xdt == WE_BF16 && odt == WE_BF16) rope_dispatch<WE_BF16, WE_BF16>(x, cs, sn, tokens, heads, pairs, pairing, out, vec, sms, st);
  else if (xdt == WE_BF16) rope_dispatch<WE_BF16, WE_F32>(x, cs, sn, tokens, heads, pairs, pairing, out, vec, sms, st);
  else if (odt == WE_BF16) rope_dispatch<WE_F32, WE_BF16>(x, cs, sn, tokens, heads, pairs, pairing, out, vec, sms, st);
  else rope_dispatch<WE_F32, WE_F32>(x, cs, sn, tokens, heads, pairs, pairing, out, vec, sms, st);
  return cudaGetLastError();
}

template <int DT, int OT, int V>
static void qk_dispatch2(const void* x, const float* w, float eps, float offset, const float* cs, const float* sn,
                         int64_t tokens, int64_t heads, int pairing, void* out, int sms, cudaStream_t st) {
  int threads = 256;
  int64_t rows = tokens * heads;
  int g = capped((rows + 7) / 8, sms, 8);
  if (pairing == WE_ROPE_INTERLEAVED)
    qknorm_rope_kernel<DT, OT, V, WE_ROPE_INTERLEAVED><<<g, threads, 0, st>>>(x, w, eps, offset, cs, sn, tokens, heads, out);
  else
    qknorm_rope_kernel<DT, OT, V, WE_ROPE_HALF><<<g, threads, 0, st>>>(x, w, eps, offset, cs, sn, tokens, heads, out);
}

template <int DT, int OT>
static bool qk_dispatch(const void* x, const float* w, float eps, float offset, const float* cs, const float* sn,
                        int64_t tokens, int64_t heads, int64_t pairs, int pairing, void* out, int sms, cudaStream_t st) {
  if (pairs * 2 == 128 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0 && ((uintptr_t)cs & 15) == 0 &&
      ((uintptr_t)sn & 15) == 0) {
    launch_qk128<DT, OT, true>(x, w, eps, offset, cs, sn, tokens, heads, pairing, out, sms, st);
    return true;
  }
  switch (pairs * 2) {
    case 64: qk_dispatch2<DT, OT, 2>(x, w, eps, offset, cs, sn, tokens, heads, pairing, out, sms, st); return true;
    case 128: qk_dispatch2<DT, OT, 4>(x, w, eps, offset, cs, sn, tokens, heads, pairing, out, sms, st); return true;
    case 256: qk_dispatch2<DT, OT, 8>(x, w, eps, offset, cs, sn, tokens, heads, pairing, out, sms, st); return true;
    default: return false;
  }
}

// Returns cudaErrorNotSupported when the head size has no fused variant (the caller then runs
// rmsnorm + rope as two passes).
cudaError_t launch_qknorm_rope_peers(const void* x, const float* w, float eps, float offset, const float* cs,
                                     const float* sn, int64_t tokens, int64_t heads, int pairing, void* const* dst,
                                     int world, int64_t row0, int sms, cudaStream_t st) {
  if (world < 1 || world > WE_PEER_MAX || heads % world || !al16(x) || ((uintptr_t)cs & 15) || ((uintptr_t)sn & 15))
    return cudaErrorNotSupported;
  PeerRows pr{};
  for (int r = 0; r < world; r++) {
    if (!dst[r] || ((uintptr_t)dst[r] & 15)) return cudaErrorNotSupported;
    pr.dst[r] = dst[r];
  }
  pr.row0 = row0;
  pr.hl = heads / world;
  const int64_t groups = (tokens * heads + 7) / 8;
  const bool tok = heads % 8 == 0;
#define WE_QKP(PAIR, TOK)                                                                                      \
  {                                                                                                            \
    auto kern = qknorm_rope128_kernel<WE_BF16, WE_BF16, PAIR, true, TOK, true>;                                \
    return launch_pdl(kern, resident_grid(kern, 256, sms, (groups + 7) / 8), 256, 0, st, x, w, eps, offset, cs, sn, \
                      tokens, heads, (void*)nullptr, pr);                                                      \
  }
  if (pairing == WE_ROPE_INTERLEAVED) {
    if (tok) WE_QKP(WE_ROPE_INTERLEAVED, true) else WE_QKP(WE_ROPE_INTERLEAVED, false)
  } else {
    if (tok) WE_QKP(WE_ROPE_HALF, true) else WE_QKP(WE_ROPE_HALF, false)
  }
#undef WE_QKP
}

cudaError_t launch_qknorm_rope(const void* x, int xdt, const float* w, float eps, float offset, const float* cs,
                               const float* sn, int64_t tokens, int64_t heads, int64_t pairs, int pairing, void* out,
                               int odt, int sms, cudaStream_t st) {
  if (pairs * 2 == 256 && !(al16(x) && al16(out))) return cudaErrorNotSupported;
  bool ok;
  if (xdt == WE_BF16 && odt == WE_BF16) ok = qk_dispatch<WE_BF16, WE_BF16>(x, w, eps, offset, cs, sn, tokens, heads, pairs, pairing, out, sms, st);
  else if (xdt == WE_BF16) ok = qk_dispatch<WE_BF16, WE_F32>(x, w, eps, offset, cs, sn, tokens, heads, pairs, pairing, out, sms, st);
  else if (odt == WE_BF16) ok = qk_dispatch<WE_F32, WE_BF16>(x, w, eps, offset, cs, sn, tokens, heads, pairs, pairing, out, sms, st);
  else ok = qk_dispatch<WE_F32, WE_F32>(x, w, eps, offset, cs, sn, tokens, heads, pairs, pairing, out, sms, st);
  if (!ok) return cudaErrorNotSupported;
  return cudaGetLastError();
}

}  // namespace we
