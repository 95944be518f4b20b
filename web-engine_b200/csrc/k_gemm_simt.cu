// CUDA-core GEMM with the full reference matmul semantics (src/kernels/matmul.ts:118-178):
// y = x . W^T * scale with f32 or bf16 x, W in f32 / bf16 / fp8 / int4-g64, row strides and offsets,
// split-K partials and accumulate mode. fp32 FMA accumulation in K order, like the reference shader.
//
// This is the exact path for f32 activations (the reference's own input type) and for layouts the
// tensor-core kernel cannot take (rows not 16-byte aligned, K not a multiple of 16 bytes, split-K).
// bf16 activations on aligned layouts go to the tcgen05 kernel (k_gemm_tc.cu).
#include "common.cuh"
#include "kernels.h"

namespace we {

constexpr int SB_M = 64, SB_N = 64, SB_K = 16, SB_T = 256;

template <int WT>
__device__ __forceinline__ float load_w(const void* w, int64_t idx, const uint16_t* gs, int64_t groups, int64_t row,
                                        int64_t kk) {
  if constexpr (WT == WE_F32) return static_cast<const float*>(w)[idx];
  else if constexpr (WT == WE_BF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(w)[idx]);
  else if constexpr (WT == WE_FP8) return e4m3_to_f32(static_cast<const uint8_t*>(w)[idx]);
  else {
    uint8_t b = static_cast<const uint8_t*>(w)[idx >> 1];
    uint32_t nib = (idx & 1) ? (b >> 4) : (b & 0xf);
    float s = __half2float(__ushort_as_half(gs[row * groups + kk / 64]));
    return int4_operand(nib, s);
  }
}

template <int XT, int WT, int YT>
__global__ void __launch_bounds__(SB_T) gemm_simt_kernel(const void* __restrict__ x, const void* __restrict__ w, void* __restrict__ y,
                                                      MatmulArgs a) {
  __shared__ float xs[SB_K][SB_M + 4];
  __shared__ float ws[SB_K][SB_N + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t row0 = (int64_t)blockIdx.y * SB_M, col0 = (int64_t)blockIdx.x * SB_N;
  int64_t kb = 0, ke = a.k;
  if (a.k_split > 1) {
    int64_t kc = ((a.k + a.k_split - 1) / a.k_split + 15) / 16 * 16;
    kb = blockIdx.z * kc;
    ke = kb + kc < a.k ? kb + kc : a.k;
  }
  const int64_t groups = a.k / 64;
  float acc[4][4] = {};
  for (int64_t k0 = kb; k0 < ke; k0 += SB_K) {
    for (int e = threadIdx.x; e < SB_M * SB_K; e += SB_T) {
      int r = e / SB_K, kk = e % SB_K;
      int64_t gr = row0 + r, gk = k0 + kk;
      xs[kk][r] = (gr < a.m && gk < ke) ? load_act<XT>(x, a.x_offset + gr * a.x_stride + gk) : 0.f;
      int64_t gc = col0 + r;
      ws[kk][r] = (gc < a.n && gk < ke) ? load_w<WT>(w, a.w_offset + gc * a.w_stride + gk, a.group_scale, groups, gc, gk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; kk++) {
      float xa[4], wb[4];
#pragma unroll
      for (int i = 0; i < 4; i++) xa[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) wb[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(xa[i], wb[j], acc[i][j]);
    }
    __syncthreads();
  }
  const int64_t zrows = a.k_split > 1 ? (int64_t)blockIdx.z * a.m : 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int64_t r = row0 + ty * 4 + i;
    if (r >= a.m) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int64_t c = col0 + tx * 4 + j;
      if (c >= a.n) continue;
      float sc = a.chan_scale ? a.chan_scale[c] : a.scale;
      float v = acc[i][j] * sc;
      if (a.bias) v += a.bias[c];
      int64_t o = a.y_offset + (zrows + r) * a.y_stride + c;
      v = act_apply(a.epi.act, v);
      if (a.epi.aux_op) {
        const int64_t oa = (zrows + r) * a.y_stride + c;  // aux is offset like y
        const float ax = a.epi.aux_dtype == WE_BF16 ? load_act<WE_BF16>(a.epi.aux, oa) : load_act<WE_F32>(a.epi.aux, oa);
        v = aux_apply(a.epi.aux_op, ax, v);
      }
      if (a.epi.gate) v *= a.epi.gate[c];
      if (a.accumulate) v += load_act<YT>(y, o);
      store_out<YT>(y, o, v);
    }
  }
}

template <int XT, int WT>
static void simt_y(const void* x, const void* w, void* y, const MatmulArgs& a, dim3 g, cudaStream_t st) {
  if (a.y_dtype == WE_BF16) gemm_simt_kernel<XT, WT, WE_BF16><<<g, SB_T, 0, st>>>(x, w, y, a);
  else gemm_simt_kernel<XT, WT, WE_F32><<<g, SB_T, 0, st>>>(x, w, y, a);
}
template <int XT>
static void simt_w(const void* x, const void* w, void* y, const MatmulArgs& a, dim3 g, cudaStream_t st) {
  switch (a.w_dtype) {
    case WE_F32: simt_y<XT, WE_F32>(x, w, y, a, g, st); break;
    case WE_BF16: simt_y<XT, WE_BF16>(x, w, y, a, g, st); break;
    case WE_FP8: simt_y<XT, WE_FP8>(x, w, y, a, g, st); break;
    default: simt_y<XT, WE_INT4G64>(x, w, y, a, g, st); break;
  }
}

cudaError_t launch_gemm_simt(const void* x, const void* w, void* y, const MatmulArgs& a, cudaStream_t st) {
  dim3 g((unsigned)((a.n + SB_N - 1) / SB_N), (unsigned)((a.m + SB_M - 1) / SB_M), (unsigned)(a.k_split > 1 ? a.k_split : 1));
  if (g.y > 65535) return cudaErrorInvalidValue;
  if (a.x_dtype == WE_BF16) simt_w<WE_BF16>(x, w, y, a, g, st);
  else simt_w<WE_F32>(x, w, y, a, g, st);
  return cudaGetLastError();
}

}  // namespace we
