// Shared device helpers for the web-engine B200 kernels (sm_100a only).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/we_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "web-engine B200 kernels target sm_100a only"
#endif

namespace we {

// Device error word codes (written by bounded waits; read by we_device_error).
enum : uint32_t {
  DEV_ERR_NONE = 0,
  DEV_ERR_TIMEOUT_PRODUCER = 1,
  DEV_ERR_TIMEOUT_MMA = 2,
  DEV_ERR_TIMEOUT_EPILOGUE = 3,
  DEV_ERR_TIMEOUT_DRAIN = 4,
  DEV_ERR_TIMEOUT_PEER = 5,  // a peer exchange waited longer than its timeout for another rank's flag
};

// ---- element decode / encode ----
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// e4m3fn byte -> f32 (exact). Same decode as src/kernels/fp8.ts:12-20 (NaN codes not special-cased).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  uint32_t e = (b >> 3) & 0xfu, m = b & 7u;
  float normal = __uint_as_float(((e + 120u) << 23) | (m << 20));
  float sub = float(m) * 0.001953125f;  // m/8 * 2^-6
  float v = e == 0 ? sub : normal;
  return (b & 0x80u) ? -v : v;
}

// two e4m3 values (low byte first) -> two f32, by the hardware converter (exact)
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint16_t two) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(two, __NV_E4M3);
  __half2 hh = *reinterpret_cast<__half2*>(&h);
  return __half22float2(hh);
}

// f32 -> e4m3, round to nearest even, saturating to +-448 (NaN -> 0x7f)
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

template <int DT>
__device__ __forceinline__ float load_act(const void* p, int64_t i) {
  if constexpr (DT == WE_F32) return static_cast<const float*>(p)[i];
  else return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
}
template <int DT>
__device__ __forceinline__ void store_out(void* p, int64_t i, float v) {
  if constexpr (DT == WE_F32) static_cast<float*>(p)[i] = v;
  else static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
}

// int4 group-64 operand: bf16_rne(q * float(s)), q two's complement nibble
__device__ __forceinline__ float int4_operand(uint32_t nib, float s) {
  int q = int(nib ^ 8u) - 8;
  return bf16_bits_to_f32(f32_to_bf16_bits(float(q) * s));
}

// 8 values of an activation row as floats: one 16-byte load for bf16, two for f32
template <int DT>
__device__ __forceinline__ void load8(const void* p, int64_t i, float v[8]) {
  if constexpr (DT == WE_BF16) {
    uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  } else {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    float4 a = q[0], b = q[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}
template <int DT>
__device__ __forceinline__ void store8(void* p, int64_t i, const float v[8]) {
  if constexpr (DT == WE_BF16) {
    uint4 u = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = u;
  } else {
    float4* q = reinterpret_cast<float4*>(static_cast<float*>(p) + i);
    q[0] = make_float4(v[0], v[1], v[2], v[3]);
    q[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}
__device__ __forceinline__ void load8f(const float* p, int64_t i, float v[8]) {
  const float4* q = reinterpret_cast<const float4*>(p + i);
  float4 a = q[0], b = q[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ---- the per-value steps of a block (src/kernels/elementwise.ts:22-29) ----
__device__ __forceinline__ float sigmoid_ref(float v) { return 1.f / (1.f + expf(-v)); }
// PyTorch GELU(approximate="tanh"), tanh written with exp and clamped like the reference shader
__device__ __forceinline__ float gelu_tanh_ref(float v) {
  const float u = fminf(fmaxf(0.7978845608028654f * (v + 0.044715f * v * v * v), -15.f), 15.f);
  const float e = expf(2.f * u);
  return 0.5f * v * (1.f + (e - 1.f) / (e + 1.f));
}
__device__ __forceinline__ float act_apply(int act, float v) {
  return act == WE_ACT_GELU_TANH ? gelu_tanh_ref(v) : (act == WE_ACT_SILU ? v * sigmoid_ref(v) : v);
}
__device__ __forceinline__ float aux_apply(int op, float aux, float v) {
  return op == WE_AUX_SIGMOID_GATE ? aux * sigmoid_ref(v) : (op == WE_AUX_SWIGLU ? aux * sigmoid_ref(aux) * v : v);
}

// The GEMM epilogue's forms of the same functions, on the hardware exp2 / reciprocal approximations
// (__expf, __fdividef: a few ulp): tanh-GELU through the identity 0.5 (1 + tanh u) = 1 / (1 + e^(-2u)), so
// gelu(v) = v / (1 + e^(-2u)). Both limits are exact: e^(-2u) -> inf gives -0, -> 0 gives v.
__device__ __forceinline__ float sigmoid_fast(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }
__device__ __forceinline__ float gelu_tanh_fast(float v) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * v, v * v, v);
  return __fdividef(v, 1.f + __expf(-2.f * u));
}

// The hardware 2^x and 1/x (MUFU.EX2, MUFU.RCP; subnormal results flush to zero).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// GELU (tanh form) of two values with packed f32x2 arithmetic: v sigma(2u) = v / (1 + 2^x), where
// x = -2 log2(e) sqrt(2/pi) (v + 0.044715 v^3) = v (K1 + K2 v^2). Same function as gelu_tanh_fast, about half the
// instructions: the GEMM epilogue that applies it is bound by instruction issue.
__device__ __forceinline__ float2 gelu_tanh2(float2 v) {
  constexpr float K1 = -2.302208198144325f, K2 = -0.1029432395800235f;
  const float2 x = __fmul2_rn(v, __ffma2_rn(__fmul2_rn(v, v), make_float2(K2, K2), make_float2(K1, K1)));
  const float2 d = __fadd2_rn(make_float2(ex2_ftz(x.x), ex2_ftz(x.y)), make_float2(1.f, 1.f));
  return __fmul2_rn(v, make_float2(rcp_ftz(d.x), rcp_ftz(d.y)));
}
// SiLU of two values: v / (1 + 2^(-v log2 e)).
__device__ __forceinline__ float2 silu2(float2 v) {
  constexpr float NL2E = -1.4426950408889634f;
  const float2 x = __fmul2_rn(v, make_float2(NL2E, NL2E));
  const float2 d = __fadd2_rn(make_float2(ex2_ftz(x.x), ex2_ftz(x.y)), make_float2(1.f, 1.f));
  return __fmul2_rn(v, make_float2(rcp_ftz(d.x), rcp_ftz(d.y)));
}

// Grid of a row-loop kernel: as many CTAs as fit on the SMs at once (each then walks its rows, and a kernel that
// prefetches its next row keeps those loads in flight), at most one per row.
template <typename K>
static inline unsigned resident_grid(K kernel, int threads, int sms, int64_t rows, size_t smem = 0) {
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem) != cudaSuccess || per < 1) per = 1;
  const int64_t g = (int64_t)per * sms;
  return (unsigned)(rows < g ? rows : g);
}

// ---- warp reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- programmatic dependent launch (griddepcontrol) ----
// A kernel launched by launch_pdl may begin while the kernel before it in the stream is still finishing: its CTAs
// are placed as that kernel's CTAs leave the SMs, so the launch latency and the block scheduling overlap the
// previous kernel's tail. Such a kernel calls pdl_wait() in every CTA before its first global memory access (read
// or write): the wait returns once the previous kernel has completed and its writes are visible, and calling it
// unconditionally keeps "this kernel completed" implying "every earlier kernel completed" for the next one.
// pdl_launch_dependents() lets the next kernel's CTAs be placed once every CTA of this one has started.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// WE_PDL=0 launches the pdl kernels as ordinary stream-ordered launches (their pdl_wait then returns at once).
static inline bool pdl_enabled() {
  static const bool on = [] {
    const char* env = getenv("WE_PDL");
    return !(env && env[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem,
                                     cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// the programmatic-serialization attribute for a launch that sets its own other attributes
static inline void pdl_attribute(cudaLaunchAttribute& a) {
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
}

// ---- cp.async: a thread's own global -> shared copies, in flight without holding registers ----
// A thread that reads back only the bytes it copied itself needs no barrier: cp.async.wait_group orders them.
// `smem` is a shared-memory address (__cvta_generic_to_shared).
__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// max over the warp's 32 lanes of |v| (sm_100a redux.sync; NaN lanes are ignored, as fmaxf does)
__device__ __forceinline__ float warp_max_abs(float v) {
  float r;
  asm volatile("redux.sync.max.abs.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Exponent e of the activation split's row scale 2^e for a row maximum |x| = amax: the smallest e with
// amax 2^-e <= 448 when amax's mantissa is at most 1.75 (E - 9), else one more (E - 8), amax = f 2^E, f in [0.5, 1).
// Normal amax by its bits, the rest (0, subnormal, inf, NaN) by frexpf.
__device__ __forceinline__ int split_exponent(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const uint32_t ex = (b >> 23) & 0xffu;
  if (ex != 0u && ex != 0xffu && !(b >> 31)) return (int)ex - 126 - ((b & 0x7fffffu) <= 0x600000u ? 9 : 8);
  if (!(amax > 0.f)) return 0;
  int E;
  const float f = frexpf(amax, &E);
  return (2.f * f <= 1.75f) ? E - 9 : E - 8;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

}  // namespace we
