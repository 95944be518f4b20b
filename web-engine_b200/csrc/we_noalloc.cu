// we_matmul_fp8_noalloc: the bf16 x fp8 linear (activation split + tcgen05 GEMM) for callers that cannot
// allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at all: a real-time or serving loop whose device
// memory budget is fixed when it starts, or an embedding runtime (a framework plugin that is handed only
// streams and tensor pointers) whose own allocator owns every byte of device memory. The regular path (we_matmul /
// we_linear_forward) takes its scratch for the activation split from the context's pool, and that
// pool grows with cudaMalloc. This entry point needs no context and allocates nothing. Its scratch is
// one file-scope device array of WE_NOALLOC_SCRATCH_BYTES, which the CUDA runtime creates on every GPU
// that loads this library and which stays there until the process exits.
//
// The array's name is a host-side stand-in in host code, not a device address. Its device address is
// looked up with cudaGetSymbolAddress, with the device current, once per CUDA context: the set-up is keyed
// by the current context's unique ID (cuCtxGetId), so a context created after cudaDeviceReset, or a
// non-primary context a host made with cuCtxCreate, gets its own lookup instead of an address that belongs
// to another context.
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

// The shared scratch of every call on a device: the e4m3 activation planes and the row scales.
static __device__ __align__(256) uint8_t g_noalloc_scratch[WE_NOALLOC_SCRATCH_BYTES];
// Device error word for the GEMM's bounded waits (cleared at the start of every call).
static __device__ __align__(256) uint32_t g_noalloc_err[4];

constexpr int kMaxDevices = 64;
struct DeviceSlots {
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch in the context ctx_id
  uint32_t* err = nullptr;     // device address of g_noalloc_err in the context ctx_id
  int sms = 0;
  unsigned long long ctx_id = 0;
  bool ready = false;
};
DeviceSlots g_slots[kMaxDevices];
std::mutex g_setup;

int report(char* errbuf, size_t errlen, int code, const char* fmt, long long a = 0, long long b = 0) {
  if (errbuf && errlen) snprintf(errbuf, errlen, fmt, a, b);
  return code;
}

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

// The unique ID of the calling thread's current CUDA context (driver entry points, no libcuda link).
bool current_context_id(unsigned long long* id) {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  if (!get_current || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int we_matmul_fp8_noalloc(void* stream, const void* x, int64_t m, int64_t k, int64_t x_stride,
                                     const uint8_t* w, int64_t n, float scale, const float* chan_scale,
                                     const float* bias, void* y, int64_t y_stride, int32_t y_dtype, uint32_t flags,
                                     char* errbuf, size_t errlen) {
  if (errbuf && errlen) errbuf[0] = 0;
  if (m < 0 || n < 0 || k < 0) return report(errbuf, errlen, WE_EINVAL, "m, n and k must not be negative");
  if (x_stride < 0 || (x_stride > 0 && x_stride < k))
    return report(errbuf, errlen, WE_EINVAL, "x_stride must be 0 or at least k (%lld), got %lld", k, x_stride);
  if (y_stride < 0 || (y_stride > 0 && y_stride < n))
    return report(errbuf, errlen, WE_EINVAL, "y_stride must be 0 or at least n (%lld), got %lld", n, y_stride);
  if (m == 0 || n == 0) return WE_OK;
  if (!x || !w || !y) return report(errbuf, errlen, WE_EINVAL, "x, w and y must be device pointers");
  if (y_dtype != WE_F32 && y_dtype != WE_BF16) return report(errbuf, errlen, WE_EINVAL, "y must be f32 or bf16");
  if (k % 16 != 0)
    return report(errbuf, errlen, WE_EINVAL, "K must be a multiple of 16 for the tensor-core path, got %lld", k);
  if (((uintptr_t)w & 15) != 0) return report(errbuf, errlen, WE_EINVAL, "w must be 16-byte aligned");
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
    return report(errbuf, errlen, WE_EINVAL, "m, n and k must be below 2^31");
  const int terms = (flags & WE_MM_FP8_FAST) ? 1 : 2;
  const size_t plane = round256((size_t)m * (size_t)k);
  const size_t need = (size_t)terms * plane + round256((size_t)m * 4);
  if (need > (size_t)WE_NOALLOC_SCRATCH_BYTES)
    return report(errbuf, errlen, WE_EINVAL,
                  "activation split needs %lld bytes of scratch; the static scratch holds %lld (reduce m * k)",
                  (long long)need, (long long)WE_NOALLOC_SCRATCH_BYTES);

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return report(errbuf, errlen, WE_ECUDA, "no current CUDA device (or device index >= 64)");
  cudaError_t e = cudaSuccess;
  unsigned long long ctx_id = 0;
  if (!current_context_id(&ctx_id)) {
    // no context is current on this thread yet: a symbol lookup makes the runtime bind the device's primary
    // context (it allocates nothing beyond the module's own arrays)
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_err);
    if (e != cudaSuccess || !current_context_id(&ctx_id))
      return report(errbuf, errlen, WE_ECUDA, "no usable CUDA context (error %lld)", (long long)e);
  }
  DeviceSlots slot;
  {
    // once per device and context, with that device current: the device addresses of the file-scope arrays
    std::lock_guard<std::mutex> lock(g_setup);
    DeviceSlots* s = &g_slots[dev];
    if (!s->ready || s->ctx_id != ctx_id) {
      s->ready = false;
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess)
        return report(errbuf, errlen, WE_ECUDA, "cudaGetSymbolAddress(scratch) failed (error %lld)", (long long)e);
      s->scratch = static_cast<uint8_t*>(p);
      e = cudaGetSymbolAddress(&p, g_noalloc_err);
      if (e != cudaSuccess)
        return report(errbuf, errlen, WE_ECUDA, "cudaGetSymbolAddress(error word) failed (error %lld)", (long long)e);
      s->err = static_cast<uint32_t*>(p);
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      s->sms = sms > 0 ? sms : 148;
      s->ctx_id = ctx_id;
      s->ready = true;
    }
    slot = *s;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* hi = slot.scratch;
  uint8_t* lo = terms > 1 ? slot.scratch + plane : nullptr;
  float* rs = reinterpret_cast<float*>(slot.scratch + (size_t)terms * plane);

  // the error word must start at zero; the split overwrites every scratch byte the GEMM reads
  e = cudaMemsetAsync(slot.err, 0, sizeof(uint32_t), st);
  if (e == cudaSuccess)
    e = we::launch_quant_act(x, WE_BF16, m, k, x_stride ? x_stride : k, terms, hi, lo, rs, slot.sms, st);
  if (e != cudaSuccess) return report(errbuf, errlen, WE_ECUDA, "activation split launch failed (error %lld)", (long long)e);

  we::TcGemmArgs t{};
  t.m = m;
  t.n = n;
  t.k = k;
  t.kind_f16 = 0;
  t.terms = terms;
  t.x[0] = hi;
  t.x[1] = lo ? lo : hi;
  t.x_stride_bytes = k;
  t.w = w;
  t.w_stride_bytes = k;
  t.row_scale = rs;
  t.scale = scale;
  t.chan_scale = chan_scale;
  t.bias = bias;
  t.y = y;
  t.y_stride = y_stride ? y_stride : n;
  t.y_dtype = y_dtype;
  t.accumulate = (flags & WE_MM_ACCUMULATE) ? 1 : 0;
  t.dev_err = slot.err;
  if (!we::gemm_tc_supported(t))
    return report(errbuf, errlen, WE_EINVAL,
                  "the tcgen05 GEMM cannot take this layout: K %% 16 == 0, w 16-byte aligned, m, n, k below 2^31");
  e = we::launch_gemm_tc(t, slot.sms, st);
  if (e == cudaErrorNotSupported)
    return report(errbuf, errlen, WE_EINVAL,
                  "the tcgen05 GEMM refused this layout (its TMA descriptors need 16-byte aligned rows of w)");
  if (e != cudaSuccess) return report(errbuf, errlen, WE_ECUDA, "tcgen05 GEMM launch failed (error %lld)", (long long)e);

  if (flags & WE_NOALLOC_SYNC) {
    uint32_t code = 0;
    e = cudaMemcpyAsync(&code, slot.err, sizeof(code), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return report(errbuf, errlen, WE_ECUDA, "synchronising the stream failed (error %lld)", (long long)e);
    if (code) return report(errbuf, errlen, WE_ETIMEOUT, "a bounded wait in the GEMM gave up (code %lld)", (long long)code);
  }
  return WE_OK;
}
