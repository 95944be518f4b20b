// Latent <-> token layout of the step driver (src/model/transformer.ts:53-82), on the device so a step's
// latent goes host -> HBM once and never comes back through the CPU for reshaping.
//
//   patchify:   latent [C, H, W] -> tokens [ceil(H/2) * ceil(W/2), 4C], feature (c, patch row, patch col);
//               an odd H or W wraps to row / column 0 (ComfyUI pad_to_patch_size, transformer.ts:55-69)
//   unpatchify: the inverse; the padding is cropped off (transformer.ts:72-82)
//
// Pure data movement, one thread per output element: the writes are coalesced, the reads are a 2-strided
// gather that stays in L1/L2 (a 1024x1024 image's latent is 1 MB). Bit-exact by construction.
#include "common.cuh"
#include "kernels.h"

namespace we {

template <int IT, int OT>
__global__ void patchify_kernel(const void* __restrict__ latent, void* __restrict__ tokens, int64_t C, int64_t H,
                                int64_t W, int64_t cols, int64_t total) {
  const int64_t feat = 4 * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / feat, f = i - tok * feat;
    const int64_t ch = f >> 2, pr = (f >> 1) & 1, pc = f & 1;
    const int64_t r = tok / cols, c = tok - r * cols;
    const int64_t y = (2 * r + pr) % H, x = (2 * c + pc) % W;
    store_out<OT>(tokens, i, load_act<IT>(latent, (ch * H + y) * W + x));
  }
}

template <int IT, int OT>
__global__ void unpatchify_kernel(const void* __restrict__ tokens, void* __restrict__ latent, int64_t C, int64_t H,
                                  int64_t W, int64_t cols, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ch = i / (H * W), rem = i - ch * H * W;
    const int64_t y = rem / W, x = rem - y * W;
    const int64_t tok = (y >> 1) * cols + (x >> 1);
    store_out<OT>(latent, i, load_act<IT>(tokens, tok * 4 * C + ch * 4 + (y & 1) * 2 + (x & 1)));
  }
}

#define WE_LAYOUT_LAUNCH(KERNEL)                                                                                  \
  template <int IT>                                                                                             \
  static void KERNEL##_out(const void* in, void* out, int odt, int64_t C, int64_t H, int64_t W, int64_t cols,    \
                           int64_t total, unsigned grid, cudaStream_t st) {                                    \
    if (odt == WE_BF16) KERNEL##_kernel<IT, WE_BF16><<<grid, 256, 0, st>>>(in, out, C, H, W, cols, total);     \
    else KERNEL##_kernel<IT, WE_F32><<<grid, 256, 0, st>>>(in, out, C, H, W, cols, total);                     \
  }
WE_LAYOUT_LAUNCH(patchify)
WE_LAYOUT_LAUNCH(unpatchify)
#undef WE_LAYOUT_LAUNCH

static unsigned layout_grid(int64_t total, int sms) {
  int64_t g = (total + 255) / 256, cap = (int64_t)sms * 8;
  return (unsigned)(g < cap ? (g > 0 ? g : 1) : cap);
}

cudaError_t launch_patchify(const void* latent, int ldt, int64_t C, int64_t H, int64_t W, void* tokens, int tdt,
                            int sms, cudaStream_t st) {
  const int64_t rows = (H + 1) / 2, cols = (W + 1) / 2, total = rows * cols * 4 * C;
  const unsigned g = layout_grid(total, sms);
  if (ldt == WE_BF16) patchify_out<WE_BF16>(latent, tokens, tdt, C, H, W, cols, total, g, st);
  else patchify_out<WE_F32>(latent, tokens, tdt, C, H, W, cols, total, g, st);
  return cudaGetLastError();
}

cudaError_t launch_unpatchify(const void* tokens, int tdt, int64_t C, int64_t H, int64_t W, void* latent, int ldt,
                              int sms, cudaStream_t st) {
  const int64_t cols = (W + 1) / 2, total = C * H * W;
  const unsigned g = layout_grid(total, sms);
  if (tdt == WE_BF16) unpatchify_out<WE_BF16>(tokens, latent, ldt, C, H, W, cols, total, g, st);
  else unpatchify_out<WE_F32>(tokens, latent, ldt, C, H, W, cols, total, g, st);
  return cudaGetLastError();
}

}  // namespace we

namespace we {

// Head-group exchange layout of sequence parallelism: rows [tokens, groups * hg, row_bytes] (token-major, a
// rank's token shard with every head) <-> [groups, tokens, hg, row_bytes] (head-group-major: chunk g is what
// rank g receives). `to_groups` picks the direction. One thread moves 16 bytes; row_bytes % 16 == 0.
__global__ void head_groups_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t tokens,
                                   int64_t groups, int64_t hg_vec, int to_groups, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    // i indexes the token-major layout: (t, g, v) with v < hg_vec 16-byte words per (token, group)
    const int64_t v = i % hg_vec, tg = i / hg_vec;
    const int64_t g = tg % groups, t = tg / groups;
    const int64_t j = (g * tokens + t) * hg_vec + v;  // the same word in the group-major layout
    if (to_groups) dst[j] = src[i];
    else dst[i] = src[j];
  }
}

cudaError_t launch_head_groups(const void* src, void* dst, int64_t tokens, int64_t groups, int64_t group_bytes,
                               int to_groups, int sms, cudaStream_t st) {
  const int64_t hg_vec = group_bytes / 16, total = tokens * groups * hg_vec;
  if (total <= 0) return cudaSuccess;
  const unsigned g = layout_grid(total, sms);
  head_groups_kernel<<<g, 256, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), tokens, groups,
                                        hg_vec, to_groups, total);
  return cudaGetLastError();
}

}  // namespace we
