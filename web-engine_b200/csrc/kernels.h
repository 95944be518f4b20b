// Host-side launch interfaces of the web-engine B200 kernels (internal to the library).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/we_b200.h"

namespace we {

// Fused epilogue steps after v = acc * scales + bias (see we_epilogue in the public header).
struct EpiOps {
  int act = 0;
  int aux_op = 0;
  int aux_dtype = 0;
  const void* aux = nullptr;  // [m, n] with y's stride (already offset like y)
  const float* gate = nullptr;
};

// Resolved matmul arguments (values, not bytes; strides already defaulted).
struct MatmulArgs {
  int64_t m, n, k;
  int64_t x_stride, w_stride, y_stride, x_offset, w_offset, y_offset;
  int64_t k_split;
  float scale;
  const float* chan_scale;
  const uint16_t* group_scale;
  const float* bias;
  int x_dtype, w_dtype, y_dtype;
  int accumulate;
  EpiOps epi;
};

cudaError_t launch_gemm_simt(const void* x, const void* w, void* y, const MatmulArgs& a, cudaStream_t st);

// tcgen05 GEMM: y[m, n] = (sum over terms of X_t[m, :] . W[n, :]) * row_scale[m] * (chan_scale[n] | scale)
// (+ bias[n]) (+ y if accumulate). kind_f16: X and W bf16 (one term); else X terms and W e4m3.
struct TcGemmArgs {
  const void* w;            // [n, k] (fp8 bytes or bf16), rows w_stride_bytes apart
  int64_t w_stride_bytes;
  const void* x[2];         // terms, [m, k], rows x_stride_bytes apart
  int64_t x_stride_bytes;
  int terms;                // 1 or 2 (fp8 only)
  int kind_f16;             // 1: bf16 x bf16 (kind::f16); 0: e4m3 x e4m3 (kind::f8f6f4)
  int64_t m, n, k;          // k in elements
  const float* row_scale;   // [m] or null
  const float* chan_scale;  // [n] or null
  float scale;
  const float* bias;        // [n] or null
  void* y;
  int64_t y_stride;         // values
  int y_dtype;
  int accumulate;
  EpiOps epi;
  uint32_t* dev_err;        // device error word
  void* ys[3];              // split output (ys[0] set): channels [seg_end[i-1], seg_end[i]) to ys[i], rows as
  int64_t seg_end[3];       // wide as the part apart; inner ends multiples of 256 (no tile straddles two parts)
  // second weight set (nseg > 0): token rows [row_end[i-1], row_end[i]) use set row_set[i]; set 1 takes w2 (same
  // shape and stride as w), chan_scale2 / scale2, bias2 and gate2 (gate2 present iff epi.gate is)
  const void* w2;
  const float* chan_scale2;
  float scale2;
  const float* bias2;
  const float* gate2;
  int nseg;
  int64_t row_end[WE_GEMM_MAX_SEGMENTS];
  int row_set[WE_GEMM_MAX_SEGMENTS];
  // int4 group-64 weights unpacked inside the GEMM (kind_f16 = 1): w is packed [n, k / 2] (low nibble = even k),
  // group_scale f16 [n, k / 64]; k % 64 == 0, one weight set
  int int4;
  const uint16_t* group_scale;
  // peer output (peer = 1): split-output part peer_part (the whole output without a split) is stored into other
  // GPUs' memory, head by head (128 channels): head h of the part goes to rank o = h / hl, hl = part width /
  // (128 peer_world), at peer_dst[o] + ((peer_row0 + row) hl + h - o hl) 128 values (bf16 y only, no aux, no
  // accumulate); the kernel fences its stores at system scope before it ends
  int peer;
  int peer_part;
  int peer_world;
  int64_t peer_row0;
  void* peer_dst[WE_PEER_MAX];
};
// Returns cudaErrorNotSupported when the layout cannot go through TMA (alignment) so the caller can
// use the CUDA-core kernel instead.
cudaError_t launch_gemm_tc(const TcGemmArgs& a, int sms, cudaStream_t st);
bool gemm_tc_supported(const TcGemmArgs& a);

cudaError_t launch_unpack_fp8_f32(const uint8_t* in, int64_t n, float scale, float* out, int sms, cudaStream_t st);
cudaError_t launch_unpack_fp8_bf16(const uint8_t* in, int64_t n, uint16_t* out, int sms, cudaStream_t st);
cudaError_t launch_unpack_int4(const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k, uint16_t* out,
                               int sms, cudaStream_t st);
cudaError_t launch_quant_fp8(const void* w, int dt, int64_t n, int64_t k, bool per_channel, uint8_t* q, float* scales,
                             unsigned int* amax_scratch, int sms, cudaStream_t st);
cudaError_t launch_quant_int4(const void* w, int dt, int64_t n, int64_t k, uint8_t* packed, uint16_t* scales, int sms,
                              cudaStream_t st);
cudaError_t launch_quant_act(const void* x, int dt, int64_t m, int64_t k, int64_t stride, int terms, uint8_t* hi,
                             uint8_t* lo, float* row_scale, int sms, cudaStream_t st);

cudaError_t launch_rmsnorm(const void* x, int xdt, const float* w, const float* sc, const float* sh, int64_t rows,
                           int64_t d, float eps, float offset, void* out, int odt, int sms, cudaStream_t st);
cudaError_t launch_rope(const void* x, int xdt, const float* cs, const float* sn, int64_t tokens, int64_t heads,
                        int64_t pairs, int pairing, void* out, int odt, int sms, cudaStream_t st);
// bf16 rows of 128-wide heads, norm + RoPE, each row stored into the exchange region of the rank that attends its
// head (dst[rank], [world x tokens, heads / world, 128], this rank's tokens from row0)
cudaError_t launch_qknorm_rope_peers(const void* x, const float* w, float eps, float offset, const float* cs,
                                     const float* sn, int64_t tokens, int64_t heads, int pairing, void* const* dst,
                                     int world, int64_t row0, int sms, cudaStream_t st);
cudaError_t launch_qknorm_rope(const void* x, int xdt, const float* w, float eps, float offset, const float* cs,
                               const float* sn, int64_t tokens, int64_t heads, int64_t pairs, int pairing, void* out,
                               int odt, int sms, cudaStream_t st);

cudaError_t launch_elementwise(int op, const void* a, const void* b, const float* g, int64_t n, int64_t d, int dt,
                               void* out, int ot, int sms, cudaStream_t st);
cudaError_t launch_norm_split(const void* x, int xdt, const float* w, const float* sc, const float* sh, int64_t rows,
                              int64_t d, float eps, float offset, int terms, uint8_t* hi, uint8_t* lo, float* rs,
                              int sms, cudaStream_t st);

cudaError_t launch_add_norm_split(const float* x, const float* r, float* xo, const float* w, const float* sc,
                                  const float* sh, int64_t rows, int64_t d, float eps, float offset, int terms,
                                  uint8_t* hi, uint8_t* lo, float* rs, int sms, cudaStream_t st);

// k_layout.cu: latent <-> tokens (2x2 patches, odd sizes wrap / crop)
cudaError_t launch_patchify(const void* latent, int ldt, int64_t C, int64_t H, int64_t W, void* tokens, int tdt,
                            int sms, cudaStream_t st);
cudaError_t launch_unpatchify(const void* tokens, int tdt, int64_t C, int64_t H, int64_t W, void* latent, int ldt,
                              int sms, cudaStream_t st);
cudaError_t launch_head_groups(const void* src, void* dst, int64_t tokens, int64_t groups, int64_t group_bytes,
                               int to_groups, int sms, cudaStream_t st);

// attention(q [T, H, D], k, v [T, Hkv, D]) -> out [T, H, D]
struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t tokens, heads, kv_heads, dim;
  int causal;
  int dtype, out_dtype;
};
bool flash_attention_supported(const AttnArgs& a);
// key splits for a grid that would not fill `sms` SMs (1 = none), the scratch they need, and the launch (the flash
// kernel, then the combine kernel when splits > 1)
int flash_attention_splits(const AttnArgs& a, int sms);
int64_t flash_attention_scratch_bytes(const AttnArgs& a, int splits);
cudaError_t launch_flash_attention(const AttnArgs& a, int splits, void* scratch, uint32_t* err, cudaStream_t st);
cudaError_t launch_attention_simt(const AttnArgs& a, int sms, cudaStream_t st);

}  // namespace we
