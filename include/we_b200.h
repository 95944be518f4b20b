/*
 * web-engine B200: the C ABI of the quantized-linear / RMSNorm / RoPE hot path.
 *
 * This is the drop-in boundary for the operator layer of dotstories/web-engine:
 * src/model/ops.ts (linear, norm, noMod, rotate) on top of src/gpu/graph.ts (Graph),
 * and the kernel-level entry points of src/kernels/{matmul,fp8,rmsnorm,rope}.ts.
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and returns an int
 * status (WE_OK or an error code); the message of the last error of a context is
 * we_last_error(ctx). The reference's synchronous `throw new Error(...)` cases map to
 * WE_EINVAL with the same message text.
 *
 * Memory: device buffers are plain device pointers. Buffers made by we_buffer() belong
 * to the context's pool (the Graph analog) and are freed by we_free / we_release /
 * we_destroy. Pointers from elsewhere (cudaMalloc, torch) may be passed to every op.
 *
 * Ordering: all work of a context runs in order on its stream (we_set_stream); the
 * calls are asynchronous except we_read and we_sync. A context is used by one host
 * thread at a time (the reference is single-threaded JS).
 */
#ifndef WE_B200_H
#define WE_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- status codes ---------------- */
enum {
  WE_OK = 0,
  WE_EINVAL = 1,      /* bad shape/format/layout: the reference's throw cases */
  WE_ENOMEM = 2,      /* device allocation failed */
  WE_ECUDA = 3,       /* a CUDA runtime/driver call failed */
  WE_ENCCL = 4,       /* a collective failed */
  WE_ETIMEOUT = 5,    /* a bounded device-side wait gave up (see we_device_error) */
  WE_EUNSUPPORTED = 6, /* valid request that this build does not implement */
  WE_EIO = 7           /* a file could not be opened, read or mapped */
};

/* ---------------- element types ---------------- */
enum {
  WE_F32 = 0,
  WE_BF16 = 1,
  WE_FP8 = 2,     /* float8_e4m3fn, 1 byte per value (src/kernels/fp8.ts: 4 per u32, little-endian) */
  WE_INT4G64 = 3, /* symmetric int4, 2 per byte (low nibble = even k), f16 scale per 64 values of K */
  WE_F16 = 4
};

typedef struct we_ctx we_ctx;

/* ---------------- context (src/gpu/compute.ts getDevice; src/gpu/graph.ts constructor) ---------------- */
/* Makes a context on CUDA device `device` with its own stream. flags: reserved, pass 0. */
int we_init(int device, uint32_t flags, we_ctx** out);
/* Frees every buffer of the context (Graph.destroy, src/gpu/graph.ts:148-154) and the context. */
int we_destroy(we_ctx* ctx);
const char* we_last_error(const we_ctx* ctx);
/* Runs later work on `stream` (a cudaStream_t; NULL = the context's own stream). Waits for the old one. */
int we_set_stream(we_ctx* ctx, void* stream);
void* we_get_stream(const we_ctx* ctx);
/* Waits for all queued work (device.queue.onSubmittedWorkDone). */
int we_sync(we_ctx* ctx);
/* Device-side error word of the context: 0, or the code a kernel's bounded wait recorded. Cleared on read. */
int we_device_error(we_ctx* ctx, uint32_t* code);
/* Number of streaming multiprocessors of the context's device. */
int we_num_sms(const we_ctx* ctx);

/* ---------------- memory: the Graph analog (src/gpu/graph.ts:26-155) ---------------- */
/* Graph.buffer(data | bytes) (graph.ts:38-54): a device buffer of `bytes` (rounded up to 4),
   filled with `host` when non-NULL, else zeroed. Reuses a pooled buffer of the same size. */
int we_buffer(we_ctx* ctx, size_t bytes, const void* host, void** out);
/* queue.writeBuffer: copy `bytes` from host to device (in order with the queued work). */
int we_write(we_ctx* ctx, void* dst, const void* host, size_t bytes);
/* Graph.read (graph.ts:109-119): runs everything queued, then copies `bytes` back. Synchronous. */
int we_read(we_ctx* ctx, const void* src, void* host, size_t bytes);
/* Graph.copy (graph.ts:93-98): device-to-device copy, in order with the queued work. */
int we_copy(we_ctx* ctx, const void* src, size_t src_offset, void* dst, size_t dst_offset, size_t bytes);
/* A strided device-to-device copy (no reference counterpart): `rows` rows of `width` bytes, src rows src_pitch bytes
   apart, dst rows dst_pitch apart, in order with the queued work. Cuts column slices out of row-major tensors (the
   K slice of a weight for tensor parallelism). */
int we_copy_2d(we_ctx* ctx, const void* src, size_t src_pitch, void* dst, size_t dst_pitch, size_t width, size_t rows);
/* Graph.mark (graph.ts:122): how many buffers the context owns now. */
size_t we_mark(we_ctx* ctx);
/* Graph.release (graph.ts:127-132): frees every buffer made since `mark`, except `keep`. */
int we_release(we_ctx* ctx, size_t mark, void* const* keep, size_t nkeep);
/* Graph.free (graph.ts:135-139): frees one buffer made by we_buffer. */
int we_free(we_ctx* ctx, void* buf);
/* the largest group of ranks that share memory (peer exchange, peer outputs) */
#define WE_PEER_MAX 8

/* Graph.stats (graph.ts:33): buffers created vs taken from the pool, bytes created; plus the number of
   kernels this context launched, and how many matmuls ran on the tcgen05 and CUDA-core kernels. */
typedef struct {
  uint64_t created, reused, created_bytes;
  uint64_t launches, tc_gemms, simt_gemms;
} we_stats;
int we_get_stats(const we_ctx* ctx, we_stats* out);

/* ---------------- matmul: matmulWgsl + matmulParams (src/kernels/matmul.ts:118-214) ---------------- */
enum {
  WE_MM_ACCUMULATE = 1u << 0, /* y += x . W^T * scale instead of y = (matmul.ts:145) */
  WE_MM_FP8_FAST = 1u << 1,   /* bf16 x with fp8 W: one e4m3 term per activation (fp8 tensor peak, ~3% rms
                                 per-element activation error) instead of the exact two-term split */
  WE_MM_FORCE_SIMT = 1u << 2  /* use the CUDA-core kernel even where the tensor-core kernel applies */
};
/* Epilogue operations fused into a matmul (the per-value steps of a block, src/kernels/elementwise.ts:38-84),
   applied to v = x . W^T * scale + bias in this order:
     act:    WE_ACT_GELU_TANH (geluTanh) | WE_ACT_SILU (silu) | WE_ACT_NONE
     aux_op: WE_AUX_SIGMOID_GATE  v = aux * sigmoid(v)  (sigmoidGate with this matmul as the gate)
             WE_AUX_SWIGLU        v = silu(aux) * v     (swiglu with this matmul as "up", aux = gate)
             aux: [m, n] in aux_dtype with y's row stride
     gate:   v = gate[col] * v                          (gatedAdd's g, with WE_MM_ACCUMULATE: y += g h)
   A zero-initialised we_epilogue does nothing. */
enum { WE_ACT_NONE = 0, WE_ACT_GELU_TANH = 1, WE_ACT_SILU = 2 };
enum { WE_AUX_NONE = 0, WE_AUX_SIGMOID_GATE = 1, WE_AUX_SWIGLU = 2 };
typedef struct {
  int32_t act;
  int32_t aux_op;
  int32_t aux_dtype; /* WE_F32 | WE_BF16 */
  const void* aux;
  const float* gate;
} we_epilogue;
typedef struct {
  int64_t m, n, k;
  /* Row strides and offsets in values (matmul.ts:185-195). 0 stride = contiguous (k, k, n). */
  int64_t x_stride, w_stride, y_stride, x_offset, w_offset, y_offset;
  int64_t k_split;          /* > 1: K slices, partials [k_split, m, y_stride] (matmul.ts:155-159) */
  float scale;              /* per-tensor weight scale (the reference's scalar weight_scale) */
  const float* chan_scale;  /* optional device [n]: per-output-channel scale, replaces `scale` */
  const uint16_t* group_scale; /* WE_INT4G64: device f16 [n, k/64] */
  const float* bias;        /* optional device f32 [n], added after scaling (ops.ts:65) */
  int32_t x_dtype;          /* WE_F32 | WE_BF16 */
  int32_t w_dtype;          /* WE_F32 | WE_BF16 | WE_FP8 | WE_INT4G64 */
  int32_t y_dtype;          /* WE_F32 | WE_BF16 */
  uint32_t flags;           /* WE_MM_* */
  we_epilogue epi;          /* fused per-value steps (zero = none) */
} we_matmul_desc;
/* y[m, n] = x[m, k] . W^T * scale (+ bias) with W [n, k] like nn.Linear. Validation as matmulParams
   (matmul.ts:205-207): "K must be a multiple of 4, got 6" etc. Replaces matmulWgsl/matmulParams/
   matmulWorkgroups and the one-shots matmulFp8/matmulBf16/matmulF32 (matmul.ts:223-265). */
int we_matmul(we_ctx* ctx, const we_matmul_desc* desc, const void* x, const void* w, void* y);
/* The matmulParams validation alone (throws in the reference): WE_OK or WE_EINVAL with the message. */
int we_matmul_check(we_ctx* ctx, const we_matmul_desc* desc);
/* The tcgen05 GEMM on activations already split into e4m3 terms (we_quantize_act, or a producer that
   writes the split directly): y = (x_hi + x_lo) . W^T * row_scale[m] * (chan_scale[n] | scale) (+ bias)
   (+ y with WE_MM_ACCUMULATE). x_lo NULL = one term. K % 16 == 0, rows 16-byte aligned. The matmul
   of matmulWgsl (src/kernels/matmul.ts:118-178) with its activation quantisation hoisted out. */
#define WE_GEMM_MAX_SEGMENTS 32
typedef struct {
  int64_t m, n, k;
  const uint8_t* x_hi;
  const uint8_t* x_lo;
  const float* row_scale;
  const uint8_t* w;
  float scale;
  const float* chan_scale;
  const float* bias;
  void* y;
  int64_t y_stride; /* values; 0 = n */
  int32_t y_dtype;  /* WE_F32 | WE_BF16 */
  uint32_t flags;   /* WE_MM_ACCUMULATE */
  we_epilogue epi;  /* fused per-value steps (zero = none) */
  /* Split output (part_n[0] > 0; y and y_stride unused): the first part_n[0] channels go to y_parts[0], the next
     part_n[1] to y_parts[1], the rest (part_n[2]) to y_parts[2], each with rows part_n[i] values apart, so one
     GEMM over concatenated weights (the q, k and v projections) fills separate buffers. The parts' widths sum
     to n; the boundaries between parts are multiples of 32 (an epilogue warp's channels); no aux operand. */
  void* y_parts[3];
  int64_t part_n[3];
  /* Two weight sets (nseg > 0): token rows [row_end[i - 1], row_end[i]) use set row_set[i] (row_end increasing, the
     last one m, at most WE_GEMM_MAX_SEGMENTS segments). Set 0 is w, scale / chan_scale, bias and epi.gate above;
     set 1 is w2 (same [n, k] layout), scale2 / chan_scale2, bias2 and gate2 (given iff epi.gate is). One GEMM
     then runs a double block's text and image rows, or every image of a batch, each with its own weights. Inner
     boundaries must be multiples of 64 rows (of 256 for the 2-SM kernel to be used). */
  const uint8_t* w2;
  float scale2;
  const float* chan_scale2;
  const float* bias2;
  const float* gate2;
  int32_t nseg;
  int64_t row_end[WE_GEMM_MAX_SEGMENTS];
  int32_t row_set[WE_GEMM_MAX_SEGMENTS];
  /* Peer output (peer_world > 0; no counterpart in the reference, which runs on one GPU): the channels of part
     peer_part (of the whole output without a split; that part's y_parts entry is then not used) are heads of 128,
     and head h goes straight into the memory of rank o = h / hl, hl = the part's width / (128 peer_world): row r
     of this GEMM to peer_dst[o] + ((peer_row0 + r) hl + h % hl) 128 values, i.e. rank o's [every rank's tokens,
     hl heads, 128] block (sequence parallelism: the GEMM's epilogue does the head scatter over NVLink, tile by
     tile, while the other tiles are computed). bf16 y, no aux operand, no WE_MM_ACCUMULATE, the part's width a
     multiple of 128 peer_world and its first channel of 128, peer_dst[0 .. peer_world) 16-byte aligned (from
     we_peer_remote). The stores are fenced at system scope; a flag barrier after the kernel (we_peer_exchange with
     no copies) makes them visible to the other ranks. */
  void* peer_dst[WE_PEER_MAX];
  int32_t peer_world;
  int32_t peer_part;
  int64_t peer_row0;
} we_gemm_fp8_desc;
int we_gemm_fp8(we_ctx* ctx, const we_gemm_fp8_desc* desc);
/* kSplitFor (src/model/ops.ts:42-45). */
int64_t we_ksplit_for(int64_t m, int64_t n, int64_t k);

/* ---------------- the operator API: src/model/ops.ts ---------------- */
/* Linear (ops.ts:24-32): W [n, k] as stored, scalar or per-channel scale, optional bias and LoRA. */
typedef struct we_linear {
  const void* weight;
  int32_t dtype;               /* WE_FP8 | WE_BF16 | WE_F32 | WE_INT4G64 */
  float scale;
  const float* chan_scale;     /* optional [n] */
  const uint16_t* group_scale; /* WE_INT4G64 */
  int64_t n, k;
  const float* bias;           /* optional [n] */
  const struct we_linear* lora_down; /* optional [rank, k] */
  const struct we_linear* lora_up;   /* optional [n, rank], scale = strength * alpha / rank */
} we_linear;
/* linear (ops.ts:61-73): y = x . W^T (+ bias) (+ up.scale (x . down^T) . up^T), a new pooled buffer
   [m, n] of y_dtype. LoRA shape errors: "LoRA shapes do not fit the linear layer". */
int we_linear_forward(we_ctx* ctx, const void* x, int32_t x_dtype, const we_linear* w, int64_t m,
                      int32_t y_dtype, uint32_t flags, void** y);
/* linear from host memory to host memory: y_host [m, n] = linear(x_host [m, k]). One call does the upload of x,
   the linear and the read-back of y. A caller of ops.ts:61-73 does the same with queue.writeBuffer before the
   dispatch and a mapped read after it (graph.ts:37-47, graph.ts:108-119). Rows go in chunks of chunk_rows
   (0: about m / 12, a multiple of 128) through three streams, so the host -> device copy of chunk c + 1, the GEMM
   of chunk c and the device -> host copy of chunk c - 1 overlap. Returns when y_host holds the result. Copies
   overlap only when both host buffers are page-locked (cudaHostAlloc / cudaHostRegister); pageable buffers give
   the same result. Each chunk is the linear of its rows, as we_linear_forward computes it for that many rows.
   Refused while capturing. */
int we_linear_host(we_ctx* ctx, const void* x_host, int32_t x_dtype, const we_linear* w, int64_t m,
                   int32_t y_dtype, uint32_t flags, void* y_host, int64_t chunk_rows);
/* Mod (ops.ts:75): scale/shift device vectors of length d (NULL = zeros). */
typedef struct {
  const float* scale;
  const float* shift;
} we_mod;
/* noMod (ops.ts:85): two zeroed pooled buffers of d floats. */
int we_no_mod(we_ctx* ctx, int64_t d, we_mod* out);
/* norm (ops.ts:78-82): RMSNorm rows of length d with modulation, a new pooled buffer. */
int we_norm(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, int64_t rows, int64_t d,
            const we_mod* mod, float eps, float offset, int32_t out_dtype, void** out);
/* Rope (ops.ts:87): tables [tokens, pairs]. */
typedef struct {
  const float* cos;
  const float* sin;
  int64_t pairs, tokens;
} we_rope;
enum { WE_ROPE_INTERLEAVED = 0, WE_ROPE_HALF = 1 };
/* rotate (ops.ts:89-93): x [tokens, heads, 2 pairs] -> a new pooled buffer. */
int we_rotate(we_ctx* ctx, const void* x, int32_t x_dtype, int64_t heads, const we_rope* rope, int32_t pairing,
              int32_t out_dtype, void** out);

/* ---------------- kernel-level entry points ---------------- */
/* rmsnormWgsl (src/kernels/rmsnorm.ts:13-48):
   out = x / sqrt(mean(x^2) + eps) * (offset + weight) * (1 + scale) + shift, per row of d. */
int we_rmsnorm(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, const float* scale,
               const float* shift, int64_t rows, int64_t d, float eps, float offset, void* out, int32_t out_dtype);
/* ropeKernel (src/kernels/rope.ts:59-77), interleaved or half pairing. */
int we_rope_apply(we_ctx* ctx, const void* x, int32_t x_dtype, const float* cos, const float* sin, int64_t tokens,
                  int64_t heads, int64_t pairs, int32_t pairing, void* out, int32_t out_dtype);
/* The block's q/k path in one pass (src/model/block.ts:53-56, norm then rotate): per head row of
   2*pairs values, RMSNorm (offset, eps) with `weight` [2 pairs], then RoPE. */
int we_qknorm_rope(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, float eps, float offset,
                   const float* cos, const float* sin, int64_t tokens, int64_t heads, int64_t pairs,
                   int32_t pairing, void* out, int32_t out_dtype);
/* we_qknorm_rope for sequence parallelism, with the head scatter done by the kernel's own stores (no reference
   counterpart: the reference runs on one GPU). x: this rank's bf16 rows [tokens, heads, 128] (interleaved or half
   pairing); the normalised, rotated bf16 row of (token t, head h) is written straight into the memory of the rank
   that attends head h, o = h / (heads / world), at dst[o] + ((dst_row0 + t) (heads / world) + h % (heads / world))
   128 values: dst[r] is rank r's q (or k) block in its exchange region (we_peer_remote + offset), laid out
   [world x tokens, heads / world, 128]. The stores are fenced at system scope; a flag barrier after the kernel
   (we_peer_exchange with no copies) makes them visible to the other ranks. */
int we_qknorm_rope_peers(we_ctx* ctx, const void* x, const float* weight, float eps, float offset, const float* cos,
                         const float* sin, int64_t tokens, int64_t heads, int32_t pairing, void* const* dst,
                         int32_t world, int64_t dst_row0);
/* ropeTables (src/kernels/rope.ts:20-36) on the host in float64: pos [tokens, naxes], axes (even),
   cos/sin [tokens, pairs] f32. Returns pairs, or -1 ("Every RoPE axis needs an even number of dims"). */
int64_t we_rope_tables(const int64_t* pos, int64_t tokens, int32_t naxes, const int64_t* axes, double theta,
                       float* cos, float* sin);
/* positions (src/kernels/rope.ts:14-18): text tokens at (0,0,0), then image tokens (0, row, col). */
int we_positions(int64_t text, int64_t rows, int64_t cols, int64_t* pos);

/* unpackFp8 (src/kernels/fp8.ts:24-36): out[i] = e4m3(bytes[i]) * scale, f32. */
int we_unpack_fp8(we_ctx* ctx, const uint8_t* bytes, int64_t n, float scale, float* out);
/* The same decode to bf16 (exact: every e4m3 value is a bf16 value), scale 1. */
int we_unpack_fp8_bf16(we_ctx* ctx, const uint8_t* bytes, int64_t n, uint16_t* out);
/* int4 group-64 operand decode: out[n, k] = bf16_rne(q * f16 scale). */
int we_unpack_int4(we_ctx* ctx, const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k,
                   uint16_t* out);

/* Weight quantisers (load-time helpers; no reference counterpart beyond the per-tensor fp8 format):
   fp8 per output channel (per_channel = 1: s_n = max|W[n,:]| / 448) or per tensor (s = max|W| / 448),
   q = e4m3 round-to-nearest-even, saturating. scales: [n] (or [1]) f32. */
int we_quantize_fp8(we_ctx* ctx, const void* w, int32_t w_dtype, int64_t n, int64_t k, int32_t per_channel,
                    uint8_t* q, float* scales);
/* int4 group 64: s = f16_rne(max|W_group| / 7), q = clamp(rint(W / s), -8, 7). */
int we_quantize_int4(we_ctx* ctx, const void* w, int32_t w_dtype, int64_t n, int64_t k, uint8_t* packed,
                     uint16_t* scales);
/* Activation split for the fp8 tensor-core path: per row a power-of-two scale 2^e (e smallest with
   max|x| 2^-e <= 448), hi = e4m3(x 2^-e), lo = e4m3(x 2^-e - hi) (terms = 2; exact for bf16 input),
   row_scale[m] = 2^e. lo may be NULL when terms = 1. */
int we_quantize_act(we_ctx* ctx, const void* x, int32_t x_dtype, int64_t m, int64_t k, int64_t x_stride,
                    int32_t terms, uint8_t* hi, uint8_t* lo, float* row_scale);

/* ---------------- elementwise (src/kernels/elementwise.ts:38-84, ops.ts:95-113) ----------------
   out[i] = swiglu: silu(a) b | sigmoidGate: a sigmoid(b) | gatedAdd: a + g[i % d] b | addBias: a + g[i % d]
          | geluTanh: GELU(a), tanh form | add: a + b | silu: a sigmoid(a), over n values (b, g unused where
   the formula has none). */
enum {
  WE_EW_SWIGLU = 0,
  WE_EW_SIGMOID_GATE = 1,
  WE_EW_GATED_ADD = 2,
  WE_EW_ADD_BIAS = 3,
  WE_EW_GELU_TANH = 4,
  WE_EW_ADD = 5,
  WE_EW_SILU = 6
};
int we_elementwise(we_ctx* ctx, int32_t op, const void* a, const void* b, const float* g, int64_t n, int64_t d,
                   int32_t dtype, void* out, int32_t out_dtype);
/* The op form (ops.ts elementwise()): out is a new pooled buffer of n values. */
int we_ew(we_ctx* ctx, int32_t op, const void* a, const void* b, const float* g, int64_t n, int64_t d, int32_t dtype,
          int32_t out_dtype, void** out);
/* norm() followed by the e4m3 activation split of its bf16-rounded output, in one pass: the planes and row
   scales equal we_rmsnorm(out_dtype = bf16) then we_quantize_act up to the summation order of the row's sum of
   squares and the modulation's rounding (y = fma(x inv, (offset + w)(1 + scale), shift), the product of the two
   factors rounded once): a 1-ulp bf16 difference in rare values. d % 8 == 0, d <= 8192, 16-byte aligned. */
int we_norm_split(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, const float* scale,
                  const float* shift, int64_t rows, int64_t d, float eps, float offset, int32_t terms, uint8_t* hi,
                  uint8_t* lo, float* row_scale);

/* ---------------- CUDA graphs (no reference counterpart: WebGPU records its command buffers each time) ----------------
   we_capture_begin starts capturing the context's stream (a stream set with we_set_stream, not the legacy default
   stream); every op of this library issued until we_capture_end is recorded, not run. Buffers the ops take while
   capturing come from a pool of the capture's own and belong to the graph afterwards (a replay writes them; they
   stay valid, with their addresses, until we_graph_destroy); host data uploaded while capturing is copied into
   pinned memory the graph owns. Buffers made before the capture and used by it must outlive the graph.
   we_read and we_sync refuse while capturing. we_graph_launch replays on the context's stream. */
typedef struct we_graph we_graph;
int we_capture_begin(we_ctx* ctx);
int we_capture_end(we_ctx* ctx, we_graph** out);
int we_graph_launch(we_ctx* ctx, we_graph* graph);
int we_graph_destroy(we_ctx* ctx, we_graph* graph);

/* The residual add of a block fused with the next norm + split: xo = x + r (f32 rows), then the planes and row
   scales of norm(xo) exactly as we_norm_split computes them from xo. f32 only; d <= 8192, d % 8 == 0,
   16-byte aligned rows. */
int we_add_norm_split(we_ctx* ctx, const float* x, const float* r, float* xo, const float* weight, const float* scale,
                      const float* shift, int64_t rows, int64_t d, float eps, float offset, int32_t terms, uint8_t* hi,
                      uint8_t* lo, float* row_scale);

/* ---------------- latent <-> tokens: patchify / unpatchify (src/model/transformer.ts:53-82) ----------------
   tokens [ceil(H/2) * ceil(W/2), 4 channels] <- latent [channels, H, W]: 2x2 patches, features in (channel, patch
   row, patch column) order; an odd H or W wraps to row / column 0 (patchify, transformer.ts:59-69). unpatchify is
   the inverse and crops the padding off (transformer.ts:72-82). f32 or bf16 on either side; bit-exact moves. */
int we_patchify(we_ctx* ctx, const void* latent, int32_t latent_dtype, int64_t channels, int64_t height, int64_t width,
                void* tokens, int32_t tokens_dtype);
int we_unpatchify(we_ctx* ctx, const void* tokens, int32_t tokens_dtype, int64_t channels, int64_t height,
                  int64_t width, void* latent, int32_t latent_dtype);

/* Sequence-parallel exchange layout (no reference counterpart: the reference runs on one GPU). rows holds
   [tokens, groups, group_bytes] (a token shard with every head), groups holds [groups, tokens, group_bytes]
   (chunk g = the heads of rank g, what an all-to-all sends to rank g). to_groups = 1 moves rows -> groups, 0 the
   reverse. group_bytes must be a multiple of 16 and both buffers 16-byte aligned. */
int we_head_groups(we_ctx* ctx, const void* rows, void* groups, int64_t tokens, int64_t n_groups, int64_t group_bytes,
                   int32_t to_groups);

/* ---------------- attention: attention() (src/kernels/attention.ts:20-51) ----------------
   softmax(q k^T / sqrt(dim)) v per head with grouped-query heads (query head h uses kv head
   h / (heads / kv_heads)); q [tokens, heads, dim], k, v [tokens, kv_heads, dim] -> out [tokens, heads, dim].
   causal = 1: query i sees keys 0..i (the text encoder). "heads must be a multiple of kvHeads" otherwise.
   bf16 with dim 128 and no mask runs the tcgen05 flash-attention kernel; the rest runs on CUDA cores in
   fp32 (the reference's exact semantics for f32 buffers). */
int we_attention(we_ctx* ctx, const void* q, const void* k, const void* v, int32_t dtype, int64_t tokens,
                 int64_t heads, int64_t kv_heads, int64_t dim, int32_t causal, void* out, int32_t out_dtype);
/* The same as an op: out is a new pooled buffer [tokens, heads, dim] of out_dtype. */
int we_attend(we_ctx* ctx, const void* q, const void* k, const void* v, int32_t dtype, int64_t tokens, int64_t heads,
              int64_t kv_heads, int64_t dim, int32_t causal, int32_t out_dtype, void** out);

/* ---------------- layer streaming: src/model/weights.ts:94-131 (loadTransformer) ----------------
   The reference uploads every block once and keeps it resident. A streamer instead keeps `slots` device
   buffers and copies layer l (host[l], bytes[l]) into slot l % slots with cudaMemcpyAsync on its own copy
   stream, overlapped with compute on the context stream. The host ranges are page-locked by the streamer
   (cudaHostRegister) unless WE_STREAM_HOST_PINNED says they already are. */
typedef struct we_streamer we_streamer;
enum { WE_STREAM_HOST_PINNED = 1u };
int we_streamer_create(we_ctx* ctx, const void* const* host, const size_t* bytes, int32_t layers, int32_t slots,
                       uint32_t flags, we_streamer** out);
/* Layer `layer`'s device copy: work queued on the context stream after this call sees its bytes. Also starts
   copying the following layers (wrapping to layer 0) into slots that no acquired layer holds. A layer whose
   slot is still held by another acquired layer is refused ("release it first"). */
int we_streamer_acquire(we_streamer* s, int32_t layer, void** dev);
/* The work using `layer` is queued: its slot may be refilled once that work has run. */
int we_streamer_release(we_streamer* s, int32_t layer);
int we_streamer_stats(const we_streamer* s, uint64_t* copies, uint64_t* bytes_copied);
int we_streamer_destroy(we_streamer* s);

/* ---------------- peer memory for sequence parallelism (no counterpart in the reference) ----------------
   The reference runs on one GPU. With one image's rows split over the GPUs of a node, its attention needs an
   all-to-all of q, k, v and o per block. Each rank creates an exchange region of `bytes` in its own HBM
   (we_peer_create), exports it (we_peer_export: an opaque blob of WE_PEER_HANDLE_BYTES), gathers every rank's
   blob by any host channel, and opens them (we_peer_open, blobs in rank order; a blob equal to this rank's own
   export maps to its own memory). we_peer_exchange then runs ONE kernel on the context's stream: for each copy,
   peer p and row i it copies chunk_bytes from
       src + p * src_peer_stride + i * src_row_stride                      (this rank's memory)
   to  region_p + dst_offset + rank * dst_rank_stride + i * dst_row_stride  (rank p's region, over NVLink),
   and then meets every rank at a flag barrier in the same memory, so kernels after it on the stream see every
   rank's chunks. Every rank must issue the same exchanges in the same order. The barrier's wait is bounded by
   timeout_ns (0: 2 s); on timeout the kernel sets the context's device error word (we_device_error) and returns.
   Sources, chunks and strides must be multiples of 16 bytes; a copy may not run past the region. The kernel
   can be captured in a CUDA graph (its epoch lives on the device). */
#define WE_PEER_HANDLE_BYTES 128
typedef struct we_peer we_peer;
typedef struct {
  const void* src;
  int64_t rows;             /* rows per peer */
  int64_t chunk_bytes;      /* bytes per (peer, row) */
  int64_t src_row_stride, src_peer_stride;
  int64_t dst_offset, dst_row_stride, dst_rank_stride;
} we_peer_copy;
int we_peer_create(we_ctx* ctx, int32_t rank, int32_t world, size_t bytes, we_peer** out);
int we_peer_export(const we_peer* peer, void* handle);
int we_peer_open(we_peer* peer, const void* handles);
void* we_peer_region(const we_peer* peer);
/* Rank `rank`'s exchange region as this process maps it (its own region for rank == this rank; NULL before
   we_peer_open or for a rank outside the group): the destination of kernels that store straight into a peer's
   region (we_qknorm_rope_peers, the peer output of we_gemm_fp8). */
void* we_peer_remote(const we_peer* peer, int32_t rank);
int we_peer_exchange(we_ctx* ctx, we_peer* peer, const we_peer_copy* copies, int32_t ncopies, uint64_t timeout_ns);
int we_peer_destroy(we_peer* peer);

/* ---------------- collectives (no counterpart in the reference: it runs on one GPU) ----------------
   NCCL communicators over NVLink / NVSwitch, one per context (one process per GPU), for the multi-GPU paths: the
   tensor-parallel linears (all-gather of token shards, reduce-scatter of partial sums), the sequence-parallel
   attention exchange (all-to-all) and timing reductions. NCCL is loaded when first needed (dlopen libnccl.so.2);
   without it these calls return WE_EUNSUPPORTED. Rank 0 makes the unique id (we_comm_unique_id, WE_COMM_ID_BYTES)
   and any host channel carries it to the other ranks, which all call we_comm_init with it. The communicator is
   non-blocking: each collective returns once queued on the context's stream (device buffers, stream order). A host
   deadline (timeout_ms, 0 = 60 s) bounds init and every call: a rank that never joins, or an NCCL error, aborts the
   communicator and returns WE_ETIMEOUT / WE_ENCCL, with the message in we_comm_last_error; an aborted communicator
   refuses further calls. Every rank must issue the same collectives in the same order. */
#define WE_COMM_ID_BYTES 128
typedef struct we_comm we_comm;
enum { WE_REDUCE_SUM = 0, WE_REDUCE_MAX = 1 };
int we_comm_unique_id(void* id);
int we_comm_init(we_ctx* ctx, int32_t nranks, int32_t rank, const void* id, uint64_t timeout_ms, we_comm** out);
int we_comm_destroy(we_comm* comm);
int we_comm_abort(we_comm* comm);
int we_comm_rank(const we_comm* comm, int32_t* rank, int32_t* nranks);
const char* we_comm_last_error(const we_comm* comm);
/* y [nranks * bytes] = every rank's x [bytes], in rank order */
int we_all_gather(we_comm* comm, const void* x, void* y, size_t bytes);
/* y [count] = this rank's count values of the element-wise sum over ranks of x [nranks * count] (f32 | bf16 | f16) */
int we_reduce_scatter(we_comm* comm, const void* x, void* y, size_t count, int32_t dtype);
/* y [count] = the element-wise sum or max over ranks of x [count] (f32 | bf16 | f16); x == y allowed */
int we_all_reduce(we_comm* comm, const void* x, void* y, size_t count, int32_t dtype, int32_t op);
/* y [nranks * bytes_per_rank]: chunk p of y is chunk rank of rank p's x (an all-to-all of equal chunks) */
int we_all_to_all(we_comm* comm, const void* x, void* y, size_t bytes_per_rank);
/* every rank reaches this point: an all-reduce of one word, then a bounded wait for the context's stream */
int we_comm_barrier(we_comm* comm);
/* waits for the context's stream, bounded by the timeout, watching for asynchronous NCCL errors */
int we_comm_wait(we_comm* comm);

/* ---------------- allocation-free linear (no counterpart in the reference) ----------------
   For callers that cannot allocate device memory: a serving loop whose memory budget is fixed when it
   starts, or a host runtime (a plugin handed only streams and pointers) whose allocator owns all of it.
   y = x . W^T * scale (+ bias) for bf16 x [m, k] (row stride x_stride values: 0 = k, else >= k) and e4m3
   W [n, k] with f32 scale or per-channel chan_scale [n], into y [m, n] (row stride y_stride: 0 = n, else
   >= n): the same activation split and tcgen05 GEMM as we_matmul, but with no context and no allocation.
   The split lives in one static device array of WE_NOALLOC_SCRATCH_BYTES that every GPU loading this
   library holds until the process exits; calls needing more (2 m k + 4 m bytes, m k + 4 m with
   WE_MM_FP8_FAST) return WE_EINVAL, and so do layouts the tensor-core GEMM cannot take (K % 16 != 0, w
   not 16-byte aligned), with a message. All calls on a device share that array, so calls that overlap on
   the GPU (other streams, other threads) race: serialise them. The first call in each CUDA context (per
   device; again after cudaDeviceReset, or in a context the host made itself) looks up the array's device
   address with that device current; make that first call before any stream capture. `stream` is a
   cudaStream_t of the current context. flags: WE_MM_FP8_FAST, WE_MM_ACCUMULATE, WE_NOALLOC_SYNC (wait for
   the stream, read the GEMM's error word on it, and return WE_ETIMEOUT if a bounded wait gave up). Without
   WE_NOALLOC_SYNC the call returns once the work is queued and a bounded-wait timeout goes unreported (the
   next call clears the word). errbuf (may be NULL) receives a message on failure. */
#define WE_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
enum { WE_NOALLOC_SYNC = 1u << 3 };
int we_matmul_fp8_noalloc(void* stream, const void* x, int64_t m, int64_t k, int64_t x_stride, const uint8_t* w,
                          int64_t n, float scale, const float* chan_scale, const float* bias, void* y,
                          int64_t y_stride, int32_t y_dtype, uint32_t flags, char* errbuf, size_t errlen);

/* ---------------- weights: .safetensors files (src/weights/safetensors.ts:1-70) ----------------
   The file is untrusted: we_st_open checks every offset and size before use, with the reference's checks and
   messages (readHeader, safetensors.ts:27-64): "File is too small to be a .safetensors file", "Bad header size: N"
   (over 100 MB or past the end), "Header is not valid JSON", "Header is not an object", "<name>: unknown dtype D",
   "<name>: bad shape", "<name>: bad data_offsets", "<name>: has N bytes, its shape needs M bytes", "<name>: data
   goes past the end of the file", "<a> and <b> overlap". Those return WE_EINVAL, OS failures WE_EIO, with the
   message in err. The data region is mapped read-only; nothing is read until a tensor is asked for. */
typedef struct we_st we_st;
typedef struct {
  const char* name;  /* owned by the we_st */
  const char* dtype; /* "F32", "BF16", "F16", "F8_E4M3", "F8_E5M2", "I64", ... "BOOL" */
  int32_t ndim;
  int64_t shape[8]; /* the first min(ndim, 8) dimensions */
  int64_t offset;   /* absolute byte offset of the data in the file */
  int64_t size;     /* bytes */
} we_st_tensor;

int we_st_open(const char* path, we_st** out, char* err, size_t err_len);
int64_t we_st_count(const we_st* st);
/* the i-th tensor in header order */
int we_st_tensor_at(const we_st* st, int64_t i, we_st_tensor* out);
/* WE_EINVAL when the file has no tensor of that name */
int we_st_find(const we_st* st, const char* name, we_st_tensor* out);
int64_t we_st_metadata_count(const we_st* st);
int we_st_metadata_at(const we_st* st, int64_t i, const char** key, const char** value);
/* readTensor (safetensors.ts:67-70): the first min(limit, size) bytes of a tensor (limit < 0: all) into host memory */
int we_st_read(const we_st* st, const char* name, void* dst, int64_t limit);
/* The tensor's bytes into device memory on the context's stream: the mapped file is copied through two pinned
   32 MB staging chunks, each chunk's DMA overlapping the host copy of the next. The loader's device upload of a
   linear layer (loadLinear's graph.buffer, src/model/weights.ts:26-50). */
int we_st_upload(we_ctx* ctx, we_st* st, const char* name, void* device_dst);
void we_st_close(we_st* st);

#ifdef __cplusplus
}
#endif
#endif
