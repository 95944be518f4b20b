// The C ABI of the web-engine B200 hot path (include/we_b200.h): context, the Graph-style buffer
// pool, argument validation with the reference's error messages, and dispatch to the kernels.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <cstring>
#include <deque>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.h"

struct we_ctx {
  int device = 0;
  int sms = 148;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  std::string err;
  // Graph analog (src/gpu/graph.ts:26-155): buffers in creation order, a free pool keyed by size
  std::vector<void*> owned;
  std::unordered_map<size_t, std::vector<void*>> pool;
  std::unordered_map<void*, size_t> sizes;  // every buffer this context allocated
  we_stats stats{0, 0, 0, 0, 0, 0};
  uint32_t* dev_err = nullptr;  // device error word written by bounded waits
  unsigned int* amax_word = nullptr;
  // Pinned staging ring for host -> device uploads. Like WebGPU's queue.writeBuffer, an upload copies the
  // caller's data before returning and the DMA then runs in stream order: a copy straight from pageable
  // memory would first wait for the whole stream, and the GPU would idle while the host catches up.
  struct Staged {
    size_t begin, end;
    cudaEvent_t done;
  };
  char* stage = nullptr;
  size_t stage_head = 0;
  std::deque<Staged> staged;
  std::vector<cudaEvent_t> spare_events;
  // Stream capture (we_capture_begin / we_capture_end). Buffers taken while capturing come from, and go back to,
  // a pool of the capture's own and belong to the graph afterwards: a replay writes them, so nothing else may
  // be handed them. Uploads made while capturing read from pinned copies the graph owns.
  bool capturing = false;
  std::unordered_map<size_t, std::vector<void*>> cap_pool;
  std::vector<void*> cap_bufs;
  std::vector<void*> cap_host;
  uint64_t cap_launches0 = 0;
  std::vector<we_graph*> graphs;  // live graphs, destroyed with the context
  // we_linear_host's copy engines: host -> device and device -> host streams beside the compute stream, and
  // the events that order one call's row chunks between the three (created on first use)
  cudaStream_t h2d = nullptr, d2h = nullptr;
  std::vector<cudaEvent_t> io_events;
};

struct we_graph {
  cudaGraphExec_t exec = nullptr;
  std::vector<void*> bufs;  // device buffers the graph reads and writes
  std::vector<void*> host;  // pinned sources of its uploads
  uint64_t launches = 0;    // kernels of this library in one replay
};

namespace {

int fail(we_ctx* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}
int cuda_fail(we_ctx* c, cudaError_t e, const char* what) {
  return fail(c, e == cudaErrorMemoryAllocation ? WE_ENOMEM : WE_ECUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}
#define CK(call, what)                      \
  do {                                      \
    cudaError_t e_ = (call);                \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
  } while (0)
// a kernel launch of this library: checked and counted in we_stats.launches
#define LK(call, what)        \
  do {                        \
    CK(call, what);           \
    ctx->stats.launches++;    \
  } while (0)

size_t round4(size_t b) { return std::max<size_t>(4, (b + 3) / 4 * 4); }

constexpr size_t kStageBytes = 16u << 20;  // uploads up to half of this go through the staging ring

// Host -> device copy of `bytes` at `host` into `dst`, in stream order, without waiting for the stream: small
// uploads are copied into the pinned ring first (waiting only for earlier copies still reading the region to
// be overwritten), large ones go straight from the caller's memory.
int upload(we_ctx* ctx, void* dst, const void* host, size_t bytes, const char* what) {
  if (bytes == 0) return WE_OK;
  if (ctx->capturing) {  // the graph replays the copy from a pinned copy of its own
    void* pin = nullptr;
    CK(cudaHostAlloc(&pin, bytes, cudaHostAllocDefault), "capture upload copy");
    ctx->cap_host.push_back(pin);
    std::memcpy(pin, host, bytes);
    CK(cudaMemcpyAsync(dst, pin, bytes, cudaMemcpyHostToDevice, ctx->stream), what);
    return WE_OK;
  }
  if (bytes > kStageBytes / 2) {
    CK(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, ctx->stream), what);
    return WE_OK;
  }
  if (!ctx->stage) CK(cudaHostAlloc(reinterpret_cast<void**>(&ctx->stage), kStageBytes, cudaHostAllocDefault),
                      "staging ring");
  const size_t len = (bytes + 255) & ~size_t(255);
  const size_t off = ctx->stage_head + len <= kStageBytes ? ctx->stage_head : 0;
  for (auto it = ctx->staged.begin(); it != ctx->staged.end();) {
    if (it->begin < off + len && off < it->end) {
      CK(cudaEventSynchronize(it->done), "staging wait");
      ctx->spare_events.push_back(it->done);
      it = ctx->staged.erase(it);
    } else {
      ++it;
    }
  }
  while (!ctx->staged.empty() && cudaEventQuery(ctx->staged.front().done) == cudaSuccess) {
    ctx->spare_events.push_back(ctx->staged.front().done);
    ctx->staged.pop_front();
  }
  std::memcpy(ctx->stage + off, host, bytes);
  CK(cudaMemcpyAsync(dst, ctx->stage + off, bytes, cudaMemcpyHostToDevice, ctx->stream), what);
  cudaEvent_t ev;
  if (ctx->spare_events.empty()) {
    CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "staging event");
  } else {
    ev = ctx->spare_events.back();
    ctx->spare_events.pop_back();
  }
  const cudaError_t e = cudaEventRecord(ev, ctx->stream);
  if (e != cudaSuccess) {
    ctx->spare_events.push_back(ev);
    return cuda_fail(ctx, e, "staging event");
  }
  ctx->staged.push_back({off, off + len, ev});
  ctx->stage_head = off + len;
  return WE_OK;
}

// Takes a pooled buffer of exactly `size` bytes or allocates one (graph.ts:41-45).
int pool_take(we_ctx* ctx, size_t size, void** out, bool* reused) {
  auto& pool = ctx->capturing ? ctx->cap_pool : ctx->pool;
  auto it = pool.find(size);
  if (it != pool.end() && !it->second.empty()) {
    *out = it->second.back();
    it->second.pop_back();
    *reused = true;
    return WE_OK;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, size);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(ctx, WE_ENOMEM, "cudaMalloc of " + std::to_string(size) + " bytes failed: " + cudaGetErrorString(e));
  }
  ctx->sizes[p] = size;
  if (ctx->capturing) ctx->cap_bufs.push_back(p);
  *out = p;
  *reused = false;
  return WE_OK;
}
void pool_put(we_ctx* ctx, void* p) {
  const bool mine = ctx->capturing && std::find(ctx->cap_bufs.begin(), ctx->cap_bufs.end(), p) != ctx->cap_bufs.end();
  (mine ? ctx->cap_pool : ctx->pool)[ctx->sizes[p]].push_back(p);
}

void graph_free(we_graph* g) {
  if (g->exec) cudaGraphExecDestroy(g->exec);
  for (void* b : g->bufs) cudaFree(b);
  for (void* h : g->host) cudaFreeHost(h);
  delete g;
}

// A temporary of the library (activation split, decoded int4 weights): from the pool, not owned by
// the caller, returned to the pool right after the work using it is queued (stream order keeps it safe).
struct Scratch {
  we_ctx* ctx;
  std::vector<void*> bufs;
  explicit Scratch(we_ctx* c) : ctx(c) {}
  int take(size_t bytes, void** out) {
    bool reused;
    size_t size = (bytes + 255) / 256 * 256;
    int rc = pool_take(ctx, size, out, &reused);
    if (rc == WE_OK) bufs.push_back(*out);
    return rc;
  }
  ~Scratch() {
    for (void* p : bufs) pool_put(ctx, p);
  }
};

// New output buffer of an op (ops.ts: graph.buffer(bytes)); contents are fully overwritten by the op.
int op_output(we_ctx* ctx, size_t bytes, void** out) {
  bool reused;
  size_t size = round4(bytes);
  int rc = pool_take(ctx, size, out, &reused);
  if (rc != WE_OK) return rc;
  if (reused) ctx->stats.reused++;
  else {
    ctx->stats.created++;
    ctx->stats.created_bytes += size;
  }
  ctx->owned.push_back(*out);
  return WE_OK;
}

size_t dsize(int dt) { return dt == WE_F32 ? 4 : (dt == WE_BF16 || dt == WE_F16) ? 2 : 1; }
bool act_dtype_ok(int dt) { return dt == WE_F32 || dt == WE_BF16; }

}  // namespace

// helpers shared with the other translation units of the library (we_stream.cu)
int we_ctx_fail(we_ctx* ctx, int code, const std::string& msg) { return fail(ctx, code, msg); }
cudaStream_t we_ctx_stream(we_ctx* ctx) { return ctx->stream; }
int we_ctx_device(we_ctx* ctx) { return ctx->device; }
uint32_t* we_ctx_dev_err(we_ctx* ctx) { return ctx->dev_err; }
void we_ctx_count_launch(we_ctx* ctx) { ctx->stats.launches++; }
bool we_ctx_capturing(const we_ctx* ctx) { return ctx->capturing; }

extern "C" {

// ---------------- context ----------------
int we_init(int device, uint32_t flags, we_ctx** out) {
  (void)flags;
  if (!out) return WE_EINVAL;
  *out = nullptr;
  we_ctx* ctx = new we_ctx();
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    delete ctx;
    return WE_ECUDA;
  }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (major != 10) {
    delete ctx;
    return WE_EUNSUPPORTED;  // sm_100a kernels only
  }
  ctx->sms = sms > 0 ? sms : 148;
  if (cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->dev_err, 16) != cudaSuccess || cudaMemset(ctx->dev_err, 0, 16) != cudaSuccess) {
    delete ctx;
    return WE_ECUDA;
  }
  ctx->amax_word = reinterpret_cast<unsigned int*>(ctx->dev_err + 2);
  ctx->stream = ctx->own;
  *out = ctx;
  return WE_OK;
}

int we_destroy(we_ctx* ctx) {
  if (!ctx) return WE_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (we_graph* g : ctx->graphs) graph_free(g);
  for (auto& st : ctx->staged) cudaEventDestroy(st.done);
  for (cudaEvent_t ev : ctx->spare_events) cudaEventDestroy(ev);
  if (ctx->stage) cudaFreeHost(ctx->stage);
  for (cudaEvent_t ev : ctx->io_events) cudaEventDestroy(ev);
  if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
  if (ctx->d2h) cudaStreamDestroy(ctx->d2h);
  for (auto& kv : ctx->sizes) cudaFree(kv.first);
  cudaFree(ctx->dev_err);
  cudaStreamDestroy(ctx->own);
  delete ctx;
  return WE_OK;
}

const char* we_last_error(const we_ctx* ctx) { return ctx ? ctx->err.c_str() : "no context"; }

int we_set_stream(we_ctx* ctx, void* stream) {
  if (!ctx) return WE_EINVAL;
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own;
  return WE_OK;
}
void* we_get_stream(const we_ctx* ctx) { return ctx ? ctx->stream : nullptr; }

int we_sync(we_ctx* ctx) {
  if (!ctx) return WE_EINVAL;
  if (ctx->capturing) return fail(ctx, WE_EINVAL, "cannot synchronize while capturing a graph");
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return WE_OK;
}

int we_device_error(we_ctx* ctx, uint32_t* code) {
  if (!ctx || !code) return WE_EINVAL;
  CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  CK(cudaMemcpy(code, ctx->dev_err, 4, cudaMemcpyDeviceToHost), "read device error word");
  CK(cudaMemset(ctx->dev_err, 0, 4), "clear device error word");
  return WE_OK;
}

int we_num_sms(const we_ctx* ctx) { return ctx ? ctx->sms : 0; }

// ---------------- memory (Graph) ----------------
int we_buffer(we_ctx* ctx, size_t bytes, const void* host, void** out) {
  if (!ctx || !out) return WE_EINVAL;
  int rc = op_output(ctx, bytes, out);
  if (rc != WE_OK) return rc;
  size_t size = ctx->sizes[*out];
  if (host) {
    rc = upload(ctx, *out, host, bytes, "upload");
    if (rc != WE_OK) return rc;
    if (size > bytes) CK(cudaMemsetAsync(static_cast<char*>(*out) + bytes, 0, size - bytes, ctx->stream), "pad");
  } else {
    CK(cudaMemsetAsync(*out, 0, size, ctx->stream), "zero buffer");
  }
  return WE_OK;
}

int we_write(we_ctx* ctx, void* dst, const void* host, size_t bytes) {
  if (!ctx) return WE_EINVAL;
  return upload(ctx, dst, host, bytes, "we_write");
}

int we_read(we_ctx* ctx, const void* src, void* host, size_t bytes) {
  if (!ctx) return WE_EINVAL;
  if (ctx->capturing) return fail(ctx, WE_EINVAL, "cannot read back while capturing a graph");
  CK(cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "we_read");
  CK(cudaStreamSynchronize(ctx->stream), "we_read sync");
  return WE_OK;
}

int we_copy(we_ctx* ctx, const void* src, size_t so, void* dst, size_t dof, size_t bytes) {
  if (!ctx) return WE_EINVAL;
  CK(cudaMemcpyAsync(static_cast<char*>(dst) + dof, static_cast<const char*>(src) + so, bytes,
                     cudaMemcpyDeviceToDevice, ctx->stream),
     "we_copy");
  return WE_OK;
}

int we_copy_2d(we_ctx* ctx, const void* src, size_t src_pitch, void* dst, size_t dst_pitch, size_t width,
               size_t rows) {
  if (!ctx) return WE_EINVAL;
  if (width > src_pitch || width > dst_pitch) return fail(ctx, WE_EINVAL, "we_copy_2d: a row is wider than its pitch");
  if (!width || !rows) return WE_OK;
  CK(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, rows, cudaMemcpyDeviceToDevice, ctx->stream),
     "we_copy_2d");
  return WE_OK;
}

size_t we_mark(we_ctx* ctx) { return ctx ? ctx->owned.size() : 0; }

int we_release(we_ctx* ctx, size_t mark, void* const* keep, size_t nkeep) {
  if (!ctx) return WE_EINVAL;
  if (mark > ctx->owned.size()) return fail(ctx, WE_EINVAL, "mark is beyond the buffers of this graph");
  std::vector<void*> later(ctx->owned.begin() + mark, ctx->owned.end());
  ctx->owned.resize(mark);
  for (void* b : later) {
    bool kept = false;
    for (size_t i = 0; i < nkeep; i++) kept |= keep[i] == b;
    if (kept) ctx->owned.push_back(b);
    else pool_put(ctx, b);
  }
  return WE_OK;
}

int we_free(we_ctx* ctx, void* buf) {
  if (!ctx) return WE_EINVAL;
  auto it = std::find(ctx->owned.begin(), ctx->owned.end(), buf);
  if (it == ctx->owned.end()) return fail(ctx, WE_EINVAL, "buffer is not owned by this graph");
  ctx->owned.erase(it);
  pool_put(ctx, buf);
  return WE_OK;
}

int we_get_stats(const we_ctx* ctx, we_stats* out) {
  if (!ctx || !out) return WE_EINVAL;
  *out = ctx->stats;
  return WE_OK;
}

// ---------------- matmul ----------------
int64_t we_ksplit_for(int64_t m, int64_t n, int64_t k) {
  const int64_t TILE = 128, BUSY = 256, MIN_SLICE = 256;
  int64_t tiles = ((m + TILE - 1) / TILE) * ((n + TILE - 1) / TILE);
  int64_t v = std::min((BUSY + tiles - 1) / tiles, k / MIN_SLICE);
  return std::max<int64_t>(1, v);
}

int we_matmul_check(we_ctx* ctx, const we_matmul_desc* d) {
  if (!d) return fail(ctx, WE_EINVAL, "no matmul description");
  const int64_t xs = d->x_stride ? d->x_stride : d->k, ws = d->w_stride ? d->w_stride : d->k;
  // matmulParams (src/kernels/matmul.ts:205-207)
  const std::pair<const char*, int64_t> four[] = {{"K", d->k}, {"xStride", xs}, {"wStride", ws},
                                                  {"xOffset", d->x_offset}, {"wOffset", d->w_offset}};
  for (auto& kv : four)
    if (kv.second % 4)
      return fail(ctx, WE_EINVAL, std::string(kv.first) + " must be a multiple of 4, got " + std::to_string(kv.second));
  if (d->m < 0 || d->n < 0 || d->k < 0) return fail(ctx, WE_EINVAL, "m, n and k must not be negative");
  if (!act_dtype_ok(d->x_dtype)) return fail(ctx, WE_EINVAL, "x must be f32 or bf16");
  if (!act_dtype_ok(d->y_dtype)) return fail(ctx, WE_EINVAL, "y must be f32 or bf16");
  if (d->w_dtype < WE_F32 || d->w_dtype > WE_INT4G64) return fail(ctx, WE_EINVAL, "unknown weight format");
  if (d->w_dtype == WE_INT4G64) {
    if (d->k % 64) return fail(ctx, WE_EINVAL, "K must be a multiple of 64 for int4 group-64 weights, got " + std::to_string(d->k));
    if (ws != d->k || d->w_offset) return fail(ctx, WE_EINVAL, "int4 group-64 weights must be contiguous [n, k]");
    if (!d->group_scale) return fail(ctx, WE_EINVAL, "int4 group-64 weights need group scales");
    if ((uintptr_t)d->group_scale & 1) return fail(ctx, WE_EINVAL, "int4 group scales must be 2-byte aligned f16");
  }
  if (d->k_split > 1 && d->bias) return fail(ctx, WE_EINVAL, "bias is not supported with kSplit");
  if (d->epi.act < WE_ACT_NONE || d->epi.act > WE_ACT_SILU) return fail(ctx, WE_EINVAL, "unknown activation");
  if (d->epi.aux_op < WE_AUX_NONE || d->epi.aux_op > WE_AUX_SWIGLU) return fail(ctx, WE_EINVAL, "unknown aux op");
  if (d->epi.aux_op && (!d->epi.aux || !act_dtype_ok(d->epi.aux_dtype)))
    return fail(ctx, WE_EINVAL, "the aux op needs an f32 or bf16 aux tensor");
  if (d->k_split > 1 && (d->epi.act || d->epi.aux_op || d->epi.gate))
    return fail(ctx, WE_EINVAL, "fused epilogue steps are not supported with kSplit");
  return WE_OK;
}

static int matmul_impl(we_ctx* ctx, const we_matmul_desc* d, const void* x, const void* w, void* y) {
  int rc = we_matmul_check(ctx, d);
  if (rc != WE_OK) return rc;
  if (d->m == 0 || d->n == 0) return WE_OK;
  we::MatmulArgs a;
  a.m = d->m;
  a.n = d->n;
  a.k = d->k;
  a.x_stride = d->x_stride ? d->x_stride : d->k;
  a.w_stride = d->w_stride ? d->w_stride : d->k;
  a.y_stride = d->y_stride ? d->y_stride : d->n;
  a.x_offset = d->x_offset;
  a.w_offset = d->w_offset;
  a.y_offset = d->y_offset;
  a.k_split = d->k_split > 1 ? d->k_split : 1;
  a.scale = d->scale;
  a.chan_scale = d->chan_scale;
  a.group_scale = d->group_scale;
  a.bias = d->bias;
  a.x_dtype = d->x_dtype;
  a.w_dtype = d->w_dtype;
  a.y_dtype = d->y_dtype;
  a.accumulate = (d->flags & WE_MM_ACCUMULATE) ? 1 : 0;
  a.epi.act = d->epi.act;
  a.epi.aux_op = d->epi.aux_op;
  a.epi.aux_dtype = d->epi.aux_dtype;
  a.epi.aux = d->epi.aux ? static_cast<const char*>(d->epi.aux) + a.y_offset * dsize(d->epi.aux_dtype) : nullptr;
  a.epi.gate = d->epi.gate;
  cudaStream_t st = ctx->stream;

  const bool tc_candidate = !(d->flags & WE_MM_FORCE_SIMT) && a.x_dtype == WE_BF16 && a.k_split == 1 && a.k > 0 &&
                            a.w_dtype != WE_F32;
  if (tc_candidate) {
    Scratch scratch(ctx);
    we::TcGemmArgs t{};
    t.m = a.m;
    t.n = a.n;
    t.k = a.k;
    t.scale = a.scale;
    t.chan_scale = a.chan_scale;
    t.bias = a.bias;
    t.y = static_cast<char*>(y) + a.y_offset * dsize(a.y_dtype);
    t.y_stride = a.y_stride;
    t.y_dtype = a.y_dtype;
    t.accumulate = a.accumulate;
    t.epi = a.epi;
    t.dev_err = ctx->dev_err;
    bool ready = false;
    if (a.w_dtype == WE_FP8) {
      t.kind_f16 = 0;
      t.terms = (d->flags & WE_MM_FP8_FAST) ? 1 : 2;
      t.w = static_cast<const uint8_t*>(w) + a.w_offset;
      t.w_stride_bytes = a.w_stride;
      t.x_stride_bytes = a.k;  // the split writes contiguous [m, k] rows (TMA needs k % 16 == 0)
      t.x[0] = t.x[1] = reinterpret_cast<void*>(256);  // layout probe before doing the split
      if (we::gemm_tc_supported(t)) {
        void *hi, *lo = nullptr, *rs;
        if ((rc = scratch.take((size_t)(a.m * a.k), &hi)) != WE_OK) return rc;
        if (t.terms > 1 && (rc = scratch.take((size_t)(a.m * a.k), &lo)) != WE_OK) return rc;
        if ((rc = scratch.take((size_t)a.m * 4, &rs)) != WE_OK) return rc;
        const char* xp = static_cast<const char*>(x) + a.x_offset * 2;
        LK(we::launch_quant_act(xp, WE_BF16, a.m, a.k, a.x_stride, t.terms, (uint8_t*)hi, (uint8_t*)lo, (float*)rs,
                                ctx->sms, st),
           "activation split");
        t.x[0] = hi;
        t.x[1] = lo ? lo : hi;
        t.row_scale = (const float*)rs;
        ready = true;
      }
    } else if (a.w_dtype == WE_BF16) {
      t.kind_f16 = 1;
      t.terms = 1;
      t.w = static_cast<const uint16_t*>(w) + a.w_offset;
      t.w_stride_bytes = a.w_stride * 2;
      t.x[0] = t.x[1] = static_cast<const uint16_t*>(x) + a.x_offset;
      t.x_stride_bytes = a.x_stride * 2;
      ready = we::gemm_tc_supported(t);
    } else if (a.w_dtype == WE_INT4G64) {
      t.kind_f16 = 1;
      t.terms = 1;
      t.w_stride_bytes = a.k * 2;
      t.x[0] = t.x[1] = static_cast<const uint16_t*>(x) + a.x_offset;
      t.x_stride_bytes = a.x_stride * 2;
      // In-kernel unpack (the GEMM's converter warps write bf16_rne(q * s) into shared memory) converts each weight
      // once per 256-token tile; decoding W to bf16 in HBM first converts it once and costs n k 4 bytes of traffic.
      // Measured on config 2's shapes: the in-kernel form wins with one token tile and at least sms / 2 weight-row
      // tiles (M <= 256, N = 12288: 49 against 58 us), decoding wins everywhere else (M = 4608: 0.27 against 0.43 ms).
      // Both give the same bf16 operand, so the choice changes no value.
      bool fuse = a.m <= 256 && ((a.n + 127) / 128) * 2 >= ctx->sms;
      if (const char* env = getenv("WE_TC_I4"))  // tuning / test override: 1 in-kernel unpack, 0 decode first
        fuse = atoi(env) == 1;
      t.int4 = 1;
      t.w = w;
      t.group_scale = a.group_scale;
      ready = fuse && we::gemm_tc_supported(t);
      t.int4 = 0;
      t.w = reinterpret_cast<void*>(256);
      if (ready) {
        t.int4 = 1;
        t.w = w;
      } else if (((uintptr_t)w & 3) == 0 && we::gemm_tc_supported(t)) {
        // packed weights 4- but not 16-byte aligned: decode to bf16 first (the decode reads 4-byte words); less
        // aligned packed weights go to the CUDA-core kernel, which reads bytes
        void* wb;
        if ((rc = scratch.take((size_t)(a.n * a.k * 2), &wb)) != WE_OK) return rc;
        LK(we::launch_unpack_int4(static_cast<const uint8_t*>(w), a.group_scale, a.n, a.k, (uint16_t*)wb, ctx->sms, st),
           "int4 decode");
        t.w = wb;
        ready = true;
      }
    }
    if (ready) {
      cudaError_t e = we::launch_gemm_tc(t, ctx->sms, st);
      if (e == cudaSuccess) {
        ctx->stats.launches++;
        ctx->stats.tc_gemms++;
        return WE_OK;
      }
      if (e != cudaErrorNotSupported) return cuda_fail(ctx, e, "tcgen05 gemm");
    }
  }
  LK(we::launch_gemm_simt(x, w, y, a, st), "simt gemm");
  ctx->stats.simt_gemms++;
  return WE_OK;
}

int we_matmul(we_ctx* ctx, const we_matmul_desc* d, const void* x, const void* w, void* y) {
  if (!ctx) return WE_EINVAL;
  return matmul_impl(ctx, d, x, w, y);
}

int we_gemm_fp8(we_ctx* ctx, const we_gemm_fp8_desc* d) {
  if (!ctx) return WE_EINVAL;
  const bool split = d && d->part_n[0] > 0;
  if (!d || !d->x_hi || !d->w || (!d->y && !split)) return fail(ctx, WE_EINVAL, "we_gemm_fp8: missing operand");
  if (!act_dtype_ok(d->y_dtype)) return fail(ctx, WE_EINVAL, "y must be f32 or bf16");
  int64_t ends[3] = {0, 0, 0};
  if (split) {
    bool ok = !d->epi.aux_op;
    int64_t end = 0;
    for (int i = 0; i < 3; i++) {
      if (d->part_n[i] < 0) ok = false;
      if (d->part_n[i] > 0 && !d->y_parts[i]) ok = false;
      if (i > 0 && d->part_n[i] > 0 && end % 32) ok = false;  // a boundary inside an epilogue warp's 32 channels
      end += d->part_n[i];
      ends[i] = end;
    }
    if (!ok || end != d->n)
      return fail(ctx, WE_EINVAL, "split output needs parts whose widths sum to n, boundaries at multiples of 32, "
                                  "a buffer for every part and no aux operand");
  }
  if (d->nseg < 0 || d->nseg > WE_GEMM_MAX_SEGMENTS)
    return fail(ctx, WE_EINVAL, "two weight sets take 1 to " + std::to_string(WE_GEMM_MAX_SEGMENTS) + " row segments");
  if (d->nseg > 0) {
    bool ok = (!d->epi.gate) == (!d->gate2), any1 = false;
    for (int i = 0; i < d->nseg; i++) {
      ok = ok && d->row_end[i] > (i ? d->row_end[i - 1] : 0) && (d->row_set[i] == 0 || d->row_set[i] == 1);
      any1 = any1 || d->row_set[i] == 1;
    }
    ok = ok && d->row_end[d->nseg - 1] == d->m && (!any1 || d->w2);
    if (!ok)
      return fail(ctx, WE_EINVAL, "row segments must increase to m, name set 0 or 1, have w2 for set 1, and give "
                                  "gate2 iff epi.gate");
  }
  if (d->peer_world != 0) {
    const int pp = d->peer_part;
    bool ok = d->peer_world > 0 && d->peer_world <= WE_PEER_MAX && d->y_dtype == WE_BF16 && !d->epi.aux_op &&
              !(d->flags & WE_MM_ACCUMULATE) && pp >= 0 && pp < (split ? 3 : 1);
    if (ok) {
      const int64_t lo = split && pp ? ends[pp - 1] : 0, hi = split ? ends[pp] : d->n;
      ok = hi > lo && lo % 128 == 0 && (hi - lo) % (128 * (int64_t)d->peer_world) == 0 && d->peer_row0 >= 0;
      for (int r = 0; ok && r < d->peer_world; r++) ok = d->peer_dst[r] && (uintptr_t)d->peer_dst[r] % 16 == 0;
    }
    if (!ok)
      return fail(ctx, WE_EINVAL, "peer output needs bf16 y, no aux operand or accumulate, a part of heads of 128 "
                                  "that split over 1 to 8 ranks, and a 16-byte aligned destination per rank");
  }
  if (d->m == 0 || d->n == 0) return WE_OK;
  we::TcGemmArgs t{};
  t.m = d->m;
  t.n = d->n;
  t.k = d->k;
  t.kind_f16 = 0;
  if (d->peer_world > 0) {
    t.peer = 1;
    t.peer_part = d->peer_part;
    t.peer_world = d->peer_world;
    t.peer_row0 = d->peer_row0;
    for (int r = 0; r < d->peer_world; r++) t.peer_dst[r] = d->peer_dst[r];
  }
  if (d->nseg > 0) {
    t.w2 = d->w2 ? d->w2 : d->w;
    t.scale2 = d->scale2;
    t.chan_scale2 = d->chan_scale2;
    t.bias2 = d->bias2;
    t.gate2 = d->gate2;
    t.nseg = d->nseg;
    for (int i = 0; i < d->nseg; i++) {
      t.row_end[i] = d->row_end[i];
      t.row_set[i] = d->row_set[i];
    }
  }
  t.terms = d->x_lo ? 2 : 1;
  t.x[0] = d->x_hi;
  t.x[1] = d->x_lo ? d->x_lo : d->x_hi;
  t.x_stride_bytes = d->k;
  t.w = d->w;
  t.w_stride_bytes = d->k;
  t.row_scale = d->row_scale;
  t.scale = d->scale;
  t.chan_scale = d->chan_scale;
  t.bias = d->bias;
  t.y = d->y;
  t.y_stride = d->y_stride ? d->y_stride : d->n;
  if (split) {
    for (int i = 0; i < 3; i++) {
      t.ys[i] = d->y_parts[i];
      t.seg_end[i] = ends[i];
    }
    t.y = d->y_parts[0];
    t.y_stride = d->part_n[0];
  }
  t.y_dtype = d->y_dtype;
  t.accumulate = (d->flags & WE_MM_ACCUMULATE) ? 1 : 0;
  t.epi.act = d->epi.act;
  t.epi.aux_op = d->epi.aux_op;
  t.epi.aux_dtype = d->epi.aux_dtype;
  t.epi.aux = d->epi.aux;
  t.epi.gate = d->epi.gate;
  t.dev_err = ctx->dev_err;
  if (!we::gemm_tc_supported(t))
    return fail(ctx, WE_EINVAL, "we_gemm_fp8 needs K a multiple of 16 and 16-byte aligned operands");
  const cudaError_t e = we::launch_gemm_tc(t, ctx->sms, ctx->stream);
  if (e == cudaErrorNotSupported && t.nseg > 0)
    return fail(ctx, WE_EINVAL, "row segment boundaries must be multiples of 64 rows");
  CK(e, "tcgen05 gemm");
  ctx->stats.launches++;
  ctx->stats.tc_gemms++;
  return WE_OK;
}

// ---------------- ops ----------------
static int sum_partials(we_ctx* ctx, const float* partials, int64_t split, int64_t count, float* out);

// The linear's GEMM descriptor for m rows, and its shape checks (LoRA included), before anything is enqueued.
static int linear_check(we_ctx* ctx, int32_t x_dtype, const we_linear* w, int64_t m, int32_t y_dtype, uint32_t flags) {
  if (w->lora_down || w->lora_up) {
    const we_linear *down = w->lora_down, *up = w->lora_up;
    if (!down || !up || down->k != w->k || up->n != w->n || up->k != down->n || down->n % 4)
      return fail(ctx, WE_EINVAL, "LoRA shapes do not fit the linear layer");
  }
  we_matmul_desc d{};
  d.m = m;
  d.n = w->n;
  d.k = w->k;
  d.scale = w->scale;
  d.chan_scale = w->chan_scale;
  d.group_scale = w->group_scale;
  d.bias = w->bias;
  d.x_dtype = x_dtype;
  d.w_dtype = w->dtype;
  d.y_dtype = y_dtype;
  d.flags = flags & (WE_MM_FP8_FAST | WE_MM_FORCE_SIMT);
  return we_matmul_check(ctx, &d);
}

static int linear_into(we_ctx* ctx, const void* x, int32_t x_dtype, const we_linear* w, int64_t m, int32_t y_dtype,
                       uint32_t flags, void* y);

int we_linear_forward(we_ctx* ctx, const void* x, int32_t x_dtype, const we_linear* w, int64_t m, int32_t y_dtype,
                      uint32_t flags, void** y) {
  if (!ctx || !w || !y) return WE_EINVAL;
  int rc = linear_check(ctx, x_dtype, w, m, y_dtype, flags);
  if (rc != WE_OK) return rc;
  if ((rc = op_output(ctx, (size_t)(m * w->n) * dsize(y_dtype), y)) != WE_OK) return rc;
  return linear_into(ctx, x, x_dtype, w, m, y_dtype, flags, *y);
}

// y[m, n] = linear(x) into an existing buffer: the body of we_linear_forward, also run per row chunk by
// we_linear_host.
static int linear_into(we_ctx* ctx, const void* x, int32_t x_dtype, const we_linear* w, int64_t m, int32_t y_dtype,
                       uint32_t flags, void* y) {
  int rc;
  we_matmul_desc d{};
  d.m = m;
  d.n = w->n;
  d.k = w->k;
  d.scale = w->scale;
  d.chan_scale = w->chan_scale;
  d.group_scale = w->group_scale;
  d.bias = w->bias;
  d.x_dtype = x_dtype;
  d.w_dtype = w->dtype;
  d.y_dtype = y_dtype;
  d.flags = flags & (WE_MM_FP8_FAST | WE_MM_FORCE_SIMT);
  if ((rc = matmul_impl(ctx, &d, x, w->weight, y)) != WE_OK) return rc;
  if (!w->lora_down) return WE_OK;
  // narrowLinear (ops.ts:48-58): t = x . down^T, split over K when narrow, then y += up.scale t . up^T
  const we_linear *down = w->lora_down, *up = w->lora_up;
  Scratch scratch(ctx);
  void* t;
  if ((rc = scratch.take((size_t)(m * down->n) * 4, &t)) != WE_OK) return rc;
  const int64_t split = we_ksplit_for(m, down->n, down->k);
  we_matmul_desc dd{};
  dd.m = m;
  dd.n = down->n;
  dd.k = down->k;
  dd.scale = down->scale;
  dd.chan_scale = down->chan_scale;
  dd.group_scale = down->group_scale;
  dd.x_dtype = x_dtype;
  dd.w_dtype = down->dtype;
  dd.y_dtype = WE_F32;
  if (split == 1) {
    if ((rc = matmul_impl(ctx, &dd, x, down->weight, t)) != WE_OK) return rc;
  } else {
    void* parts;
    if ((rc = scratch.take((size_t)(split * m * down->n) * 4, &parts)) != WE_OK) return rc;
    dd.k_split = split;
    if ((rc = matmul_impl(ctx, &dd, x, down->weight, parts)) != WE_OK) return rc;
    if ((rc = sum_partials(ctx, (const float*)parts, split, m * down->n, (float*)t)) != WE_OK) return rc;
  }
  we_matmul_desc du{};
  du.m = m;
  du.n = up->n;
  du.k = up->k;
  du.scale = up->scale;
  du.chan_scale = up->chan_scale;
  du.group_scale = up->group_scale;
  du.x_dtype = WE_F32;
  du.w_dtype = up->dtype;
  du.y_dtype = y_dtype;
  du.flags = WE_MM_ACCUMULATE;
  return matmul_impl(ctx, &du, t, up->weight, y);
}

int we_linear_host(we_ctx* ctx, const void* x_host, int32_t x_dtype, const we_linear* w, int64_t m,
                   int32_t y_dtype, uint32_t flags, void* y_host, int64_t chunk_rows) {
  if (!ctx || !w || m < 0 || chunk_rows < 0 || (m > 0 && (!x_host || !y_host))) return WE_EINVAL;
  if (ctx->capturing) return fail(ctx, WE_EINVAL, "cannot read back while capturing a graph");
  int rc = linear_check(ctx, x_dtype, w, m, y_dtype, flags);
  if (rc != WE_OK || m == 0) return rc;
  // about 12 chunks: at config 2 (4608 x 12288 bf16 out) 8, 12, 18 and 36 chunks measured 2.25, 2.21, 2.27 and
  // 2.39 ms; fewer chunks lengthen the first upload and the last read-back, more add per-copy overhead
  if (chunk_rows == 0) chunk_rows = std::max<int64_t>(128, ((m + 11) / 12 + 127) / 128 * 128);
  const int64_t chunks = (m + chunk_rows - 1) / chunk_rows;
  const size_t xrow = (size_t)w->k * dsize(x_dtype), yrow = (size_t)w->n * dsize(y_dtype);
  if (!ctx->h2d) CK(cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking), "copy stream");
  if (!ctx->d2h) CK(cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking), "copy stream");
  while (ctx->io_events.size() < (size_t)(2 * chunks + 2)) {
    cudaEvent_t ev;
    CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
    ctx->io_events.push_back(ev);
  }
  cudaEvent_t* ev = ctx->io_events.data();  // [0] start, [1] end, [2 + 2c] x chunk c in, [3 + 2c] y chunk c out
  Scratch scratch(ctx);
  void *xd, *yd;
  if ((rc = scratch.take((size_t)m * xrow, &xd)) != WE_OK) return rc;
  if ((rc = scratch.take((size_t)m * yrow, &yd)) != WE_OK) return rc;
  // Before the scratch goes back to the pool (a stream-ordered reuse on the compute stream), the compute stream
  // waits for the last device -> host copy; on an error part-way, the copies already enqueued finish first.
  struct Drain {
    we_ctx* c;
    bool ok = false;
    ~Drain() {
      if (ok) return;
      cudaStreamSynchronize(c->h2d);
      cudaStreamSynchronize(c->d2h);
    }
  } drain{ctx};
  // the pooled buffers may still be read by earlier work of the compute stream
  CK(cudaEventRecord(ev[0], ctx->stream), "cudaEventRecord");
  CK(cudaStreamWaitEvent(ctx->h2d, ev[0], 0), "cudaStreamWaitEvent");
  for (int64_t c = 0; c < chunks; c++) {  // every input chunk goes first: the link runs ahead of the GEMMs
    const int64_t r0 = c * chunk_rows, rows = std::min(chunk_rows, m - r0);
    CK(cudaMemcpyAsync(static_cast<char*>(xd) + r0 * xrow, static_cast<const char*>(x_host) + r0 * xrow,
                       rows * xrow, cudaMemcpyHostToDevice, ctx->h2d),
       "host -> device chunk");
    CK(cudaEventRecord(ev[2 + 2 * c], ctx->h2d), "cudaEventRecord");
  }
  for (int64_t c = 0; c < chunks; c++) {
    const int64_t r0 = c * chunk_rows, rows = std::min(chunk_rows, m - r0);
    CK(cudaStreamWaitEvent(ctx->stream, ev[2 + 2 * c], 0), "cudaStreamWaitEvent");
    if ((rc = linear_into(ctx, static_cast<const char*>(xd) + r0 * xrow, x_dtype, w, rows, y_dtype, flags,
                          static_cast<char*>(yd) + r0 * yrow)) != WE_OK)
      return rc;
    CK(cudaEventRecord(ev[3 + 2 * c], ctx->stream), "cudaEventRecord");
    CK(cudaStreamWaitEvent(ctx->d2h, ev[3 + 2 * c], 0), "cudaStreamWaitEvent");
    CK(cudaMemcpyAsync(static_cast<char*>(y_host) + r0 * yrow, static_cast<char*>(yd) + r0 * yrow, rows * yrow,
                       cudaMemcpyDeviceToHost, ctx->d2h),
       "device -> host chunk");
  }
  CK(cudaEventRecord(ev[1], ctx->d2h), "cudaEventRecord");
  CK(cudaStreamWaitEvent(ctx->stream, ev[1], 0), "cudaStreamWaitEvent");
  drain.ok = true;
  CK(cudaStreamSynchronize(ctx->stream), "we_linear_host sync");
  return WE_OK;
}

int we_no_mod(we_ctx* ctx, int64_t d, we_mod* out) {
  if (!ctx || !out) return WE_EINVAL;
  void *s, *h;
  int rc = we_buffer(ctx, (size_t)d * 4, nullptr, &s);
  if (rc != WE_OK) return rc;
  if ((rc = we_buffer(ctx, (size_t)d * 4, nullptr, &h)) != WE_OK) return rc;
  out->scale = (const float*)s;
  out->shift = (const float*)h;
  return WE_OK;
}

int we_rmsnorm(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, const float* scale, const float* shift,
               int64_t rows, int64_t d, float eps, float offset, void* out, int32_t out_dtype) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(out_dtype)) return fail(ctx, WE_EINVAL, "x and out must be f32 or bf16");
  if (d <= 0 || rows < 0) return fail(ctx, WE_EINVAL, "rows and d must be positive");
  if (rows == 0) return WE_OK;
  LK(we::launch_rmsnorm(x, x_dtype, weight, scale, shift, rows, d, eps, offset, out, out_dtype, ctx->sms, ctx->stream),
     "rmsnorm");
  return WE_OK;
}

int we_norm(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, int64_t rows, int64_t d, const we_mod* mod,
            float eps, float offset, int32_t out_dtype, void** out) {
  if (!ctx || !out) return WE_EINVAL;
  int rc = op_output(ctx, (size_t)(rows * d) * dsize(out_dtype), out);
  if (rc != WE_OK) return rc;
  return we_rmsnorm(ctx, x, x_dtype, weight, mod ? mod->scale : nullptr, mod ? mod->shift : nullptr, rows, d, eps,
                    offset, *out, out_dtype);
}

int we_rope_apply(we_ctx* ctx, const void* x, int32_t x_dtype, const float* cos, const float* sin, int64_t tokens,
                  int64_t heads, int64_t pairs, int32_t pairing, void* out, int32_t out_dtype) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(out_dtype)) return fail(ctx, WE_EINVAL, "x and out must be f32 or bf16");
  if (pairing != WE_ROPE_INTERLEAVED && pairing != WE_ROPE_HALF) return fail(ctx, WE_EINVAL, "unknown pairing");
  if (tokens < 0 || heads < 0 || pairs < 0) return fail(ctx, WE_EINVAL, "negative size");
  if (tokens == 0 || heads == 0 || pairs == 0) return WE_OK;
  LK(we::launch_rope(x, x_dtype, cos, sin, tokens, heads, pairs, pairing, out, out_dtype, ctx->sms, ctx->stream), "rope");
  return WE_OK;
}

int we_rotate(we_ctx* ctx, const void* x, int32_t x_dtype, int64_t heads, const we_rope* rope, int32_t pairing,
              int32_t out_dtype, void** out) {
  if (!ctx || !rope || !out) return WE_EINVAL;
  int rc = op_output(ctx, (size_t)(rope->tokens * heads * rope->pairs * 2) * dsize(out_dtype), out);
  if (rc != WE_OK) return rc;
  return we_rope_apply(ctx, x, x_dtype, rope->cos, rope->sin, rope->tokens, heads, rope->pairs, pairing, *out,
                       out_dtype);
}

int we_qknorm_rope(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, float eps, float offset,
                   const float* cos, const float* sin, int64_t tokens, int64_t heads, int64_t pairs, int32_t pairing,
                   void* out, int32_t out_dtype) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(x_dtype) || !act_dtype_ok(out_dtype)) return fail(ctx, WE_EINVAL, "x and out must be f32 or bf16");
  if (pairing != WE_ROPE_INTERLEAVED && pairing != WE_ROPE_HALF) return fail(ctx, WE_EINVAL, "unknown pairing");
  if (tokens == 0 || heads == 0 || pairs == 0) return WE_OK;
  cudaError_t e = we::launch_qknorm_rope(x, x_dtype, weight, eps, offset, cos, sin, tokens, heads, pairs, pairing, out,
                                         out_dtype, ctx->sms, ctx->stream);
  if (e == cudaErrorNotSupported) {
    // no fused variant for this head size: norm into `out` (f32 keeps the intermediate exact), rotate in place
    Scratch scratch(ctx);
    void* tmp;
    int rc = scratch.take((size_t)(tokens * heads * pairs * 2) * 4, &tmp);
    if (rc != WE_OK) return rc;
    LK(we::launch_rmsnorm(x, x_dtype, weight, nullptr, nullptr, tokens * heads, pairs * 2, eps, offset, tmp, WE_F32,
                          ctx->sms, ctx->stream),
       "qk norm");
    LK(we::launch_rope(tmp, WE_F32, cos, sin, tokens, heads, pairs, pairing, out, out_dtype, ctx->sms, ctx->stream),
       "qk rope");
    return WE_OK;
  }
  CK(e, "qknorm_rope");
  ctx->stats.launches++;
  return WE_OK;
}

int we_qknorm_rope_peers(we_ctx* ctx, const void* x, const float* weight, float eps, float offset, const float* cos,
                         const float* sin, int64_t tokens, int64_t heads, int32_t pairing, void* const* dst,
                         int32_t world, int64_t dst_row0) {
  if (!ctx) return WE_EINVAL;
  if (!x || !weight || !cos || !sin || !dst) return fail(ctx, WE_EINVAL, "qk norm + RoPE to peers: missing buffer");
  if (pairing != WE_ROPE_INTERLEAVED && pairing != WE_ROPE_HALF) return fail(ctx, WE_EINVAL, "unknown pairing");
  if (world < 1 || world > WE_PEER_MAX || heads % world)
    return fail(ctx, WE_EINVAL, "the heads must split evenly over 1 to 8 ranks");
  if (tokens == 0 || heads == 0) return WE_OK;
  cudaError_t e = we::launch_qknorm_rope_peers(x, weight, eps, offset, cos, sin, tokens, heads, pairing, dst, world,
                                               dst_row0, ctx->sms, ctx->stream);
  if (e == cudaErrorNotSupported)
    return fail(ctx, WE_EINVAL, "qk norm + RoPE to peers needs 16-byte aligned rows, tables and destinations");
  CK(e, "qknorm_rope_peers");
  ctx->stats.launches++;
  return WE_OK;
}

int64_t we_rope_tables(const int64_t* pos, int64_t tokens, int32_t naxes, const int64_t* axes, double theta, float* cos,
                       float* sin) {
  int64_t pairs = 0;
  for (int a = 0; a < naxes; a++) {
    if (axes[a] % 2) return -1;
    pairs += axes[a] / 2;
  }
  if (!cos || !sin) return pairs;
  for (int64_t t = 0; t < tokens; t++) {
    int64_t pair = 0;
    for (int a = 0; a < naxes; a++) {
      const int64_t dim = axes[a];
      for (int64_t j = 0; j < dim / 2; j++, pair++) {
        const double angle = (double)pos[t * naxes + a] * pow(theta, -(double)(2 * j) / (double)dim);
        cos[t * pairs + pair] = (float)::cos(angle);
        sin[t * pairs + pair] = (float)::sin(angle);
      }
    }
  }
  return pairs;
}

int we_positions(int64_t text, int64_t rows, int64_t cols, int64_t* pos) {
  if (!pos || text < 0 || rows < 0 || cols < 0) return WE_EINVAL;
  int64_t t = 0;
  for (int64_t i = 0; i < text; i++, t++) pos[3 * t] = pos[3 * t + 1] = pos[3 * t + 2] = 0;
  for (int64_t i = 0; i < rows * cols; i++, t++) {
    pos[3 * t] = 0;
    pos[3 * t + 1] = i / cols;
    pos[3 * t + 2] = i % cols;
  }
  return WE_OK;
}

// ---------------- elementwise / norm + split ----------------
int we_elementwise(we_ctx* ctx, int32_t op, const void* a, const void* b, const float* g, int64_t n, int64_t d,
                   int32_t dtype, void* out, int32_t out_dtype) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(dtype) || !act_dtype_ok(out_dtype)) return fail(ctx, WE_EINVAL, "inputs and out must be f32 or bf16");
  if (op < WE_EW_SWIGLU || op > WE_EW_SILU) return fail(ctx, WE_EINVAL, "unknown elementwise op");
  const bool needs_b = op == WE_EW_SWIGLU || op == WE_EW_SIGMOID_GATE || op == WE_EW_GATED_ADD || op == WE_EW_ADD;
  const bool needs_g = op == WE_EW_GATED_ADD || op == WE_EW_ADD_BIAS;
  if ((needs_b && !b) || (needs_g && (!g || d <= 0))) return fail(ctx, WE_EINVAL, "missing input of the elementwise op");
  if (n <= 0) return WE_OK;
  LK(we::launch_elementwise(op, a, needs_b ? b : nullptr, needs_g ? g : nullptr, n, d > 0 ? d : 1, dtype, out, out_dtype,
                            ctx->sms, ctx->stream),
     "elementwise");
  return WE_OK;
}

int we_ew(we_ctx* ctx, int32_t op, const void* a, const void* b, const float* g, int64_t n, int64_t d, int32_t dtype,
          int32_t out_dtype, void** out) {
  if (!ctx || !out) return WE_EINVAL;
  int rc = op_output(ctx, (size_t)n * dsize(out_dtype), out);
  if (rc != WE_OK) return rc;
  return we_elementwise(ctx, op, a, b, g, n, d, dtype, *out, out_dtype);
}

int we_norm_split(we_ctx* ctx, const void* x, int32_t x_dtype, const float* weight, const float* scale,
                  const float* shift, int64_t rows, int64_t d, float eps, float offset, int32_t terms, uint8_t* hi,
                  uint8_t* lo, float* row_scale) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(x_dtype)) return fail(ctx, WE_EINVAL, "x must be f32 or bf16");
  if (terms != 1 && terms != 2) return fail(ctx, WE_EINVAL, "terms must be 1 or 2");
  if (terms == 2 && !lo) return fail(ctx, WE_EINVAL, "two terms need a lo buffer");
  if (rows <= 0) return WE_OK;
  cudaError_t e = we::launch_norm_split(x, x_dtype, weight, scale, shift, rows, d, eps, offset, terms, hi, lo,
                                        row_scale, ctx->sms, ctx->stream);
  if (e == cudaErrorNotSupported)
    return fail(ctx, WE_EINVAL, "norm + split needs d % 8 == 0, d <= 8192 and 16-byte aligned rows");
  CK(e, "norm + split");
  ctx->stats.launches++;
  return WE_OK;
}

int we_add_norm_split(we_ctx* ctx, const float* x, const float* r, float* xo, const float* weight, const float* scale,
                      const float* shift, int64_t rows, int64_t d, float eps, float offset, int32_t terms, uint8_t* hi,
                      uint8_t* lo, float* row_scale) {
  if (!ctx) return WE_EINVAL;
  if (!x || !r || !xo || !weight || !hi || !row_scale) return fail(ctx, WE_EINVAL, "add + norm + split: missing buffer");
  if (terms != 1 && terms != 2) return fail(ctx, WE_EINVAL, "terms must be 1 or 2");
  if (terms == 2 && !lo) return fail(ctx, WE_EINVAL, "two terms need a lo buffer");
  if (rows <= 0) return WE_OK;
  cudaError_t e = we::launch_add_norm_split(x, r, xo, weight, scale, shift, rows, d, eps, offset, terms, hi, lo,
                                            row_scale, ctx->sms, ctx->stream);
  if (e == cudaErrorNotSupported)
    return fail(ctx, WE_EINVAL, "add + norm + split needs d <= 8192, d % 8 == 0 and 16-byte aligned rows");
  CK(e, "add + norm + split");
  ctx->stats.launches++;
  return WE_OK;
}

// ---------------- CUDA graphs: capture a sequence of this library's ops once, replay it ----------------
int we_capture_begin(we_ctx* ctx) {
  if (!ctx) return WE_EINVAL;
  if (ctx->capturing) return fail(ctx, WE_EINVAL, "a capture is already open");
  if (ctx->stream == nullptr) return fail(ctx, WE_EINVAL, "cannot capture the legacy default stream");
  CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed), "begin capture");
  ctx->capturing = true;
  ctx->cap_launches0 = ctx->stats.launches;
  return WE_OK;
}

int we_capture_end(we_ctx* ctx, we_graph** out) {
  if (!ctx || !out) return WE_EINVAL;
  if (!ctx->capturing) return fail(ctx, WE_EINVAL, "no capture is open");
  *out = nullptr;
  ctx->capturing = false;
  we_graph* g = new we_graph();
  g->bufs.swap(ctx->cap_bufs);
  g->host.swap(ctx->cap_host);
  g->launches = ctx->stats.launches - ctx->cap_launches0;
  ctx->cap_pool.clear();
  // the graph's buffers leave the context: no release or free may hand them to anything else
  for (void* b : g->bufs) {
    ctx->sizes.erase(b);
    auto it = std::find(ctx->owned.begin(), ctx->owned.end(), b);
    if (it != ctx->owned.end()) ctx->owned.erase(it);
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&g->exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    cudaGetLastError();
    graph_free(g);
    return cuda_fail(ctx, e, "end capture");
  }
  ctx->graphs.push_back(g);
  *out = g;
  return WE_OK;
}

int we_graph_launch(we_ctx* ctx, we_graph* g) {
  if (!ctx || !g) return WE_EINVAL;
  if (ctx->capturing) return fail(ctx, WE_EINVAL, "cannot replay a graph while capturing");
  CK(cudaGraphLaunch(g->exec, ctx->stream), "graph launch");
  ctx->stats.launches += g->launches;
  return WE_OK;
}

int we_graph_destroy(we_ctx* ctx, we_graph* g) {
  if (!ctx || !g) return WE_EINVAL;
  auto it = std::find(ctx->graphs.begin(), ctx->graphs.end(), g);
  if (it == ctx->graphs.end()) return fail(ctx, WE_EINVAL, "graph is not owned by this context");
  CK(cudaStreamSynchronize(ctx->stream), "graph destroy");  // no replay of it is still running
  ctx->graphs.erase(it);
  graph_free(g);
  return WE_OK;
}

// ---------------- latent <-> tokens ----------------
static int layout_check(we_ctx* ctx, const void* a, const void* b, int32_t adt, int32_t bdt, int64_t c, int64_t h,
                        int64_t w) {
  if (!a || !b) return fail(ctx, WE_EINVAL, "patchify: missing buffer");
  if (!act_dtype_ok(adt) || !act_dtype_ok(bdt)) return fail(ctx, WE_EINVAL, "patchify: f32 or bf16 only");
  if (c <= 0 || h <= 0 || w <= 0) return fail(ctx, WE_EINVAL, "patchify: channels, height and width must be positive");
  return WE_OK;
}

int we_patchify(we_ctx* ctx, const void* latent, int32_t latent_dtype, int64_t channels, int64_t height, int64_t width,
                void* tokens, int32_t tokens_dtype) {
  if (!ctx) return WE_EINVAL;
  int rc = layout_check(ctx, latent, tokens, latent_dtype, tokens_dtype, channels, height, width);
  if (rc != WE_OK) return rc;
  LK(we::launch_patchify(latent, latent_dtype, channels, height, width, tokens, tokens_dtype, ctx->sms, ctx->stream),
     "patchify");
  return WE_OK;
}

int we_unpatchify(we_ctx* ctx, const void* tokens, int32_t tokens_dtype, int64_t channels, int64_t height,
                  int64_t width, void* latent, int32_t latent_dtype) {
  if (!ctx) return WE_EINVAL;
  int rc = layout_check(ctx, tokens, latent, tokens_dtype, latent_dtype, channels, height, width);
  if (rc != WE_OK) return rc;
  LK(we::launch_unpatchify(tokens, tokens_dtype, channels, height, width, latent, latent_dtype, ctx->sms, ctx->stream),
     "unpatchify");
  return WE_OK;
}

int we_head_groups(we_ctx* ctx, const void* rows, void* groups, int64_t tokens, int64_t n_groups, int64_t group_bytes,
                   int32_t to_groups) {
  if (!ctx) return WE_EINVAL;
  if (!rows || !groups) return fail(ctx, WE_EINVAL, "head groups: missing buffer");
  if (group_bytes <= 0 || group_bytes % 16 || ((uintptr_t)rows | (uintptr_t)groups) % 16)
    return fail(ctx, WE_EINVAL, "head groups need 16-byte groups and 16-byte aligned buffers");
  if (tokens < 0 || n_groups <= 0) return fail(ctx, WE_EINVAL, "head groups: bad sizes");
  // to_groups reads rows and writes groups; the reverse reads groups and writes rows
  LK(we::launch_head_groups(to_groups ? rows : groups, to_groups ? groups : const_cast<void*>(rows), tokens, n_groups,
                            group_bytes, to_groups ? 1 : 0, ctx->sms, ctx->stream),
     "head groups");
  return WE_OK;
}

// ---------------- attention ----------------
int we_attention(we_ctx* ctx, const void* q, const void* k, const void* v, int32_t dtype, int64_t tokens, int64_t heads,
                 int64_t kv_heads, int64_t dim, int32_t causal, void* out, int32_t out_dtype) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(dtype) || !act_dtype_ok(out_dtype)) return fail(ctx, WE_EINVAL, "q/k/v and out must be f32 or bf16");
  if (kv_heads <= 0 || heads % kv_heads) return fail(ctx, WE_EINVAL, "heads must be a multiple of kvHeads");
  if (dim <= 0 || dim > 256) return fail(ctx, WE_EINVAL, "dim must be in 1..256");
  if (tokens <= 0 || heads <= 0) return WE_OK;
  we::AttnArgs a{q, k, v, out, tokens, heads, kv_heads, dim, causal ? 1 : 0, dtype, out_dtype};
  if (we::flash_attention_supported(a)) {
    const int splits = we::flash_attention_splits(a, ctx->sms);
    Scratch scratch(ctx);
    void* part = nullptr;
    if (splits > 1) {
      int rc = scratch.take((size_t)we::flash_attention_scratch_bytes(a, splits), &part);
      if (rc != WE_OK) return rc;
    }
    cudaError_t e = we::launch_flash_attention(a, splits, part, ctx->dev_err, ctx->stream);
    if (e == cudaSuccess) {
      ctx->stats.launches += splits > 1 ? 2 : 1;
      return WE_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_fail(ctx, e, "flash attention");
  }
  LK(we::launch_attention_simt(a, ctx->sms, ctx->stream), "attention");
  return WE_OK;
}

int we_attend(we_ctx* ctx, const void* q, const void* k, const void* v, int32_t dtype, int64_t tokens, int64_t heads,
              int64_t kv_heads, int64_t dim, int32_t causal, int32_t out_dtype, void** out) {
  if (!ctx || !out) return WE_EINVAL;
  if (kv_heads <= 0 || heads % kv_heads) return fail(ctx, WE_EINVAL, "heads must be a multiple of kvHeads");
  int rc = op_output(ctx, (size_t)(tokens * heads * dim) * dsize(out_dtype), out);
  if (rc != WE_OK) return rc;
  return we_attention(ctx, q, k, v, dtype, tokens, heads, kv_heads, dim, causal, *out, out_dtype);
}

// ---------------- unpack / quantise ----------------
int we_unpack_fp8(we_ctx* ctx, const uint8_t* bytes, int64_t n, float scale, float* out) {
  if (!ctx) return WE_EINVAL;
  if (n <= 0) return WE_OK;
  LK(we::launch_unpack_fp8_f32(bytes, n, scale, out, ctx->sms, ctx->stream), "unpack fp8");
  return WE_OK;
}

int we_unpack_fp8_bf16(we_ctx* ctx, const uint8_t* bytes, int64_t n, uint16_t* out) {
  if (!ctx) return WE_EINVAL;
  if (n <= 0) return WE_OK;
  LK(we::launch_unpack_fp8_bf16(bytes, n, out, ctx->sms, ctx->stream), "unpack fp8 -> bf16");
  return WE_OK;
}

int we_unpack_int4(we_ctx* ctx, const uint8_t* packed, const uint16_t* scales, int64_t n, int64_t k, uint16_t* out) {
  if (!ctx) return WE_EINVAL;
  if (k % 64) return fail(ctx, WE_EINVAL, "K must be a multiple of 64 for int4 group-64 weights, got " + std::to_string(k));
  if (((uintptr_t)packed & 3) || ((uintptr_t)out & 15))
    return fail(ctx, WE_EINVAL, "int4 decode needs 4-byte aligned input and 16-byte aligned output");
  if (n <= 0) return WE_OK;
  LK(we::launch_unpack_int4(packed, scales, n, k, out, ctx->sms, ctx->stream), "unpack int4");
  return WE_OK;
}

int we_quantize_fp8(we_ctx* ctx, const void* w, int32_t w_dtype, int64_t n, int64_t k, int32_t per_channel, uint8_t* q,
                    float* scales) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(w_dtype)) return fail(ctx, WE_EINVAL, "weights to quantise must be f32 or bf16");
  if (n <= 0 || k <= 0) return WE_OK;
  CK(we::launch_quant_fp8(w, w_dtype, n, k, per_channel != 0, q, scales, ctx->amax_word, ctx->sms, ctx->stream),
     "quantise fp8");
  ctx->stats.launches += per_channel ? 1 : 2;
  return WE_OK;
}

int we_quantize_int4(we_ctx* ctx, const void* w, int32_t w_dtype, int64_t n, int64_t k, uint8_t* packed,
                     uint16_t* scales) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(w_dtype)) return fail(ctx, WE_EINVAL, "weights to quantise must be f32 or bf16");
  if (k % 64) return fail(ctx, WE_EINVAL, "K must be a multiple of 64 for int4 group-64 weights, got " + std::to_string(k));
  if (n <= 0 || k <= 0) return WE_OK;
  LK(we::launch_quant_int4(w, w_dtype, n, k, packed, scales, ctx->sms, ctx->stream), "quantise int4");
  return WE_OK;
}

int we_quantize_act(we_ctx* ctx, const void* x, int32_t x_dtype, int64_t m, int64_t k, int64_t x_stride, int32_t terms,
                    uint8_t* hi, uint8_t* lo, float* row_scale) {
  if (!ctx) return WE_EINVAL;
  if (!act_dtype_ok(x_dtype)) return fail(ctx, WE_EINVAL, "x must be f32 or bf16");
  if (terms != 1 && terms != 2) return fail(ctx, WE_EINVAL, "terms must be 1 or 2");
  if (terms == 2 && !lo) return fail(ctx, WE_EINVAL, "two terms need a lo buffer");
  if (m <= 0 || k <= 0) return WE_OK;
  LK(we::launch_quant_act(x, x_dtype, m, k, x_stride ? x_stride : k, terms, hi, lo, row_scale, ctx->sms, ctx->stream),
     "activation split");
  return WE_OK;
}

}  // extern "C"

// layerSum with unit weights (src/kernels/text.ts:67-84 as used by narrowLinear, ops.ts:55-57)
__global__ void sum_partials_kernel(const float* __restrict__ p, int64_t split, int64_t count, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int64_t z = 0; z < split; z++) s += p[z * count + i];
    out[i] = s;
  }
}
static int sum_partials(we_ctx* ctx, const float* partials, int64_t split, int64_t count, float* out) {
  int64_t g = std::min<int64_t>((count + 255) / 256, (int64_t)ctx->sms * 8);
  sum_partials_kernel<<<(unsigned)std::max<int64_t>(g, 1), 256, 0, ctx->stream>>>(partials, split, count, out);
  LK(cudaGetLastError(), "sum partials");
  return WE_OK;
}
