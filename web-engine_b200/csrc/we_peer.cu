// Peer memory of the GPUs of one node, for sequence parallelism without a collective library on the data path.
//
// The reference runs on one GPU. When one image's step is split over N GPUs by token rows, attention needs every
// token of a head: q, k and v go from token shards to head shards and the output comes back (an all-to-all each).
// Here each rank owns an exchange region in its HBM, exported with CUDA IPC and opened by every other rank of the
// node. One kernel (peer_exchange_kernel) copies each (peer, row) chunk of the sources straight into the owning
// rank's region over NVLink (plain 16-byte peer stores, no multicast), then the ranks meet at a flag barrier
// in the same memory:
//   * every CTA fences its stores (system scope) and counts itself done; the last CTA bumps this rank's
//     epoch (a device counter, so a captured graph replays correctly), writes it into slot `rank` of every
//     rank's flag array, and waits until its own flag array holds the epoch from every rank;
//   * the next kernel on the stream therefore sees every peer's chunks. Each wait is bounded: after the
//     timeout the kernel records DEV_ERR_TIMEOUT_PEER in the context's error word and returns.
// A rank cannot run two exchanges ahead of another (each exchange waits for all flags), so regions that the
// caller uses in alternation (even / odd blocks) are never written while a peer still reads them.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

// defined in we_api.cu
int we_ctx_fail(we_ctx* ctx, int code, const std::string& msg);
cudaStream_t we_ctx_stream(we_ctx* ctx);
uint32_t* we_ctx_dev_err(we_ctx* ctx);
void we_ctx_count_launch(we_ctx* ctx);

namespace {
constexpr int MAXC = 4;       // copies per launch
constexpr int SYNC_WORDS = 16;  // flags[WE_PEER_MAX], then epoch and the CTA counter of this rank

struct CopyArgs {
  const char* src;
  int64_t rows, words;  // rows per peer, 16-byte words per (peer, row) chunk
  int64_t src_row, src_peer, dst_off, dst_row, dst_rank;  // bytes
};
struct ExchangeArgs {
  CopyArgs c[MAXC];
  int64_t first[MAXC + 1];  // prefix sums of world * rows over the copies: chunk index ranges
  char* base[WE_PEER_MAX];
  uint32_t* flags[WE_PEER_MAX];
  uint32_t* local_sync;
  uint32_t* err;
  int ncopies, rank, world;
  uint64_t timeout_ns;
};

// One warp per (copy, peer, row) chunk; its lanes stride the chunk's 16-byte words.
__global__ void __launch_bounds__(256) peer_exchange_kernel(const __grid_constant__ ExchangeArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = a.first[a.ncopies];
  for (int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < total; q += warps) {
    int c = 0;
    while (c + 1 < a.ncopies && q >= a.first[c + 1]) c++;
    const CopyArgs& cp = a.c[c];
    const int64_t local = q - a.first[c];
    const int p = (int)(local / cp.rows);
    const int64_t i = local - (int64_t)p * cp.rows;
    const uint4* s = reinterpret_cast<const uint4*>(cp.src + p * cp.src_peer + i * cp.src_row);
    uint4* d = reinterpret_cast<uint4*>(a.base[p] + cp.dst_off + a.rank * cp.dst_rank + i * cp.dst_row);
    for (int64_t w = lane; w < cp.words; w += 32) d[w] = s[w];
  }
  // barrier: the last CTA of this rank signals every rank and waits for all of them
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t* epoch = a.local_sync + WE_PEER_MAX;
  uint32_t* done = a.local_sync + WE_PEER_MAX + 1;
  if (atomicAdd(done, 1u) != gridDim.x - 1) return;
  __threadfence_system();
  *done = 0;
  const uint32_t e = *epoch + 1;
  *epoch = e;
  for (int p = 0; p < a.world; p++) {
    volatile uint32_t* f = a.flags[p] + a.rank;
    *f = e;
  }
  __threadfence_system();
  const uint64_t t0 = we::global_timer_ns();
  for (int p = 0; p < a.world; p++) {
    volatile uint32_t* f = a.local_sync + p;
    while ((int32_t)(*f - e) < 0) {
      if (we::global_timer_ns() - t0 > a.timeout_ns) {
        atomicCAS(a.err, 0u, (uint32_t)we::DEV_ERR_TIMEOUT_PEER);
        return;
      }
    }
  }
  __threadfence_system();
}
}  // namespace

struct we_peer {
  we_ctx* ctx = nullptr;
  int rank = 0, world = 1;
  size_t bytes = 0;
  char* region = nullptr;     // this rank's exchange region
  uint32_t* sync = nullptr;   // this rank's flags + epoch + counter
  char* base[WE_PEER_MAX] = {};
  uint32_t* flags[WE_PEER_MAX] = {};
  std::vector<void*> opened;  // IPC mappings to close
};

#define PCK(call, what)                                                                                  \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess) return we_ctx_fail(ctx, WE_ECUDA, std::string(what) + ": " + cudaGetErrorString(e_)); \
  } while (0)

int we_peer_create(we_ctx* ctx, int32_t rank, int32_t world, size_t bytes, we_peer** out) {
  if (!ctx || !out) return WE_EINVAL;
  *out = nullptr;
  if (world < 1 || world > WE_PEER_MAX || rank < 0 || rank >= world)
    return we_ctx_fail(ctx, WE_EINVAL, "peer groups hold 1 to 8 ranks, and rank must be below world");
  we_peer* p = new we_peer;
  p->ctx = ctx;
  p->rank = rank;
  p->world = world;
  p->bytes = (bytes + 255) / 256 * 256;
  cudaError_t e = cudaMalloc(&p->region, p->bytes ? p->bytes : 256);
  if (e == cudaSuccess) e = cudaMalloc(&p->sync, SYNC_WORDS * 4);
  if (e == cudaSuccess) e = cudaMemset(p->sync, 0, SYNC_WORDS * 4);
  if (e != cudaSuccess) {
    cudaFree(p->region);
    cudaFree(p->sync);
    delete p;
    return we_ctx_fail(ctx, e == cudaErrorMemoryAllocation ? WE_ENOMEM : WE_ECUDA,
                       std::string("peer region: ") + cudaGetErrorString(e));
  }
  p->base[rank] = p->region;
  p->flags[rank] = p->sync;
  *out = p;
  return WE_OK;
}

int we_peer_export(const we_peer* p, void* handle) {
  if (!p || !handle) return WE_EINVAL;
  we_ctx* ctx = p->ctx;
  cudaIpcMemHandle_t h[2];
  PCK(cudaIpcGetMemHandle(&h[0], p->region), "cudaIpcGetMemHandle");
  PCK(cudaIpcGetMemHandle(&h[1], p->sync), "cudaIpcGetMemHandle");
  static_assert(sizeof(h) <= WE_PEER_HANDLE_BYTES, "handle blob");
  memset(handle, 0, WE_PEER_HANDLE_BYTES);
  memcpy(handle, h, sizeof(h));
  return WE_OK;
}

int we_peer_open(we_peer* p, const void* handles) {
  if (!p || !handles) return WE_EINVAL;
  we_ctx* ctx = p->ctx;
  unsigned char own[WE_PEER_HANDLE_BYTES];
  int rc = we_peer_export(p, own);
  if (rc != WE_OK) return rc;
  for (int r = 0; r < p->world; r++) {
    const unsigned char* h = static_cast<const unsigned char*>(handles) + (size_t)r * WE_PEER_HANDLE_BYTES;
    if (r == p->rank || memcmp(h, own, WE_PEER_HANDLE_BYTES) == 0) {  // this rank's own memory
      p->base[r] = p->region;
      p->flags[r] = p->sync;
      continue;
    }
    cudaIpcMemHandle_t m[2];
    memcpy(m, h, sizeof(m));
    void *region = nullptr, *sync = nullptr;
    PCK(cudaIpcOpenMemHandle(&region, m[0], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle (region)");
    p->opened.push_back(region);
    PCK(cudaIpcOpenMemHandle(&sync, m[1], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle (flags)");
    p->opened.push_back(sync);
    p->base[r] = static_cast<char*>(region);
    p->flags[r] = static_cast<uint32_t*>(sync);
  }
  return WE_OK;
}

void* we_peer_region(const we_peer* p) { return p ? p->region : nullptr; }
void* we_peer_remote(const we_peer* p, int32_t rank) {
  return p && rank >= 0 && rank < p->world ? p->base[rank] : nullptr;
}

int we_peer_exchange(we_ctx* ctx, we_peer* p, const we_peer_copy* copies, int32_t ncopies, uint64_t timeout_ns) {
  if (!ctx || !p || (ncopies > 0 && !copies)) return WE_EINVAL;
  if (ncopies < 0 || ncopies > MAXC) return we_ctx_fail(ctx, WE_EINVAL, "an exchange takes 0 to 4 copies");
  for (int r = 0; r < p->world; r++)
    if (!p->base[r]) return we_ctx_fail(ctx, WE_EINVAL, "the peer group is not open (we_peer_open)");
  ExchangeArgs a{};
  a.first[0] = 0;
  for (int c = 0; c < ncopies; c++) {
    const we_peer_copy& x = copies[c];
    const bool aligned = ((uintptr_t)x.src % 16 == 0) && x.chunk_bytes % 16 == 0 && x.src_row_stride % 16 == 0 &&
                         x.src_peer_stride % 16 == 0 && x.dst_offset % 16 == 0 && x.dst_row_stride % 16 == 0 &&
                         x.dst_rank_stride % 16 == 0;
    if (!aligned) return we_ctx_fail(ctx, WE_EINVAL, "peer copies need 16-byte aligned sources, chunks and strides");
    if (x.rows < 0 || x.chunk_bytes < 0) return we_ctx_fail(ctx, WE_EINVAL, "negative peer copy size");
    // the last byte written in any region stays inside it
    if (x.rows > 0 && x.chunk_bytes > 0) {
      const int64_t last = x.dst_offset + (int64_t)(p->world - 1) * x.dst_rank_stride + (x.rows - 1) * x.dst_row_stride +
                           x.chunk_bytes;
      if (x.dst_offset < 0 || x.dst_rank_stride < 0 || x.dst_row_stride < 0 || last > (int64_t)p->bytes)
        return we_ctx_fail(ctx, WE_EINVAL, "peer copy runs past the exchange region");
    }
    a.c[c] = CopyArgs{static_cast<const char*>(x.src), x.rows, x.chunk_bytes / 16, x.src_row_stride, x.src_peer_stride,
                      x.dst_offset, x.dst_row_stride, x.dst_rank_stride};
    a.first[c + 1] = a.first[c] + (int64_t)p->world * x.rows;
  }
  a.ncopies = ncopies;
  for (int c = ncopies; c < MAXC; c++) a.first[c + 1] = a.first[c];
  for (int r = 0; r < p->world; r++) {
    a.base[r] = p->base[r];
    a.flags[r] = p->flags[r];
  }
  a.local_sync = p->sync;
  a.err = we_ctx_dev_err(ctx);
  a.rank = p->rank;
  a.world = p->world;
  a.timeout_ns = timeout_ns ? timeout_ns : 2000000000ull;
  int sms = we_num_sms(ctx);
  const int64_t chunks = a.first[ncopies];
  int64_t grid = (chunks + 7) / 8;
  if (grid > (int64_t)sms * 4) grid = (int64_t)sms * 4;
  if (grid < 1) grid = 1;
  peer_exchange_kernel<<<(unsigned)grid, 256, 0, we_ctx_stream(ctx)>>>(a);
  PCK(cudaGetLastError(), "peer exchange launch");
  we_ctx_count_launch(ctx);
  return WE_OK;
}

int we_peer_destroy(we_peer* p) {
  if (!p) return WE_OK;
  cudaStreamSynchronize(we_ctx_stream(p->ctx));
  for (void* m : p->opened) cudaIpcCloseMemHandle(m);
  cudaFree(p->region);
  cudaFree(p->sync);
  delete p;
  return WE_OK;
}
