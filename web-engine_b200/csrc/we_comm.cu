// Collectives behind the C ABI: NCCL communicators over NVLink / NVSwitch, one per context (one process per GPU).
//
// The reference runs on one GPU and has no collective layer; this file gives the multi-GPU paths (tensor-parallel
// linears, sequence-parallel attention, timing reductions) a communicator that the host reaches through the same
// C ABI as every op, with no framework in between. NCCL is loaded at run time (dlopen of libnccl.so.2): the
// library itself loads on hosts without NCCL, and a process that already holds an NCCL library (a framework's)
// shares it. The communicator is non-blocking (ncclConfig_t.blocking = 0): every call returns once its work is
// queued on the context's stream, and a host-side deadline turns a rank that never joins, or a collective that
// never completes, into WE_ETIMEOUT after aborting the communicator, instead of a hang.
#include <dlfcn.h>
#include <stdlib.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <chrono>
#include <string>
#include <thread>

#include "common.cuh"
#include "kernels.h"

// defined in we_api.cu
int we_ctx_fail(we_ctx* ctx, int code, const std::string& msg);
cudaStream_t we_ctx_stream(we_ctx* ctx);
int we_ctx_device(we_ctx* ctx);

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    // WE_NCCL_LIBRARY names the NCCL to use (a path); otherwise the loader's search for libnccl.so.2. A process
    // holds one library of that soname, so it must be the newest NCCL that anything in the process needs.
    void* h = nullptr;
    if (const char* path = getenv("WE_NCCL_LIBRARY")) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      a.why = std::string("NCCL is not available (dlopen libnccl.so.2: ") + dlerror() + ")";
      return a;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) all = false;
    };
    sym(a.get_unique_id, "ncclGetUniqueId");
    sym(a.init_rank_config, "ncclCommInitRankConfig");
    sym(a.destroy, "ncclCommDestroy");
    sym(a.abort, "ncclCommAbort");
    sym(a.async_error, "ncclCommGetAsyncError");
    sym(a.all_gather, "ncclAllGather");
    sym(a.reduce_scatter, "ncclReduceScatter");
    sym(a.all_reduce, "ncclAllReduce");
    sym(a.send, "ncclSend");
    sym(a.recv, "ncclRecv");
    sym(a.group_start, "ncclGroupStart");
    sym(a.group_end, "ncclGroupEnd");
    sym(a.error_string, "ncclGetErrorString");
    a.ok = all;
    if (!all) a.why = "the NCCL library lacks an entry point this build needs";
    return a;
  }();
  return api;
}

bool dtype_of(int32_t dt, ncclDataType_t* out, size_t* esz) {
  switch (dt) {
    case WE_F32: *out = ncclFloat32; *esz = 4; return true;
    case WE_BF16: *out = ncclBfloat16; *esz = 2; return true;
    case WE_F16: *out = ncclFloat16; *esz = 2; return true;
    case WE_FP8: *out = ncclUint8; *esz = 1; return true;  // bytes (all-gather / all-to-all only)
    default: return false;
  }
}

}  // namespace

struct we_comm {
  we_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, nranks = 1;
  uint64_t timeout_ms = 60000;
  bool aborted = false;
  std::string err;
};

namespace {

int comm_fail(we_comm* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

// Polls the communicator until its last call is no longer in progress; aborts it when the deadline passes.
int settle(we_comm* c, ncclResult_t r, const char* what) {
  const NcclApi& a = nccl();
  if (r != ncclSuccess && r != ncclInProgress)
    return comm_fail(c, WE_ENCCL, std::string(what) + ": " + a.error_string(r));
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = a.async_error(c->comm, &st);
    if (q != ncclSuccess) return comm_fail(c, WE_ENCCL, std::string(what) + ": " + a.error_string(q));
    if (st == ncclSuccess) return WE_OK;
    if (st != ncclInProgress) {
      a.abort(c->comm);
      c->comm = nullptr;
      c->aborted = true;
      return comm_fail(c, WE_ENCCL, std::string(what) + ": " + a.error_string(st));
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if ((uint64_t)ms > c->timeout_ms) {
      a.abort(c->comm);
      c->comm = nullptr;
      c->aborted = true;
      return comm_fail(c, WE_ETIMEOUT, std::string(what) + ": no progress within the timeout; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int usable(we_comm* c) {
  if (!c) return WE_EINVAL;
  if (c->aborted || !c->comm) return comm_fail(c, WE_ENCCL, "the communicator was aborted");
  return WE_OK;
}

}  // namespace

extern "C" int we_comm_unique_id(void* id) {
  if (!id) return WE_EINVAL;
  const NcclApi& a = nccl();
  if (!a.ok) return WE_EUNSUPPORTED;
  ncclUniqueId u;
  if (a.get_unique_id(&u) != ncclSuccess) return WE_ENCCL;
  memcpy(id, &u, sizeof(u));
  return WE_OK;
}

extern "C" int we_comm_init(we_ctx* ctx, int32_t nranks, int32_t rank, const void* id, uint64_t timeout_ms,
                            we_comm** out) {
  if (!ctx || !id || !out || nranks < 1 || rank < 0 || rank >= nranks) return WE_EINVAL;
  *out = nullptr;
  const NcclApi& a = nccl();
  if (!a.ok) return WE_EUNSUPPORTED;
  we_comm* c = new we_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->nranks = nranks;
  c->timeout_ms = timeout_ms ? timeout_ms : 60000;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(we_ctx_device(ctx));
  ncclResult_t r = a.init_rank_config(&c->comm, nranks, u, rank, &cfg);
  int rc = settle(c, r, "ncclCommInitRankConfig");
  cudaSetDevice(dev);
  if (rc != WE_OK) {
    std::string msg = c->err;
    if (c->comm) a.abort(c->comm);
    delete c;
    return we_ctx_fail(ctx, rc, msg);
  }
  *out = c;
  return WE_OK;
}

extern "C" int we_comm_destroy(we_comm* c) {
  if (!c) return WE_OK;
  const NcclApi& a = nccl();
  if (c->comm && a.ok) a.destroy(c->comm);
  delete c;
  return WE_OK;
}

extern "C" int we_comm_abort(we_comm* c) {
  if (!c) return WE_EINVAL;
  const NcclApi& a = nccl();
  if (c->comm && a.ok) a.abort(c->comm);
  c->comm = nullptr;
  c->aborted = true;
  return WE_OK;
}

extern "C" const char* we_comm_last_error(const we_comm* c) { return c ? c->err.c_str() : "no communicator"; }

extern "C" int we_comm_rank(const we_comm* c, int32_t* rank, int32_t* nranks) {
  if (!c) return WE_EINVAL;
  if (rank) *rank = c->rank;
  if (nranks) *nranks = c->nranks;
  return WE_OK;
}

extern "C" int we_all_gather(we_comm* c, const void* x, void* y, size_t bytes) {
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  if ((!x || !y) && bytes) return comm_fail(c, WE_EINVAL, "we_all_gather: missing buffer");
  return settle(c, nccl().all_gather(x, y, bytes, ncclUint8, c->comm, we_ctx_stream(c->ctx)),
                "ncclAllGather");
}

extern "C" int we_reduce_scatter(we_comm* c, const void* x, void* y, size_t count, int32_t dtype) {
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  ncclDataType_t t;
  size_t esz;
  if (!dtype_of(dtype, &t, &esz) || dtype == WE_FP8) return comm_fail(c, WE_EINVAL, "reduce-scatter takes f32, bf16 or f16");
  return settle(c, nccl().reduce_scatter(x, y, count, t, ncclSum, c->comm, we_ctx_stream(c->ctx)),
                "ncclReduceScatter");
}

extern "C" int we_all_reduce(we_comm* c, const void* x, void* y, size_t count, int32_t dtype, int32_t op) {
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  ncclDataType_t t;
  size_t esz;
  if (!dtype_of(dtype, &t, &esz) || dtype == WE_FP8) return comm_fail(c, WE_EINVAL, "all-reduce takes f32, bf16 or f16");
  if (op != WE_REDUCE_SUM && op != WE_REDUCE_MAX) return comm_fail(c, WE_EINVAL, "all-reduce op is sum or max");
  return settle(c, nccl().all_reduce(x, y, count, t, op == WE_REDUCE_MAX ? ncclMax : ncclSum, c->comm,
                                     we_ctx_stream(c->ctx)),
                "ncclAllReduce");
}

extern "C" int we_all_to_all(we_comm* c, const void* x, void* y, size_t bytes_per_rank) {
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  const NcclApi& a = nccl();
  cudaStream_t st = we_ctx_stream(c->ctx);
  a.group_start();
  ncclResult_t r = ncclSuccess;
  for (int p = 0; p < c->nranks && r == ncclSuccess; p++) {
    r = a.send(static_cast<const char*>(x) + p * bytes_per_rank, bytes_per_rank, ncclUint8, p, c->comm, st);
    if (r == ncclSuccess || r == ncclInProgress)
      r = a.recv(static_cast<char*>(y) + p * bytes_per_rank, bytes_per_rank, ncclUint8, p, c->comm, st);
    if (r == ncclInProgress) r = ncclSuccess;
  }
  ncclResult_t e = a.group_end();
  if (r != ncclSuccess) return settle(c, r, "ncclSend/ncclRecv");
  return settle(c, e, "ncclGroupEnd (all-to-all)");
}

extern "C" int we_comm_barrier(we_comm* c) {
  // an all-reduce of one word on the context's stream, then a wait for the stream bounded by the timeout
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  void* word = nullptr;
  if ((rc = we_buffer(c->ctx, 4, nullptr, &word)) != WE_OK) return comm_fail(c, rc, "barrier scratch");
  rc = we_all_reduce(c, word, word, 1, WE_F32, WE_REDUCE_SUM);
  if (rc == WE_OK) rc = we_comm_wait(c);
  we_free(c->ctx, word);
  return rc;
}

extern "C" int we_comm_wait(we_comm* c) {
  // waits for the context's stream, polling the communicator for asynchronous errors, bounded by the timeout
  int rc = usable(c);
  if (rc != WE_OK) return rc;
  const NcclApi& a = nccl();
  cudaStream_t st = we_ctx_stream(c->ctx);
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return WE_OK;
    if (q != cudaErrorNotReady) return comm_fail(c, WE_ECUDA, std::string("stream: ") + cudaGetErrorString(q));
    ncclResult_t s = ncclSuccess;
    if (a.async_error(c->comm, &s) == ncclSuccess && s != ncclSuccess && s != ncclInProgress) {
      a.abort(c->comm);
      c->comm = nullptr;
      c->aborted = true;
      return comm_fail(c, WE_ENCCL, std::string("asynchronous NCCL error: ") + a.error_string(s));
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if ((uint64_t)ms > c->timeout_ms) {
      a.abort(c->comm);
      c->comm = nullptr;
      c->aborted = true;
      return comm_fail(c, WE_ETIMEOUT, "the stream did not finish within the timeout; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}
