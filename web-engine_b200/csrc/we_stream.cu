// Layer streaming: pinned host memory -> HBM on a side stream, double- (or N-) buffered against compute.
//
// The reference loads every block's weights once and keeps them on the GPU (src/model/weights.ts:94-131,
// a per-block onSubmittedWorkDone bounding host RAM). On B200 the weights of a 12B model also fit in HBM,
// but a batch of images can be served with only a few layers resident: layer l is copied into slot
// l % slots by cudaMemcpyAsync on the streamer's copy stream while the context's stream computes on the
// layers before it. Events order the two streams: a slot is refilled only after the compute that used
// its previous layer has run (`freed`), and compute on a layer waits only for that layer's copy (`ready`).
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

// defined in we_api.cu
int we_ctx_fail(we_ctx* ctx, int code, const std::string& msg);
cudaStream_t we_ctx_stream(we_ctx* ctx);

struct we_streamer {
  we_ctx* ctx = nullptr;
  cudaStream_t copy = nullptr;
  std::vector<const void*> host;
  std::vector<size_t> bytes;
  std::vector<void*> slot_mem;
  std::vector<cudaEvent_t> ready, freed;
  std::vector<int> slot_layer;   // layer loaded (or loading) in each slot, -1 = none
  std::vector<bool> slot_busy;   // acquired and not released yet
  std::vector<bool> freed_valid; // `freed` has been recorded at least once
  std::vector<void*> registered; // host ranges this streamer page-locked
  uint64_t copies = 0, bytes_copied = 0;
};

namespace {

int sfail(we_streamer* s, int code, const std::string& msg) { return we_ctx_fail(s ? s->ctx : nullptr, code, msg); }

#define SCK(call, what)                                                                             \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) return sfail(s, WE_ECUDA, std::string(what) + ": " + cudaGetErrorString(e_)); \
  } while (0)

int load(we_streamer* s, int layer, int slot) {
  if (s->freed_valid[slot]) SCK(cudaStreamWaitEvent(s->copy, s->freed[slot], 0), "wait for the slot's last use");
  SCK(cudaMemcpyAsync(s->slot_mem[slot], s->host[layer], s->bytes[layer], cudaMemcpyHostToDevice, s->copy),
      "layer copy");
  SCK(cudaEventRecord(s->ready[slot], s->copy), "record layer ready");
  s->slot_layer[slot] = layer;
  s->copies++;
  s->bytes_copied += s->bytes[layer];
  return WE_OK;
}

}  // namespace

extern "C" {

int we_streamer_create(we_ctx* ctx, const void* const* host, const size_t* bytes, int32_t layers, int32_t slots,
                       uint32_t flags, we_streamer** out) {
  if (!ctx || !host || !bytes || !out) return WE_EINVAL;
  *out = nullptr;
  if (layers < 1 || slots < 1) return we_ctx_fail(ctx, WE_EINVAL, "a streamer needs at least one layer and one slot");
  if (slots > layers) slots = layers;
  we_streamer* s = new we_streamer();
  s->ctx = ctx;
  size_t max_bytes = 0;
  for (int l = 0; l < layers; l++) {
    if (!host[l] || !bytes[l]) {
      delete s;
      return we_ctx_fail(ctx, WE_EINVAL, "layer " + std::to_string(l) + " has no host bytes");
    }
    s->host.push_back(host[l]);
    s->bytes.push_back(bytes[l]);
    if (bytes[l] > max_bytes) max_bytes = bytes[l];
    if (!(flags & WE_STREAM_HOST_PINNED)) {
      cudaError_t e = cudaHostRegister(const_cast<void*>(host[l]), bytes[l], cudaHostRegisterDefault);
      if (e == cudaSuccess) s->registered.push_back(const_cast<void*>(host[l]));
      else cudaGetLastError();  // already page-locked (or not lockable): copies still work, just staged
    }
  }
  cudaError_t e = cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking);
  for (int i = 0; i < slots && e == cudaSuccess; i++) {
    void* p = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    e = cudaMalloc(&p, (max_bytes + 255) / 256 * 256);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
    s->slot_mem.push_back(p);
    s->ready.push_back(a);
    s->freed.push_back(b);
    s->slot_layer.push_back(-1);
    s->slot_busy.push_back(false);
    s->freed_valid.push_back(false);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    we_streamer_destroy(s);
    return we_ctx_fail(ctx, WE_ENOMEM, std::string("streamer set-up failed: ") + cudaGetErrorString(e));
  }
  *out = s;
  return WE_OK;
}

int we_streamer_acquire(we_streamer* s, int32_t layer, void** dev) {
  if (!s || !dev) return WE_EINVAL;
  const int layers = (int)s->host.size(), slots = (int)s->slot_mem.size();
  if (layer < 0 || layer >= layers) return sfail(s, WE_EINVAL, "layer " + std::to_string(layer) + " out of range");
  const int slot = layer % slots;
  if (s->slot_busy[slot] && s->slot_layer[slot] != layer)
    return sfail(s, WE_EINVAL, "slot of layer " + std::to_string(layer) + " still holds layer " +
                                   std::to_string(s->slot_layer[slot]) + ": release it first");
  if (s->slot_layer[slot] != layer) {
    int rc = load(s, layer, slot);
    if (rc != WE_OK) return rc;
  }
  SCK(cudaStreamWaitEvent(we_ctx_stream(s->ctx), s->ready[slot], 0), "wait for the layer");
  s->slot_busy[slot] = true;
  // prefetch the layers after this one (wrapping to the next pass) into slots nobody holds
  for (int j = 1; j < slots; j++) {
    const int next = (layer + j) % layers, ns = next % slots;
    if (ns == slot || s->slot_busy[ns] || s->slot_layer[ns] == next) continue;
    int rc = load(s, next, ns);
    if (rc != WE_OK) return rc;
  }
  *dev = s->slot_mem[slot];
  return WE_OK;
}

int we_streamer_release(we_streamer* s, int32_t layer) {
  if (!s) return WE_EINVAL;
  const int slots = (int)s->slot_mem.size();
  if (layer < 0 || layer >= (int)s->host.size()) return sfail(s, WE_EINVAL, "layer out of range");
  const int slot = layer % slots;
  if (!s->slot_busy[slot] || s->slot_layer[slot] != layer)
    return sfail(s, WE_EINVAL, "layer " + std::to_string(layer) + " is not acquired");
  SCK(cudaEventRecord(s->freed[slot], we_ctx_stream(s->ctx)), "record slot free");
  s->freed_valid[slot] = true;
  s->slot_busy[slot] = false;
  return WE_OK;
}

int we_streamer_stats(const we_streamer* s, uint64_t* copies, uint64_t* bytes_copied) {
  if (!s) return WE_EINVAL;
  if (copies) *copies = s->copies;
  if (bytes_copied) *bytes_copied = s->bytes_copied;
  return WE_OK;
}

int we_streamer_destroy(we_streamer* s) {
  if (!s) return WE_OK;
  if (s->copy) cudaStreamSynchronize(s->copy);
  cudaStreamSynchronize(we_ctx_stream(s->ctx));
  for (size_t i = 0; i < s->slot_mem.size(); i++) {
    if (s->slot_mem[i]) cudaFree(s->slot_mem[i]);
    if (s->ready[i]) cudaEventDestroy(s->ready[i]);
    if (s->freed[i]) cudaEventDestroy(s->freed[i]);
  }
  for (void* p : s->registered) cudaHostUnregister(p);
  if (s->copy) cudaStreamDestroy(s->copy);
  delete s;
  return WE_OK;
}

}  // extern "C"
