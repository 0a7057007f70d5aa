// Block-weight prefetcher: host -> device copies of whole transformer blocks on
// a dedicated copy stream, ordered against the compute stream with events.
//
// Replaces the synchronous per-tensor `.to(device)` of the reference's
// offloader (src/krea2_svdquant/runtime/block_offload.py:56-63, 157-173).
// The caller keeps each block's weights in one pinned host arena and owns
// `num_slots` device slots; a block's upload is one cudaMemcpyAsync into a
// slot.  Per slot:
//   ready[slot]  recorded on the copy stream after the upload (and after any
//                work the caller enqueues on the copy stream, e.g. a repack)
//   free[slot]   recorded on the compute stream after the last use of the slot
// An upload into a slot waits (on the GPU) for free[slot]; compute waits (on
// the GPU, or on the host with a time limit) for ready[slot].
#include <chrono>
#include <thread>

#include "svdq_common.cuh"

struct svdq_prefetcher {
  int device = 0;
  int num_slots = 0;
  cudaStream_t copy = nullptr;
  cudaEvent_t* ready = nullptr;
  cudaEvent_t* freed = nullptr;
  bool* ready_recorded = nullptr;
  bool* free_recorded = nullptr;
};

namespace {

int slot_ok(const svdq_prefetcher* p, int slot, const char* who) {
  if (!p) return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, std::string(who) + ": prefetcher is NULL");
  if (slot < 0 || slot >= p->num_slots)
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, std::string(who) + ": slot out of range");
  return SVDQ_OK;
}

// Make the prefetcher's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  int st = SVDQ_OK;
  explicit DeviceGuard(int dev) {
    st = svdq::check_cuda(cudaGetDevice(&prev), "prefetcher: current device");
    if (!st && prev != dev) st = svdq::check_cuda(cudaSetDevice(dev), "prefetcher: set device");
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

void destroy_fields(svdq_prefetcher* p) {
  for (int i = 0; i < p->num_slots; ++i) {
    if (p->ready && p->ready[i]) cudaEventDestroy(p->ready[i]);
    if (p->freed && p->freed[i]) cudaEventDestroy(p->freed[i]);
  }
  delete[] p->ready;
  delete[] p->freed;
  delete[] p->ready_recorded;
  delete[] p->free_recorded;
  if (p->copy) cudaStreamDestroy(p->copy);
}

}  // namespace

extern "C" int svdq_prefetcher_create(int device, int num_slots, svdq_prefetcher** out) {
  using namespace svdq;
  SVDQ_REQUIRE(out, "svdq_prefetcher_create: out is NULL");
  SVDQ_REQUIRE(num_slots > 0 && num_slots <= 64, "svdq_prefetcher_create: num_slots must be in [1, 64]");
  *out = nullptr;
  DeviceGuard g(device);
  if (g.st) return g.st;
  auto* p = new svdq_prefetcher();
  p->device = device;
  p->num_slots = num_slots;
  p->ready = new cudaEvent_t[num_slots]();
  p->freed = new cudaEvent_t[num_slots]();
  p->ready_recorded = new bool[num_slots]();
  p->free_recorded = new bool[num_slots]();
  int lo = 0, hi = 0;
  int st = check_cuda(cudaDeviceGetStreamPriorityRange(&lo, &hi), "svdq_prefetcher_create: priority range");
  // the copy stream gets the lowest priority: compute work is never queued behind an upload
  if (!st) st = check_cuda(cudaStreamCreateWithPriority(&p->copy, cudaStreamNonBlocking, lo),
                           "svdq_prefetcher_create: copy stream");
  for (int i = 0; !st && i < num_slots; ++i) {
    st = check_cuda(cudaEventCreateWithFlags(&p->ready[i], cudaEventDisableTiming), "svdq_prefetcher_create: event");
    if (!st)
      st = check_cuda(cudaEventCreateWithFlags(&p->freed[i], cudaEventDisableTiming), "svdq_prefetcher_create: event");
  }
  if (st) {
    destroy_fields(p);
    delete p;
    return st;
  }
  *out = p;
  return SVDQ_OK;
}

extern "C" int svdq_prefetcher_copy_stream(svdq_prefetcher* p, cudaStream_t* out) {
  if (!p || !out) return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_prefetcher_copy_stream: NULL argument");
  *out = p->copy;
  return SVDQ_OK;
}

extern "C" int svdq_prefetch_begin(svdq_prefetcher* p, int slot, void* dev_dst, const void* host_src, size_t bytes) {
  using namespace svdq;
  int st = slot_ok(p, slot, "svdq_prefetch_begin");
  if (st) return st;
  SVDQ_REQUIRE(dev_dst && host_src, "svdq_prefetch_begin: NULL buffer");
  DeviceGuard g(p->device);
  if (g.st) return g.st;
  cudaPointerAttributes a{};
  st = check_cuda(cudaPointerGetAttributes(&a, host_src), "svdq_prefetch_begin: host pointer attributes");
  if (st) return st;
  if (a.type != cudaMemoryTypeHost)
    return set_error(SVDQ_ERR_INVALID_ARGUMENT,
                     "svdq_prefetch_begin: host_src is not pinned host memory (the copy would not be asynchronous)");
  if (p->free_recorded[slot]) {
    st = check_cuda(cudaStreamWaitEvent(p->copy, p->freed[slot], 0), "svdq_prefetch_begin: wait for slot release");
    if (st) return st;
  }
  if (bytes > 0) {
    st = check_cuda(cudaMemcpyAsync(dev_dst, host_src, bytes, cudaMemcpyHostToDevice, p->copy),
                    "svdq_prefetch_begin: upload");
    if (st) return st;
  }
  return SVDQ_OK;
}

// Marks the slot ready: everything enqueued on the copy stream so far (the upload and
// any follow-up work the caller put there) completes before ready[slot].
extern "C" int svdq_prefetch_commit(svdq_prefetcher* p, int slot) {
  using namespace svdq;
  int st = slot_ok(p, slot, "svdq_prefetch_commit");
  if (st) return st;
  DeviceGuard g(p->device);
  if (g.st) return g.st;
  st = check_cuda(cudaEventRecord(p->ready[slot], p->copy), "svdq_prefetch_commit: record");
  if (!st) p->ready_recorded[slot] = true;
  return st;
}

// Orders `compute` after ready[slot].  timeout_ms < 0: a device-side wait only (the host
// does not block).  timeout_ms >= 0: the host first polls for completion for at most
// timeout_ms and returns SVDQ_ERR_TIMEOUT if the upload has not finished by then.
extern "C" int svdq_prefetch_wait(svdq_prefetcher* p, int slot, cudaStream_t compute, int timeout_ms) {
  using namespace svdq;
  int st = slot_ok(p, slot, "svdq_prefetch_wait");
  if (st) return st;
  if (!p->ready_recorded[slot]) return set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_prefetch_wait: slot was never committed");
  DeviceGuard g(p->device);
  if (g.st) return g.st;
  if (timeout_ms >= 0) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      const cudaError_t q = cudaEventQuery(p->ready[slot]);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return check_cuda(q, "svdq_prefetch_wait: query");
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
        return set_error(SVDQ_ERR_TIMEOUT, "svdq_prefetch_wait: upload of slot " + std::to_string(slot) +
                                                " not finished within " + std::to_string(timeout_ms) + " ms");
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  return check_cuda(cudaStreamWaitEvent(compute, p->ready[slot], 0), "svdq_prefetch_wait: stream wait");
}

// Records the end of the slot's use on `compute`; the next upload into the slot waits for it.
extern "C" int svdq_prefetch_release(svdq_prefetcher* p, int slot, cudaStream_t compute) {
  using namespace svdq;
  int st = slot_ok(p, slot, "svdq_prefetch_release");
  if (st) return st;
  DeviceGuard g(p->device);
  if (g.st) return g.st;
  st = check_cuda(cudaEventRecord(p->freed[slot], compute), "svdq_prefetch_release: record");
  if (!st) p->free_recorded[slot] = true;
  return st;
}

// Waits (host, at most timeout_ms; < 0 = no limit) until every upload enqueued so far is done.
extern "C" int svdq_prefetcher_sync(svdq_prefetcher* p, int timeout_ms) {
  using namespace svdq;
  SVDQ_REQUIRE(p, "svdq_prefetcher_sync: prefetcher is NULL");
  DeviceGuard g(p->device);
  if (g.st) return g.st;
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = cudaStreamQuery(p->copy);
    if (q == cudaSuccess) return SVDQ_OK;
    if (q != cudaErrorNotReady) return check_cuda(q, "svdq_prefetcher_sync: query");
    if (timeout_ms >= 0 && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return set_error(SVDQ_ERR_TIMEOUT, "svdq_prefetcher_sync: uploads not finished within " +
                                             std::to_string(timeout_ms) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

extern "C" int svdq_prefetcher_destroy(svdq_prefetcher* p) {
  if (!p) return SVDQ_OK;
  {
    DeviceGuard g(p->device);
    if (p->copy) cudaStreamSynchronize(p->copy);
    destroy_fields(p);
  }
  delete p;
  return SVDQ_OK;
}
