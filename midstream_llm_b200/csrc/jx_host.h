// Host-only helpers shared across translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace jx {

// Unique id of the calling thread's current CUDA context (cuCtxGetId), or 0 if it cannot be read.
// Ids are never reused within a process, so a context torn down and created again (cudaDeviceReset)
// gets a new one.
uint64_t current_context_id();

// Device address of a file-scope __device__ variable on the current device, looked up with that device
// current and cached per device. The cache is keyed on the context id, so after a device reset (which
// reloads the module at a new address) the next call looks the address up again.
class SymbolCache {
 public:
  void* get(const void* symbol);

 private:
  struct Entry {
    void* ptr = nullptr;
    uint64_t ctx = 0;
  };
  std::mutex mu_;
  Entry entries_[64];
};

// Device address of this device's status word (kernels write error codes there).
int* status_ptr();

// Runs `fn` (returning cudaError_t) the first time it is reached on the current device: function
// attributes such as the dynamic shared-memory limit are per device. A race between two host threads
// may run it twice, which is harmless for idempotent setup.
template <typename Fn>
inline cudaError_t once_per_device(std::atomic<uint64_t>& done, Fn&& fn) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = fn();
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Status codes written by kernels whose bounded waits expired.
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusGemmProducerWait = 101,
  kStatusGemmMmaWait = 102,
  kStatusGemmEpilogueWait = 103,
  kStatusEmbedBadId = 201,
  kStatusCeBadTarget = 202,
  kStatusNormWait = 501,  // the staged RMSNorm backward's row-copy wait
};

// Builds a 2-D fp16 TMA descriptor with 128-byte (or 64-byte) swizzle.
//   inner: elements along the contiguous dimension, outer: rows,
//   ld: elements between consecutive rows, box: {box_inner, box_outer}
//   (box_inner * 2 bytes <= swizzle_bytes).
bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128);

// The same for fp32 tensors (box_inner * 4 bytes <= swizzle_bytes; 128- or 64-byte swizzle).
bool make_tmap_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128);

}  // namespace jx
