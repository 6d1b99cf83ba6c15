// Host-only helpers shared across translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace jx {

// Device address of this device's status word (kernels write error codes there).
int* status_ptr();

// Status codes written by kernels whose bounded waits expired.
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusGemmProducerWait = 101,
  kStatusGemmMmaWait = 102,
  kStatusGemmEpilogueWait = 103,
  kStatusEmbedBadId = 201,
};

// Builds a 2-D fp16 TMA descriptor with 128-byte swizzle.
//   inner: elements along the contiguous dimension, outer: rows,
//   ld: elements between consecutive rows, box: {box_inner, box_outer}.
bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer);

// The same for fp32 tensors (box_inner * 4 bytes <= swizzle_bytes; 128- or 64-byte swizzle).
bool make_tmap_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128);

}  // namespace jx
