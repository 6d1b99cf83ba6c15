// Single-token causal attention against a KV cache (incremental decoding).
//
// The reference generates by re-running the whole context for every new token
// (Midstream-LLM src/jishui/generate_torch.py:279-285, model(tokens)[0, -1]),
// i.e. SDPA of the last query over all keys (model_torch.py:48). Here the keys
// and values of earlier positions are kept in a cache [max_len, H*64] per layer,
// and the new query attends to positions 0 .. len-1, the last of which (the new
// token) is read from the fresh q/k/v projection row and appended to the cache.
//
// Split over keys: CTA (s, h, b) scores keys [s*128, min(len, (s+1)*128)) of head
// h of sequence b with one key per thread (its 64-dim dot product in fp32),
// computes the chunk's max m, sum l = sum exp(score - m) and o = sum exp(..) v
// (each warp accumulates 32 keys' values, four keys per 16-byte step), and writes
// (m, l, o[64]) to a workspace; a second kernel merges the chunks. Memory-bound
// on the cache: 256 B per key and head.
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace dec {

constexpr int D = 64;
constexpr int kChunk = 128;
constexpr int kThreads = 128;
constexpr int kPartFloats = 2 + D;  // m, l, o[64]

__global__ void __launch_bounds__(kThreads) attn_decode_part_kernel(
    const __half* __restrict__ qkv, int64_t ld_qkv, __half* __restrict__ kcache, __half* __restrict__ vcache,
    int64_t ld_cache, int64_t cache_batch_stride, int len, const int* __restrict__ len_dev, int H,
    float scale_log2, float* __restrict__ part, int nsplit) {
  __shared__ float sq[D];
  __shared__ float sp[kChunk];
  __shared__ float sred[kThreads / 32];
  __shared__ float so[kThreads / 32][D];
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (len_dev) len = *len_dev;  // graph replays: the length lives in device memory
  if (s * kChunk >= len) {      // a chunk past the current length (fixed grid of a replayed graph)
    float* dst = part + (((int64_t)b * H + h) * nsplit + s) * kPartFloats;
    if (tid < kPartFloats) dst[tid] = tid == 0 ? -INFINITY : 0.f;
    return;
  }
  const int d = H * D;
  const __half* qrow = qkv + (int64_t)b * ld_qkv;  // this sequence's new q | k | v row
  __half* kc = kcache + (int64_t)b * cache_batch_stride + h * D;
  __half* vc = vcache + (int64_t)b * cache_batch_stride + h * D;
  if (tid < D) sq[tid] = __half2float(qrow[h * D + tid]);
  const int k0 = s * kChunk, k1 = min(len, k0 + kChunk);
  // The last chunk holds the new token: append its key / value to the cache.
  if (k1 == len && tid < D) {
    kc[(int64_t)(len - 1) * ld_cache + tid] = qrow[d + h * D + tid];
    vc[(int64_t)(len - 1) * ld_cache + tid] = qrow[2 * d + h * D + tid];
  }
  __syncthreads();
  // Scores: one key per thread (log2 domain).
  const int key = k0 + tid;
  float sc = -INFINITY;
  if (key < k1) {
    const __half* kr = (key == len - 1) ? qrow + d + h * D : kc + (int64_t)key * ld_cache;
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(kr + c * 8);
      const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(hp[j]);
        acc = fmaf(f.x, sq[c * 8 + 2 * j], acc);
        acc = fmaf(f.y, sq[c * 8 + 2 * j + 1], acc);
      }
    }
    sc = acc * scale_log2;
  }
  // Chunk max.
  float m = warp_max(sc);
  if (lane == 0) sred[warp] = m;
  __syncthreads();
  m = sred[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, sred[w]);
  const float p = (key < k1) ? exp2f(sc - m) : 0.f;
  sp[tid] = p;
  float l = warp_sum(p);
  __syncthreads();  // sred reuse and sp visible
  if (lane == 0) sred[warp] = l;
  // o = sum p_k v_k: warp w takes keys k0 + w*32 .. +32, four keys per step: lane l reads
  // 8 dims (16 bytes) at (l & 7) * 8 of key (l >> 3); the four key groups are summed at the end.
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = 0.f;
  const int kg = lane >> 3, dd = (lane & 7) * 8;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int i = it * 4 + kg;
    const int k = k0 + warp * 32 + i;
    if (k < k1) {
      const __half* vr = (k == len - 1) ? qrow + 2 * d + h * D : vc + (int64_t)k * ld_cache;
      const uint4 u = *reinterpret_cast<const uint4*>(vr + dd);
      const __half2* hv = reinterpret_cast<const __half2*>(&u);
      const float pk = sp[warp * 32 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v = __half22float2(hv[j]);
        o[2 * j] = fmaf(pk, v.x, o[2 * j]);
        o[2 * j + 1] = fmaf(pk, v.y, o[2 * j + 1]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    o[j] += __shfl_xor_sync(0xffffffffu, o[j], 8);
    o[j] += __shfl_xor_sync(0xffffffffu, o[j], 16);
  }
  if (lane < 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) so[warp][dd + j] = o[j];
  __syncthreads();
  float* dst = part + (((int64_t)b * H + h) * nsplit + s) * kPartFloats;
  if (tid < D) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) acc += so[w][tid];
    dst[2 + tid] = acc;
  }
  if (tid == 0) {
    float lt = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) lt += sred[w];
    dst[0] = m;
    dst[1] = lt;
  }
}

// out[b][h*64 + c] = f16(sum_s o_s[c] 2^(m_s - M) / sum_s l_s 2^(m_s - M)).
__global__ void attn_decode_combine_kernel(const float* __restrict__ part, int nsplit, int H, __half* __restrict__ out,
                                           int64_t ld_out) {
  const int h = blockIdx.x, b = blockIdx.y, c = threadIdx.x;
  const float* pp = part + ((int64_t)b * H + h) * nsplit * kPartFloats;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pp[s * kPartFloats]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    if (pp[s * kPartFloats + 1] == 0.f) continue;  // empty chunk
    const float w = exp2f(pp[s * kPartFloats] - M);
    l += pp[s * kPartFloats + 1] * w;
    o += pp[s * kPartFloats + 2 + c] * w;
  }
  out[(int64_t)b * ld_out + h * D + c] = __float2half_rn(o / l);
}

}  // namespace dec
}  // namespace jx

using namespace jx;

extern "C" int64_t jx_attn_decode_workspace_bytes(int B, int H, int max_len) {
  const int64_t nsplit = (max_len + dec::kChunk - 1) / dec::kChunk;
  return (int64_t)B * H * nsplit * dec::kPartFloats * (int64_t)sizeof(float);
}

extern "C" int jx_attn_decode(const void* qkv, int64_t ld_qkv, void* kcache, void* vcache, int64_t ld_cache,
                              int64_t cache_batch_stride, int B, int len, const int* len_dev, int H, int Dh,
                              float scale, void* workspace, void* out, int64_t ld_out, jx_stream_t stream) {
  JX_CHECK_ARG(qkv && kcache && vcache && workspace && out, "jx_attn_decode: NULL argument");
  JX_CHECK_ARG(Dh == 64, "jx_attn_decode: head_dim must be 64 (got %d)", Dh);
  JX_CHECK_ARG(B > 0 && B <= 65535 && H > 0 && H <= 65535 && len > 0, "jx_attn_decode: bad shape");
  // With len_dev the length is read on the device and `len` is its upper bound (the grid size).
  JX_CHECK_ARG(aligned16(qkv) && aligned16(kcache) && aligned16(vcache) && ld_qkv % 8 == 0 && ld_cache % 8 == 0 &&
                   cache_batch_stride % 8 == 0 && aligned16(workspace),
               "jx_attn_decode: rows must be 16-byte aligned");
  const int nsplit = (len + dec::kChunk - 1) / dec::kChunk;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dec::attn_decode_part_kernel<<<dim3(nsplit, H, B), dec::kThreads, 0, s>>>(
      static_cast<const __half*>(qkv), ld_qkv, static_cast<__half*>(kcache), static_cast<__half*>(vcache), ld_cache,
      cache_batch_stride, len, len_dev, H, scale * 1.4426950408889634f, static_cast<float*>(workspace), nsplit);
  JX_CHECK_LAUNCH("jx_attn_decode");
  dec::attn_decode_combine_kernel<<<dim3(H, B), dec::D, 0, s>>>(static_cast<const float*>(workspace), nsplit, H,
                                                                 static_cast<__half*>(out), ld_out);
  JX_CHECK_LAUNCH("jx_attn_decode: combine");
  return JX_OK;
}
