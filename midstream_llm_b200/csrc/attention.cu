// Row statistics for the causal attention backward (the forward and backward
// themselves are the tcgen05 kernels in attention_tc.cu).
//
// Reference: Midstream-LLM src/jishui/model_torch.py:48,
// F.scaled_dot_product_attention(q, k, v, is_causal=True) on fp16 q/k/v under
// autocast. Its backward recomputes the probabilities from the saved
// log-sum-exp (the flash formulation) and needs, per query row,
//   Delta = sum_c dO[c] * O[c]      (the softmax-gradient correction term).
// This kernel also writes -LSE * log2(e) beside it, the per-query offset of the
// base-2 exponent P = 2^(S * scale * log2(e) - LSE * log2(e)), so the backward's
// softmax warps read it instead of rescaling LSE for every key.
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace attn {

constexpr int D = 64;

// delta[b,h,t] = sum_c dO[t, h*64+c] * O[t, h*64+c]; neg_lse_log2[b,h,t] = -lse[b,h,t] * log2(e).
// One thread per (token, head); the 32 lanes of a warp take 32 consecutive tokens of one head, so the
// [B, H, T] outputs (and the lse reads) are coalesced. Each thread reads its head's 128 bytes of O and
// dO as eight 16-byte loads through the read-only cache: the first load of a row brings its line,
// the rest hit it.
__global__ void attn_delta_kernel(const __half* __restrict__ out, const __half* __restrict__ dout,
                                  const float* __restrict__ lse, float* __restrict__ delta,
                                  float* __restrict__ neg_lse_log2, int B, int T, int H) {
  const int warps_per_head = (T + 31) / 32;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t bh = warp / warps_per_head;  // (batch, head)
  if (bh >= (int64_t)B * H) return;
  const int t = (int)(warp - bh * warps_per_head) * 32 + lane;
  if (t >= T) return;
  const int b = (int)(bh / H), h = (int)(bh - (int64_t)b * H);
  const int d = H * D;
  const int64_t off = ((int64_t)b * T + t) * d + h * D;
  uint4 a[8], g[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    a[k] = __ldg(reinterpret_cast<const uint4*>(out + off) + k);
    g[k] = __ldg(reinterpret_cast<const uint4*>(dout + off) + k);
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const __half2* ah = reinterpret_cast<const __half2*>(&a[k]);
    const __half2* gh = reinterpret_cast<const __half2*>(&g[k]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 af = __half22float2(ah[j]), gf = __half22float2(gh[j]);
      s += af.x * gf.x + af.y * gf.y;
    }
  }
  const int64_t i = bh * T + t;
  delta[i] = s;
  neg_lse_log2[i] = -lse[i] * 1.4426950408889634f;
}

void launch_delta(const __half* out, const __half* dout, const float* lse, float* delta, float* neg_lse_log2, int B,
                  int T, int H, cudaStream_t s) {
  const int64_t threads = (int64_t)B * H * ((T + 31) / 32) * 32;
  attn_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(out, dout, lse, delta, neg_lse_log2, B, T, H);
}

}  // namespace attn
}  // namespace jx
