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

// delta[b,h,t] = sum_c dO[t, h*64+c] * O[t, h*64+c]; eight threads per
// (token, head), 16-byte loads. neg_lse_log2[b,h,t] = -lse[b,h,t] * log2(e).
__global__ void attn_delta_kernel(const __half* __restrict__ out, const __half* __restrict__ dout,
                                  const float* __restrict__ lse, float* __restrict__ delta,
                                  float* __restrict__ neg_lse_log2, int B, int T, int H) {
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t item = gid >> 3;  // (token, head)
  const int sub = threadIdx.x & 7;
  const int64_t total = (int64_t)B * T * H;
  float s = 0.f;
  if (item < total) {
    const int h = (int)(item % H);
    const int64_t tok = item / H;
    const int d = H * D;
    const int64_t off = tok * d + h * D + sub * 8;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(out + off));
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(dout + off));
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 af = __half22float2(ah[j]), gf = __half22float2(gh[j]);
      s += af.x * gf.x + af.y * gf.y;
    }
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  if (item < total && sub == 0) {
    const int h = (int)(item % H);
    const int64_t tok = item / H;
    const int b = (int)(tok / T), t = (int)(tok % T);
    const int64_t i = ((int64_t)b * H + h) * T + t;
    delta[i] = s;
    neg_lse_log2[i] = -lse[i] * 1.4426950408889634f;
  }
}

void launch_delta(const __half* out, const __half* dout, const float* lse, float* delta, float* neg_lse_log2, int B,
                  int T, int H, cudaStream_t s) {
  const int64_t threads = (int64_t)B * T * H * 8;
  attn_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(out, dout, lse, delta, neg_lse_log2, B, T, H);
}

}  // namespace attn
}  // namespace jx
