// Causal flash attention backward, head_dim 64 (the forward is in attention_tc.cu).
//
// Reference: Midstream-LLM src/jishui/model_torch.py:48,
// F.scaled_dot_product_attention(q, k, v, is_causal=True) with scale
// 1/sqrt(head_dim) on fp16 q/k/v under autocast; the backward recomputes the
// probabilities from the saved log-sum-exp (the flash formulation), so only
// O and LSE are kept between forward and backward.
//
// Q/K/V are read in place from the fused projection output qkv [B*T, 3*H*64]
// (row = token, q|k|v column blocks, head h at column h*64 of each block);
// O is written token-major [B*T, H*64], which is what the output projection
// consumes. No transposes, no [B,H,T,T] buffer.
//
// The backward uses warp-level mma.sync (m16n8k16, fp16 in / fp32 acc) with
// K/V tiles staged through XOR-swizzled shared memory by cp.async.
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace attn {

constexpr int D = 64;

__device__ __forceinline__ int swz(int r, int chunk) { return r * 64 + ((chunk ^ (r & 7)) << 3); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load a [rows x 64] fp16 tile (row stride ld elements) into swizzled smem.
template <int ROWS, int NT>
__device__ __forceinline__ void load_tile(__half* s, const __half* g, int64_t ld, int tid) {
#pragma unroll
  for (int i = tid; i < ROWS * 8; i += NT) {
    const int r = i >> 3, c = i & 7;
    cp_async16(s + swz(r, c), g + (int64_t)r * ld + c * 8);
  }
}

// A-operand fragments (16 rows x 64 cols) of a swizzled tile, rows r0..r0+15.
__device__ __forceinline__ void load_afrag(uint32_t (&f)[4][4], const __half* s, int r0, int lane) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) ldsm_x4(f[ks], s + swz(r0 + (lane & 15), ks * 2 + (lane >> 4)));
}

// acc[16 x 64] += A(16 x 64, k = tile columns) * T^T where T is a 64x64 swizzled tile
// whose rows are the n index (B = rows of T, "non-transposed").
__device__ __forceinline__ void mma_abt(float (&acc)[8][4], const uint32_t (&a)[4][4], const __half* t, int lane) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm_x4(b, t + swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
      mma16816(acc[2 * np], a[ks], b[0], b[1]);
      mma16816(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// acc[16 x 64] += P(16 x 64, k = tile rows, given as C-layout fp32) * T where T is a
// 64x64 swizzled tile indexed [k][n] ("transposed" ldmatrix).
__device__ __forceinline__ void mma_pt(float (&acc)[8][4], const float (&p)[8][4], const __half* t, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_h2(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_h2(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_h2(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_h2(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int dp = 0; dp < 4; ++dp) {
      uint32_t b[4];
      ldsm_x4_t(b, t + swz(kk * 16 + (lane & 15), dp * 2 + (lane >> 4)));
      mma16816(acc[2 * dp], a, b[0], b[1]);
      mma16816(acc[2 * dp + 1], a, b[2], b[3]);
    }
  }
}

__device__ __forceinline__ void zero(float (&a)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) a[i][j] = 0.f;
}

__device__ __forceinline__ float r16(float x) { return __half2float(__float2half_rn(x)); }

// delta[b,h,t] = sum_c dO[t, h*64+c] * O[t, h*64+c]; eight threads per
// (token, head), 16-byte loads.
__global__ void attn_delta_kernel(const __half* __restrict__ out, const __half* __restrict__ dout,
                                  float* __restrict__ delta, int B, int T, int H) {
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
    delta[((int64_t)b * H + h) * T + t] = s;
  }
}

void launch_delta(const __half* out, const __half* dout, float* delta, int B, int T, int H, cudaStream_t s) {
  const int64_t threads = (int64_t)B * T * H * 8;
  attn_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(out, dout, delta, B, T, H);
}

}  // namespace attn
}  // namespace jx

