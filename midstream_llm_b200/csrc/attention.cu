// Causal flash attention, head_dim 64, forward and backward.
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
// This version uses warp-level mma.sync (m16n8k16, fp16 in / fp32 acc) with
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

// ---------------------------------------------------------------------------
// Forward: one CTA per (128-query block, head, batch); 8 warps x 16 queries.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) attn_fwd_kernel(const __half* __restrict__ qkv, __half* __restrict__ out,
                                                       float* __restrict__ lse, int T, int H, float scale_log2) {
  __shared__ __align__(128) __half sQ[128 * 64];
  __shared__ __align__(128) __half sK[2][64 * 64];
  __shared__ __align__(128) __half sV[2][64 * 64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = T / 128;
  const int qb = nqb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int d = H * D;
  const int64_t ld = 3 * (int64_t)d;
  const int q0 = qb * 128;
  const __half* qbase = qkv + (int64_t)b * T * ld + h * D;
  const __half* kbase = qbase + d;
  const __half* vbase = qbase + 2 * d;

  load_tile<128, 256>(sQ, qbase + (int64_t)q0 * ld, ld, tid);
  load_tile<64, 256>(sK[0], kbase, ld, tid);
  load_tile<64, 256>(sV[0], vbase, ld, tid);
  cp_commit();

  const int nkt = (q0 + 128) / 64;
  const int row0 = q0 + warp * 16 + (lane >> 2);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[8][4];
  zero(o);
  uint32_t qf[4][4];

  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) {
      load_tile<64, 256>(sK[(kt + 1) & 1], kbase + (int64_t)(kt + 1) * 64 * ld, ld, tid);
      load_tile<64, 256>(sV[(kt + 1) & 1], vbase + (int64_t)(kt + 1) * 64 * ld, ld, tid);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kt == 0) load_afrag(qf, sQ, warp * 16, lane);
    const int buf = kt & 1;
    const int k0 = kt * 64;
    if (k0 <= q0 + warp * 16 + 15) {  // some key of this tile is visible to this warp's rows
      float s[8][4];
      zero(s);
      mma_abt(s, qf, sK[buf], lane);
      const bool diag = k0 + 63 > q0 + warp * 16;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int key = k0 + nt * 8 + (lane & 3) * 2 + j;
          float a = s[nt][j] * scale_log2, c = s[nt][2 + j] * scale_log2;
          if (diag) {
            if (key > row0) a = -INFINITY;
            if (key > row0 + 8) c = -INFINITY;
          }
          s[nt][j] = a;
          s[nt][2 + j] = c;
          mx0 = fmaxf(mx0, a);
          mx1 = fmaxf(mx1, c);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          s[nt][j] = exp2f(s[nt][j] - mn0);
          s[nt][2 + j] = exp2f(s[nt][2 + j] - mn1);
          rs0 += s[nt][j];
          rs1 += s[nt][2 + j];
        }
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        o[nt][0] *= al0;
        o[nt][1] *= al0;
        o[nt][2] *= al1;
        o[nt][3] *= al1;
      }
      mma_pt(o, s, sV[buf], lane);
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  __half* ob = out + (int64_t)b * T * d + h * D;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + (lane & 3) * 2;
    *reinterpret_cast<__half2*>(ob + (int64_t)row0 * d + c) = __floats2half2_rn(o[nt][0] * inv0, o[nt][1] * inv0);
    *reinterpret_cast<__half2*>(ob + (int64_t)(row0 + 8) * d + c) =
        __floats2half2_rn(o[nt][2] * inv1, o[nt][3] * inv1);
  }
  if ((lane & 3) == 0) {
    const float ln2 = 0.69314718055994530942f;
    float* lb = lse + ((int64_t)b * H + h) * T;
    lb[row0] = (m0 + log2f(l0)) * ln2;
    lb[row0 + 8] = (m1 + log2f(l1)) * ln2;
  }
}

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

// Inverse RoPE of a gradient pair held by one thread: columns c (first half)
// and c+32 (second half) of a head at sequence position pos.
__device__ __forceinline__ void rope_bwd_pair(float& g1, float& g2, const float* cs, const float* sn, int pos, int c) {
  const float co = __ldg(cs + (int64_t)pos * 32 + c), si = __ldg(sn + (int64_t)pos * 32 + c);
  const float a = __fadd_rn(__fmul_rn(g1, co), __fmul_rn(g2, si));
  const float bb = __fsub_rn(__fmul_rn(g2, co), __fmul_rn(g1, si));
  g1 = a;
  g2 = bb;
}

// Store a 16x64 fp32 accumulator (C layout, rows row0 / row0+8) as fp16,
// scaled, optionally rotated back through RoPE.
__device__ __forceinline__ void store_grad_rows(__half* dst, int64_t ld, int row0, float (&acc)[8][4], float scale,
                                                const float* cs, const float* sn, int pos0, int lane) {
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nt][j] = r16(acc[nt][j] * scale);
  if (cs) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = nt * 8 + (lane & 3) * 2 + j;
        rope_bwd_pair(acc[nt][j], acc[nt + 4][j], cs, sn, pos0, c);
        rope_bwd_pair(acc[nt][2 + j], acc[nt + 4][2 + j], cs, sn, pos0 + 8, c);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + (lane & 3) * 2;
    *reinterpret_cast<__half2*>(dst + (int64_t)row0 * ld + c) = __floats2half2_rn(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<__half2*>(dst + (int64_t)(row0 + 8) * ld + c) = __floats2half2_rn(acc[nt][2], acc[nt][3]);
  }
}

// ---------------------------------------------------------------------------
// Backward, dK/dV: one CTA per (64-key block, head, batch); 4 warps x 16 keys.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(const __half* __restrict__ qkv,
                                                            const __half* __restrict__ dout,
                                                            const float* __restrict__ lse,
                                                            const float* __restrict__ delta, __half* __restrict__ dqkv,
                                                            int T, int H, float scale, float scale_log2,
                                                            const float* rope_cos, const float* rope_sin) {
  __shared__ __align__(128) __half sQ[2][64 * 64];
  __shared__ __align__(128) __half sO[2][64 * 64];  // dO tiles
  __shared__ __align__(128) __half sKV[64 * 64];
  __shared__ __align__(16) float sL[2][64];
  __shared__ __align__(16) float sD[2][64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkb = T / 64;
  const int kb = nkb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int d = H * D;
  const int64_t ld = 3 * (int64_t)d;
  const int k0 = kb * 64;
  const __half* qbase = qkv + (int64_t)b * T * ld + h * D;
  const __half* kbase = qbase + d;
  const __half* vbase = qbase + 2 * d;
  const __half* obase = dout + (int64_t)b * T * d + h * D;
  const float* lb = lse + ((int64_t)b * H + h) * T;
  const float* db = delta + ((int64_t)b * H + h) * T;
  const float log2e = 1.4426950408889634f;

  uint32_t kf[4][4], vf[4][4];
  load_tile<64, 128>(sKV, kbase + (int64_t)k0 * ld, ld, tid);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  load_afrag(kf, sKV, warp * 16, lane);
  __syncthreads();
  load_tile<64, 128>(sKV, vbase + (int64_t)k0 * ld, ld, tid);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  load_afrag(vf, sKV, warp * 16, lane);

  float dk[8][4], dv[8][4];
  zero(dk);
  zero(dv);
  const int key0 = k0 + warp * 16 + (lane >> 2);  // keys key0 and key0+8
  const int qt0 = k0 / 64;
  const int nqt = T / 64;

  auto load_q = [&](int qt, int buf) {
    load_tile<64, 128>(sQ[buf], qbase + (int64_t)qt * 64 * ld, ld, tid);
    load_tile<64, 128>(sO[buf], obase + (int64_t)qt * 64 * d, d, tid);
    if (tid < 16) cp_async16(&sL[buf][tid * 4], lb + qt * 64 + tid * 4);
    else if (tid < 32) cp_async16(&sD[buf][(tid - 16) * 4], db + qt * 64 + (tid - 16) * 4);
  };
  load_q(qt0, 0);
  cp_commit();
  for (int qt = qt0; qt < nqt; ++qt) {
    const int buf = (qt - qt0) & 1;
    if (qt + 1 < nqt) {
      load_q(qt + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int q0 = qt * 64;
    // S^T = K Q^T  [16 keys x 64 queries]
    float s[8][4];
    zero(s);
    mma_abt(s, kf, sQ[buf], lane);
    float dp[8][4];
    zero(dp);
    mma_abt(dp, vf, sO[buf], lane);
    const bool diag = (q0 < k0 + 64);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int qi = nt * 8 + (lane & 3) * 2 + j;
        const int q = q0 + qi;
        const float L = sL[buf][qi] * log2e, Dl = sD[buf][qi];
        float p0 = exp2f(s[nt][j] * scale_log2 - L);
        float p1 = exp2f(s[nt][2 + j] * scale_log2 - L);
        if (diag) {
          if (q < key0) p0 = 0.f;
          if (q < key0 + 8) p1 = 0.f;
        }
        s[nt][j] = p0;
        s[nt][2 + j] = p1;
        dp[nt][j] = p0 * (dp[nt][j] - Dl);
        dp[nt][2 + j] = p1 * (dp[nt][2 + j] - Dl);
      }
    }
    mma_pt(dv, s, sO[buf], lane);
    mma_pt(dk, dp, sQ[buf], lane);
    __syncthreads();
  }
  __half* gb = dqkv + (int64_t)b * T * ld + h * D;
  store_grad_rows(gb + 2 * d, ld, key0, dv, 1.0f, nullptr, nullptr, 0, lane);
  store_grad_rows(gb + d, ld, key0, dk, scale, rope_cos, rope_sin, key0, lane);
}

// ---------------------------------------------------------------------------
// Backward, dQ: one CTA per (64-query block, head, batch); 4 warps x 16 queries.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const __half* __restrict__ qkv,
                                                          const __half* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          const float* __restrict__ delta, __half* __restrict__ dqkv,
                                                          int T, int H, float scale, float scale_log2,
                                                          const float* rope_cos, const float* rope_sin) {
  __shared__ __align__(128) __half sK[2][64 * 64];
  __shared__ __align__(128) __half sV[2][64 * 64];
  __shared__ __align__(128) __half sA[64 * 64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = T / 64;
  const int qb = nqb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int d = H * D;
  const int64_t ld = 3 * (int64_t)d;
  const int q0 = qb * 64;
  const __half* qbase = qkv + (int64_t)b * T * ld + h * D;
  const __half* kbase = qbase + d;
  const __half* vbase = qbase + 2 * d;
  const __half* obase = dout + (int64_t)b * T * d + h * D;
  const float log2e = 1.4426950408889634f;

  uint32_t qf[4][4], of[4][4];
  load_tile<64, 128>(sA, qbase + (int64_t)q0 * ld, ld, tid);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  load_afrag(qf, sA, warp * 16, lane);
  __syncthreads();
  load_tile<64, 128>(sA, obase + (int64_t)q0 * d, d, tid);
  load_tile<64, 128>(sK[0], kbase, ld, tid);
  load_tile<64, 128>(sV[0], vbase, ld, tid);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  load_afrag(of, sA, warp * 16, lane);

  const int row0 = q0 + warp * 16 + (lane >> 2);
  const float* lb = lse + ((int64_t)b * H + h) * T;
  const float* db = delta + ((int64_t)b * H + h) * T;
  const float L0 = lb[row0] * log2e, L1 = lb[row0 + 8] * log2e;
  const float D0 = db[row0], D1 = db[row0 + 8];
  float dq[8][4];
  zero(dq);
  const int nkt = q0 / 64 + 1;
  for (int kt = 0; kt < nkt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) {
      load_tile<64, 128>(sK[buf ^ 1], kbase + (int64_t)(kt + 1) * 64 * ld, ld, tid);
      load_tile<64, 128>(sV[buf ^ 1], vbase + (int64_t)(kt + 1) * 64 * ld, ld, tid);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int k0 = kt * 64;
    float s[8][4], dp[8][4];
    zero(s);
    zero(dp);
    mma_abt(s, qf, sK[buf], lane);
    mma_abt(dp, of, sV[buf], lane);
    const bool diag = (k0 + 63 > q0);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = k0 + nt * 8 + (lane & 3) * 2 + j;
        float p0 = exp2f(s[nt][j] * scale_log2 - L0);
        float p1 = exp2f(s[nt][2 + j] * scale_log2 - L1);
        if (diag) {
          if (key > row0) p0 = 0.f;
          if (key > row0 + 8) p1 = 0.f;
        }
        dp[nt][j] = p0 * (dp[nt][j] - D0);
        dp[nt][2 + j] = p1 * (dp[nt][2 + j] - D1);
      }
    }
    mma_pt(dq, dp, sK[buf], lane);
    __syncthreads();
  }
  __half* gb = dqkv + (int64_t)b * T * ld + h * D;
  store_grad_rows(gb, ld, row0, dq, scale, rope_cos, rope_sin, row0, lane);
}

}  // namespace attn
}  // namespace jx

using namespace jx;
using namespace jx::attn;

extern "C" int jx_attn_fwd(const void* qkv, void* out, float* lse, int B, int T, int H, int Dh, float scale,
                           jx_stream_t stream) {
  JX_CHECK_ARG(qkv && out && lse, "jx_attn_fwd: NULL argument");
  JX_CHECK_ARG(Dh == 64, "jx_attn_fwd: head_dim must be 64 (got %d)", Dh);
  JX_CHECK_ARG(B > 0 && H > 0 && T > 0 && T % 128 == 0, "jx_attn_fwd: T must be a positive multiple of 128 (got %d)", T);
  JX_CHECK_ARG(aligned16(qkv) && aligned16(out), "jx_attn_fwd: buffers must be 16-byte aligned");
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(T / 128, H, B);
  attn_fwd_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(qkv), static_cast<__half*>(out), lse, T, H, scale_log2);
  JX_CHECK_LAUNCH("jx_attn_fwd");
  return JX_OK;
}

extern "C" int jx_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, float* delta,
                           void* dqkv, int B, int T, int H, int Dh, float scale, const float* rope_cos,
                           const float* rope_sin, jx_stream_t stream) {
  JX_CHECK_ARG(qkv && out && dout && lse && delta && dqkv, "jx_attn_bwd: NULL argument");
  JX_CHECK_ARG(Dh == 64, "jx_attn_bwd: head_dim must be 64 (got %d)", Dh);
  JX_CHECK_ARG(B > 0 && H > 0 && T > 0 && T % 128 == 0, "jx_attn_bwd: T must be a positive multiple of 128");
  JX_CHECK_ARG(aligned16(qkv) && aligned16(out) && aligned16(dout) && aligned16(dqkv) && aligned16(lse) &&
                   aligned16(delta),
               "jx_attn_bwd: buffers must be 16-byte aligned");
  JX_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr), "jx_attn_bwd: pass both RoPE tables or neither");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t threads = (int64_t)B * T * H * 8;
  attn_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(out),
                                                                static_cast<const __half*>(dout), delta, B, T, H);
  JX_CHECK_LAUNCH("jx_attn_bwd: delta");
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(T / 64, H, B);
  attn_bwd_dkdv_kernel<<<grid, 128, 0, s>>>(static_cast<const __half*>(qkv), static_cast<const __half*>(dout), lse,
                                            delta, static_cast<__half*>(dqkv), T, H, scale, scale_log2, rope_cos,
                                            rope_sin);
  JX_CHECK_LAUNCH("jx_attn_bwd: dkdv");
  attn_bwd_dq_kernel<<<grid, 128, 0, s>>>(static_cast<const __half*>(qkv), static_cast<const __half*>(dout), lse,
                                          delta, static_cast<__half*>(dqkv), T, H, scale, scale_log2, rope_cos,
                                          rope_sin);
  JX_CHECK_LAUNCH("jx_attn_bwd: dq");
  return JX_OK;
}
