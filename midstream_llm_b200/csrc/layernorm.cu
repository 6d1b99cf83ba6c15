// LayerNorm (with optional bias) forward/backward over an fp16 residual stream.
//
// Follows nn.LayerNorm as the reference decoder builds it for norm_type
// "layernorm" (Midstream-LLM src/jishui/model_torch.py:12-15) under fp16
// autocast: layer_norm runs in fp32 (the fp16 input is widened exactly, gain
// and bias are the fp32 parameters), and its fp32 output is rounded to fp16
// once, by the cast in front of the next fp16 GEMM. In backward the fp16
// gradient is widened, the fp32 layer-norm backward runs, and the input
// gradient is rounded to fp16 (the backward of that widening cast) before it
// joins the fp16 residual gradient. dgamma / dbeta are fp32 sums.
//
// One warp per row; each lane owns NV 8-element (16-byte) vectors, so a row is
// read once with coalesced 16-byte loads and kept in registers; mean and
// variance are two passes over those registers (biased variance, as torch).
// HBM traffic per row: fwd 2*cols*2 bytes (+8 bytes of statistics), bwd
// 3*cols*2 bytes (+cols*2 with the residual gradient).
#include "jx_common.cuh"
#include "jx_host.h"

extern "C" int jx_rmsnorm_bwd_parts(int64_t rows);

namespace jx {
namespace ln {

constexpr int kWarps = 8;

__device__ __forceinline__ float2 h2f2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

template <int NV>
__global__ void __launch_bounds__(kWarps * 32) layernorm_fwd_kernel(const __half* __restrict__ x,
                                                                    const float* __restrict__ gamma,
                                                                    const float* __restrict__ beta,
                                                                    __half* __restrict__ y,
                                                                    float* __restrict__ mean_out,
                                                                    float* __restrict__ rstd_out, int64_t rows,
                                                                    int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + row * cols;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t* w = &u.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = h2f2(w[j]);
        v[i][2 * j] = f.x;
        v[i][2 * j + 1] = f.y;
        s += f.x + f.y;
      }
    }
  }
  const float mean = warp_sum(s) / (float)cols;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float dlt = v[i][j] - mean;
        ss += dlt * dlt;
      }
  }
  const float rs = rsqrtf(warp_sum(ss) / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = *reinterpret_cast<const float2*>(gamma + c + 2 * j);
        float y0 = (v[i][2 * j] - mean) * rs * g.x;
        float y1 = (v[i][2 * j + 1] - mean) * rs * g.y;
        if (beta) {
          const float2 b = *reinterpret_cast<const float2*>(beta + c + 2 * j);
          y0 += b.x;
          y1 += b.y;
        }
        __half2 h = __floats2half2_rn(y0, y1);
        o[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(y + row * cols + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rs;
  }
}

// Backward: per row xhat = (x - mean) * rstd, g = dy * gamma,
// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), rounded to fp16 and added
// to the fp16 residual gradient; per-block fp32 partials of dgamma = sum dy*xhat
// and dbeta = sum dy (deterministic: fixed rows per block, fixed tree).
template <int NV>
__global__ void __launch_bounds__(kWarps * 32) layernorm_bwd_kernel(const __half* __restrict__ dy,
                                                                    const __half* __restrict__ x,
                                                                    const float* __restrict__ mean_in,
                                                                    const float* __restrict__ rstd_in,
                                                                    const float* __restrict__ gamma,
                                                                    const __half* __restrict__ dresid,
                                                                    __half* __restrict__ dx,
                                                                    float* __restrict__ dgamma_part,
                                                                    float* __restrict__ dbeta_part, int64_t rows,
                                                                    int cols) {
  extern __shared__ float red[];  // [kWarps][cols]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float dg[NV][8], db[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dg[i][j] = db[i][j] = 0.f;

  for (int64_t row = blockIdx.x * (int64_t)kWarps + warp; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const float mu = mean_in[row], rs = rstd_in[row];
    uint4 xq[NV], dq[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        dq[i] = *reinterpret_cast<const uint4*>(dy + row * cols + c);
        xq[i] = *reinterpret_cast<const uint4*>(x + row * cols + c);
      }
    }
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const uint32_t* xw = &xq[i].x;
        const uint32_t* dw = &dq[i].x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = h2f2(xw[j]), df = h2f2(dw[j]);
          const float2 g = *reinterpret_cast<const float2*>(gamma + c + 2 * j);
          const float xh0 = (xf.x - mu) * rs, xh1 = (xf.y - mu) * rs;
          dg[i][2 * j] += df.x * xh0;
          dg[i][2 * j + 1] += df.y * xh1;
          db[i][2 * j] += df.x;
          db[i][2 * j + 1] += df.y;
          const float g0 = df.x * g.x, g1 = df.y * g.y;
          sg += g0 + g1;
          sgx += g0 * xh0 + g1 * xh1;
        }
      }
    }
    const float a = warp_sum(sg) / (float)cols;
    const float b = warp_sum(sgx) / (float)cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const uint32_t* xw = &xq[i].x;
        const uint32_t* dw = &dq[i].x;
        uint4 rq = make_uint4(0, 0, 0, 0);
        if (dresid) rq = *reinterpret_cast<const uint4*>(dresid + row * cols + c);
        const uint32_t* rw = &rq.x;
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = h2f2(xw[j]), df = h2f2(dw[j]);
          const float2 g = *reinterpret_cast<const float2*>(gamma + c + 2 * j);
          const float xh0 = (xf.x - mu) * rs, xh1 = (xf.y - mu) * rs;
          float o0 = __half2float(__float2half_rn(rs * (df.x * g.x - a - xh0 * b)));
          float o1 = __half2float(__float2half_rn(rs * (df.y * g.y - a - xh1 * b)));
          if (dresid) {
            const float2 rf = h2f2(rw[j]);
            o0 += rf.x;
            o1 += rf.y;
          }
          __half2 h = __floats2half2_rn(o0, o1);
          o[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(dx + row * cols + c) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // Block reduction of the partials across warps: dgamma, then dbeta through the same buffer.
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && !dbeta_part) break;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols)
#pragma unroll
        for (int j = 0; j < 8; ++j) red[warp * cols + c + j] = pass ? db[i][j] : dg[i][j];
    }
    __syncthreads();
    float* part = pass ? dbeta_part : dgamma_part;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += red[w * cols + c];
      part[(int64_t)blockIdx.x * cols + c] = s;
    }
    __syncthreads();
  }
}

}  // namespace ln
}  // namespace jx

using namespace jx;
using namespace jx::ln;

#define JX_LN_NV_CASES(X) X(1) X(2) X(3) X(4) X(5) X(6) X(8) X(12) X(16)

static int ln_pick_nv(int cols) {
  const int nv = (cols + 255) / 256;
  const int allowed[] = {1, 2, 3, 4, 5, 6, 8, 12, 16};
  for (int a : allowed)
    if (nv <= a) return a;
  return -1;
}

extern "C" int jx_layernorm_fwd(const void* x, const float* gamma, const float* beta, void* y, float* mean,
                                float* rstd, int64_t rows, int cols, float eps, jx_stream_t stream) {
  JX_CHECK_ARG(x && gamma && y && mean && rstd, "jx_layernorm_fwd: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0 && cols <= 4096,
               "jx_layernorm_fwd: cols must be a multiple of 8 in (0, 4096] (got %d)", cols);
  JX_CHECK_ARG(aligned16(x) && aligned16(y) && aligned16(gamma) && (!beta || aligned16(beta)),
               "jx_layernorm_fwd: buffers must be 16-byte aligned");
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  __half* yh = static_cast<__half*>(y);
  switch (ln_pick_nv(cols)) {
#define X(N)                                                                                               \
  case N:                                                                                                  \
    layernorm_fwd_kernel<N><<<grid, kWarps * 32, 0, s>>>(xh, gamma, beta, yh, mean, rstd, rows, cols, eps); \
    break;
    JX_LN_NV_CASES(X)
#undef X
    default:
      jx::set_error("jx_layernorm_fwd: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_layernorm_fwd");
  return JX_OK;
}

extern "C" int jx_layernorm_bwd(const void* dy, const void* x, const float* mean, const float* rstd,
                                const float* gamma, const void* dresid, void* dx, float* dgamma_part,
                                float* dbeta_part, int64_t rows, int cols, jx_stream_t stream) {
  JX_CHECK_ARG(dy && x && mean && rstd && gamma && dx && dgamma_part, "jx_layernorm_bwd: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0 && cols <= 4096,
               "jx_layernorm_bwd: cols must be a multiple of 8 in (0, 4096]");
  JX_CHECK_ARG(aligned16(dy) && aligned16(x) && aligned16(dx) && aligned16(gamma) && (!dresid || aligned16(dresid)),
               "jx_layernorm_bwd: buffers must be 16-byte aligned");
  const int grid = jx_rmsnorm_bwd_parts(rows);  // the partial count the caller allocated
  const size_t smem = (size_t)kWarps * cols * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* dyh = static_cast<const __half*>(dy);
  const __half* xh = static_cast<const __half*>(x);
  const __half* drh = static_cast<const __half*>(dresid);
  __half* dxh = static_cast<__half*>(dx);
  switch (ln_pick_nv(cols)) {
#define X(N)                                                                                                  \
  case N:                                                                                                     \
    if (smem > 48 * 1024)                                                                                     \
      cudaFuncSetAttribute(layernorm_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);  \
    layernorm_bwd_kernel<N><<<grid, kWarps * 32, smem, s>>>(dyh, xh, mean, rstd, gamma, drh, dxh, dgamma_part, \
                                                            dbeta_part, rows, cols);                          \
    break;
    JX_LN_NV_CASES(X)
#undef X
    default:
      jx::set_error("jx_layernorm_bwd: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_layernorm_bwd");
  return JX_OK;
}
