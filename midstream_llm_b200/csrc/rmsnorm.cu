// RMSNorm forward/backward with optional residual-add fusion.
//
// Follows nn.RMSNorm as the reference decoder uses it under fp16 autocast
// (Midstream-LLM src/jishui/model_torch.py:12-15, 72-73): the residual
// stream is fp16, the statistics are computed in fp32, the normalised value is
// rounded to fp16 before the fp32 gain multiplies it, and the result feeds an
// fp16 GEMM (so it is rounded to fp16 once more here).
//
// One warp per row; each lane owns NV 8-element (16-byte) vectors, so a row
// of `cols` fp16 values is read once with coalesced 16-byte loads and kept in
// registers. HBM traffic per row: fwd 2*cols*2 bytes (+2*cols*2 with the
// residual), bwd 3*cols*2 bytes (+cols*2 with the residual gradient).
#include <mutex>

#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace rms {

constexpr int kWarps = 8;
constexpr int kMaxParts = 296;

__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float r16(float x) { return __half2float(__float2half_rn(x)); }

template <int NV>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(const __half* __restrict__ x,
                                                                  const __half* __restrict__ resid,
                                                                  __half* __restrict__ sum_out,
                                                                  const float* __restrict__ gamma,
                                                                  __half* __restrict__ y, float* __restrict__ rstd,
                                                                  int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + row * cols;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols) {
      load8(xr + c, v[i]);
      if (resid) {
        float r[8];
        load8(resid + row * cols + c, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = r16(v[i][j] + r[j]);
        store8(sum_out + row * cols + c, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = warp_sum(ss);
  const float rs = 1.0f / sqrtf(ss / (float)cols + eps);
  if (lane == 0) rstd[row] = rs;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols) {
      float o[8];
      const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
      const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r16(v[i][j] * rs) * g[j];
      store8(y + row * cols + c, o);
    }
  }
}

__device__ __forceinline__ float2 h2f2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// dx = f16(dresid + f16(rstd * (gh - xhat * mean(gh * xhat)))), gh = f16(dy * gamma),
// xhat = x * rstd; dgamma partial += dy * f16(xhat). Rows are held as packed
// fp16 (4 registers per 8 values) to keep occupancy high.
template <int NV>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_kernel(const __half* __restrict__ dy,
                                                                  const __half* __restrict__ x,
                                                                  const float* __restrict__ rstd,
                                                                  const float* __restrict__ gamma,
                                                                  const __half* __restrict__ dresid,
                                                                  __half* __restrict__ dx,
                                                                  float* __restrict__ dgamma_part, int64_t rows,
                                                                  int cols) {
  extern __shared__ float red[];  // [kWarps][cols]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float dg[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dg[i][j] = 0.f;

  for (int64_t row = blockIdx.x * (int64_t)kWarps + warp; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const float rs = rstd[row];
    uint4 xq[NV], dq[NV], rq[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        dq[i] = *reinterpret_cast<const uint4*>(dy + row * cols + c);
        xq[i] = *reinterpret_cast<const uint4*>(x + row * cols + c);
        if (dresid) rq[i] = *reinterpret_cast<const uint4*>(dresid + row * cols + c);
      }
    }
    float dot = 0.f;
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
          const float xh0 = xf.x * rs, xh1 = xf.y * rs;
          dg[i][2 * j] += df.x * r16(xh0);
          dg[i][2 * j + 1] += df.y * r16(xh1);
          dot += r16(df.x * g.x) * xh0 + r16(df.y * g.y) * xh1;
        }
      }
    }
    dot = warp_sum(dot) / (float)cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const uint32_t* xw = &xq[i].x;
        const uint32_t* dw = &dq[i].x;
        const uint32_t* rw = &rq[i].x;
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = h2f2(xw[j]), df = h2f2(dw[j]);
          const float2 g = *reinterpret_cast<const float2*>(gamma + c + 2 * j);
          float o0 = r16(rs * (r16(df.x * g.x) - xf.x * rs * dot));
          float o1 = r16(rs * (r16(df.y * g.y) - xf.y * rs * dot));
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
  // Block reduction of the dgamma partials across warps.
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * cols + c + j] = dg[i][j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w * cols + c];
    dgamma_part[(int64_t)blockIdx.x * cols + c] = s;
  }
}

// dgamma[c] (+)= sum_p part[p][c]: 32 columns x 32 part-groups per block (each thread sums
// every 32nd part with two independent accumulators, so its loads overlap), then a fixed tree
// over the groups: deterministic order.
__global__ void __launch_bounds__(1024) dgamma_reduce_kernel(const float* __restrict__ part, int nparts, int cols,
                                                             float* __restrict__ dgamma, int accumulate) {
  __shared__ float red[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s0 = 0.f, s1 = 0.f;
  if (c < cols) {
    int p = ty;
    for (; p + 32 < nparts; p += 64) {
      s0 += part[(int64_t)p * cols + c];
      s1 += part[(int64_t)(p + 32) * cols + c];
    }
    if (p < nparts) s0 += part[(int64_t)p * cols + c];
  }
  red[ty][tx] = s0 + s1;
  __syncthreads();
  if (ty == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) t += red[j][tx];
    dgamma[c] = accumulate ? dgamma[c] + t : t;
  }
}

template <template <int> class K>
struct Dispatch;

}  // namespace rms
}  // namespace jx

using namespace jx;
using namespace jx::rms;

extern "C" int jx_rmsnorm_bwd_parts(int64_t rows) {
  int64_t b = (rows + kWarps - 1) / kWarps;
  return (int)(b < kMaxParts ? (b < 1 ? 1 : b) : kMaxParts);
}

#define JX_RMS_NV_CASES(X) X(1) X(2) X(3) X(4) X(5) X(6) X(8) X(12) X(16)

static int pick_nv(int cols) {
  const int nv = (cols + 255) / 256;
  const int allowed[] = {1, 2, 3, 4, 5, 6, 8, 12, 16};
  for (int a : allowed)
    if (nv <= a) return a;
  return -1;
}

extern "C" int jx_rmsnorm_fwd(const void* x, const void* resid, void* sum_out, const float* gamma, void* y,
                              float* rstd, int64_t rows, int cols, float eps, jx_stream_t stream) {
  JX_CHECK_ARG(x && gamma && y && rstd, "jx_rmsnorm_fwd: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0 && cols <= 4096, "jx_rmsnorm_fwd: cols must be a multiple of 8 in (0, 4096] (got %d)", cols);
  JX_CHECK_ARG(!resid || sum_out, "jx_rmsnorm_fwd: residual input needs sum_out");
  JX_CHECK_ARG(aligned16(x) && aligned16(y) && aligned16(gamma) && (!resid || (aligned16(resid) && aligned16(sum_out))),
               "jx_rmsnorm_fwd: buffers must be 16-byte aligned");
  const int nv = pick_nv(cols);
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const __half* rh = static_cast<const __half*>(resid);
  __half* sh = static_cast<__half*>(sum_out);
  __half* yh = static_cast<__half*>(y);
  switch (nv) {
#define X(N)                                                                                       \
  case N:                                                                                          \
    rmsnorm_fwd_kernel<N><<<grid, kWarps * 32, 0, s>>>(xh, rh, sh, gamma, yh, rstd, rows, cols, eps); \
    break;
    JX_RMS_NV_CASES(X)
#undef X
    default:
      jx::set_error("jx_rmsnorm_fwd: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_rmsnorm_fwd");
  return JX_OK;
}

extern "C" int jx_rmsnorm_bwd(const void* dy, const void* x, const float* rstd, const float* gamma, const void* dresid,
                              void* dx, float* dgamma_part, int64_t rows, int cols, jx_stream_t stream) {
  JX_CHECK_ARG(dy && x && rstd && gamma && dx && dgamma_part, "jx_rmsnorm_bwd: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0 && cols <= 4096, "jx_rmsnorm_bwd: cols must be a multiple of 8 in (0, 4096]");
  JX_CHECK_ARG(aligned16(dy) && aligned16(x) && aligned16(dx) && aligned16(gamma) && (!dresid || aligned16(dresid)),
               "jx_rmsnorm_bwd: buffers must be 16-byte aligned");
  const int nv = pick_nv(cols);
  const int grid = jx_rmsnorm_bwd_parts(rows);
  const size_t smem = (size_t)kWarps * cols * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* dyh = static_cast<const __half*>(dy);
  const __half* xh = static_cast<const __half*>(x);
  const __half* drh = static_cast<const __half*>(dresid);
  __half* dxh = static_cast<__half*>(dx);
  switch (nv) {
#define X(N)                                                                                     \
  case N:                                                                                        \
    if (smem > 48 * 1024)                                                                        \
      cudaFuncSetAttribute(rmsnorm_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                           (int)smem);                                                           \
    rmsnorm_bwd_kernel<N><<<grid, kWarps * 32, smem, s>>>(dyh, xh, rstd, gamma, drh, dxh, dgamma_part, rows, \
                                                          cols);                                 \
    break;
    JX_RMS_NV_CASES(X)
#undef X
    default:
      jx::set_error("jx_rmsnorm_bwd: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd");
  return JX_OK;
}

extern "C" int jx_rmsnorm_dgamma_reduce(const float* dgamma_part, int nparts, int cols, float* dgamma, int accumulate,
                                        jx_stream_t stream) {
  JX_CHECK_ARG(dgamma_part && dgamma && nparts > 0 && cols > 0, "jx_rmsnorm_dgamma_reduce: bad argument");
  dgamma_reduce_kernel<<<(cols + 31) / 32, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      dgamma_part, nparts, cols, dgamma, accumulate);
  JX_CHECK_LAUNCH("jx_rmsnorm_dgamma_reduce");
  return JX_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free RMSNorm backward.
//
// Some callers cannot allocate device memory at all: a host runtime that binds
// this library through the C ABI without a device allocator of its own, or one
// that runs under a fixed, pre-reserved memory budget and must not call
// cudaMalloc / cudaFree (which can synchronise the whole device and stall other
// streams). jx_rmsnorm_bwd needs a caller-provided scratch buffer for the
// per-block dgamma partials; this variant keeps that scratch in a fixed
// file-scope device array instead, so the caller passes only inputs and
// outputs. The array holds kNoAllocMaxParts x kNoAllocMaxCols floats
// (296 x 1024 x 4 B = 1.16 MiB) and stays resident on every GPU that loads the
// library until the process exits.
// ---------------------------------------------------------------------------
namespace jx {
namespace rms {

constexpr int kNoAllocMaxCols = 1024;
constexpr int kNoAllocMaxParts = kMaxParts;

static __device__ __align__(256) float g_noalloc_dgamma_part[kNoAllocMaxParts * kNoAllocMaxCols];

// Device address of g_noalloc_dgamma_part, looked up with the device current by the first call made on
// that device and cached per device; the cache is keyed on the CUDA context, so a device reset (which
// reloads the module at a new address) triggers a fresh lookup instead of a stale pointer.
static SymbolCache g_noalloc_cache;

static int noalloc_scratch(float** out) {
  void* p = g_noalloc_cache.get(reinterpret_cast<const void*>(&g_noalloc_dgamma_part));
  JX_CHECK_ARG(p != nullptr, "jx_rmsnorm_bwd_noalloc: cannot look up the device address of the scratch array");
  *out = static_cast<float*>(p);
  return JX_OK;
}

}  // namespace rms
}  // namespace jx

extern "C" int jx_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* rstd, const float* gamma,
                                      const void* dresid, void* dx, float* dgamma, int accumulate, int64_t rows,
                                      int cols, jx_stream_t stream) {
  JX_CHECK_ARG(dy && x && rstd && gamma && dx && dgamma, "jx_rmsnorm_bwd_noalloc: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0, "jx_rmsnorm_bwd_noalloc: cols must be a positive multiple of 8");
  JX_CHECK_ARG(cols <= kNoAllocMaxCols,
               "jx_rmsnorm_bwd_noalloc: cols %d exceeds the built-in scratch limit of %d columns; use jx_rmsnorm_bwd "
               "with a caller-provided scratch buffer",
               cols, kNoAllocMaxCols);
  JX_CHECK_ARG(aligned16(dy) && aligned16(x) && aligned16(dx) && aligned16(gamma) && (!dresid || aligned16(dresid)),
               "jx_rmsnorm_bwd_noalloc: buffers must be 16-byte aligned");
  float* part = nullptr;
  const int rc = noalloc_scratch(&part);
  if (rc != JX_OK) return rc;
  const int nv = pick_nv(cols);
  const int grid = jx_rmsnorm_bwd_parts(rows);  // <= kNoAllocMaxParts
  const size_t smem = (size_t)kWarps * cols * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* dyh = static_cast<const __half*>(dy);
  const __half* xh = static_cast<const __half*>(x);
  const __half* drh = static_cast<const __half*>(dresid);
  __half* dxh = static_cast<__half*>(dx);
  // Every block overwrites its own row of partials and the reduction reads only
  // those rows, so nothing left in the array by an earlier call is ever read.
  switch (nv) {
#define X(N)                                                                                                    \
  case N:                                                                                                       \
    rmsnorm_bwd_kernel<N><<<grid, kWarps * 32, smem, s>>>(dyh, xh, rstd, gamma, drh, dxh, part, rows, cols); \
    break;
    X(1) X(2) X(3) X(4)
#undef X
    default:
      jx::set_error("jx_rmsnorm_bwd_noalloc: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd_noalloc");
  dgamma_reduce_kernel<<<(cols + 31) / 32, 1024, 0, s>>>(part, grid, cols, dgamma, accumulate);
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd_noalloc: reduce");
  return JX_OK;
}
