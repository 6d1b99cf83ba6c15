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
constexpr int kFwdBlocksPerSm = 2;  // forward grid: blocks of kWarps warps resident per SM (96 registers)

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

// Grid-stride over rows (a grid of a few resident blocks per SM): each warp loads its next row
// (and residual row) into registers before it finishes the current one, so a load round trip
// overlaps every row's arithmetic and stores instead of being waited out per row.
template <int NV>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(const __half* __restrict__ x,
                                                                  const __half* __restrict__ resid,
                                                                  __half* __restrict__ sum_out,
                                                                  const float* __restrict__ gamma,
                                                                  __half* __restrict__ y, float* __restrict__ rstd,
                                                                  int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t step = (int64_t)gridDim.x * kWarps;
  int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 xq[NV], rq[NV];
  auto load_row = [&](int64_t r) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        xq[i] = *reinterpret_cast<const uint4*>(x + r * cols + c);
        if (resid) rq[i] = *reinterpret_cast<const uint4*>(resid + r * cols + c);
      }
    }
  };
  load_row(row);
  for (; row < rows; row += step) {
    float v[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const __half2* h = reinterpret_cast<const __half2*>(&xq[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h[j]);
          v[i][2 * j] = f.x;
          v[i][2 * j + 1] = f.y;
        }
        if (resid) {
          const __half2* rh = reinterpret_cast<const __half2*>(&rq[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(rh[j]);
            v[i][2 * j] = r16(v[i][2 * j] + f.x);
            v[i][2 * j + 1] = r16(v[i][2 * j + 1] + f.y);
          }
        }
      }
    }
    if (row + step < rows) load_row(row + step);  // the next row is in flight during this one
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        if (resid) store8(sum_out + row * cols + c, v[i]);
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

// The same backward with its row inputs staged in shared memory: a persistent grid (one block of
// kSWarps warps per SM), each warp walking rows w, w + W, w + 2W, ... (W warps in the grid) and
// keeping the dy / x / dresid rows of its next kStages - 1 rows in flight as bulk copies (one
// mbarrier per stage) while it computes the current one. The register-staged kernel above issues a
// row's loads only when it starts the row, so each warp waits out a full memory round trip per row;
// here the next row is already landing. Arithmetic and rounding points are those of
// rmsnorm_bwd_kernel; each lane reads its 8-column chunks back from shared memory (consecutive lanes,
// consecutive 16 bytes) and writes dx with coalesced 16-byte stores.
constexpr int kSWarps = 16;
constexpr int kStages = 2;
constexpr int kStagedMaxCols = 1024;  // 3 rows x 2 KiB x 2 stages x 16 warps = 192 KiB of staging

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int NV>
__global__ void __launch_bounds__(kSWarps * 32, 1) rmsnorm_bwd_staged_kernel(
    const __half* __restrict__ dy, const __half* __restrict__ x, const float* __restrict__ rstd,
    const float* __restrict__ gamma, const __half* __restrict__ dresid, __half* __restrict__ dx,
    float* __restrict__ dgamma_part, int64_t rows, int cols, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nin = dresid ? 3 : 2;                       // rows staged per stage: dy, x (, dresid)
  const uint32_t row_bytes = (uint32_t)cols * 2;
  const uint32_t stage_bytes = nin * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kSWarps * kStages * stage_bytes);
  float2* gs = reinterpret_cast<float2*>(bars + kSWarps * kStages);  // gamma, as column pairs
  for (int c = threadIdx.x * 2; c < cols; c += blockDim.x * 2) gs[c >> 1] = *reinterpret_cast<const float2*>(gamma + c);
  __syncthreads();
  uint8_t* ring = smem + (size_t)warp * kStages * stage_bytes;
  uint64_t* wbar = bars + warp * kStages;
  if (lane == 0)
    for (int s = 0; s < kStages; ++s) mbar_init(&wbar[s], 1);
  fence_barrier_init();
  __syncwarp();

  const int64_t step = (int64_t)gridDim.x * kSWarps;
  const int64_t first = (int64_t)blockIdx.x * kSWarps + warp;
  const int64_t nrows = first < rows ? (rows - first + step - 1) / step : 0;  // this warp's rows
  auto issue = [&](int64_t k) {  // lane 0: the k-th row of this warp into stage k % kStages
    const int64_t row = first + k * step;
    const int s = (int)(k % kStages);
    uint8_t* dst = ring + s * stage_bytes;
    mbar_expect_tx(&wbar[s], stage_bytes);
    bulk_copy_g2s(dst, dy + row * cols, row_bytes, &wbar[s]);
    bulk_copy_g2s(dst + row_bytes, x + row * cols, row_bytes, &wbar[s]);
    if (dresid) bulk_copy_g2s(dst + 2 * row_bytes, dresid + row * cols, row_bytes, &wbar[s]);
  };
  if (lane == 0)
    for (int64_t k = 0; k < kStages && k < nrows; ++k) issue(k);

  float dg[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dg[i][j] = 0.f;

  float rs_batch = 0.f;  // lane l holds rstd of this warp's row 32 * (k / 32) + l
  int64_t k = 0;
  for (; k < nrows; ++k) {
    if ((k & 31) == 0) {
      const int64_t kk = k + lane;
      rs_batch = kk < nrows ? rstd[first + kk * step] : 0.f;
    }
    const float rs = __shfl_sync(0xffffffffu, rs_batch, (int)(k & 31));
    const float2 rs2 = make_float2(rs, rs);
    const int s = (int)(k % kStages);
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&wbar[s], (uint32_t)((k / kStages) & 1), status, kStatusNormWait) ? 1 : 0;
    if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    const uint8_t* st = ring + s * stage_bytes;
    const int64_t row = first + k * step;
    // Pairs of columns in paired fp32 operations (non-contracted, the same roundings as above):
    // xh = x * rs, gh = f16(dy * gamma), dgamma += dy * f16(xh), dot += gh * xh.
    float2 dot2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const uint4 dq = *reinterpret_cast<const uint4*>(st + c * 2);
        const uint4 xq = *reinterpret_cast<const uint4*>(st + row_bytes + c * 2);
        const uint32_t* xw = &xq.x;
        const uint32_t* dw = &dq.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = h2f2(xw[j]), df = h2f2(dw[j]);
          const float2 g = gs[(c >> 1) + j];
          const float2 xh = __fmul2_rn(xf, rs2);
          const float2 gh = __half22float2(__float22half2_rn(__fmul2_rn(df, g)));
          const float2 d2 = __ffma2_rn(df, __half22float2(__float22half2_rn(xh)), make_float2(dg[i][2 * j], dg[i][2 * j + 1]));
          dg[i][2 * j] = d2.x;
          dg[i][2 * j + 1] = d2.y;
          dot2 = __ffma2_rn(gh, xh, dot2);
        }
      }
    }
    const float dot = warp_sum(dot2.x + dot2.y) / (float)cols;
    const float2 ndot2 = make_float2(-dot, -dot);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < cols) {
        const uint4 dq = *reinterpret_cast<const uint4*>(st + c * 2);
        const uint4 xq = *reinterpret_cast<const uint4*>(st + row_bytes + c * 2);
        uint4 rq = make_uint4(0, 0, 0, 0);
        if (dresid) rq = *reinterpret_cast<const uint4*>(st + 2 * row_bytes + c * 2);
        const uint32_t* xw = &xq.x;
        const uint32_t* dw = &dq.x;
        const uint32_t* rw = &rq.x;
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = h2f2(xw[j]), df = h2f2(dw[j]);
          const float2 g = gs[(c >> 1) + j];
          const float2 gh = __half22float2(__float22half2_rn(__fmul2_rn(df, g)));
          // dx = f16(rs * (gh - xh * dot)) (+ dresid, added in fp32 and rounded once more)
          const float2 v = __ffma2_rn(__fmul2_rn(xf, rs2), ndot2, gh);
          float2 w = __fmul2_rn(rs2, v);
          if (dresid) w = __fadd2_rn(__half22float2(__float22half2_rn(w)), h2f2(rw[j]));
          __half2 h = __float22half2_rn(w);
          o[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(dx + row * cols + c) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncwarp();  // every lane has read the stage
    if (lane == 0 && k + kStages < nrows) {
      fence_proxy_async_smem();  // generic reads of the stage before the async-proxy refill
      issue(k + kStages);
    }
  }
  // After an abandoned wait (k < nrows), copies may still be in flight: let them land first.
  if (lane == 0)
    for (int64_t kk = k; kk < nrows && kk < k + kStages; ++kk)
      mbar_wait(&wbar[kk % kStages], (uint32_t)((kk / kStages) & 1), nullptr, 0);
  __syncthreads();  // the staging area becomes the dgamma reduction buffer
  float* red = reinterpret_cast<float*>(smem);  // [kSWarps][cols]
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < cols)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * cols + c + j] = dg[i][j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kSWarps; ++w) sum += red[w * cols + c];
    dgamma_part[(int64_t)blockIdx.x * cols + c] = sum;
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

// Blocks of the norm backward kernels (each writes one dgamma / dbeta partial row): one per SM, at
// most kMaxParts, fewer for short inputs. The staged kernel keeps one block per SM resident.
extern "C" int jx_rmsnorm_bwd_parts(int64_t rows) {
  int n = num_sms();
  if (n > kMaxParts) n = kMaxParts;
  const int64_t b = (rows + kWarps - 1) / kWarps;
  return (int)(b < n ? (b < 1 ? 1 : b) : n);
}

static size_t staged_smem(int cols, bool resid) {
  return (size_t)kSWarps * kStages * (resid ? 3 : 2) * cols * 2 + kSWarps * kStages * sizeof(uint64_t) +
         (size_t)cols * sizeof(float);
}
static cudaError_t staged_smem_attr() {
  const int bytes = (int)staged_smem(kStagedMaxCols, true);
  cudaError_t e = cudaFuncSetAttribute(rmsnorm_bwd_staged_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rmsnorm_bwd_staged_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rmsnorm_bwd_staged_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(rmsnorm_bwd_staged_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e;
}

#define JX_RMS_NV_CASES(X) X(1) X(2) X(3) X(4) X(5) X(6) X(8) X(12) X(16)

static int pick_nv(int cols) {
  const int nv = (cols + 255) / 256;
  const int allowed[] = {1, 2, 3, 4, 5, 6, 8, 12, 16};
  for (int a : allowed)
    if (nv <= a) return a;
  return -1;
}

// The staged backward (cols <= kStagedMaxCols), shared by jx_rmsnorm_bwd and jx_rmsnorm_bwd_noalloc.
static int launch_staged_bwd(const __half* dyh, const __half* xh, const float* rstd, const float* gamma,
                             const __half* drh, __half* dxh, float* dgamma_part, int64_t rows, int cols,
                             cudaStream_t s) {
  const int nv = pick_nv(cols);
  const int grid = jx_rmsnorm_bwd_parts(rows);
  static std::atomic<uint64_t> attr_set{0};
  JX_CUDA_TRY(once_per_device(attr_set, staged_smem_attr), "jx_rmsnorm_bwd");
  const size_t ssmem = staged_smem(cols, drh != nullptr);
  int* st = status_ptr();
  switch (nv) {
#define X(N)                                                                                                   \
  case N:                                                                                                      \
    rmsnorm_bwd_staged_kernel<N><<<grid, kSWarps * 32, ssmem, s>>>(dyh, xh, rstd, gamma, drh, dxh, dgamma_part, rows, \
                                                                  cols, st);                                   \
    break;
    X(1) X(2) X(3) X(4)
#undef X
    default:
      jx::set_error("jx_rmsnorm_bwd: unsupported cols %d", cols);
      return JX_ERR_UNSUPPORTED;
  }
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd");
  return JX_OK;
}

extern "C" int jx_rmsnorm_fwd(const void* x, const void* resid, void* sum_out, const float* gamma, void* y,
                              float* rstd, int64_t rows, int cols, float eps, jx_stream_t stream) {
  JX_CHECK_ARG(x && gamma && y && rstd, "jx_rmsnorm_fwd: NULL argument");
  JX_CHECK_ARG(rows > 0 && cols > 0 && cols % 8 == 0 && cols <= 4096, "jx_rmsnorm_fwd: cols must be a multiple of 8 in (0, 4096] (got %d)", cols);
  JX_CHECK_ARG(!resid || sum_out, "jx_rmsnorm_fwd: residual input needs sum_out");
  JX_CHECK_ARG(aligned16(x) && aligned16(y) && aligned16(gamma) && (!resid || (aligned16(resid) && aligned16(sum_out))),
               "jx_rmsnorm_fwd: buffers must be 16-byte aligned");
  const int nv = pick_nv(cols);
  const int64_t blocks = (rows + kWarps - 1) / kWarps;
  const int64_t resident = (int64_t)num_sms() * kFwdBlocksPerSm;
  const unsigned grid = (unsigned)(blocks < resident ? blocks : resident);
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
  if (cols <= kStagedMaxCols) return launch_staged_bwd(dyh, xh, rstd, gamma, drh, dxh, dgamma_part, rows, cols, s);
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
  const int grid = jx_rmsnorm_bwd_parts(rows);  // <= kNoAllocMaxParts
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* dyh = static_cast<const __half*>(dy);
  const __half* xh = static_cast<const __half*>(x);
  const __half* drh = static_cast<const __half*>(dresid);
  __half* dxh = static_cast<__half*>(dx);
  // Every block overwrites its own row of partials and the reduction reads only
  // those rows, so nothing left in the array by an earlier call is ever read.
  const int rc2 = launch_staged_bwd(dyh, xh, rstd, gamma, drh, dxh, part, rows, cols, s);
  if (rc2 != JX_OK) return rc2;
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd_noalloc");
  dgamma_reduce_kernel<<<(cols + 31) / 32, 1024, 0, s>>>(part, grid, cols, dgamma, accumulate);
  JX_CHECK_LAUNCH("jx_rmsnorm_bwd_noalloc: reduce");
  return JX_OK;
}
