// Fused GradScaler unscale + non-finite check + global grad norm, and the
// AdamW update over flat parameter/moment buffers.
//
// Reference semantics (Midstream-LLM src/jishui/pretrain_torch.py:218-233):
//   scaler.unscale_(opt)         g <- g * inv_scale, found_inf if any g non-finite
//   clip_grad_norm_(params, c)   total = ||g||_2, coef = min(c/(total+1e-6), 1), g <- g * coef
//   scaler.step(opt)             AdamW(fused=True) update unless found_inf
//   scaler.update()              growth/backoff of the loss scale
// Here the stats pass reads the raw (scaled) gradients once and, as
// GradScaler.unscale_ does, writes them back unscaled (so `.grad` holds what
// torch's own clip_grad_norm_ expects); the clip coefficient is folded into
// the update pass, so clipped gradients are never written to HBM. The AdamW arithmetic follows torch's fused AdamW
// (double-precision hyper-parameters, fp32 state): p -= lr*wd*p;
// m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*g*g;
// p -= (lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps).
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace opt {

constexpr int kThreads = 512;
constexpr int kMaxParts = 1184;  // 8 blocks per SM on a 148-SM part

template <bool F16>
__device__ __forceinline__ void load_grad4(const void* g, int64_t i, float (&v)[4]) {
  if constexpr (F16) {
    const __half2* p = reinterpret_cast<const __half2*>(static_cast<const __half*>(g) + i);
    const float2 a = __half22float2(p[0]);
    const float2 b = __half22float2(p[1]);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  } else {
    const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(g) + i);
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
  }
}

template <bool F16>
__device__ __forceinline__ float load_grad1(const void* g, int64_t i) {
  if constexpr (F16)
    return __half2float(static_cast<const __half*>(g)[i]);
  else
    return static_cast<const float*>(g)[i];
}

template <bool F16>
__global__ void __launch_bounds__(kThreads) grad_stats_kernel(const void* __restrict__ grad, int64_t n,
                                                              const float* __restrict__ inv_scale,
                                                              float* __restrict__ partial,
                                                              float* __restrict__ found_inf,
                                                              float* __restrict__ unscaled) {
  const float inv = *inv_scale;
  float ss = 0.f;
  bool bad = false;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float v[4];
    load_grad4<F16>(grad, i * 4, v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] *= inv;
      bad |= !isfinite(v[j]);
      ss += v[j] * v[j];
    }
    if (unscaled) reinterpret_cast<float4*>(unscaled)[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float u = load_grad1<F16>(grad, i) * inv;
    bad |= !isfinite(u);
    ss += u * u;
    if (unscaled) unscaled[i] = u;
  }
  __shared__ float red[kThreads / 32];
  ss = warp_sum(ss);
  const unsigned anybad = __any_sync(0xffffffffu, bad);
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = ss;
    if (anybad) *found_inf = 1.0f;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) partial[blockIdx.x] = t;
  }
}

__global__ void grad_finalize_kernel(const float* __restrict__ partial, int nparts, float max_norm,
                                     float* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += partial[i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
    const float total = sqrtf((float)t);
    float coef = 1.0f;
    if (max_norm > 0.f) {
      coef = max_norm / (total + 1e-6f);
      coef = fminf(coef, 1.0f);
    }
    out[0] = total;
    out[1] = coef;
  }
}

struct AdamHyper {
  double lr, beta1, beta2, eps, wd;
};

// step_state[0] += 1 unless the update is skipped; [1] = 1 - beta1^step,
// [2] = sqrt(1 - beta2^step) (double precision, then rounded to fp32).
__global__ void adamw_prepare_kernel(float* __restrict__ state, const float* __restrict__ found_inf, double beta1,
                                     double beta2) {
  if (found_inf && *found_inf != 0.f) return;
  const float step = state[0] + 1.0f;
  state[0] = step;
  state[1] = (float)(1.0 - pow(beta1, (double)step));
  state[2] = (float)sqrt(1.0 - pow(beta2, (double)step));
}

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, const AdamHyper& h, float bc1,
                                         float bc2_sqrt) {
  p = (float)((double)p - h.lr * h.wd * (double)p);
  m = (float)(h.beta1 * (double)m + (1.0 - h.beta1) * (double)g);
  v = (float)(h.beta2 * (double)v + (1.0 - h.beta2) * (double)g * (double)g);
  const float step_size = (float)(h.lr / (double)bc1);
  const float denom = (float)((double)(sqrtf(v) / bc2_sqrt) + h.eps);
  p -= step_size * m / denom;
}

template <bool F16>
__global__ void __launch_bounds__(kThreads) adamw_kernel(float* __restrict__ p, const void* __restrict__ grad,
                                                         float* __restrict__ m, float* __restrict__ v,
                                                         __half* __restrict__ p16, int64_t n,
                                                         const float* __restrict__ inv_scale,
                                                         const float* __restrict__ clip,
                                                         const float* __restrict__ found_inf,
                                                         const float* __restrict__ state, AdamHyper h) {
  if (found_inf && *found_inf != 0.f) return;
  const float bc1 = state[1], bc2s = state[2];
  const float inv = inv_scale ? *inv_scale : 1.0f;
  const float coef = clip ? *clip : 1.0f;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float g[4];
    load_grad4<F16>(grad, i * 4, g);
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x;
    float* ma = &mm.x;
    float* va = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) adam_one(pa[j], (g[j] * inv) * coef, ma[j], va[j], h, bc1, bc2s);
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16) {
      __half2* d = reinterpret_cast<__half2*>(p16 + i * 4);
      d[0] = __floats2half2_rn(pp.x, pp.y);
      d[1] = __floats2half2_rn(pp.z, pp.w);
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float pv = p[i], mv = m[i], vv = v[i];
    adam_one(pv, (load_grad1<F16>(grad, i) * inv) * coef, mv, vv, h, bc1, bc2s);
    p[i] = pv;
    m[i] = mv;
    v[i] = vv;
    if (p16) p16[i] = __float2half_rn(pv);
  }
}

__global__ void scaler_update_kernel(float* scale, int* tracker, const float* found_inf, float growth, float backoff,
                                     int interval) {
  if (*found_inf != 0.f) {
    *scale = *scale * backoff;
    *tracker = 0;
  } else {
    const int t = *tracker + 1;
    if (t == interval) {
      *scale = *scale * growth;
      *tracker = 0;
    } else {
      *tracker = t;
    }
  }
}

__global__ void cast_kernel(const float* __restrict__ src, __half* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 f = reinterpret_cast<const float4*>(src)[i];
    __half2* d = reinterpret_cast<__half2*>(dst + i * 4);
    d[0] = __floats2half2_rn(f.x, f.y);
    d[1] = __floats2half2_rn(f.z, f.w);
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = __float2half_rn(src[i]);
}

__global__ void transpose_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int64_t rows,
                                 int64_t cols) {
  __shared__ __half tile[32][33];
  const int64_t c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][i];
  }
}

static int blocks_for(int64_t n) {
  int64_t b = (n / 4 + kThreads - 1) / kThreads;
  if (b < 1) b = 1;
  const int64_t cap = (int64_t)num_sms() * 8;
  return (int)(b < cap ? b : cap);
}

}  // namespace opt
}  // namespace jx

using namespace jx;
using namespace jx::opt;

extern "C" int jx_grad_stats_parts(int64_t n) {
  int64_t b = (n / 4 + kThreads - 1) / kThreads;
  if (b < 1) b = 1;
  return (int)(b < kMaxParts ? b : kMaxParts);
}

extern "C" int jx_grad_stats(const void* grad, int grad_is_f16, int64_t n, const float* inv_scale, float* partial,
                             float* found_inf, float* unscaled_out, jx_stream_t stream) {
  JX_CHECK_ARG(grad && inv_scale && partial && found_inf && n > 0, "jx_grad_stats: bad argument");
  JX_CHECK_ARG(aligned16(grad) && (!unscaled_out || aligned16(unscaled_out)),
               "jx_grad_stats: grad and unscaled_out must be 16-byte aligned");
  JX_CHECK_ARG(!unscaled_out || !grad_is_f16 || (const void*)unscaled_out != grad,
               "jx_grad_stats: f16 gradients cannot be unscaled in place into f32");
  const int grid = jx_grad_stats_parts(n);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (grad_is_f16)
    grad_stats_kernel<true><<<grid, kThreads, 0, s>>>(grad, n, inv_scale, partial, found_inf, unscaled_out);
  else
    grad_stats_kernel<false><<<grid, kThreads, 0, s>>>(grad, n, inv_scale, partial, found_inf, unscaled_out);
  JX_CHECK_LAUNCH("jx_grad_stats");
  return JX_OK;
}

extern "C" int jx_grad_finalize(const float* partial, int nparts, float max_norm, float* out, jx_stream_t stream) {
  JX_CHECK_ARG(partial && out && nparts > 0, "jx_grad_finalize: bad argument");
  grad_finalize_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(partial, nparts, max_norm, out);
  JX_CHECK_LAUNCH("jx_grad_finalize");
  return JX_OK;
}

extern "C" int jx_adamw_step(float* p, const void* grad, int grad_is_f16, float* m, float* v, void* p16, int64_t n,
                             const float* inv_scale, const float* clip, const float* found_inf, float* step_state,
                             float lr, float beta1, float beta2, float eps, float weight_decay, jx_stream_t stream) {
  JX_CHECK_ARG(p && grad && m && v && step_state && n > 0, "jx_adamw_step: bad argument");
  JX_CHECK_ARG(aligned16(p) && aligned16(grad) && aligned16(m) && aligned16(v) && (!p16 || ((uintptr_t)p16 & 7) == 0),
               "jx_adamw_step: buffers must be 16-byte aligned (p16 8-byte)");
  AdamHyper h;
  h.lr = lr;
  h.beta1 = beta1;
  h.beta2 = beta2;
  h.eps = eps;
  h.wd = weight_decay;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  adamw_prepare_kernel<<<1, 1, 0, s>>>(step_state, found_inf, (double)beta1, (double)beta2);
  JX_CHECK_LAUNCH("jx_adamw_step: prepare");
  const int grid = blocks_for(n);
  __half* ph = static_cast<__half*>(p16);
  if (grad_is_f16)
    adamw_kernel<true><<<grid, kThreads, 0, s>>>(p, grad, m, v, ph, n, inv_scale, clip, found_inf, step_state, h);
  else
    adamw_kernel<false><<<grid, kThreads, 0, s>>>(p, grad, m, v, ph, n, inv_scale, clip, found_inf, step_state, h);
  JX_CHECK_LAUNCH("jx_adamw_step");
  return JX_OK;
}

extern "C" int jx_scaler_update(float* scale, int* growth_tracker, const float* found_inf, float growth_factor,
                                float backoff_factor, int growth_interval, jx_stream_t stream) {
  JX_CHECK_ARG(scale && growth_tracker && found_inf && growth_interval > 0, "jx_scaler_update: bad argument");
  scaler_update_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(scale, growth_tracker, found_inf,
                                                                          growth_factor, backoff_factor,
                                                                          growth_interval);
  JX_CHECK_LAUNCH("jx_scaler_update");
  return JX_OK;
}

extern "C" int jx_cast_f32_f16(const float* src, void* dst16, int64_t n, jx_stream_t stream) {
  JX_CHECK_ARG(src && dst16 && n > 0 && aligned16(src) && ((uintptr_t)dst16 & 7) == 0, "jx_cast_f32_f16: bad argument");
  cast_kernel<<<blocks_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(src, static_cast<__half*>(dst16),
                                                                                       n);
  JX_CHECK_LAUNCH("jx_cast_f32_f16");
  return JX_OK;
}

extern "C" int jx_transpose_f16(const void* src, void* dst, int64_t rows, int64_t cols, jx_stream_t stream) {
  JX_CHECK_ARG(src && dst && rows > 0 && cols > 0, "jx_transpose_f16: bad argument");
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(src), static_cast<__half*>(dst), rows, cols);
  JX_CHECK_LAUNCH("jx_transpose_f16");
  return JX_OK;
}
