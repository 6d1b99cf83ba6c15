// Token embedding gather / scatter-add and the cross-entropy kernels over
// fp16 logits.
//
// Embedding: Midstream-LLM src/jishui/model_torch.py:89-93 (fp32 table row,
// cast to the fp16 autocast dtype; the fp16 table copy holds exactly those
// values). Backward accumulates the fp16 row gradients into the fp32 table
// gradient, which the tied head's dE also lands in (model_torch.py:98).
//
// Cross-entropy: model_torch.py:102-104, F.cross_entropy(logits.float(), t)
// with mean reduction: per row lse = max + log(sum exp(x - max)), loss = lse -
// x[target]; the backward writes f16((softmax - onehot) * dloss / count) over
// the logits in place, which is what the `.float()` cast's backward hands the
// fp16 head GEMM.
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace ec {

constexpr int kWarps = 8;

__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, int64_t ntok, const __half* __restrict__ table,
                                 int64_t vocab, int cols, __half* __restrict__ out, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (t >= ntok) return;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && lane == 0 && status) atomicExch(status, kStatusEmbedBadId);
  for (int c = lane * 8; c < cols; c += 256) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (ok) v = *reinterpret_cast<const uint4*>(table + id * cols + c);
    *reinterpret_cast<uint4*>(out + t * cols + c) = v;
  }
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, int64_t ntok, const __half* __restrict__ dout,
                                 int64_t vocab, int cols, float* __restrict__ dtable) {
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (t >= ntok) return;
  const int64_t id = ids[t];
  if (id < 0 || id >= vocab) return;
  for (int c = lane * 4; c < cols; c += 128) {
    const __half2* src = reinterpret_cast<const __half2*>(dout + t * cols + c);
    const float2 a = __half22float2(src[0]);
    const float2 b = __half22float2(src[1]);
    atomicAdd(reinterpret_cast<float4*>(dtable + id * cols + c), make_float4(a.x, a.y, b.x, b.y));
  }
}

// Loss of one row from its log-sum-exp and target. A target outside [0, vocab) that is not ignore_index
// (torch's cross_entropy rejects it) gives a NaN loss, so the mean loss is NaN and the trainer refuses the
// update, and records kStatusCeBadTarget in the device status word; the backward gives such a row no
// gradient (ce_target_valid).
__device__ __forceinline__ bool ce_target_valid(int64_t t, int vocab) { return t >= 0 && t < vocab; }

__device__ __forceinline__ float target_loss(int64_t t, int64_t ignore_index, int vocab, float lse_row,
                                             const __half* row_logits, int* status) {
  if (t == ignore_index) return 0.f;
  if (!ce_target_valid(t, vocab)) {
    if (status) atomicExch(status, kStatusCeBadTarget);
    return __int_as_float(0x7fc00000);
  }
  return lse_row - __half2float(row_logits[t]);
}

// One warp per row: online max / sum-of-exp over the row with 16-byte loads.
__global__ void ce_fwd_kernel(const __half* __restrict__ logits, int64_t rows, int vocab, int64_t ld,
                              const int64_t* __restrict__ targets, int64_t ignore_index, float* __restrict__ lse,
                              float* __restrict__ row_loss, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int nvec = vocab / 8;
  for (int i = lane; i < nvec; i += 32) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + i * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    float bm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) bm = fmaxf(bm, v[j]);
    if (bm > m) {
      s *= expf(m - bm);
      m = bm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += expf(v[j] - m);
  }
  for (int c = nvec * 8 + lane; c < vocab; c += 32) {
    const float v = __half2float(x[c]);
    if (v > m) {
      s *= expf(m - v);
      m = v;
    }
    s += expf(v - m);
  }
  const float gm = warp_max(m);
  s = (m == -INFINITY) ? 0.f : s * expf(m - gm);
  s = warp_sum(s);
  if (lane == 0) {
    const float l = gm + logf(s);
    lse[row] = l;
    row_loss[row] = target_loss(targets[row], ignore_index, vocab, l, x, status);
  }
}

// The same statistics from per-block partials: the head GEMM (kHeadCE epilogue) leaves, for every row and
// 128-column block b, (m_b, s_b) = (max, sum exp(v - m_b)) of the fp16 logits; one warp per row merges them
// (lse = M + log sum_b s_b exp(m_b - M)) and reads the target's logit, so the logits are not read again.
__global__ void ce_fwd_parts_kernel(const float2* __restrict__ parts, int nblk, const __half* __restrict__ logits,
                                    int64_t rows, int vocab, int64_t ld, const int64_t* __restrict__ targets,
                                    int64_t ignore_index, float* __restrict__ lse, float* __restrict__ row_loss,
                                    int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float2* pr = parts + row * nblk;
  float m = -INFINITY, s = 0.f;
  for (int b = lane; b < nblk; b += 32) {
    const float2 q = pr[b];
    if (q.y == 0.f) continue;
    const float nm = fmaxf(m, q.x);
    s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + q.y * expf(q.x - nm);
    m = nm;
  }
  const float gm = warp_max(m);
  s = (m == -INFINITY) ? 0.f : s * expf(m - gm);
  s = warp_sum(s);
  if (lane == 0) {
    const float l = gm + logf(s);
    lse[row] = l;
    row_loss[row] = target_loss(targets[row], ignore_index, vocab, l, logits + row * ld, status);
  }
}

// Deterministic single-block sum of the per-row losses and of counted rows.
__global__ void ce_loss_kernel(const float* __restrict__ row_loss, const int64_t* __restrict__ targets,
                               int64_t ignore_index, int64_t rows, float* __restrict__ out, int accumulate) {
  __shared__ float s_sum[32], s_cnt[32];
  float sum = 0.f, cnt = 0.f;
  for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
    sum += row_loss[i];
    cnt += (targets[i] != ignore_index) ? 1.f : 0.f;
  }
  sum = warp_sum(sum);
  cnt = warp_sum(cnt);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    s_sum[warp] = sum;
    s_cnt[warp] = cnt;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    sum = lane < nw ? s_sum[lane] : 0.f;
    cnt = lane < nw ? s_cnt[lane] : 0.f;
    sum = warp_sum(sum);
    cnt = warp_sum(cnt);
    if (lane == 0) {
      const float t = accumulate ? out[0] + sum : sum;
      const float c = accumulate ? out[1] + cnt : cnt;
      out[0] = t;
      out[1] = c;
      out[2] = t / c;
    }
  }
}

__global__ void ce_bwd_kernel(__half* __restrict__ logits, int64_t rows, int vocab, int64_t ld,
                              const int64_t* __restrict__ targets, int64_t ignore_index, const float* __restrict__ lse,
                              const float* __restrict__ grad_loss, const float* __restrict__ count) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  __half* x = logits + row * ld;
  const int64_t t = targets[row];
  const float cnt = *count;
  const float g = (t == ignore_index || !ce_target_valid(t, vocab) || cnt <= 0.f) ? 0.f : (*grad_loss) / cnt;
  const float l = lse[row];
  const int nvec = vocab / 8;
  for (int i = lane; i < nvec; i += 32) {
    uint4 raw = *reinterpret_cast<const uint4*>(x + i * 8);
    __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(h[j]);
      const int c0 = i * 8 + 2 * j;
      float a = expf(f.x - l) - (c0 == t ? 1.f : 0.f);
      float b = expf(f.y - l) - (c0 + 1 == t ? 1.f : 0.f);
      h[j] = __floats2half2_rn(a * g, b * g);
    }
    *reinterpret_cast<uint4*>(x + i * 8) = raw;
  }
  for (int c = nvec * 8 + lane; c < vocab; c += 32) {
    const float v = __half2float(x[c]);
    x[c] = __float2half_rn((expf(v - l) - (c == t ? 1.f : 0.f)) * g);
  }
}

}  // namespace ec
}  // namespace jx

using namespace jx;
using namespace jx::ec;

extern "C" int jx_embed_fwd(const int64_t* ids, int64_t ntok, const void* table16, int64_t vocab, int cols,
                            void* out16, jx_stream_t stream) {
  JX_CHECK_ARG(ids && table16 && out16 && ntok > 0 && vocab > 0, "jx_embed_fwd: bad argument");
  JX_CHECK_ARG(cols % 8 == 0 && aligned16(table16) && aligned16(out16), "jx_embed_fwd: cols%%8 and 16B alignment required");
  const unsigned grid = (unsigned)((ntok + kWarps - 1) / kWarps);
  embed_fwd_kernel<<<grid, kWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ids, ntok, static_cast<const __half*>(table16), vocab, cols, static_cast<__half*>(out16), status_ptr());
  JX_CHECK_LAUNCH("jx_embed_fwd");
  return JX_OK;
}

extern "C" int jx_embed_bwd(const int64_t* ids, int64_t ntok, const void* dout16, int64_t vocab, int cols,
                            float* dtable, jx_stream_t stream) {
  JX_CHECK_ARG(ids && dout16 && dtable && ntok > 0 && vocab > 0, "jx_embed_bwd: bad argument");
  JX_CHECK_ARG(cols % 4 == 0 && ((uintptr_t)dtable & 15) == 0 && ((uintptr_t)dout16 & 7) == 0,
               "jx_embed_bwd: cols%%4 and alignment required");
  const unsigned grid = (unsigned)((ntok + kWarps - 1) / kWarps);
  embed_bwd_kernel<<<grid, kWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ids, ntok, static_cast<const __half*>(dout16), vocab, cols, dtable);
  JX_CHECK_LAUNCH("jx_embed_bwd");
  return JX_OK;
}

extern "C" int jx_ce_fwd(const void* logits16, int64_t rows, int vocab, int64_t ld, const int64_t* targets,
                         int64_t ignore_index, float* lse, float* row_loss, jx_stream_t stream) {
  JX_CHECK_ARG(logits16 && targets && lse && row_loss && rows > 0 && vocab > 0, "jx_ce_fwd: bad argument");
  JX_CHECK_ARG(ld % 8 == 0 && aligned16(logits16), "jx_ce_fwd: ld%%8 and 16B alignment required");
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  ce_fwd_kernel<<<grid, kWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(logits16), rows, vocab, ld, targets, ignore_index, lse, row_loss, status_ptr());
  JX_CHECK_LAUNCH("jx_ce_fwd");
  return JX_OK;
}

extern "C" int jx_ce_fwd_parts(const void* parts, int nblk, const void* logits16, int64_t rows, int vocab, int64_t ld,
                               const int64_t* targets, int64_t ignore_index, float* lse, float* row_loss,
                               jx_stream_t stream) {
  JX_CHECK_ARG(parts && logits16 && targets && lse && row_loss && rows > 0 && vocab > 0 && nblk == (vocab + 127) / 128,
               "jx_ce_fwd_parts: bad argument (nblk must be ceil(vocab / 128))");
  JX_CHECK_ARG(((uintptr_t)parts & 7) == 0, "jx_ce_fwd_parts: parts must be 8-byte aligned");
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  ce_fwd_parts_kernel<<<grid, kWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const float2*>(parts), nblk, static_cast<const __half*>(logits16), rows, vocab, ld, targets,
      ignore_index, lse, row_loss, status_ptr());
  JX_CHECK_LAUNCH("jx_ce_fwd_parts");
  return JX_OK;
}

extern "C" int jx_ce_loss(const float* row_loss, const int64_t* targets, int64_t ignore_index, int64_t rows,
                          float* loss_sum_count, int accumulate, jx_stream_t stream) {
  JX_CHECK_ARG(row_loss && targets && loss_sum_count && rows > 0, "jx_ce_loss: bad argument");
  ce_loss_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(row_loss, targets, ignore_index, rows,
                                                                        loss_sum_count, accumulate);
  JX_CHECK_LAUNCH("jx_ce_loss");
  return JX_OK;
}

extern "C" int jx_ce_bwd(void* logits16, int64_t rows, int vocab, int64_t ld, const int64_t* targets,
                         int64_t ignore_index, const float* lse, const float* grad_loss, const float* count,
                         jx_stream_t stream) {
  JX_CHECK_ARG(logits16 && targets && lse && grad_loss && count && rows > 0 && vocab > 0, "jx_ce_bwd: bad argument");
  JX_CHECK_ARG(ld % 8 == 0 && aligned16(logits16), "jx_ce_bwd: ld%%8 and 16B alignment required");
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  ce_bwd_kernel<<<grid, kWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(logits16), rows, vocab, ld, targets, ignore_index, lse, grad_loss, count);
  JX_CHECK_LAUNCH("jx_ce_bwd");
  return JX_OK;
}
