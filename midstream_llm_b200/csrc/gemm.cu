// Persistent tcgen05 GEMM for the Jishui decoder's dense contractions.
//
// acc[m][n] = sum_k A[m][k] * B[n][k]; fp16 operands staged by TMA into
// 128B-swizzled shared memory, fp32 accumulators in tensor memory (TMEM).
// One CTA per SM (persistent), 320 threads:
//   warp 0      TMA producer (one elected lane) filling a 4-stage ring,
//   warp 1      TMEM allocator + MMA issuer (one elected lane),
//   warps 2..9  epilogue: tcgen05.ld from TMEM -> fused math -> global stores
//               (two warps per TMEM lane quarter, each on half of the columns).
// The accumulator is double-buffered in TMEM (2 x 256 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Both operands may be K-major or MN-major in global memory; MN-major
// operands (the dgrad / wgrad products of backward) are consumed directly
// through the descriptor's major bit instead of being transposed in HBM.
//
// Fused epilogues (reference call sites in Midstream-LLM):
//   kF16      plain / residual add         model_torch.py:49,60,72-73,98
//   kHeadCE   tied head (plain fp16 logits) + per-(row, 128-column block) max and sum of exp of
//             the fp16 logits, the partial statistics of F.cross_entropy (model_torch.py:102-104)
//   kRope     q|k|v projection + RoPE      model_torch.py:18-25,41-44
//   kSwigluF  gate|up projection + SwiGLU  model_torch.py:59-60
//   kSwigluB  down dgrad + SwiGLU backward (autograd of model_torch.py:60)
//   kWgrad    weight gradient in f32, rounded through f16 as an fp16
//             autocast Linear's weight gradient is before it reaches .grad
#include <math.h>
#include <stdio.h>

#include <mutex>

#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer warp + MMA warp + epilogue warps
constexpr uint32_t kABytes = BM * BK * 2;  // 16 KiB
constexpr uint32_t kBBytes = BN * BK * 2;  // 32 KiB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kStageOutBytes = 32 * 128;  // one 32-row x 64-col fp16 output sub-tile per epilogue warp
constexpr size_t kSmemBytes = 1024 /*align slack*/ + STAGES * kStageBytes + kEpiWarps * kStageOutBytes + 256 /*barriers*/;

enum Epi : int { kF16 = 0, kRope = 1, kSwigluF = 2, kSwigluB = 3, kWgrad = 4, kHeadCE = 5 };

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, num_kb;
  int swiglu_F;  // kSwigluF: row offset of the up half inside B; kSwigluB: F
  // outputs
  __half* C;
  int64_t ldc;
  const __half* resid;
  int64_t ld_resid;
  __half* out1;
  __half* out2;
  int64_t ld_out;
  const __half* aux0;
  const __half* aux1;
  int64_t ld_aux;
  const float* rope_cos;
  const float* rope_sin;
  int rope_seq;
  int rope_cols;
  float2* ce_parts;  // kHeadCE: [M][ce_nblk] (max, sum exp(v - max)) of each 128-column block
  int ce_nblk;
  int rope_tma;  // kRope, 2-SM: cos / sin rows of a warp read as one TMA box each (rope_seq % 32 == 0)
  float* G;
  int64_t ldg;
  int accumulate;
  float* ws;
  int* status;
  long long wait_budget;  // clock64 cycles a barrier wait may take before the kernel gives up (~2 s)
  int skip_loads;         // test hook (jx_gemm_wait_test): the producer issues no loads
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, const Params& p,
                                         int code) {
  const long long start = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*abort_flag) return false;
      if (clock64() - start > p.wait_budget) {
        *abort_flag = 1;
        if (p.status) atomicExch(p.status, code);
        return false;
      }
    }
  }
}

// Warp-wide wait where only lane 0 polls (all 32 lanes active); the accumulator
// it guards lives in TMEM, read after tcgen05.fence::after_thread_sync.
__device__ __forceinline__ bool warp_wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              const Params& p, int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, abort_flag, p, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& mb, int& nb, int& s) {
  const int per_split = p.tiles_m * p.tiles_n;
  s = t / per_split;
  int tt = t - s * per_split;
  // Grouped raster: 16 M-blocks share each sweep over N for L2 reuse of B.
  constexpr int GM = 16;
  const int group_span = GM * p.tiles_n;
  const int g = tt / group_span;
  const int r = tt - g * group_span;
  const int rows = min(GM, p.tiles_m - g * GM);
  mb = g * GM + r % rows;
  nb = r / rows;
}

__device__ __forceinline__ float h2f_round(float x) { return __half2float(__float2half_rn(x)); }

// Round a and b to fp16 and back (round to nearest even), two values per packed conversion.
__device__ __forceinline__ void round2(float& a, float& b) {
  const float2 f = __half22float2(__floats2half2_rn(a, b));
  a = f.x;
  b = f.y;
}

template <int N>
__device__ __forceinline__ void round_all(float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 2) round2(v[i], v[i + 1]);
}

// Raw 16-byte loads of 32 consecutive fp16 values of one row (zero outside [M, N)).
__device__ __forceinline__ void load_raw32(const __half* base, int64_t ld, int row, int col, int M, int N,
                                           uint4 (&r)[4]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (row < M && col + g * 8 + 8 <= N)
      r[g] = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)row * ld + col + g * 8));
    else
      r[g] = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void unpack32(const uint4 (&r)[4], float (&v)[32]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const __half2* h = reinterpret_cast<const __half2*>(&r[g]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(h[j]);
      v[g * 8 + 2 * j] = f.x;
      v[g * 8 + 2 * j + 1] = f.y;
    }
  }
}

// Store 32 consecutive fp32 values of row `row` starting at column `col` as fp16.
__device__ __forceinline__ void store_row32_f16(__half* base, int64_t ld, int row, int col, int M, int N,
                                                const float (&v)[32]) {
  if (row >= M) return;
  __half* dst = base + (int64_t)row * ld + col;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (col + g * 8 + 8 <= N) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 h = __floats2half2_rn(v[g * 8 + 2 * j], v[g * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(dst + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void to_f32(const uint32_t (&r)[32], float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// silu(x) = x / (1 + e^-x) with the fast exp and division; the result is rounded
// to fp16, where the difference to the correctly rounded fp32 form is below half an
// fp16 ulp except at rounding ties. (The backward's sigmoid: swiglu_bwd_pair.)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// SwiGLU backward of two adjacent columns with autograd's fp16 rounding points:
//   d = f16(dact), ds = f16(d * u), dup = f16(d * f16(g * sig)),
//   dgate = f16(f32(ds) * sig * (1 + g * (1 - sig))), sig = 1 / (1 + e^-g) in fp32.
// A product of two fp16 values is exact in fp32, so rounding it once to fp16 is the fp16
// multiply (__hmul2_rn); the fp32 chain of dgate uses paired, non-contracted operations.
// g2 / u2 / dg2 / du2 hold fp16 pairs (column c in the low half, c + 1 in the high half).
__device__ __forceinline__ void swiglu_bwd_pair(float d0, float d1, uint32_t g2, uint32_t u2, uint32_t& dg2,
                                                uint32_t& du2) {
  const __half2 dh = __floats2half2_rn(d0, d1);
  const __half2 gh = *reinterpret_cast<const __half2*>(&g2);
  const __half2 uh = *reinterpret_cast<const __half2*>(&u2);
  const float2 one = make_float2(1.0f, 1.0f);
  const float2 g = __half22float2(gh);
  const float2 t = __fmul2_rn(g, make_float2(-kLog2e, -kLog2e));
  const float2 y = __fadd2_rn(make_float2(ex2_approx(t.x), ex2_approx(t.y)), one);
  const float2 sig = make_float2(rcp_approx(y.x), rcp_approx(y.y));
  const __half2 du = __hmul2_rn(dh, __float22half2_rn(__fmul2_rn(g, sig)));
  const float2 ds = __half22float2(__hmul2_rn(dh, uh));
  const float2 om = __ffma2_rn(sig, make_float2(-1.0f, -1.0f), one);  // 1 - sig, rounded once
  const float2 q = __fadd2_rn(one, __fmul2_rn(g, om));
  const __half2 dg = __float22half2_rn(__fmul2_rn(__fmul2_rn(ds, sig), q));
  dg2 = *reinterpret_cast<const uint32_t*>(&dg);
  du2 = *reinterpret_cast<const uint32_t*>(&du);
}

// Word i (fp16 pair i) of 32 consecutive fp16 values held as four 16-byte vectors.
__device__ __forceinline__ uint32_t pair_word(const uint4 (&q)[4], int i) {
  const uint4& v = q[i >> 2];
  return (i & 3) == 0 ? v.x : (i & 3) == 1 ? v.y : (i & 3) == 2 ? v.z : v.w;
}

// TMA store of one staged [32 rows x 64 cols] fp16 sub-tile (128B-swizzled).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Per-warp staging of output sub-tiles: thread `lane` owns staging row `lane`
// (tile row 32q + lane); 64 fp16 columns = 8 16-byte chunks, XOR-swizzled by
// row as the 128B-swizzled TMA box expects. One lane issues the TMA store.
struct Stager {
  uint8_t* buf;
  int lane;
  __device__ __forceinline__ void begin() {  // the previous store has finished reading the buffer
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }
  __device__ __forceinline__ void put32(int part, const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __half2 h = __floats2half2_rn(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t*>(&h);
      }
      const int c = part * 4 + j;
      *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  // 32 values already packed as fp16 pairs (16 words).
  __device__ __forceinline__ void put_packed(int part, const uint32_t (&w)[16]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = part * 4 + j;
      *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
  }
  __device__ __forceinline__ void flush(const CUtensorMap* map, int x, int y) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, buf, x, y);
      bulk_commit();
    }
  }
  // 32 fp32 values of this lane's row (a 32 x 32 fp32 box, 128B-swizzled).
  __device__ __forceinline__ void put_f32(const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
  // Adds the staged box to global memory (TMA reduce-add; out-of-range rows / columns are clipped).
  __device__ __forceinline__ void flush_add(const CUtensorMap* map, int x, int y) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                       reinterpret_cast<uint64_t>(map)),
                   "r"(smem_u32(buf)), "r"(x), "r"(y)
                   : "memory");
      bulk_commit();
    }
  }
};

// Per-warp TMA staging of the epilogue's row-wise inputs (gate and up boxes of 32 rows x 64
// columns, 128B-swizzled): one mbarrier, its phase, and the two tensor maps.
constexpr uint32_t kAuxWarpBytes = 2 * 32 * 64 * 2;  // gate + up box of 32 rows x 64 fp16 columns

struct AuxTma {
  uint8_t* buf;
  uint64_t* bar;
  uint32_t phase;
  const CUtensorMap* gate;
  const CUtensorMap* up;
  volatile int* abort_flag;
  __device__ __forceinline__ void issue(int x, int y) {  // lane 0 only
    fence_proxy_async_smem();  // earlier generic reads of the buffer happen before the refill
    mbar_expect_tx(bar, kAuxWarpBytes);
    tma_load_2d(buf, gate, bar, x, y);
    tma_load_2d(buf + kAuxWarpBytes / 2, up, bar, x, y);
  }
};

struct OutMaps {
  const CUtensorMap* c0;
  const CUtensorMap* c1;
  const CUtensorMap* c2;
};

// Epilogue of one 128 x 256 accumulator tile. Eight warps drain it: warp
// quarter q (= warp % 4) owns TMEM lanes / tile rows [32q, 32q+32), and half
// h owns half of the columns (for kSwigluF: half of the gate and of the up
// columns; for kRope: two of the four heads). Each thread owns one row; fp16
// outputs go out through per-warp shared-memory staging and TMA stores
// (out-of-range rows/columns are clipped by the tensor map), the fp32
// weight-gradient output with direct 16-byte accesses.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, const OutMaps& om, Stager& st, uint32_t tacc,
                                              int quarter, int half, int lane, int mb, int nb, int split, AuxTma* aux = nullptr) {
  const int row = mb * BM + quarter * 32 + lane;
  const int yrow = mb * BM + quarter * 32;  // first row of this warp's TMA boxes
  const uint32_t tl = tacc + (static_cast<uint32_t>(quarter * 32) << 16);
  if constexpr (EPI == kF16 || EPI == kHeadCE || EPI == kWgrad) {
    float ce_m = -INFINITY, ce_s = 0.f;  // kHeadCE: running statistics of this thread's 128-column block
#pragma unroll 1
    for (int cp = 0; cp < 2; ++cp) {
      const int c0 = half * 4 + cp * 2;  // first of two 32-column chunks
      const int col0 = nb * BN + c0 * 32;
      if (col0 >= p.N) break;
      uint32_t r0[32], r1[32];
      tmem_ld32(tl + c0 * 32, r0);
      tmem_ld32(tl + c0 * 32 + 32, r1);
      uint4 q0[4], q1[4];
      if (EPI == kF16 && p.resid) {
        load_raw32(p.resid, p.ld_resid, row, col0, p.M, p.N, q0);
        load_raw32(p.resid, p.ld_resid, row, col0 + 32, p.M, p.N, q1);
      }
      tmem_ld_wait();
      float v0[32], v1[32];
      to_f32(r0, v0);
      to_f32(r1, v1);
      if constexpr (EPI == kHeadCE) {
        // The logits are stored as fp16: the statistics are taken over the rounded values, columns past N
        // (zero accumulators) excluded; sum exp(v - m) = sum 2^((v - m) log2 e).
        round_all(v0);
        round_all(v1);
        const int nv0 = min(32, p.N - col0), nv1 = min(32, p.N - col0 - 32);
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < nv0) m = fmaxf(m, v0[i]);
          if (i < nv1) m = fmaxf(m, v1[i]);
        }
        const float ml = m * kLog2e;
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < nv0) sum += ex2_approx(fmaf(v0[i], kLog2e, -ml));
          if (i < nv1) sum += ex2_approx(fmaf(v1[i], kLog2e, -ml));
        }
        const float nm = fmaxf(ce_m, m);
        ce_s = (ce_m == -INFINITY ? 0.f : ce_s * ex2_approx((ce_m - nm) * kLog2e)) + sum * ex2_approx((m - nm) * kLog2e);
        ce_m = nm;
      }
      if constexpr (EPI == kF16 || EPI == kHeadCE) {
        if (p.resid) {
          float a[32], b[32];
          unpack32(q0, a);
          unpack32(q1, b);
          round_all(v0);
          round_all(v1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v0[i] = a[i] + v0[i];
            v1[i] = b[i] + v1[i];
          }
        }
        st.begin();
        st.put32(0, v0);
        st.put32(1, v1);
        st.flush(om.c0, col0, yrow);
      } else {
        if (p.splits > 1) {
          // Split-K: this split's fp32 partial is added into the one shared workspace by TMA reduce-add
          // (32 x 32 boxes through the warp's staging buffer), so the partial sums meet in L2.
          (void)split;
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            st.begin();
            st.put_f32(part ? v1 : v0);
            st.flush_add(om.c0, col0 + part * 32, yrow);
          }
          continue;
        }
        if (row >= p.M) continue;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int col = col0 + part * 32;
          const float* v = part ? v1 : v0;
          {
            float* dst = p.G + (int64_t)row * p.ldg + col;
            float vr[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) vr[i] = v[i];
            round_all(vr);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              if (col + g * 4 + 4 <= p.N) {
                float4 o = make_float4(vr[g * 4], vr[g * 4 + 1], vr[g * 4 + 2], vr[g * 4 + 3]);
                if (p.accumulate) {
                  const float4 old = *reinterpret_cast<const float4*>(dst + g * 4);
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                *reinterpret_cast<float4*>(dst + g * 4) = o;
              }
            }
          }
        }
      }
    }
    if constexpr (EPI == kHeadCE) {
      const int blk_col = nb * BN + half * 128;
      if (row < p.M && blk_col < p.N) p.ce_parts[(int64_t)row * p.ce_nblk + blk_col / 128] = make_float2(ce_m, ce_s);
    }
  } else if constexpr (EPI == kRope) {
    const int pos = p.rope_seq > 0 ? row % p.rope_seq : 0;
    // Staged: the caller requested this warp's cos / sin box (rows yrow % rope_seq .. +31, 128B-swizzled).
    if (aux && nb * BN + half * 128 < p.rope_cols) {
      if (!warp_wait_bar(aux->bar, aux->phase, aux->abort_flag, p, kStatusGemmEpilogueWait)) return;
      aux->phase ^= 1u;
    }
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      const int h = half * 2 + hh;
      const int col = nb * BN + h * 64;
      if (col >= p.N) break;
      uint32_t ra[32], rb[32];
      tmem_ld32(tl + h * 64, ra);
      tmem_ld32(tl + h * 64 + 32, rb);
      tmem_ld_wait();
      float a[32], b[32];
      to_f32(ra, a);
      to_f32(rb, b);
      if (col < p.rope_cols && row < p.M) {
        const float4* cs = reinterpret_cast<const float4*>(p.rope_cos + (int64_t)pos * 32);
        const float4* sn = reinterpret_cast<const float4*>(p.rope_sin + (int64_t)pos * 32);
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          float4 c4, s4;
          if (aux) {
            const int off = lane * 128 + ((i4 ^ (lane & 7)) << 4);
            c4 = *reinterpret_cast<const float4*>(aux->buf + off);
            s4 = *reinterpret_cast<const float4*>(aux->buf + kAuxWarpBytes / 2 + off);
          } else {
            c4 = __ldg(cs + i4);
            s4 = __ldg(sn + i4);
          }
          const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = i4 * 4 + j;
            float x0 = a[i], x1 = b[i];
            round2(x0, x1);
            a[i] = __fsub_rn(__fmul_rn(x0, cc[j]), __fmul_rn(x1, ss[j]));
            b[i] = __fadd_rn(__fmul_rn(x0, ss[j]), __fmul_rn(x1, cc[j]));
          }
        }
      }
      st.begin();
      st.put32(0, a);
      st.put32(1, b);
      st.flush(om.c0, col, yrow);
    }
    if (aux) __syncwarp();  // every lane's box reads done before the next tile's refill
  } else if constexpr (EPI == kSwigluF) {
    const int F = p.swiglu_F;
    const int col = nb * 128 + half * 64;  // 64 gate columns (and the matching up columns)
    if (col < F) {
      uint32_t rg0[32], rg1[32], ru0[32], ru1[32];
      tmem_ld32(tl + half * 64, rg0);
      tmem_ld32(tl + half * 64 + 32, rg1);
      tmem_ld32(tl + 128 + half * 64, ru0);
      tmem_ld32(tl + 128 + half * 64 + 32, ru1);
      tmem_ld_wait();
      float g0[32], g1[32], u0[32], u1[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        g0[i] = __uint_as_float(rg0[i]);
        g1[i] = __uint_as_float(rg1[i]);
        u0[i] = __uint_as_float(ru0[i]);
        u1[i] = __uint_as_float(ru1[i]);
      }
      round_all(g0);
      round_all(g1);
      round_all(u0);
      round_all(u1);
      st.begin();
      st.put32(0, g0);
      st.put32(1, g1);
      st.flush(om.c0, col, yrow);
      st.begin();
      st.put32(0, u0);
      st.put32(1, u1);
      st.flush(om.c1, col, yrow);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        g0[i] = silu_f(g0[i]);
        g1[i] = silu_f(g1[i]);
      }
      round_all(g0);
      round_all(g1);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        g0[i] = __fmul_rn(g0[i], u0[i]);
        g1[i] = __fmul_rn(g1[i], u1[i]);
      }
      st.begin();
      st.put32(0, g0);
      st.put32(1, g1);
      st.flush(om.c2, col, yrow);
    }
  } else if constexpr (EPI == kSwigluB) {
    // The 1-SM kernel's form (the 2-SM kernel pipelines its own, swiglu_bwd_epilogue2): the gate / up
    // rows straight from global memory, 64-column outputs through the warp's staging buffer.
    const int F = p.swiglu_F;
#pragma unroll 1
    for (int cp = 0; cp < 2; ++cp) {
      const int c0 = half * 4 + cp * 2;
      const int col0 = nb * BN + c0 * 32;
      if (col0 >= F) break;
      uint32_t pdg[2][16], pdu[2][16];
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t r[32];
        tmem_ld32(tl + c0 * 32 + part * 32, r);
        uint4 gq[4], uq[4];
        load_raw32(p.aux0, p.ld_aux, row, col0 + part * 32, p.M, F, gq);
        load_raw32(p.aux1, p.ld_aux, row, col0 + part * 32, p.M, F, uq);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          swiglu_bwd_pair(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]), pair_word(gq, i), pair_word(uq, i),
                          pdg[part][i], pdu[part][i]);
      }
      st.begin();
      st.put_packed(0, pdg[0]);
      st.put_packed(1, pdg[1]);
      st.flush(om.c0, col0, yrow);
      st.begin();
      st.put_packed(0, pdu[0]);
      st.put_packed(1, pdu[1]);
      st.flush(om.c1, col0, yrow);
    }
  }
  (void)aux;
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC0, const __grid_constant__ CUtensorMap tmC1,
                const __grid_constant__ CUtensorMap tmC2, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kABytes;
  uint8_t* sOut = smem + STAGES * kStageBytes;  // kEpiWarps x 4 KiB output staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + kEpiWarps * kStageOutBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n * p.splits;

  if (warp == 0) {
    if (lane == 0 && !p.skip_loads) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb, s;
        tile_coords(p, t, mb, nb, s);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t stage = it % STAGES;
          const uint32_t parity = ((it / STAGES) & 1u) ^ 1u;
          if (!wait_bar(&empty[stage], parity, abort_flag, p, kStatusGemmProducerWait)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], kStageBytes);
          uint8_t* a_dst = smA + stage * kABytes;
          uint8_t* b_dst = smB + stage * kBBytes;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, mb * BM);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], mb * BM, kb * BK);
            tma_load_2d(a_dst + 8192, &tmA, &full[stage], mb * BM + 64, kb * BK);
          }
          if constexpr (!B_MN) {
            if constexpr (EPI == kSwigluF) {
              tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, nb * 128);
              tma_load_2d(b_dst + 16384, &tmB, &full[stage], kb * BK, p.swiglu_F + nb * 128);
            } else {
              tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, nb * BN);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], nb * BN + j * 64, kb * BK);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        int mb, nb, s;
        tile_coords(p, t, mb, nb, s);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int acc = local & 1;
        if (!wait_bar(&acc_empty[acc], ((local >> 1) & 1) ^ 1, abort_flag, p, kStatusGemmMmaWait)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t stage = it % STAGES;
          if (!wait_bar(&full[stage], (it / STAGES) & 1u, abort_flag, p, kStatusGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * kABytes);
          const uint32_t b_base = smem_u32(smB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
    }
  } else {
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;    // which half of the tile's columns
    Stager st{sOut + (warp - 2) * kStageOutBytes, lane};
    const OutMaps om{&tmC0, &tmC1, &tmC2};
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mb, nb, s;
      tile_coords(p, t, mb, nb, s);
      const int acc = local & 1;
      if (!warp_wait_bar(&acc_full[acc], (local >> 1) & 1, abort_flag, p, kStatusGemmEpilogueWait)) break;
      tc_fence_after();
      epilogue_tile<EPI>(p, om, st, tmem_base + acc * BN, quarter, half, lane, mb, nb, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (lane == 0) bulk_wait_all();  // outstanding output stores complete before the CTA retires
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M 256, N 256, K 16). CTA rank r holds rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile
// (half of N) in its own shared memory; the pair of tensor cores exchanges the
// B halves, and each CTA's TMEM receives its 128 rows x all 256 columns, which
// its own epilogue warps drain exactly as in the 1-SM kernel. Per k-block each
// SM therefore stages 32 KiB instead of 48 KiB, which buys a 6-stage ring.
// Protocol (one leader, CTA rank 0):
//   both producers   wait their own `empty` slot, TMA (cta_group::2 form, no
//                    multicast) into their own smem, completing on the leader's
//                    `full` barrier; only the leader arms it with the pair's bytes,
//   leader MMA       waits `full`, issues the pair MMA, commits `empty` and
//                    `acc_full` to both CTAs (commit multicast),
//   both epilogues   drain their TMEM half and arrive on the leader's `acc_empty`.
// ---------------------------------------------------------------------------
constexpr int STAGES2 = 6;
constexpr uint32_t kAHalf = 128 * BK * 2;  // 16 KiB
constexpr uint32_t kBHalf = 128 * BK * 2;  // 16 KiB
constexpr uint32_t kStage2Bytes = kAHalf + kBHalf;
// The SwiGLU-backward and RoPE epilogues read their row-wise inputs (gate / up boxes, cos / sin
// rows) through TMA into per-warp shared memory (kAuxWarpBytes per epilogue warp), paid for with a
// 4-stage ring.
template <int EPI>
__host__ __device__ constexpr bool has_aux2() { return EPI == kSwigluB || EPI == kRope; }
template <int EPI>
__host__ __device__ constexpr int stages2() { return has_aux2<EPI>() ? 4 : STAGES2; }
template <int EPI>
__host__ __device__ constexpr size_t smem2_bytes() {
  return 1024 + stages2<EPI>() * kStage2Bytes + kEpiWarps * kStageOutBytes +
         (has_aux2<EPI>() ? kEpiWarps * kAuxWarpBytes : 0) + 320;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t smem_dst, const CUtensorMap* map, uint32_t leader_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this shared offset in both CTAs of the pair once the issued MMAs complete.
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tile_coords2(const Params& p, int t, int& mb2, int& nb, int& s) {
  const int tiles_m2 = (p.tiles_m + 1) / 2;
  const int per_split = tiles_m2 * p.tiles_n;
  s = t / per_split;
  const int tt = t - s * per_split;
  constexpr int GM = 8;  // 8 pair-rows (2048 rows of A) share each sweep over N
  const int group_span = GM * p.tiles_n;
  const int g = tt / group_span;
  const int r = tt - g * group_span;
  const int rows = min(GM, tiles_m2 - g * GM);
  mb2 = g * GM + r % rows;
  nb = r / rows;
}

// SwiGLU-backward epilogue of the 2-SM kernel. Each epilogue warp walks its parts (32 rows x 32
// columns: tile columns nb*256 + half*128 + 32j, j < 4) in order across its tiles. A part's gate / up
// boxes (32 x 32 fp16 each, 64B-swizzled, 4 KiB together) land in one of the warp's two slots,
// requested two parts ahead and across tile boundaries, so the loads overlap the arithmetic of the
// parts before; dgate and dup leave through the two halves of the warp's 4 KiB staging buffer by
// two TMA stores, so a part waits only for the stores of the part before it. The accumulator is
// released once its last part is in registers.
constexpr uint32_t kSwbSlotBytes = 2 * 32 * 32 * 2;  // gate + up box of one part
static_assert(2 * kSwbSlotBytes == kAuxWarpBytes && kSwbSlotBytes == kStageOutBytes, "per-warp buffer sizes");

// This warp's first column and row in tile t, and how many of its four parts hold columns < F.
__device__ __forceinline__ void swb_coords(const Params& p, int t, int half, int quarter, uint32_t rank, int& x0,
                                           int& y, int& n) {
  int mb2, nb, s;
  tile_coords2(p, t, mb2, nb, s);
  x0 = nb * BN + half * 128;
  y = (mb2 * 2 + (int)rank) * BM + quarter * 32;
  n = min(4, max(0, (p.swiglu_F - x0 + 31) / 32));
}

// The next part a warp requests: tile t (first column x0, first row y, n parts in the warp's columns),
// part j; parts requested so far.
struct SwbCursor {
  int t, j, n, x0, y, requested;
};

__device__ __forceinline__ int swb_chunk(int lane, int c) {  // 64B swizzle: 16-byte chunk c of row `lane`
  return lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4);
}

__device__ __forceinline__ void swiglu_bwd_epilogue2(const Params& p, const CUtensorMap* gate_map,
                                                     const CUtensorMap* up_map, const CUtensorMap* dgate_map,
                                                     const CUtensorMap* dup_map, uint8_t* slots, uint64_t* slot_bars,
                                                     uint8_t* stage, uint32_t tmem_base, uint64_t* acc_full,
                                                     uint32_t leader_acc_empty0, uint32_t leader_acc_empty1,
                                                     volatile int* abort_flag, int cluster_id, int num_clusters,
                                                     int num_tiles, int half, int quarter, uint32_t rank, int lane) {
  SwbCursor rq{cluster_id, 0, 0, 0, 0, 0};
  if (rq.t < num_tiles) swb_coords(p, rq.t, half, quarter, rank, rq.x0, rq.y, rq.n);
  // Requests the next part's boxes into slot (requested & 1); the warp has finished reading that slot.
  auto request = [&]() {
    while (rq.j >= rq.n) {
      if (rq.t >= num_tiles) return;
      rq.t += num_clusters;
      rq.j = 0;
      if (rq.t >= num_tiles) return;
      swb_coords(p, rq.t, half, quarter, rank, rq.x0, rq.y, rq.n);
    }
    if (lane == 0) {  // the caller has fenced the warp's generic reads of the slot against this refill
      const int sl = rq.requested & 1;
      const int x = rq.x0 + rq.j * 32;
      mbar_expect_tx(&slot_bars[sl], kSwbSlotBytes);
      tma_load_2d(slots + sl * kSwbSlotBytes, gate_map, &slot_bars[sl], x, rq.y);
      tma_load_2d(slots + sl * kSwbSlotBytes + kSwbSlotBytes / 2, up_map, &slot_bars[sl], x, rq.y);
    }
    ++rq.requested;
    ++rq.j;
  };
  request();
  request();
  int consumed = 0, local = 0;
  bool ok = true;
  for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++local) {
    const int acc = local & 1;
    if (!warp_wait_bar(&acc_full[acc], (local >> 1) & 1, abort_flag, p, kStatusGemmEpilogueWait)) break;
    tc_fence_after();
    const uint32_t tl = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
    int x0, y, nparts;
    swb_coords(p, t, half, quarter, rank, x0, y, nparts);
    bool released = false;
#pragma unroll 1
    for (int j = 0; j < nparts; ++j) {
      const int x = x0 + j * 32;
      const bool last = j == nparts - 1;
      uint32_t r[32];
      tmem_ld32(tl + (half * 4 + j) * 32, r);
      const int sl = consumed & 1;
      if (!warp_wait_bar(&slot_bars[sl], (consumed >> 1) & 1, abort_flag, p, kStatusGemmEpilogueWait)) {
        tmem_ld_wait();
        ok = false;
        break;
      }
      const uint8_t* src = slots + sl * kSwbSlotBytes;
      tmem_ld_wait();
      if (last) {  // the accumulator is in registers: the MMA may refill it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc ? leader_acc_empty1 : leader_acc_empty0);
        released = true;
      }
      if (lane == 0) bulk_wait_read_all();  // the previous part's stores have left the staging buffer
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // one 16-byte chunk (8 columns) of gate / up in, dgate / dup out
        const uint4 gq = *reinterpret_cast<const uint4*>(src + swb_chunk(lane, c));
        const uint4 uq = *reinterpret_cast<const uint4*>(src + kSwbSlotBytes / 2 + swb_chunk(lane, c));
        const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
        uint32_t dg[4], du[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = 4 * c + i;
          swiglu_bwd_pair(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]), gw[i], uw[i], dg[i], du[i]);
        }
        *reinterpret_cast<uint4*>(stage + swb_chunk(lane, c)) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
        *reinterpret_cast<uint4*>(stage + kSwbSlotBytes / 2 + swb_chunk(lane, c)) = make_uint4(du[0], du[1], du[2], du[3]);
      }
      // All lanes have read the slot and written the staging buffer: the slot is refilled (two parts
      // ahead) and the results leave, both by the async proxy.
      fence_proxy_async_smem();
      __syncwarp();
      request();
      ++consumed;
      if (lane == 0) {
        tma_store_2d(dgate_map, stage, x, y);
        tma_store_2d(dup_map, stage + kSwbSlotBytes / 2, x, y);
        bulk_commit();
      }
    }
    if (ok && !released) {  // no part of this tile in this warp's columns
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc ? leader_acc_empty1 : leader_acc_empty0);
    }
  }
  // Requests still in flight (after an abandoned wait): let them land before the CTA leaves.
  for (; consumed < rq.requested; ++consumed)
    if (lane == 0) mbar_wait(&slot_bars[consumed & 1], (consumed >> 1) & 1, nullptr, 0);
  __syncwarp();
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC0, const __grid_constant__ CUtensorMap tmC1,
                 const __grid_constant__ CUtensorMap tmC2, const __grid_constant__ CUtensorMap tmX0,
                 const __grid_constant__ CUtensorMap tmX1, const Params p) {
  constexpr int S2 = stages2<EPI>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S2 * kAHalf;
  uint8_t* sOut = smem + S2 * kStage2Bytes;
  uint8_t* sAux = sOut + kEpiWarps * kStageOutBytes;  // kSwigluB / kRope: [kEpiWarps][gate | up] or [cos | sin]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sAux + (has_aux2<EPI>() ? kEpiWarps * kAuxWarpBytes : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + S2;
  uint64_t* acc_full = bars + 2 * S2;
  uint64_t* acc_empty = bars + 2 * S2 + 2;
  uint64_t* aux_full = bars + 2 * S2 + 4;  // two per epilogue warp (kSwigluB: one per slot; kRope: the first)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S2 + 4 + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = (rank == 0);

  if (threadIdx.x == 0) {
    for (int w = 0; w < 2 * kEpiWarps; ++w) mbar_init(&aux_full[w], 1);
    for (int s = 0; s < S2; ++s) {
      mbar_init(&full[s], 1);   // leader's producer arms it; both CTAs' TMA bytes complete it
      mbar_init(&empty[s], 1);  // the leader's MMA commit arrives in both CTAs
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // epilogue warps of both CTAs (used in the leader)
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive / TMA completion
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m2 = (p.tiles_m + 1) / 2;
  const int num_tiles = tiles_m2 * p.tiles_n * p.splits;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        int mb2, nb, s;
        tile_coords2(p, t, mb2, nb, s);
        const int m0 = mb2 * 256 + rank * 128;  // this CTA's A rows
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t stage = it % S2;
          if (!wait_bar(&empty[stage], ((it / S2) & 1u) ^ 1u, abort_flag, p, kStatusGemmProducerWait)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = map_to_rank(smem_u32(&full[stage]), 0);
          if (leader) mbar_expect_tx(&full[stage], 2 * kStage2Bytes);
          const uint32_t a_dst = smem_u32(smA + stage * kAHalf);
          const uint32_t b_dst = smem_u32(smB + stage * kBHalf);
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, leader_full, kb * BK, m0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, leader_full, m0, kb * BK);
            tma_load_2d_pair(a_dst + 8192, &tmA, leader_full, m0 + 64, kb * BK);
          }
          if constexpr (!B_MN) {
            int brow;
            if constexpr (EPI == kSwigluF)
              brow = (rank == 0 ? 0 : p.swiglu_F) + nb * 128;  // CTA 0: gate rows, CTA 1: up rows
            else
              brow = nb * BN + rank * 128;
            tma_load_2d_pair(b_dst, &tmB, leader_full, kb * BK, brow);
          } else {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              tma_load_2d_pair(b_dst + j * 8192, &tmB, leader_full, nb * BN + rank * 128 + j * 64, kb * BK);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16_f32(256, BN, A_MN, B_MN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++local) {
        int mb2, nb, s;
        tile_coords2(p, t, mb2, nb, s);
        const int kb0 = s * p.kb_per_split;
        const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        const int acc = local & 1;
        if (!wait_bar(&acc_empty[acc], ((local >> 1) & 1) ^ 1, abort_flag, p, kStatusGemmMmaWait)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t stage = it % S2;
          if (!wait_bar(&full[stage], (it / S2) & 1u, abort_flag, p, kStatusGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * kAHalf);
          const uint32_t b_base = smem_u32(smB + stage * kBHalf);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma2_f16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma2_commit_both(&empty[stage]);
        }
        if (ok) umma2_commit_both(&acc_full[acc]);
      }
    }
  } else if constexpr (EPI == kSwigluB) {
    const uint32_t leader_acc_empty0 = map_to_rank(smem_u32(&acc_empty[0]), 0);
    const uint32_t leader_acc_empty1 = map_to_rank(smem_u32(&acc_empty[1]), 0);
    swiglu_bwd_epilogue2(p, &tmX0, &tmX1, &tmC0, &tmC1, sAux + (warp - 2) * kAuxWarpBytes, &aux_full[2 * (warp - 2)],
                         sOut + (warp - 2) * kStageOutBytes, tmem_base, acc_full, leader_acc_empty0, leader_acc_empty1,
                         abort_flag, cluster_id, num_clusters, num_tiles, (warp - 2) >> 2, warp & 3, rank, lane);
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    Stager st{sOut + (warp - 2) * kStageOutBytes, lane};
    const OutMaps om{&tmC0, &tmC1, &tmC2};
    const uint32_t leader_acc_empty0 = map_to_rank(smem_u32(&acc_empty[0]), 0);
    const uint32_t leader_acc_empty1 = map_to_rank(smem_u32(&acc_empty[1]), 0);
    AuxTma aux{sAux + (warp - 2) * kAuxWarpBytes, &aux_full[warp - 2], 0u, &tmX0, &tmX1, abort_flag};
    int local = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters, ++local) {
      int mb2, nb, s;
      tile_coords2(p, t, mb2, nb, s);
      const int acc = local & 1;
      if constexpr (EPI == kRope) {
        // The cos / sin rows of this warp's 32 token rows (consecutive positions).
        const int y = (mb2 * 2 + (int)rank) * BM + quarter * 32;
        if (p.rope_tma && nb * BN + half * 128 < p.rope_cols && lane == 0) aux.issue(0, y % p.rope_seq);
      }
      if (!warp_wait_bar(&acc_full[acc], (local >> 1) & 1, abort_flag, p, kStatusGemmEpilogueWait)) break;
      tc_fence_after();
      epilogue_tile<EPI>(p, om, st, tmem_base + acc * BN, quarter, half, lane, mb2 * 2 + (int)rank, nb, s,
                         (EPI == kRope && p.rope_tma) ? &aux : nullptr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc ? leader_acc_empty1 : leader_acc_empty0);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// Split-K finish for the weight gradient: G (+)= f32(f16(ws)), ws holding the sum of every split's
// partial (added by the splits' TMA reduces into the zeroed workspace).
__global__ void wgrad_reduce_kernel(const float* __restrict__ ws, int M, int N, float* __restrict__ G, int64_t ldg,
                                    int accumulate) {
  const int64_t total4 = (int64_t)M * N / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    const int row = (int)(e / N);
    const int col = (int)(e - (int64_t)row * N);
    const float4 acc = *reinterpret_cast<const float4*>(ws + e);
    float* dst = G + (int64_t)row * ldg + col;
    float4 o = make_float4(h2f_round(acc.x), h2f_round(acc.y), h2f_round(acc.z), h2f_round(acc.w));
    if (accumulate) {
      float4 old = *reinterpret_cast<float4*>(dst);
      o.x += old.x;
      o.y += old.y;
      o.z += old.z;
      o.w += old.w;
    }
    *reinterpret_cast<float4*>(dst) = o;
  }
}

// ---------------------------------------------------------------------------
// Small-M products (M <= 8, A and B K-major): C[m][n] = sum_k A[m][k] B[n][k],
// for incremental decoding. The tensor-core tiles are 128 rows high, so for a
// handful of rows the product is a weight-bandwidth problem: every CTA streams
// one pair of B rows with 16-byte loads (its warps and lanes split K),
// accumulates in fp32 for all M rows of A (L1-resident), reduces across the CTA
// and applies the same epilogue as the tiled kernel (fp16 rounding points
// included). A pair is the
// two rows an epilogue needs together: (2q, 2q+1) for the plain / residual
// epilogue, the RoPE partners (64h + c, 64h + c + 32) for q/k/v, and the gate /
// up rows (q, F + q) for SwiGLU.
// ---------------------------------------------------------------------------
constexpr int kGemvMaxM = 8;
constexpr int kGemvWarps = 4;

template <int EPI>
__device__ __forceinline__ void gemv_pair_rows(const Params& p, int q, int& r0, int& r1) {
  if constexpr (EPI == kRope) {
    r0 = (q / 32) * 64 + (q % 32);
    r1 = r0 + 32;
  } else if constexpr (EPI == kSwigluF) {
    r0 = q;
    r1 = p.swiglu_F + q;
  } else {
    r0 = 2 * q;
    r1 = 2 * q + 1;
  }
}

template <int EPI>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const __half* __restrict__ A, int64_t lda,
                                                               const __half* __restrict__ B, int64_t ldb, Params p) {
  __shared__ float red[kGemvWarps][kGemvMaxM][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x;  // one pair of B rows per CTA, K split across its warps
  int r0, r1;
  gemv_pair_rows<EPI>(p, q, r0, r1);
  float acc[kGemvMaxM][2];
#pragma unroll
  for (int m = 0; m < kGemvMaxM; ++m) acc[m][0] = acc[m][1] = 0.f;
  const __half* b0 = B + (int64_t)r0 * ldb;
  const __half* b1 = B + (int64_t)r1 * ldb;
  for (int k = (warp * 32 + lane) * 8; k < p.K; k += kGemvWarps * 256) {
    const uint4 u0 = __ldg(reinterpret_cast<const uint4*>(b0 + k));
    const uint4 u1 = __ldg(reinterpret_cast<const uint4*>(b1 + k));
    const __half2* w0 = reinterpret_cast<const __half2*>(&u0);
    const __half2* w1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
    for (int m = 0; m < kGemvMaxM; ++m) {
      if (m >= p.M) break;
      const uint4 ua = __ldg(reinterpret_cast<const uint4*>(A + (int64_t)m * lda + k));
      const __half2* xa = reinterpret_cast<const __half2*>(&ua);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = __half22float2(xa[j]), f0 = __half22float2(w0[j]), f1 = __half22float2(w1[j]);
        acc[m][0] = fmaf(x.x, f0.x, fmaf(x.y, f0.y, acc[m][0]));
        acc[m][1] = fmaf(x.x, f1.x, fmaf(x.y, f1.y, acc[m][1]));
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kGemvMaxM; ++m) {
    const float s0 = warp_sum(acc[m][0]), s1 = warp_sum(acc[m][1]);
    if (lane == 0) {
      red[warp][m][0] = s0;
      red[warp][m][1] = s1;
    }
  }
  __syncthreads();
  const int m = threadIdx.x;  // thread m writes row m of the pair
  if (m >= p.M) return;
  float t0 = 0.f, t1 = 0.f;
#pragma unroll
  for (int w = 0; w < kGemvWarps; ++w) {
    t0 += red[w][m][0];
    t1 += red[w][m][1];
  }
  float v0 = h2f_round(t0), v1 = h2f_round(t1);
  if constexpr (EPI == kF16) {
    if (p.resid) {
      v0 += __half2float(p.resid[(int64_t)m * p.ld_resid + r0]);
      v1 += __half2float(p.resid[(int64_t)m * p.ld_resid + r1]);
    }
    p.C[(int64_t)m * p.ldc + r0] = __float2half_rn(v0);
    p.C[(int64_t)m * p.ldc + r1] = __float2half_rn(v1);
  } else if constexpr (EPI == kRope) {
    if (r0 < p.rope_cols) {
      const int pos = p.rope_seq > 0 ? m % p.rope_seq : 0;
      const int c = q % 32;
      const float cc = __ldg(p.rope_cos + (int64_t)pos * 32 + c), ss = __ldg(p.rope_sin + (int64_t)pos * 32 + c);
      const float a = __fsub_rn(__fmul_rn(v0, cc), __fmul_rn(v1, ss));
      const float bb = __fadd_rn(__fmul_rn(v0, ss), __fmul_rn(v1, cc));
      v0 = a;
      v1 = bb;
    }
    p.C[(int64_t)m * p.ldc + r0] = __float2half_rn(v0);
    p.C[(int64_t)m * p.ldc + r1] = __float2half_rn(v1);
  } else {  // kSwigluF: v0 = gate, v1 = up
    p.C[(int64_t)m * p.ld_out + q] = __float2half_rn(v0);
    p.out1[(int64_t)m * p.ld_out + q] = __float2half_rn(v1);
    p.out2[(int64_t)m * p.ld_out + q] = __float2half_rn(__fmul_rn(h2f_round(silu_f(v0)), v1));
  }
}

template <int EPI>
int launch_gemv(const void* A, int64_t lda, const void* B, int64_t ldb, const Params& p, int pairs, cudaStream_t s,
                const char* name) {
  JX_CHECK_ARG(A && B && aligned16(A) && aligned16(B) && lda % 8 == 0 && ldb % 8 == 0 && p.K % 8 == 0,
               "%s: small-M operands must be 16-byte aligned with K, lda, ldb multiples of 8", name);
  JX_CHECK_ARG(pairs > 0 && pairs <= 0x7fffffff, "%s: bad shape", name);
  gemv_kernel<EPI><<<pairs, kGemvWarps * 32, 0, s>>>(static_cast<const __half*>(A), lda,
                                                     static_cast<const __half*>(B), ldb, p);
  JX_CHECK_LAUNCH(name);
  return JX_OK;
}

}  // namespace gemm

// ---------------------------------------------------------------------------
// TMA descriptor construction through the driver entry point (no -lcuda).
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace gemm {

// 0: choose (2-SM when there are at least two 128-row blocks), 1: force 1-SM, 2: force 2-SM.
// A test / diagnostic switch, kept per host thread (jx_gemm_set_mode).
static thread_local int g_gemm_mode = 0;

template <int EPI, bool A_MN, bool B_MN>
static int launch(const void* A, int64_t lda, const void* B, int64_t ldb, Params p, cudaStream_t stream,
                  const char* name) {
  JX_CHECK_ARG(A && B, "%s: NULL operand", name);
  JX_CHECK_ARG(p.M > 0 && p.N > 0 && p.K > 0, "%s: empty shape M=%d N=%d K=%d", name, p.M, p.N, p.K);
  JX_CHECK_ARG(aligned16(A) && aligned16(B), "%s: operands must be 16-byte aligned", name);
  JX_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0, "%s: leading dimensions must be multiples of 8 (lda=%lld ldb=%lld)",
               name, (long long)lda, (long long)ldb);
  CUtensorMap ta, tb;
  bool ok;
  if (!A_MN)
    ok = make_tmap_f16(&ta, A, p.K, p.M, lda, BK, BM);
  else
    ok = make_tmap_f16(&ta, A, p.M, p.K, lda, 64, BK);
  JX_CHECK_ARG(ok, "%s: cannot encode TMA descriptor for A", name);
  const int b_rows = (EPI == kSwigluF) ? 2 * p.swiglu_F : p.N;
  const bool two_sm = !p.skip_loads && ((g_gemm_mode == 2) || (g_gemm_mode == 0 && p.M > BM));
  if (!B_MN)
    ok = make_tmap_f16(&tb, B, p.K, b_rows, ldb, BK, (EPI == kSwigluF || two_sm) ? 128 : BN);
  else
    ok = make_tmap_f16(&tb, B, b_rows, p.K, ldb, 64, BK);
  JX_CHECK_ARG(ok, "%s: cannot encode TMA descriptor for B", name);
  // Output descriptors: [rows, cols] fp16 boxes of 32 rows x 64 columns (one epilogue warp's sub-tile).
  CUtensorMap tc0 = ta, tc1 = ta, tc2 = ta;
  if constexpr (EPI == kF16 || EPI == kHeadCE || EPI == kRope) {
    ok = make_tmap_f16(&tc0, p.C, p.N, p.M, p.ldc, 64, 32);
  } else if constexpr (EPI == kSwigluF) {
    ok = make_tmap_f16(&tc0, p.C, p.swiglu_F, p.M, p.ld_out, 64, 32) &&
         make_tmap_f16(&tc1, p.out1, p.swiglu_F, p.M, p.ld_out, 64, 32) &&
         make_tmap_f16(&tc2, p.out2, p.swiglu_F, p.M, p.ld_out, 64, 32);
  } else if constexpr (EPI == kSwigluB) {
    // 2-SM kernel: 32 x 32 boxes (64B swizzle) per part; 1-SM kernel: 32 x 64 staging boxes.
    const uint32_t bx = two_sm ? 32 : 64;
    const int sw = two_sm ? 64 : 128;
    ok = make_tmap_f16(&tc0, p.C, p.swiglu_F, p.M, p.ldc, bx, 32, sw) &&
         make_tmap_f16(&tc1, p.C + p.swiglu_F, p.swiglu_F, p.M, p.ldc, bx, 32, sw);
  }
  if constexpr (EPI == kWgrad) {
    if (p.splits > 1) ok = make_tmap_f32(&tc0, p.ws, p.N, p.M, p.N, 32, 32);
  }
  JX_CHECK_ARG(ok, "%s: cannot encode TMA descriptor for the output", name);
  // The 2-SM SwiGLU-backward epilogue's gate / up inputs, read as 32 x 32 boxes (64B swizzle).
  CUtensorMap tx0 = tc0, tx1 = tc0;
  if constexpr (EPI == kSwigluB) {
    if (two_sm)
      ok = make_tmap_f16(&tx0, p.aux0, p.swiglu_F, p.M, p.ld_aux, 32, 32, 64) &&
           make_tmap_f16(&tx1, p.aux1, p.swiglu_F, p.M, p.ld_aux, 32, 32, 64);
  }
  // The RoPE epilogue's cos / sin tables ([rope_seq, 32] fp32): a warp's 32 rows are 32 consecutive
  // positions when rope_seq is a multiple of 32, one 32 x 32 box per table.
  if constexpr (EPI == kRope) {
    p.rope_tma = two_sm && p.rope_seq % 32 == 0;
    if (p.rope_tma)
      ok = make_tmap_f32(&tx0, p.rope_cos, 32, p.rope_seq, 32, 32, 32) &&
           make_tmap_f32(&tx1, p.rope_sin, 32, p.rope_seq, 32, 32, 32);
  }
  JX_CHECK_ARG(ok, "%s: cannot encode TMA descriptor for an epilogue input", name);

  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (EPI == kSwigluF) ? (p.swiglu_F + 127) / 128 : (p.N + BN - 1) / BN;
  p.num_kb = (p.K + BK - 1) / BK;
  if (p.splits < 1) p.splits = 1;
  if (p.splits > p.num_kb) p.splits = p.num_kb;
  p.kb_per_split = (p.num_kb + p.splits - 1) / p.splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.status = status_ptr();

  if (two_sm) {
    // Resident clusters per device, per template instantiation (0 = not measured yet).
    static std::atomic<int> max_clusters[64];
    int dev = 0;
    JX_CUDA_TRY(cudaGetDevice(&dev), name);
    std::atomic<int>& slot = max_clusters[dev & 63];
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem2_bytes<EPI>();
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    if (slot.load(std::memory_order_acquire) == 0) {
      JX_CUDA_TRY(cudaFuncSetAttribute(gemm2_kernel<EPI, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem2_bytes<EPI>()),
                  name);
      cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
      int n = 0;
      JX_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, gemm2_kernel<EPI, A_MN, B_MN>, &cfg), name);
      slot.store(n > 0 ? n : 1, std::memory_order_release);
    }
    int max_cl = slot.load(std::memory_order_acquire);
    if (max_cl > persistent_sms() / 2) max_cl = persistent_sms() / 2;
    const int tiles2 = ((p.tiles_m + 1) / 2) * p.tiles_n * p.splits;
    const int clusters = tiles2 < max_cl ? tiles2 : max_cl;
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    JX_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm2_kernel<EPI, A_MN, B_MN>, ta, tb, tc0, tc1, tc2, tx0, tx1, p), name);
    JX_CHECK_LAUNCH(name);
    return JX_OK;
  }
  static std::atomic<uint64_t> attr_set{0};  // per template instantiation
  JX_CUDA_TRY(once_per_device(attr_set, [] {
                return cudaFuncSetAttribute(gemm_kernel<EPI, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)kSmemBytes);
              }),
              name);
  const int tiles = p.tiles_m * p.tiles_n * p.splits;
  const int grid = tiles < persistent_sms() ? tiles : persistent_sms();
  gemm_kernel<EPI, A_MN, B_MN><<<grid, kThreads, kSmemBytes, stream>>>(ta, tb, tc0, tc1, tc2, p);
  JX_CHECK_LAUNCH(name);
  return JX_OK;
}

static Params base_params(int M, int N, int K) {
  Params p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = 1;
  p.wait_budget = 1ll << 32;
  return p;
}

}  // namespace gemm
}  // namespace jx

using namespace jx;
using namespace jx::gemm;

extern "C" int jx_gemm_f16(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                           int M, int N, int K, void* C, int64_t ldc, const void* resid, int64_t ld_resid,
                           jx_stream_t stream) {
  JX_CHECK_ARG(C && aligned16(C) && ldc % 8 == 0 && N % 8 == 0, "jx_gemm_f16: C must be 16B aligned, ldc%%8==0, N%%8==0");
  JX_CHECK_ARG(!resid || (aligned16(resid) && ld_resid % 8 == 0), "jx_gemm_f16: bad residual");
  Params p = base_params(M, N, K);
  p.C = static_cast<__half*>(C);
  p.ldc = ldc;
  p.resid = static_cast<const __half*>(resid);
  p.ld_resid = ld_resid;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (M <= kGemvMaxM && !a_mn_major && !b_mn_major && N % 2 == 0)
    return launch_gemv<kF16>(A, lda, B, ldb, p, N / 2, s, "jx_gemm_f16");
  if (!a_mn_major && !b_mn_major) return launch<kF16, false, false>(A, lda, B, ldb, p, s, "jx_gemm_f16");
  if (!a_mn_major && b_mn_major) return launch<kF16, false, true>(A, lda, B, ldb, p, s, "jx_gemm_f16");
  if (a_mn_major && !b_mn_major) return launch<kF16, true, false>(A, lda, B, ldb, p, s, "jx_gemm_f16");
  return launch<kF16, true, true>(A, lda, B, ldb, p, s, "jx_gemm_f16");
}

extern "C" int jx_gemm_f16_ce_parts(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, void* C,
                                    int64_t ldc, void* parts, jx_stream_t stream) {
  JX_CHECK_ARG(C && aligned16(C) && ldc % 8 == 0 && N % 8 == 0,
               "jx_gemm_f16_ce_parts: C must be 16B aligned, ldc%%8==0, N%%8==0");
  JX_CHECK_ARG(parts && ((uintptr_t)parts & 7) == 0, "jx_gemm_f16_ce_parts: parts must be 8-byte aligned");
  Params p = base_params(M, N, K);
  p.C = static_cast<__half*>(C);
  p.ldc = ldc;
  p.ce_parts = static_cast<float2*>(parts);
  p.ce_nblk = (N + 127) / 128;
  return launch<kHeadCE, false, false>(A, lda, B, ldb, p, reinterpret_cast<cudaStream_t>(stream), "jx_gemm_f16_ce_parts");
}

extern "C" int jx_gemm_qkv_rope(const void* X, int64_t ldx, const void* W, int M, int hidden, int K, void* C,
                                int64_t ldc, const float* rope_cos, const float* rope_sin, int seq_len,
                                int head_dim, jx_stream_t stream) {
  JX_CHECK_ARG(head_dim == 64, "jx_gemm_qkv_rope: head_dim must be 64 (got %d)", head_dim);
  JX_CHECK_ARG(hidden % 64 == 0, "jx_gemm_qkv_rope: hidden must be a multiple of 64");
  JX_CHECK_ARG(rope_cos && rope_sin && seq_len > 0, "jx_gemm_qkv_rope: missing RoPE tables");
  JX_CHECK_ARG(aligned16(rope_cos) && aligned16(rope_sin), "jx_gemm_qkv_rope: RoPE tables must be 16-byte aligned");
  JX_CHECK_ARG(C && aligned16(C) && ldc % 8 == 0, "jx_gemm_qkv_rope: bad output");
  Params p = base_params(M, 3 * hidden, K);
  p.C = static_cast<__half*>(C);
  p.ldc = ldc;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.rope_seq = seq_len;
  p.rope_cols = 2 * hidden;
  if (M <= kGemvMaxM)
    return launch_gemv<kRope>(X, ldx, W, K, p, 3 * hidden / 2, reinterpret_cast<cudaStream_t>(stream),
                              "jx_gemm_qkv_rope");
  return launch<kRope, false, false>(X, ldx, W, K, p, reinterpret_cast<cudaStream_t>(stream), "jx_gemm_qkv_rope");
}

extern "C" int jx_gemm_swiglu_fwd(const void* X, int64_t ldx, const void* Wgu, int M, int F, int K, void* gate,
                                  void* up, void* act, int64_t ld_out, jx_stream_t stream) {
  JX_CHECK_ARG(gate && up && act && aligned16(gate) && aligned16(up) && aligned16(act),
               "jx_gemm_swiglu_fwd: outputs must be 16-byte aligned");
  JX_CHECK_ARG(F % 8 == 0 && ld_out % 8 == 0, "jx_gemm_swiglu_fwd: F and ld_out must be multiples of 8");
  Params p = base_params(M, 2 * F, K);
  p.swiglu_F = F;
  p.C = static_cast<__half*>(gate);
  p.out1 = static_cast<__half*>(up);
  p.out2 = static_cast<__half*>(act);
  p.ld_out = ld_out;
  if (M <= kGemvMaxM)
    return launch_gemv<kSwigluF>(X, ldx, Wgu, K, p, F, reinterpret_cast<cudaStream_t>(stream), "jx_gemm_swiglu_fwd");
  return launch<kSwigluF, false, false>(X, ldx, Wgu, K, p, reinterpret_cast<cudaStream_t>(stream),
                                        "jx_gemm_swiglu_fwd");
}

extern "C" int jx_gemm_swiglu_bwd(const void* dY, int64_t lddy, const void* Wd, int M, int F, int K, const void* gate,
                                  const void* up, int64_t ld_gu, void* dgu, int64_t ld_dgu, jx_stream_t stream) {
  JX_CHECK_ARG(gate && up && dgu && aligned16(gate) && aligned16(up) && aligned16(dgu),
               "jx_gemm_swiglu_bwd: buffers must be 16-byte aligned");
  JX_CHECK_ARG(F % 8 == 0 && ld_gu % 8 == 0 && ld_dgu % 8 == 0, "jx_gemm_swiglu_bwd: F, ld_gu, ld_dgu must be multiples of 8");
  JX_CHECK_ARG(ld_gu >= F && ld_dgu >= 2 * (int64_t)F, "jx_gemm_swiglu_bwd: rows shorter than F (gate / up) or 2F (dgu)");
  Params p = base_params(M, F, K);
  p.swiglu_F = F;
  p.C = static_cast<__half*>(dgu);
  p.ldc = ld_dgu;
  p.aux0 = static_cast<const __half*>(gate);
  p.aux1 = static_cast<const __half*>(up);
  p.ld_aux = ld_gu;
  // dact[m][f] = sum_k dY[m][k] * Wd[k][f]: B is Wd read MN-major.
  return launch<kSwigluB, false, true>(dY, lddy, Wd, F, p, reinterpret_cast<cudaStream_t>(stream),
                                       "jx_gemm_swiglu_bwd");
}

extern "C" int64_t jx_gemm_wgrad_workspace_bytes(int N, int K, int splits) {
  if (splits <= 1) return 0;
  return (int64_t)N * K * (int64_t)sizeof(float);  // one fp32 accumulator, whatever the split count
}

extern "C" int jx_gemm_wgrad(const void* dY, int64_t lddy, const void* X, int64_t ldx, int T, int N, int K, float* G,
                             int64_t ldg, int accumulate, int splits, void* workspace, jx_stream_t stream) {
  JX_CHECK_ARG(G && ((uintptr_t)G & 15) == 0 && ldg % 4 == 0 && K % 8 == 0, "jx_gemm_wgrad: bad gradient buffer");
  JX_CHECK_ARG(splits >= 1, "jx_gemm_wgrad: splits must be >= 1");
  JX_CHECK_ARG(splits == 1 || (workspace && ((uintptr_t)workspace & 15) == 0),
               "jx_gemm_wgrad: splits > 1 needs a 16-byte aligned workspace");
  // acc[n][k] = sum_t dY[t][n] * X[t][k]: both operands MN-major, reduction over tokens.
  Params p = base_params(N, K, T);
  p.G = G;
  p.ldg = ldg;
  p.accumulate = accumulate;
  p.splits = splits;
  p.ws = static_cast<float*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Clamp the split count exactly as launch() does so the reduction sees the same value.
  const int num_kb = (T + BK - 1) / BK;
  int sp = splits > num_kb ? num_kb : splits;
  const int per = (num_kb + sp - 1) / sp;
  sp = (num_kb + per - 1) / per;
  p.splits = sp;
  if (sp > 1)
    JX_CUDA_TRY(cudaMemsetAsync(workspace, 0, (size_t)N * K * sizeof(float), s), "jx_gemm_wgrad: clear workspace");
  int rc = launch<kWgrad, true, true>(dY, lddy, X, ldx, p, s, "jx_gemm_wgrad");
  if (rc != JX_OK || sp == 1) return rc;
  const int64_t total4 = (int64_t)N * K / 4;
  int blocks = (int)((total4 + 255) / 256);
  if (blocks > num_sms() * 8) blocks = num_sms() * 8;
  wgrad_reduce_kernel<<<blocks, 256, 0, s>>>(static_cast<const float*>(workspace), N, K, G, ldg, accumulate);
  JX_CHECK_LAUNCH("jx_gemm_wgrad: reduce");
  return JX_OK;
}

extern "C" int jx_gemm_set_mode(int mode) {
  JX_CHECK_ARG(mode >= 0 && mode <= 2, "jx_gemm_set_mode: mode must be 0 (auto), 1 (1-SM) or 2 (2-SM)");
  jx::gemm::g_gemm_mode = mode;
  return JX_OK;
}

extern "C" int jx_gemm_wait_test(const void* A, const void* B, void* C, int64_t wait_budget_cycles,
                                 jx_stream_t stream) {
  JX_CHECK_ARG(C && aligned16(C), "jx_gemm_wait_test: C must be 16-byte aligned");
  JX_CHECK_ARG(wait_budget_cycles > 0 && wait_budget_cycles <= (1ll << 32),
               "jx_gemm_wait_test: wait budget must be in (0, 2^32] cycles");
  // One 128 x 256 x 64 tile on the 1-SM kernel with its TMA loads withheld: the MMA thread's wait for the
  // first stage runs out, sets the abort flag and the status word, and every warp leaves through the
  // normal teardown (no copy is in flight, the TMEM is released).
  Params p = base_params(128, 256, 64);
  p.C = static_cast<__half*>(C);
  p.ldc = 256;
  p.wait_budget = wait_budget_cycles;
  p.skip_loads = 1;
  return launch<kF16, false, false>(A, 64, B, 64, p, reinterpret_cast<cudaStream_t>(stream), "jx_gemm_wait_test");
}
