// Causal flash attention on the 5th-generation tensor cores (tcgen05),
// head_dim 64: forward and backward.
//
// Reference: Midstream-LLM src/jishui/model_torch.py:48,
// F.scaled_dot_product_attention(q, k, v, is_causal=True), scale 1/sqrt(64),
// fp16 operands, fp32 softmax; the forward saves O and the natural-log LSE per
// row, the backward recomputes the probabilities from them.
//
// Forward: a persistent kernel, one CTA per SM. A work item is a
// pair of 128-query tiles (A = 2p, B = 2p+1) of one (head, batch); the CTAs
// take items from a global counter, heaviest first within chunks of 32
// (head, batch) pairs, and the loads of the next item overlap the last key
// tiles and the output of the current one.
// 320 threads:
//   warp 0     TMA producer: Q_A, Q_B per item, K_j / V_j (128 keys) into a 4-stage ring,
//   warp 1     TMEM allocator + MMA issuer, ping-ponging the two tiles:
//                S_w = Q_w K_j^T (M 128, N 128, K 64, operands in shared memory) -> TMEM,
//                O_w += P_w V_j  (M 128, N 64, K 128, P_w read from TMEM),
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B (one query row per
//              thread): the S row in registers (one TMEM round trip), row max,
//              P_w (fp16 pairs) stored back to TMEM;
//              O_w accumulates in TMEM across key tiles and is rescaled there only
//              when the row max grows by more than 2^8.
// S of the next key tile is computed while the softmax of this one runs, and
// while one warpgroup runs its softmax the tensor core works on the other's tile.
// q/k/v are read in place from the fused projection output [B*T, 3*H*64] by
// one TMA descriptor; O is written token-major [B*T, H*64].
#include <algorithm>
#include <type_traits>

#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace fa {

constexpr int D = 64;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int KV_STAGES = 4;
constexpr int kFwdThreads = 320;
constexpr uint32_t kTileBytes = BKV * D * 2;  // 16 KiB (one [128 x 64] fp16 tile)
constexpr uint32_t kPBytes = BQ * BKV * 2;    // 32 KiB (backward P^T / dS^T staging)
constexpr uint32_t kTmemCols = 512;
// smem: Q_A, Q_B | K stages | V stages | barriers
constexpr size_t kSmemBytes = 1024 + 2 * kTileBytes + 2 * KV_STAGES * kTileBytes + 512;

constexpr int kItemSlots = 4;
constexpr int kItemConsumers = 9;  // the MMA thread + 8 softmax warps

struct ItemRing {
  uint64_t full[kItemSlots], empty[kItemSlots];
  int idx[kItemSlots];
};

enum Status : int { kFaProducer = 301, kFaMma = 302, kFaSoftmax = 303 };

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], p_empty[2];  // per query tile (A, B)
  ItemRing items;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status, int code) {
  const long long start = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*abort_flag) return false;
      if (clock64() - start > (1ll << 32)) {
        *abort_flag = 1;
        if (status) atomicExch(status, code);
        return false;
      }
    }
  }
}

// Warp-wide wait where only lane 0 polls the barrier (all 32 lanes must be active).
// Used for barriers that publish TMEM contents or free a resource; the other
// lanes are ordered after lane 0's acquire by __syncwarp, and TMEM reads that
// follow are ordered by tcgen05.fence::after_thread_sync.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wait(bar, parity, abort_flag, status, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---------------------------------------------------------------------------
// Work distribution of the persistent forward. Work items are numbered in
// chunks of whole (head, batch) pairs; inside a chunk the heaviest items of all
// its pairs come first (the longest causal rows), then the next lighter, so the
// CTAs running at the same time share the K/V tiles of one chunk in L2 while
// each chunk still ends on its lightest items. The producer
// warp of each CTA takes the next number from a global counter (zeroed on the
// stream before the launch) and hands it to the MMA and softmax warps through
// a small ring of slots in shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ring_init(ItemRing* r) {
  for (int s = 0; s < kItemSlots; ++s) {
    mbar_init(&r->full[s], 1);
    mbar_init(&r->empty[s], kItemConsumers);
  }
}

// Producer: publish work number idx as this CTA's n-th item (false if the wait gave up).
__device__ __forceinline__ bool ring_publish(ItemRing* r, uint32_t n, int idx, volatile int* abort_flag, int* status,
                                             int code) {
  const int s = n % kItemSlots;
  if (!wait(&r->empty[s], ((n / kItemSlots) & 1) ^ 1, abort_flag, status, code)) return false;
  *reinterpret_cast<volatile int*>(&r->idx[s]) = idx;
  mbar_arrive(&r->full[s]);  // release: the slot store is visible to the waiting consumers
  return true;
}

// Consumer (one thread): the n-th item's work number, or -1 if the wait gave up.
__device__ __forceinline__ int ring_take(ItemRing* r, uint32_t n, volatile int* abort_flag, int* status, int code) {
  const int s = n % kItemSlots;
  if (!wait(&r->full[s], (n / kItemSlots) & 1, abort_flag, status, code)) return -1;
  const int idx = *reinterpret_cast<volatile int*>(&r->idx[s]);
  mbar_arrive(&r->empty[s]);
  return idx;
}

// Consumer (whole warp): lane 0 takes the slot, the number is broadcast.
__device__ __forceinline__ int ring_take_warp(ItemRing* r, uint32_t n, volatile int* abort_flag, int* status,
                                              int code) {
  int idx = 0;
  if ((threadIdx.x & 31) == 0) idx = ring_take(r, n, abort_flag, status, code);
  return __shfl_sync(0xffffffffu, idx, 0);
}

// Work number -> (chunk of `chunk` pairs, item rank inside the chunk, pair). Pair p is
// (head p % H, batch p / H). Returns the rank (0 = heaviest) and sets *pair.
__device__ __forceinline__ int chunked_rank(int idx, int per_pair, int chunk, int pairs, int* pair) {
  const int ci = idx / (chunk * per_pair);
  const int first = ci * chunk;
  const int n = min(chunk, pairs - first);
  const int local = idx - ci * chunk * per_pair;
  *pair = first + local % n;
  return local / n;
}

constexpr int kFwdChunk = 32;  // (head, batch) pairs per chunk of the forward

struct FwdItem {
  int pr, h, b;
};

__device__ __forceinline__ FwdItem fwd_decode(int idx, int npairs, int H, int B) {
  int pair;
  const int rank = chunked_rank(idx, npairs, kFwdChunk, H * B, &pair);
  return FwdItem{npairs - 1 - rank, pair % H, pair / H};
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, __half* __restrict__ out, float* __restrict__ lse,
                       int* __restrict__ work_counter, int B, int T, int H, float scale_log2, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                         // [2] query tiles
  uint8_t* sK = sQ + 2 * kTileBytes;
  uint8_t* sV = sK + KV_STAGES * kTileBytes;
  Bars* bars = reinterpret_cast<Bars*>(sV + KV_STAGES * kTileBytes);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = T / (2 * BQ);
  const int d = H * D;
  const int total = npairs * H * B;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bars->s_full[w], 1);
      mbar_init(&bars->s_free[w], 4);
      mbar_init(&bars->p_full[w], 4);
      mbar_init(&bars->p_empty[w], 1);
    }
    ring_init(&bars->items);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // TMEM columns of query-tile slot w: S at w*256 + [0,128), P (fp16 pairs) at
  // w*256 + [128,192), O at w*256 + [192,256).

  if (warp < 2) {
    if (warp == 0 && lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      uint32_t kv = 0;
      for (uint32_t round = 0;; ++round) {
        const int idx = atomicAdd(work_counter, 1);
        if (!ring_publish(&bars->items, round, idx, abort_flag, status, kFaProducer) || idx >= total) break;
        const FwdItem it = fwd_decode(idx, npairs, H, B);
        const int row_base = it.b * T;
        // The query tiles are free once the previous item's last S MMAs completed.
        if (!wait(&bars->q_empty, (round & 1) ^ 1, abort_flag, status, kFaProducer)) break;
        mbar_expect_tx(&bars->q_full, 2 * kTileBytes);
        tma_load_2d(sQ, &tm_qkv, &bars->q_full, it.h * D, row_base + (2 * it.pr) * BQ);
        tma_load_2d(sQ + kTileBytes, &tm_qkv, &bars->q_full, it.h * D, row_base + (2 * it.pr + 1) * BQ);
        const int n = 2 * it.pr + 2;
        bool ok = true;
        for (int j = 0; j < n; ++j, ++kv) {
          const int s = kv % KV_STAGES;
          if (!wait(&bars->kv_empty[s], ((kv / KV_STAGES) & 1) ^ 1, abort_flag, status, kFaProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars->kv_full[s], 2 * kTileBytes);
          tma_load_2d(sK + s * kTileBytes, &tm_qkv, &bars->kv_full[s], d + it.h * D, row_base + j * BKV);
          tma_load_2d(sV + s * kTileBytes, &tm_qkv, &bars->kv_full[s], 2 * d + it.h * D, row_base + j * BKV);
        }
        if (!ok) break;
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(BQ, BKV, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(BQ, D, false, true);
      uint32_t kv = 0;
      uint32_t ns[2] = {0, 0}, np[2] = {0, 0};  // S tiles issued / P V products issued per slot
      // Descriptors built once, advanced by constant additions per product.
      const uint64_t dQ0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dK0 = smem_desc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dV0 = smem_desc_sw128(smem_u32(sV), 8192, 1024);
      auto issue_s = [&](int w, uint32_t kvi) -> bool {
        const int s = kvi % KV_STAGES;
        if (!wait(&bars->kv_full[s], (kvi / KV_STAGES) & 1, abort_flag, status, kFaMma)) return false;
        if (!wait(&bars->s_free[w], (ns[w] & 1) ^ 1, abort_flag, status, kFaMma)) return false;
        tc_fence_after();
        const uint64_t a = desc_adv(dQ0, w * kTileBytes), bk = desc_adv(dK0, s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + w * 256, desc_adv(a, kk * 32), desc_adv(bk, kk * 32), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&bars->s_full[w]);
        ++ns[w];
        return true;
      };
      auto issue_pv = [&](int w, uint32_t kvi, bool first) -> bool {
        const int s = kvi % KV_STAGES;
        if (!wait(&bars->p_full[w], np[w] & 1, abort_flag, status, kFaMma)) return false;
        tc_fence_after();
        const uint64_t bv = desc_adv(dV0, s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // P from TMEM (16 keys = 8 packed columns per step); V [128 keys x 64 hd] read
          // MN-major (hd contiguous), 16 keys = two 8-row groups.
          const uint64_t bdesc = desc_adv(bv, kk * 2048);
          umma_f16_ts(tmem + w * 256 + 192, tmem + w * 256 + 128 + kk * 8, bdesc, idesc_o,
                      (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->p_empty[w]);
        ++np[w];
        return true;
      };
      bool ok = true;
      for (uint32_t round = 0; ok; ++round) {
        const int idx = ring_take(&bars->items, round, abort_flag, status, kFaMma);
        if (idx < 0 || idx >= total) break;
        const FwdItem it = fwd_decode(idx, npairs, H, B);
        const int nA = 2 * it.pr + 1, nB = 2 * it.pr + 2;
        ok = wait(&bars->q_full, round & 1, abort_flag, status, kFaMma);
        if (ok) ok = issue_s(0, kv) && issue_s(1, kv);
        for (int j = 0; j < nB && ok; ++j) {
          // S of the next key tile goes ahead of this tile's P V: the softmax has already
          // moved S_j into registers, so the tensor core computes S_{j+1} while it runs.
          if (j < nA) {
            if (j + 1 < nA && !(ok = issue_s(0, kv + j + 1))) break;
            if (!(ok = issue_pv(0, kv + j, j == 0))) break;
          }
          if (j + 1 < nB) {
            if (!(ok = issue_s(1, kv + j + 1))) break;
            if (j + 1 == nB - 1) umma_commit(&bars->q_empty);  // last S of this item issued
          }
          if (!(ok = issue_pv(1, kv + j, j == 0))) break;
          umma_commit(&bars->kv_empty[(kv + j) % KV_STAGES]);
        }
        kv += nB;
      }
    }
  } else {
    // Softmax: warpgroup w (0: warps 2-5, 1: warps 6-9); thread owns query row r of its tile.
    // The output accumulates in TMEM; it is rescaled there only when a row's running
    // max grows by more than 2^8, otherwise P is formed against the stale max (P <= 256).
    const int w = (warp - 2) >> 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + w * 256 + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr float kRescaleThreshold = 8.0f;  // log2 units
    uint32_t g = 0;                            // S tiles consumed by this slot
    bool ok = true;
    for (uint32_t round = 0; ok; ++round) {
      const int idx = ring_take_warp(&bars->items, round, abort_flag, status, kFaSoftmax);
      if (idx < 0 || idx >= total) break;
      const FwdItem it = fwd_decode(idx, npairs, H, B);
      const int qt = 2 * it.pr + w;  // query tile index
      const int q = qt * BQ + r;     // position in the sequence
      const int n = qt + 1;          // key tiles 0 .. qt
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++g) {
        if (!warp_wait(&bars->s_full[w], g & 1, abort_flag, status, kFaSoftmax)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[BKV];
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) tmem_ld32(lane_base + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->s_free[w]);  // S is in registers; the next S may overwrite it
        const bool diag = (j == n - 1);
        const int lim = diag ? q - j * BKV : BKV;  // columns <= lim are visible
        float mp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
        if (!diag) {
#pragma unroll
          for (int i = 0; i < BKV; i += 2)
            mp[(i >> 1) & 7] = max3(mp[(i >> 1) & 7], __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
        } else {
#pragma unroll
          for (int i = 0; i < BKV; ++i) mp[i & 7] = fmaxf(mp[i & 7], i <= lim ? __uint_as_float(sr[i]) : -INFINITY);
        }
        const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
        const float m_cand = mx * scale_log2;
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m = m_cand;
        } else if (m_cand > m + kRescaleThreshold) {
          alpha = ex2(m - m_cand);
          m = m_cand;
          rescale = true;
        }
        // P V of the previous tile must be done before P is overwritten or O is rescaled
        // (for j = 0 the previous item's epilogue waited for it).
        if (j > 0 && !warp_wait(&bars->p_empty[w], (g - 1) & 1, abort_flag, status, kFaSoftmax)) { ok = false; break; }
        tc_fence_after();
        // P = exp2(s*scale - m) as fp16 pairs into TMEM (64 columns, two stores of 32); 8 partial row sums.
        // (Computing all exponentials before this wait needs 64 more live registers and spills; measured slower.)
        float sp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) sp[u] = 0.f;
        const float neg_m = -m;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t pw[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int i0 = hf * 64 + 2 * e;
            float p0 = ex2(fmaf(__uint_as_float(sr[i0]), scale_log2, neg_m));
            float p1 = ex2(fmaf(__uint_as_float(sr[i0 + 1]), scale_log2, neg_m));
            if (diag) {
              if (i0 > lim) p0 = 0.f;
              if (i0 + 1 > lim) p1 = 0.f;
            }
            sp[(2 * e) & 7] += p0;
            sp[(2 * e + 1) & 7] += p1;
            __half2 hp = __floats2half2_rn(p0, p1);
            pw[e] = *reinterpret_cast<uint32_t*>(&hp);
          }
          tmem_st32(lane_base + 128 + hf * 32, pw);
        }
        const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
        // Rare: bring the TMEM output to the new max.
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t orr[32];
            tmem_ld32(lane_base + 192 + hf * 32, orr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
            tmem_st32(lane_base + 192 + hf * 32, orr);
          }
        }
        l = l * alpha + sum;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[w]);
      }
      if (ok && !warp_wait(&bars->p_empty[w], (g - 1) & 1, abort_flag, status, kFaSoftmax)) ok = false;
      if (!ok) break;
      tc_fence_after();
      const float inv = 1.f / l;
      __half* dst = out + (int64_t)(it.b * T + q) * d + it.h * D;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t orr[32];
        tmem_ld32(lane_base + 192 + hf * 32, orr);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __half2 hv = __floats2half2_rn(__uint_as_float(orr[c * 8 + 2 * e]) * inv,
                                           __uint_as_float(orr[c * 8 + 2 * e + 1]) * inv);
            wv[e] = *reinterpret_cast<uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(dst + hf * 32 + c * 8) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
      lse[((int64_t)it.b * H + it.h) * T + q] = (m + __log2f(l)) * 0.69314718055994530942f;
      // The O reads above complete before the next item's first P V overwrites O: that
      // product waits for this warp's next p_full arrival, issued after tcgen05.wait::ld.
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Backward on tcgen05: a persistent kernel, one CTA per SM. A work item is one
// 128-key block kb of one (head, batch); the CTAs take items from a global
// counter, heaviest first (key block kb meets T/128 - kb query tiles) within
// chunks of kBwdChunk (head, batch) pairs, so the last items anywhere are the
// one-tile blocks. The key block's K and V stay in shared memory (two buffers,
// one per item parity, so the next item's K / V load during this one's last
// tiles); dK and dV accumulate in TMEM across the query tiles i = kb .. T/128-1.
// Each query tile (Q_i, dO_i, -LSE_i log2(e), Delta_i: a two-slot ring filled
// by TMA, running on across items) is processed as two halves of 64 queries,
// pipelined against each other:
//   S^T_h  = K Q_h^T   (M 128 keys, N 64 queries, K 64)    TMEM [64h, 64h+64)
//   dP^T_h = V dO_h^T  (M 128, N 64, K 64)                 TMEM [128+64h, ...)
//   softmax warps of half h: P^T = exp(S^T*scale - LSE), dS^T = P^T (dP^T - Delta);
//                  both written back to TMEM as fp16 pairs over the columns just
//                  read, and dS^T also to 128B-swizzled shared memory (two buffers)
//   dV += P^T_h dO_h   (M 128, N 64, K 64; P^T from TMEM, dO read MN-major)   TMEM [256,320)
//   dK += dS^T_h Q_h   (M 128, N 64, K 64; dS^T from TMEM, Q read MN-major)   TMEM [320,384)
//   then S^T_h / dP^T_h of the next tile (of this item, or of the next item
//   during this item's last tile): the tensor core runs one thread's products
//   in issue order, so they follow the dV / dK reads of those columns.
//   dQ_i = dS K        (M 128 queries, N 64, K 128 keys; dS^T in shared memory
//                       read MN-major as the A operand, K read MN-major)     TMEM [384,512), two buffers
//   dQ_i is added to an fp32 accumulator in global memory by TMA reduce-add
//   (each warp stages its 32 x 32 block as two 64B-swizzled 32 x 16 halves)
//   while the products of the next tile run.
// At the end of an item the softmax warps drain dK / dV from TMEM (then the
// next item's first dV / dK products may overwrite them) and store them while
// the next item's first scores are computed.
// Warps: 0 TMA producer, 1 MMA issuer, 2..9 softmax / epilogue (two warps per
// TMEM lane quarter, each on half of the query columns).
// ---------------------------------------------------------------------------
constexpr int kBwdThreads = 320;
constexpr int kBwdChunk = 32;  // (head, batch) pairs per chunk of the backward's work order
constexpr uint32_t kDqStageBytes = 32 * 16 * 4;  // one warp's [32 rows x 16 cols] fp32 half of its dQ block
constexpr size_t kBwdSmem = 1024 + 4 * kTileBytes /*K,V x2*/ + 4 * kTileBytes /*Q,dO x2*/ + 2 * kPBytes /*dS^T x2*/ +
                            8 * kDqStageBytes /*dQ staging*/ + 2 * 2 * BQ * sizeof(float) /*-LSE log2e, Delta x2*/ +
                            512;

struct BwdBars {
  uint64_t kv_full[2], kv_empty[2];  // per K / V buffer (item parity)
  uint64_t q_full[2], q_empty[2];    // per query-tile ring slot
  uint64_t sdp_full[2], p_full[2];   // per query half
  uint64_t grads_done, dq_free[2], acc_drained;
  ItemRing items;
  uint32_t tmem_base;
  int abort;
};

struct BwdItem {
  int kb, h, b;
};

__device__ __forceinline__ BwdItem bwd_decode(int idx, int nqb, int H, int B) {
  int pair;
  const int kb = chunked_rank(idx, nqb, kBwdChunk, H * B, &pair);
  return BwdItem{kb, pair % H, pair / H};
}

// TMEM column (relative to the S^T or dP^T base) of the fp16 pair holding queries
// 2c, 2c+1 of K step kk (16 queries): the softmax warp of column half h writes the
// pairs of queries [64h, 64h+64) as two 16-column chunks at 64h and 64h+16.
__device__ __forceinline__ uint32_t pair_col(int kk) { return (kk >> 2) * 64 + (kk & 3) * 8; }

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ float h16(float x) { return __half2float(__float2half_rn(x)); }

// Inverse RoPE of one gradient pair (first-half column c, second-half column c+32) at position pos.
__device__ __forceinline__ void rope_back(float& g1, float& g2, const float* cs, const float* sn, int pos, int c) {
  const float co = __ldg(cs + (int64_t)pos * 32 + c), si = __ldg(sn + (int64_t)pos * 32 + c);
  const float a = __fadd_rn(__fmul_rn(g1, co), __fmul_rn(g2, si));
  const float b = __fsub_rn(__fmul_rn(g2, co), __fmul_rn(g1, si));
  g1 = a;
  g2 = b;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ neg_lse_log2, const float* __restrict__ delta,
                       float* __restrict__ dq_acc, __half* __restrict__ dqkv, int* __restrict__ work_counter, int B,
                       int T, int H, float scale, float scale_log2, const float* __restrict__ rope_cos,
                       const float* __restrict__ rope_sin, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem;                       // [2 buffers][K | V]
  uint8_t* sQ = sKV + 4 * kTileBytes;        // query-tile ring, 2 slots
  uint8_t* sO = sQ + 2 * kTileBytes;         // dO, 2 slots
  uint8_t* sSt = sO + 2 * kTileBytes;        // dS^T [128 keys x 128 queries], 2 buffers (tile parity)
  uint8_t* sDq = sSt + 2 * kPBytes;          // [8 warps][32 x 16] fp32 dQ staging (64B-swizzled)
  float* sL = reinterpret_cast<float*>(sDq + 8 * kDqStageBytes);  // [2][128] -LSE log2(e)
  float* sD = sL + 2 * BQ;                                   // [2][128] Delta
  BwdBars* bars = reinterpret_cast<BwdBars*>(sD + 2 * BQ);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = T / BQ;
  const int d = H * D;
  const int total = nqb * H * B;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->q_empty[s], 1);
      mbar_init(&bars->sdp_full[s], 1);
      mbar_init(&bars->p_full[s], 4);
      mbar_init(&bars->dq_free[s], 8);
    }
    mbar_init(&bars->grads_done, 1);
    mbar_init(&bars->acc_drained, 8);
    ring_init(&bars->items);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_do);
      uint32_t g = 0;  // query tiles loaded so far (the ring runs on across items)
      for (uint32_t n = 0;; ++n) {
        const int idx = atomicAdd(work_counter, 1);
        if (!ring_publish(&bars->items, n, idx, abort_flag, status, kFaProducer) || idx >= total) break;
        const BwdItem it = bwd_decode(idx, nqb, H, B);
        const int row_base = it.b * T;
        const int kvb = n & 1;
        if (!wait(&bars->kv_empty[kvb], ((n >> 1) & 1) ^ 1, abort_flag, status, kFaProducer)) break;
        uint8_t* kv = sKV + kvb * 2 * kTileBytes;
        mbar_expect_tx(&bars->kv_full[kvb], 2 * kTileBytes);
        tma_load_2d(kv, &tm_qkv, &bars->kv_full[kvb], d + it.h * D, row_base + it.kb * BKV);
        tma_load_2d(kv + kTileBytes, &tm_qkv, &bars->kv_full[kvb], 2 * d + it.h * D, row_base + it.kb * BKV);
        const float* lse_bh = neg_lse_log2 + ((int64_t)it.b * H + it.h) * T;
        const float* delta_bh = delta + ((int64_t)it.b * H + it.h) * T;
        bool ok = true;
        for (int qi = it.kb; qi < nqb; ++qi, ++g) {
          const int s = g & 1;
          if (!wait(&bars->q_empty[s], ((g >> 1) & 1) ^ 1, abort_flag, status, kFaProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars->q_full[s], 2 * kTileBytes + 2 * BQ * sizeof(float));
          tma_load_2d(sQ + s * kTileBytes, &tm_qkv, &bars->q_full[s], it.h * D, row_base + qi * BQ);
          tma_load_2d(sO + s * kTileBytes, &tm_do, &bars->q_full[s], it.h * D, row_base + qi * BQ);
          bulk_load(sL + s * BQ, lse_bh + qi * BQ, BQ * sizeof(float), &bars->q_full[s]);
          bulk_load(sD + s * BQ, delta_bh + qi * BQ, BQ * sizeof(float), &bars->q_full[s]);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_sq = idesc_f16_f32(BKV, BQ / 2, false, false);
      constexpr uint32_t id_kn = idesc_f16_f32(BKV, D, false, true);
      constexpr uint32_t id_q = idesc_f16_f32(BQ, D, true, true);
      // Shared-memory descriptors are built once and advanced by constant additions: one
      // thread issues every product, and an N = 64 product is shorter than building two
      // descriptors from addresses. K / V descriptors are for buffer 0 (+ 2 tiles for buffer 1).
      const uint64_t dK = smem_desc_sw128(smem_u32(sKV), 16, 1024);               // K-major A of S^T
      const uint64_t dV = smem_desc_sw128(smem_u32(sKV + kTileBytes), 16, 1024);  // K-major A of dP^T
      const uint64_t dKmn = smem_desc_sw128(smem_u32(sKV), 8192, 1024);           // MN-major B of dQ
      const uint64_t dQk = smem_desc_sw128(smem_u32(sQ), 16, 1024);               // K-major B of S^T (slot 0)
      const uint64_t dOk = smem_desc_sw128(smem_u32(sO), 16, 1024);
      const uint64_t dQmn = smem_desc_sw128(smem_u32(sQ), 8192, 1024);  // MN-major B of dK
      const uint64_t dOmn = smem_desc_sw128(smem_u32(sO), 8192, 1024);  // MN-major B of dV
      const uint64_t dSt = smem_desc_sw128(smem_u32(sSt), 16384, 1024); // MN-major A of dQ (buffer 0)
      // S^T / dP^T of query half hf of ring tile g with K / V buffer kvb: M 128 keys, N 64
      // queries, into TMEM columns [64 hf, 64 hf + 64) and [128 + 64 hf, ...).
      auto issue_sdp = [&](uint32_t g, auto hc, auto slot_c, int kvb) {
        constexpr int hf = decltype(hc)::value;
        constexpr int SL = decltype(slot_c)::value;  // ring slot of tile g (g & 1)
        (void)g;
        const uint32_t off = SL * kTileBytes + hf * 8192;
        const uint32_t kvo = kvb * 2 * kTileBytes;
        const uint64_t bq = desc_adv(dQk, off), bo = desc_adv(dOk, off);
        const uint64_t ak = desc_adv(dK, kvo), av = desc_adv(dV, kvo);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16(tmem + hf * 64, desc_adv(ak, kk * 32), desc_adv(bq, kk * 32), id_sq, kk > 0 ? 1u : 0u);
          umma_f16(tmem + 128 + hf * 64, desc_adv(av, kk * 32), desc_adv(bo, kk * 32), id_sq, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->sdp_full[hf]);
      };
      uint32_t g = 0;  // query tiles processed (ring slot and TMEM / shared buffer parities)
      bool ok = true;
      int idx = ring_take(&bars->items, 0, abort_flag, status, kFaMma);
      if (idx >= 0 && idx < total) {
        ok = wait(&bars->kv_full[0], 0, abort_flag, status, kFaMma) &&
             wait(&bars->q_full[0], 0, abort_flag, status, kFaMma);
        if (ok) {
          tc_fence_after();
          issue_sdp(0, std::integral_constant<int, 0>{}, std::integral_constant<int, 0>{}, 0);
          issue_sdp(0, std::integral_constant<int, 1>{}, std::integral_constant<int, 0>{}, 0);
        }
      }
      for (uint32_t n = 0; ok && idx >= 0 && idx < total; ++n) {
        const BwdItem it = bwd_decode(idx, nqb, H, B);
        const int ntiles = nqb - it.kb;
        const int kvb = n & 1;
        const uint64_t kmn = desc_adv(dKmn, kvb * 2 * kTileBytes);
        int next = -1;  // the following item, taken during this item's last tile
        for (int t = 0; t < ntiles && ok; ++t, ++g) {
          // The ring slot (g & 1) is a compile-time constant in each copy of the tile body.
          auto tile = [&](auto sc) {
            constexpr int S = decltype(sc)::value;
            const uint64_t bq = desc_adv(dQmn, S * kTileBytes), bo = desc_adv(dOmn, S * kTileBytes);
            // The half index is a compile-time constant in each copy of the body (TMEM columns, descriptor
            // offsets and barrier addresses fold into immediates).
            auto half = [&](auto hc) {
              constexpr int hf = decltype(hc)::value;
              // P^T / dS^T of this half are in TMEM (over its S^T / dP^T columns).
              if (!(ok = wait(&bars->p_full[hf], S, abort_flag, status, kFaMma))) return;
              // The first dV / dK products of an item overwrite the accumulators: the previous
              // item's epilogue has read them.
              if (t == 0 && hf == 0 && n > 0 && !(ok = wait(&bars->acc_drained, (n - 1) & 1, abort_flag, status, kFaMma)))
                return;
              tc_fence_after();
  #pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int kk = hf * 4 + j;  // 16 queries per step
                const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
                umma_f16_ts(tmem + 256, tmem + pair_col(kk), desc_adv(bo, kk * 2048), id_kn, acc);
                umma_f16_ts(tmem + 320, tmem + 128 + pair_col(kk), desc_adv(bq, kk * 2048), id_kn, acc);
              }
              if (hf == 1) umma_commit(&bars->q_empty[S]);  // Q / dO / LSE / Delta of this slot are no longer read
              // The next tile's scores of this half overwrite the columns dV / dK just read; the
              // tensor core runs a thread's products in issue order.
              if (t + 1 < ntiles) {
                if (hf == 0) {
                  if (!(ok = wait(&bars->q_full[1 - S], ((g + 1) >> 1) & 1, abort_flag, status, kFaMma))) return;
                  tc_fence_after();
                }
                issue_sdp(g + 1, hc, std::integral_constant<int, 1 - S>{}, kvb);
              } else {
                if (hf == 0) {
                  next = ring_take(&bars->items, n + 1, abort_flag, status, kFaMma);
                  if (next < 0) {
                    ok = false;
                    return;
                  }
                  if (next < total) {
                    if (!(ok = wait(&bars->kv_full[kvb ^ 1], ((n + 1) >> 1) & 1, abort_flag, status, kFaMma) &&
                               wait(&bars->q_full[1 - S], ((g + 1) >> 1) & 1, abort_flag, status, kFaMma)))
                      return;
                    tc_fence_after();
                  }
                }
                if (next < total) issue_sdp(g + 1, hc, std::integral_constant<int, 1 - S>{}, kvb ^ 1);  // next item's first tile
              }
            };
            half(std::integral_constant<int, 0>{});
            if (ok) half(std::integral_constant<int, 1>{});
            if (!ok) return;
            if (!(ok = wait(&bars->dq_free[S], ((g >> 1) & 1) ^ 1, abort_flag, status, kFaMma))) return;
            tc_fence_after();
            const uint64_t sbuf = desc_adv(dSt, S * kPBytes);
  #pragma unroll
            for (int kk = 0; kk < BKV / 16; ++kk) {
              // dS^T read MN-major: queries contiguous (two 64-query halves 16 KiB apart), 16 keys per step.
              umma_f16(tmem + 384 + S * D, desc_adv(sbuf, kk * 2048), desc_adv(kmn, kk * 2048), id_q,
                       kk > 0 ? 1u : 0u);
            }
            umma_commit(&bars->grads_done);
            if (t + 1 == ntiles) umma_commit(&bars->kv_empty[kvb]);  // K / V of this item are no longer read
          };
          if (g & 1)
            tile(std::integral_constant<int, 1>{});
          else
            tile(std::integral_constant<int, 0>{});
        }
        idx = next;
      }
    }
  } else {
    const int quarter = warp & 3;         // TMEM lane quarter
    const int colh = (warp - 2) >> 2;     // which half of the query columns
    const int r = quarter * 32 + lane;    // key row (S^T / dP^T / dK / dV) or query row (dQ)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // dQ of ring tile gp: TMEM lanes are query rows; this warp adds 32 of the 64 columns of its
    // 32 rows (from global row qrow) to the fp32 accumulator: two 16-column halves, each staged in
    // shared memory (64B swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)) and added by one
    // TMA reduce.
    uint8_t* dq_stage = sDq + (warp - 2) * kDqStageBytes;
    auto drain_dq = [&](uint32_t gp, int head, int qrow) {
      const int buf = gp & 1;
      tc_fence_after();
      uint32_t qr[32];
      tmem_ld32(lane_base + 384 + buf * D + colh * 32, qr);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->dq_free[buf]);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the staging was read
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int w = part * 16 + c * 4;
          *reinterpret_cast<uint4*>(dq_stage + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(qr[w], qr[w + 1], qr[w + 2], qr[w + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          asm volatile(
              "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                  reinterpret_cast<uint64_t>(&tm_dq)),
              "r"(smem_u32(dq_stage)), "r"(head * D + colh * 32 + part * 16), "r"(qrow)
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
    };
    uint8_t* srow0 = sSt + colh * 16384 + (r >> 3) * 1024 + (r & 7) * 128;  // this thread's dS^T row
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t n = 0; ok; ++n) {
      const int idx = ring_take_warp(&bars->items, n, abort_flag, status, kFaSoftmax);
      if (idx < 0) break;
      if (idx >= total) break;
      const BwdItem it = bwd_decode(idx, nqb, H, B);
      const int ntiles = nqb - it.kb;
      const int key = it.kb * BKV + r;
      const int row_base = it.b * T;
      const int dq_row0 = row_base + quarter * 32;  // + qi * BQ: this warp's first dQ row of tile qi
      for (int t = 0; t < ntiles && ok; ++t, ++g) {
        const int s = g & 1, qi = it.kb + t;
        const bool diag = (t == 0);
        if (!wait(&bars->q_full[s], (g >> 1) & 1, abort_flag, status, kFaSoftmax)) { ok = false; break; }
        if (!warp_wait(&bars->sdp_full[colh], g & 1, abort_flag, status, kFaSoftmax)) { ok = false; break; }
        uint8_t* srow = srow0 + s * kPBytes;
        tc_fence_after();
        const float* Ls = sL + s * BQ;
        const float* Ds = sD + s * BQ;
        const int lim = diag ? key - qi * BQ : -1;  // on the diagonal tile, queries at index < lim are masked
        // The diagonal tile masks queries before this thread's key; the other tiles compile without the test.
        auto softmax_tile = [&](auto diag_tag) {
          constexpr bool kDiag = decltype(diag_tag)::value;
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            // 32 queries: S^T / dP^T in, P^T / dS^T (fp16 pairs) back over the first 16 columns of
            // this warp's half (already read), dS^T also to shared memory.
            const int q0 = colh * 64 + ch * 32;
            uint32_t sr[32], dr[32];
            tmem_ld32(lane_base + q0, sr);
            tmem_ld32(lane_base + 128 + q0, dr);
            tmem_ld_wait();
            uint32_t pw[16], sw[16];
#pragma unroll
            for (int gq = 0; gq < 8; ++gq) {  // 4 queries per group: -LSE log2(e) / Delta as float4 (broadcast reads)
              const float4 L4 = *reinterpret_cast<const float4*>(Ls + q0 + gq * 4);
              const float4 D4 = *reinterpret_cast<const float4*>(Ds + q0 + gq * 4);
              const float nl[4] = {L4.x, L4.y, L4.z, L4.w};
              const float dl[4] = {D4.x, D4.y, D4.z, D4.w};
              float pv[4], dv[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int qc = gq * 4 + u;
                float p = ex2(fmaf(__uint_as_float(sr[qc]), scale_log2, nl[u]));
                if (kDiag && q0 + qc < lim) p = 0.f;
                pv[u] = p;
                dv[u] = p * (__uint_as_float(dr[qc]) - dl[u]);
              }
              __half2 hp0 = __floats2half2_rn(pv[0], pv[1]), hp1 = __floats2half2_rn(pv[2], pv[3]);
              __half2 hs0 = __floats2half2_rn(dv[0], dv[1]), hs1 = __floats2half2_rn(dv[2], dv[3]);
              pw[gq * 2] = *reinterpret_cast<uint32_t*>(&hp0);
              pw[gq * 2 + 1] = *reinterpret_cast<uint32_t*>(&hp1);
              sw[gq * 2] = *reinterpret_cast<uint32_t*>(&hs0);
              sw[gq * 2 + 1] = *reinterpret_cast<uint32_t*>(&hs1);
            }
            tmem_st16(lane_base + colh * 64 + ch * 16, pw);
            tmem_st16(lane_base + 128 + colh * 64 + ch * 16, sw);
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 4 chunks of 8 queries
              const int off = ((ch * 4 + c) ^ (r & 7)) << 4;
              *reinterpret_cast<uint4*>(srow + off) = make_uint4(sw[c * 4], sw[c * 4 + 1], sw[c * 4 + 2], sw[c * 4 + 3]);
            }
          }
        };
        if (diag)
          softmax_tile(std::true_type{});
        else
          softmax_tile(std::false_type{});
        tmem_st_wait();
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[colh]);
        // The previous tile's dQ completed before this tile's scores; reduce it while this tile's products run.
        if (t > 0) {
          if (!warp_wait(&bars->grads_done, (g - 1) & 1, abort_flag, status, kFaSoftmax)) { ok = false; break; }
          drain_dq(g - 1, it.h, dq_row0 + (qi - 1) * BQ);
        }
      }
      if (!ok) break;
      // The item's last dQ, then dK (warps with colh 0, scaled, rotated back through RoPE) and dV (colh 1).
      if (!warp_wait(&bars->grads_done, (g - 1) & 1, abort_flag, status, kFaSoftmax)) break;
      drain_dq(g - 1, it.h, dq_row0 + (nqb - 1) * BQ);
      tc_fence_after();
      uint32_t ar[64];
      const uint32_t col = colh == 0 ? 320u : 256u;
      tmem_ld32(lane_base + col, *reinterpret_cast<uint32_t(*)[32]>(&ar[0]));
      tmem_ld32(lane_base + col + 32, *reinterpret_cast<uint32_t(*)[32]>(&ar[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_drained);  // the next item's first dV / dK products may overwrite them
      float v[64];
      const float sc = colh == 0 ? scale : 1.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = h16(__uint_as_float(ar[i]) * sc);
      if (colh == 0 && rope_cos) {
#pragma unroll
        for (int c = 0; c < 32; ++c) rope_back(v[c], v[c + 32], rope_cos, rope_sin, key, c);
      }
      __half* dst = dqkv + (int64_t)(row_base + key) * (3 * d) + (colh == 0 ? d : 2 * d) + it.h * D;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __half2 hv = __floats2half2_rn(v[c * 8 + 2 * e], v[c * 8 + 2 * e + 1]);
          w[e] = *reinterpret_cast<uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(dst + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // dQ reduces complete
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// dqkv[:, h*64 + c] = f16(RoPE^-1(f16(dq_acc * scale))) for the query part; one
// thread per (row, head, group of 8 rotation pairs), 16-byte accesses.
__global__ void attn_dq_finish_kernel(const float* __restrict__ dq_acc, __half* __restrict__ dqkv, int64_t rows, int H,
                                      int T, float scale, const float* __restrict__ rope_cos,
                                      const float* __restrict__ rope_sin) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = rows * H * 4;
  if (i >= total) return;
  const int grp = (int)(i & 3);
  const int64_t rh = i >> 2;
  const int h = (int)(rh % H);
  const int64_t row = rh / H;
  const int d = H * D;
  const float* src = dq_acc + row * d + h * D + grp * 8;
  float g1[8], g2[8];
  const float4 a0 = *reinterpret_cast<const float4*>(src), a1 = *reinterpret_cast<const float4*>(src + 4);
  const float4 b0 = *reinterpret_cast<const float4*>(src + 32), b1 = *reinterpret_cast<const float4*>(src + 36);
  const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  const int pos = (int)(row % T);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    g1[j] = h16(av[j] * scale);
    g2[j] = h16(bv[j] * scale);
    if (rope_cos) rope_back(g1[j], g2[j], rope_cos, rope_sin, pos, grp * 8 + j);
  }
  uint32_t w1[4], w2[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __half2 x = __floats2half2_rn(g1[2 * e], g1[2 * e + 1]);
    __half2 y = __floats2half2_rn(g2[2 * e], g2[2 * e + 1]);
    w1[e] = *reinterpret_cast<uint32_t*>(&x);
    w2[e] = *reinterpret_cast<uint32_t*>(&y);
  }
  __half* dst = dqkv + row * (3 * d) + h * D + grp * 8;
  *reinterpret_cast<uint4*>(dst) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  *reinterpret_cast<uint4*>(dst + 32) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
}

}  // namespace fa
}  // namespace jx

using namespace jx;
using namespace jx::fa;

extern "C" int64_t jx_attn_fwd_workspace_bytes(int B, int T, int H, int Dh) {
  (void)B, (void)T, (void)H, (void)Dh;
  return 256;  // the work counter of the persistent kernel
}

extern "C" int jx_attn_fwd(const void* qkv, void* out, float* lse, void* workspace, int B, int T, int H, int Dh,
                           float scale, jx_stream_t stream) {
  JX_CHECK_ARG(qkv && out && lse && workspace, "jx_attn_fwd: NULL argument");
  JX_CHECK_ARG(Dh == 64, "jx_attn_fwd: head_dim must be 64 (got %d)", Dh);
  JX_CHECK_ARG(B > 0 && H > 0 && T > 0 && T % 256 == 0, "jx_attn_fwd: T must be a positive multiple of 256 (got %d)", T);
  JX_CHECK_ARG(aligned16(qkv) && aligned16(out) && aligned16(workspace), "jx_attn_fwd: buffers must be 16-byte aligned");
  JX_CHECK_ARG((int64_t)(T / 256) * H * B < (1LL << 30), "jx_attn_fwd: too many work items");
  const int64_t rows = (int64_t)B * T;
  const int64_t cols = 3LL * H * D;
  CUtensorMap tm;
  JX_CHECK_ARG(make_tmap_f16(&tm, qkv, cols, rows, cols, D, BKV), "jx_attn_fwd: cannot encode TMA descriptor");
  static std::atomic<uint64_t> attr_set{0};
  JX_CUDA_TRY(once_per_device(attr_set, [] {
                return cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)kSmemBytes);
              }),
              "jx_attn_fwd: smem attribute");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* counter = static_cast<int*>(workspace);
  JX_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(int), s), "jx_attn_fwd: clear work counter");
  const float scale_log2 = scale * 1.4426950408889634f;
  const int64_t items = (int64_t)(T / (2 * BQ)) * H * B;
  const int grid = (int)std::min<int64_t>(items, persistent_sms());
  attn_fwd_tc_kernel<<<grid, kFwdThreads, kSmemBytes, s>>>(tm, static_cast<__half*>(out), lse, counter, B, T, H,
                                                           scale_log2, status_ptr());
  JX_CHECK_LAUNCH("jx_attn_fwd");
  return JX_OK;
}

extern "C" int64_t jx_attn_bwd_workspace_bytes(int B, int T, int H, int Dh) {
  // Delta, -LSE log2(e), the fp32 dQ accumulator, the work counter of the persistent kernel.
  return 2 * (int64_t)B * H * T * 4 + (int64_t)B * T * H * Dh * 4 + 256;
}

// Delta = rowsum(dO * O), computed by attn_delta_kernel in attention.cu.
namespace jx {
namespace attn {
void launch_delta(const __half* out, const __half* dout, const float* lse, float* delta, float* neg_lse_log2, int B,
                  int T, int H, cudaStream_t s);
}
}  // namespace jx

extern "C" int jx_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, void* workspace,
                           void* dqkv, int B, int T, int H, int Dh, float scale, const float* rope_cos,
                           const float* rope_sin, jx_stream_t stream) {
  JX_CHECK_ARG(qkv && out && dout && lse && workspace && dqkv, "jx_attn_bwd: NULL argument");
  JX_CHECK_ARG(Dh == 64, "jx_attn_bwd: head_dim must be 64 (got %d)", Dh);
  JX_CHECK_ARG(B > 0 && H > 0 && T > 0 && T % 128 == 0, "jx_attn_bwd: T must be a positive multiple of 128");
  JX_CHECK_ARG(aligned16(qkv) && aligned16(out) && aligned16(dout) && aligned16(dqkv) && aligned16(lse) &&
                   aligned16(workspace),
               "jx_attn_bwd: buffers must be 16-byte aligned");
  JX_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr), "jx_attn_bwd: pass both RoPE tables or neither");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* delta = static_cast<float*>(workspace);
  float* nl2 = delta + (int64_t)B * H * T;
  float* dq_acc = nl2 + (int64_t)B * H * T;
  const int64_t rows = (int64_t)B * T;
  const int d = H * D;
  CUtensorMap tq, tdo;
  JX_CHECK_ARG(make_tmap_f16(&tq, qkv, 3LL * d, rows, 3LL * d, D, BKV), "jx_attn_bwd: cannot encode TMA descriptor");
  JX_CHECK_ARG(make_tmap_f16(&tdo, dout, d, rows, d, D, BQ), "jx_attn_bwd: cannot encode TMA descriptor");
  int* counter = reinterpret_cast<int*>(dq_acc + rows * d);
  CUtensorMap tdq;
  JX_CHECK_ARG(make_tmap_f32(&tdq, dq_acc, d, rows, d, 16, 32, 64),
               "jx_attn_bwd: cannot encode TMA descriptor for the dQ accumulator");
  JX_CHECK_ARG((int64_t)(T / BQ) * H * B < (1LL << 30), "jx_attn_bwd: too many work items");
  // One clear for the dQ accumulator and the work counter behind it.
  JX_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, (size_t)rows * d * sizeof(float) + sizeof(int), s),
              "jx_attn_bwd: clear dq accumulator");
  jx::attn::launch_delta(static_cast<const __half*>(out), static_cast<const __half*>(dout), lse, delta, nl2, B, T, H, s);
  JX_CHECK_LAUNCH("jx_attn_bwd: delta");
  static std::atomic<uint64_t> attr_set{0};
  JX_CUDA_TRY(once_per_device(attr_set, [] {
                return cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)kBwdSmem);
              }),
              "jx_attn_bwd: smem attribute");
  const int64_t items = (int64_t)(T / BQ) * H * B;
  const int grid = (int)std::min<int64_t>(items, persistent_sms());
  attn_bwd_tc_kernel<<<grid, kBwdThreads, kBwdSmem, s>>>(tq, tdo, tdq, nl2, delta, dq_acc, static_cast<__half*>(dqkv),
                                                        counter, B, T, H, scale, scale * 1.4426950408889634f,
                                                        rope_cos, rope_sin, status_ptr());
  JX_CHECK_LAUNCH("jx_attn_bwd");
  const int64_t groups = rows * H * 4;
  attn_dq_finish_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, s>>>(dq_acc, static_cast<__half*>(dqkv), rows, H, T,
                                                                        scale, rope_cos, rope_sin);
  JX_CHECK_LAUNCH("jx_attn_bwd: dq finish");
  return JX_OK;
}
