/*
 * jishui_b200.h — C ABI of the B200 (sm_100a) kernels behind the Jishui
 * decoder training step.
 *
 * Conventions shared by every entry point:
 *   - All tensors are device pointers owned by the caller (torch allocates
 *     them). Sizes and leading dimensions are in elements.
 *   - "f16" buffers hold IEEE binary16, "f32" buffers binary32.
 *   - Each call is stream-ordered on `stream` (the caller's current CUDA
 *     stream) and never synchronises the host.
 *   - The return value is JX_OK (0) or a negative JX_ERR_* code; the text of
 *     the most recent failure on the calling thread is returned by
 *     jx_last_error().
 *   - The library allocates no device memory on any call. Scratch space (the
 *     split-K partials of the weight-gradient GEMM, the attention backward's
 *     dQ accumulator) is passed in by the caller; the *_workspace_bytes()
 *     queries give its size.
 *
 * Reference interfaces replaced (paths are inside the Midstream-LLM project):
 *   src/jishui/model_torch.py:12-15   nn.RMSNorm            -> jx_rmsnorm_fwd / jx_rmsnorm_bwd
 *   src/jishui/model_torch.py:18-25   rope()                -> jx_gemm_qkv_rope epilogue, jx_attn_bwd rope_* args
 *   src/jishui/model_torch.py:41-43   q/k/v nn.Linear       -> jx_gemm_qkv_rope, jx_gemm_f16, jx_gemm_wgrad
 *   src/jishui/model_torch.py:48      F.scaled_dot_product_attention(is_causal=True) -> jx_attn_fwd / jx_attn_bwd
 *   src/jishui/model_torch.py:49,72   o_proj + residual add -> jx_gemm_f16 (residual epilogue)
 *   src/jishui/model_torch.py:59-60   SwiGLU                -> jx_gemm_swiglu_fwd / jx_gemm_swiglu_bwd
 *   src/jishui/model_torch.py:89-93   nn.Embedding + cast   -> jx_embed_fwd / jx_embed_bwd
 *   src/jishui/model_torch.py:98      tied head F.linear    -> jx_gemm_f16 (+ jx_gemm_wgrad for dE)
 *   src/jishui/model_torch.py:102-104 F.cross_entropy(logits.float()) -> jx_ce_fwd (or jx_gemm_f16_ce_parts +
 *                                     jx_ce_fwd_parts) / jx_ce_loss / jx_ce_bwd
 *   src/jishui/pretrain_torch.py:218-219 GradScaler.unscale_ + clip_grad_norm_ -> jx_grad_stats / jx_grad_finalize
 *   src/jishui/pretrain_torch.py:119-120,231 AdamW(fused=True).step -> jx_adamw_step
 */
#ifndef JISHUI_B200_H_
#define JISHUI_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* jx_stream_t; /* == cudaStream_t */

#define JX_OK 0
#define JX_ERR_INVALID -1     /* bad argument, shape or alignment */
#define JX_ERR_UNSUPPORTED -2 /* valid but not implemented for this shape */
#define JX_ERR_LAUNCH -3      /* CUDA launch / runtime error */

/* Library version (major*10000 + minor*100 + patch). */
int jx_version(void);
/* Text of the last error on this host thread ("" if none). */
const char* jx_last_error(void);
/* Number of kernels this library has launched in this process. */
int64_t jx_launch_count(void);
/* Device-side status word: non-zero when a kernel abandoned work after a
 * bounded wait expired (code identifies the wait: 101-103 GEMM producer / MMA /
 * epilogue, 301-303 attention producer / MMA / softmax, 501 the staged RMSNorm
 * backward's row copies) or met a bad input (201 token id, 202 target, 401 / 402
 * packed-row column / source). Reads and optionally clears it; synchronises the
 * current device. */
int jx_device_status(int* status_out, int clear);
/* Number of SMs that the persistent kernels (GEMM, attention) launched from the
 * calling host thread leave free, e.g. for NCCL's collective kernels while
 * gradient buckets are in flight during a data-parallel backward (0 by default,
 * at most 64; results do not depend on it). No counterpart in the reference. */
int jx_set_sm_reserve(int sms);

/* ---- RMSNorm (model_torch.py:12-15, nn.RMSNorm, eps from ModelConfig.norm_eps) ----
 * Forward: s = x (+ resid if resid != NULL, stored to sum_out as f16);
 *   rstd[r] = 1/sqrt(mean(s^2) + eps);  y = f16( f16(s*rstd) * gamma ).
 * x, resid, sum_out, y: f16 [rows, cols] contiguous; gamma f32 [cols]; rstd f32 [rows].
 * cols must be a multiple of 8 and <= 4096. */
int jx_rmsnorm_fwd(const void* x, const void* resid, void* sum_out, const float* gamma, void* y, float* rstd,
                   int64_t rows, int cols, float eps, jx_stream_t stream);
/* Backward: dx = f16( dresid + f16(d rmsnorm/dx . dy) ) (dresid optional).
 * dy is f16 [rows, cols]; x is the forward input s; dgamma_part is f32
 * [nparts, cols] with nparts = jx_rmsnorm_bwd_parts(rows) (one per SM of the
 * current device, at most 296, fewer for short inputs); reduce it with
 * jx_rmsnorm_dgamma_reduce. */
int jx_rmsnorm_bwd_parts(int64_t rows);
int jx_rmsnorm_bwd(const void* dy, const void* x, const float* rstd, const float* gamma, const void* dresid,
                   void* dx, float* dgamma_part, int64_t rows, int cols, jx_stream_t stream);
/* dgamma (+)= sum over parts (accumulate != 0 adds to the existing value). */
int jx_rmsnorm_dgamma_reduce(const float* dgamma_part, int nparts, int cols, float* dgamma, int accumulate,
                             jx_stream_t stream);
/* ---- LayerNorm (model_torch.py:12-15, norm_type "layernorm"; fp32 under autocast) ----
 * y = f16((x - mean) * rstd * gamma + beta) with fp32 statistics of the f16 row x
 * (biased variance, rstd = 1/sqrt(var + eps)); beta may be NULL (norm_bias false).
 * mean, rstd: f32 [rows], saved for the backward. cols: multiple of 8, <= 4096. */
int jx_layernorm_fwd(const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                     int64_t rows, int cols, float eps, jx_stream_t stream);
/* dx = f16(f16(layer-norm input gradient in fp32) + dresid) (dresid may be NULL);
 * dgamma_part / dbeta_part: f32 [nparts, cols], nparts = jx_rmsnorm_bwd_parts(rows),
 * reduced with jx_rmsnorm_dgamma_reduce; dbeta_part may be NULL. */
int jx_layernorm_bwd(const void* dy, const void* x, const float* mean, const float* rstd, const float* gamma,
                     const void* dresid, void* dx, float* dgamma_part, float* dbeta_part, int64_t rows, int cols,
                     jx_stream_t stream);
/* RMSNorm backward that allocates nothing and needs no scratch from the caller:
 * for callers that cannot allocate device memory (a runtime bound through this
 * C ABI without a device allocator of its own, or one held to a fixed memory
 * budget that must not call cudaMalloc/cudaFree, which can synchronise the
 * device). Same results as jx_rmsnorm_bwd followed by jx_rmsnorm_dgamma_reduce
 * into `dgamma` (accumulate != 0 adds to it). The dgamma partials live in a
 * fixed device array of 296 x 1024 floats (1.16 MiB) inside the library, held
 * on every GPU that loads it until the process exits; cols above 1024 are
 * rejected with JX_ERR_INVALID. The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress with the device current), so
 * make a first call on each device before any stream capture. The looked-up
 * address is cached per device and keyed on the CUDA context, so after a
 * device reset (cudaDeviceReset) the next call looks it up again. All calls share
 * the one array: calls that overlap on the GPU (e.g. on two streams at once)
 * race; nothing from an earlier call is read, so no clearing is needed.
 * This entry point has no counterpart in the reference project. */
int jx_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* rstd, const float* gamma, const void* dresid,
                           void* dx, float* dgamma, int accumulate, int64_t rows, int cols, jx_stream_t stream);

/* ---- Embedding (model_torch.py:89-93): out[t] = table16[ids[t]] ----
 * Ids outside [0, vocab) produce zero rows and set the device status word. */
int jx_embed_fwd(const int64_t* ids, int64_t ntok, const void* table16, int64_t vocab, int cols, void* out16,
                 jx_stream_t stream);
/* dtable[ids[t]] += f32(dout16[t]) (fp32 atomics). */
int jx_embed_bwd(const int64_t* ids, int64_t ntok, const void* dout16, int64_t vocab, int cols, float* dtable,
                 jx_stream_t stream);

/* ---- Dense GEMMs on tcgen05 (fp16 operands, fp32 accumulation in TMEM) ----
 * Logical product acc[m][n] = sum_k A[m][k] * B[n][k].
 * a_mn_major = 0: A stored [M][K] (row stride lda); 1: A stored [K][M].
 * b_mn_major = 0: B stored [N][K] (row stride ldb); 1: B stored [K][N].
 * All leading dimensions must be multiples of 8, bases 16-byte aligned,
 * N a multiple of 8. */
/* C16[m][n] = f16(acc) or, with resid != NULL, f16(resid[m][n] + f16(acc)). */
int jx_gemm_f16(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major, int M, int N,
                int K, void* C, int64_t ldc, const void* resid, int64_t ld_resid, jx_stream_t stream);
/* Fused q/k/v projection with RoPE (model_torch.py:18-25, 41-44): C = [q|k|v] f16
 * [M, 3*hidden], with the first 2*hidden columns rotated per head_dim-wide
 * head (half-split pairs) at position (row % seq_len), using tables
 * cos/sin f32 [seq_len, head_dim/2]. W is the stacked [3*hidden, K] f16 weight. */
int jx_gemm_qkv_rope(const void* X, int64_t ldx, const void* W, int M, int hidden, int K, void* C, int64_t ldc,
                     const float* rope_cos, const float* rope_sin, int seq_len, int head_dim, jx_stream_t stream);
/* SwiGLU forward (model_torch.py:59-60): Wgu is [gate; up] f16 [2F, K];
 * writes gate = f16(X Wg^T), up = f16(X Wu^T), act = f16(f16(silu(gate)) * up),
 * each f16 [M, F] with leading dimension ld_out. */
int jx_gemm_swiglu_fwd(const void* X, int64_t ldx, const void* Wgu, int M, int F, int K, void* gate, void* up,
                       void* act, int64_t ld_out, jx_stream_t stream);
/* SwiGLU backward through the down projection: dact = f16(dY Wd) with dY f16
 * [M, K] and Wd f16 [K, F]; then dgu[:, 0:F] = d gate, dgu[:, F:2F] = d up
 * (f16 [M, 2F], leading dimension ld_dgu). */
int jx_gemm_swiglu_bwd(const void* dY, int64_t lddy, const void* Wd, int M, int F, int K, const void* gate,
                       const void* up, int64_t ld_gu, void* dgu, int64_t ld_dgu, jx_stream_t stream);
/* Weight gradient: G[n][k] (+)= f32( f16( sum_t dY[t][n] * X[t][k] ) ) with
 * dY f16 [T, N], X f16 [T, K], G f32 [N, K] (leading dimension ldg).
 * The product is rounded to f16 before it is added, as an fp16 autocast
 * Linear's weight gradient is. `splits` > 1 splits the T reduction across
 * CTAs, whose fp32 partials are added into one accumulator (zeroed by the call)
 * before the f16 rounding; it needs `workspace` of
 * jx_gemm_wgrad_workspace_bytes(N, K, splits) = N*K*4 bytes. */
int64_t jx_gemm_wgrad_workspace_bytes(int N, int K, int splits);
/* Kernel choice for all GEMM entry points: 0 (default) runs the 2-SM
 * kernel (a CTA pair per 256 x 256 tile, tcgen05 cta_group::2) whenever M
 * spans at least two 128-row blocks and the 1-SM kernel otherwise; 1 forces
 * the 1-SM kernel, 2 the 2-SM kernel. A test / diagnostic switch: it is kept
 * per host thread (it affects only calls made from the thread that set it),
 * and both kernels give identical results. */
int jx_gemm_set_mode(int mode);
/* Failure-detection test hook (no counterpart in the reference: it exercises this
 * library's bounded waits). Runs the 1-SM GEMM kernel on one 128 x 256 x 64 tile
 * (A [128][64], B [256][64], C [128][256] f16) with its TMA loads withheld, so the
 * MMA thread's wait for the first operand stage expires after wait_budget_cycles
 * (clock64 cycles, at most 2^32; the production kernels allow 2^32, about 2 s).
 * The kernel then records 102 in the device status word (jx_device_status), every
 * warp leaves through the normal teardown and C is left unwritten; the context
 * stays usable. */
int jx_gemm_wait_test(const void* A, const void* B, void* C, int64_t wait_budget_cycles, jx_stream_t stream);
int jx_gemm_wgrad(const void* dY, int64_t lddy, const void* X, int64_t ldx, int T, int N, int K, float* G,
                  int64_t ldg, int accumulate, int splits, void* workspace, jx_stream_t stream);

/* ---- Causal attention (model_torch.py:48, SDPA is_causal=True) ----
 * qkv: f16 [B*T, 3*H*D] rows (q | k | v, head h at column h*D of each part).
 * out: f16 [B*T, H*D]. lse: f32 [B, H, T] (natural-log logsumexp of the scaled scores).
 * D must be 64; T a multiple of 256 (forward) / 128 (backward).
 * `workspace` is caller scratch of jx_attn_fwd_workspace_bytes(B, T, H, D) bytes (the
 * work counter of the persistent kernel, cleared by the call on `stream`); calls that
 * may run concurrently need separate workspaces. */
int64_t jx_attn_fwd_workspace_bytes(int B, int T, int H, int D);
int jx_attn_fwd(const void* qkv, void* out, float* lse, void* workspace, int B, int T, int H, int D, float scale,
                jx_stream_t stream);
/* Backward: writes dqkv f16 [B*T, 3*H*D]. `workspace` is caller scratch of
 * jx_attn_bwd_workspace_bytes(B, T, H, D) bytes (the row sums dO.O and an fp32
 * dQ accumulator; the call clears what must start at zero).
 * If rope_cos/rope_sin are non-NULL the q/k gradients are rotated back
 * through RoPE (the inverse rotation) before they are stored. */
int64_t jx_attn_bwd_workspace_bytes(int B, int T, int H, int D);
int jx_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, void* workspace, void* dqkv,
                int B, int T, int H, int D, float scale, const float* rope_cos, const float* rope_sin,
                jx_stream_t stream);

/* ---- Incremental decoding (generate_torch.py:279-285 re-runs model(tokens)[0, -1]) ----
 * Causal attention of one new token per sequence against a KV cache: qkv is the new token's
 * projection row (q | k | v, RoPE applied; row b at qkv + b*ld_qkv), kcache / vcache hold
 * positions 0 .. len-2 (row stride ld_cache, sequence stride cache_batch_stride); the new k / v are
 * appended at position len-1. out: f16 [B, H*64] (row stride ld_out). workspace: caller scratch of
 * jx_attn_decode_workspace_bytes(B, H, max_len) bytes with max_len >= len. head_dim must be 64.
 * If len_dev is non-NULL the length is read from that device int (for CUDA-graph replays) and `len`
 * is only its upper bound, which sets the grid. */
int64_t jx_attn_decode_workspace_bytes(int B, int H, int max_len);
int jx_attn_decode(const void* qkv, int64_t ld_qkv, void* kcache, void* vcache, int64_t ld_cache,
                   int64_t cache_batch_stride, int B, int len, const int* len_dev, int H, int D, float scale,
                   void* workspace, void* out, int64_t ld_out, jx_stream_t stream);

/* ---- Packed corpus rows (data.py:233-379 row filling, pretrain_torch.py:38-40 widening) ----
 * out: int64 [rows, width]. Row r is covered by runs[row_start[r] .. row_start[r+1]) (int64 triples
 * dst column, src token index into `tokens` (uint16 [ntokens]) or -(eod + 1), count), sorted by dst.
 * A column outside every run, or a src beyond ntokens, writes -1 and records a device status. */
int jx_pack_rows(const void* tokens, int64_t ntokens, const int64_t* runs, const int32_t* row_start, int rows,
                 int width, int64_t* out, jx_stream_t stream);

/* ---- Cross-entropy over f16 logits (model_torch.py:102-104) ----
 * Per row: lse = log(sum exp(logit)), loss = lse - logit[target]; rows whose
 * target == ignore_index give loss 0 and are excluded from the mean. A target
 * outside [0, vocab) that is not ignore_index (torch rejects it) gives a NaN
 * row loss, so the mean is NaN, and sets the device status word to 202
 * (jx_device_status); jx_ce_bwd gives such a row a zero gradient. */
int jx_ce_fwd(const void* logits16, int64_t rows, int vocab, int64_t ld, const int64_t* targets, int64_t ignore_index,
              float* lse, float* row_loss, jx_stream_t stream);
/* The tied head with the cross-entropy statistics in its epilogue: C = A B^T as jx_gemm_f16 (A [M, K],
 * B [N, K], both K-major, no residual) and parts [M][ceil(N/128)] of float pairs (max, sum exp(v - max))
 * over each 128-column block of the f16 logits v. jx_ce_fwd_parts then gives what jx_ce_fwd gives without
 * reading the logits again (nblk = ceil(vocab / 128); only the target logit is read). */
int jx_gemm_f16_ce_parts(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, void* C,
                         int64_t ldc, void* parts, jx_stream_t stream);
int jx_ce_fwd_parts(const void* parts, int nblk, const void* logits16, int64_t rows, int vocab, int64_t ld,
                    const int64_t* targets, int64_t ignore_index, float* lse, float* row_loss, jx_stream_t stream);
/* loss_sum_count[0] = sum of row losses, [1] = number of counted rows,
 * [2] = [0]/[1], the mean loss (deterministic order); accumulate != 0 adds
 * to the existing sum and count. The buffer holds 3 floats. */
int jx_ce_loss(const float* row_loss, const int64_t* targets, int64_t ignore_index, int64_t rows,
               float* loss_sum_count, int accumulate, jx_stream_t stream);
/* In place: logits16 <- f16( (exp(logit - lse) - onehot(target)) * g ),
 * g = (*grad_loss) / (*count), i.e. the gradient of mean CE scaled by the
 * incoming gradient of the loss. */
int jx_ce_bwd(void* logits16, int64_t rows, int vocab, int64_t ld, const int64_t* targets, int64_t ignore_index,
              const float* lse, const float* grad_loss, const float* count, jx_stream_t stream);

/* ---- GradScaler unscale + inf check + global norm, then AdamW ----
 * Stats over a flat gradient buffer (grad_is_f16 selects f16 or f32 input):
 * partial[b] = sum over the block's slice of (g*inv_scale)^2, found_inf set to 1
 * if any element is not finite. nparts = jx_grad_stats_parts(n).
 * unscaled_out (f32 [n], may be NULL, may alias an f32 grad) receives
 * g*inv_scale: GradScaler.unscale_ leaves unscaled gradients in `.grad`, so a
 * caller's own torch.nn.utils.clip_grad_norm_ sees what it sees in the
 * reference (pretrain_torch.py:218-219). */
int jx_grad_stats_parts(int64_t n);
int jx_grad_stats(const void* grad, int grad_is_f16, int64_t n, const float* inv_scale, float* partial,
                  float* found_inf, float* unscaled_out, jx_stream_t stream);
/* total_norm = sqrt(sum partial); clip = min(max_norm/(total_norm+1e-6), 1)
 * (clip_grad_norm_ semantics; max_norm <= 0 disables clipping: clip = 1).
 * out[0] = total_norm, out[1] = clip coefficient. */
int jx_grad_finalize(const float* partial, int nparts, float max_norm, float* out, jx_stream_t stream);
/* One decoupled-weight-decay Adam step over flat buffers, skipped entirely
 * (no writes, step count unchanged) when *found_inf != 0. Gradient used:
 * (g * inv_scale) * clip (either pointer may be NULL for 1). step_state is a
 * device f32[4]: [0] holds the number of completed updates and is advanced on
 * the device before the bias corrections 1-beta^step are formed, as torch's
 * fused AdamW advances its per-parameter step tensors; [1..3] are scratch.
 * p16 (optional) receives f16(p_new), the weight copy the GEMMs read. */
int jx_adamw_step(float* p, const void* grad, int grad_is_f16, float* m, float* v, void* p16, int64_t n,
                  const float* inv_scale, const float* clip, const float* found_inf, float* step_state, float lr,
                  float beta1, float beta2, float eps, float weight_decay, jx_stream_t stream);
/* GradScaler.update(): if found_inf: scale *= backoff, tracker = 0; else
 * tracker += 1 and at growth_interval scale *= growth, tracker = 0. */
int jx_scaler_update(float* scale, int* growth_tracker, const float* found_inf, float growth_factor,
                     float backoff_factor, int growth_interval, jx_stream_t stream);

/* ---- Utilities ---- */
/* dst16[i] = f16(src32[i]). */
int jx_cast_f32_f16(const float* src, void* dst16, int64_t n, jx_stream_t stream);
/* dst16 [cols, rows] = transpose(src16 [rows, cols]). */
int jx_transpose_f16(const void* src, void* dst, int64_t rows, int64_t cols, jx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* JISHUI_B200_H_ */
