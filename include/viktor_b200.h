/*
 * viktor_b200 -- C ABI of the B200 (sm_100a) decoder inference kernels.
 *
 * Every entry point takes plain device pointers, sizes and strides, launches on the given CUDA stream
 * (cudaStream_t passed as void*, NULL = legacy default stream) and returns an int status.  Nothing here
 * allocates device memory or synchronises the host, so every call can be captured into a CUDA graph; the
 * caller owns all buffers, including the decode-attention workspace.
 *
 * Data types: "bf16" buffers hold __nv_bfloat16, "f32" float, "i32" int32_t, "i64" int64_t, "u8" uint8_t.
 * Layouts are row-major and contiguous unless a stride is given.  The decoder geometry the kernels are built
 * for is the Viktor decoder: d_model 512, 8 query heads, 2 KV heads, head_dim 64 (GQA group 4).
 *
 * Each function names the reference interface (GHSSHG/Viktor, path:line) whose semantics it implements.
 */
#ifndef VIKTOR_B200_H
#define VIKTOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------------------------------------- */
#define VK_OK 0
#define VK_ERR_ARG (-1)         /* unsupported shape, null or misaligned pointer, bad size */
#define VK_ERR_CUDA (-2)        /* a CUDA launch or runtime call failed */
#define VK_ERR_UNSUPPORTED (-3) /* geometry the kernels are not built for */

/* Device error word bits (set by kernels, read with vk_read_device_errors). */
#define VK_DEVERR_WAIT_FULL 1u   /* a consumer gave up waiting for a TMA stage */
#define VK_DEVERR_WAIT_EMPTY 2u  /* a producer gave up waiting for a free stage */
#define VK_DEVERR_WAIT_ACCUM 4u  /* an epilogue gave up waiting for the tensor-core accumulator */
#define VK_DEVERR_BOUNDS 8u      /* an index (token, position, cache row) was out of range; access skipped */

/* Library version as major*10000 + minor*100 + patch. */
int vk_version(void);

/* Reads (and with clear != 0, clears) the device error word of the current device.  Synchronous. */
int vk_read_device_errors(uint32_t* bits, int clear);

/* Enables (1) or disables (0) programmatic dependent launch between consecutive kernels.  Default 1. */
int vk_set_pdl(int enable);

/* Test hook of the failure path (no reference counterpart; the reference's inference path has no device-side
 * waits).  Launches one CTA whose thread waits on an mbarrier that nothing arrives on, bounded by limit_ns
 * (0 < limit_ns <= 1e9): the wait runs out, the kernel sets VK_DEVERR_WAIT_FULL in the device error word,
 * stores the nanoseconds it waited in *waited_ns (device, u64, may be NULL) and returns, leaving the context
 * usable.  No copy is in flight while it waits. */
int vk_test_bounded_wait(uint64_t limit_ns, unsigned long long* waited_ns, void* stream);

/* ---- fused row ops: viktor/triton_ops.py ------------------------------------------------------------------ */

/* viktor/triton_ops.py:34-40 add_rmsnorm.  x [n, d] bf16 (updated in place by += delta when delta != NULL),
 * w [d] bf16, h [n, d] bf16 out: h = RMSNorm(x) * w.  d in {512}. */
int vk_add_rmsnorm(void* x, const void* delta, const void* w, void* h, int64_t n, int d, float eps,
                   void* stream);

/* viktor/triton_ops.py:163-169 embed_rmsnorm.  tok [n] i64, emb [V, d] bf16, w [d]; x, h [n, d] bf16 out. */
int vk_embed_rmsnorm(const int64_t* tok, const void* emb, int64_t vocab, const void* w, void* x, void* h,
                     int64_t n, int d, float eps, void* stream);

/* viktor/triton_ops.py:94-108 qkv_rope_cache.  qkv [n, (H + 2 Hkv) * 64] bf16; q_norm_w, k_norm_w [64] bf16;
 * cos, sin [rope_len, 32] f32; pos, seq [n] i32 (cache position and cache row of each token); rope_pos [n] i32
 * or NULL (= pos); q [n, H, 64] bf16 out; k_cache, v_cache: one layer, element (row, p, kvh, d) at
 * row * stride_cb + p * stride_cs + kvh * 64 + d; k_out, v_out [n, Hkv, 64] bf16 or NULL. */
int vk_qkv_rope_cache(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos,
                      const float* sin, int rope_len, const int32_t* pos, const int32_t* rope_pos,
                      const int32_t* seq, void* q, void* k_cache, void* v_cache, void* k_out, void* v_out,
                      int64_t n, int64_t stride_cb, int64_t stride_cs, int cache_rows, int cache_len, float eps,
                      int n_heads, int n_kv_heads, int head_dim, void* stream);

/* viktor/triton_ops.py:138-146 linear, on tcgen05 tensor cores.  x [M, K] bf16, w [N, K] bf16 (nn.Linear
 * layout).  swiglu = 0: y [M, N] (bf16, or f32 when out_f32).  swiglu = 1: w is gate_up with N = 2F rows (gate
 * rows first) and y [M, F] bf16 = silu(gate) * up.  K a multiple of 64; with swiglu, F a multiple of 64. */
int vk_linear(const void* x, const void* w, void* y, int64_t M, int N, int K, int swiglu, int out_f32,
              void* stream);

/* viktor/triton_ops.py:223-229 swiglu.  gu [n, 2F] bf16 (gate | up) -> out [n, F] bf16. */
int vk_swiglu(const void* gu, void* out, int64_t n, int F, void* stream);

/* viktor/triton_ops.py:200-209 greedy_update (+ viktor/engine.py:79-89 _select at temperature 0).
 * logits [B, V] f32 (row stride ld_logits); bias [V] f32; is_tail, is_homo [V] u8; tok, run, pos, plen,
 * rope_off [B] i64; out [B, out_cols] i64 (row stride out_stride); pos32, seqlens, rpos32 [B] i32.
 * When emb != NULL, additionally writes the next decode step's input: x = emb[new tok] ([B, 512] bf16) and its
 * per-64-column sums of squares ssq ([B, 8] f32), which the first layer's folded RMSNorm consumes (the
 * embed_rmsnorm of viktor/fast_decoder.py:80-81, fused). */
int vk_greedy_update(const float* logits, int64_t ld_logits, const float* bias, const uint8_t* is_tail,
                     const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run, int64_t* pos,
                     const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                     int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos,
                     int pad, const void* emb, void* x, float* ssq, void* stream);

/* viktor/engine.py:79-89 _select at temperature > 0 (Gumbel-max sampling) + the state advance of
 * vk_greedy_update.  Arguments as vk_greedy_update, plus noise [B, V] f32 uniform draws in [0, 1) (row stride
 * ld_noise >= V; the torch.rand_like of viktor/engine.py:82, drawn by the caller) and temperature > 0:
 * score = (logits + bias) / temperature - log(-log(max(noise, 1e-20))), argmax (ties to the lower index),
 * then the grammar. */
int vk_sample_update(const float* logits, int64_t ld_logits, const float* bias, const uint8_t* is_tail,
                     const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run, int64_t* pos,
                     const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                     int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos,
                     int pad, const void* emb, void* x, float* ssq, const float* noise, int64_t ld_noise,
                     float temperature, void* stream);

/* ---- attention: viktor/decode_attention.py, flash_attn calls of viktor/fast_decoder.py ------------------- */

/* Workspace bytes vk_decode_attention needs for nq queries over a cache of S positions. */
size_t vk_decode_attention_workspace_bytes(int nq, int S);

/* viktor/decode_attention.py:41-53 decode_attention (and flash_attn_with_kvcache, viktor/fast_decoder.py:88).
 * q [nq, 8, 64] bf16; k_cache/v_cache: one layer, (row, p, kvh, d) at row * stride_kb + p * stride_ks +
 * kvh * 64 + d with stride_ks >= 128; query i attends cache row row0 + i, positions [0, lengths[i]),
 * 1 <= lengths[i] <= S (i32); out [nq, 8, 64] bf16.  workspace: vk_decode_attention_workspace_bytes(nq, S)
 * bytes, 16-byte aligned, ZERO-FILLED once before first use (it holds per-query tickets that every call
 * returns to zero). */
int vk_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* lengths,
                        void* out, int nq, int row0, int cache_rows, int S, int64_t stride_kb, int64_t stride_ks,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---- opt-in INT8 prefix KV (the reference's analysis.md:95 proposal; no reference kernel exists) ------------
 * The prefix of a chunk (its prefilled positions) is written once; an int8 copy halves the bytes decode
 * attention reads for it, while generated tokens stay bf16.  Per channel c of one layer and row (both KV heads,
 * 128 channels): s_c = max_{p < start} |x[p][c]| / 127, stored byte u = clamp(rint(x / s_c), -127, 127) + 128.
 * k8 [cache_rows][S8][128] u8 (position-major), v8t [cache_rows][S8 / 128][128][128] u8 (channel-major within
 * each tile of 128 positions: byte (c, p) of a row at (p / 128) * 16384 + c * 128 + p % 128), sk/sv
 * [cache_rows][128] f32; S8 a multiple of 128. */

/* Quantizes positions [0, starts[i]) (0 <= starts[i] <= min(S, S8), i32) of cache row row0 + i, i < n, of one
 * layer (same cache layout as vk_decode_attention) into k8/v8t/sk/sv. */
int vk_kv_quantize(const void* k_cache, const void* v_cache, int cache_rows, int S, int64_t stride_kb,
                   int64_t stride_ks, const int32_t* starts, int row0, int n, void* k8, void* v8t, float* sk,
                   float* sv, int S8, void* stream);

/* Workspace bytes vk_decode_attention_i8 needs (zero-filled once before first use, like vk_decode_attention's). */
size_t vk_decode_attention_i8_workspace_bytes(int nq, int S8, int max_tail);

/* vk_decode_attention with positions [0, starts[i]) of query i read from the int8 copy (vk_kv_quantize) and
 * [starts[i], lengths[i]) from the bf16 cache.  Requires 0 <= starts[i] < lengths[i] <= S, starts[i] <= S8 and
 * lengths[i] - starts[i] <= max_tail (violations set the device error flag and skip the query). */
int vk_decode_attention_i8(const void* q, const void* k_cache, const void* v_cache, const void* k8,
                           const void* v8t, const float* sk, const float* sv, const int32_t* starts,
                           const int32_t* lengths, void* out, int nq, int row0, int cache_rows, int S,
                           int64_t stride_kb, int64_t stride_ks, int S8, int max_tail, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Decode attention for callers that cannot allocate device memory.  No counterpart in the reference: it is
 * vk_decode_attention with its split-K workspace taken from a fixed array inside this library instead of from
 * the caller.  Meant for hosts that hand a kernel only its inputs and outputs and have no way to obtain a
 * workspace: plugin or custom-op interfaces of inference servers that own all device memory, FFI callers
 * without a CUDA allocator of their own, code that must not allocate once serving has started.
 * Limits: nq <= 256 queries and S <= 4096 cache positions; larger requests return VK_ERR_ARG with a message on
 * stderr.  The array (8.25 MiB) lives on every GPU that loads the library until the process exits.  The first
 * call on a device looks up the array's device address and keeps it for the life of the process; make that first
 * call before any stream capture, and do not use this entry point on a device after cudaDeviceReset (the kept
 * address would no longer be mapped).  `stream` must belong to the current device (VK_ERR_ARG otherwise).
 * Every call clears the per-query tickets it uses and then shares the device's array with all other calls on
 * that device: calls whose executions overlap on the same GPU (for example on concurrent streams) corrupt each
 * other's results — issue them in order on one stream per device.  Each device has its own array. */
int vk_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* lengths,
                                void* out, int nq, int row0, int cache_rows, int S, int64_t stride_kb,
                                int64_t stride_ks, void* stream);

/* Test hook: fills the current device's noalloc tickets with a nonzero byte pattern on `stream`, the state an
 * aborted call could leave behind, so that a test can check that the next vk_decode_attention_noalloc clears
 * them (stale tickets would keep every split from merging and leave the output unwritten). */
int vk_test_noalloc_poison(void* stream);

/* flash_attn_varlen_func(q, k, v, cu, cu, max_len, max_len, causal=True) of viktor/fast_decoder.py:73, with K
 * and V read from the cache rows the prefill just wrote.  q, out [n_tok, 8, 64] bf16 packed by cu_seqlens
 * [nseq + 1] (i32, device); sequence b attends cache row row0 + b, positions [0, T_b).  max_seqlen = max T_b. */
int vk_prefill_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cu_seqlens,
                         int nseq, int max_seqlen, int64_t n_tok, int row0, int cache_rows, int S,
                         int64_t stride_kb, int64_t stride_ks, void* out, void* stream);

/* ---- tensor-core projections with fused epilogues (the B200 forms of viktor/fast_decoder.py:33-60) -------
 *
 * Folded RMSNorm.  The decoder's pre-norm GEMMs compute (RMSNorm(x) * w) . W^T.  Here they run on the residual x
 * itself with w folded into W's columns once (W' = bf16(W * w), vk_fold_norm_weight), and the epilogue scales row
 * i by rsqrt(sum(ssq[i, 0..7]) / 512 + eps).  ssq [M, 8] f32 holds the sums of squares of the eight 64-column
 * blocks of each 512-wide row of x; vk_linear_residual, vk_row_ssq and the fused greedy step produce it. */

/* (RMSNorm(x) * w) . W^T with W' = W diag(w) given (w_folded): x [M, 512] bf16, ssq [M, 8] f32.  Output as in
 * vk_linear (swiglu / out_f32).  Replaces add_rmsnorm's h followed by linear (viktor/fast_decoder.py:56,
 * viktor/engine.py:96). */
int vk_linear_rmsnorm(const void* x, const float* ssq, float eps, const void* w_folded, void* y, int64_t M, int N,
                      int K, int swiglu, int out_f32, void* stream);

/* q, K/V <- (RMSNorm(x) * w_attn) . W_qkv^T followed by the qkv_rope_cache epilogue (arguments as in
 * vk_qkv_rope_cache; eps is the QK-norm epsilon; q_norm_w and k_norm_w 16-byte aligned).  ssq NULL: x is used
 * as given (w_qkv not folded).
 * Replaces add_rmsnorm + linear + qkv_rope_cache of viktor/fast_decoder.py:41-47. */
int vk_linear_qkv_rope_cache(const void* x, const float* ssq, float norm_eps, const void* w_qkv,
                             const void* q_norm_w, const void* k_norm_w, const float* cos, const float* sin,
                             int rope_len, const int32_t* pos, const int32_t* rope_pos, const int32_t* seq, void* q,
                             void* k_cache, void* v_cache, void* k_out, void* v_out, int64_t M, int64_t stride_cb,
                             int64_t stride_cs, int cache_rows, int cache_len, float eps, int n_heads,
                             int n_kv_heads, void* stream);

/* x += bf16(a [M, K] . w [512, K]^T) in place (bf16), and ssq_out [M, 8] f32 = sums of squares of the new rows'
 * 64-column blocks.  The residual half of linear + add_rmsnorm (viktor/fast_decoder.py:55,57-59). */
int vk_linear_residual(const void* a, const void* w, void* x, float* ssq_out, int64_t M, int K, void* stream);

/* viktor/fast_decoder.py:55,57-59 as one call: x += a . w^T (bf16) and h = RMSNorm(x) * norm_w ([M, 512] bf16).
 * ssq_scratch [M, 8] f32 receives the row sums of squares.  K a multiple of 64. */
int vk_linear_add_rmsnorm(const void* a, const void* w, void* x, const void* norm_w, void* h, float* ssq_scratch,
                          int64_t M, int K, float eps, void* stream);

/* y = act(x [M, K] . w [N, K]^T + bias) as bf16; act 0 = identity, 1 = GELU (erf); N a multiple of 64.  Row i of
 * the result goes to row row_map[i] of y (row_map NULL = identity; ldy = row stride of y).  The projector of
 * viktor/model.py:35 and the packed-prefill scatter of viktor/engine.py:163-164. */
int vk_linear_bias_act(const void* x, const void* w, const void* bias, void* y, int64_t ldy,
                       const int32_t* row_map, int64_t M, int N, int K, int act, void* stream);

/* ssq [n, 8] f32 = sums of squares of the eight 64-column blocks of each row of x [n, 512] bf16. */
int vk_row_ssq(const void* x, float* ssq, int64_t n, int d, void* stream);

/* h = bf16(x * rsqrt(sum(ssq[row]) / 512 + eps) * w): RMSNorm from precomputed sums of squares. */
int vk_ssq_rmsnorm(const void* x, const float* ssq, const void* w, void* h, int64_t n, int d, float eps,
                   void* stream);

/* out [N, K] bf16 = bf16(w [N, K] * norm_w [K]): folds an RMSNorm weight into the GEMM that consumes it. */
int vk_fold_norm_weight(const void* w, const void* norm_w, void* out, int64_t N, int K, void* stream);

/* ---- layout helpers --------------------------------------------------------------------------------------- */
int vk_cast_f32_bf16(const float* src, void* dst, int64_t n, void* stream);
/* dst[i, :] = src[idx[i], :] for rows of row_bytes (multiple of 16), src has src_rows rows. */
int vk_gather_rows(const void* src, const int64_t* idx, void* dst, int64_t n, int row_bytes, int64_t src_rows,
                   void* stream);
/* dst[dst_idx[i], :] = src[src_idx[i], :] for rows of row_bytes (multiple of 16); a NULL index is the
 * identity.  Indices are i64 and bounds-checked against src_rows / dst_rows. */
int vk_copy_rows(const void* src, const int64_t* src_idx, int64_t src_rows, void* dst, const int64_t* dst_idx,
                 int64_t dst_rows, int64_t n, int row_bytes, void* stream);
/* The decode head in one kernel: lm_head + selection + state advance + next embedding.  x_final [B, 512] bf16
 * and ssq_final [B, 8] f32 are the final residual and its per-64-column sums of squares; head_w [V, 512] bf16
 * is the lm_head with the final RMSNorm weight folded in (logits = rsqrt(mean(x^2) + eps) * x . head_w^T, fp32,
 * as the fp32-output linear of viktor/engine.py:95-96); V <= 512.  The remaining arguments are those of
 * vk_sample_update; noise = NULL selects greedily (vk_greedy_update).  x / ssq may alias x_final / ssq_final
 * (each row is read before it is overwritten with the next token's embedding).
 * limit [B] i64 or NULL: per-row output cap; the token of output column >= limit[b] becomes EOS (a stand-in for
 * a model that ends its read there; the reference's grammar has no such rule, NULL keeps it exact).
 * shrink_done != 0: a row whose new token is EOS or PAD gets seqlens = 1 instead of pos + 1.  That row's next
 * output is PAD whatever the step computes (viktor/engine.py:88), so its attention then reads one cached
 * position instead of its whole row; no output token changes. */
int vk_head_select(const void* x_final, const float* ssq_final, float eps, const void* head_w, const float* bias,
                   const uint8_t* is_tail, const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run,
                   int64_t* pos, const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                   int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos, int pad,
                   const void* emb, void* x, float* ssq, const float* noise, int64_t ld_noise, float temperature,
                   const int64_t* limit, int shrink_done, void* stream);

/* The packed prefill layout of viktor/engine.py:145-159, built on the device from the prefix lengths of one
 * sub-batch (lens [n] i32 on the device, 1 <= n <= 4096; total = sum(lens) + n, known to the caller).
 * Sequence b occupies packed rows cu[b] .. cu[b+1]-1: its lens[b] frames, then BOS.  Writes cu [n+1] i32,
 * frame_idx [sum(lens)] i32 (packed row of each frame; NULL allowed when there are no frames), last [n] i64
 * (BOS rows), pos / seq [total] i32 (position in the sequence, cache row row0 + b), rpos [total] i32
 * (pos * pos_scale; NULL to skip) and lengths [n] i32 (lens + 1).  If the lengths do not add up to total (or
 * one is negative) nothing is written and the device error word records a range error. */
int vk_prefill_plan(const int32_t* lens, int n, int row0, int pos_scale, int64_t total, int32_t* cu,
                    int32_t* frame_idx, int64_t* last, int32_t* pos, int32_t* seq, int32_t* rpos, int32_t* lengths,
                    void* stream);
/* x[rows[i], :] = emb[token, :] (d bf16 values per row). */
int vk_scatter_embed(void* x, const int64_t* rows, int64_t n, int64_t x_rows, const void* emb, int64_t token,
                     int d, void* stream);


/* ---- host-side stitching of chunk calls (scripts/basecall_viktor.py:31-108; no device work) -----------------
 * Edit-distance alignment with edlib's semantics (the reference's aligner): mode 0 NW (global), 1 SHW (query
 * against a prefix of the target), 2 HW (query against an infix); k >= 0 caps the distance (above it: -1).
 * out[3] = distance, start and end (inclusive, -1: no target base) of the first best location; with
 * cigar != NULL (cigar_cap >= qlen + tlen + 1) the alignment path as extended CIGAR operations, one character
 * per column ('=', 'X', 'I' = query base not in the target, 'D' = target base not in the query), NUL-ended. */
int vk_align(const char* query, int qlen, const char* target, int tlen, int mode, int k, int* out, char* cigar,
             int cigar_cap);

/* scripts/basecall_viktor.py:31-54 overlap_cut: calls a, b of adjacent chunks sharing ov_frames encoder frames,
 * rate = bases per frame of a; keep a[:cut[0]] + b[cut[1]:]. */
int vk_overlap_cut(const char* a, int la, const char* b, int lb, int ov_frames, double rate, int* cut);

/* scripts/basecall_viktor.py:96-108 stitch: the n calls of one read, concatenated (call i is
 * calls[offsets[i], offsets[i + 1])), spans [n][2] their (start, end) samples, stride samples per encoder frame.
 * Writes the read's sequence to out (cap bytes) and its length to out_len; out == NULL only reports the length. */
int vk_stitch(const char* calls, const int64_t* offsets, const int64_t* spans, int n, int stride, char* out,
              int64_t cap, int64_t* out_len);

#ifdef __cplusplus
}
#endif

#endif /* VIKTOR_B200_H */
