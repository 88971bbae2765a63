// Row-wise kernels of the decoder path: RMSNorm variants, the standalone QK-norm/RoPE/cache op, SwiGLU,
// greedy token selection with its grammar, and small layout kernels (cast, gather, scatter).
// Rounding follows the reference: bf16 storage between ops, fp32 math inside an op
// (viktor/triton_ops.py:9).
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace ew {

VK_DEV void load8(const __nv_bfloat16* src, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z); v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
}

VK_DEV float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// One warp per row, d a multiple of 256 (each lane holds d/32 elements as 16-byte chunks).
// x = bf16(x + delta) in place (if delta), h = bf16(x * rsqrt(mean(x^2) + eps) * w)   (viktor/triton_ops.py:17-31)
// With tok != nullptr the row is first replaced by emb[tok[row]] (viktor/triton_ops.py:149-160).
template <int D>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(__nv_bfloat16* x, const __nv_bfloat16* delta,
                                                           const int64_t* tok, const __nv_bfloat16* emb,
                                                           int64_t vocab, const __nv_bfloat16* w,
                                                           __nv_bfloat16* h, int64_t n, float eps) {
  constexpr int PER = D / 32;  // elements per lane
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();
  if (row >= n) return;
  float v[PER];
  __nv_bfloat16* xr = x + row * D;
  const __nv_bfloat16* src = xr;
  if (tok) {
    int64_t t = tok[row];
    if (t < 0 || t >= vocab) {
      if (lane == 0) raise_error(ERR_BOUNDS);
      t = 0;
    }
    src = emb + t * D;
  }
#pragma unroll
  for (int c = 0; c < PER / 8; ++c) {
    const int col = (c * 32 + lane) * 8;
    uint4 u = *reinterpret_cast<const uint4*>(src + col);
    v[c * 8 + 0] = bf16_lo(u.x); v[c * 8 + 1] = bf16_hi(u.x);
    v[c * 8 + 2] = bf16_lo(u.y); v[c * 8 + 3] = bf16_hi(u.y);
    v[c * 8 + 4] = bf16_lo(u.z); v[c * 8 + 5] = bf16_hi(u.z);
    v[c * 8 + 6] = bf16_lo(u.w); v[c * 8 + 7] = bf16_hi(u.w);
    if (delta) {
      uint4 dd = *reinterpret_cast<const uint4*>(delta + row * D + col);
      v[c * 8 + 0] = bf16_round(v[c * 8 + 0] + bf16_lo(dd.x)); v[c * 8 + 1] = bf16_round(v[c * 8 + 1] + bf16_hi(dd.x));
      v[c * 8 + 2] = bf16_round(v[c * 8 + 2] + bf16_lo(dd.y)); v[c * 8 + 3] = bf16_round(v[c * 8 + 3] + bf16_hi(dd.y));
      v[c * 8 + 4] = bf16_round(v[c * 8 + 4] + bf16_lo(dd.z)); v[c * 8 + 5] = bf16_round(v[c * 8 + 5] + bf16_hi(dd.z));
      v[c * 8 + 6] = bf16_round(v[c * 8 + 6] + bf16_lo(dd.w)); v[c * 8 + 7] = bf16_round(v[c * 8 + 7] + bf16_hi(dd.w));
    }
    if (delta || tok) {
      uint4 o;
      o.x = pack_bf16x2(v[c * 8 + 0], v[c * 8 + 1]);
      o.y = pack_bf16x2(v[c * 8 + 2], v[c * 8 + 3]);
      o.z = pack_bf16x2(v[c * 8 + 4], v[c * 8 + 5]);
      o.w = pack_bf16x2(v[c * 8 + 6], v[c * 8 + 7]);
      *reinterpret_cast<uint4*>(xr + col) = o;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
  for (int c = 0; c < PER / 8; ++c) {
    const int col = (c * 32 + lane) * 8;
    uint4 wu = *reinterpret_cast<const uint4*>(w + col);
    float wv[8] = {bf16_lo(wu.x), bf16_hi(wu.x), bf16_lo(wu.y), bf16_hi(wu.y),
                   bf16_lo(wu.z), bf16_hi(wu.z), bf16_lo(wu.w), bf16_hi(wu.w)};
    uint4 o;
    o.x = pack_bf16x2(v[c * 8 + 0] * r * wv[0], v[c * 8 + 1] * r * wv[1]);
    o.y = pack_bf16x2(v[c * 8 + 2] * r * wv[2], v[c * 8 + 3] * r * wv[3]);
    o.z = pack_bf16x2(v[c * 8 + 4] * r * wv[4], v[c * 8 + 5] * r * wv[5]);
    o.w = pack_bf16x2(v[c * 8 + 6] * r * wv[6], v[c * 8 + 7] * r * wv[7]);
    *reinterpret_cast<uint4*>(h + row * D + col) = o;
  }
  pdl_launch_dependents();
}

// Standalone QK-norm + RoPE + cache write (viktor/triton_ops.py:52-108): one thread per (token, head).
__global__ void __launch_bounds__(128) qkv_rope_cache_kernel(
    const __nv_bfloat16* qkv, const __nv_bfloat16* qw, const __nv_bfloat16* kw, const float* cos, const float* sin,
    int rope_len, const int32_t* pos, const int32_t* rope_pos, const int32_t* seq, __nv_bfloat16* q,
    __nv_bfloat16* kc, __nv_bfloat16* vc, __nv_bfloat16* ko, __nv_bfloat16* vo, int64_t n, int64_t stride_cb,
    int64_t stride_cs, int cache_rows, int cache_len, float eps, int H, int HKV) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int NH = H + 2 * HKV;
  pdl_wait();
  if (gid >= n * NH) return;
  const int64_t t = gid / NH;
  const int hd = static_cast<int>(gid % NH);
  const int p = pos[t], rp = rope_pos ? rope_pos[t] : p, sq = seq[t];
  if (p < 0 || p >= cache_len || sq < 0 || sq >= cache_rows || rp < 0 || rp >= rope_len) {
    raise_error(ERR_BOUNDS);
    return;
  }
  float v[64];
  const __nv_bfloat16* src = qkv + (t * NH + hd) * 64;
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    uint4 u = *reinterpret_cast<const uint4*>(src + i);
    v[i] = bf16_lo(u.x); v[i + 1] = bf16_hi(u.x); v[i + 2] = bf16_lo(u.y); v[i + 3] = bf16_hi(u.y);
    v[i + 4] = bf16_lo(u.z); v[i + 5] = bf16_hi(u.z); v[i + 6] = bf16_lo(u.w); v[i + 7] = bf16_hi(u.w);
  }
  auto store64 = [&](__nv_bfloat16* dst) {
#pragma unroll
    for (int i = 0; i < 64; i += 8) {
      uint4 o;
      o.x = pack_bf16x2(v[i], v[i + 1]); o.y = pack_bf16x2(v[i + 2], v[i + 3]);
      o.z = pack_bf16x2(v[i + 4], v[i + 5]); o.w = pack_bf16x2(v[i + 6], v[i + 7]);
      *reinterpret_cast<uint4*>(dst + i) = o;
    }
  };
  if (hd < H + HKV) {
    const __nv_bfloat16* wn = hd < H ? qw : kw;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) ss += v[i] * v[i];
    const float r = rsqrtf(ss * (1.0f / 64.0f) + eps);
    const float* cr = cos + static_cast<int64_t>(rp) * 32;
    const float* sr = sin + static_cast<int64_t>(rp) * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float y1 = bf16_round(v[i] * r * __bfloat162float(wn[i]));
      const float y2 = bf16_round(v[i + 32] * r * __bfloat162float(wn[i + 32]));
      v[i] = y1 * cr[i] - y2 * sr[i];
      v[i + 32] = y1 * sr[i] + y2 * cr[i];
    }
  }
  if (hd < H) {
    store64(q + (t * H + hd) * 64);
    return;
  }
  const bool is_k = hd < H + HKV;
  const int kvh = is_k ? hd - H : hd - H - HKV;
  store64((is_k ? kc : vc) + static_cast<int64_t>(sq) * stride_cb + static_cast<int64_t>(p) * stride_cs + kvh * 64);
  __nv_bfloat16* packed = is_k ? ko : vo;
  if (packed) store64(packed + (t * HKV + kvh) * 64);
}

// silu(gate) * up with the silu output rounded to bf16 (viktor/triton_ops.py:212-220).
__global__ void swiglu_kernel(const __nv_bfloat16* gu, __nv_bfloat16* out, int64_t n, int F) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  if (i >= n * F) return;
  const int64_t row = i / F;
  const int col = static_cast<int>(i % F);
  const float g = __bfloat162float(gu[row * 2 * F + col]);
  const float u = __bfloat162float(gu[row * 2 * F + F + col]);
  const float act = bf16_round(silu(g));
  out[i] = __float2bfloat16_rn(act * u);
}

// Greedy selection + grammar + state advance, one CTA (128 threads) per sequence
// (viktor/triton_ops.py:172-197, viktor/engine.py:79-89).  With x/h set, the chosen token's embedding and its
// first-layer RMSNorm are written for the next decode step (viktor/triton_ops.py:149-160).
struct GreedyArgs {
  const float* logits;
  int64_t ld_logits;
  const float* bias;
  const uint8_t* is_tail;
  const uint8_t* is_homo;
  int homo_stop;
  int64_t* tok;
  int64_t* run;
  int64_t* pos;
  const int64_t* plen;
  const int64_t* rope_off;
  int64_t* out;
  int64_t out_stride;
  int64_t out_cols;
  int32_t* pos32;
  int32_t* seqlens;
  int32_t* rpos32;
  int B, V, eos, pad;
  // optional fused embedding of the chosen token: x = emb[tok] and its per-64-column sums of squares
  const __nv_bfloat16* emb;
  __nv_bfloat16* x;
  float* ssq;
  // optional sampling (temperature > 0): uniform [0, 1) draws [B, V] (row stride ld_noise)
  const float* noise;
  int64_t ld_noise;
  float temperature;
  // optional fused lm_head: logits = rsqrt(mean(x^2) + eps) * x . head_w^T from the final residual (head_w is
  // the lm_head with the final norm folded in, [V, D] bf16); `logits` is then not read
  const __nv_bfloat16* head_x;
  const float* head_ssq;
  const __nv_bfloat16* head_w;
  float head_eps;
  // optional per-row output cap: row b's token in output column limit[b] (and any later one) is EOS, so the row
  // emits at most limit[b] tokens before it ends (nullptr = no cap)
  const int64_t* limit;
  // 1: a row whose next input token is EOS or PAD gets seqlens = 1 for the next step.  Its next output is PAD
  // whatever that step computes, so its attention reads one position instead of its whole cache row.
  int shrink_done;
};
constexpr int kHeadMaxV = 512;  // vocabulary of the fused head (the 4-mer vocabulary has 343 tokens)

template <int D>
__global__ void __launch_bounds__(128) greedy_kernel(GreedyArgs a) {
  __shared__ float sv[4];
  __shared__ int si[4];
  __shared__ int64_t chosen;
  __shared__ float slog[kHeadMaxV];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();
  if (b >= a.B) return;
  if (a.head_w) {
    // logits of this row: lane j of every warp holds x[16j .. 16j + 15]; warp w computes tokens w, w + 4, ...
    static_assert(D == 512, "fused head: 16 columns per lane");
    float xv[16];
    load8(a.head_x + static_cast<int64_t>(b) * D + lane * 16, xv);
    load8(a.head_x + static_cast<int64_t>(b) * D + lane * 16 + 8, xv + 8);
    const float4* sp = reinterpret_cast<const float4*>(a.head_ssq + static_cast<int64_t>(b) * 8);
    const float4 s0 = sp[0], s1 = sp[1];
    const float r = rsqrtf((((s0.x + s0.y) + (s0.z + s0.w)) + ((s1.x + s1.y) + (s1.z + s1.w))) * (1.0f / D) +
                           a.head_eps);
    for (int v = warp; v < a.V; v += 4) {
      float wv[16];
      load8(a.head_w + static_cast<int64_t>(v) * D + lane * 16, wv);
      load8(a.head_w + static_cast<int64_t>(v) * D + lane * 16 + 8, wv + 8);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc = fmaf(xv[i], wv[i], acc);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) slog[v] = acc * r;
    }
    __syncthreads();
  }
  // state of this sequence, loaded while the argmax runs
  int64_t prev = 0, run0 = 0, p = 0, pl = 0, roff = 0;
  if (tid == 0) {
    prev = a.tok[b];
    run0 = a.run[b];
    p = a.pos[b];
    pl = a.plen[b];
    roff = a.rope_off[b];
  }
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = tid; v < a.V; v += 128) {
    float z = (a.head_w ? slog[v] : a.logits[static_cast<int64_t>(b) * a.ld_logits + v]) + a.bias[v];
    if (a.noise) {  // Gumbel-max sampling, op for op as viktor/engine.py:81-82 (fp32 division and logarithms)
      const float u = fmaxf(a.noise[static_cast<int64_t>(b) * a.ld_noise + v], 1e-20f);
      z = z / a.temperature - logf(-logf(u));
    }
    if (z > best || (z == best && v < bi)) {
      best = z;
      bi = v;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < 4; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    if (bi == 0x7fffffff) bi = 0;
    int64_t nxt = bi;
    const bool prev_ok = prev >= 0 && prev < a.V;
    if (!prev_ok) raise_error(ERR_BOUNDS);
    if (prev_ok && a.is_tail[prev]) nxt = a.eos;  // a tail must be last
    if (a.homo_stop > 0) {
      const bool same = (nxt == prev) && a.is_homo[nxt];
      const int64_t run = same ? run0 + 1 : 0;
      a.run[b] = run;
      if (run + 1 >= a.homo_stop) nxt = a.eos;
    }
    const int64_t col = p - pl;
    if (a.limit && col >= a.limit[b]) nxt = a.eos;  // the row's output cap: end it here
    if (prev == a.eos || prev == a.pad) nxt = a.pad;
    if (col >= 0 && col < a.out_cols)
      a.out[static_cast<int64_t>(b) * a.out_stride + col] = nxt;
    else
      raise_error(ERR_BOUNDS);
    a.tok[b] = nxt;
    p += 1;
    a.pos[b] = p;
    a.pos32[b] = static_cast<int32_t>(p);
    a.seqlens[b] = (a.shrink_done && (nxt == a.eos || nxt == a.pad)) ? 1 : static_cast<int32_t>(p + 1);
    a.rpos32[b] = static_cast<int32_t>(p + roff);
    chosen = nxt;
  }
  __syncthreads();
  if (a.x == nullptr) return;
  // fused embedding of the chosen token for the next step: x = emb[tok] and the sums of squares of its eight
  // 64-column blocks (consumed by the folded attention norm of layer 0)
  constexpr int PER = D / 128;
  const int64_t t = chosen;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const __nv_bfloat16 v = a.emb[t * D + tid * PER + i];
    const float f = __bfloat162float(v);
    ss += f * f;
    a.x[static_cast<int64_t>(b) * D + tid * PER + i] = v;
  }
  // 64 columns = 16 threads (PER = 4): reduce over groups of 16 lanes
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((tid & 15) == 0) a.ssq[static_cast<int64_t>(b) * 8 + tid / 16] = ss;
}

// Per-row sums of squares of the eight 64-column blocks of x [n, 512] (bf16), one warp per row.
__global__ void __launch_bounds__(256) row_ssq_kernel(const __nv_bfloat16* x, float* ssq, int64_t n) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();
  if (row >= n) return;
  // lane holds columns [16*lane, 16*lane + 16): four lanes per 64-column block
  float v[16];
  load8(x + row * 512 + lane * 16, v);
  load8(x + row * 512 + lane * 16 + 8, v + 8);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) ss += v[i] * v[i];
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  if ((lane & 3) == 0) ssq[row * 8 + lane / 4] = ss;
  pdl_launch_dependents();
}

// h = bf16(x * rsqrt(sum(ssq[row]) / 512 + eps) * w), 8 elements per thread.
__global__ void ssq_rmsnorm_kernel(const __nv_bfloat16* x, const float* ssq, const __nv_bfloat16* w,
                                   __nv_bfloat16* h, int64_t n, float eps) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  if (i >= n * 64) return;
  const int64_t row = i / 64;
  const int c = static_cast<int>(i % 64) * 8;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += ssq[row * 8 + k];
  const float r = rsqrtf(s / 512.f + eps);
  float v[8], wv[8], o[8];
  load8(x + row * 512 + c, v);
  load8(w + c, wv);
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = v[k] * r * wv[k];
  uint4 u;
  u.x = pack_bf16x2(o[0], o[1]);
  u.y = pack_bf16x2(o[2], o[3]);
  u.z = pack_bf16x2(o[4], o[5]);
  u.w = pack_bf16x2(o[6], o[7]);
  *reinterpret_cast<uint4*>(h + row * 512 + c) = u;
}

// out[n][k] = bf16(w[n][k] * norm_w[k]) (product of two bf16 values in fp32, rounded once).
__global__ void fold_norm_kernel(const __nv_bfloat16* w, const __nv_bfloat16* nw, __nv_bfloat16* out, int64_t N,
                                 int K) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N * K) return;
  out[i] = __float2bfloat16_rn(__bfloat162float(w[i]) * __bfloat162float(nw[i % K]));
}

__global__ void cast_f32_bf16_kernel(const float* src, __nv_bfloat16* dst, int64_t n) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    *reinterpret_cast<uint2*>(dst + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  } else {
    for (int64_t k = i; k < n; ++k) dst[k] = __float2bfloat16_rn(src[k]);
  }
}

// dst[i] = src[idx[i]] for rows of row_bytes (a multiple of 16).
__global__ void gather_rows_kernel(const uint8_t* src, const int64_t* idx, uint8_t* dst, int64_t n, int row_bytes,
                                   int64_t src_rows) {
  const int64_t r = blockIdx.x;
  pdl_wait();
  if (r >= n) return;
  const int64_t s = idx[r];
  if (s < 0 || s >= src_rows) {
    if (threadIdx.x == 0) raise_error(ERR_BOUNDS);
    return;
  }
  for (int c = threadIdx.x * 16; c < row_bytes; c += blockDim.x * 16)
    *reinterpret_cast<uint4*>(dst + r * row_bytes + c) = *reinterpret_cast<const uint4*>(src + s * row_bytes + c);
}

// dst[dst_idx[i]] = src[src_idx[i]] (either index may be null = identity).
__global__ void copy_rows_kernel(const uint8_t* src, const int64_t* sidx, int64_t src_rows, uint8_t* dst,
                                 const int64_t* didx, int64_t dst_rows, int64_t n, int row_bytes) {
  const int64_t r = blockIdx.x;
  pdl_wait();
  if (r >= n) return;
  const int64_t s = sidx ? sidx[r] : r;
  const int64_t d = didx ? didx[r] : r;
  if (s < 0 || s >= src_rows || d < 0 || d >= dst_rows) {
    if (threadIdx.x == 0) raise_error(ERR_BOUNDS);
    return;
  }
  for (int c = threadIdx.x * 16; c < row_bytes; c += blockDim.x * 16)
    *reinterpret_cast<uint4*>(dst + d * row_bytes + c) = *reinterpret_cast<const uint4*>(src + s * row_bytes + c);
}

// x[rows[i]] = emb[token] (the BOS rows of the packed prefill, viktor/engine.py:165).
__global__ void scatter_embed_kernel(__nv_bfloat16* x, const int64_t* rows, int64_t n, int64_t x_rows,
                                     const __nv_bfloat16* emb, int64_t token, int D) {
  const int64_t r = blockIdx.x;
  pdl_wait();
  if (r >= n) return;
  const int64_t dr = rows[r];
  if (dr < 0 || dr >= x_rows) {
    if (threadIdx.x == 0) raise_error(ERR_BOUNDS);
    return;
  }
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(x + dr * D + c) = *reinterpret_cast<const uint4*>(emb + token * D + c);
}

// ---- packed prefill plan (viktor/engine.py:145-159), built on the device from the prefix lengths ----------
// Sequence b occupies packed rows cu[b] .. cu[b+1]-1: its lens[b] frames, then BOS.  Every CTA scans the n
// lengths itself (n is a sub-batch, at most kPlanMaxSeq), then the grid strides over the packed rows.
constexpr int kPlanMaxSeq = 4096;
constexpr int kPlanThreads = 256;

struct PlanArgs {
  const int32_t* lens;   // [n]
  int n, row0, pos_scale;
  int64_t total;         // sum(lens) + n, as the caller sized the outputs
  int32_t* cu;           // [n + 1]
  int32_t* frame_idx;    // [sum(lens)]: packed row of each frame (may be null when there are no frames)
  int64_t* last;         // [n]: packed row of each BOS
  int32_t* pos;          // [total]: position inside the sequence
  int32_t* seq;          // [total]: cache row (row0 + b)
  int32_t* rpos;         // [total] RoPE position pos * pos_scale, or null
  int32_t* lengths;      // [n]: lens + 1
};

__global__ void __launch_bounds__(kPlanThreads) prefill_plan_kernel(PlanArgs a) {
  __shared__ int64_t scu[kPlanMaxSeq + 1];
  __shared__ int64_t warp_tot[kPlanThreads / 32];
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  if (tid == 0) bad = 0;
  __syncthreads();
  // exclusive scan of (lens + 1): each thread owns kPer consecutive sequences
  constexpr int kPer = kPlanMaxSeq / kPlanThreads;
  int64_t local[kPer];
  int64_t sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    int64_t v = 0;
    if (b < a.n) {
      const int L = a.lens[b];
      if (L < 0) bad = 1;
      v = static_cast<int64_t>(L < 0 ? 0 : L) + 1;
    }
    local[i] = sum;
    sum += v;
  }
  int64_t incl = sum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int64_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int64_t base = incl - sum;
  for (int w = 0; w < warp; ++w) base += warp_tot[w];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    if (b <= a.n) scu[b] = base + local[i];
  }
  if (tid == kPlanThreads - 1 && a.n == kPlanMaxSeq) scu[kPlanMaxSeq] = base + sum;  // no thread starts there
  __syncthreads();
  if (scu[a.n] != a.total || bad) {  // the caller's sizes disagree with the lengths: write nothing
    if (blockIdx.x == 0 && tid == 0) raise_error(ERR_BOUNDS);
    return;
  }
  if (blockIdx.x == 0) {
    for (int b = tid; b <= a.n; b += kPlanThreads) a.cu[b] = static_cast<int32_t>(scu[b]);
    for (int b = tid; b < a.n; b += kPlanThreads) {
      a.last[b] = scu[b + 1] - 1;
      a.lengths[b] = static_cast<int32_t>(scu[b + 1] - scu[b]);
    }
  }
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kPlanThreads + tid; t < a.total;
       t += static_cast<int64_t>(gridDim.x) * kPlanThreads) {
    int lo = 0, hi = a.n - 1;  // last b with scu[b] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (scu[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int p = static_cast<int>(t - scu[b]);
    a.pos[t] = p;
    a.seq[t] = a.row0 + b;
    if (a.rpos) a.rpos[t] = p * a.pos_scale;
    if (t < scu[b + 1] - 1 && a.frame_idx) a.frame_idx[scu[b] - b + p] = static_cast<int32_t>(t);
  }
}

}  // namespace ew
}  // namespace vk
