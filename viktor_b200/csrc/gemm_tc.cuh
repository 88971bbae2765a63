// tcgen05 GEMM for the decoder projections:  C[M, N] = A[M, K] * B[N, K]^T  (bf16 in, fp32 accumulate in TMEM).
//
// One CTA computes one 128 x BN tile over a K range.  Warp roles (192 threads):
//   warp 0      TMA producer (one elected lane): A and B K-major tiles, 128-byte swizzle, up to 4-deep ring
//   warp 1      TMEM allocator + MMA issuer (one elected lane): tcgen05.mma kind::f16, M=128, N=BN, K=16 x 4
//   warps 2..5  epilogue (thread = one accumulator row = one TMEM lane)
//
// Split-K across a thread-block cluster (NK > 1): the NK CTAs of a cluster share one output tile and each
// accumulates K/NK of the contraction.  Partial tiles are staged in shared memory and reduced on chip through
// distributed shared memory: CTA k sums rows [k*128/NK, (k+1)*128/NK) over all NK peers and runs the epilogue on
// them.  Small-M (decode) GEMMs thereby spread over 100-200 CTAs that each stream only 24-72 KB, instead of a few
// CTAs streaming hundreds of KB.
//
// Folded RMSNorm: a GEMM whose input is RMSNorm(x) * w runs on x itself with w folded into the weight columns
// (W' = W diag(w), done once when the weights are loaded); the epilogue scales each row by
// r = rsqrt(mean(x^2) + eps), with mean(x^2) assembled from the per-64-column sums of squares (ssq) that the
// producer of x wrote.  That keeps every epilogue tile-local.
//
// Fused epilogues (each restates a reference op on the GEMM output):
//   STORE_BF16 / STORE_F32   y = r * acc (viktor/triton_ops.py:111-146 without SwiGLU; fp32 logits)
//   BIAS_ACT                 y = act(bf16(acc + bias)), act = identity | GELU(erf), optional output row map
//                            (projector, viktor/model.py:35; packed-prefill scatter, viktor/engine.py:163-165)
//   SWIGLU                   B rows = [gate block | up block]: y = bf16(bf16(silu(bf16(r g))) * bf16(r u))
//                            (viktor/triton_ops.py:129-134, :212-220)
//   QKV_ROPE                 per 64-column head of bf16(r * acc): QK-RMSNorm, RoPE, q store, K/V cache write
//                            (viktor/triton_ops.py:43-91)
//   ADD_RESID                x = bf16(x + bf16(acc)) in place and the new row's per-64-column sums of squares
//                            (the residual half of viktor/triton_ops.py:17-31; the norm half is folded forward)
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
// Stages of the TMA ring for large M (many tiles per SM): wide tiles get three so that two CTAs fit on an SM
// (one's epilogue then overlaps the other's mainloop); narrow tiles get four.  Small-M (decode) launches have
// at most one tile per SM and are bound by load latency: they take as many stages as shared memory holds, up
// to kMaxStages, so that most or all of a CTA's K blocks are in flight at once.
__host__ __device__ constexpr int max_stages_for(int bn) { return bn >= 128 ? 3 : 4; }
constexpr int kSmemBudget = 232448;  // dynamic shared memory one CTA may use on sm_100
constexpr int kSsqSlots = 8;  // sums of squares per 512-wide residual row, one per 64-column block

enum Epi : int { STORE_BF16 = 0, STORE_F32 = 1, BIAS_ACT = 2, SWIGLU = 3, QKV_ROPE = 4, ADD_RESID = 5 };

struct EpiArgs {
  void* y;
  int64_t ldy;
  int n_valid;                     // output columns that exist (STORE_*, BIAS_ACT)
  const int32_t* row_map;          // BIAS_ACT: output row of each input row (nullptr = identity)
  const __nv_bfloat16* bias;       // BIAS_ACT
  int act;                         // BIAS_ACT: 0 identity, 1 GELU(erf)
  const float* ssq_in;             // folded RMSNorm of A: [M, 8] sums of squares (nullptr = no norm)
  float eps;
  // QKV_ROPE
  __nv_bfloat16* q_out;            // [M, H, 64]
  __nv_bfloat16* k_cache;          // one layer: element (row, p, kvh, d) at row*stride_cb + p*stride_cs + kvh*64 + d
  __nv_bfloat16* v_cache;
  __nv_bfloat16* k_out;            // optional packed [M, Hkv, 64]
  __nv_bfloat16* v_out;
  const int32_t* pos;              // cache position of each token
  const int32_t* rope_pos;         // RoPE position of each token (nullptr = pos)
  const int32_t* seq;              // cache row of each token
  const __nv_bfloat16* q_norm_w;   // [64]
  const __nv_bfloat16* k_norm_w;   // [64]
  const float* cos;                // [rope_len, 32]
  const float* sin;
  int rope_len;
  int cache_rows, cache_len;
  int64_t stride_cb, stride_cs;
  int n_heads, n_kv_heads;
  float qk_eps;
  // ADD_RESID
  __nv_bfloat16* x;                // residual [M, 512], updated in place
  float* ssq_out;                  // [M, 8]
};

// Shared-memory layout (bytes from the 1024-aligned base), identical in every CTA of a launch.
//   [0, pipe)          TMA ring; after the mainloop, this CTA's fp32 partial tile [128][BN+4] (split-K)
//   [recv_off, ...)    split-K: slices of the reduced rows received from the peers [NK-1][BM/NK][BN+4]
//   [bar_off, ...)     mbarriers, TMEM address
struct SmemLayout {
  int stages, stage_bytes, a_bytes, recv_off, bar_off, total;
  __host__ __device__ SmemLayout(int bn, int nk, int stages_, int epi) {
    stages = stages_;
    a_bytes = BM * BK * 2;
    stage_bytes = a_bytes + bn * BK * 2;
    int pipe = stages * stage_bytes;
    const int staging = nk > 1 ? BM * (bn + 4) * 4 : 0;
    if (staging > pipe) pipe = staging;
    pipe = (pipe + 1023) & ~1023;
    (void)epi;
    recv_off = pipe;  // split-K: the NK-1 slices [BM/nk][bn+4] fp32 sent by the peers
    bar_off = recv_off + (nk > 1 ? (nk - 1) * (BM / nk) * (bn + 4) * 4 : 0);
    total = bar_off + 256 + 1024;  // barriers + alignment slack
  }
};

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  return bn <= 32 ? 32u : (bn <= 64 ? 64u : (bn <= 128 ? 128u : (bn <= 256 ? 256u : 512u)));
}

VK_DEV void store_bf16x8(__nv_bfloat16* dst, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = u;
}
VK_DEV void load_bf16x8(const __nv_bfloat16* src, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x);
  v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z);
  v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
}

VK_DEV float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// Row scale of a folded RMSNorm: rsqrt(mean(x^2) + eps) from the producer's eight partial sums.
VK_DEV float row_rscale(const EpiArgs& ep, int row) {
  if (!ep.ssq_in) return 1.f;
  const float4* p = reinterpret_cast<const float4*>(ep.ssq_in + static_cast<int64_t>(row) * kSsqSlots);
  const float4 a = p[0], b = p[1];
  const float s = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
  return rsqrtf(s * (1.0f / 512.0f) + ep.eps);
}

// QK-RMSNorm + RoPE of one 64-wide head held by this thread (viktor/triton_ops.py:44-49).
VK_DEV void norm_rope_head(float* v, const __nv_bfloat16* w, const float* c, const float* s, float eps) {
  float ss8[8];  // eight independent chains: the 64-term sum is a latency chain otherwise
#pragma unroll
  for (int k = 0; k < 8; ++k) ss8[k] = v[k] * v[k];
#pragma unroll
  for (int i = 8; i < 64; i += 8)
#pragma unroll
    for (int k = 0; k < 8; ++k) ss8[k] = fmaf(v[i + k], v[i + k], ss8[k]);
  const float ss = ((ss8[0] + ss8[1]) + (ss8[2] + ss8[3])) + ((ss8[4] + ss8[5]) + (ss8[6] + ss8[7]));
  const float r = rsqrtf(ss * (1.0f / 64.0f) + eps);
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    float wa[8], wb[8];  // 16-byte loads of the norm weights (the pointer is 16-byte aligned)
    load_bf16x8(w + i, wa);
    load_bf16x8(w + i + 32, wb);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float y1 = bf16_round(v[i + e] * r * wa[e]);
      const float y2 = bf16_round(v[i + e + 32] * r * wb[e]);
      v[i + e] = y1 * c[i + e] - y2 * s[i + e];
      v[i + e + 32] = y1 * s[i + e] + y2 * c[i + e];
    }
  }
}

// Per-row inputs of the QKV_ROPE epilogue (cache position, RoPE position, cache row, the cos / sin row), loaded
// once per row so that a caller can fetch them before its accumulator is ready.
struct QkvRow {
  int p, rp, sq;
  bool ok;  // every index in range
  float c[32], s[32];
};

VK_DEV void load_qkv_row(const EpiArgs& ep, int row, QkvRow& q) {
  q.p = ep.pos[row];
  q.rp = ep.rope_pos ? ep.rope_pos[row] : q.p;
  q.sq = ep.seq[row];
  q.ok = q.p >= 0 && q.p < ep.cache_len && q.sq >= 0 && q.sq < ep.cache_rows && q.rp >= 0 && q.rp < ep.rope_len;
  const int64_t rp = q.ok ? q.rp : 0;
  const float4* cp = reinterpret_cast<const float4*>(ep.cos + rp * 32);
  const float4* sp = reinterpret_cast<const float4*>(ep.sin + rp * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 a = cp[i], b = sp[i];
    q.c[4 * i] = a.x; q.c[4 * i + 1] = a.y; q.c[4 * i + 2] = a.z; q.c[4 * i + 3] = a.w;
    q.s[4 * i] = b.x; q.s[4 * i + 1] = b.y; q.s[4 * i + 2] = b.z; q.s[4 * i + 3] = b.w;
  }
}

// QKV_ROPE epilogue of global head gh (64 values in v, row scale r): round to bf16, QK-norm + RoPE for q and k
// heads, then q to q_out and k / v into the cache (and the packed copies when asked).
VK_DEV void qkv_head(const EpiArgs& ep, int row, int gh, float* v, float r, const QkvRow& q) {
  const int H = ep.n_heads, HKV = ep.n_kv_heads;
  if (!q.ok) {
    raise_error(ERR_BOUNDS);
    return;
  }
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = bf16_round(v[i] * r);  // the qkv linear output is stored in bf16
  if (gh < H + HKV) norm_rope_head(v, gh < H ? ep.q_norm_w : ep.k_norm_w, q.c, q.s, ep.qk_eps);
  if (gh < H) {
    __nv_bfloat16* qp = ep.q_out + (static_cast<int64_t>(row) * H + gh) * 64;
#pragma unroll
    for (int i = 0; i < 64; i += 8) store_bf16x8(qp + i, v + i);
  } else if (gh < H + 2 * HKV) {
    const bool is_k = gh < H + HKV;
    const int kvh = is_k ? gh - H : gh - H - HKV;
    __nv_bfloat16* cache = is_k ? ep.k_cache : ep.v_cache;
    __nv_bfloat16* dst =
        cache + static_cast<int64_t>(q.sq) * ep.stride_cb + static_cast<int64_t>(q.p) * ep.stride_cs + kvh * 64;
#pragma unroll
    for (int i = 0; i < 64; i += 8) store_bf16x8(dst + i, v + i);
    __nv_bfloat16* packed = is_k ? ep.k_out : ep.v_out;
    if (packed) {
      __nv_bfloat16* pd = packed + (static_cast<int64_t>(row) * HKV + kvh) * 64;
#pragma unroll
      for (int i = 0; i < 64; i += 8) store_bf16x8(pd + i, v + i);
    }
  }
}

// ADD_RESID epilogue of the 64 columns c0.. of one row: x += bf16(v) (bf16 rounding), with the residual's 64
// bf16 values given in xr (loaded by the caller), and the block's sum of squares to ssq_out.
VK_DEV void add_resid_block(const EpiArgs& ep, int row, int c0, const float* v, const uint4* xr, int N) {
  __nv_bfloat16* xp = ep.x + static_cast<int64_t>(row) * N + c0;
  float ss8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // independent chains (see norm_rope_head)
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    const uint4 u = xr[i / 8];
    float xo[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                   bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      xo[e] = bf16_round(xo[e] + bf16_round(v[i + e]));
      ss8[e] = fmaf(xo[e], xo[e], ss8[e]);
    }
    store_bf16x8(xp + i, xo);
  }
  ep.ssq_out[static_cast<int64_t>(row) * kSsqSlots + c0 / 64] =
      ((ss8[0] + ss8[1]) + (ss8[2] + ss8[3])) + ((ss8[4] + ss8[5]) + (ss8[6] + ss8[7]));
}

// Number of epilogue chunks of a BN tile and their width.  A chunk is 64 consecutive columns (BN < 64: BN
// columns); for SWIGLU it is 32 gate columns and the 32 matching up columns.
template <int BN>
struct Chunks {
  static constexpr int W = BN < 64 ? BN : 64;
  static constexpr int COUNT = BN < 64 ? 1 : BN / 64;
};

// Applies the epilogue to chunk `ch` of row `row` (v holds W values; SWIGLU: 32 gate then 32 up).
template <int BN, int EPI>
VK_DEV void epi_chunk(const EpiArgs& ep, int row, int n_tile, int ch, float* v, float r, int N) {
  constexpr int W = Chunks<BN>::W;
  if (EPI == STORE_BF16 || EPI == STORE_F32 || EPI == BIAS_ACT) {
    const int col = n_tile * BN + ch * W;
    const int64_t orow = (EPI == BIAS_ACT && ep.row_map) ? ep.row_map[row] : row;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      if (EPI == BIAS_ACT) {
        const float t = bf16_round(v[i] + (col + i < ep.n_valid ? __bfloat162float(ep.bias[col + i]) : 0.f));
        v[i] = ep.act == 1 ? gelu_erf(t) : t;
      } else {
        v[i] *= r;
      }
    }
    if (EPI == STORE_F32) {
      float* yp = reinterpret_cast<float*>(ep.y) + orow * ep.ldy + col;
      if (col + W <= ep.n_valid && (ep.ldy & 3) == 0) {
#pragma unroll
        for (int i = 0; i < W; i += 4)
          *reinterpret_cast<float4*>(yp + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
        for (int i = 0; i < W; ++i)
          if (col + i < ep.n_valid) yp[i] = v[i];
      }
    } else {
      __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(ep.y) + orow * ep.ldy + col;
      if (col + W <= ep.n_valid && (ep.ldy & 7) == 0) {
#pragma unroll
        for (int i = 0; i < W; i += 8) store_bf16x8(yp + i, v + i);
      } else {
        for (int i = 0; i < W; ++i)
          if (col + i < ep.n_valid) yp[i] = __float2bfloat16_rn(v[i]);
      }
    }
  } else if (EPI == SWIGLU) {
    const int F = N / 2;
    const int o0 = n_tile * (BN / 2) + ch * 32;
    float out[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float gb = bf16_round(v[i] * r);
      out[i] = bf16_round(silu(gb)) * bf16_round(v[32 + i] * r);
    }
    if (o0 + 32 <= F) {
      __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(ep.y) + static_cast<int64_t>(row) * ep.ldy + o0;
#pragma unroll
      for (int i = 0; i < 32; i += 8) store_bf16x8(yp + i, out + i);
    }
  } else if (EPI == ADD_RESID) {
    const int c0 = n_tile * BN + ch * 64;
    const uint4* xp = reinterpret_cast<const uint4*>(ep.x + static_cast<int64_t>(row) * N + c0);
    uint4 xr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[i] = xp[i];
    add_resid_block(ep, row, c0, v, xr, N);
  } else if (EPI == QKV_ROPE) {
    QkvRow q;
    load_qkv_row(ep, row, q);
    qkv_head(ep, row, n_tile * (BN / 64) + ch, v, r, q);
  }
}

// Split-K epilogue: each thread owns 8 consecutive output columns of one row (SWIGLU: 8 gate + the 8 matching
// up columns, producing 8 outputs).  Groups of 8 consecutive lanes cover one 64-column block (one head for
// QKV_ROPE), so row-wide reductions over a block are 3 butterfly shuffles.  Every lane of a warp executes the
// shuffles; `active` masks the memory traffic of lanes without a row.
VK_DEV float group8_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

// Epilogue inputs of one thread's reduced row (split-K), loaded before the accumulator is ready.
// Everything the epilogue reads from global memory is loaded here, before the accumulator wait, for every pass
// a thread makes (up to two): under a saturated memory system each such load is a long round trip, so none may
// sit between the split-K exchange and the stores.
struct RowInputs {
  float r;                       // folded-norm row scale
  int pos, rpos, seq;            // QKV_ROPE
  float c[8], s[8];              // QKV_ROPE: cos / sin of the eight rotation angles this thread applies
  float wn[8];                   // QKV_ROPE: the QK-norm weights of this thread's eight columns of its head
  float xres[8];                 // ADD_RESID: this thread's eight residual columns
};

template <int BN, int EPI>
VK_DEV RowInputs load_row_inputs(const EpiArgs& ep, int row, int n_tile, int g8, int N, bool valid) {
  RowInputs in;
  in.r = (valid && EPI != ADD_RESID) ? row_rscale(ep, row) : 1.f;
  in.pos = in.rpos = in.seq = 0;
  if (EPI == QKV_ROPE) {
    if (valid) {
      in.pos = ep.pos[row];
      in.rpos = ep.rope_pos ? ep.rope_pos[row] : in.pos;
      in.seq = ep.seq[row];
    }
    const int rp = (valid && in.rpos >= 0 && in.rpos < ep.rope_len) ? in.rpos : 0;
    const int d0 = (g8 & 3) * 8;  // position within the rotated half
    const float4* cp = reinterpret_cast<const float4*>(ep.cos + static_cast<int64_t>(rp) * 32 + d0);
    const float4* sp = reinterpret_cast<const float4*>(ep.sin + static_cast<int64_t>(rp) * 32 + d0);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    in.c[0] = c0.x; in.c[1] = c0.y; in.c[2] = c0.z; in.c[3] = c0.w;
    in.c[4] = c1.x; in.c[5] = c1.y; in.c[6] = c1.z; in.c[7] = c1.w;
    in.s[0] = s0.x; in.s[1] = s0.y; in.s[2] = s0.z; in.s[3] = s0.w;
    in.s[4] = s1.x; in.s[5] = s1.y; in.s[6] = s1.z; in.s[7] = s1.w;
    const int gh = n_tile * (BN / 64) + g8 / 8;  // head of this thread's columns
    if (gh < ep.n_heads + ep.n_kv_heads) {
      load_bf16x8((gh < ep.n_heads ? ep.q_norm_w : ep.k_norm_w) + (g8 & 7) * 8, in.wn);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) in.wn[i] = 0.f;
    }
  }
  if (EPI == ADD_RESID) {
    if (valid) {
      load_bf16x8(ep.x + static_cast<int64_t>(row) * N + n_tile * BN + g8 * 8, in.xres);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) in.xres[i] = 0.f;
    }
  }
  return in;
}

template <int BN, int EPI>
VK_DEV void epi_group8(const EpiArgs& ep, int row, int n_tile, int g8, float* v, const RowInputs& in, int N,
                       bool active) {
  const float r = in.r;
  if (EPI == STORE_BF16 || EPI == STORE_F32) {
    const int col = n_tile * BN + g8 * 8;
    if (!active) return;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= r;
    if (EPI == STORE_F32) {
      float* yp = reinterpret_cast<float*>(ep.y) + static_cast<int64_t>(row) * ep.ldy + col;
      if (col + 8 <= ep.n_valid && (ep.ldy & 3) == 0) {
        *reinterpret_cast<float4*>(yp) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(yp + 4) = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        for (int i = 0; i < 8; ++i)
          if (col + i < ep.n_valid) yp[i] = v[i];
      }
    } else {
      __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(ep.y) + static_cast<int64_t>(row) * ep.ldy + col;
      if (col + 8 <= ep.n_valid && (ep.ldy & 7) == 0) {
        store_bf16x8(yp, v);
      } else {
        for (int i = 0; i < 8; ++i)
          if (col + i < ep.n_valid) yp[i] = __float2bfloat16_rn(v[i]);
      }
    }
  } else if (EPI == SWIGLU) {
    const int o0 = n_tile * (BN / 2) + g8 * 8;
    if (!active || o0 + 8 > N / 2) return;
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = bf16_round(silu(bf16_round(v[i] * r))) * bf16_round(v[8 + i] * r);
    store_bf16x8(reinterpret_cast<__nv_bfloat16*>(ep.y) + static_cast<int64_t>(row) * ep.ldy + o0, out);
  } else if (EPI == ADD_RESID) {
    const int c0 = n_tile * BN + g8 * 8;
    float ss = 0.f;
    if (active) {
      __nv_bfloat16* xp = ep.x + static_cast<int64_t>(row) * N + c0;
      float xo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xo[e] = bf16_round(in.xres[e] + bf16_round(v[e]));
        ss += xo[e] * xo[e];
      }
      store_bf16x8(xp, xo);
    }
    ss = group8_sum(ss);
    if (active && (g8 & 7) == 0) ep.ssq_out[static_cast<int64_t>(row) * kSsqSlots + c0 / 64] = ss;
  } else if (EPI == QKV_ROPE) {
    const int H = ep.n_heads, HKV = ep.n_kv_heads;
    const int gh = n_tile * (BN / 64) + g8 / 8;
    const int j = g8 & 7;  // 8-column group within the head
    const int p = in.pos, sq = in.seq;
    if (active && (p < 0 || p >= ep.cache_len || sq < 0 || sq >= ep.cache_rows || in.rpos < 0 ||
                   in.rpos >= ep.rope_len)) {
      raise_error(ERR_BOUNDS);
      active = false;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = bf16_round(v[i] * r);  // the qkv linear output is stored in bf16
    if (gh < H + HKV) {  // uniform across the 8-lane group
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
      ss = group8_sum(ss);
      const float rr = rsqrtf(ss * (1.0f / 64.0f) + ep.qk_eps);
      float y[8], other[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = bf16_round(v[i] * rr * in.wn[i]);
#pragma unroll
      for (int i = 0; i < 8; ++i) other[i] = __shfl_xor_sync(0xffffffffu, y[i], 4);
#pragma unroll
      for (int i = 0; i < 8; ++i)  // first half: y1*c - y2*s; second half: y1*s + y2*c (y1 from the partner)
        v[i] = j < 4 ? y[i] * in.c[i] - other[i] * in.s[i] : other[i] * in.s[i] + y[i] * in.c[i];
    }
    if (!active) return;
    if (gh < H) {
      store_bf16x8(ep.q_out + (static_cast<int64_t>(row) * H + gh) * 64 + j * 8, v);
    } else if (gh < H + 2 * HKV) {
      const bool is_k = gh < H + HKV;
      const int kvh = is_k ? gh - H : gh - H - HKV;
      __nv_bfloat16* cache = is_k ? ep.k_cache : ep.v_cache;
      store_bf16x8(cache + static_cast<int64_t>(sq) * ep.stride_cb + static_cast<int64_t>(p) * ep.stride_cs +
                       kvh * 64 + j * 8,
                   v);
      __nv_bfloat16* packed = is_k ? ep.k_out : ep.v_out;
      if (packed) store_bf16x8(packed + (static_cast<int64_t>(row) * HKV + kvh) * 64 + j * 8, v);
    }
  }
}

// TMEM column of element i of chunk ch (SWIGLU chunks gather gate and up halves).
template <int BN, int EPI>
VK_DEV int chunk_col(int ch, int i) {
  constexpr int W = Chunks<BN>::W;
  if (EPI == SWIGLU) return i < 32 ? ch * 32 + i : BN / 2 + ch * 32 + (i - 32);
  return ch * W + i;
}

template <int BN, int EPI, int NK>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                int K, int stages, EpiArgs ep) {
  const SmemLayout L(BN, NK, stages, EPI);
  constexpr int B_BOX_BYTES = (EPI == SWIGLU ? BN / 2 : BN) * BK * 2;
  constexpr int SROW = BN + 4;   // staging row stride (floats)
  constexpr int R = BM / NK;     // rows each CTA reduces
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr int W = Chunks<BN>::W;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accum = empty + kMaxStages;
  uint64_t* tmem_free = accum + 1;
  uint64_t* recv_bar = tmem_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  float* staging = reinterpret_cast<float*>(smem);
  float* recv = reinterpret_cast<float*>(smem + L.recv_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = NK > 1 ? static_cast<int>(blockIdx.x) : 0;
  const int n_tile = blockIdx.y, m0 = blockIdx.z * BM;
  const int nkb = K / BK / NK;
  const int kb0 = ks * nkb;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_init(tmem_free, 4);
    mbar_init(recv_bar, 1);
    if (NK > 1) mbar_expect_tx(recv_bar, static_cast<uint32_t>((NK - 1) * R * SROW * 4));
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (NK > 1) cluster_arrive();  // (phase A) this CTA's receive barrier is initialised
  // Let the next kernel of the stream start its prologue (barriers, TMEM, weight loads) now; it waits for this
  // grid's completion before touching anything this grid writes.
  pdl_launch_dependents();

  bool ok = true;  // producer / MMA lanes: false once a wait ran out
  if (warp == 0) {
    if (lane == 0) {
      // The B operand (weights) does not depend on the previous kernel: start it before waiting on it.  Weights
      // are re-read every step: keep them in L2 ahead of streamed data.
      const uint64_t keep = l2_policy_evict_last();
      const int pre = nkb < stages ? nkb : stages;
      for (int i = 0; i < pre; ++i) {
        uint8_t* sB = smem + i * L.stage_bytes + L.a_bytes;
        const int kx = (kb0 + i) * BK;
        mbar_expect_tx(&full[i], L.stage_bytes);
        if (EPI == SWIGLU) {
          tma_load_2d_hint(sB, &tmB, &full[i], kx, n_tile * (BN / 2), keep);
          tma_load_2d_hint(sB + B_BOX_BYTES, &tmB, &full[i], kx, N / 2 + n_tile * (BN / 2), keep);
        } else {
          tma_load_2d_hint(sB, &tmB, &full[i], kx, n_tile * BN, keep);
        }
      }
      // The rest of this CTA's weight tiles: into L2 now, so the loads after the wait do not go to HBM.
      for (int i = pre; i < nkb; ++i) {
        const int kx = (kb0 + i) * BK;
        if (EPI == SWIGLU) {
          tma_prefetch_l2_2d(&tmB, kx, n_tile * (BN / 2));
          tma_prefetch_l2_2d(&tmB, kx, N / 2 + n_tile * (BN / 2));
        } else {
          tma_prefetch_l2_2d(&tmB, kx, n_tile * BN);
        }
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) tma_load_2d(smem + i * L.stage_bytes, &tmA, &full[i], (kb0 + i) * BK, m0);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        uint8_t* sA = smem + s * L.stage_bytes;
        uint8_t* sB = sA + L.a_bytes;
        const int kx = (kb0 + i) * BK;
        mbar_expect_tx(&full[s], L.stage_bytes);
        tma_load_2d(sA, &tmA, &full[s], kx, m0);
        if (EPI == SWIGLU) {
          tma_load_2d_hint(sB, &tmB, &full[s], kx, n_tile * (BN / 2), keep);
          tma_load_2d_hint(sB + B_BOX_BYTES, &tmB, &full[s], kx, N / 2 + n_tile * (BN / 2), keep);
        } else {
          tma_load_2d_hint(sB, &tmB, &full[s], kx, n_tile * BN, keep);
        }
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (!mbar_wait(&full[s], ph)) {
          raise_error(ERR_WAIT_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sdesc_k_sw128(smem_u32(smem + s * L.stage_bytes));
        const uint64_t bd = sdesc_k_sw128(smem_u32(smem + s * L.stage_bytes + L.a_bytes));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) umma_bf16(tmem_base, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(accum);
    }
  } else {
    pdl_wait();
  }
  __syncwarp();

  // ---------------- epilogue ----------------
  // tcgen05.ld is warp-collective: every lane of an epilogue warp issues the same loads; only global stores
  // depend on the row being inside M.  Inputs that do not depend on the accumulator (row scales, positions,
  // RoPE angles, the residual) are loaded before the accumulator wait, while the MMAs run: everything they
  // read was written before the previous grid completed.
  const bool epi_warp = warp >= 2;
  const int quarter = warp & 3;
  const int row_local = quarter * 32 + lane;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  bool have_acc = false;
  auto wait_accum = [&]() {
    if (epi_warp) {
      have_acc = __all_sync(0xffffffffu, mbar_wait(accum, 0));
      if (!have_acc && lane == 0) raise_error(ERR_WAIT_ACCUM);
      tc_fence_after();
    }
  };
  // An epilogue warp is done with TMEM: the MMA warp may free it once all four have said so.
  auto release_tmem = [&]() {
    if (epi_warp) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_free);
    }
  };

  if (NK == 1) {
    const int row = m0 + row_local;
    const bool row_ok = row < M;
    const float r = (epi_warp && row_ok && EPI != BIAS_ACT && EPI != ADD_RESID) ? row_rscale(ep, row) : 1.f;
    wait_accum();
    if (epi_warp && have_acc) {
#pragma unroll 1
      for (int ch = 0; ch < Chunks<BN>::COUNT; ++ch) {
        float v[64];
#pragma unroll
        for (int q = 0; q < W; q += 16) tmem_ld16(taddr + chunk_col<BN, EPI>(ch, q), v + q);
        tmem_wait_ld();
        if (row_ok) epi_chunk<BN, EPI>(ep, row, n_tile, ch, v, r, N);
      }
    }
    release_tmem();
  } else {
    // Split-K: every CTA of the cluster stages its fp32 partial tile [128][SROW] in its own shared memory and
    // hands rows [p*R, p*R + R) to CTA p with one bulk copy (the copy engine moves them between the SMs); CTA ks
    // waits until its NK-1 slices have landed, sums them with its own in the order p = 0..NK-1 and applies the
    // epilogue.  Each thread owns 8 output columns of one reduced row (SWIGLU: 8 gate + the 8 matching up
    // columns).  The only cluster-wide wait on this path is before exit: no CTA may leave while a copy still
    // reads its staging tile.
    constexpr int WOUT = EPI == SWIGLU ? BN / 2 : BN;
    constexpr int TPR = WOUT / 8;                 // threads per reduced row
    constexpr int RPP = 128 / TPR;                // reduced rows per pass
    constexpr int PASSES = (R + RPP - 1) / RPP;
    constexpr int NV = EPI == SWIGLU ? 16 : 8;    // values per thread and pass
    constexpr uint32_t SLICE = R * SROW * 4;      // bytes of one slice
    static_assert((TPR & (TPR - 1)) == 0 && TPR <= 128, "epilogue thread mapping");
    static_assert(SLICE % 16 == 0, "bulk copies move multiples of 16 bytes");
    const int t = epi_warp ? static_cast<int>(threadIdx.x) - 64 : 0;
    const int g8 = t & (TPR - 1);
    RowInputs in0, in1;  // the inputs of passes 0 and 1
    if (epi_warp) {
      const int rl0 = t / TPR, row0 = m0 + ks * R + rl0;
      in0 = load_row_inputs<BN, EPI>(ep, row0, n_tile, g8, N, rl0 < R && row0 < M);
      if (PASSES > 1) {
        const int rl1 = RPP + t / TPR, row1 = m0 + ks * R + rl1;
        in1 = load_row_inputs<BN, EPI>(ep, row1, n_tile, g8, N, rl1 < R && row1 < M);
      }
    }
    wait_accum();
    if (epi_warp) {
      // stage (on a failed accumulator wait the slices are still sent, so that no peer waits in vain)
      if (have_acc) {
        constexpr int CW = BN < 64 ? BN : 64;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += CW) {
          float v[CW];
#pragma unroll
          for (int q = 0; q < CW; q += 16) tmem_ld16(taddr + c0 + q, v + q);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(staging + row_local * SROW + c0);
#pragma unroll
          for (int i = 0; i < CW / 4; ++i)
            dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
      release_tmem();
      fence_proxy_async();                          // staging stores -> visible to the copy engine
      asm volatile("bar.sync 1, 128;" ::: "memory");  // all 128 rows staged
      cluster_wait();                               // (phase A) every peer's receive barrier is initialised
      if (t < NK && t != ks) {
        const int slot = ks < t ? ks : ks - 1;      // where CTA t keeps the slice from this CTA
        bulk_copy_to_peer(dsmem_addr(recv + slot * (SLICE / 4), static_cast<uint32_t>(t)),
                          smem_u32(staging + t * R * SROW), SLICE,
                          dsmem_addr(recv_bar, static_cast<uint32_t>(t)));
      }
      const bool got = mbar_wait(recv_bar, 0);
      if (!got && t == 0) raise_error(ERR_WAIT_FULL);
      __syncwarp();
      cluster_arrive_relaxed();                     // (phase B) this CTA's slices have all arrived
      auto do_pass = [&](int pass, const RowInputs& in) {
        const int rl = pass * RPP + t / TPR;
        const int row = m0 + ks * R + rl;
        const bool active = have_acc && got && rl < R && row < M;
        const int rs = rl < R ? rl : 0;
        float v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = 0.f;
#pragma unroll
        for (int p = 0; p < NK; ++p) {
          const float* src = p == ks ? staging + (ks * R + rs) * SROW : recv + ((p < ks ? p : p - 1) * R + rs) * SROW;
          src += g8 * 8;
#pragma unroll
          for (int qd = 0; qd < NV / 4; ++qd) {
            const float4 x = *reinterpret_cast<const float4*>(src + (qd & 1) * 4 + (qd >> 1) * (BN / 2));
            v[4 * qd] += x.x;
            v[4 * qd + 1] += x.y;
            v[4 * qd + 2] += x.z;
            v[4 * qd + 3] += x.w;
          }
        }
        epi_group8<BN, EPI>(ep, row, n_tile, g8, v, in, N, active);
      };
      do_pass(0, in0);
      if (PASSES > 1) do_pass(1, in1);
#pragma unroll 1
      for (int pass = 2; pass < PASSES; ++pass) {  // (more than two passes: wide tiles with few splits)
        const int rl = pass * RPP + t / TPR, row = m0 + ks * R + rl;
        do_pass(pass, load_row_inputs<BN, EPI>(ep, row, n_tile, g8, N, rl < R && row < M));
      }
    } else {
      __syncwarp();
      cluster_wait();            // (phase A)
      cluster_arrive_relaxed();  // (phase B)
    }
    __syncwarp();
    cluster_wait();  // (phase B) every slice of the cluster has landed: no copy still reads this CTA's staging
  }

  if (warp == 1) {
    // free TMEM only after the four epilogue warps have finished reading it
    if (!mbar_wait(tmem_free, 0) && lane == 0) raise_error(ERR_WAIT_ACCUM);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Persistent GEMM for large M (prefill): one CTA per SM walks the output tiles (BN = 256, N fastest, so the
// CTAs that run together share A row blocks in L2).  Warp 0 streams A/B stages through a 4-deep TMA ring across
// tile boundaries, warp 1 issues the MMAs into one of two TMEM accumulators (2 x 256 of the 512 columns), and
// eight epilogue warps (two per TMEM lane quarter, each taking half of the tile's 64-column chunks) drain the
// other accumulator, so a tile's epilogue overlaps the next tile's K loop.  Epilogues as gemm_kernel (NK = 1).
constexpr int kPBN = 256;
constexpr int kPStages = 4;
constexpr int kPThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kPStageBytes = BM * BK * 2 + kPBN * BK * 2;  // 48 KB
constexpr int kPBarOff = kPStages * kPStageBytes;
constexpr int kPSmemBytes = kPBarOff + 256 + 1024;
constexpr uint32_t kPTmemCols = 512;

template <int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                           int N, int K, EpiArgs ep) {
  constexpr int BN = kPBN;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BOX_BYTES = (EPI == SWIGLU ? BN / 2 : BN) * BK * 2;
  constexpr int W = Chunks<BN>::W;
  constexpr int CPS = Chunks<BN>::COUNT / 2;  // chunks per epilogue warp set
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPBarOff);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;   // [2] accumulator ready (tcgen05.commit)
  uint64_t* acc_empty = acc_full + 2;      // [2] accumulator drained (8 epilogue warps)
  uint64_t* tmem_free = acc_empty + 2;     // every epilogue warp is done with TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_free + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (EPI == SWIGLU ? N / 2 : N) / (EPI == SWIGLU ? BN / 2 : BN);
  const int m_tiles = (M + BM - 1) / BM;
  const int tiles = n_tiles * m_tiles;
  const int nkb = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    mbar_init(tmem_free, 8);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kPTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int n_tile = t % n_tiles, m0 = (t / n_tiles) * BM;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kPStages;
          if (it >= kPStages && !mbar_wait(&empty[s], ((it / kPStages) & 1) ^ 1)) {
            raise_error(ERR_WAIT_EMPTY);
            ok = false;
            break;
          }
          uint8_t* sA = smem + s * kPStageBytes;
          uint8_t* sB = sA + A_BYTES;
          const int kx = kb * BK;
          mbar_expect_tx(&full[s], kPStageBytes);
          tma_load_2d(sA, &tmA, &full[s], kx, m0);
          if (EPI == SWIGLU) {
            tma_load_2d_hint(sB, &tmB, &full[s], kx, n_tile * (BN / 2), keep);
            tma_load_2d_hint(sB + B_BOX_BYTES, &tmB, &full[s], kx, N / 2 + n_tile * (BN / 2), keep);
          } else {
            tma_load_2d_hint(sB, &tmB, &full[s], kx, n_tile * BN, keep);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      uint32_t it = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int ab = i & 1;
        if (i >= 2 && !mbar_wait(&acc_empty[ab], ((i >> 1) - 1) & 1)) {
          raise_error(ERR_WAIT_ACCUM);
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tmem_base + ab * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kPStages;
          if (!mbar_wait(&full[s], (it / kPStages) & 1)) {
            raise_error(ERR_WAIT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_k_sw128(smem_u32(smem + s * kPStageBytes));
          const uint64_t bd = sdesc_k_sw128(smem_u32(smem + s * kPStageBytes + A_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_bf16(dacc, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
    }
  } else {
    // epilogue warps 2..9: lane quarter (warp % 4), column half (warp set)
    const int quarter = warp & 3;
    const int set = (warp - 2) >> 2;
    const int row_local = quarter * 32 + lane;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int ab = i & 1;
      const int n_tile = t % n_tiles, m0 = (t / n_tiles) * BM;
      const int row = m0 + row_local;
      const bool row_ok = row < M;
      const float r = (row_ok && EPI != BIAS_ACT && EPI != ADD_RESID) ? row_rscale(ep, row) : 1.f;
      // the epilogue's other global inputs do not depend on the accumulator: fetch them while the MMAs run
      QkvRow qr;
      uint4 xr[CPS][8];
      if (EPI == QKV_ROPE && row_ok) load_qkv_row(ep, row, qr);
      if (EPI == ADD_RESID && row_ok) {
#pragma unroll
        for (int cc = 0; cc < CPS; ++cc) {
          const uint4* xp = reinterpret_cast<const uint4*>(ep.x + static_cast<int64_t>(row) * N + n_tile * BN +
                                                           (set * CPS + cc) * 64);
#pragma unroll
          for (int k = 0; k < 8; ++k) xr[cc][k] = xp[k];
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (i >> 1) & 1))) {
        if (lane == 0) raise_error(ERR_WAIT_ACCUM);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ab * BN + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
      for (int cc = 0; cc < CPS; ++cc) {
        const int ch = set * CPS + cc;
        float v[64];
#pragma unroll
        for (int q = 0; q < W; q += 16) tmem_ld16(taddr + chunk_col<BN, EPI>(ch, q), v + q);
        tmem_wait_ld();
        if (row_ok) {
          if (EPI == QKV_ROPE)
            qkv_head(ep, row, n_tile * (BN / 64) + ch, v, r, qr);
          else if (EPI == ADD_RESID)
            add_resid_block(ep, row, n_tile * BN + ch * 64, v, xr[cc], N);
          else
            epi_chunk<BN, EPI>(ep, row, n_tile, ch, v, r, N);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_free);
  }
  if (warp == 1) {
    // free TMEM once the epilogue warps are done (they waited on the last accumulator, i.e. on every MMA)
    if (!mbar_wait(tmem_free, 0) && lane == 0) raise_error(ERR_WAIT_ACCUM);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kPTmemCols);
  }
}

}  // namespace gemm
}  // namespace vk
