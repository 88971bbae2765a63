// Single-query GQA decode attention over the bf16 KV cache (replaces viktor/decode_attention.py:11-53 and the
// flash_attn_with_kvcache call of viktor/fast_decoder.py:88-89).
//
//   out[b, h, :] = softmax(q[b, h] . K[b, :L_b, h / 4]^T / 8) . V[b, :L_b, h / 4]
//
// The kernel is bound by HBM reads of the cache, so the design is about keeping enough bytes in flight:
//  * split-K over the prefix: CTA (split, b) owns positions [split * chunk, min(+chunk, L_b)) of sequence b and
//    both KV heads; ~2 x 148 CTAs are resident at a time (96 KB of TMA ring each).  The host picks the longest
//    chunk (1024, 512 or 256 positions) that still gives a full wave of CTAs: long chunks amortise each CTA's
//    pipeline fill and split merge (measured: 0.92-0.95 of the copy bandwidth at 1024 vs 0.85 at 256).
//  * a TMA warp streams 64-position tiles of K and V (one 8 KB box per KV head, 128-byte swizzle) into a
//    2-stage mbarrier ring; positions past the cache end read as zero.
//  * four compute warps each take 16 positions of a tile.  Scores are computed transposed on the warp tensor
//    cores: S^T[16 pos x 8 heads] = K[16 x (2 x 64)] . Qbd[(2 x 64) x 8], with Qbd block-diagonal (query head
//    n only sees KV head n / 4), so both KV heads and all 8 query heads go through one MMA chain.  The fp32
//    online softmax (exp2, scale folded with log2 e) runs on the accumulator fragments; probabilities are
//    rounded to bf16 (as the reference does before its P.V dot) and transposed in registers (movmatrix)
//    into the B operand of O^T[(2 x 64) x 8] += V^T . P^T.
//  * warps are merged through shared memory; splits are merged by the last CTA of each sequence to finish
//    (threadfence + atomic ticket, no waiting), which also resets the ticket for the next launch.
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace attn {

constexpr int kTile = 64;          // positions per TMA tile
constexpr int kMinChunk = 256;     // shortest split (positions per CTA); the workspace is sized for it
constexpr int kStages = 2;          // 2 x 32 KB per CTA, 2 CTAs per SM (3 stages measured slower in the full step)
constexpr int kThreads = 160;      // 4 compute warps + 1 TMA warp
constexpr int kBoxBytes = 64 * 128;            // 64 positions x 64 bf16 (one KV head)
constexpr int kStageBytes = 4 * kBoxBytes;     // K h0, K h1, V h0, V h1
constexpr int kCombineOff = kStages * kStageBytes;
constexpr int kCombineBytes = (4 * 8 * 2 + 4 * 8 * 64) * 4;
constexpr int kBarOff = kCombineOff + kCombineBytes;
constexpr int kSmemBytes = kBarOff + 128 + 1024;
static_assert(kBarOff % 16 == 0 && kCombineOff % 16 == 0, "shared-memory layout alignment");

struct DecodeArgs {
  const __nv_bfloat16* q;   // [nq, 8, 64]
  __nv_bfloat16* out;       // [nq, 8, 64]
  const int32_t* lengths;   // [nq], 1 <= L <= S
  int row0;                 // cache row of query i is row0 + i
  int nq;
  int max_splits;
  int S;
  float* ws_o;              // [nq, max_splits, 8, 64]
  float* ws_ml;             // [nq, max_splits, 8, 2]
  int* counters;            // [nq], zero between launches
  float scale_log2;
  int chunk;                // positions per split: 256, 512 or 1024
  // int8 prefix (decode_attn_i8_kernel only): positions [0, starts[b]) of row b come from an int8 copy of the
  // prefix in at most n8max splits; the bf16 cache serves [starts[b], L_b), at most max_tail positions.
  const int32_t* starts;
  int n8max;
  int max_tail;
  const float* sk;          // [rows][128] per-channel K scale of the prefix
  const float* sv;          // [rows][128] per-channel V scale
  int S8;                   // int8 prefix capacity (positions, a multiple of 128)
};

VK_DEV void named_bar_compute() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Merges the four compute warps' partial results of one split (running max, sum and O^T per query head),
// then either writes the output (single split) or stores the split's partial result in its workspace slot; the
// last split of the row to finish (atomic ticket) merges all of them and resets the ticket.  vscale: per-channel
// V scale of an int8 split (nullptr for bf16).  Called by the 128 compute threads only.
VK_DEV void finish_split(const DecodeArgs& a, int b, int slot_split, int nsplit, float m0, float m1, float l0, float l1,
                         float (&o)[8][4], float* cm, float* cl, float* co, int* last_flag, const float* vscale) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int tid = threadIdx.x;  // 0..127
  // ---- merge the four warps ----
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  if (g == 0) {
    cm[warp * 8 + 2 * t4] = m0;
    cm[warp * 8 + 2 * t4 + 1] = m1;
    cl[warp * 8 + 2 * t4] = l0;
    cl[warp * 8 + 2 * t4 + 1] = l1;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    if ((t4 >> 1) == (mt >> 2)) {  // accumulator columns of this thread belong to KV head mt / 4
      const int d = (mt & 3) * 16 + g;
      float* c0 = co + (warp * 8 + 2 * t4) * 64;
      float* c1 = c0 + 64;
      c0[d] = o[mt][0];
      c1[d] = o[mt][1];
      c0[d + 8] = o[mt][2];
      c1[d + 8] = o[mt][3];
    }
  }
  named_bar_compute();

  const int hh = tid >> 4, d0 = (tid & 15) * 4;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, cm[w * 8 + hh]);
  float Ls = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float f = exp2f(cm[w * 8 + hh] - M);
    Ls += f * cl[w * 8 + hh];
    const float* cw = co + (w * 8 + hh) * 64 + d0;
#pragma unroll
    for (int i = 0; i < 4; ++i) O[i] += f * cw[i];
  }
  __nv_bfloat16* op = a.out + static_cast<int64_t>(b) * 512 + hh * 64 + d0;
  if (vscale) {  // int8 V: O = sv[channel] * sum_p P v8 (the channel of query head hh is (hh / 4) * 64 + d)
    const float4 svv = *reinterpret_cast<const float4*>(vscale + (hh >> 2) * 64 + d0);
    O[0] *= svv.x;
    O[1] *= svv.y;
    O[2] *= svv.z;
    O[3] *= svv.w;
  }
  if (nsplit == 1) {
    const float inv = 1.f / Ls;
    *reinterpret_cast<uint2*>(op) = make_uint2(pack_bf16x2(O[0] * inv, O[1] * inv), pack_bf16x2(O[2] * inv, O[3] * inv));
    return;
  }
  const int64_t slot = (static_cast<int64_t>(b) * a.max_splits + slot_split) * 8 + hh;
  *reinterpret_cast<float4*>(a.ws_o + slot * 64 + d0) = make_float4(O[0], O[1], O[2], O[3]);
  if (d0 == 0) *reinterpret_cast<float2*>(a.ws_ml + slot * 2) = make_float2(M, Ls);
  __threadfence();
  named_bar_compute();
  if (tid == 0) *last_flag = (atomicAdd(&a.counters[b], 1) == nsplit - 1);
  named_bar_compute();
  if (!*last_flag) return;
  __threadfence();
  const int64_t base = static_cast<int64_t>(b) * a.max_splits * 8 + hh;
  // one pass over the splits, four at a time (their loads in flight together), merged with a running maximum
  float Mt = -INFINITY, Lt = 0.f, Ot[4] = {0.f, 0.f, 0.f, 0.f};
  for (int sp0 = 0; sp0 < nsplit; sp0 += 4) {
    float2 ml[4];
    float4 ov[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int sp = sp0 + k < nsplit ? sp0 + k : sp0;
      ml[k] = __ldcg(reinterpret_cast<const float2*>(a.ws_ml + (base + sp * 8) * 2));
      ov[k] = __ldcg(reinterpret_cast<const float4*>(a.ws_o + (base + sp * 8) * 64 + d0));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (sp0 + k >= nsplit) break;
      const float Mn = fmaxf(Mt, ml[k].x);
      const float fa = exp2f(Mt - Mn), fb = exp2f(ml[k].x - Mn);
      Lt = Lt * fa + ml[k].y * fb;
      Ot[0] = Ot[0] * fa + ov[k].x * fb;
      Ot[1] = Ot[1] * fa + ov[k].y * fb;
      Ot[2] = Ot[2] * fa + ov[k].z * fb;
      Ot[3] = Ot[3] * fa + ov[k].w * fb;
      Mt = Mn;
    }
  }
  const float inv = 1.f / Lt;
  *reinterpret_cast<uint2*>(op) = make_uint2(pack_bf16x2(Ot[0] * inv, Ot[1] * inv), pack_bf16x2(Ot[2] * inv, Ot[3] * inv));
  if (tid == 0) a.counters[b] = 0;
}

// ---- bf16 tiles ------------------------------------------------------------------------------------------------
// Block-diagonal Q operand of sequence b: B[k = (h, d)][n = query head], nonzero where n / 4 == h.
VK_DEV void bf16_qbd(const DecodeArgs& a, int b, uint32_t (&qb)[8][2]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const __nv_bfloat16* qp = a.q + static_cast<int64_t>(b) * 512 + g * 64;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int dbase = (ks & 3) * 16;
    const bool mine = (g >> 2) == (ks >> 2);
    qb[ks][0] = mine ? *reinterpret_cast<const uint32_t*>(qp + dbase + 2 * t4) : 0u;
    qb[ks][1] = mine ? *reinterpret_cast<const uint32_t*>(qp + dbase + 2 * t4 + 8) : 0u;
  }
}

// TMA loads of the 64-position bf16 tile at p0 (K and V, both KV heads) into stage st, completing on bar.
VK_DEV void bf16_load(const CUtensorMap* tmK, const CUtensorMap* tmV, uint64_t* bar, uint8_t* st, int p0, int crow,
                      uint64_t policy) {
  mbar_expect_tx(bar, kStageBytes);
  tma_load_4d_hint(st, tmK, bar, 0, 0, p0, crow, policy);
  tma_load_4d_hint(st + kBoxBytes, tmK, bar, 0, 1, p0, crow, policy);
  tma_load_4d_hint(st + 2 * kBoxBytes, tmV, bar, 0, 0, p0, crow, policy);
  tma_load_4d_hint(st + 3 * kBoxBytes, tmV, bar, 0, 1, p0, crow, policy);
}

// Online-softmax update of (m, l, o) over this warp's 16 positions of the bf16 tile staged at st (positions
// tile_p0 .. tile_p0 + 63; those at or past L are masked).
VK_DEV void bf16_tile(uint32_t st, int tile_p0, int L, float scale_log2, const uint32_t (&qb)[8][2], float& m0,
                      float& m1, float& l0, float& l1, float (&o)[8][4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int j = lane >> 3, rr = lane & 7;
  // ---- S^T = K . Qbd ----
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int row = 16 * warp + (j & 1) * 8 + rr;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t base = st + (ks >> 2) * kBoxBytes;
      const int chunk = (ks & 3) * 2 + (j >> 1);
      uint32_t af[4];
      ldsm_x4(base + row * 128 + ((chunk ^ (row & 7)) << 4), af[0], af[1], af[2], af[3]);
      mma_bf16_16816(sc, af, qb[ks][0], qb[ks][1]);
    }
  }
  // ---- online softmax over this warp's 16 positions ----
  const int pa = tile_p0 + 16 * warp + g, pb = pa + 8;
  const float s00 = pa < L ? sc[0] * scale_log2 : -INFINITY;
  const float s01 = pa < L ? sc[1] * scale_log2 : -INFINITY;
  const float s10 = pb < L ? sc[2] * scale_log2 : -INFINITY;
  const float s11 = pb < L ? sc[3] * scale_log2 : -INFINITY;
  float tm0 = fmaxf(s00, s10), tm1 = fmaxf(s01, s11);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
    tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
  }
  const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
  const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
  const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
  const float p00 = exp2f(s00 - mu0), p10 = exp2f(s10 - mu0);
  const float p01 = exp2f(s01 - mu1), p11 = exp2f(s11 - mu1);
  l0 = l0 * al0 + p00 + p10;
  l1 = l1 * al1 + p01 + p11;
  m0 = mn0;
  m1 = mn1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o[i][0] *= al0;
    o[i][2] *= al0;
    o[i][1] *= al1;
    o[i][3] *= al1;
  }
  const uint32_t pb0 = movmatrix_t(pack_bf16x2(p00, p01));
  const uint32_t pb1 = movmatrix_t(pack_bf16x2(p10, p11));
  // ---- O^T += V^T . P^T ----
  const bool partial = tile_p0 + kTile > L;
  const int kp = tile_p0 + 16 * warp + 2 * t4;
  const uint32_t mk0 = (kp < L ? 0x0000FFFFu : 0u) | (kp + 1 < L ? 0xFFFF0000u : 0u);
  const uint32_t mk1 = (kp + 8 < L ? 0x0000FFFFu : 0u) | (kp + 9 < L ? 0xFFFF0000u : 0u);
  {
    const int prow = 16 * warp + (j >> 1) * 8 + rr;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const uint32_t base = st + (2 + (mt >> 2)) * kBoxBytes;
      const int chunk = (mt & 3) * 2 + (j & 1);
      uint32_t af[4];
      ldsm_x4_t(base + prow * 128 + ((chunk ^ (prow & 7)) << 4), af[0], af[1], af[2], af[3]);
      if (partial) {  // rows past the sequence may hold stale data: zero them, not just their weights
        af[0] &= mk0;
        af[1] &= mk0;
        af[2] &= mk1;
        af[3] &= mk1;
      }
      mma_bf16_16816(o[mt], af, pb0, pb1);
    }
  }
}

// ---- bf16 split -------------------------------------------------------------------------------------------------
// Positions [p_begin, p_end) of row b (both KV heads, all 8 query heads) from the bf16 cache; the partial result
// goes to workspace slot slot_split of the row's nsplit.  p_begin + chunk >= p_end and chunk is a multiple of
// kTile, so the tiles of a split stay inside it (the last one may run past L, which is masked).
VK_DEV void bf16_split(const CUtensorMap* tmK, const CUtensorMap* tmV, const DecodeArgs& a, uint8_t* smem, int b,
                       int L, int p_begin, int p_end, int slot_split, int nsplit) {
  float* cm = reinterpret_cast<float*>(smem + kCombineOff);   // [4][8]
  float* cl = cm + 32;                                        // [4][8]
  float* co = cl + 32;                                        // [4][8][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  int* last_flag = reinterpret_cast<int*>(empty + kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (p_end - p_begin + kTile - 1) / kTile;
  const int crow = a.row0 + b;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(tmK);
      tma_prefetch_desc(tmV);
      const uint64_t stream_policy = l2_policy_evict_first();  // the cache is read once per step
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        const uint32_t ph = (t / kStages) & 1;
        if (t >= kStages && !mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          break;
        }
        bf16_load(tmK, tmV, &full[s], smem + s * kStageBytes, p_begin + t * kTile, crow, stream_policy);
      }
    }
    return;
  }

  // ---------------- compute warps 0..3 ----------------
  uint32_t qb[8][2];
  bf16_qbd(a, b, qb);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2*t4, 2*t4 + 1
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    const uint32_t ph = (t / kStages) & 1;
    if (!mbar_wait(&full[s], ph)) {
      raise_error(ERR_WAIT_FULL);
      break;
    }
    bf16_tile(smem_u32(smem + s * kStageBytes), p_begin + t * kTile, L, a.scale_log2, qb, m0, m1, l0, l1, o);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  finish_split(a, b, slot_split, nsplit, m0, m1, l0, l1, o, cm, cl, co, last_flag, nullptr);
}

// ---- int8 split ---------------------------------------------------------------------------------------------------
// The prefix copy holds excess-128 bytes u = round(x / s_c) + 128 with one scale s_c per channel (both KV heads,
// 128 channels): K8 position-major [rows][S8][128], V8T channel-major in tiles of 128 positions,
// [rows][S8 / 128][128 channels][128 positions], so that a 128-position tile of either is one contiguous 16 KB
// TMA box (128-byte swizzle).  The warp MMAs run in fp16: ldmatrix hands each thread four
// consecutive bytes of a row, which two byte permutes and one packed fp16 subtract turn into exact fp16 values
// (0x6400 | u is 1024 + u; minus 1152 leaves u - 128).  Those four bytes are taken as the k slots
// {2t, 2t+1, 2t+8, 2t+9} of the MMA fragment; the other operand follows the same order:
//  * S^T = K8 . Qbd': Qbd' carries q * s_c (the K scales folded into the query) at the matching channels;
//  * O^T += V8T . P^T: the k slots are positions, so the S^T rows are loaded in the order
//    pi(r) = {0,1,4,5,8,9,12,13,2,3,6,7,10,11,14,15}[r], which makes the transposed P fragment line up;
//    the V scales multiply O when the split finishes.
constexpr int kTile8 = 128;                 // positions per int8 tile
constexpr int kStages8 = 2;                 // int8 splits: 2 x 32 KB ring (3 measured no faster)
constexpr int kCombineOff8 = kStages8 * kStageBytes;
constexpr int kBarOff8 = kCombineOff8 + kCombineBytes;
constexpr int kSmemBytes8 = (kBarOff8 > kBarOff ? kBarOff8 : kBarOff) + 128 + 1024;  // holds both split layouts
constexpr int kBox8Bytes = 128 * 128;       // K8: 128 positions x 128 channels; V8T: 128 channels x 128 positions
static_assert(2 * kBox8Bytes == kStageBytes, "an int8 stage has the size of a bf16 stage");

VK_DEV uint32_t u8x2_to_f16x2(uint32_t w, uint32_t sel) {
  const uint32_t h = __byte_perm(w, 0x64646464u, sel);
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
  return r;
}
VK_DEV uint32_t u8_lo(uint32_t w) { return u8x2_to_f16x2(w, 0x4140); }  // bytes 0, 1
VK_DEV uint32_t u8_hi(uint32_t w) { return u8x2_to_f16x2(w, 0x4342); }  // bytes 2, 3
VK_DEV uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
VK_DEV void mma_f16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Positions per int8 split of a prefix of `start` positions cut into at most n8max splits (multiple of kTile8).
VK_DEV int i8_chunk(int start, int n8max) {
  const int per = (start + n8max - 1) / n8max;
  return (per + kTile8 - 1) / kTile8 * kTile8;
}

// Qbd' of sequence b (cache row crow), fp16.
VK_DEV void i8_qbd(const DecodeArgs& a, int b, int crow, uint32_t (&qb)[8][2]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  // Qbd' in fp16: k step ks covers channels 16 ks .. 16 ks + 15 (KV head ks / 4); this thread's k slots 2 t4,
  // 2 t4 + 1 hold channels 4 t4, 4 t4 + 1 and slots 2 t4 + 8, 2 t4 + 9 channels 4 t4 + 2, 4 t4 + 3.
  const __nv_bfloat16* qp = a.q + static_cast<int64_t>(b) * 512 + g * 64;
  const float* skp = a.sk + static_cast<int64_t>(crow) * 128 + (g >> 2) * 64;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d0 = (ks & 3) * 16 + 4 * t4;
    if ((g >> 2) == (ks >> 2)) {
      const uint2 qv = *reinterpret_cast<const uint2*>(qp + d0);
      const float4 scl = *reinterpret_cast<const float4*>(skp + d0);
      qb[ks][0] = pack_f16x2(bf16_lo(qv.x) * scl.x, bf16_hi(qv.x) * scl.y);
      qb[ks][1] = pack_f16x2(bf16_lo(qv.y) * scl.z, bf16_hi(qv.y) * scl.w);
    } else {
      qb[ks][0] = qb[ks][1] = 0u;
    }
  }
}

// TMA loads of the 128-position int8 tile at p0 (one 16 KB box of K8 and one of V8T) into stage st.
VK_DEV void i8_load(const CUtensorMap* tmK8, const CUtensorMap* tmV8, uint64_t* bar, uint8_t* st, int p0, int crow,
                    uint64_t policy) {
  mbar_expect_tx(bar, kStageBytes);
  tma_load_3d_hint(st, tmK8, bar, 0, p0, crow, policy);
  tma_load_4d_hint(st + kBox8Bytes, tmV8, bar, 0, 0, p0 / kTile8, crow, policy);
}

// Online-softmax update of (m, l, o) over this warp's 32 positions of the int8 tile staged at st (positions
// tile_p0 .. tile_p0 + 127; those at or past p_end are masked).
VK_DEV void i8_tile(uint32_t st, int tile_p0, int p_end, float scale_log2, const uint32_t (&qb)[8][2], float& m0,
                    float& m1, float& l0, float& l1, float (&o)[8][4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int j = lane >> 3, rr = lane & 7;       // ldmatrix: this lane addresses row rr of matrix j
  const int mrow = rr + (j & 1) * 8;            // MMA row of that address (matrices: rows 0-7, 8-15, 0-7, 8-15)
  const int kpos = ((mrow & 6) << 1) | ((mrow >> 3) << 1) | (mrow & 1);   // pi(mrow)
  const int pg = ((g & 6) << 1) | (g & 1);      // pi(g); pi(g + 8) = pg | 2
  const int wp0 = tile_p0 + 32 * warp;   // this warp's 32 positions: two blocks of 16
  // ---- S^T = K8 . Qbd' ----
  // four independent accumulator chains (two blocks x the two KV heads' k steps), summed at the end
  float sc[2][4], sh[2][2][4];
#pragma unroll
  for (int sb = 0; sb < 2; ++sb) {
#pragma unroll
    for (int h = 0; h < 2; ++h) sh[sb][h][0] = sh[sb][h][1] = sh[sb][h][2] = sh[sb][h][3] = 0.f;
    const int row = 32 * warp + 16 * sb + kpos;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const int chunk = 2 * kc + (j >> 1);
      uint32_t r0, r1, r2, r3;
      ldsm_x4(st + row * 128 + ((chunk ^ (row & 7)) << 4), r0, r1, r2, r3);
      const uint32_t a0[4] = {u8_lo(r0), u8_lo(r1), u8_hi(r0), u8_hi(r1)};
      mma_f16_16816(sh[sb][kc >> 1], a0, qb[2 * kc][0], qb[2 * kc][1]);
      const uint32_t a1[4] = {u8_lo(r2), u8_lo(r3), u8_hi(r2), u8_hi(r3)};
      mma_f16_16816(sh[sb][kc >> 1], a1, qb[2 * kc + 1][0], qb[2 * kc + 1][1]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) sc[sb][e] = sh[sb][0][e] + sh[sb][1][e];
  }
  // ---- online softmax over the warp's 32 positions ----
  float sl[2][4];
#pragma unroll
  for (int sb = 0; sb < 2; ++sb) {
    const int pa = wp0 + 16 * sb + pg, pb = pa + 2;
    sl[sb][0] = pa < p_end ? sc[sb][0] * scale_log2 : -INFINITY;
    sl[sb][1] = pa < p_end ? sc[sb][1] * scale_log2 : -INFINITY;
    sl[sb][2] = pb < p_end ? sc[sb][2] * scale_log2 : -INFINITY;
    sl[sb][3] = pb < p_end ? sc[sb][3] * scale_log2 : -INFINITY;
  }
  float tm0 = fmaxf(fmaxf(sl[0][0], sl[0][2]), fmaxf(sl[1][0], sl[1][2]));
  float tm1 = fmaxf(fmaxf(sl[0][1], sl[0][3]), fmaxf(sl[1][1], sl[1][3]));
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
    tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
  }
  const float mn0 = fmaxf(m0, tm0), mn1 = fmaxf(m1, tm1);
  const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
  const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
  uint32_t pfrag[2][2];
  float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
  for (int sb = 0; sb < 2; ++sb) {
    const float p00 = exp2f(sl[sb][0] - mu0), p10 = exp2f(sl[sb][2] - mu0);
    const float p01 = exp2f(sl[sb][1] - mu1), p11 = exp2f(sl[sb][3] - mu1);
    ls0 += p00 + p10;
    ls1 += p01 + p11;
    pfrag[sb][0] = movmatrix_t(pack_f16x2(p00, p01));
    pfrag[sb][1] = movmatrix_t(pack_f16x2(p10, p11));
  }
  l0 = l0 * al0 + ls0;
  l1 = l1 * al1 + ls1;
  m0 = mn0;
  m1 = mn1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o[i][0] *= al0;
    o[i][2] *= al0;
    o[i][1] *= al1;
    o[i][3] *= al1;
  }
  // ---- O^T += V8T . P^T (positions past the prefix have P = 0 and finite bytes) ----
  {
    const int vchunk = 2 * warp + (j >> 1);   // matrices: (channels 0-7, block 0), (8-15, 0), (0-7, 1), (8-15, 1)
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int ch = 16 * mt + mrow;
      uint32_t r0, r1, r2, r3;
      ldsm_x4(st + kBox8Bytes + ch * 128 + ((vchunk ^ (ch & 7)) << 4), r0, r1, r2, r3);
      const uint32_t a0[4] = {u8_lo(r0), u8_lo(r1), u8_hi(r0), u8_hi(r1)};
      mma_f16_16816(o[mt], a0, pfrag[0][0], pfrag[0][1]);
      const uint32_t a1[4] = {u8_lo(r2), u8_lo(r3), u8_hi(r2), u8_hi(r3)};
      mma_f16_16816(o[mt], a1, pfrag[1][0], pfrag[1][1]);
    }
  }
}

VK_DEV void i8_split(const CUtensorMap* tmK8, const CUtensorMap* tmV8, const DecodeArgs& a, uint8_t* smem, int b,
                     int p_begin, int p_end, int slot_split, int nsplit) {
  float* cm = reinterpret_cast<float*>(smem + kCombineOff8);
  float* cl = cm + 32;
  float* co = cl + 32;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff8);
  uint64_t* empty = full + kStages8;
  int* last_flag = reinterpret_cast<int*>(empty + kStages8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (p_end - p_begin + kTile8 - 1) / kTile8;
  const int crow = a.row0 + b;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages8; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(tmK8);
      tma_prefetch_desc(tmV8);
      const uint64_t stream_policy = l2_policy_evict_first();
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages8;
        const uint32_t ph = (t / kStages8) & 1;
        if (t >= kStages8 && !mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          break;
        }
        i8_load(tmK8, tmV8, &full[s], smem + s * kStageBytes, p_begin + t * kTile8, crow, stream_policy);
      }
    }
    return;
  }

  uint32_t qb[8][2];
  i8_qbd(a, b, crow, qb);
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages8;
    const uint32_t ph = (t / kStages8) & 1;
    if (!mbar_wait(&full[s], ph)) {
      raise_error(ERR_WAIT_FULL);
      break;
    }
    i8_tile(smem_u32(smem + s * kStageBytes), p_begin + t * kTile8, p_end, a.scale_log2, qb, m0, m1, l0, l1, o);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  finish_split(a, b, slot_split, nsplit, m0, m1, l0, l1, o, cm, cl, co, last_flag,
               a.sv + static_cast<int64_t>(crow) * 128);
}

VK_DEV uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// bf16 cache only: CTA (split, b) covers positions [split * chunk, +chunk) of row b.
__global__ void __launch_bounds__(kThreads, 2)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  const int b = blockIdx.y, split = blockIdx.x;
  pdl_launch_dependents();
  if (threadIdx.x == 128 && b < a.nq) {
    // While the previous kernel finishes: the first tiles of this split into L2.  Cache rows older than this
    // step's newest position were written by earlier grids; the prefetch only warms L2 (the loads after the
    // wait read whatever L2 then holds).
    // The row's length as last written (this step's, or the previous step's if the kernel that advances it is
    // still running: at most one position short) only bounds the prefetch, so tiles past the row's end (splits
    // past it, rows that have ended) are not pulled from HBM.
    const int p0 = split * a.chunk, crow = a.row0 + b;
    const int len_hint = *reinterpret_cast<const volatile int32_t*>(a.lengths + b);
    for (int t = 0; t < kStages; ++t)
      if (p0 + t * kTile <= len_hint)
        for (int h = 0; h < 2; ++h) {
          tma_prefetch_l2_4d(&tmK, 0, h, p0 + t * kTile, crow);
          tma_prefetch_l2_4d(&tmV, 0, h, p0 + t * kTile, crow);
        }
  }
  pdl_wait();  // q, lengths and the newest cache row come from the previous kernel
  if (b >= a.nq) return;
  const int L = a.lengths[b];
  if (L <= 0 || L > a.S) {
    if (split == 0 && threadIdx.x == 0) raise_error(ERR_BOUNDS);
    return;
  }
  const int p_begin = split * a.chunk;
  if (p_begin >= L) return;
  bf16_split(&tmK, &tmV, a, smem, b, L, p_begin, min(p_begin + a.chunk, L), split, (L + a.chunk - 1) / a.chunk);
}

// int8 prefix + bf16 rest.  CTA (b, x): x < n8max is int8 split x of the prefix [0, starts[b]) (splits of
// i8_chunk positions); the others are bf16 splits of chunk positions over [starts[b], L_b).  All splits of a row
// share its workspace slots (int8 first) and its merge ticket.
__global__ void __launch_bounds__(kThreads, 2)
    decode_attn_i8_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmK8, const __grid_constant__ CUtensorMap tmV8,
                          DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  const int b = blockIdx.x, x = blockIdx.y;  // splits outermost: the long int8 splits start first
  pdl_launch_dependents();
  if (threadIdx.x == 128 && b < a.nq && x < a.n8max) {
    // the int8 prefix is written once, before decoding: warm L2 with this split's first tiles before the wait
    const int p0 = x * i8_chunk(a.S8, a.n8max), crow = a.row0 + b;
    for (int t = 0; t < kStages8; ++t)
      if (p0 + t * kTile8 < a.S8) {
        tma_prefetch_l2_3d(&tmK8, 0, p0 + t * kTile8, crow);
        tma_prefetch_l2_4d(&tmV8, 0, 0, p0 / kTile8 + t, crow);
      }
  }
  pdl_wait();
  if (b >= a.nq) return;
  const int L = a.lengths[b], start = a.starts[b];
  if (L <= 0 || L > a.S || start < 0 || start >= L || start > a.S8 || L - start > a.max_tail) {
    if (x == 0 && threadIdx.x == 0) raise_error(ERR_BOUNDS);
    return;
  }
  const int c8 = i8_chunk(start, a.n8max);
  const int n8 = start > 0 ? (start + c8 - 1) / c8 : 0;
  const int n16 = (L - start + a.chunk - 1) / a.chunk;
  if (x < a.n8max) {
    if (x >= n8) return;
    i8_split(&tmK8, &tmV8, a, smem, b, x * c8, min(x * c8 + c8, start), x, n8 + n16);
  } else {
    const int split = x - a.n8max;
    if (split >= n16) return;
    const int p_begin = start + split * a.chunk;
    bf16_split(&tmK, &tmV, a, smem, b, L, p_begin, min(p_begin + a.chunk, L), n8 + split, n8 + n16);
  }
}

// ---- int8 prefix quantisation -------------------------------------------------------------------------------------
// Block (i, which): row row0 + i of one layer's K (which 0) or V (which 1) cache, positions [0, starts[i]).
// Per channel c: m_c = max |x|, scale s_c = m_c / 127 (0 for an all-zero channel), byte
// u = clamp(rint(x * (127 / m_c)), -127, 127) + 128 (fp32, round to nearest even).  K8 rows are written
// position-major; V goes through a shared-memory transpose (128 positions at a time) into the channel-major
// tiles of V8T.  Positions [starts[i], round_up(starts[i], 128)) of V8T get the byte for 0.
struct QuantArgs {
  const __nv_bfloat16* k;   // [rows][S][128] bf16 layer cache (element strides stride_kb, stride_ks)
  const __nv_bfloat16* v;
  int64_t stride_kb, stride_ks;
  const int32_t* starts;    // [n]
  int row0, n, S, S8;
  uint8_t* k8;              // [rows][S8][128]
  uint8_t* v8t;             // [rows][S8 / 128][128][128]
  float* sk;                // [rows][128]
  float* sv;
};
constexpr int kQuantThreads = 256;

VK_DEV uint32_t quant_byte(float x, float inv) {
  const float q = fminf(fmaxf(rintf(x * inv), -127.f), 127.f);
  return static_cast<uint32_t>(static_cast<int>(q) + 128);
}

__global__ void __launch_bounds__(kQuantThreads) kv_quantize_kernel(QuantArgs a) {
  __shared__ float red[16][128];
  __shared__ float inv_s[128];
  __shared__ __align__(16) uint8_t tr[128][128 + 16];
  const int i = blockIdx.x, which = blockIdx.y;
  pdl_wait();  // the cache rows come from the previous kernels
  if (i >= a.n) return;
  const int row = a.row0 + i;
  const int start = a.starts[i];
  if (start < 0 || start > a.S || start > a.S8) {
    if (threadIdx.x == 0 && which == 0) raise_error(ERR_BOUNDS);
    return;
  }
  const __nv_bfloat16* src = (which ? a.v : a.k) + static_cast<int64_t>(row) * a.stride_kb;
  const int t = threadIdx.x, cg = t & 15, pr = t >> 4;   // channels 8 cg .. 8 cg + 7, positions pr + 16 k
  float mx[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  // eight rows per thread per round, their loads issued together (the pass is bound by load latency)
  for (int p0 = 0; p0 < start; p0 += 128) {
    uint4 w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int p = p0 + pr + 16 * k;
      w[k] = p < start ? __ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(p) * a.stride_ks + 8 * cg))
                       : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t ws[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mx[2 * e] = fmaxf(mx[2 * e], fabsf(bf16_lo(ws[e])));
        mx[2 * e + 1] = fmaxf(mx[2 * e + 1], fabsf(bf16_hi(ws[e])));
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[pr][8 * cg + e] = mx[e];
  __syncthreads();
  if (t < 128) {
    float m = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) m = fmaxf(m, red[r][t]);
    (which ? a.sv : a.sk)[static_cast<int64_t>(row) * 128 + t] = __fdiv_rn(m, 127.f);
    inv_s[t] = m > 0.f ? __fdiv_rn(127.f, m) : 0.f;
  }
  __syncthreads();
  float inv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) inv[e] = inv_s[8 * cg + e];
  if (which == 0) {
    uint8_t* dst = a.k8 + static_cast<int64_t>(row) * a.S8 * 128;
    for (int p0 = 0; p0 < start; p0 += 128) {
      uint4 w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int p = p0 + pr + 16 * k;
        w[k] = p < start
                   ? __ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(p) * a.stride_ks + 8 * cg))
                   : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int p = p0 + pr + 16 * k;
        if (p >= start) break;
        const uint32_t ws[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
        uint32_t out[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t lo = quant_byte(bf16_lo(ws[e]), inv[2 * e]);
          const uint32_t hi = quant_byte(bf16_hi(ws[e]), inv[2 * e + 1]);
          out[e >> 1] |= (lo | (hi << 8)) << ((e & 1) * 16);
        }
        *reinterpret_cast<uint2*>(dst + static_cast<int64_t>(p) * 128 + 8 * cg) = make_uint2(out[0], out[1]);
      }
    }
  } else {
    uint8_t* dst = a.v8t + static_cast<int64_t>(row) * 128 * a.S8;
    for (int p0 = 0; p0 < start; p0 += 128) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int pl = pr + 16 * k, p = p0 + pl;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (p < start)
          w = __ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(p) * a.stride_ks + 8 * cg));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          tr[8 * cg + 2 * e][pl] = static_cast<uint8_t>(quant_byte(bf16_lo(ws[e]), inv[2 * e]));
          tr[8 * cg + 2 * e + 1][pl] = static_cast<uint8_t>(quant_byte(bf16_hi(ws[e]), inv[2 * e + 1]));
        }
      }
      __syncthreads();
      const int c = t >> 1, off = (t & 1) * 64;
      uint8_t* tile = dst + static_cast<int64_t>(p0) * 128;  // the 16 KB tile of positions p0 .. p0 + 127
#pragma unroll
      for (int k = 0; k < 4; ++k)
        *reinterpret_cast<uint4*>(tile + c * 128 + off + 16 * k) =
            *reinterpret_cast<const uint4*>(&tr[c][off + 16 * k]);
      __syncthreads();
    }
  }
}

}  // namespace attn
}  // namespace vk
