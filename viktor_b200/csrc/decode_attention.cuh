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
};

VK_DEV void named_bar_compute() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 2)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* cm = reinterpret_cast<float*>(smem + kCombineOff);   // [4][8]
  float* cl = cm + 32;                                        // [4][8]
  float* co = cl + 32;                                        // [4][8][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  int* last_flag = reinterpret_cast<int*>(empty + kStages);

  const int b = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_launch_dependents();
  if (threadIdx.x == 128 && b < a.nq) {
    // While the previous kernel finishes: the first tiles of this split into L2.  Cache rows older than this
    // step's newest position were written by earlier grids; the prefetch only warms L2 (the loads after the
    // wait read whatever L2 then holds).
    const int p0 = split * a.chunk, crow = a.row0 + b;
    for (int t = 0; t < kStages; ++t)
      for (int h = 0; h < 2; ++h) {
        tma_prefetch_l2_4d(&tmK, 0, h, p0 + t * kTile, crow);
        tma_prefetch_l2_4d(&tmV, 0, h, p0 + t * kTile, crow);
      }
  }
  pdl_wait();  // q, lengths and the newest cache row come from the previous kernel
  if (b >= a.nq) return;
  const int L = a.lengths[b];
  const int p_begin = split * a.chunk;
  if (L <= 0 || L > a.S || p_begin >= L) {
    if (split == 0 && threadIdx.x == 0 && (L <= 0 || L > a.S)) raise_error(ERR_BOUNDS);
    return;
  }
  const int p_end = min(p_begin + a.chunk, L);
  const int ntiles = (p_end - p_begin + kTile - 1) / kTile;
  const int nsplit = (L + a.chunk - 1) / a.chunk;
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
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t stream_policy = l2_policy_evict_first();  // the cache is read once per step
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        const uint32_t ph = (t / kStages) & 1;
        if (t >= kStages && !mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          break;
        }
        uint8_t* st = smem + s * kStageBytes;
        const int p0 = p_begin + t * kTile;
        mbar_expect_tx(&full[s], kStageBytes);
        tma_load_4d_hint(st, &tmK, &full[s], 0, 0, p0, crow, stream_policy);
        tma_load_4d_hint(st + kBoxBytes, &tmK, &full[s], 0, 1, p0, crow, stream_policy);
        tma_load_4d_hint(st + 2 * kBoxBytes, &tmV, &full[s], 0, 0, p0, crow, stream_policy);
        tma_load_4d_hint(st + 3 * kBoxBytes, &tmV, &full[s], 0, 1, p0, crow, stream_policy);
      }
    }
    return;
  }

  // ---------------- compute warps 0..3 ----------------
  const int g = lane >> 2, t4 = lane & 3;
  // Block-diagonal Q operand: B[k = (h, d)][n = query head], nonzero where n / 4 == h.
  uint32_t qb[8][2];
  {
    const __nv_bfloat16* qp = a.q + static_cast<int64_t>(b) * 512 + g * 64;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int dbase = (ks & 3) * 16;
      const bool mine = (g >> 2) == (ks >> 2);
      qb[ks][0] = mine ? *reinterpret_cast<const uint32_t*>(qp + dbase + 2 * t4) : 0u;
      qb[ks][1] = mine ? *reinterpret_cast<const uint32_t*>(qp + dbase + 2 * t4 + 8) : 0u;
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2*t4, 2*t4 + 1
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const int j = lane >> 3, rr = lane & 7;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    const uint32_t ph = (t / kStages) & 1;
    if (!mbar_wait(&full[s], ph)) {
      raise_error(ERR_WAIT_FULL);
      break;
    }
    const uint32_t st = smem_u32(smem + s * kStageBytes);
    const int tile_p0 = p_begin + t * kTile;
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
    const float s00 = pa < L ? sc[0] * a.scale_log2 : -INFINITY;
    const float s01 = pa < L ? sc[1] * a.scale_log2 : -INFINITY;
    const float s10 = pb < L ? sc[2] * a.scale_log2 : -INFINITY;
    const float s11 = pb < L ? sc[3] * a.scale_log2 : -INFINITY;
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

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

  const int tid = threadIdx.x;  // 0..127
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
  if (nsplit == 1) {
    const float inv = 1.f / Ls;
    *reinterpret_cast<uint2*>(op) = make_uint2(pack_bf16x2(O[0] * inv, O[1] * inv), pack_bf16x2(O[2] * inv, O[3] * inv));
    return;
  }
  const int64_t slot = (static_cast<int64_t>(b) * a.max_splits + split) * 8 + hh;
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

}  // namespace attn
}  // namespace vk
