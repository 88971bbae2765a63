// Varlen causal GQA attention for the packed prefill (replaces flash_attn_varlen_func(..., causal=True) of
// viktor/fast_decoder.py:73).
//
//   q       packed [n_tok, 8, 64] (token i of sequence b at cu_seqlens[b] + i)
//   K, V    read straight from the KV cache rows the qkv epilogue just wrote (row0 + b, positions 0..T_b-1)
//   out     packed [n_tok, 8, 64]
//
// CTA = (64-query tile, query head, sequence); largest tiles are scheduled first.  A TMA warp loads the query
// tile once and streams 64-key tiles of the matching KV head through a 3-stage ring; four compute warps own
// 16 query rows each and run the FlashAttention-2 recurrence on the warp tensor cores (S = Q K^T, fp32 online
// softmax with exp2, P rounded to bf16, O += P V).  The causal mask only touches the diagonal tile.
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace pattn {

constexpr int kStages = 3;
constexpr int kThreads = 160;
constexpr int kBox = 64 * 128;                 // 64 rows x 64 bf16
constexpr int kQOff = 0;
constexpr int kStageOff = kBox;                // stage s: K at kStageOff + s*2*kBox, V right after
constexpr int kBarOff = kStageOff + kStages * 2 * kBox;
constexpr int kSmemBytes = kBarOff + 128 + 1024;
static_assert(kBarOff % 16 == 0 && kStageOff % 1024 == 0, "shared-memory layout alignment");

struct PrefillArgs {
  const int32_t* cu_seqlens;  // [nseq + 1]
  int nseq;
  int row0;                   // cache row of sequence 0
  int n_qtiles;               // grid.x: max over sequences of ceil(T_b / 64)
  int S;                      // cache positions per row
  __nv_bfloat16* out;         // [n_tok, 8, 64]
  float scale_log2;
};

__global__ void __launch_bounds__(kThreads)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* qbar = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* full = qbar + 1;
  uint64_t* empty = full + kStages;

  const int qt = a.n_qtiles - 1 - static_cast<int>(blockIdx.x);
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq >> 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_wait();
  const int t0 = a.cu_seqlens[b];
  const int T = a.cu_seqlens[b + 1] - t0;
  if (qt * 64 >= T) return;
  if (T > a.S) {
    if (threadIdx.x == 0 && qt == 0) raise_error(ERR_BOUNDS);
    return;
  }
  const int nk = qt + 1;  // key tiles 0..qt
  const int crow = a.row0 + b;

  if (threadIdx.x == 0) {
    mbar_init(qbar, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 4) {
    if (lane == 0) {
      mbar_expect_tx(qbar, kBox);
      tma_load_3d(smem + kQOff, &tmQ, qbar, 0, hq, t0 + qt * 64);
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (kt / kStages) & 1;
        if (kt >= kStages && !mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          break;
        }
        uint8_t* st = smem + kStageOff + s * 2 * kBox;
        mbar_expect_tx(&full[s], 2 * kBox);
        tma_load_4d(st, &tmK, &full[s], 0, hkv, kt * 64, crow);
        tma_load_4d(st + kBox, &tmV, &full[s], 0, hkv, kt * 64, crow);
      }
    }
    return;
  }

  const int g = lane >> 2, t4 = lane & 3;
  const int j = lane >> 3, rr = lane & 7;
  if (!mbar_wait(qbar, 0)) {
    raise_error(ERR_WAIT_FULL);
    return;
  }
  uint32_t qa[4][4];
  {
    const uint32_t qs = smem_u32(smem + kQOff);
    const int row = 16 * warp + (j & 1) * 8 + rr;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int chunk = 2 * ks + (j >> 1);
      ldsm_x4(qs + row * 128 + ((chunk ^ (row & 7)) << 4), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
    }
  }
  const int qa_pos = qt * 64 + 16 * warp + g, qb_pos = qa_pos + 8;  // sequence positions of rows g, g+8
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int kt = 0; kt < nk; ++kt) {
    const int s = kt % kStages;
    const uint32_t ph = (kt / kStages) & 1;
    if (!mbar_wait(&full[s], ph)) {
      raise_error(ERR_WAIT_FULL);
      break;
    }
    const uint32_t ks_base = smem_u32(smem + kStageOff + s * 2 * kBox);
    const uint32_t vs_base = ks_base + kBox;
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int krow = 16 * np + (j >> 1) * 8 + rr;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int chunk = 2 * ks + (j & 1);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(ks_base + krow * 128 + ((chunk ^ (krow & 7)) << 4), r0, r1, r2, r3);
        mma_bf16_16816(sc[2 * np], qa[ks], r0, r1);
        mma_bf16_16816(sc[2 * np + 1], qa[ks], r2, r3);
      }
    }
    const bool diag = kt == qt;
    float tmA = -INFINITY, tmB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int kp = kt * 64 + 8 * nt + 2 * t4;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float va = sc[nt][e] * a.scale_log2, vb = sc[nt][2 + e] * a.scale_log2;
        if (diag) {
          if (kp + e > qa_pos) va = -INFINITY;
          if (kp + e > qb_pos) vb = -INFINITY;
        }
        sc[nt][e] = va;
        sc[nt][2 + e] = vb;
        tmA = fmaxf(tmA, va);
        tmB = fmaxf(tmB, vb);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, off));
      tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, off));
    }
    const float nA = fmaxf(mA, tmA), nB = fmaxf(mB, tmB);
    const float uA = nA == -INFINITY ? 0.f : nA, uB = nB == -INFINITY ? 0.f : nB;
    const float alA = exp2f(mA - uA), alB = exp2f(mB - uB);
    mA = nA;
    mB = nB;
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = exp2f(sc[nt][0] - uA);
      sc[nt][1] = exp2f(sc[nt][1] - uA);
      sc[nt][2] = exp2f(sc[nt][2] - uB);
      sc[nt][3] = exp2f(sc[nt][3] - uB);
      sA += sc[nt][0] + sc[nt][1];
      sB += sc[nt][2] + sc[nt][3];
    }
    lA = lA * alA + sA;
    lB = lB * alB + sB;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= alA;
      o[i][1] *= alA;
      o[i][2] *= alB;
      o[i][3] *= alB;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]);
      pa[1] = pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]);
      pa[2] = pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
      const int vrow = 16 * kk + (j & 1) * 8 + rr;
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int chunk = 2 * dp + (j >> 1);
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vs_base + vrow * 128 + ((chunk ^ (vrow & 7)) << 4), r0, r1, r2, r3);
        mma_bf16_16816(o[2 * dp], pa, r0, r1);
        mma_bf16_16816(o[2 * dp + 1], pa, r2, r3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, off);
    lB += __shfl_xor_sync(0xffffffffu, lB, off);
  }
  const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
  if (qa_pos < T) {
    __nv_bfloat16* op = a.out + (static_cast<int64_t>(t0 + qa_pos) * 8 + hq) * 64 + 2 * t4;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      *reinterpret_cast<uint32_t*>(op + 8 * nt) = pack_bf16x2(o[nt][0] * iA, o[nt][1] * iA);
  }
  if (qb_pos < T) {
    __nv_bfloat16* op = a.out + (static_cast<int64_t>(t0 + qb_pos) * 8 + hq) * 64 + 2 * t4;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      *reinterpret_cast<uint32_t*>(op + 8 * nt) = pack_bf16x2(o[nt][2] * iB, o[nt][3] * iB);
  }
}

}  // namespace pattn
}  // namespace vk
