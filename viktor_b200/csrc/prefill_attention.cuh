// Varlen causal GQA attention for the packed prefill on the 5th-generation tensor cores (replaces
// flash_attn_varlen_func(..., causal=True) of viktor/fast_decoder.py:73).
//
//   q       packed [n_tok, 8, 64] (token i of sequence b at cu_seqlens[b] + i)
//   K, V    read straight from the KV cache rows the qkv epilogue just wrote (row0 + b, positions 0..T_b-1)
//   out     packed [n_tok, 8, 64]
//
// CTA = (128-query tile, query head, sequence), largest tiles first, two CTAs per SM.  Warp roles:
//   warp 0      TMA: the query tile once, then 128-key K and V tiles of the matching KV head (2-stage ring)
//   warp 1      TMEM allocation and the MMA issue (one elected lane), per key tile j:
//                 S_j  = Q K_j^T    tcgen05.mma M=128 N=128 K=64, A and B from shared memory -> TMEM S (fp32)
//                 O   += P_j V_j    tcgen05.mma M=128 N=64 K=128, A = P_j from TMEM (bf16), B = the V tile as
//                                   an MN-major operand straight from its TMA tile -> TMEM O (fp32)
//   warps 2-5   softmax, one query row per thread (TMEM lane = row): the score row in one TMEM round trip,
//               row max, exp2, P_j rounded to bf16 into TMEM, and the FlashAttention rescale of the TMEM
//               accumulator (O *= alpha, lazily: only when a row's reference maximum moved) before O += P_j V_j.
// S_{j+1} is computed while the softmax warps work on tile j.  TMEM holds S (128 columns), P (64) and O (64):
// 256 columns, so two CTAs share an SM.  The causal mask only touches the diagonal tile.  P is rounded to
// bf16 before P.V and the row sums use the unrounded fp32 probabilities, as the FlashAttention-2 kernel the
// reference calls does.
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace pattn {

constexpr int kBQ = 128;                       // queries per CTA = TMEM lanes
constexpr int kBK = 128;                       // keys per tile
constexpr int kStages = 2;                     // K/V ring depth
constexpr int kThreads = 192;
constexpr int kTileBytes = 128 * 128;          // 128 rows x 64 bf16 (Q, K or V tile)
constexpr int kQOff = 0;
constexpr int kKVOff = kTileBytes;                         // stage s: K at kKVOff + 2s tiles, V right after
constexpr int kBarOff = kKVOff + kStages * 2 * kTileBytes;
constexpr int kSmemBytes = kBarOff + 128 + 1024;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192;
static_assert(kKVOff % 1024 == 0 && kBarOff % 1024 == 0, "tiles must be 1024-aligned");

struct PrefillArgs {
  const int32_t* cu_seqlens;  // [nseq + 1]
  int nseq;
  int row0;                   // cache row of sequence 0
  int n_qtiles;               // grid.x: max over sequences of ceil(T_b / 128)
  int S;                      // cache positions per row
  __nv_bfloat16* out;         // [n_tok, 8, 64]
  float scale_log2;
};

// Shared-memory descriptor of an MN-major operand tile written by TMA with 128-byte swizzle: rows of 128
// bytes (64 bf16 along MN), 8-row swizzle atoms 1024 bytes apart along K; the MN extent is one atom.
VK_DEV uint64_t sdesc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (one MN atom: unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: next 8 K rows
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

__global__ void __launch_bounds__(kThreads, 2)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;   // S_j in TMEM
  uint64_t* s_free = s_full + 1;           // the softmax warps have read S_j
  uint64_t* p_full = s_free + 1;           // P_j in TMEM and O rescaled
  uint64_t* o_full = p_full + 1;           // O += P_j V_j done (P and O free again)
  uint64_t* tmem_free = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_free + 1);

  const int qt = a.n_qtiles - 1 - static_cast<int>(blockIdx.x);
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq >> 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_wait();
  const int t0 = a.cu_seqlens[b];
  const int T = a.cu_seqlens[b + 1] - t0;
  if (qt * kBQ >= T) return;
  if (T > a.S) {
    if (threadIdx.x == 0 && qt == 0) raise_error(ERR_BOUNDS);
    return;
  }
  const int nkv = qt + 1;  // key tiles 0..qt
  const int crow = a.row0 + b;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(tmem_free, 4);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(q_full, kTileBytes);
      tma_load_3d(smem + kQOff, &tmQ, q_full, 0, hq, t0 + qt * kBQ);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) & 1) ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          break;
        }
        uint8_t* kt = smem + kKVOff + s * 2 * kTileBytes;
        mbar_expect_tx(&kv_full[s], 2 * kTileBytes);
        tma_load_4d(kt, &tmK, &kv_full[s], 0, hkv, j * kBK, crow);
        tma_load_4d(kt + kTileBytes, &tmV, &kv_full[s], 0, hkv, j * kBK, crow);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kBQ, kBK);
      constexpr uint32_t idesc_o = idesc_bf16_f32(kBQ, 64) | (1u << 16);  // B (V) is MN-major
      const uint64_t qd = sdesc_k_sw128(smem_u32(smem + kQOff));
      bool ok = mbar_wait(q_full, 0);
      if (!ok) raise_error(ERR_WAIT_FULL);
      auto issue_pv = [&](int k) {
        if (!mbar_wait(p_full, k & 1)) {
          raise_error(ERR_WAIT_FULL);
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + kKVOff + (k % kStages) * 2 * kTileBytes + kTileBytes);
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks)
          umma_bf16_tmem_a(tmem_base + kColO, tmem_base + kColP + ks * 8, sdesc_mn_sw128(v_base + ks * 2048),
                           idesc_o, (k | ks) != 0);
        umma_commit(o_full);
        umma_commit(&kv_empty[k % kStages]);
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&kv_full[s], (j / kStages) & 1) || (j >= 1 && !mbar_wait(s_free, (j - 1) & 1))) {
          raise_error(ERR_WAIT_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t kd = sdesc_k_sw128(smem_u32(smem + kKVOff + s * 2 * kTileBytes));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) umma_bf16(tmem_base + kColS, qd + 2 * ks, kd + 2 * ks, idesc_s, ks != 0);
        umma_commit(s_full);
        if (j >= 1) issue_pv(j - 1);
      }
      if (ok) issue_pv(nkv - 1);
    }
  } else {
    // ---------------- softmax warps ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qpos = qt * kBQ + row;  // position of this row's query in its sequence
    const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, ok && mbar_wait(s_full, j & 1));
      if (!ok) {
        if (lane == 0) raise_error(ERR_WAIT_ACCUM);
        break;
      }
      tc_fence_after();
      const bool diag = j == qt;
      const int key0 = j * kBK;
      // the whole score row in one round trip to TMEM; then S may be overwritten by S_{j+1}
      float v[kBK];
#pragma unroll
      for (int c0 = 0; c0 < kBK; c0 += 16) tmem_ld16(trow + kColS + c0, v + c0);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      // row max of the raw scores (the scale is positive); the causal mask only on the diagonal tile
      if (diag) {
#pragma unroll
        for (int i = 0; i < kBK; ++i)
          if (key0 + i > qpos) v[i] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = v[k];
#pragma unroll
      for (int i = 8; i < kBK; i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(mx8[k], v[i + k]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * a.scale_log2;
      // Lazy rescale: the exponentials keep using the row's current reference maximum m unless the tile's
      // maximum exceeds it by more than 8 (log2 units); then probabilities stay below 2^8, exact in fp32 and
      // bf16-rounded with the same relative error, and most tiles need no accumulator rescale.
      const float m_new = (mx > m + 8.f || m == -INFINITY) ? fmaxf(m, mx) : m;
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m - mu);
      // O += P_{j-1} V_{j-1} must have finished before P_j and the rescale overwrite P and O
      if (j >= 1) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_full, (j - 1) & 1));
        if (!ok) {
          if (lane == 0) raise_error(ERR_WAIT_ACCUM);
          break;
        }
        tc_fence_after();
      }
      // P_j = exp2(s * scale - mu) (bf16) into TMEM, 32 keys per store; partial row sums for ILP.  Scores are
      // taken in pairs with packed fp32x2 arithmetic (the softmax warps are bound by their instruction issue: an
      // FMA-pipe polynomial for part of the exponentials, to unload MUFU, measured slower).
      const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-mu, -mu);
      float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int c0 = 0; c0 < kBK; c0 += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 t = __ffma2_rn(make_float2(v[c0 + i], v[c0 + i + 1]), sc2, nm2);
          const float2 p = make_float2(fast_exp2(t.x), fast_exp2(t.y));
          rs4[(i >> 1) & 3] = __fadd2_rn(rs4[(i >> 1) & 3], p);
          pk[i / 2] = pack_bf16x2(p.x, p.y);
        }
        tmem_st16(trow + kColP + c0 / 2, pk);
      }
      const float2 rs2 = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
      const float rs = rs2.x + rs2.y;
      // rescale the accumulator when this warp's row maxima moved (alpha = 1 otherwise)
      if (j >= 1 && !__all_sync(0xffffffffu, alpha == 1.f)) {
        float o[64];
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) tmem_ld16(trow + kColO + c0, o + c0);
        tmem_wait_ld();
        uint32_t ob[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) ob[i] = __float_as_uint(o[i] * alpha);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) tmem_st16(trow + kColO + c0, ob + c0);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l = alpha * l + rs;
      m = m_new;
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_full, (nkv - 1) & 1));
      if (!ok && lane == 0) raise_error(ERR_WAIT_ACCUM);
    }
    if (ok) {
      tc_fence_after();
      float o[64];
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) tmem_ld16(trow + kColO + c0, o + c0);
      tmem_wait_ld();
      if (qpos < T) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* op = a.out + (static_cast<int64_t>(t0 + qpos) * 8 + hq) * 64;
#pragma unroll
        for (int i = 0; i < 64; i += 8) {
          uint4 u;
          u.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
          u.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
          u.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
          u.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(op + i) = u;
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_free);
  }

  if (warp == 1) {
    // free TMEM once the softmax warps are done with it (they waited on every MMA)
    if (!mbar_wait(tmem_free, 0) && lane == 0) raise_error(ERR_WAIT_ACCUM);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace pattn
}  // namespace vk
