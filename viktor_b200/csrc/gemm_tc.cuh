// tcgen05 GEMM for the decoder projections:  C[M, N] = A[M, K] * B[N, K]^T  (bf16 in, fp32 accumulate in TMEM).
//
// One CTA computes one 128 x BN tile.  Warp roles (192 threads):
//   warp 0      TMA producer (one elected lane): A and B K-major tiles, 128-byte swizzle, STAGES-deep ring
//   warp 1      TMEM allocator + MMA issuer (one elected lane): tcgen05.mma kind::f16, M=128, N=BN, K=16 x 4
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (thread = one output row = one TMEM lane), then the
//               fused epilogue writes the result straight to global memory.
//
// Fused epilogues (each restates a reference op on the GEMM output, see the per-epilogue comments):
//   STORE_BF16 / STORE_F32   plain y = acc (viktor/triton_ops.py:111-146 without SwiGLU; fp32 logits)
//   BIAS_ACT                 y = act(bf16(acc + bias)), act = identity | GELU(erf); optional output row map
//                            (projector, viktor/model.py:35, and the packed-prefill scatter, viktor/engine.py:163-165)
//   SWIGLU                   B rows = [gate block | up block]: y = bf16(bf16(silu(bf16 g)) * bf16 u)
//                            (viktor/triton_ops.py:129-134, :212-220)
//   QKV_ROPE                 per 64-column head: QK-RMSNorm, RoPE, q store, K/V cache write
//                            (viktor/triton_ops.py:43-91)
//   ADD_RMSNORM              x += bf16(acc) in place; h = bf16(x * rsqrt(mean(x^2) + eps) * w).  The row spans
//                            the N/BN CTAs of a thread-block cluster; per-row partial sums of squares are
//                            exchanged through distributed shared memory (viktor/triton_ops.py:17-31)
#pragma once

#include "vk_common.cuh"

namespace vk {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

enum Epi : int { STORE_BF16 = 0, STORE_F32 = 1, BIAS_ACT = 2, SWIGLU = 3, QKV_ROPE = 4, ADD_RMSNORM = 5 };

struct EpiArgs {
  // STORE_*, BIAS_ACT, SWIGLU
  void* y;
  int64_t ldy;
  int n_valid;                     // output columns that exist (STORE_*: <= N)
  const int32_t* row_map;          // BIAS_ACT: output row of each input row (nullptr = identity)
  const __nv_bfloat16* bias;       // BIAS_ACT
  int act;                         // BIAS_ACT: 0 identity, 1 GELU(erf)
  // QKV_ROPE
  __nv_bfloat16* q_out;            // [M, H, 64]
  __nv_bfloat16* k_cache;          // one layer: [rows, S, Hkv, 64] with the strides below
  __nv_bfloat16* v_cache;
  __nv_bfloat16* k_out;            // optional packed [M, Hkv, 64]
  __nv_bfloat16* v_out;
  const int32_t* pos;              // cache position of each token
  const int32_t* rope_pos;         // RoPE position of each token
  const int32_t* seq;              // cache row of each token
  const __nv_bfloat16* q_norm_w;   // [64]
  const __nv_bfloat16* k_norm_w;   // [64]
  const float* cos;                // [rope_len, 32]
  const float* sin;
  int rope_len;
  int cache_rows, cache_len;       // bounds of the cache (rows, positions)
  int64_t stride_cb, stride_cs;    // cache strides in elements
  int n_heads, n_kv_heads;
  float eps;
  // ADD_RMSNORM
  __nv_bfloat16* x;                // residual [M, N], updated in place
  const __nv_bfloat16* norm_w;     // [N]
  __nv_bfloat16* h_out;            // [M, N]
};

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int RED_OFF = BAR_OFF + 256;
  static constexpr int TOTAL = RED_OFF + BM * 4 + 1024;  // + alignment slack
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
VK_DEV float silu(float g) { return g * (1.0f / (1.0f + __expf(-g))); }

// QK-RMSNorm + RoPE of one 64-wide head held by this thread (viktor/triton_ops.py:44-49).
VK_DEV void norm_rope_head(float* v, const __nv_bfloat16* w, const float* c, const float* s, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) ss += v[i] * v[i];
  const float r = rsqrtf(ss * (1.0f / 64.0f) + eps);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float y1 = bf16_round(v[i] * r * __bfloat162float(w[i]));
    const float y2 = bf16_round(v[i + 32] * r * __bfloat162float(w[i + 32]));
    v[i] = y1 * c[i] - y2 * s[i];
    v[i + 32] = y1 * s[i] + y2 * c[i];
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                int K, EpiArgs ep) {
  using L = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + L::RED_OFF);
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m0 = blockIdx.y * BM;
  const int num_kb = K / BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
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

  if (warp == 0) {
    if (lane == 0) {
      // Weights do not depend on the previous kernel: start them before waiting on it.
      const int pre = num_kb < STAGES ? num_kb : STAGES;
      for (int kb = 0; kb < pre; ++kb) {
        uint8_t* sB = smem + kb * L::STAGE_BYTES + L::A_BYTES;
        mbar_expect_tx(&full[kb], L::STAGE_BYTES);
        if (EPI == SWIGLU) {
          tma_load_2d(sB, &tmB, &full[kb], kb * BK, n_tile * (BN / 2));
          tma_load_2d(sB + L::B_BYTES / 2, &tmB, &full[kb], kb * BK, N / 2 + n_tile * (BN / 2));
        } else {
          tma_load_2d(sB, &tmB, &full[kb], kb * BK, n_tile * BN);
        }
      }
      pdl_wait();
      for (int kb = 0; kb < pre; ++kb) tma_load_2d(smem + kb * L::STAGE_BYTES, &tmA, &full[kb], kb * BK, m0);
      for (int kb = pre; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (*abort_flag) break;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          raise_error(ERR_WAIT_EMPTY);
          *abort_flag = 1;
          break;
        }
        uint8_t* sA = smem + s * L::STAGE_BYTES;
        uint8_t* sB = sA + L::A_BYTES;
        mbar_expect_tx(&full[s], L::STAGE_BYTES);
        tma_load_2d(sA, &tmA, &full[s], kb * BK, m0);
        if (EPI == SWIGLU) {
          tma_load_2d(sB, &tmB, &full[s], kb * BK, n_tile * (BN / 2));
          tma_load_2d(sB + L::B_BYTES / 2, &tmB, &full[s], kb * BK, N / 2 + n_tile * (BN / 2));
        } else {
          tma_load_2d(sB, &tmB, &full[s], kb * BK, n_tile * BN);
        }
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) {
          raise_error(ERR_WAIT_FULL);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sdesc_k_sw128(smem_u32(smem + s * L::STAGE_BYTES));
        const uint64_t bd = sdesc_k_sw128(smem_u32(smem + s * L::STAGE_BYTES + L::A_BYTES));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) umma_bf16(tmem_base, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(accum);
    }
    __syncwarp();
  } else {
    pdl_wait();
  }

  // ---------------- epilogue (warps 2..5) ----------------
  // tcgen05.ld is warp-collective: every lane of an epilogue warp issues the same loads; only the global
  // stores are predicated on the row being inside M.
  __syncwarp();
  const bool epi_warp = warp >= 2;
  const int quarter = warp & 3;
  const int row_local = quarter * 32 + lane;
  const int row = m0 + row_local;
  const bool row_ok = row < M;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  bool have_acc = false;
  if (epi_warp) {
    have_acc = __all_sync(0xffffffffu, mbar_wait(accum, 0));
    if (!have_acc && lane == 0) {
      raise_error(ERR_WAIT_ACCUM);
      *abort_flag = 1;
    }
    tc_fence_after();
  }
  pdl_launch_dependents();

  if (EPI == ADD_RMSNORM) {
    // Phase 1: x_new = bf16(x + bf16(acc)) over this CTA's BN columns; partial sum of squares.
    const int n0 = n_tile * BN;
    if (epi_warp && have_acc) {
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(taddr + c, v);
        tmem_wait_ld();
        if (row_ok) {
          __nv_bfloat16* xp = ep.x + static_cast<int64_t>(row) * N + n0 + c;
          float xo[16];
          load_bf16x8(xp, xo);
          load_bf16x8(xp + 8, xo + 8);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xo[i] = bf16_round(xo[i] + bf16_round(v[i]));
            ss += xo[i] * xo[i];
          }
          store_bf16x8(xp, xo);
          store_bf16x8(xp + 8, xo + 8);
        }
      }
      red[row_local] = ss;
    }
    cluster_sync();
    // Phase 2: full-row sum of squares from every CTA of the cluster, then h = bf16(x * r * w).
    if (epi_warp && have_acc && row_ok) {
      const uint32_t cs = static_cast<uint32_t>(N / BN);
      float tot = 0.f;
      for (uint32_t r = 0; r < cs; ++r) tot += ld_dsmem_f32(&red[row_local], r);
      const float rr = rsqrtf(tot / static_cast<float>(N) + ep.eps);
      const __nv_bfloat16* xp = ep.x + static_cast<int64_t>(row) * N + n0;
      __nv_bfloat16* hp = ep.h_out + static_cast<int64_t>(row) * N + n0;
#pragma unroll 1
      for (int c = 0; c < BN; c += 8) {
        float xv[8], hv[8];
        load_bf16x8(xp + c, xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) hv[i] = xv[i] * rr * __bfloat162float(ep.norm_w[n0 + c + i]);
        store_bf16x8(hp + c, hv);
      }
    }
    cluster_sync();
  } else if (epi_warp && have_acc) {
    if (EPI == STORE_BF16 || EPI == STORE_F32 || EPI == BIAS_ACT) {
      const int n0 = n_tile * BN;
      const int64_t orow = (EPI == BIAS_ACT && ep.row_map && row_ok) ? ep.row_map[row] : row;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(taddr + c, v);
        tmem_wait_ld();
        if (!row_ok) continue;
        const int col = n0 + c;
        if (EPI == BIAS_ACT) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float t = bf16_round(v[i] + (col + i < ep.n_valid ? __bfloat162float(ep.bias[col + i]) : 0.f));
            v[i] = ep.act == 1 ? gelu_erf(t) : t;
          }
        }
        if (EPI == STORE_F32) {
          float* yp = reinterpret_cast<float*>(ep.y) + orow * ep.ldy + col;
          if (col + 16 <= ep.n_valid && (ep.ldy & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(yp + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 16; ++i)
              if (col + i < ep.n_valid) yp[i] = v[i];
          }
        } else {
          __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(ep.y) + orow * ep.ldy + col;
          if (col + 16 <= ep.n_valid && (ep.ldy & 7) == 0) {
            store_bf16x8(yp, v);
            store_bf16x8(yp + 8, v + 8);
          } else {
            for (int i = 0; i < 16; ++i)
              if (col + i < ep.n_valid) yp[i] = __float2bfloat16_rn(v[i]);
          }
        }
      }
    } else if (EPI == SWIGLU) {
      const int F = N / 2;
      const int o0 = n_tile * (BN / 2);
      __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(ep.y) + static_cast<int64_t>(row) * ep.ldy + o0;
#pragma unroll 1
      for (int c = 0; c < BN / 2; c += 16) {
        float g[16], u[16];
        tmem_ld16(taddr + c, g);
        tmem_ld16(taddr + BN / 2 + c, u);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float gb = bf16_round(g[i]);
          g[i] = bf16_round(silu(gb)) * bf16_round(u[i]);
        }
        if (row_ok && o0 + c + 16 <= F) {
          store_bf16x8(yp + c, g);
          store_bf16x8(yp + c + 8, g + 8);
        }
      }
    } else if (EPI == QKV_ROPE) {
      const int H = ep.n_heads, HKV = ep.n_kv_heads;
      const int p = row_ok ? ep.pos[row] : 0;
      const int rp = row_ok ? (ep.rope_pos ? ep.rope_pos[row] : p) : 0;
      const int sq = row_ok ? ep.seq[row] : 0;
      const bool in_cache = p >= 0 && p < ep.cache_len && sq >= 0 && sq < ep.cache_rows;
      const bool in_rope = rp >= 0 && rp < ep.rope_len;
      const bool ok = row_ok && in_cache && in_rope;
      if (row_ok && !(in_cache && in_rope)) raise_error(ERR_BOUNDS);
      float c[32], s[32];
      {
        const float4* cp = reinterpret_cast<const float4*>(ep.cos + static_cast<int64_t>(ok ? rp : 0) * 32);
        const float4* sp = reinterpret_cast<const float4*>(ep.sin + static_cast<int64_t>(ok ? rp : 0) * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 a = cp[i], b = sp[i];
          c[4 * i] = a.x; c[4 * i + 1] = a.y; c[4 * i + 2] = a.z; c[4 * i + 3] = a.w;
          s[4 * i] = b.x; s[4 * i + 1] = b.y; s[4 * i + 2] = b.z; s[4 * i + 3] = b.w;
        }
      }
#pragma unroll 1
      for (int hh = 0; hh < BN / 64; ++hh) {
        const int gh = n_tile * (BN / 64) + hh;
        float v[64];
        tmem_ld16(taddr + hh * 64, v);
        tmem_ld16(taddr + hh * 64 + 16, v + 16);
        tmem_ld16(taddr + hh * 64 + 32, v + 32);
        tmem_ld16(taddr + hh * 64 + 48, v + 48);
        tmem_wait_ld();
        if (!ok) continue;
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = bf16_round(v[i]);  // the qkv linear output is stored in bf16
        if (gh < H) {
          norm_rope_head(v, ep.q_norm_w, c, s, ep.eps);
          __nv_bfloat16* qp = ep.q_out + (static_cast<int64_t>(row) * H + gh) * 64;
#pragma unroll
          for (int i = 0; i < 64; i += 8) store_bf16x8(qp + i, v + i);
        } else if (gh < H + 2 * HKV) {
          const bool is_k = gh < H + HKV;
          const int kvh = is_k ? gh - H : gh - H - HKV;
          if (is_k) norm_rope_head(v, ep.k_norm_w, c, s, ep.eps);
          __nv_bfloat16* cache = is_k ? ep.k_cache : ep.v_cache;
          __nv_bfloat16* dst =
              cache + static_cast<int64_t>(sq) * ep.stride_cb + static_cast<int64_t>(p) * ep.stride_cs + kvh * 64;
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
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace vk
