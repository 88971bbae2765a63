// C ABI of the viktor_b200 kernels (declared in include/viktor_b200.h).  Single translation unit: the kernel
// headers are included here so that all kernels share one device error word without relocatable device code.
#include <algorithm>
#include <cstring>
#include <utility>

#include "decode_attention.cuh"
#include "elementwise.cuh"
#include "gemm_tc.cuh"
#include "prefill_attention.cuh"
#include "stitch_host.h"
#include "vk_host.cuh"

namespace vk {

static int g_pdl = 1;

#ifndef VK_ATTN_MAX_CHUNK
#define VK_ATTN_MAX_CHUNK 1024
#endif

// Per-device record of kernels whose dynamic shared-memory limit has been raised.  The first launch of each
// kernel on a device must happen outside stream capture (engines warm up eagerly before capturing).
template <typename K>
static bool ensure_smem(K kernel, int bytes) {
  struct Entry {
    const void* fn;
    uint64_t mask;
  };
  static Entry table[64];
  static int used = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = 1ull << (dev & 63);
  const void* fn = reinterpret_cast<const void*>(kernel);
  int i = 0;
  for (; i < used; ++i)
    if (table[i].fn == fn) break;
  if (i < used && (table[i].mask & bit)) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (i == used) {
    if (used == 64) return true;
    table[used++] = Entry{fn, 0};
  }
  table[i].mask |= bit;
  return true;
}

template <typename... KArgs, typename... Args>
static int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, int cluster_x,
                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (g_pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = cluster_x;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    fprintf(stderr, "viktor_b200: launch failed: %s\n", cudaGetErrorString(e));
    return VK_ERR_CUDA;
  }
  return VK_OK;
}

// SMs of the current device (cached per device); 0 if the runtime cannot tell.
static int device_sm_count() {
  static int sm_count[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!sm_count[dev] && cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return sm_count[dev];
}

static inline unsigned blocks_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

constexpr int64_t kSmallM = 4096;  // decode-sized GEMMs: narrow tiles + split-K clusters; prefill: wide tiles

// ---- GEMM dispatch ----------------------------------------------------------------------------------------
template <int BN, int EPI, int NK>
static int run_gemm_nk(const void* A, const void* B, int64_t M, int N, int K, const gemm::EpiArgs& ep, int n_tiles,
                       int64_t b_rows, void* stream) {
  using gemm::SmemLayout;
  const int nkb = K / gemm::BK / NK;
  int cap = gemm::max_stages_for(BN);
  if (M <= kSmallM) {
    cap = gemm::kMaxStages;
    while (cap > 2 && SmemLayout(BN, NK, cap, EPI).total > gemm::kSmemBudget) --cap;
  }
  const int stages = nkb < cap ? nkb : cap;
  const SmemLayout L(BN, NK, stages, EPI);
  CUtensorMap ta, tb;
  const uint32_t b_box = EPI == gemm::SWIGLU ? BN / 2 : BN;
  if (!make_map_kmajor(&ta, A, static_cast<uint64_t>(M), K, K, gemm::BM)) return VK_ERR_ARG;
  if (!make_map_kmajor(&tb, B, static_cast<uint64_t>(b_rows), K, K, b_box)) return VK_ERR_ARG;
  auto kern = gemm::gemm_kernel<BN, EPI, NK>;
  if (!ensure_smem(kern, gemm::kSmemBudget)) return VK_ERR_CUDA;
  dim3 grid(NK, n_tiles, static_cast<unsigned>((M + gemm::BM - 1) / gemm::BM));
  return launch(kern, grid, dim3(gemm::kThreads), L.total, stream, NK, ta, tb, static_cast<int>(M), N, K, stages,
                ep);
}

// Split-K factor for small-M GEMMs.  A decode GEMM is bound by latency (load round trips, the epilogue), not
// by throughput, so it is split over K as far as one wave allows: the largest power of two, at most
// VK_MAX_SPLITK (a build-time tuning constant, 8 by default), with tiles x splits CTAs on at most one SM each
// and every split at least two 64-wide K blocks.  (Measured on B200, full decode steps with two row groups in
// one CUDA graph: a second wave costs more than the shorter K loop saves, and one-block splits cost more in
// the reduction than they save in the K loop.)
#ifndef VK_MAX_SPLITK
#define VK_MAX_SPLITK 8
#endif
static int pick_nk(int64_t M, int n_tiles, int K) {
  const int64_t tiles = n_tiles * ((M + gemm::BM - 1) / gemm::BM);
  const int kb = K / gemm::BK;
  const int sms = device_sm_count();
  int nk = 1;
  while (nk < VK_MAX_SPLITK && tiles * nk * 2 <= sms && kb % (nk * 2) == 0 && kb / (nk * 2) >= 2) nk *= 2;
  return nk;
}

template <int BN, int EPI>
static int run_gemm(const void* A, const void* B, int64_t M, int N, int K, const gemm::EpiArgs& ep, int n_tiles,
                    int64_t b_rows, int nk, void* stream) {
  if (M <= 0 || M > (int64_t(1) << 31) - 128) return VK_ERR_ARG;
  if (K <= 0 || K % gemm::BK != 0 || (K / gemm::BK) % nk != 0) return VK_ERR_ARG;
  if (!aligned16(A) || !aligned16(B)) return VK_ERR_ARG;
  switch (nk) {
    case 1: return run_gemm_nk<BN, EPI, 1>(A, B, M, N, K, ep, n_tiles, b_rows, stream);
    case 2: return run_gemm_nk<BN, EPI, 2>(A, B, M, N, K, ep, n_tiles, b_rows, stream);
    case 4: return run_gemm_nk<BN, EPI, 4>(A, B, M, N, K, ep, n_tiles, b_rows, stream);
    case 8: return run_gemm_nk<BN, EPI, 8>(A, B, M, N, K, ep, n_tiles, b_rows, stream);
    default: return VK_ERR_ARG;
  }
}

// Large-M GEMMs (prefill): the persistent BN = 256 kernel when N fits its tiles.
#ifndef VK_PERSISTENT_GEMM
#define VK_PERSISTENT_GEMM 1
#endif
template <int EPI>
static bool persistent_fits(int64_t M, int N) {
  if (!VK_PERSISTENT_GEMM || M <= 0 || M > (int64_t(1) << 31) - 128) return false;
  return EPI == gemm::SWIGLU ? (N / 2) % (gemm::kPBN / 2) == 0 && N % 2 == 0 : N % gemm::kPBN == 0;
}

template <int EPI>
static int run_gemm_persistent(const void* A, const void* B, int64_t M, int N, int K, const gemm::EpiArgs& ep,
                               int64_t b_rows, void* stream) {
  if (K <= 0 || K % gemm::BK != 0) return VK_ERR_ARG;
  if (!aligned16(A) || !aligned16(B)) return VK_ERR_ARG;
  CUtensorMap ta, tb;
  const uint32_t b_box = EPI == gemm::SWIGLU ? gemm::kPBN / 2 : gemm::kPBN;
  if (!make_map_kmajor(&ta, A, static_cast<uint64_t>(M), K, K, gemm::BM)) return VK_ERR_ARG;
  if (!make_map_kmajor(&tb, B, static_cast<uint64_t>(b_rows), K, K, b_box)) return VK_ERR_ARG;
  const int sms = device_sm_count();
  if (sms <= 0) return VK_ERR_CUDA;
  const int64_t n_tiles = (EPI == gemm::SWIGLU ? N / 2 : N) / b_box;
  const int64_t tiles = n_tiles * ((M + gemm::BM - 1) / gemm::BM);
  auto kern = gemm::gemm_persistent_kernel<EPI>;
  if (!ensure_smem(kern, gemm::kPSmemBytes)) return VK_ERR_CUDA;
  return launch(kern, dim3(static_cast<unsigned>(tiles < sms ? tiles : sms)), dim3(gemm::kPThreads),
                gemm::kPSmemBytes, stream, 1, ta, tb, static_cast<int>(M), N, K, ep);
}

static gemm::EpiArgs epi_zero() {
  gemm::EpiArgs e;
  memset(&e, 0, sizeof(e));
  return e;
}

// Failure-path probe: one CTA whose first thread waits on an mbarrier that nothing arrives on (no copy in flight,
// no other thread involved).  The bounded wait gives up after limit_ns, the thread records ERR_WAIT_FULL exactly
// as a pipeline wait that ran out does, writes how long it waited and the kernel returns normally.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, unsigned long long* waited_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    const bool done = mbar_wait_for(&bar, 0, limit_ns);
    if (!done) raise_error(ERR_WAIT_FULL);
    if (waited_ns) *waited_ns = globaltimer() - t0;
  }
}


}  // namespace vk

using namespace vk;

extern "C" {

int vk_version(void) { return 100; }

int vk_read_device_errors(uint32_t* bits, int clear) {
  if (!bits) return VK_ERR_ARG;
  if (cudaMemcpyFromSymbol(bits, vk::g_error_word, sizeof(uint32_t)) != cudaSuccess) return VK_ERR_CUDA;
  if (clear) {
    const uint32_t z = 0;
    if (cudaMemcpyToSymbol(vk::g_error_word, &z, sizeof(uint32_t)) != cudaSuccess) return VK_ERR_CUDA;
  }
  return VK_OK;
}

int vk_set_pdl(int enable) {
  vk::g_pdl = enable ? 1 : 0;
  return VK_OK;
}

int vk_test_bounded_wait(uint64_t limit_ns, unsigned long long* waited_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > vk::kWaitLimitNs) return VK_ERR_ARG;
  bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, waited_ns);
  return cudaGetLastError() == cudaSuccess ? VK_OK : VK_ERR_CUDA;
}

int vk_add_rmsnorm(void* x, const void* delta, const void* w, void* h, int64_t n, int d, float eps, void* stream) {
  if (n < 0 || d != 512 || !x || !w || !h) return n == 0 ? VK_OK : VK_ERR_ARG;
  if (n == 0) return VK_OK;
  if (!aligned16(x) || !aligned16(w) || !aligned16(h) || (delta && !aligned16(delta))) return VK_ERR_ARG;
  return launch(ew::rmsnorm_rows_kernel<512>, dim3(blocks_for(n, 8)), dim3(256), 0, stream, 1,
                static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(delta),
                static_cast<const int64_t*>(nullptr), static_cast<const __nv_bfloat16*>(nullptr), int64_t(0),
                static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(h), n, eps);
}

int vk_embed_rmsnorm(const int64_t* tok, const void* emb, int64_t vocab, const void* w, void* x, void* h, int64_t n,
                     int d, float eps, void* stream) {
  if (n == 0) return VK_OK;
  if (n < 0 || d != 512 || !tok || !emb || !w || !x || !h || vocab <= 0) return VK_ERR_ARG;
  if (!aligned16(emb) || !aligned16(w) || !aligned16(x) || !aligned16(h)) return VK_ERR_ARG;
  return launch(ew::rmsnorm_rows_kernel<512>, dim3(blocks_for(n, 8)), dim3(256), 0, stream, 1,
                static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(nullptr), tok,
                static_cast<const __nv_bfloat16*>(emb), vocab, static_cast<const __nv_bfloat16*>(w),
                static_cast<__nv_bfloat16*>(h), n, eps);
}

int vk_qkv_rope_cache(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos,
                      const float* sin, int rope_len, const int32_t* pos, const int32_t* rope_pos,
                      const int32_t* seq, void* q, void* k_cache, void* v_cache, void* k_out, void* v_out,
                      int64_t n, int64_t stride_cb, int64_t stride_cs, int cache_rows, int cache_len, float eps,
                      int n_heads, int n_kv_heads, int head_dim, void* stream) {
  if (n == 0) return VK_OK;
  if (head_dim != 64 || n_heads <= 0 || n_kv_heads <= 0) return VK_ERR_UNSUPPORTED;
  if (n < 0 || !qkv || !q_norm_w || !k_norm_w || !cos || !sin || !pos || !seq || !q || !k_cache || !v_cache)
    return VK_ERR_ARG;
  if (!aligned16(qkv) || !aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || stride_cs % 8 ||
      stride_cb % 8 || (k_out && !aligned16(k_out)) || (v_out && !aligned16(v_out)))
    return VK_ERR_ARG;
  const int64_t threads = n * (n_heads + 2 * n_kv_heads);
  return launch(ew::qkv_rope_cache_kernel, dim3(blocks_for(threads, 128)), dim3(128), 0, stream, 1,
                static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(q_norm_w),
                static_cast<const __nv_bfloat16*>(k_norm_w), cos, sin, rope_len, pos, rope_pos, seq,
                static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k_cache),
                static_cast<__nv_bfloat16*>(v_cache), static_cast<__nv_bfloat16*>(k_out),
                static_cast<__nv_bfloat16*>(v_out), n, stride_cb, stride_cs, cache_rows, cache_len, eps, n_heads,
                n_kv_heads);
}

// Shared body of vk_linear / vk_linear_rmsnorm: plain or SwiGLU GEMM, bf16 or f32 out, optional folded norm.
static int linear_impl(const void* x, const float* ssq, float eps, const void* w, void* y, int64_t M, int N, int K,
                       int swiglu, int out_f32, void* stream) {
  if (M == 0) return VK_OK;
  if (!x || !w || !y || N <= 0 || M < 0) return VK_ERR_ARG;
  if (ssq && (K != 512 || !aligned16(ssq))) return VK_ERR_ARG;
  gemm::EpiArgs ep = epi_zero();
  ep.y = y;
  ep.ssq_in = ssq;
  ep.eps = eps;
  if (swiglu) {
    if (out_f32 || N % 2) return VK_ERR_ARG;
    const int F = N / 2;
    ep.ldy = F;
    ep.n_valid = F;
    if (M <= kSmallM) {
      if (F % 64) return VK_ERR_ARG;
      // narrow tiles (32 outputs) while they fit in one wave, for more CTAs in flight; else 64 outputs
      if ((F / 32) * ((M + gemm::BM - 1) / gemm::BM) <= device_sm_count())
        return run_gemm<64, gemm::SWIGLU>(x, w, M, N, K, ep, F / 32, N, pick_nk(M, F / 32, K), stream);
      return run_gemm<128, gemm::SWIGLU>(x, w, M, N, K, ep, F / 64, N, pick_nk(M, F / 64, K), stream);
    }
    if (F % 64) return VK_ERR_ARG;
    if (persistent_fits<gemm::SWIGLU>(M, N)) return run_gemm_persistent<gemm::SWIGLU>(x, w, M, N, K, ep, N, stream);
    return run_gemm<128, gemm::SWIGLU>(x, w, M, N, K, ep, F / 64, N, 1, stream);
  }
  ep.ldy = N;
  ep.n_valid = N;
  if (out_f32) {
    if (N <= 16) return run_gemm<16, gemm::STORE_F32>(x, w, M, N, K, ep, 1, N, pick_nk(M, 1, K), stream);
    const int nt = (N + 127) / 128;
    return run_gemm<128, gemm::STORE_F32>(x, w, M, N, K, ep, nt, N, M <= kSmallM ? pick_nk(M, nt, K) : 1, stream);
  }
  if (N <= 64 || M <= kSmallM) {
    const int nt = (N + 63) / 64;
    return run_gemm<64, gemm::STORE_BF16>(x, w, M, N, K, ep, nt, N, M <= kSmallM ? pick_nk(M, nt, K) : 1, stream);
  }
  if (persistent_fits<gemm::STORE_BF16>(M, N))
    return run_gemm_persistent<gemm::STORE_BF16>(x, w, M, N, K, ep, N, stream);
  return run_gemm<128, gemm::STORE_BF16>(x, w, M, N, K, ep, (N + 127) / 128, N, 1, stream);
}

int vk_linear(const void* x, const void* w, void* y, int64_t M, int N, int K, int swiglu, int out_f32,
              void* stream) {
  return linear_impl(x, nullptr, 0.f, w, y, M, N, K, swiglu, out_f32, stream);
}

int vk_linear_rmsnorm(const void* x, const float* ssq, float eps, const void* w_folded, void* y, int64_t M, int N,
                      int K, int swiglu, int out_f32, void* stream) {
  if (M != 0 && !ssq) return VK_ERR_ARG;
  return linear_impl(x, ssq, eps, w_folded, y, M, N, K, swiglu, out_f32, stream);
}

int vk_swiglu(const void* gu, void* out, int64_t n, int F, void* stream) {
  if (n == 0) return VK_OK;
  if (!gu || !out || n < 0 || F <= 0) return VK_ERR_ARG;
  return launch(ew::swiglu_kernel, dim3(blocks_for(n * F, 256)), dim3(256), 0, stream, 1,
                static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), n, F);
}

// Fields shared by the selection entry points (viktor/triton_ops.py:172-209, viktor/engine.py:79-89).
static ew::GreedyArgs greedy_args(const float* logits, int64_t ld_logits, const float* bias, const uint8_t* is_tail,
                                  const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run, int64_t* pos,
                                  const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                                  int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V,
                                  int eos, int pad, const void* emb, void* x, float* ssq) {
  ew::GreedyArgs a;
  memset(&a, 0, sizeof(a));
  a.logits = logits;
  a.ld_logits = ld_logits;
  a.bias = bias;
  a.is_tail = is_tail;
  a.is_homo = is_homo;
  a.homo_stop = homo_stop;
  a.tok = tok;
  a.run = run;
  a.pos = pos;
  a.plen = plen;
  a.rope_off = rope_off;
  a.out = out;
  a.out_stride = out_stride;
  a.out_cols = out_cols;
  a.pos32 = pos32;
  a.seqlens = seqlens;
  a.rpos32 = rpos32;
  a.B = B;
  a.V = V;
  a.eos = eos;
  a.pad = pad;
  a.emb = static_cast<const __nv_bfloat16*>(emb);
  a.x = static_cast<__nv_bfloat16*>(emb ? x : nullptr);
  a.ssq = ssq;
  a.temperature = 1.f;
  return a;
}

static bool greedy_state_ok(const float* bias, const uint8_t* is_tail, const uint8_t* is_homo, const int64_t* tok,
                            const int64_t* run, const int64_t* pos, const int64_t* plen, const int64_t* rope_off,
                            const int64_t* out, const int32_t* pos32, const int32_t* seqlens, const int32_t* rpos32,
                            int B, int V, const void* emb, const void* x, const float* ssq) {
  return B > 0 && V > 0 && bias && is_tail && is_homo && tok && run && pos && plen && rope_off && out && pos32 &&
         seqlens && rpos32 && (!emb || (x && ssq));
}

int vk_greedy_update(const float* logits, int64_t ld_logits, const float* bias, const uint8_t* is_tail,
                     const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run, int64_t* pos,
                     const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                     int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos,
                     int pad, const void* emb, void* x, float* ssq, void* stream) {
  if (B == 0) return VK_OK;
  if (!logits || !greedy_state_ok(bias, is_tail, is_homo, tok, run, pos, plen, rope_off, out, pos32, seqlens, rpos32,
                                  B, V, emb, x, ssq))
    return VK_ERR_ARG;
  const ew::GreedyArgs a = greedy_args(logits, ld_logits, bias, is_tail, is_homo, homo_stop, tok, run, pos, plen,
                                       rope_off, out, out_stride, out_cols, pos32, seqlens, rpos32, B, V, eos, pad,
                                       emb, x, ssq);
  return launch(ew::greedy_kernel<512>, dim3(B), dim3(128), 0, stream, 1, a);
}

int vk_prefill_plan(const int32_t* lens, int n, int row0, int pos_scale, int64_t total, int32_t* cu,
                    int32_t* frame_idx, int64_t* last, int32_t* pos, int32_t* seq, int32_t* rpos, int32_t* lengths,
                    void* stream) {
  if (n <= 0 || n > ew::kPlanMaxSeq || row0 < 0 || pos_scale < 1 || total < n || total > (int64_t(1) << 31) - 1 ||
      !lens || !cu || !last || !pos || !seq || !lengths || (total > n && !frame_idx))
    return VK_ERR_ARG;
  ew::PlanArgs a;
  a.lens = lens;
  a.n = n;
  a.row0 = row0;
  a.pos_scale = pos_scale;
  a.total = total;
  a.cu = cu;
  a.frame_idx = frame_idx;
  a.last = last;
  a.pos = pos;
  a.seq = seq;
  a.rpos = rpos;
  a.lengths = lengths;
  const int sms = device_sm_count();
  if (sms <= 0) return VK_ERR_CUDA;
  const int64_t want = (total + ew::kPlanThreads - 1) / ew::kPlanThreads;
  const unsigned grid = static_cast<unsigned>(want < 2 * sms ? want : 2 * sms);
  return launch(ew::prefill_plan_kernel, dim3(grid), dim3(ew::kPlanThreads), 0, stream, 1, a);
}

int vk_sample_update(const float* logits, int64_t ld_logits, const float* bias, const uint8_t* is_tail,
                     const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run, int64_t* pos,
                     const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                     int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos,
                     int pad, const void* emb, void* x, float* ssq, const float* noise, int64_t ld_noise,
                     float temperature, void* stream) {
  if (B == 0) return VK_OK;
  if (!logits || !greedy_state_ok(bias, is_tail, is_homo, tok, run, pos, plen, rope_off, out, pos32, seqlens, rpos32,
                                  B, V, emb, x, ssq) ||
      !noise || ld_noise < V || !(temperature > 0.f) || !(temperature < INFINITY))
    return VK_ERR_ARG;
  ew::GreedyArgs a = greedy_args(logits, ld_logits, bias, is_tail, is_homo, homo_stop, tok, run, pos, plen, rope_off,
                                 out, out_stride, out_cols, pos32, seqlens, rpos32, B, V, eos, pad, emb, x, ssq);
  a.noise = noise;
  a.ld_noise = ld_noise;
  a.temperature = temperature;
  return launch(ew::greedy_kernel<512>, dim3(B), dim3(128), 0, stream, 1, a);
}

int vk_head_select(const void* x_final, const float* ssq_final, float eps, const void* head_w, const float* bias,
                   const uint8_t* is_tail, const uint8_t* is_homo, int homo_stop, int64_t* tok, int64_t* run,
                   int64_t* pos, const int64_t* plen, const int64_t* rope_off, int64_t* out, int64_t out_stride,
                   int64_t out_cols, int32_t* pos32, int32_t* seqlens, int32_t* rpos32, int B, int V, int eos, int pad,
                   const void* emb, void* x, float* ssq, const float* noise, int64_t ld_noise, float temperature,
                   const int64_t* limit, int shrink_done, void* stream) {
  if (B == 0) return VK_OK;
  if (!x_final || !ssq_final || !head_w || V > ew::kHeadMaxV || !aligned16(x_final) || !aligned16(ssq_final) ||
      !aligned16(head_w) ||
      !greedy_state_ok(bias, is_tail, is_homo, tok, run, pos, plen, rope_off, out, pos32, seqlens, rpos32, B, V, emb,
                       x, ssq))
    return VK_ERR_ARG;
  if (noise && (ld_noise < V || !(temperature > 0.f) || !(temperature < INFINITY))) return VK_ERR_ARG;
  ew::GreedyArgs a = greedy_args(nullptr, 0, bias, is_tail, is_homo, homo_stop, tok, run, pos, plen, rope_off, out,
                                 out_stride, out_cols, pos32, seqlens, rpos32, B, V, eos, pad, emb, x, ssq);
  a.head_x = static_cast<const __nv_bfloat16*>(x_final);
  a.head_ssq = ssq_final;
  a.head_w = static_cast<const __nv_bfloat16*>(head_w);
  a.head_eps = eps;
  a.limit = limit;
  a.shrink_done = shrink_done ? 1 : 0;
  if (noise) {
    a.noise = noise;
    a.ld_noise = ld_noise;
    a.temperature = temperature;
  }
  return launch(ew::greedy_kernel<512>, dim3(B), dim3(128), 0, stream, 1, a);
}

size_t vk_decode_attention_workspace_bytes(int nq, int S) {
  if (nq <= 0 || S <= 0) return 0;
  const size_t splits = (S + attn::kMinChunk - 1) / attn::kMinChunk;
  const size_t counters = ((size_t)nq * 4 + 255) / 256 * 256;
  const size_t ml = ((size_t)nq * splits * 8 * 2 * 4 + 255) / 256 * 256;
  const size_t o = (size_t)nq * splits * 8 * 64 * 4;
  return counters + ml + o;
}

// TMA maps of one layer of the KV cache, [rows][S][2 heads][64] bf16: boxes of box_pos positions x one head.
static bool make_cache_maps(CUtensorMap* mk, CUtensorMap* mv, const void* k, const void* v, int cache_rows, int S,
                            int64_t stride_kb, int64_t stride_ks, uint32_t box_pos = 64) {
  uint64_t dims[4] = {64, 2, static_cast<uint64_t>(S), static_cast<uint64_t>(cache_rows)};
  uint64_t strides[3] = {128, static_cast<uint64_t>(stride_ks) * 2, static_cast<uint64_t>(stride_kb) * 2};
  uint32_t box[4] = {64, 1, box_pos, 1};
  return make_map_bf16(mk, k, 4, dims, strides, box, true) && make_map_bf16(mv, v, 4, dims, strides, box, true);
}

int vk_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* lengths, void* out,
                        int nq, int row0, int cache_rows, int S, int64_t stride_kb, int64_t stride_ks,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (nq == 0) return VK_OK;
  if (nq < 0 || !q || !k_cache || !v_cache || !lengths || !out || !workspace || S <= 0 || row0 < 0 ||
      row0 + nq > cache_rows || stride_ks < 128 || stride_kb < stride_ks * S)
    return VK_ERR_ARG;
  if (!aligned16(q) || !aligned16(out) || !aligned16(workspace)) return VK_ERR_ARG;
  if (workspace_bytes < vk_decode_attention_workspace_bytes(nq, S)) return VK_ERR_ARG;
  CUtensorMap mk, mv;
  if (!make_cache_maps(&mk, &mv, k_cache, v_cache, cache_rows, S, stride_kb, stride_ks)) return VK_ERR_ARG;
  const int splits = (S + attn::kMinChunk - 1) / attn::kMinChunk;  // workspace slots per query
  const int sms = device_sm_count();
  if (sms <= 0) return VK_ERR_CUDA;
  // longest split that still fills every SM with its two resident CTAs (judged on the cache length); at most
  // VK_ATTN_MAX_CHUNK positions (a build-time tuning constant)
  int chunk = VK_ATTN_MAX_CHUNK;
  while (chunk > attn::kMinChunk && static_cast<int64_t>(nq) * ((S + chunk - 1) / chunk) < 2 * sms) chunk /= 2;
  attn::DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lengths = lengths;
  a.row0 = row0;
  a.nq = nq;
  a.max_splits = splits;
  a.S = S;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.counters = reinterpret_cast<int*>(ws);
  const size_t counters = ((size_t)nq * 4 + 255) / 256 * 256;
  a.ws_ml = reinterpret_cast<float*>(ws + counters);
  a.ws_o = reinterpret_cast<float*>(ws + counters + ((size_t)nq * splits * 8 * 2 * 4 + 255) / 256 * 256);
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  a.chunk = chunk;
  if (!ensure_smem(attn::decode_attn_kernel, attn::kSmemBytes)) return VK_ERR_CUDA;
  return launch(attn::decode_attn_kernel, dim3((S + chunk - 1) / chunk, nq), dim3(attn::kThreads), attn::kSmemBytes,
                stream, 1, mk, mv, a);
}

// ---- int8 prefix KV ------------------------------------------------------------------------------------------
// Split plan of decode_attn_i8_kernel: bf16 splits of `chunk` positions and at most n8max int8 splits of about
// 2 x chunk positions (the same bytes per CTA), the longest chunk that still fills every SM twice.
struct I8Plan {
  int chunk, n8max, n16max;
};
static I8Plan i8_plan(int nq, int S8, int max_tail, int sms) {
  I8Plan p{};
  for (int c = 1024;; c /= 2) {
    p.chunk = c;
    p.n8max = (S8 + 2 * c - 1) / (2 * c);
    p.n16max = (max_tail + c - 1) / c;
    if (c == 128 || static_cast<int64_t>(nq) * (p.n8max + p.n16max) >= 2 * sms) break;
  }
  return p;
}
static size_t i8_slots_bound(int S8, int max_tail) { return (S8 + 255) / 256 + (max_tail + 127) / 128; }

size_t vk_decode_attention_i8_workspace_bytes(int nq, int S8, int max_tail) {
  if (nq <= 0 || S8 <= 0 || max_tail <= 0) return 0;
  const size_t splits = i8_slots_bound(S8, max_tail);
  const size_t counters = ((size_t)nq * 4 + 255) / 256 * 256;
  const size_t ml = ((size_t)nq * splits * 8 * 2 * 4 + 255) / 256 * 256;
  return counters + ml + (size_t)nq * splits * 8 * 64 * 4;
}

int vk_kv_quantize(const void* k_cache, const void* v_cache, int cache_rows, int S, int64_t stride_kb,
                   int64_t stride_ks, const int32_t* starts, int row0, int n, void* k8, void* v8t, float* sk,
                   float* sv, int S8, void* stream) {
  if (n == 0) return VK_OK;
  if (n < 0 || !k_cache || !v_cache || !starts || !k8 || !v8t || !sk || !sv || S <= 0 || row0 < 0 ||
      row0 + n > cache_rows || S8 <= 0 || S8 % 128 != 0 || stride_ks < 128 || stride_ks % 8 != 0 ||
      stride_kb < stride_ks * S || stride_kb % 8 != 0)
    return VK_ERR_ARG;
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(k8) || !aligned16(v8t) || !aligned16(sk) ||
      !aligned16(sv))
    return VK_ERR_ARG;
  attn::QuantArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.stride_kb = stride_kb;
  a.stride_ks = stride_ks;
  a.starts = starts;
  a.row0 = row0;
  a.n = n;
  a.S = S;
  a.S8 = S8;
  a.k8 = static_cast<uint8_t*>(k8);
  a.v8t = static_cast<uint8_t*>(v8t);
  a.sk = sk;
  a.sv = sv;
  return launch(attn::kv_quantize_kernel, dim3(n, 2), dim3(attn::kQuantThreads), 0, stream, 1, a);
}

int vk_decode_attention_i8(const void* q, const void* k_cache, const void* v_cache, const void* k8,
                           const void* v8t, const float* sk, const float* sv, const int32_t* starts,
                           const int32_t* lengths, void* out, int nq, int row0, int cache_rows, int S,
                           int64_t stride_kb, int64_t stride_ks, int S8, int max_tail, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (nq == 0) return VK_OK;
  if (nq < 0 || !q || !k_cache || !v_cache || !k8 || !v8t || !sk || !sv || !starts || !lengths || !out ||
      !workspace || S <= 0 || row0 < 0 || row0 + nq > cache_rows || stride_ks < 128 || stride_kb < stride_ks * S ||
      S8 <= 0 || S8 % 128 != 0 || max_tail <= 0 || max_tail > S)
    return VK_ERR_ARG;
  if (!aligned16(q) || !aligned16(out) || !aligned16(workspace) || !aligned16(sk) || !aligned16(sv))
    return VK_ERR_ARG;
  if (workspace_bytes < vk_decode_attention_i8_workspace_bytes(nq, S8, max_tail)) return VK_ERR_ARG;
  CUtensorMap mk, mv, mk8, mv8;
  if (!make_cache_maps(&mk, &mv, k_cache, v_cache, cache_rows, S, stride_kb, stride_ks)) return VK_ERR_ARG;
  {
    uint64_t dims[3] = {128, static_cast<uint64_t>(S8), static_cast<uint64_t>(cache_rows)};
    uint64_t strides[2] = {128, static_cast<uint64_t>(S8) * 128};
    uint32_t box[3] = {128, attn::kTile8, 1};
    if (!make_map_u8(&mk8, k8, 3, dims, strides, box, true)) return VK_ERR_ARG;
  }
  {
    uint64_t dims[4] = {attn::kTile8, 128, static_cast<uint64_t>(S8 / attn::kTile8), static_cast<uint64_t>(cache_rows)};
    uint64_t strides[3] = {attn::kTile8, attn::kTile8 * 128, static_cast<uint64_t>(S8) * 128};
    uint32_t box[4] = {attn::kTile8, 128, 1, 1};
    if (!make_map_u8(&mv8, v8t, 4, dims, strides, box, true)) return VK_ERR_ARG;
  }
  const int sms = device_sm_count();
  if (sms <= 0) return VK_ERR_CUDA;
  const I8Plan plan = i8_plan(nq, S8, max_tail, sms);
  attn::DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.lengths = lengths;
  a.row0 = row0;
  a.nq = nq;
  a.max_splits = plan.n8max + plan.n16max;
  a.S = S;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.counters = reinterpret_cast<int*>(ws);
  const size_t counters = ((size_t)nq * 4 + 255) / 256 * 256;
  a.ws_ml = reinterpret_cast<float*>(ws + counters);
  a.ws_o = reinterpret_cast<float*>(ws + counters + ((size_t)nq * a.max_splits * 8 * 2 * 4 + 255) / 256 * 256);
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  a.chunk = plan.chunk;
  a.starts = starts;
  a.n8max = plan.n8max;
  a.max_tail = max_tail;
  a.sk = sk;
  a.sv = sv;
  a.S8 = S8;
  if (!ensure_smem(attn::decode_attn_i8_kernel, attn::kSmemBytes8)) return VK_ERR_CUDA;
  return launch(attn::decode_attn_i8_kernel, dim3(nq, plan.n8max + plan.n16max), dim3(attn::kThreads),
                attn::kSmemBytes8, stream, 1, mk, mv, mk8, mv8, a);
}

}  // extern "C"

// ---- allocation-free decode attention -----------------------------------------------------------------------
// The split-K workspace of vk_decode_attention_noalloc: sized for 256 queries over 4096 cache positions (16
// splits of 256).  Zero at module load; each call clears the tickets it uses before the kernel runs.
namespace vk {
constexpr int kNoAllocMaxQ = 256;
constexpr int kNoAllocMaxS = 4096;
constexpr size_t kNoAllocSplits = (kNoAllocMaxS + attn::kMinChunk - 1) / attn::kMinChunk;
constexpr size_t kNoAllocBytes = 1024 + 256 * kNoAllocSplits * 8 * 2 * 4 + 256 * kNoAllocSplits * 8 * 64 * 4;
static __device__ __align__(256) uint8_t g_noalloc_attn_scratch[kNoAllocBytes];
}  // namespace vk

extern "C" {

int vk_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* lengths,
                                void* out, int nq, int row0, int cache_rows, int S, int64_t stride_kb,
                                int64_t stride_ks, void* stream) {
  if (nq == 0) return VK_OK;
  if (nq < 0 || nq > vk::kNoAllocMaxQ || S <= 0 || S > vk::kNoAllocMaxS) {
    fprintf(stderr,
            "viktor_b200: vk_decode_attention_noalloc supports at most %d queries and %d cache positions "
            "(got %d queries, %d positions); use vk_decode_attention with a caller-provided workspace\n",
            vk::kNoAllocMaxQ, vk::kNoAllocMaxS, nq, S);
    return VK_ERR_ARG;
  }
  const size_t need = vk_decode_attention_workspace_bytes(nq, S);
  if (need > vk::kNoAllocBytes) return VK_ERR_ARG;
  // Device address of the array, looked up once per device with that device current (host code cannot use the
  // symbol itself as a device pointer).
  static void* scratch[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VK_ERR_CUDA;
  // the array used is the current device's: a stream of another device would run against memory it cannot see
  int stream_dev = dev;
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_dev) != cudaSuccess) return VK_ERR_CUDA;
  if (stream_dev != dev) {
    fprintf(stderr, "viktor_b200: vk_decode_attention_noalloc: the stream belongs to device %d, the current device "
                    "is %d\n", stream_dev, dev);
    return VK_ERR_ARG;
  }
  if (!scratch[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, vk::g_noalloc_attn_scratch) != cudaSuccess || !p) {
      fprintf(stderr, "viktor_b200: cannot resolve the decode-attention scratch array on device %d\n", dev);
      return VK_ERR_CUDA;
    }
    scratch[dev] = p;
  }
  // the per-query tickets must start at zero (an earlier aborted call could have left them set)
  const size_t tickets = ((size_t)nq * 4 + 255) / 256 * 256;
  if (cudaMemsetAsync(scratch[dev], 0, tickets, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return VK_ERR_CUDA;
  return vk_decode_attention(q, k_cache, v_cache, lengths, out, nq, row0, cache_rows, S, stride_kb, stride_ks,
                             scratch[dev], vk::kNoAllocBytes, stream);
}

int vk_test_noalloc_poison(void* stream) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, vk::g_noalloc_attn_scratch) != cudaSuccess || !p) return VK_ERR_CUDA;
  const size_t tickets = static_cast<size_t>(vk::kNoAllocMaxQ) * 4;
  if (cudaMemsetAsync(p, 0x5A, tickets, static_cast<cudaStream_t>(stream)) != cudaSuccess) return VK_ERR_CUDA;
  return VK_OK;
}

int vk_prefill_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* cu_seqlens,
                         int nseq, int max_seqlen, int64_t n_tok, int row0, int cache_rows, int S,
                         int64_t stride_kb, int64_t stride_ks, void* out, void* stream) {
  if (nseq == 0 || n_tok == 0) return VK_OK;
  if (nseq < 0 || !q || !k_cache || !v_cache || !cu_seqlens || !out || max_seqlen <= 0 || max_seqlen > S ||
      row0 < 0 || row0 + nseq > cache_rows || stride_ks < 128 || stride_kb < stride_ks * S)
    return VK_ERR_ARG;
  if (!aligned16(q) || !aligned16(out)) return VK_ERR_ARG;
  CUtensorMap mq, mk, mv;
  {
    uint64_t dims[3] = {64, 8, static_cast<uint64_t>(n_tok)};
    uint64_t strides[2] = {128, 1024};
    uint32_t box[3] = {64, 1, pattn::kBQ};
    if (!make_map_bf16(&mq, q, 3, dims, strides, box, true)) return VK_ERR_ARG;
  }
  if (!make_cache_maps(&mk, &mv, k_cache, v_cache, cache_rows, S, stride_kb, stride_ks, pattn::kBK))
    return VK_ERR_ARG;
  pattn::PrefillArgs a;
  a.cu_seqlens = cu_seqlens;
  a.nseq = nseq;
  a.row0 = row0;
  a.n_qtiles = (max_seqlen + pattn::kBQ - 1) / pattn::kBQ;
  a.S = S;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  if (!ensure_smem(pattn::prefill_attn_kernel, pattn::kSmemBytes)) return VK_ERR_CUDA;
  return launch(pattn::prefill_attn_kernel, dim3(a.n_qtiles, 8, nseq), dim3(pattn::kThreads), pattn::kSmemBytes,
                stream, 1, mq, mk, mv, a);
}

int vk_linear_qkv_rope_cache(const void* x, const float* ssq, float norm_eps, const void* w_qkv,
                             const void* q_norm_w, const void* k_norm_w, const float* cos, const float* sin,
                             int rope_len, const int32_t* pos, const int32_t* rope_pos, const int32_t* seq, void* q,
                             void* k_cache, void* v_cache, void* k_out, void* v_out, int64_t M, int64_t stride_cb,
                             int64_t stride_cs, int cache_rows, int cache_len, float eps, int n_heads,
                             int n_kv_heads, void* stream) {
  if (M == 0) return VK_OK;
  if (n_heads != 8 || n_kv_heads != 2) return VK_ERR_UNSUPPORTED;
  if (M < 0 || !x || !w_qkv || !q_norm_w || !k_norm_w || !cos || !sin || !pos || !seq || !q || !k_cache ||
      !v_cache)
    return VK_ERR_ARG;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || stride_cs % 8 || stride_cb % 8 ||
      !aligned16(cos) || !aligned16(sin) || (k_out && !aligned16(k_out)) || (v_out && !aligned16(v_out)) ||
      (ssq && !aligned16(ssq)) || !aligned16(q_norm_w) || !aligned16(k_norm_w))
    return VK_ERR_ARG;
  gemm::EpiArgs ep = epi_zero();
  ep.ssq_in = ssq;
  ep.eps = norm_eps;
  ep.q_out = static_cast<__nv_bfloat16*>(q);
  ep.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  ep.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  ep.k_out = static_cast<__nv_bfloat16*>(k_out);
  ep.v_out = static_cast<__nv_bfloat16*>(v_out);
  ep.pos = pos;
  ep.rope_pos = rope_pos;
  ep.seq = seq;
  ep.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  ep.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  ep.cos = cos;
  ep.sin = sin;
  ep.rope_len = rope_len;
  ep.cache_rows = cache_rows;
  ep.cache_len = cache_len;
  ep.stride_cb = stride_cb;
  ep.stride_cs = stride_cs;
  ep.n_heads = n_heads;
  ep.n_kv_heads = n_kv_heads;
  ep.qk_eps = eps;
  const int N = (n_heads + 2 * n_kv_heads) * 64;
  if (M <= kSmallM)
    return run_gemm<64, gemm::QKV_ROPE>(x, w_qkv, M, N, 512, ep, N / 64, N, pick_nk(M, N / 64, 512), stream);
  if (persistent_fits<gemm::QKV_ROPE>(M, N))
    return run_gemm_persistent<gemm::QKV_ROPE>(x, w_qkv, M, N, 512, ep, N, stream);
  return run_gemm<128, gemm::QKV_ROPE>(x, w_qkv, M, N, 512, ep, N / 128, N, 1, stream);
}

int vk_linear_residual(const void* a, const void* w, void* x, float* ssq_out, int64_t M, int K, void* stream) {
  if (M == 0) return VK_OK;
  if (M < 0 || !a || !w || !x || !ssq_out) return VK_ERR_ARG;
  if (!aligned16(x) || !aligned16(ssq_out)) return VK_ERR_ARG;
  gemm::EpiArgs ep = epi_zero();
  ep.x = static_cast<__nv_bfloat16*>(x);
  ep.ssq_out = ssq_out;
  if (M <= kSmallM) return run_gemm<64, gemm::ADD_RESID>(a, w, M, 512, K, ep, 8, 512, pick_nk(M, 8, K), stream);
  if (persistent_fits<gemm::ADD_RESID>(M, 512))
    return run_gemm_persistent<gemm::ADD_RESID>(a, w, M, 512, K, ep, 512, stream);
  return run_gemm<128, gemm::ADD_RESID>(a, w, M, 512, K, ep, 4, 512, 1, stream);
}

int vk_row_ssq(const void* x, float* ssq, int64_t n, int d, void* stream) {
  if (n == 0) return VK_OK;
  if (!x || !ssq || n < 0 || d != 512 || !aligned16(x)) return VK_ERR_ARG;
  return launch(ew::row_ssq_kernel, dim3(blocks_for(n, 8)), dim3(256), 0, stream, 1,
                static_cast<const __nv_bfloat16*>(x), ssq, n);
}

int vk_ssq_rmsnorm(const void* x, const float* ssq, const void* w, void* h, int64_t n, int d, float eps,
                   void* stream) {
  if (n == 0) return VK_OK;
  if (!x || !ssq || !w || !h || n < 0 || d != 512 || !aligned16(x) || !aligned16(h)) return VK_ERR_ARG;
  return launch(ew::ssq_rmsnorm_kernel, dim3(blocks_for(n * 64, 256)), dim3(256), 0, stream, 1,
                static_cast<const __nv_bfloat16*>(x), ssq, static_cast<const __nv_bfloat16*>(w),
                static_cast<__nv_bfloat16*>(h), n, eps);
}

int vk_linear_add_rmsnorm(const void* a, const void* w, void* x, const void* norm_w, void* h, float* ssq_scratch,
                          int64_t M, int K, float eps, void* stream) {
  int rc = vk_linear_residual(a, w, x, ssq_scratch, M, K, stream);
  if (rc != VK_OK) return rc;
  return vk_ssq_rmsnorm(x, ssq_scratch, norm_w, h, M, 512, eps, stream);
}

int vk_fold_norm_weight(const void* w, const void* norm_w, void* out, int64_t N, int K, void* stream) {
  if (N == 0) return VK_OK;
  if (!w || !norm_w || !out || N < 0 || K <= 0) return VK_ERR_ARG;
  return launch(ew::fold_norm_kernel, dim3(blocks_for(N * K, 256)), dim3(256), 0, stream, 1,
                static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(norm_w),
                static_cast<__nv_bfloat16*>(out), N, K);
}

int vk_linear_bias_act(const void* x, const void* w, const void* bias, void* y, int64_t ldy, const int32_t* row_map,
                       int64_t M, int N, int K, int act, void* stream) {
  if (M == 0) return VK_OK;
  if (M < 0 || !x || !w || !bias || !y || N <= 0 || N % 64 || ldy < N || (act != 0 && act != 1)) return VK_ERR_ARG;
  gemm::EpiArgs ep = epi_zero();
  ep.y = y;
  ep.ldy = ldy;
  ep.n_valid = N;
  ep.row_map = row_map;
  ep.bias = static_cast<const __nv_bfloat16*>(bias);
  ep.act = act;
  if (M <= kSmallM) return run_gemm<64, gemm::BIAS_ACT>(x, w, M, N, K, ep, N / 64, N, 1, stream);
  if (persistent_fits<gemm::BIAS_ACT>(M, N))
    return run_gemm_persistent<gemm::BIAS_ACT>(x, w, M, N, K, ep, N, stream);
  return run_gemm<128, gemm::BIAS_ACT>(x, w, M, N, K, ep, (N + 127) / 128, N, 1, stream);
}

int vk_cast_f32_bf16(const float* src, void* dst, int64_t n, void* stream) {
  if (n == 0) return VK_OK;
  if (!src || !dst || n < 0 || !aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7)) return VK_ERR_ARG;
  return launch(ew::cast_f32_bf16_kernel, dim3(blocks_for((n + 3) / 4, 256)), dim3(256), 0, stream, 1, src,
                static_cast<__nv_bfloat16*>(dst), n);
}

int vk_gather_rows(const void* src, const int64_t* idx, void* dst, int64_t n, int row_bytes, int64_t src_rows,
                   void* stream) {
  if (n == 0) return VK_OK;
  if (!src || !idx || !dst || n < 0 || row_bytes <= 0 || row_bytes % 16 || !aligned16(src) || !aligned16(dst))
    return VK_ERR_ARG;
  return launch(ew::gather_rows_kernel, dim3(static_cast<unsigned>(n)), dim3(128), 0, stream, 1,
                static_cast<const uint8_t*>(src), idx, static_cast<uint8_t*>(dst), n, row_bytes, src_rows);
}

int vk_copy_rows(const void* src, const int64_t* src_idx, int64_t src_rows, void* dst, const int64_t* dst_idx,
                 int64_t dst_rows, int64_t n, int row_bytes, void* stream) {
  if (n == 0) return VK_OK;
  if (!src || !dst || n < 0 || row_bytes <= 0 || row_bytes % 16 || !aligned16(src) || !aligned16(dst))
    return VK_ERR_ARG;
  return launch(ew::copy_rows_kernel, dim3(static_cast<unsigned>(n)), dim3(128), 0, stream, 1,
                static_cast<const uint8_t*>(src), src_idx, src_rows, static_cast<uint8_t*>(dst), dst_idx, dst_rows, n,
                row_bytes);
}

int vk_scatter_embed(void* x, const int64_t* rows, int64_t n, int64_t x_rows, const void* emb, int64_t token, int d,
                     void* stream) {
  if (n == 0) return VK_OK;
  if (!x || !rows || !emb || n < 0 || d <= 0 || d % 8 || !aligned16(x) || !aligned16(emb) || token < 0)
    return VK_ERR_ARG;
  return launch(ew::scatter_embed_kernel, dim3(static_cast<unsigned>(n)), dim3(64), 0, stream, 1,
                static_cast<__nv_bfloat16*>(x), rows, n, x_rows, static_cast<const __nv_bfloat16*>(emb), token, d);
}

// ---- host-side stitching (no device work) ------------------------------------------------------------------
int vk_align(const char* query, int qlen, const char* target, int tlen, int mode, int k, int* out, char* cigar,
             int cigar_cap) {
  if (qlen < 0 || tlen < 0 || (qlen && !query) || (tlen && !target) || !out || mode < 0 || mode > 2)
    return VK_ERR_ARG;
  if (cigar && cigar_cap < qlen + tlen + 1) return VK_ERR_ARG;
  const vk::stitch::Alignment r = vk::stitch::align(query, qlen, target, tlen, mode, k, cigar != nullptr);
  out[0] = r.dist;
  out[1] = r.start;
  out[2] = r.end;
  if (cigar) {
    const size_t n = r.dist < 0 ? 0 : r.ops.size();
    memcpy(cigar, r.ops.data(), n);
    cigar[n] = 0;
  }
  return VK_OK;
}

int vk_overlap_cut(const char* a, int la, const char* b, int lb, int ov_frames, double rate, int* cut) {
  if (la < 0 || lb < 0 || (la && !a) || (lb && !b) || !cut) return VK_ERR_ARG;
  const vk::stitch::Cut c = vk::stitch::overlap_cut(std::string(a, a + la), std::string(b, b + lb), ov_frames, rate);
  cut[0] = c.a;
  cut[1] = c.b;
  return VK_OK;
}

int vk_stitch(const char* calls, const int64_t* offsets, const int64_t* spans, int n, int stride, char* out,
              int64_t cap, int64_t* out_len) {
  if (n < 0 || stride <= 0 || !out_len || (n && (!calls || !offsets || !spans))) return VK_ERR_ARG;
  std::vector<std::string> cs(n);
  for (int i = 0; i < n; ++i) {
    if (offsets[i + 1] < offsets[i]) return VK_ERR_ARG;
    cs[i].assign(calls + offsets[i], calls + offsets[i + 1]);
  }
  std::string res;
  int64_t cut_prev = 0;
  for (int i = 0; i < n; ++i) {
    const std::string& s = cs[i];
    if (i + 1 < n) {
      const int64_t ov = vk::stitch::floor_div(spans[2 * i + 1] - spans[2 * (i + 1)], stride);
      const int64_t frames = std::max<int64_t>(vk::stitch::floor_div(spans[2 * i + 1] - spans[2 * i], stride), 1);
      const double rate = static_cast<double>(s.size()) / static_cast<double>(frames);
      const vk::stitch::Cut c = vk::stitch::overlap_cut(s, cs[i + 1], static_cast<int>(ov), rate);
      res += vk::stitch::py_slice(s, cut_prev, c.a);
      cut_prev = c.b;
    } else {
      res += vk::stitch::py_slice(s, cut_prev, static_cast<int64_t>(s.size()));
    }
  }
  *out_len = static_cast<int64_t>(res.size());
  if (!out || cap < static_cast<int64_t>(res.size())) return out ? VK_ERR_ARG : VK_OK;
  memcpy(out, res.data(), res.size());
  return VK_OK;
}

}  // extern "C"
