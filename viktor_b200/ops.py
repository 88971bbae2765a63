"""PyTorch-facing wrappers of the C ABI, one per op.

The first group keeps the names, arguments and return values of the reference's Triton ops
(viktor/triton_ops.py) and of viktor/decode_attention.py, so code written against those modules ports by
changing the import.  The second group exposes the fused tensor-core forms this package runs on the hot path.
Every wrapper launches on the current CUDA stream of the tensors' device and raises on failure; nothing falls
back to PyTorch.
"""

from __future__ import annotations

import torch

from ._lib import call, load

_BF16 = torch.bfloat16


def _p(t):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("viktor_b200 ops need CUDA tensors (there is no CPU path)")


# ---------------------------------------------------------------- mirrors of viktor/triton_ops.py
def add_rmsnorm(x, w, eps, delta=None):
    """x [n, d] (updated in place by += delta); returns RMSNorm(x) * w.  (viktor/triton_ops.py:34-40)"""
    _check_cuda(x, w, delta)
    n, d = x.shape
    assert x.dtype == _BF16 and x.is_contiguous() and (delta is None or delta.is_contiguous())
    h = torch.empty_like(x)
    call("vk_add_rmsnorm", _p(x), _p(delta), _p(w), _p(h), n, d, eps, _stream(x))
    return h


def embed_rmsnorm(tok, emb, w, eps):
    """tok [n] token ids -> (x = emb[tok] [n, d], RMSNorm(x) * w).  (viktor/triton_ops.py:163-169)"""
    _check_cuda(tok, emb, w)
    n, d = tok.shape[0], emb.shape[1]
    tok = tok.to(torch.int64).contiguous()
    x = torch.empty(n, d, dtype=emb.dtype, device=emb.device)
    h = torch.empty_like(x)
    call("vk_embed_rmsnorm", _p(tok), _p(emb), emb.shape[0], _p(w), _p(x), _p(h), n, d, eps, _stream(emb))
    return x, h


def qkv_rope_cache(qkv, q_norm_w, k_norm_w, cos, sin, pos, seq, k_cache, v_cache, eps, n_heads, n_kv_heads,
                   head_dim, return_kv=False, rope_pos=None):
    """qkv [n, (H + 2 Hkv) * D]; pos/seq [n] int32; k_cache/v_cache [B, S, Hkv, D] (one layer).
    Returns q [n, H, D] (and packed k, v [n, Hkv, D]).  (viktor/triton_ops.py:94-108)"""
    _check_cuda(qkv, k_cache, v_cache, pos, seq)
    n = qkv.shape[0]
    assert k_cache.stride() == v_cache.stride() and k_cache.stride(-1) == 1 and k_cache.stride(-2) == head_dim
    q = torch.empty(n, n_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
    k = v = None
    if return_kv:
        k = torch.empty(n, n_kv_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        v = torch.empty_like(k)
    call("vk_qkv_rope_cache", _p(qkv.contiguous()), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin), cos.shape[0],
         _p(pos), _p(rope_pos), _p(seq), _p(q), _p(k_cache), _p(v_cache), _p(k), _p(v), n, k_cache.stride(0),
         k_cache.stride(1), k_cache.shape[0], k_cache.shape[1], eps, n_heads, n_kv_heads, head_dim, _stream(qkv))
    return (q, k, v) if return_kv else q


def linear(x, w, swiglu=False, out_dtype=None):
    """x @ w^T on tcgen05 tensor cores.  swiglu: w is gate_up [2F, K] and the result silu(gate) * up [M, F].
    out_dtype: torch.float32 for unrounded logits.  (viktor/triton_ops.py:138-146)"""
    _check_cuda(x, w)
    M, K = x.shape
    N = w.shape[0]
    out_f32 = out_dtype == torch.float32
    y = torch.empty(M, N // 2 if swiglu else N, dtype=torch.float32 if out_f32 else x.dtype, device=x.device)
    call("vk_linear", _p(x.contiguous()), _p(w.contiguous()), _p(y), M, N, K, int(bool(swiglu)), int(out_f32),
         _stream(x))
    return y


def swiglu(gu):
    """gu [n, 2F] (gate | up) -> silu(gate) * up [n, F].  (viktor/triton_ops.py:223-229)"""
    _check_cuda(gu)
    n, f2 = gu.shape
    out = torch.empty(n, f2 // 2, dtype=gu.dtype, device=gu.device)
    call("vk_swiglu", _p(gu.contiguous()), _p(out), n, f2 // 2, _stream(gu))
    return out


def greedy_update(logits, bias, is_tail, is_homo, homo_stop, tok, run, pos, plen, rope_off, out, pos32, seqlens,
                  rpos32, eos, pad, emb=None, x=None, ssq=None):
    """Greedy step bookkeeping in one kernel (viktor/triton_ops.py:200-209).  is_tail / is_homo: bool or uint8
    [V].  With emb/x/ssq also writes the next step's embedding x [B, 512] and its block sums of squares ssq [B, 8]."""
    _check_cuda(logits, tok, out)
    B, V = logits.shape
    it = is_tail.to(torch.uint8) if is_tail.dtype != torch.uint8 else is_tail
    ih = is_homo.to(torch.uint8) if is_homo.dtype != torch.uint8 else is_homo
    call("vk_greedy_update", _p(logits), logits.stride(0), _p(bias), _p(it), _p(ih), int(homo_stop), _p(tok),
         _p(run), _p(pos), _p(plen), _p(rope_off), _p(out), out.stride(0), out.shape[1], _p(pos32), _p(seqlens),
         _p(rpos32), B, V, eos, pad, _p(emb), _p(x), _p(ssq), _stream(logits))


# ---------------------------------------------------------------- mirror of viktor/decode_attention.py
_WS = {}


def decode_attention_workspace(nq: int, S: int, device) -> torch.Tensor:
    """A zero-filled workspace for decode_attention (per-query tickets return to zero after every call)."""
    nbytes = load().vk_decode_attention_workspace_bytes(nq, S)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def decode_attention(q, k, v, lengths, block=64, workspace=None, row0=0):
    """q [B, H, D]; k/v [B', S, Hkv, D] (one layer of the cache, B' >= row0 + B); lengths [B] int32 including
    the current token, 1 <= lengths <= S.  Query b attends cache row row0 + b.  (viktor/decode_attention.py:41-53)"""
    B, H, D = q.shape
    HK = k.shape[2]
    assert q.is_contiguous() and H % HK == 0 and H // HK <= 16 and D == 64
    assert q.dtype == k.dtype == v.dtype == torch.bfloat16
    assert k.stride() == v.stride() and k.stride(-1) == 1 and k.stride(-2) == D
    assert lengths.shape == (B,) and lengths.dtype == torch.int32 and lengths.is_contiguous()
    if (H, HK) != (8, 2):
        raise NotImplementedError("decode attention kernels are built for 8 query / 2 KV heads")
    S = k.shape[1]
    if workspace is None:
        # one implicit workspace per (device, shape, stream): calls on the same stream run one after another;
        # calls on different streams get different workspaces, so they never share split-K tickets or partials
        key = (q.device, B, S, _stream(q))
        workspace = _WS.get(key)
        if workspace is None:
            workspace = _WS[key] = decode_attention_workspace(B, S, q.device)
    out = torch.empty_like(q)
    call("vk_decode_attention", _p(q), _p(k), _p(v), _p(lengths), _p(out), B, row0, k.shape[0], S, k.stride(0),
         k.stride(1), _p(workspace), workspace.numel(), _stream(q))
    return out


# ---------------------------------------------------------------- opt-in INT8 prefix KV (analysis.md:95)
class PrefixKV8:
    """Int8 copy of the prefix of one layer's cache rows: k8 [rows, S8, 128] / v8t [rows, S8 / 128, 128, 128]
    uint8 (excess-128 bytes; v8t channel-major within each tile of 128 positions), sk / sv [rows, 128] float32
    per-channel scales.  S8 is rounded up to a multiple of 128."""

    def __init__(self, rows: int, S8: int, device):
        self.S8 = -(-S8 // 128) * 128
        self.k8 = torch.zeros(rows, self.S8, 128, dtype=torch.uint8, device=device)
        self.v8t = torch.zeros(rows, self.S8 // 128, 128, 128, dtype=torch.uint8, device=device)
        self.sk = torch.zeros(rows, 128, dtype=torch.float32, device=device)
        self.sv = torch.zeros(rows, 128, dtype=torch.float32, device=device)


def kv_quantize(k, v, starts, prefix: PrefixKV8, row0=0):
    """Quantizes positions [0, starts[i]) of cache rows row0 + i of one layer (k/v [B', S, 2, 64] bf16) into
    prefix: per channel s = max|x| / 127, byte = clamp(rint(x / s), -127, 127) + 128."""
    assert k.dtype == v.dtype == torch.bfloat16 and k.stride() == v.stride() and k.stride(-1) == 1
    assert k.shape[2:] == (2, 64) and k.stride(-2) == 64
    assert starts.dtype == torch.int32 and starts.is_contiguous()
    call("vk_kv_quantize", _p(k), _p(v), k.shape[0], k.shape[1], k.stride(0), k.stride(1), _p(starts), row0,
         starts.shape[0], _p(prefix.k8), _p(prefix.v8t), _p(prefix.sk), _p(prefix.sv), prefix.S8, _stream(k))


def decode_attention_i8(q, k, v, prefix: PrefixKV8, starts, lengths, max_tail, workspace=None, row0=0):
    """decode_attention with positions [0, starts[b]) read from the int8 prefix and [starts[b], lengths[b]) from
    the bf16 cache (0 <= starts < lengths, lengths - starts <= max_tail)."""
    B, H, D = q.shape
    assert (H, D) == (8, 64) and q.is_contiguous() and q.dtype == k.dtype == v.dtype == torch.bfloat16
    assert k.stride() == v.stride() and k.stride(-1) == 1 and k.shape[2:] == (2, 64) and k.stride(-2) == 64
    assert starts.dtype == lengths.dtype == torch.int32 and starts.shape == lengths.shape == (B,)
    S = k.shape[1]
    if workspace is None:
        key = ("i8", q.device, B, prefix.S8, max_tail)
        workspace = _WS.get(key)
        if workspace is None:
            nbytes = load().vk_decode_attention_i8_workspace_bytes(B, prefix.S8, max_tail)
            workspace = _WS[key] = torch.zeros(nbytes, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    call("vk_decode_attention_i8", _p(q), _p(k), _p(v), _p(prefix.k8), _p(prefix.v8t), _p(prefix.sk),
         _p(prefix.sv), _p(starts), _p(lengths), _p(out), B, row0, k.shape[0], S, k.stride(0), k.stride(1),
         prefix.S8, max_tail, _p(workspace), workspace.numel(), _stream(q))
    return out


def prefill_attention(q, k_cache, v_cache, cu_seqlens, max_seqlen, row0=0, out=None):
    """Varlen causal attention (flash_attn_varlen_func(..., causal=True), viktor/fast_decoder.py:73) over K/V
    already in the cache.  q [n_tok, 8, 64] packed by cu_seqlens [nseq + 1] int32; k_cache/v_cache one layer
    [B', S, 2, 64]; sequence b reads cache row row0 + b."""
    n_tok = q.shape[0]
    nseq = cu_seqlens.shape[0] - 1
    if out is None:
        out = torch.empty_like(q)
    call("vk_prefill_attention", _p(q), _p(k_cache), _p(v_cache), _p(cu_seqlens), nseq, int(max_seqlen), n_tok,
         row0, k_cache.shape[0], k_cache.shape[1], k_cache.stride(0), k_cache.stride(1), _p(out), _stream(q))
    return out


# ---------------------------------------------------------------- fused tensor-core forms (hot path)
def fold_norm_weight(w, norm_w):
    """W' = bf16(W * norm_w[None, :]): an RMSNorm weight folded into the GEMM that consumes the norm."""
    out = torch.empty_like(w)
    call("vk_fold_norm_weight", _p(w.contiguous()), _p(norm_w.contiguous()), _p(out), w.shape[0], w.shape[1],
         _stream(w))
    return out


def row_ssq(x, out=None):
    """[n, 8] fp32 sums of squares of the eight 64-column blocks of each row of x [n, 512]."""
    out = out if out is not None else torch.empty(x.shape[0], 8, dtype=torch.float32, device=x.device)
    call("vk_row_ssq", _p(x), _p(out), x.shape[0], x.shape[1], _stream(x))
    return out


def linear_rmsnorm(x, ssq, eps, w_folded, swiglu=False, out_dtype=None):
    """(RMSNorm(x) * w) . W^T given W' = W diag(w) and the row sums of squares of x."""
    M, K = x.shape
    N = w_folded.shape[0]
    out_f32 = out_dtype == torch.float32
    y = torch.empty(M, N // 2 if swiglu else N, dtype=torch.float32 if out_f32 else x.dtype, device=x.device)
    call("vk_linear_rmsnorm", _p(x), _p(ssq), eps, _p(w_folded), _p(y), M, N, K, int(bool(swiglu)), int(out_f32),
         _stream(x))
    return y


def linear_qkv_rope_cache(x, w_qkv, q_norm_w, k_norm_w, cos, sin, pos, seq, k_cache, v_cache, eps, rope_pos=None,
                          q_out=None, return_kv=False, ssq=None, norm_eps=1e-6, n_heads=8, n_kv_heads=2):
    """x [M, 512] . w_qkv^T with the qkv_rope_cache epilogue: returns q [M, H, 64] (and packed k, v).  With ssq,
    x is the residual and w_qkv carries the folded attention-norm weight."""
    M = x.shape[0]
    q = q_out if q_out is not None else torch.empty(M, n_heads, 64, dtype=x.dtype, device=x.device)
    k = v = None
    if return_kv:
        k = torch.empty(M, n_kv_heads, 64, dtype=x.dtype, device=x.device)
        v = torch.empty_like(k)
    call("vk_linear_qkv_rope_cache", _p(x), _p(ssq), norm_eps, _p(w_qkv), _p(q_norm_w), _p(k_norm_w), _p(cos),
         _p(sin), cos.shape[0], _p(pos), _p(rope_pos), _p(seq), _p(q), _p(k_cache), _p(v_cache), _p(k), _p(v), M,
         k_cache.stride(0), k_cache.stride(1), k_cache.shape[0], k_cache.shape[1], eps, n_heads, n_kv_heads,
         _stream(x))
    return (q, k, v) if return_kv else q


def linear_residual(a, w, x, ssq_out=None):
    """x += a . w^T (bf16, in place); returns the new rows' block sums of squares [M, 8]."""
    M, K = a.shape
    ssq = ssq_out if ssq_out is not None else torch.empty(M, 8, dtype=torch.float32, device=a.device)
    call("vk_linear_residual", _p(a), _p(w), _p(x), _p(ssq), M, K, _stream(a))
    return ssq


def linear_add_rmsnorm(a, w, x, norm_w, eps, h_out=None):
    """x += a . w^T (bf16, in place); returns h = RMSNorm(x) * norm_w.  x, h [M, 512]."""
    M, K = a.shape
    h = h_out if h_out is not None else torch.empty_like(x)
    ssq = torch.empty(M, 8, dtype=torch.float32, device=a.device)
    call("vk_linear_add_rmsnorm", _p(a), _p(w), _p(x), _p(norm_w), _p(h), _p(ssq), M, K, eps, _stream(a))
    return h


def linear_bias_act(x, w, bias, act=0, out=None, row_map=None):
    """act(x . w^T + bias) in bf16 (act 0 identity, 1 GELU-erf); row i of the result lands in out[row_map[i]]."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    call("vk_linear_bias_act", _p(x), _p(w), _p(bias), _p(out), out.stride(0), _p(row_map), M, N, K, act,
         _stream(x))
    return out


def cast_bf16(src, out=None):
    out = out if out is not None else torch.empty(src.shape, dtype=torch.bfloat16, device=src.device)
    call("vk_cast_f32_bf16", _p(src.contiguous()), _p(out), src.numel(), _stream(src))
    return out


def gather_rows(src, idx, out=None):
    n = idx.shape[0]
    row_bytes = src[0].numel() * src.element_size()
    out = out if out is not None else torch.empty((n,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    call("vk_gather_rows", _p(src), _p(idx), _p(out), n, row_bytes, src.shape[0], _stream(src))
    return out


def scatter_embed(x, rows, emb, token):
    call("vk_scatter_embed", _p(x), _p(rows), rows.shape[0], x.shape[0], _p(emb), int(token), x.shape[1],
         _stream(x))
