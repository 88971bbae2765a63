"""Inference forward of the decoder on the B200 kernels (the role of viktor/fast_decoder.py).

Tokens are packed [n_tokens, d]: prefill packs the prefixes of many variable-length chunks (cu_seqlens), a
decode step is one token per sequence.  Per layer (viktor/fast_decoder.py:33-60), with the reference's
separate ops fused into tensor-core GEMM epilogues and every RMSNorm folded into the GEMM that consumes it
(norm weight in the weight columns, 1/rms per row in the epilogue, from the block sums of squares ssq that the
producer of the residual x writes):

    q, K/V -> cache  = qkv GEMM(x, ssq)                (add_rmsnorm + linear + qkv_rope_cache)
    o                = attention(q, cache)             (prefill: varlen causal; decode / BOS-only: split-K)
    x += o W_o, ssq  = residual GEMM(o)                (linear + residual add)
    g                = gate_up GEMM(x, ssq)            (add_rmsnorm + linear + SwiGLU)
    x += g W_d, ssq  = residual GEMM(g)                (linear + residual add)

The prefill runs the last layer for the BOS rows only (viktor/fast_decoder.py:48-53): all K/V are kept, the
final signal outputs have no consumer.
"""

from __future__ import annotations

import torch

from ._lib import call
from .decoder import rope_tables

_BF16 = torch.bfloat16


def _p(t):
    return None if t is None else t.data_ptr()


def expected_shapes(cfg, d_enc: int = 512) -> dict:
    """The checkpoint entries the engine reads, name -> shape: the ``projector.*`` and ``decoder.*`` keys of the
    reference model's state dict (viktor/model.py:35, viktor/decoder.py:54-134)."""
    d, f, hd = cfg.d_model, cfg.ffn_dim, cfg.head_dim
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * hd
    shapes = {"projector.0.weight": (d, d_enc), "projector.0.bias": (d,), "projector.2.weight": (d, d),
              "projector.2.bias": (d,), "decoder.embed.weight": (cfg.vocab_size, d), "decoder.norm.weight": (d,),
              "decoder.lm_head.weight": (cfg.vocab_size, d)}
    for i in range(cfg.n_layers):
        p = f"decoder.layers.{i}."
        shapes.update({p + "attn_norm.weight": (d,), p + "attn.qkv_proj.weight": (qkv, d),
                       p + "attn.q_norm.weight": (hd,), p + "attn.k_norm.weight": (hd,),
                       p + "attn.o_proj.weight": (d, cfg.n_heads * hd), p + "mlp_norm.weight": (d,),
                       p + "gate_up.weight": (2 * f, d), p + "down.weight": (d, f)})
    return shapes


def check_state_dict(shapes: dict, cfg, d_enc: int = 512):
    """Raises ValueError unless ``shapes`` (name -> shape of the model's projector/decoder entries) has exactly
    the entries expected_shapes() lists, with those shapes.  Host only (no tensors are touched)."""
    want = expected_shapes(cfg, d_enc)
    missing = sorted(set(want) - set(shapes))
    extra = sorted(set(shapes) - set(want))
    bad = sorted(n for n in want if n in shapes and tuple(shapes[n]) != want[n])
    if missing or extra or bad:
        raise ValueError(f"checkpoint does not match the decoder: missing {missing[:4]}, unexpected {extra[:4]}, "
                         f"shape mismatch {[(n, tuple(shapes[n]), want[n]) for n in bad[:4]]}")


def model_state(model) -> dict:
    """The projector and decoder entries of a Basecaller-like model (this package's or the reference's
    viktor.model.Basecaller: anything with ``projector`` and ``decoder`` modules), keyed as in its state dict."""
    sd = {f"projector.{n}": t for n, t in model.projector.state_dict().items()}
    sd.update({f"decoder.{n}": t for n, t in model.decoder.state_dict().items()})
    return sd


class DeviceWeights:
    """bf16 device copies of the projector + decoder weights, in the layouts the kernels read, taken from the
    model's state-dict entries by their reference names.  The attention norm of each layer is folded into its
    qkv weight, the MLP norm into gate_up and the final norm into lm_head (columns scaled by the norm weight,
    rounded once to bf16)."""

    def __init__(self, model, device):
        cfg = model.decoder.cfg
        if (cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim) != (512, 8, 2, 64):
            raise NotImplementedError("the kernels are built for d_model 512, 8 query / 2 KV heads, head_dim 64")
        if cfg.ffn_dim % 128:
            raise NotImplementedError("ffn_dim must be a multiple of 128")
        sd = model_state(model)
        d_enc = sd["projector.0.weight"].shape[1] if "projector.0.weight" in sd else -1
        check_state_dict({n: tuple(t.shape) for n, t in sd.items()}, cfg, d_enc)

        def w(name):
            return sd[name].detach().to(device=device, dtype=_BF16).contiguous()

        def fold(weight, norm):
            out = torch.empty_like(weight)
            call("vk_fold_norm_weight", _p(weight), _p(norm), _p(out), weight.shape[0], weight.shape[1],
                 torch.cuda.current_stream(device).cuda_stream)
            return out

        self.cfg = cfg
        self.eps = float(cfg.norm_eps)
        self.embed = w("decoder.embed.weight")
        self.vocab = cfg.vocab_size
        # lm_head rows padded to a multiple of 16 (tensor-core N granularity); padded logits are never read
        vpad = -(-cfg.vocab_size // 16) * 16
        head = torch.zeros(vpad, cfg.d_model, dtype=_BF16, device=device)
        head[:cfg.vocab_size] = w("decoder.lm_head.weight")
        self.norm = w("decoder.norm.weight")
        self.lm_head, self.vpad = fold(head, self.norm), vpad
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"decoder.layers.{i}."
            self.layers.append(dict(qkv=fold(w(p + "attn.qkv_proj.weight"), w(p + "attn_norm.weight")),
                                    q_norm=w(p + "attn.q_norm.weight"), k_norm=w(p + "attn.k_norm.weight"),
                                    o=w(p + "attn.o_proj.weight"),
                                    gate_up=fold(w(p + "gate_up.weight"), w(p + "mlp_norm.weight")),
                                    down=w(p + "down.weight")))
        cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self.cos, self.sin = cos.to(device).contiguous(), sin.to(device).contiguous()
        self.proj = (w("projector.0.weight"), w("projector.0.bias"), w("projector.2.weight"), w("projector.2.bias"))
        self.d_enc = d_enc
        if self.d_enc % 64:
            raise NotImplementedError("encoder width must be a multiple of 64")


class FastDecoder:
    """Layer loop over the fused kernels.  All buffers are passed in; nothing is allocated per call except
    where noted."""

    def __init__(self, weights: DeviceWeights):
        self.w = weights
        self.cfg = weights.cfg

    # -- helpers -----------------------------------------------------------------------------------------------
    def _qkv(self, i, x, ssq, pos, seq, rope_pos, cache, q_out, stream):
        L = self.w.layers[i]
        kc, vc = cache.k[i], cache.v[i]
        call("vk_linear_qkv_rope_cache", _p(x), _p(ssq), self.w.eps, _p(L["qkv"]), _p(L["q_norm"]), _p(L["k_norm"]),
             _p(self.w.cos), _p(self.w.sin), self.w.cos.shape[0], _p(pos), _p(rope_pos), _p(seq), _p(q_out), _p(kc),
             _p(vc), None, None, x.shape[0], kc.stride(0), kc.stride(1), kc.shape[0], kc.shape[1], self.w.eps, 8, 2,
             stream)

    def _decode_attn(self, i, q, lengths, cache, out, workspace, row0, stream):
        kc, vc = cache.k[i], cache.v[i]
        call("vk_decode_attention", _p(q), _p(kc), _p(vc), _p(lengths), _p(out), q.shape[0], row0, kc.shape[0],
             kc.shape[1], kc.stride(0), kc.stride(1), _p(workspace), workspace.numel(), stream)

    def _mlp_tail(self, i, o, x, ssq, g, stream):
        """x += o W_o; g = swiglu(norm(x) W_gu); x += g W_d  (ssq tracks the block sums of squares of x)."""
        L = self.w.layers[i]
        M = x.shape[0]
        call("vk_linear_residual", _p(o), _p(L["o"]), _p(x), _p(ssq), M, 512, stream)
        call("vk_linear_rmsnorm", _p(x), _p(ssq), self.w.eps, _p(L["gate_up"]), _p(g), M, L["gate_up"].shape[0], 512,
             1, 0, stream)
        call("vk_linear_residual", _p(g), _p(L["down"]), _p(x), _p(ssq), M, g.shape[1], stream)

    # -- prefill -----------------------------------------------------------------------------------------------
    def prefill(self, x, ssq, pos, seq, cu_seqlens, max_seqlen, cache, q, o, g, row0=0, rope_pos=None,
                last_indices=None, lengths=None, x_last=None, ssq_last=None, q_last=None, o_last=None, g_last=None,
                workspace=None, stream=None):
        """x [n, d] packed prefix embeddings (residual stream, updated in place), ssq [n, 8] its block sums of
        squares; pos/seq [n] int32; cu_seqlens [b+1] int32.  Fills the cache rows row0.. of those sequences.
        Afterwards x holds the final residual of every row, or with last_indices [b] int64 (+ lengths [b] int32
        = T_b and the *_last buffers) x_last holds that of each sequence's last row; the matching ssq / ssq_last
        give the final norm."""
        stream = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
        n_layers = self.cfg.n_layers
        n = x.shape[0]
        for i in range(n_layers):
            self._qkv(i, x, ssq, pos, seq, rope_pos, cache, q, stream)
            kc, vc = cache.k[i], cache.v[i]
            if last_indices is not None and i == n_layers - 1:
                b = last_indices.shape[0]
                call("vk_gather_rows", _p(x), _p(last_indices), _p(x_last), b, 1024, n, stream)
                call("vk_gather_rows", _p(ssq), _p(last_indices), _p(ssq_last), b, 32, n, stream)
                call("vk_gather_rows", _p(q), _p(last_indices), _p(q_last), b, 1024, n, stream)
                self._decode_attn(i, q_last, lengths, cache, o_last, workspace, row0, stream)
                self._mlp_tail(i, o_last, x_last, ssq_last, g_last, stream)
                return
            call("vk_prefill_attention", _p(q), _p(kc), _p(vc), _p(cu_seqlens), cu_seqlens.shape[0] - 1,
                 int(max_seqlen), n, row0, kc.shape[0], kc.shape[1], kc.stride(0), kc.stride(1), _p(o), stream)
            self._mlp_tail(i, o, x, ssq, g, stream)

    # -- one decode step -----------------------------------------------------------------------------------------
    def _decode_attn_i8(self, i, q, lengths, cache, prefix, out, workspace, row0, stream):
        kc, vc = cache.k[i], cache.v[i]
        pre = prefix["layers"][i]
        call("vk_decode_attention_i8", _p(q), _p(kc), _p(vc), _p(pre.k8), _p(pre.v8t), _p(pre.sk), _p(pre.sv),
             _p(prefix["starts"]), _p(lengths), _p(out), q.shape[0], row0, kc.shape[0], kc.shape[1], kc.stride(0),
             kc.stride(1), pre.S8, prefix["max_tail"], _p(workspace), workspace.numel(), stream)

    def decode(self, x, ssq, pos32, rows, seqlens, cache, q, o, g, workspace, rope_pos=None, stream=None, row0=0,
               prefix=None):
        """One token per sequence: x [B, d] residual and ssq [B, 8] (from the previous step's greedy kernel);
        pos32/rows [B] int32 (rows = cache row of each sequence, row0 + arange(B)); seqlens = pos + 1.  Leaves
        the final residual in x (and its ssq).  prefix (int8 prefix KV): dict(layers=[PrefixKV8 per layer],
        starts=[B] int32, max_tail=int); workspace is then vk_decode_attention_i8's."""
        stream = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
        for i in range(self.cfg.n_layers):
            self._qkv(i, x, ssq, pos32, rows, rope_pos, cache, q, stream)
            if prefix is None:
                self._decode_attn(i, q, seqlens, cache, o, workspace, row0, stream)
            else:
                self._decode_attn_i8(i, q, seqlens, cache, prefix, o, workspace, row0, stream)
            self._mlp_tail(i, o, x, ssq, g, stream)

    def logits(self, x, ssq, out, stream):
        """fp32 logits of the final-normed rows of x (final norm folded into lm_head)."""
        w = self.w
        call("vk_linear_rmsnorm", _p(x), _p(ssq), w.eps, _p(w.lm_head), _p(out), x.shape[0], w.vpad, 512, 0, 1,
             stream)
