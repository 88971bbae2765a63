"""Seeded synthetic weights and encoder frames (numpy only, no device work).

Weights are a flat dict keyed exactly like the reference ``Basecaller`` state dict
(``projector.{0,2}.{weight,bias}``, ``decoder.*`` as laid out by viktor/decoder.py:54-134),
so the same dict loads into the reference model, into this package's model container and
into the CPU oracle used by the tests.

Two initialisations:

* ``"normal"``: every matrix N(0, std) (std 0.02 by default), norm weights 1, biases 0.
  This is the benchmark initialisation; greedy decoding from it is degenerate
  (near-uniform logits), so it is only used for timing.
* ``"torch"``: the PyTorch module defaults (Linear weight and bias U(+-1/sqrt(fan_in)),
  Embedding N(0, 1)) with norm weights drawn from U(0.8, 1.2) so that the weight multiply in
  every RMSNorm is exercised.  Logit margins are large enough for token-level parity.
"""

from __future__ import annotations

import numpy as np

from .config import DecoderConfig


def state_dict_shapes(cfg: DecoderConfig, d_enc: int = 512) -> dict[str, tuple[int, ...]]:
    """Parameter names and shapes of the reference Basecaller (projector + decoder)."""
    d, H, Hkv, D, F, V = cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab_size
    shapes = {
        "projector.0.weight": (d, d_enc), "projector.0.bias": (d,),
        "projector.2.weight": (d, d), "projector.2.bias": (d,),
        "decoder.embed.weight": (V, d),
    }
    for i in range(cfg.n_layers):
        p = f"decoder.layers.{i}."
        shapes.update({
            p + "attn_norm.weight": (d,),
            p + "attn.qkv_proj.weight": ((H + 2 * Hkv) * D, d),
            p + "attn.o_proj.weight": (d, H * D),
            p + "attn.q_norm.weight": (D,),
            p + "attn.k_norm.weight": (D,),
            p + "mlp_norm.weight": (d,),
            p + "gate_up.weight": (2 * F, d),
            p + "down.weight": (d, F),
        })
    shapes["decoder.norm.weight"] = (d,)
    shapes["decoder.lm_head.weight"] = (V, d)
    return shapes


def make_weights(cfg: DecoderConfig, seed: int = 0, init: str = "torch", std: float = 0.02,
                 d_enc: int = 512) -> dict[str, np.ndarray]:
    """Deterministic fp32 weights for every parameter of the projector + decoder."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in state_dict_shapes(cfg, d_enc).items():
        is_norm = name.endswith("norm.weight")
        if init == "normal":
            if is_norm:
                w = np.ones(shape, np.float32)
            elif name.endswith("bias"):
                w = np.zeros(shape, np.float32)
            else:
                w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        elif init == "torch":
            if is_norm:
                w = rng.uniform(0.8, 1.2, shape).astype(np.float32)
            elif name == "decoder.embed.weight":
                w = rng.standard_normal(shape, dtype=np.float32)
            else:
                fan_in = shape[1] if len(shape) == 2 else state_dict_shapes(cfg, d_enc)[
                    name.replace("bias", "weight")][1]
                bound = 1.0 / np.sqrt(fan_in)
                w = rng.uniform(-bound, bound, shape).astype(np.float32)
        else:
            raise ValueError(f"unknown init {init!r}")
        out[name] = w
    return out


def make_frames(lens, d_enc: int = 512, seed: int = 1) -> np.ndarray:
    """Encoder frames of len(lens) chunks, concatenated: [sum(lens), d_enc] fp32 ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((int(sum(lens)), d_enc), dtype=np.float32)


def varlen_prefix_lengths(n: int, seed: int = 2, lo: int = 128, hi: int = 2048, step: int = 128) -> list[int]:
    """Prefix lengths drawn uniformly from the multiples of ``step`` in [lo, hi] (varlen config)."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo // step, hi // step + 1, size=n) * step]
