"""Decoder weights container, static KV cache and RoPE tables.

``Decoder`` has the parameter names and shapes of viktor/decoder.py:54-134 (embed, layers[i].{attn_norm,
attn.{qkv_proj,o_proj,q_norm,k_norm}, mlp_norm, gate_up, down}, norm, lm_head), so a reference checkpoint's
``decoder.*`` state dict loads unchanged.  It carries no forward pass of its own: inference runs through
``FastDecoder`` / ``DecodeEngine`` on the CUDA kernels.

``KVCache`` keeps the reference layout [layer, batch, position, kv_head, head_dim] (viktor/decoder.py:43-51).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .config import DecoderConfig


def rope_tables(dim: int, max_len: int, theta: float):
    """cos/sin [max_len, dim/2] built in fp64 and cast to fp32 (viktor/encoder.py:30-33)."""
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    freqs = torch.arange(max_len, dtype=torch.float64)[:, None] * inv
    return freqs.cos().float(), freqs.sin().float()


class KVCache:
    """Static cache [layer, batch, position, kv_head, head_dim] (viktor/decoder.py:43-51).  Zero-filled, so
    positions never written hold finite values (the attention kernels rely on that)."""

    def __init__(self, cfg: DecoderConfig, batch: int, max_len: int, dtype, device):
        shape = (cfg.n_layers, batch, max_len, cfg.n_kv_heads, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.max_len = max_len
        self.positions = torch.arange(max_len, device=device)


class Attention(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        h, hkv, d = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.qkv_proj = nn.Linear(cfg.d_model, (h + 2 * hkv) * d, bias=False)
        self.o_proj = nn.Linear(h * d, cfg.d_model, bias=False)
        self.q_norm = nn.RMSNorm(d, eps=cfg.norm_eps)
        self.k_norm = nn.RMSNorm(d, eps=cfg.norm_eps)


class Block(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.attn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.attn = Attention(cfg)
        self.mlp_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.gate_up = nn.Linear(cfg.d_model, 2 * cfg.ffn_dim, bias=False)
        self.down = nn.Linear(cfg.ffn_dim, cfg.d_model, bias=False)


class Decoder(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layers)])
        self.norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    def head(self, h):
        return self.lm_head(h)
