"""Timed CPU baseline: the reference decoder path restated with multithreaded PyTorch CPU ops (fp32).

TEST INFRASTRUCTURE ONLY (the CPU-baseline leg of ``bench.py`` and its pinning test).  Same algorithm as
``decoder_np`` (and as the reference it cites), written with the operators the reference's own CPU path uses
(F.rms_norm, SDPA with a causal mask for prefill, SDPA over the cached prefix for decode), so the CPU number it
produces is representative of running the reference on the host cores:

* projector + packed prefix ........... viktor/model.py:35, viktor/engine.py:183-188
* layer (norm, qkv, QK-norm, RoPE) .... viktor/decoder.py:63-67, :117-120, viktor/encoder.py:30-40
* causal prefill / cached decode ...... viktor/decoder.py:81-105
* greedy selection + grammar .......... viktor/engine.py:79-89
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

PAD, BOS, EOS = 0, 1, 2


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1)


class TorchCPUModel:
    def __init__(self, cfg, weights: dict, k: int = 1):
        self.cfg = cfg
        self.w = {n: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)) for n, a in weights.items()}
        self.k = k
        inv = 1.0 / cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, dtype=torch.float64) / cfg.head_dim)
        fr = torch.arange(cfg.max_seq_len, dtype=torch.float64)[:, None] * inv
        self.cos, self.sin = fr.cos().float(), fr.sin().float()
        from .decoder_np import OracleTokenizer
        self.tok = OracleTokenizer(k)

    def _l(self, i, n):
        return self.w[f"decoder.layers.{i}.{n}"]

    def _layer(self, i, x, cos, sin, attend):
        c = self.cfg
        H, Hkv, D = c.n_heads, c.n_kv_heads, c.head_dim
        h = F.rms_norm(x, (c.d_model,), self._l(i, "attn_norm.weight"), c.norm_eps)
        qkv = (h @ self._l(i, "attn.qkv_proj.weight").T).view(*x.shape[:-1], H + 2 * Hkv, D)
        q, k, v = qkv.split([H, Hkv, Hkv], -2)
        q = _rope(F.rms_norm(q, (D,), self._l(i, "attn.q_norm.weight"), c.norm_eps), cos, sin)
        k = _rope(F.rms_norm(k, (D,), self._l(i, "attn.k_norm.weight"), c.norm_eps), cos, sin)
        o = attend(i, q, k, v)
        x = x + o.reshape(*x.shape[:-1], H * D) @ self._l(i, "attn.o_proj.weight").T
        gu = F.rms_norm(x, (c.d_model,), self._l(i, "mlp_norm.weight"), c.norm_eps) @ self._l(i, "gate_up.weight").T
        g, u = gu.chunk(2, -1)
        return x + (F.silu(g) * u) @ self._l(i, "down.weight").T

    @torch.no_grad()
    def generate(self, frames, lens, max_new, bias, max_homopolymer=None, return_margin=False):
        """DecodeEngine(backend="torch").generate (viktor/engine.py:168-220) at temperature 0.  Returns out
        [B, max_new] int64 (and with return_margin the fp32 top-2 margin of logits + bias at every selection,
        [B, max_new], the gap a bf16 path must not cross)."""
        c, tk = self.cfg, self.tok
        B = len(lens)
        frames = torch.from_numpy(np.ascontiguousarray(frames, dtype=np.float32))
        w = self.w
        prefix = F.gelu(frames @ w["projector.0.weight"].T + w["projector.0.bias"]) @ w["projector.2.weight"].T \
            + w["projector.2.bias"]
        max_len = max(lens) + 1 + max_new
        Kc = torch.zeros(c.n_layers, B, max_len, c.n_kv_heads, c.head_dim)
        Vc = torch.zeros_like(Kc)
        offs = np.concatenate([[0], np.cumsum(lens)])
        emb = w["decoder.embed.weight"]
        last = []
        for b in range(B):
            x = torch.cat([prefix[offs[b]:offs[b + 1]], emb[BOS][None]], 0)[None]  # [1, T, d]
            T = x.shape[1]
            cos, sin = self.cos[:T, None], self.sin[:T, None]

            def attend(i, q, k, v, b=b, T=T):
                Kc[i, b, :T], Vc[i, b, :T] = k[0], v[0]
                return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                      is_causal=True, enable_gqa=True).transpose(1, 2)

            for i in range(c.n_layers):
                x = self._layer(i, x, cos, sin, attend)
            last.append(F.rms_norm(x[0, -1], (c.d_model,), w["decoder.norm.weight"], c.norm_eps))
        bias = torch.as_tensor(bias, dtype=torch.float32)
        is_tail = torch.from_numpy(tk.tail_mask)
        is_homo = torch.from_numpy(tk.homo_mask)
        homo_stop = max_homopolymer // tk.k if max_homopolymer else 0
        run = torch.zeros(B, dtype=torch.long)
        head = w["decoder.lm_head.weight"]

        margins = []

        def select(logits, prev):
            z = logits + bias
            top2 = z.topk(2, -1).values
            margins.append(top2[:, 0] - top2[:, 1])
            nxt = z.argmax(-1)
            nxt = torch.where(is_tail[prev], torch.full_like(nxt, EOS), nxt)
            if homo_stop:
                run.copy_(torch.where((nxt == prev) & is_homo[nxt], run + 1, 0))
                nxt = torch.where(run + 1 >= homo_stop, torch.full_like(nxt, EOS), nxt)
            return torch.where((prev == EOS) | (prev == PAD), torch.full_like(nxt, PAD), nxt)

        out = torch.full((B, max_new), PAD, dtype=torch.long)
        tok = torch.full((B,), BOS, dtype=torch.long)
        tok = select(torch.stack(last) @ head.T, tok)
        out[:, 0] = tok
        pos = torch.tensor(lens) + 1
        positions = torch.arange(max_len)
        for step in range(1, max_new):
            x = emb[tok][:, None]  # [B, 1, d]
            cos, sin = self.cos[pos][:, None, None], self.sin[pos][:, None, None]
            rows = torch.arange(B)

            def attend(i, q, k, v):
                Kc[i, rows, pos], Vc[i, rows, pos] = k[:, 0], v[:, 0]
                mask = (positions[None, :] <= pos[:, None])[:, None, None, :]
                n = int(pos.max()) + 1  # positions past every row's current one are masked anyway
                return F.scaled_dot_product_attention(
                    q.transpose(1, 2), Kc[i, :, :n].transpose(1, 2), Vc[i, :, :n].transpose(1, 2),
                    attn_mask=mask[..., :n], enable_gqa=True).transpose(1, 2)

            for i in range(c.n_layers):
                x = self._layer(i, x, cos, sin, attend)
            h = F.rms_norm(x[:, 0], (c.d_model,), w["decoder.norm.weight"], c.norm_eps)
            tok = select(h @ head.T, tok)
            out[:, step] = tok
            pos = pos + 1
        if return_margin:
            return out.numpy(), torch.stack(margins, 1).numpy()
        return out.numpy()
