"""Greedy decoding for variable-length chunks on B200: static KV cache, packed prefill, one CUDA graph per step.

Drop-in for viktor/engine.py's ``DecodeEngine`` (constructor, ``prefill``, ``decode``, ``generate``, the
reused ``out`` buffer, the mutable ``bias`` and the ``cache`` attribute).  Semantics kept from the reference:

* each sequence's prefix is its chunk's encoder frames (projected) + BOS; prefix lengths differ and every
  sequence decodes at its own position (viktor/engine.py:6-9);
* finished sequences keep running and emit PAD, so every step is shape-static and graph-capturable;
* prefill keeps all K/V but runs the last layer for BOS only;
* grammar: a tail token is followed by EOS; a run of one homopolymer token reaching ``max_homopolymer`` bases
  gets EOS; after EOS/PAD comes PAD (viktor/engine.py:79-89);
* ``decode(steps=n)`` runs exactly n-1 steps; ``steps=None`` stops when every sequence has ended (checked every
  ``check_every`` steps) or at ``max_new_tokens``.

Every kernel here is this package's CUDA code; there is no CPU or PyTorch fallback.  One decode step is 42
launches (8 x [norm+qkv+rope+cache GEMM, attention, o GEMM+residual, norm+gate_up GEMM+SwiGLU, down
GEMM+residual], norm+lm_head GEMM, greedy+grammar+next embedding), replayed as one CUDA graph.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import call, check_device_errors, load
from .config import BOS, EOS, PAD
from .decoder import KVCache
from .fast_decoder import DeviceWeights, FastDecoder
from .ops import PrefixKV8

_BF16 = torch.bfloat16


def _p(t):
    return None if t is None else t.data_ptr()


def _masks(tokenizer, device):
    """Tail mask (viktor/tokenizer.py:24-27) and homopolymer mask (viktor/engine.py:67-68) as uint8."""
    V = tokenizer.vocab_size
    tail = torch.as_tensor(np.asarray(tokenizer.tail_mask, dtype=bool)).reshape(V)
    strings = tokenizer.strings
    homo = torch.tensor([i >= 3 and len(t) == tokenizer.k and len(set(t)) == 1 for i, t in enumerate(strings)])
    return tail.to(torch.uint8).to(device), homo.to(torch.uint8).to(device)


def prefill_plan(lens, row0=0, pos_scale=1):
    """Packed prefill layout of chunks row0.. with the given prefix lengths (viktor/engine.py:145-159).

    Sequence b occupies packed rows cu[b] .. cu[b+1]-1: its lens[b] frames then BOS.  Returns numpy arrays:
    cu [n+1] i32, frame_idx [sum(lens)] i32 (packed row of each frame), last [n] i64 (BOS rows), pos [total] i32
    (position in the sequence), seq [total] i32 (cache row), rpos [total] i32 or None (RoPE positions: frame j at
    j * pos_scale, BOS at lens[b] * pos_scale), lengths [n] i32 (= lens + 1) and the sizes."""
    n = len(lens)
    L = np.asarray(lens, dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(L + 1)]).astype(np.int64)
    total = int(offsets[-1])
    seg = np.repeat(np.arange(n), L)
    frame_idx = (np.arange(int(L.sum())) + seg).astype(np.int32)
    last = (offsets[1:] - 1).astype(np.int64)
    pos = (np.arange(total) - np.repeat(offsets[:-1], L + 1)).astype(np.int32)
    seq = np.repeat(np.arange(row0, row0 + n, dtype=np.int32), L + 1)
    rpos = None if pos_scale == 1 else (pos.astype(np.int64) * pos_scale).astype(np.int32)
    return dict(cu=offsets.astype(np.int32), frame_idx=frame_idx, last=last, pos=pos, seq=seq, rpos=rpos,
                lengths=(L + 1).astype(np.int32), total=total, frames=int(L.sum()),
                max_len=int(L.max()) + 1 if n else 0, n=n)


class DecodeEngine:
    def __init__(self, model, batch_size: int, max_new_tokens: int, max_frames: int, backend: str = "auto",
                 cuda_graph: bool = True, prefill_batch: int = 128, check_every: int = 32,
                 attention_backend: str = "auto", temperature: float = 0.0, max_homopolymer: int | None = 64,
                 device=None, decode_groups: int = 2, kv_int8: bool = False, steps_per_graph: int = 16):
        if backend not in ("auto", "cuda", "triton"):
            raise ValueError(f"backend {backend!r}: this engine runs the B200 CUDA kernels only")
        if attention_backend not in ("auto", "cuda", "triton", "flash"):
            raise ValueError(f"unknown decode attention backend: {attention_backend}")
        load()
        self.model, self.dec = model, model.decoder
        self.temperature = float(temperature)
        if device is None:
            dev = model.decoder.lm_head.weight.device
            device = dev if dev.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("DecodeEngine needs a CUDA device")
        self.device = dev = device
        self.dtype = _BF16
        self.backend = "cuda"
        self.pos_scale = int(getattr(model, "pos_scale", 1))
        self.w = DeviceWeights(model, dev)
        self.fast = FastDecoder(self.w)
        cfg = self.cfg = self.dec.cfg
        self.B, self.max_new = batch_size, max_new_tokens
        self.max_frames = max_frames
        self.prefill_batch, self.check_every = prefill_batch, check_every
        self._prefill_plans = {}
        max_len = max_frames + 1 + max_new_tokens
        assert max_len <= cfg.max_seq_len
        self.cache = KVCache(cfg, batch_size, max_len, _BF16, dev)
        B, d, V = batch_size, cfg.d_model, cfg.vocab_size

        self.tok = torch.full((B,), BOS, dtype=torch.long, device=dev)
        self.pos = torch.zeros(B, dtype=torch.long, device=dev)
        self.rope_off = torch.zeros(B, dtype=torch.long, device=dev)
        self.pos32 = torch.zeros(B, dtype=torch.int32, device=dev)
        self.rpos32 = torch.zeros(B, dtype=torch.int32, device=dev)
        self.seqlens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.rows = torch.arange(B, dtype=torch.int32, device=dev)
        self.out = torch.full((B, max_new_tokens), PAD, dtype=torch.long, device=dev)
        self.bias = torch.zeros(V, device=dev)
        self.bias[[PAD, BOS]] = float("-inf")
        tk = model.tokenizer
        self.is_tail, self.is_homo = _masks(tk, dev)
        self.homo_stop = max_homopolymer // tk.k if max_homopolymer else 0
        self.run = torch.zeros(B, dtype=torch.long, device=dev)
        self.plen = torch.zeros(B, dtype=torch.long, device=dev)
        # Per-row output cap (an extension; the reference has none): the token of output column max_tokens[b]
        # is EOS, so row b emits at most max_tokens[b] tokens before it ends.  The default, max_new_tokens, never
        # triggers.  A benchmark sets it to stand in for a trained model that ends each read at its own length.
        self.max_tokens = torch.full((B,), max_new_tokens, dtype=torch.long, device=dev)
        # Rows that have ended decode at the cost of one cached position per layer: after EOS every output is PAD
        # whatever the step computes (viktor/engine.py:88), so the selection kernel gives such a row seqlens 1
        # and its attention skips the rest of its cache row.  Output tokens are unchanged.  (Not with the int8
        # prefix mode, whose attention needs every row's length past its int8 prefix.)
        self.skip_finished = not kv_int8

        # decode-step activations: residual x and the block sums of squares of its rows (folded RMSNorms)
        self.x = torch.zeros(B, d, dtype=_BF16, device=dev)
        self.ssq = torch.ones(B, 8, dtype=torch.float32, device=dev)
        self.q = torch.zeros(B, cfg.n_heads, cfg.head_dim, dtype=_BF16, device=dev)
        self.o = torch.zeros(B, cfg.n_heads * cfg.head_dim, dtype=_BF16, device=dev)
        self.g = torch.zeros(B, cfg.ffn_dim, dtype=_BF16, device=dev)
        self.logits = torch.zeros(B, self.w.vpad, dtype=torch.float32, device=dev)
        ws_bytes = load().vk_decode_attention_workspace_bytes(B, max_len)
        self.attn_ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        # Sampled decoding (viktor/engine.py:81-82): one [B, V] draw of uniform noise per selection, made with
        # the same generator call as the reference's torch.rand_like (captured into the step's graph).
        self.noise = (torch.empty(B, self.w.vocab, dtype=torch.float32, device=dev) if self.temperature > 0
                      else None)
        # Decode groups: the batch is split into row ranges whose steps run on their own streams, so that one
        # group's latency-bound projection chain overlaps another group's bandwidth-bound attention.  Every row
        # is computed exactly as in a single group (the split changes no arithmetic).
        G = max(1, min(int(decode_groups), B))
        edges = [B * g // G for g in range(G + 1)]
        self._groups = []
        for g in range(G):
            lo, hi = edges[g], edges[g + 1]
            ws = torch.zeros(load().vk_decode_attention_workspace_bytes(hi - lo, max_len), dtype=torch.uint8,
                             device=dev)
            self._groups.append((lo, hi, ws))
        self._side_streams = [torch.cuda.Stream(dev) for _ in range(G)] if G > 1 else []
        self._copy_stream = None  # host -> device copies of prefill frames (pinned host input)
        self._pf = None  # prefill scratch, allocated on first prefill and grown when a sub-batch needs more
        # the final residual of every chunk's BOS row (and its sums of squares), kept across prefill sub-batches
        self._xcat = torch.empty(B, cfg.d_model, dtype=_BF16, device=dev)
        self._scat = torch.empty(B, 8, dtype=torch.float32, device=dev)
        # Opt-in INT8 prefix KV (the reference's analysis.md:95 proposal): after prefill, every layer's prefix
        # (frames + BOS) is copied into int8 with per-channel scales and decode attention reads that copy, while the
        # generated tokens' K/V stay bf16.  Changes the arithmetic: a mode with its own tolerance, off by default.
        self.kv_int8 = bool(kv_int8)
        if self.kv_int8:
            self.prefix8 = [PrefixKV8(B, max_frames + 1, dev) for _ in range(cfg.n_layers)]
            self.starts = torch.zeros(B, dtype=torch.int32, device=dev)
            self.max_tail = max_new_tokens + 1
            S8 = self.prefix8[0].S8
            self._ws8 = [torch.zeros(load().vk_decode_attention_i8_workspace_bytes(hi - lo, S8, self.max_tail),
                                     dtype=torch.uint8, device=dev) for lo, hi, _ in self._groups]
        self.graph = None
        self.graph_multi = None
        self.kernels_per_step = 0
        self.steps_per_graph = max(1, int(steps_per_graph))
        if cuda_graph:
            self._capture()

    # ------------------------------------------------------------------ decode step
    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _draw_noise(self):
        """The uniform draws of one selection (torch.rand_like of viktor/engine.py:82: same shape, dtype and
        generator call)."""
        self.noise.uniform_()

    def _step(self):
        """One greedy (or sampled) step for every sequence (viktor/engine.py:91-116)."""
        if self.noise is not None:
            self._draw_noise()
        if not self._side_streams:
            self._step_rows(0, self._stream())
            return
        main = torch.cuda.current_stream(self.device)
        for gi, side in enumerate(self._side_streams):
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self._step_rows(gi, side.cuda_stream)
        for side in self._side_streams:
            main.wait_stream(side)

    def _steps(self, n):
        """n decode steps.  Greedy steps of several groups run each group's n steps back to back on its own stream
        (the groups' rows are independent); sampled steps draw their noise for all rows per step, so they go through
        _step one at a time."""
        if self.noise is not None or not self._side_streams:
            for _ in range(n):
                self._step()
            return
        main = torch.cuda.current_stream(self.device)
        for side in self._side_streams:
            side.wait_stream(main)
        for _ in range(n):
            for gi, side in enumerate(self._side_streams):
                with torch.cuda.stream(side):
                    self._step_rows(gi, side.cuda_stream)
        for side in self._side_streams:
            main.wait_stream(side)

    def _step_rows(self, gi, st):
        """One decode step of the sequences in the rows [lo, hi) of decode group gi."""
        lo, hi, ws = self._groups[gi]
        r = slice(lo, hi)
        rp = None if self.pos_scale == 1 else self.rpos32[r]
        prefix = None
        if self.kv_int8:
            ws = self._ws8[gi]
            prefix = dict(layers=self.prefix8, starts=self.starts[r], max_tail=self.max_tail)
        self.fast.decode(self.x[r], self.ssq[r], self.pos32[r], self.rows[r], self.seqlens[r], self.cache, self.q[r],
                         self.o[r], self.g[r], ws, rope_pos=rp, stream=st, row0=lo, prefix=prefix)
        self._head_select(self.x[r], self.ssq[r], st, lo, hi)

    def _head_select(self, x, ssq, st, lo=0, hi=None):
        """lm_head on the final-normed rows (fp32 logits) + greedy grammar + state advance + the next step's
        embedding and its sums of squares, for the sequences in rows [lo, hi)."""
        w = self.w
        hi = self.B if hi is None else hi
        r = slice(lo, hi)
        # lm_head (final norm folded in) fused into the selection kernel, which also writes the next step's
        # embedding into self.x (x may be those same rows: each is read before it is overwritten)
        noise = (None, 0, 1.0) if self.noise is None else (_p(self.noise[r]), self.noise.stride(0), self.temperature)
        call("vk_head_select", _p(x), _p(ssq), w.eps, _p(w.lm_head), _p(self.bias), _p(self.is_tail),
             _p(self.is_homo), self.homo_stop, _p(self.tok[r]), _p(self.run[r]), _p(self.pos[r]), _p(self.plen[r]),
             _p(self.rope_off[r]), _p(self.out[r]), self.out.stride(0), self.out.shape[1], _p(self.pos32[r]),
             _p(self.seqlens[r]), _p(self.rpos32[r]), hi - lo, w.vocab, EOS, PAD, _p(w.embed), _p(self.x[r]),
             _p(self.ssq[r]), *noise, _p(self.max_tokens[r]), 1 if self.skip_finished else 0, st)

    @torch.no_grad()
    def _capture(self):
        # warm-up launches (first launch of each kernel raises its shared-memory limit) on a side stream
        saved = [t.clone() for t in (self.pos, self.pos32, self.seqlens, self.rpos32, self.tok, self.run)]
        self.pos.fill_(1)
        self.pos32.fill_(1)
        self.seqlens.fill_(2)
        self.rpos32.fill_(1)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(3):  # (with decode groups, each group also runs on its own stream here)
                self.pos.fill_(1)
                self.pos32.fill_(1)
                self.seqlens.fill_(2)
                self.rpos32.fill_(1)
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        before = _lib.launches
        with torch.cuda.graph(self.graph):
            self._step()
        self.kernels_per_step = _lib.launches - before
        # Several steps in one graph: between two graph launches the GPU idles (~13 us measured at config 2), while
        # inside a graph each decode group's next step follows its previous one on the same stream, its kernels
        # launched early (programmatic dependent launch) as within a step.
        self.graph_multi = None
        if self.steps_per_graph > 1:
            self.graph_multi = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph_multi):
                self._steps(self.steps_per_graph)
        for t, v in zip((self.pos, self.pos32, self.seqlens, self.rpos32, self.tok, self.run), saved):
            t.copy_(v)
        self.out.fill_(PAD)
        torch.cuda.synchronize(self.device)
        check_device_errors()

    # ------------------------------------------------------------------ prefill
    def _plan(self, lens, row0):
        """Packed layout of one sub-batch (viktor/engine.py:145-159), built on the device by vk_prefill_plan from
        the n prefix lengths (one small host->device copy) once per length tuple and kept on the device."""
        key = tuple(lens)
        entry = self._prefill_plans.get(row0)
        if entry is not None and entry[0] == key:
            return entry[1]
        dev, n = self.device, len(lens)
        frames = int(sum(lens))
        total = frames + n
        i32 = dict(dtype=torch.int32, device=dev)
        plan = dict(cu=torch.empty(n + 1, **i32), frame_idx=torch.empty(max(frames, 1), **i32)[:frames],
                    last=torch.empty(n, dtype=torch.int64, device=dev), pos=torch.empty(total, **i32),
                    seq=torch.empty(total, **i32), rpos=None if self.pos_scale == 1 else torch.empty(total, **i32),
                    lengths=torch.empty(n, **i32), total=total, frames=frames, max_len=max(lens) + 1, n=n)
        lens_d = torch.tensor(lens, dtype=torch.int32).to(dev, non_blocking=True)
        call("vk_prefill_plan", _p(lens_d), n, row0, self.pos_scale, total, _p(plan["cu"]), _p(plan["frame_idx"]),
             _p(plan["last"]), _p(plan["pos"]), _p(plan["seq"]), None if plan["rpos"] is None else _p(plan["rpos"]),
             _p(plan["lengths"]), self._stream())
        plan["_lens"] = lens_d  # keeps the source alive until the plan kernel has run
        self._prefill_plans[row0] = (key, plan)
        return plan

    def _prefill_buffers(self, rows, frames):
        cfg, dev = self.cfg, self.device
        pf = self._pf
        if pf is None or pf["rows"] < rows or pf["frames"] < frames:
            rows = max(rows, pf["rows"] if pf else 0)
            frames = max(frames, pf["frames"] if pf else 0)
            nb = min(self.prefill_batch, self.B)
            pf = dict(rows=rows, frames=frames,
                      fb=torch.empty(frames, self.w.d_enc, dtype=_BF16, device=dev),
                      mid=torch.empty(frames, cfg.d_model, dtype=_BF16, device=dev),
                      x=torch.empty(rows, cfg.d_model, dtype=_BF16, device=dev),
                      ssq=torch.empty(rows, 8, dtype=torch.float32, device=dev),
                      q=torch.empty(rows, cfg.n_heads, cfg.head_dim, dtype=_BF16, device=dev),
                      o=torch.empty(rows, cfg.n_heads * cfg.head_dim, dtype=_BF16, device=dev),
                      g=torch.empty(rows, cfg.ffn_dim, dtype=_BF16, device=dev),
                      xl=torch.empty(nb, cfg.d_model, dtype=_BF16, device=dev),
                      sl=torch.empty(nb, 8, dtype=torch.float32, device=dev),
                      ql=torch.empty(nb, cfg.n_heads, cfg.head_dim, dtype=_BF16, device=dev),
                      ol=torch.empty(nb, cfg.n_heads * cfg.head_dim, dtype=_BF16, device=dev),
                      gl=torch.empty(nb, cfg.ffn_dim, dtype=_BF16, device=dev))
            self._pf = pf
        return pf

    def _prefill_sub(self, frames, lens, row0, st):
        """Projector + packed prefill of chunks row0..row0+len(lens); writes the final residual of their BOS rows
        (and its sums of squares) into xcat / scat."""
        w, plan = self.w, self._plan(lens, row0)
        n, nf, total = plan["n"], plan["frames"], plan["total"]
        pf = self._prefill_buffers(total, nf)
        # frames -> bf16 (viktor/engine.py:180 .to(dtype))
        if frames.dtype == _BF16:
            fb = frames.contiguous()
        else:
            fb = pf["fb"][:nf]
            call("vk_cast_f32_bf16", _p(frames.float().contiguous()), _p(fb), nf * w.d_enc, st)
        # projector: Linear-GELU-Linear; the second GEMM scatters rows into the packed layout
        w0, b0, w1, b1 = w.proj
        mid = pf["mid"][:nf]
        x, ssq = pf["x"][:total], pf["ssq"][:total]
        call("vk_linear_bias_act", _p(fb), _p(w0), _p(b0), _p(mid), mid.stride(0), None, nf, 512, w.d_enc, 1, st)
        call("vk_linear_bias_act", _p(mid), _p(w1), _p(b1), _p(x), x.stride(0), _p(plan["frame_idx"]), nf, 512, 512,
             0, st)
        call("vk_scatter_embed", _p(x), _p(plan["last"]), n, total, _p(w.embed), BOS, 512, st)
        call("vk_row_ssq", _p(x), _p(ssq), total, 512, st)
        xl, sl = pf["xl"][:n], pf["sl"][:n]
        self.fast.prefill(x, ssq, plan["pos"], plan["seq"], plan["cu"], plan["max_len"], self.cache,
                          pf["q"][:total], pf["o"][:total], pf["g"][:total], row0=row0, rope_pos=plan["rpos"],
                          last_indices=plan["last"], lengths=plan["lengths"], x_last=xl, ssq_last=sl,
                          q_last=pf["ql"][:n], o_last=pf["ol"][:n], g_last=pf["gl"][:n], workspace=self.attn_ws,
                          stream=st)
        self._xcat[row0:row0 + n].copy_(xl)
        self._scat[row0:row0 + n].copy_(sl)
        if self.kv_int8:
            starts = plan["lengths"]  # prefix positions of each chunk: its frames and BOS
            kc, vc = self.cache.k, self.cache.v
            for i, pre in enumerate(self.prefix8):
                call("vk_kv_quantize", _p(kc[i]), _p(vc[i]), kc.shape[1], kc.shape[2], kc.stride(1), kc.stride(2),
                     _p(starts), row0, n, _p(pre.k8), _p(pre.v8t), _p(pre.sk), _p(pre.sv), pre.S8, st)
            self.starts[row0:row0 + n].copy_(starts)

    @torch.no_grad()
    def prefill(self, frames, frame_lens):
        """frames [sum(frame_lens), d_enc]: encoder frames of B chunks, concatenated (device or host tensor);
        frame_lens [B].  Fills the cache and emits the first token of every sequence (viktor/engine.py:168-201)."""
        frame_lens = [int(n) for n in frame_lens]
        assert len(frame_lens) == self.B and frames.shape[0] == sum(frame_lens)
        if max(frame_lens) > self.max_frames or min(frame_lens) < 0:
            raise ValueError(f"frame_lens must lie in [0, {self.max_frames}]")
        if self.pos_scale != 1:
            top = max(n * self.pos_scale + self.max_new for n in frame_lens)
            if top >= self.cfg.max_seq_len:
                raise ValueError("RoPE positions would exceed max_seq_len")
        st = self._stream()
        offs = np.concatenate([[0], np.cumsum(frame_lens)]).astype(np.int64)
        subs = [(lo, min(self.B, lo + self.prefill_batch)) for lo in range(0, self.B, self.prefill_batch)]
        ready = [None] * len(subs)
        if frames.device != self.device:
            if frames.is_pinned():
                # host -> device copy per sub-batch on a copy stream, so that sub-batch i + 1 crosses PCIe while
                # sub-batch i is prefilled
                if self._copy_stream is None:
                    self._copy_stream = torch.cuda.Stream(self.device)
                cur = torch.cuda.current_stream(self.device)
                dev_frames = torch.empty(frames.shape, dtype=frames.dtype, device=self.device)
                cs = self._copy_stream
                cs.wait_stream(cur)
                for i, (lo, hi) in enumerate(subs):
                    a, b = int(offs[lo]), int(offs[hi])
                    with torch.cuda.stream(cs):
                        dev_frames[a:b].copy_(frames[a:b], non_blocking=True)
                        ready[i] = torch.cuda.Event()
                        ready[i].record(cs)
                dev_frames.record_stream(cs)
                frames = dev_frames
            else:
                frames = frames.to(self.device)
        for i, (lo, hi) in enumerate(subs):
            if ready[i] is not None:
                torch.cuda.current_stream(self.device).wait_event(ready[i])
            self._prefill_sub(frames[int(offs[lo]):int(offs[hi])], frame_lens[lo:hi], lo, st)
        xcat, scat = self._xcat, self._scat
        # first token: select with prev = BOS; greedy writes column pos - plen = 0 and sets pos = plen + 1
        self.tok.fill_(BOS)
        self.run.zero_()
        self.out.fill_(PAD)
        self.plen.copy_(torch.tensor(frame_lens, device=self.device))
        self.pos.copy_(self.plen)
        self.rope_off.copy_(self.plen * (self.pos_scale - 1))
        if self.noise is not None:
            self._draw_noise()
        self._head_select(xcat, scat, st)

    # ------------------------------------------------------------------ decode loop
    @torch.no_grad()
    def decode(self, steps=None):
        """Run decode steps after prefill.  steps=None: stop when all sequences ended (checked every check_every
        steps) or at max_new_tokens.  steps=n: run exactly n-1 steps (n output tokens)."""
        n = self.max_new - 1 if steps is None else steps - 1
        k = self.steps_per_graph if self.graph_multi is not None else 1
        if steps is None and self.check_every % k:
            k = 1  # the multi-step graph must not step past a check_every poll
        i = 0
        while i < n:
            if self.graph is None:
                self._step()
                i += 1
            elif k > 1 and n - i >= k:
                self.graph_multi.replay()
                _lib.launches += k * self.kernels_per_step
                i += k
            else:
                self.graph.replay()
                _lib.launches += self.kernels_per_step
                i += 1
            if steps is None and i % self.check_every == 0 and bool(((self.tok == EOS) | (self.tok == PAD)).all()):
                break
        return self.out

    def generate(self, frames, frame_lens, steps=None):
        """Returns token ids [B, max_new_tokens] (PAD after EOS).  The buffer is reused by the next call."""
        self.prefill(frames, frame_lens)
        return self.decode(steps)

    @torch.no_grad()
    def teacher_forced_logits(self, frames, frame_lens, tokens_in):
        """Teacher forcing through the prefill kernels (the computation of viktor/model.py:55-60): sequence b
        is [projected frames_b | embed(tokens_in[b])], all layers run over every position, and the fp32 logits
        at the token positions are returned, [B, T, V].  Uses (and overwrites) the cache rows 0..B-1."""
        frame_lens = [int(n) for n in frame_lens]
        B, T = tokens_in.shape
        assert B <= self.B and frames.shape[0] == sum(frame_lens)
        w, dev, st = self.w, self.device, self._stream()
        lens = [n + T for n in frame_lens]
        if max(lens) > self.cache.max_len:
            raise ValueError("sequence longer than the cache")
        L = np.asarray(lens, dtype=np.int64)
        P = np.asarray(frame_lens, dtype=np.int64)
        offsets = np.concatenate([[0], np.cumsum(L)])
        total = int(offsets[-1])
        pos = (np.arange(total) - np.repeat(offsets[:-1], L)).astype(np.int64)
        seq = np.repeat(np.arange(B), L).astype(np.int32)
        frame_rows = np.concatenate([offsets[b] + np.arange(P[b]) for b in range(B)]).astype(np.int32)
        tok_rows = np.concatenate([offsets[b] + P[b] + np.arange(T) for b in range(B)]).astype(np.int64)
        if self.pos_scale == 1:
            rpos = None
        else:
            pb = np.repeat(P, L)
            rpos = np.where(pos < pb, pos * self.pos_scale, pos + (self.pos_scale - 1) * pb).astype(np.int32)

        def t(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        nf = int(P.sum())
        x = torch.empty(total, 512, dtype=_BF16, device=dev)
        ssq = torch.empty(total, 8, dtype=torch.float32, device=dev)
        fb = torch.empty(nf, w.d_enc, dtype=_BF16, device=dev)
        mid = torch.empty(nf, 512, dtype=_BF16, device=dev)
        frames = frames.to(dev)
        call("vk_cast_f32_bf16", _p(frames.float().contiguous()), _p(fb), nf * w.d_enc, st)
        w0, b0, w1, b1 = w.proj
        call("vk_linear_bias_act", _p(fb), _p(w0), _p(b0), _p(mid), 512, None, nf, 512, w.d_enc, 1, st)
        call("vk_linear_bias_act", _p(mid), _p(w1), _p(b1), _p(x), 512, _p(t(frame_rows)), nf, 512, 512, 0, st)
        toks = tokens_in.reshape(-1).to(dev, torch.int64).contiguous()
        call("vk_copy_rows", _p(w.embed), _p(toks), w.vocab, _p(x), _p(t(tok_rows)), total, B * T, 1024, st)
        call("vk_row_ssq", _p(x), _p(ssq), total, 512, st)
        q = torch.empty(total, 8, 64, dtype=_BF16, device=dev)
        o = torch.empty(total, 512, dtype=_BF16, device=dev)
        g = torch.empty(total, self.cfg.ffn_dim, dtype=_BF16, device=dev)
        self.fast.prefill(x, ssq, t(pos.astype(np.int32)), t(seq), t(offsets.astype(np.int32)), int(L.max()),
                          self.cache, q, o, g, row0=0, rope_pos=None if rpos is None else t(rpos), stream=st)
        rows = t(tok_rows)
        xt = torch.empty(B * T, 512, dtype=_BF16, device=dev)
        st_ = torch.empty(B * T, 8, dtype=torch.float32, device=dev)
        call("vk_gather_rows", _p(x), _p(rows), _p(xt), B * T, 1024, total, st)
        call("vk_gather_rows", _p(ssq), _p(rows), _p(st_), B * T, 32, total, st)
        logits = torch.empty(B * T, w.vpad, dtype=torch.float32, device=dev)
        self.fast.logits(xt, st_, logits, st)
        return logits[:, :w.vocab].reshape(B, T, w.vocab)

    def check_errors(self):
        """Synchronises and raises if a kernel flagged an error (bounds, timed-out wait)."""
        torch.cuda.synchronize(self.device)
        check_device_errors()
