"""Kernel-level parity on the GPU: each C-ABI op against a plain PyTorch fp32 restatement of the same op.

Tolerances follow the reference's own kernel checks (tests/gpu_check.py:32-81 of GHSSHG/Viktor): RMSNorm /
SwiGLU / QK-norm outputs within 0.05 max-abs of an fp32 reference (bf16 outputs), residual updates and V rows
exact, decode attention within 0.01 of fp32 SDPA.  GEMMs are checked against fp32 matmul of the same bf16
inputs at a relative tolerance of 1e-2 (bf16 output rounding), fp32-output GEMMs at 2e-3 relative.
"""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU too, but every test here is marked gpu
    DEV = None
else:
    DEV = torch.device("cuda")

BF = torch.bfloat16


@pytest.fixture(autouse=True)
def _errors_clear():
    from viktor_b200._lib import check_device_errors
    yield
    torch.cuda.synchronize()
    check_device_errors()


def rope_ref(x, cos, sin):
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].float(), x[..., h:].float()
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1)


def tables(S, theta=1e6, D=64):
    inv = 1.0 / theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)
    fr = torch.arange(S, dtype=torch.float64)[:, None] * inv
    return fr.cos().float().to(DEV), fr.sin().float().to(DEV)


# ------------------------------------------------------------------------------------------------ GEMMs
@pytest.mark.parametrize("M,N,K", [(1, 768, 512), (7, 512, 512), (128, 64, 512), (256, 3072, 512), (300, 512, 1536),
                                   (5000, 512, 512), (4100, 768, 512), (256, 16, 512), (256, 352, 512)])
def test_linear_bf16(M, N, K):
    from viktor_b200.ops import linear
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device=DEV, dtype=BF)
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).to(BF)
    y = linear(x, w)
    ref = x.float() @ w.float().T
    err = (y.float() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2, f"rel err {err}"


@pytest.mark.parametrize("M,N", [(4, 7), (256, 16), (256, 343), (1024, 343)])
def test_linear_f32_logits(M, N):
    from viktor_b200.ops import linear
    torch.manual_seed(N)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    w = (torch.randn(N, 512, device=DEV) / math.sqrt(512)).to(BF)
    y = linear(x, w, out_dtype=torch.float32)
    ref = x.float() @ w.float().T
    assert y.dtype == torch.float32 and y.shape == (M, N)
    assert ((y - ref).abs().max() / ref.abs().max()) < 2e-3


@pytest.mark.parametrize("M", [1, 256, 1000, 5000])
def test_linear_swiglu(M):
    from viktor_b200.ops import linear, swiglu
    torch.manual_seed(M)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    w = (torch.randn(3072, 512, device=DEV) / math.sqrt(512)).to(BF)
    y = linear(x, w, swiglu=True)
    gu = (x.float() @ w.float().T).to(BF)
    g, u = gu.float().chunk(2, -1)
    ref = F.silu(g) * u
    # outputs reach |8| here, where one bf16 ulp is 0.03: compare relative to the output range
    assert (y.float() - ref).abs().max() / ref.abs().max() < 1e-2
    # the unfused op agrees with the fused epilogue
    assert (swiglu(gu).float() - ref).abs().max() / ref.abs().max() < 1e-2


@pytest.mark.parametrize("M,K", [(3, 512), (256, 512), (256, 1536), (1000, 1536), (5000, 512)])
def test_linear_add_rmsnorm(M, K):
    from viktor_b200.ops import linear_add_rmsnorm
    torch.manual_seed(K + M)
    a = torch.randn(M, K, device=DEV, dtype=BF)
    w = (torch.randn(512, K, device=DEV) / math.sqrt(K)).to(BF)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    nw = torch.rand(512, device=DEV, dtype=BF) + 0.5
    delta = (a.float() @ w.float().T).to(BF)
    ref_x = (x.float() + delta.float()).to(BF)
    ref_h = F.rms_norm(ref_x.float(), (512,), nw.float(), 1e-6)
    xk = x.clone()
    h = linear_add_rmsnorm(a, w, xk, nw, 1e-6)
    # x differs from the fp32-matmul reference only where the bf16 rounding of delta lands differently
    assert (xk.float() - ref_x.float()).abs().max() < 0.05
    assert (h.float() - ref_h).abs().max() < 0.05


@pytest.mark.parametrize("M", [1, 200, 256, 1024, 5000])
@pytest.mark.parametrize("swiglu,N,out_f32", [(False, 768, False), (True, 3072, False), (False, 16, True),
                                              (False, 352, True)])
def test_linear_rmsnorm_folded(M, swiglu, N, out_f32):
    """(RMSNorm(x) * w) . W^T computed from x, its block sums of squares and W' = W diag(w) (split-K clusters at
    small M)."""
    from viktor_b200.ops import fold_norm_weight, linear_rmsnorm, row_ssq
    torch.manual_seed(M + N)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    nw = (torch.rand(512, device=DEV) + 0.5).to(BF)
    w = (torch.randn(N, 512, device=DEV) / math.sqrt(512)).to(BF)
    ssq = row_ssq(x)
    assert torch.allclose(ssq, x.float().view(M, 8, 64).square().sum(-1), rtol=1e-5, atol=1e-3)
    y = linear_rmsnorm(x, ssq, 1e-6, fold_norm_weight(w, nw), swiglu=swiglu,
                       out_dtype=torch.float32 if out_f32 else None)
    h = F.rms_norm(x.float(), (512,), nw.float(), 1e-6)
    full = h @ w.float().T
    if swiglu:
        g, u = full.chunk(2, -1)
        ref = F.silu(g) * u
    else:
        ref = full
    err = (y.float() - ref).abs().max() / ref.abs().max()
    assert err < 1.5e-2, f"rel err {err}"


@pytest.mark.parametrize("M,K", [(1, 512), (256, 512), (256, 1536), (1024, 1536), (5000, 512)])
def test_linear_residual(M, K):
    from viktor_b200.ops import linear_residual
    torch.manual_seed(M * K)
    a = torch.randn(M, K, device=DEV, dtype=BF)
    w = (torch.randn(512, K, device=DEV) / math.sqrt(K)).to(BF)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    ref_x = (x.float() + (a.float() @ w.float().T).to(BF).float()).to(BF)
    xk = x.clone()
    ssq = linear_residual(a, w, xk)
    assert (xk.float() - ref_x.float()).abs().max() < 0.05
    assert torch.allclose(ssq, xk.float().view(M, 8, 64).square().sum(-1), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("M", [5, 256, 4500])
def test_linear_bias_act(M):
    from viktor_b200.ops import linear_bias_act
    torch.manual_seed(M)
    x = torch.randn(M, 512, device=DEV, dtype=BF)
    w = (torch.randn(512, 512, device=DEV) / math.sqrt(512)).to(BF)
    b = (torch.randn(512, device=DEV) * 0.1).to(BF)
    y = linear_bias_act(x, w, b, act=1)
    ref = F.gelu((x.float() @ w.float().T + b.float()).to(BF).float())
    assert (y.float() - ref).abs().max() < 0.05
    rows = torch.randperm(M + 3, device=DEV)[:M].int()
    out = torch.zeros(M + 3, 512, device=DEV, dtype=BF)
    linear_bias_act(x, w, b, act=0, out=out, row_map=rows)
    ref0 = (x.float() @ w.float().T + b.float())
    assert (out[rows.long()].float() - ref0).abs().max() < 0.05


# ------------------------------------------------------------------------------------------------ row ops
def test_add_rmsnorm_and_embed():
    from viktor_b200.ops import add_rmsnorm, embed_rmsnorm
    torch.manual_seed(0)
    n, d = 1000, 512
    x = torch.randn(n, d, device=DEV, dtype=BF)
    delta = torch.randn(n, d, device=DEV, dtype=BF)
    w = torch.rand(d, device=DEV, dtype=BF)
    ref_x = x + delta
    ref = F.rms_norm(ref_x.float(), (d,), w.float(), 1e-6)
    xk = x.clone()
    h = add_rmsnorm(xk, w, 1e-6, delta=delta)
    assert torch.equal(xk, ref_x)
    assert (h.float() - ref).abs().max() < 0.05
    emb = torch.randn(343, d, device=DEV, dtype=BF)
    tok = torch.randint(0, 343, (77,), device=DEV)
    xe, he = embed_rmsnorm(tok, emb, w, 1e-6)
    assert torch.equal(xe, emb[tok])
    assert (he.float() - F.rms_norm(emb[tok].float(), (d,), w.float(), 1e-6)).abs().max() < 0.05


def _qkv_reference(qkv, qw, kw, cos, sin, rpos, H=8, HKV=2, D=64):
    n = qkv.shape[0]
    qr, kr, vr = qkv.view(n, H + 2 * HKV, D).split([H, HKV, HKV], 1)
    c, s = cos[rpos.long()][:, None], sin[rpos.long()][:, None]
    rq = rope_ref(F.rms_norm(qr.float(), (D,), qw.float(), 1e-6).to(BF), c, s)
    rk = rope_ref(F.rms_norm(kr.float(), (D,), kw.float(), 1e-6).to(BF), c, s)
    return rq, rk, vr


@pytest.mark.parametrize("fused", [False, True, "normed"])
@pytest.mark.parametrize("n", [200, 1000, 5000])
def test_qkv_rope_cache(fused, n):
    from viktor_b200.ops import fold_norm_weight, linear_qkv_rope_cache, qkv_rope_cache, row_ssq
    torch.manual_seed(n)
    H, HKV, D, S, R = 8, 2, 64, 6000, 4
    qw, kw = torch.rand(D, device=DEV, dtype=BF), torch.rand(D, device=DEV, dtype=BF)
    cos, sin = tables(2 * S, theta=1e4)
    pos = torch.randperm(S, device=DEV)[:n].int()  # distinct slots: every cache write is checkable
    rpos = (pos * 2).int()
    seq = torch.randint(0, R, (n,), device=DEV, dtype=torch.int32)
    kc = torch.zeros(R, S, HKV, D, device=DEV, dtype=BF)
    vc = torch.zeros_like(kc)
    if fused == "normed":  # attention RMSNorm folded into the qkv weight
        xin = torch.randn(n, 512, device=DEV, dtype=BF)
        an = (torch.rand(512, device=DEV) + 0.5).to(BF)
        wq = (torch.randn((H + 2 * HKV) * D, 512, device=DEV) / math.sqrt(512)).to(BF)
        q, k, v = linear_qkv_rope_cache(xin, fold_norm_weight(wq, an), qw, kw, cos, sin, pos, seq, kc, vc, 1e-6,
                                        rope_pos=rpos, return_kv=True, ssq=row_ssq(xin))
        qkv = (F.rms_norm(xin.float(), (512,), an.float(), 1e-6) @ wq.float().T).to(BF)
    elif fused:
        hin = torch.randn(n, 512, device=DEV, dtype=BF)
        wq = (torch.randn((H + 2 * HKV) * D, 512, device=DEV) / math.sqrt(512)).to(BF)
        q, k, v = linear_qkv_rope_cache(hin, wq, qw, kw, cos, sin, pos, seq, kc, vc, 1e-6, rope_pos=rpos,
                                        return_kv=True)
        qkv = (hin.float() @ wq.float().T).to(BF)
    else:
        qkv = torch.randn(n, (H + 2 * HKV) * D, device=DEV, dtype=BF)
        q, k, v = qkv_rope_cache(qkv, qw, kw, cos, sin, pos, seq, kc, vc, 1e-6, H, HKV, D, return_kv=True,
                                 rope_pos=rpos)
    rq, rk, vr = _qkv_reference(qkv, qw, kw, cos, sin, rpos)
    assert (q.float() - rq).abs().max() < 0.05
    assert (k.float() - rk).abs().max() < 0.05
    if fused:
        assert (v.float() - vr.float()).abs().max() < 0.06
    else:
        assert torch.equal(v, vr)
    assert torch.equal(kc[seq.long(), pos.long()], k) and torch.equal(vc[seq.long(), pos.long()], v)


# ------------------------------------------------------------------------------------------------ attention
def _sdpa_ref(q, k, v, lens, row0=0):
    B, H, D = q.shape
    S, HKV = k.shape[1], k.shape[2]
    kk, vv = k[row0:row0 + B], v[row0:row0 + B]
    mask = (torch.arange(S, device=DEV)[None] < lens[:, None].long())[:, None, None]
    return F.scaled_dot_product_attention(q[:, :, None].float(), kk.transpose(1, 2).float().repeat_interleave(H // HKV, 1),
                                          vv.transpose(1, 2).float().repeat_interleave(H // HKV, 1),
                                          attn_mask=mask)[:, :, 0]


@pytest.mark.parametrize("S", [1300, 3200, 4096])  # 4096: the decoder's max_seq_len
def test_decode_attention(S):
    from viktor_b200.ops import decode_attention
    torch.manual_seed(S)
    B, H, HKV, D = 64, 8, 2, 64
    edge = torch.tensor([1, 63, 64, 65, 255, 256, 257, 511, 512, 513, S - 1, S])
    lens = torch.cat([edge, torch.randint(1, S + 1, (B - len(edge),))]).int().to(DEV)
    q = torch.randn(B, H, D, device=DEV, dtype=BF)
    k, v = (torch.randn(B, S, HKV, D, device=DEV, dtype=BF) for _ in range(2))
    for _ in range(2):  # the second call reuses the workspace tickets the first one returned to zero
        out = decode_attention(q, k, v, lens)
        err = (out.float() - _sdpa_ref(q, k, v, lens)).abs().max()
        assert err < 0.01, f"max |out - fp32 ref| {err}"


def test_decode_attention_ignores_stale_rows_and_row_offset():
    """Positions past each length hold NaN here: they must not leak into the output (the reference masks its
    V loads the same way).  Queries read cache rows row0.. of a larger cache."""
    from viktor_b200.ops import decode_attention
    torch.manual_seed(1)
    B, S, row0 = 16, 700, 5
    lens = torch.randint(1, S + 1, (B,)).int().to(DEV)
    q = torch.randn(B, 8, 64, device=DEV, dtype=BF)
    k, v = (torch.randn(B + 8, S, 2, 64, device=DEV, dtype=BF) for _ in range(2))
    pos = torch.arange(S, device=DEV)
    stale = pos[None, :] >= lens[:, None].long()
    kn, vn = k.clone(), v.clone()
    kn[row0:row0 + B][stale] = float("nan")
    vn[row0:row0 + B][stale] = float("nan")
    out = decode_attention(q, kn, vn, lens, row0=row0)
    ref = _sdpa_ref(q, k, v, lens, row0=row0)
    assert torch.isfinite(out).all()
    assert (out.float() - ref).abs().max() < 0.01


def test_prefill_attention():
    from viktor_b200.ops import prefill_attention
    torch.manual_seed(3)
    lens = [1, 63, 64, 65, 127, 128, 129, 200, 256, 777, 2049]
    S, R, row0 = 2100, 14, 2
    n = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    q = torch.randn(n, 8, 64, device=DEV, dtype=BF)
    kc, vc = (torch.randn(R, S, 2, 64, device=DEV, dtype=BF) for _ in range(2))
    out = prefill_attention(q, kc, vc, cu, max(lens), row0=row0)
    for b, T in enumerate(lens):
        t0 = int(cu[b])
        qb = q[t0:t0 + T].transpose(0, 1).float()[None]
        kb = kc[row0 + b, :T].transpose(0, 1).float().repeat_interleave(4, 0)[None]
        vb = vc[row0 + b, :T].transpose(0, 1).float().repeat_interleave(4, 0)[None]
        ref = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True)[0].transpose(0, 1)
        err = (out[t0:t0 + T].float() - ref).abs().max()
        assert err < 0.02, f"seq {b} (T={T}) err {err}"


def test_prefill_attention_at_max_seq_len():
    """A sequence of the decoder's maximum length (4096 positions: 32 query tiles, the diagonal tile full) next
    to a single-token one, in a cache of exactly 4096 positions."""
    from viktor_b200.ops import prefill_attention
    torch.manual_seed(4)
    lens = [4096, 1, 1500]
    S, R = 4096, 3
    n = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    q = torch.randn(n, 8, 64, device=DEV, dtype=BF)
    kc, vc = (torch.randn(R, S, 2, 64, device=DEV, dtype=BF) for _ in range(2))
    out = prefill_attention(q, kc, vc, cu, max(lens))
    for b, T in enumerate(lens):
        t0 = int(cu[b])
        qb = q[t0:t0 + T].transpose(0, 1).float()[None]
        kb = kc[b, :T].transpose(0, 1).float().repeat_interleave(4, 0)[None]
        vb = vc[b, :T].transpose(0, 1).float().repeat_interleave(4, 0)[None]
        ref = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True)[0].transpose(0, 1)
        err = (out[t0:t0 + T].float() - ref).abs().max()
        assert err < 0.02, f"seq {b} (T={T}) err {err}"


# ------------------------------------------------------------------------------------------------ greedy
def test_greedy_update_grammar():
    """Tail -> EOS, homopolymer run -> EOS, after EOS/PAD -> PAD, ties to the left, state advance and the
    fused next-token embedding (viktor/triton_ops.py:172-197)."""
    from viktor_b200.ops import greedy_update
    from viktor_b200.config import KmerTokenizer
    tk = KmerTokenizer(4)
    V, B = tk.vocab_size, 6
    logits = torch.zeros(B, V, device=DEV)
    AAAA = tk.ids["AAAA"]
    tail_A = tk.ids["A"]
    logits[0, 10] = 5.0                    # plain argmax
    logits[1, 20] = 5.0                    # prev is a tail -> EOS
    logits[2, AAAA] = 5.0                  # prev AAAA, run reaches homo_stop -> EOS
    logits[3, 7] = logits[3, 9] = 5.0      # tie -> lower index
    logits[4, 30] = 5.0                    # prev EOS -> PAD
    logits[5, 40] = 5.0                    # prev PAD -> PAD
    bias = torch.zeros(V, device=DEV)
    bias[:2] = float("-inf")
    tok = torch.tensor([5, tail_A, AAAA, 3, 2, 0], device=DEV)
    run = torch.tensor([0, 0, 2, 0, 0, 0], device=DEV)
    plen = torch.tensor([10, 11, 12, 13, 14, 15], device=DEV)
    pos = plen + 3
    rope_off = torch.tensor([0, 1, 2, 3, 4, 5], device=DEV)
    out = torch.zeros(B, 8, dtype=torch.long, device=DEV)
    pos32, seqlens, rpos32 = (torch.zeros(B, dtype=torch.int32, device=DEV) for _ in range(3))
    emb = torch.randn(V, 512, device=DEV, dtype=BF)
    x = torch.zeros(B, 512, device=DEV, dtype=BF)
    ssq = torch.zeros(B, 8, device=DEV)
    greedy_update(logits, bias, torch.from_numpy(tk.tail_mask).to(DEV), torch.from_numpy(tk.homo_mask).to(DEV),
                  4, tok, run, pos, plen, rope_off, out, pos32, seqlens, rpos32, 2, 0, emb=emb, x=x, ssq=ssq)
    assert tok.tolist() == [10, 2, 2, 7, 0, 0]
    assert out[:, 3].tolist() == [10, 2, 2, 7, 0, 0]
    assert run.tolist() == [0, 0, 3, 0, 0, 0]
    assert pos.tolist() == (plen + 4).tolist()
    assert pos32.tolist() == (plen + 4).tolist() and seqlens.tolist() == (plen + 5).tolist()
    assert rpos32.tolist() == (plen + 4 + rope_off).tolist()
    assert torch.equal(x, emb[tok])
    ref_ssq = emb[tok].float().view(B, 8, 64).square().sum(-1)
    assert torch.allclose(ssq, ref_ssq, rtol=1e-5, atol=1e-4)


def test_head_select_equals_lm_head_then_greedy():
    """vk_head_select (lm_head with the folded final norm fused into the selection kernel) picks the tokens of
    fp32 logits r * x . W^T followed by vk_greedy_update, and advances the same state, for both vocabularies."""
    from viktor_b200._lib import call
    from viktor_b200.config import KmerTokenizer
    from viktor_b200.engine import _masks
    for k, B in ((1, 64), (4, 48)):
        tk = KmerTokenizer(k)
        V = tk.vocab_size
        g = torch.Generator(device="cuda").manual_seed(7 + k)
        x = torch.randn(B, 512, generator=g, device=DEV).to(BF)
        xf = x.float()
        ssq = torch.stack([(xf[:, 64 * i:64 * (i + 1)] ** 2).sum(1) for i in range(8)], 1).contiguous()
        w = (torch.randn(V, 512, generator=g, device=DEV) * 0.3).to(BF)
        r = torch.rsqrt(ssq.sum(1, keepdim=True) / 512 + 1e-6)
        logits = (xf @ w.float().t()) * r
        bias = torch.zeros(V, device=DEV)
        bias[:2] = float("-inf")
        tail, homo = _masks(tk, torch.device(DEV))
        emb = torch.randn(V, 512, generator=g, device=DEV).to(BF)
        st = torch.cuda.current_stream().cuda_stream

        def state():
            return dict(tok=torch.randint(3, V, (B,), generator=g, device=DEV), run=torch.zeros(B, dtype=torch.long, device=DEV),
                        pos=torch.full((B,), 10, dtype=torch.long, device=DEV), plen=torch.full((B,), 9, dtype=torch.long, device=DEV),
                        roff=torch.zeros(B, dtype=torch.long, device=DEV), out=torch.zeros(B, 8, dtype=torch.long, device=DEV),
                        p32=torch.zeros(B, dtype=torch.int32, device=DEV), sl=torch.zeros(B, dtype=torch.int32, device=DEV),
                        rp=torch.zeros(B, dtype=torch.int32, device=DEV), x=torch.empty(B, 512, dtype=BF, device=DEV),
                        ssq=torch.empty(B, 8, device=DEV))
        s1 = state()
        s2 = {key: v.clone() for key, v in s1.items()}
        p = lambda t: t.data_ptr()
        call("vk_greedy_update", p(logits), logits.stride(0), p(bias), p(tail), p(homo), 0, p(s1["tok"]), p(s1["run"]),
             p(s1["pos"]), p(s1["plen"]), p(s1["roff"]), p(s1["out"]), 8, 8, p(s1["p32"]), p(s1["sl"]), p(s1["rp"]), B, V,
             2, 0, p(emb), p(s1["x"]), p(s1["ssq"]), st)
        call("vk_head_select", p(x), p(ssq), 1e-6, p(w), p(bias), p(tail), p(homo), 0, p(s2["tok"]), p(s2["run"]),
             p(s2["pos"]), p(s2["plen"]), p(s2["roff"]), p(s2["out"]), 8, 8, p(s2["p32"]), p(s2["sl"]), p(s2["rp"]), B, V,
             2, 0, p(emb), p(s2["x"]), p(s2["ssq"]), None, 0, 1.0, None, 0, st)
        torch.cuda.synchronize()
        top2 = (logits + bias).topk(2, 1).values
        clear = (top2[:, 0] - top2[:, 1]) > 1e-3
        assert clear.float().mean() > 0.9
        assert torch.equal(s1["tok"][clear], s2["tok"][clear])
        for key in ("pos", "p32", "sl", "rp"):
            assert torch.equal(s1[key], s2[key])
        assert torch.equal(s1["x"][clear], s2["x"][clear])


def test_head_select_output_cap_and_finished_rows():
    """The per-row output cap (limit) ends a row with EOS at column limit[b]; with shrink_done, rows whose new
    token is EOS or PAD get seqlens 1 (their next output is PAD regardless), the others pos + 1; tokens, pos and
    the output row are what they are without shrink_done."""
    from viktor_b200._lib import call
    from viktor_b200.config import KmerTokenizer
    from viktor_b200.engine import _masks
    tk = KmerTokenizer(1)
    V, B = tk.vocab_size, 8
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(B, 512, generator=g, device=DEV).to(BF)
    xf = x.float()
    ssq = torch.stack([(xf[:, 64 * i:64 * (i + 1)] ** 2).sum(1) for i in range(8)], 1).contiguous()
    w = (torch.randn(V, 512, generator=g, device=DEV) * 0.3).to(BF)
    bias = torch.zeros(V, device=DEV)
    bias[:3] = float("-inf")  # PAD, BOS, EOS never chosen by the argmax
    tail, homo = _masks(tk, torch.device(DEV))
    emb = torch.randn(V, 512, generator=g, device=DEV).to(BF)
    st = torch.cuda.current_stream().cuda_stream
    # rows at output columns 0..7 (pos - plen); row 6 had emitted EOS, row 7 PAD
    plen = torch.full((B,), 100, dtype=torch.long, device=DEV)
    col = torch.arange(8, dtype=torch.long, device=DEV)
    limit = torch.tensor([0, 5, 2, 9, 4, 6, 1, 1], dtype=torch.long, device=DEV)
    prev = torch.tensor([1, 3, 4, 5, 6, 3, 2, 0], dtype=torch.long, device=DEV)
    outs = {}
    for shrink in (0, 1):
        s = dict(tok=prev.clone(), run=torch.zeros(B, dtype=torch.long, device=DEV), pos=plen + col, plen=plen,
                 roff=torch.zeros(B, dtype=torch.long, device=DEV),
                 out=torch.full((B, 8), -1, dtype=torch.long, device=DEV),
                 p32=torch.zeros(B, dtype=torch.int32, device=DEV), sl=torch.zeros(B, dtype=torch.int32, device=DEV),
                 rp=torch.zeros(B, dtype=torch.int32, device=DEV), x=torch.empty(B, 512, dtype=BF, device=DEV),
                 ssq=torch.empty(B, 8, device=DEV))
        p = lambda t: t.data_ptr()
        call("vk_head_select", p(x), p(ssq), 1e-6, p(w), p(bias), p(tail), p(homo), 0, p(s["tok"]), p(s["run"]),
             p(s["pos"]), p(s["plen"]), p(s["roff"]), p(s["out"]), 8, 8, p(s["p32"]), p(s["sl"]), p(s["rp"]), B, V,
             2, 0, p(emb), p(s["x"]), p(s["ssq"]), None, 0, 1.0, p(limit), shrink, st)
        torch.cuda.synchronize()
        outs[shrink] = s
    a, b = outs[0], outs[1]
    tok = b["tok"].cpu().tolist()
    # col >= limit -> EOS (rows 0, 2, 4); below the cap: a base (rows 1, 3, 5); after EOS / PAD: PAD (rows 6, 7)
    assert [tok[i] for i in (0, 2, 4)] == [2, 2, 2]
    assert tok[1] >= 3 and tok[3] >= 3 and tok[5] >= 3
    assert tok[6] == 0 and tok[7] == 0
    for key in ("tok", "pos", "p32", "out", "rp"):
        assert torch.equal(a[key], b[key]), key
    assert torch.equal(a["sl"], (plen + col + 2).int())
    ended = torch.tensor([t in (0, 2) for t in tok], device=DEV)
    assert torch.equal(b["sl"], torch.where(ended, torch.ones_like(a["sl"]), a["sl"]))
