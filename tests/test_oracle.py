"""The CPU oracle reproduces the reference's own outputs (golden fixtures made by importing the reference)."""

import numpy as np
import pytest

from golden_io import CASES, load
from oracle import OracleConfig, OracleModel


def oracle_for(g):
    m = g["meta"]
    return OracleModel(OracleConfig(**m["cfg"]), g["weights"], k=m["k"], pos_scale=m["pos_scale"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_teacher_forced_logits_match_reference(name):
    g = load(name)
    om = oracle_for(g)
    offs = np.concatenate([[0], np.cumsum(g["meta"]["lens"])])
    for b in range(len(g["meta"]["lens"])):
        got = om.logits(g["frames"][offs[b]:offs[b + 1]], g["tf_tokens"][b])
        np.testing.assert_allclose(got, g["tf_logits"][b], atol=2e-4, rtol=1e-4)


@pytest.mark.parametrize("name", CASES)
def test_oracle_greedy_tokens_match_reference(name):
    g = load(name)
    m = g["meta"]
    om = oracle_for(g)
    noise = None if g["noise"] is None else (lambda i: g["noise"][i])
    out, margin = om.generate(g["frames"], m["lens"], m["max_new"], steps=m["max_new"], bias=g["bias"],
                              max_homopolymer=m["max_homopolymer"], temperature=m["temperature"], noise=noise)
    np.testing.assert_array_equal(out, g["tokens"])
    # every decided token had a clear fp32 margin, so the comparison is meaningful
    assert np.nanmin(margin) > 1e-4


def test_tokenizer_matches_reference_layout():
    from viktor_b200.config import EOS, KmerTokenizer
    import random
    for k in (1, 4):
        tok = KmerTokenizer(k)
        assert tok.vocab_size == 3 + sum(4 ** j for j in range(1, k + 1))
        rng = random.Random(k)
        for n in range(0, 23):
            s = "".join(rng.choice("ACGT") for _ in range(n))
            ids = tok.encode(s)
            assert len(ids) == -(-n // k)
            assert not any(tok.tail_mask[i] for i in ids[:-1])
            assert tok.decode(ids + [EOS, 5]) == s
            assert int(tok.n_bases[ids].sum()) == n


@pytest.mark.parametrize("name", ["base_theta1e6", "kmer4", "homopolymer", "base_b8"])
def test_torch_cpu_baseline_port_matches_reference(name):
    """The port timed as the CPU baseline produces the reference's greedy tokens."""
    from oracle.decoder_torch import TorchCPUModel
    g = load(name)
    m = g["meta"]
    if m["pos_scale"] != 1 or m["temperature"] > 0:
        pytest.skip("the timed port covers pos_scale 1, greedy")
    tm = TorchCPUModel(OracleConfig(**m["cfg"]), g["weights"], k=m["k"])
    out = tm.generate(g["frames"], m["lens"], m["max_new"], g["bias"], m["max_homopolymer"])
    np.testing.assert_array_equal(out, g["tokens"])


def test_kv_int8_oracle_known_answers():
    """The int8 prefix rule on hand-computed columns: s = max|x| / 127, byte = rint(x * 127 / max) + 128 (half to
    even), an all-zero channel has scale 0 and bytes 128; dequantized attention over an exactly representable
    prefix equals the bf16 attention."""
    from oracle.kv_int8_np import decode_attention, decode_attention_i8, quantize_prefix
    x = np.zeros((3, 128), np.float32)
    x[:, 0] = [-1.0, 0.5, 1.0]
    x[:, 2] = [2.0, -0.01, 0.0]
    u, s = quantize_prefix(x)
    assert u[:, 0].tolist() == [1, 192, 255]
    assert u[:, 1].tolist() == [128, 128, 128] and s[1] == 0
    assert u[:, 2].tolist() == [255, 127, 128]
    assert s[0] == np.float32(1) / np.float32(127) and s[2] == np.float32(2) / np.float32(127)
    rng = np.random.default_rng(0)
    k = rng.integers(-127, 128, (40, 2, 64)).astype(np.float32)
    k[0] = 127.0  # every channel's maximum is 127: the prefix quantizes without error
    v = rng.integers(-127, 128, (40, 2, 64)).astype(np.float32)
    v[0] = -127.0
    q = rng.standard_normal((8, 64)).astype(np.float32) * 0.05
    got, *_ = decode_attention_i8(q, k, v, 30)
    assert np.allclose(got, decode_attention(q, k, v), atol=1e-9)
