"""Drop-in on the model side: the engine reads exactly the checkpoint entries of the reference model.

tests/golden/reference_state_dict.json lists the ``projector.*`` / ``decoder.*`` state-dict names and shapes of
the stock ``viktor.Basecaller`` (recorded from the reference by make_state_dict_map.py, for the single-base and
4-mer vocabularies).  Here, on the CPU: the engine's weight reader accepts that map as it is, and nothing else
(a missing, unexpected or mis-shaped entry is an error), and this package's own ``Basecaller`` carries the same
entries.  tests/test_gpu_engine.py builds an engine from a model assembled from that map alone.
"""

import json
import os

import pytest
import torch

from viktor_b200.config import DecoderConfig, KmerTokenizer
from viktor_b200.fast_decoder import check_state_dict, expected_shapes, model_state

HERE = os.path.dirname(os.path.abspath(__file__))
MAP = json.load(open(os.path.join(HERE, "golden", "reference_state_dict.json")))


def reference_like_model(params, k, weights=None):
    """A model object built from nothing but the reference's state-dict map: nested plain modules named after the
    dotted keys, plus the attributes DecodeEngine reads (decoder.cfg, tokenizer, pos_scale).  Stands in for
    viktor.Basecaller where the reference package is absent."""
    tok = KmerTokenizer(k)
    root = torch.nn.Module()
    for name, shape in params.items():
        mod = root
        *path, leaf = name.split(".")
        for part in path:
            if not hasattr(mod, part):
                mod.add_module(part, torch.nn.Module())
            mod = getattr(mod, part)
        data = torch.zeros(shape) if weights is None else torch.as_tensor(weights[name]).float()
        mod.register_parameter(leaf, torch.nn.Parameter(data, requires_grad=False))
    root.decoder.cfg = DecoderConfig(vocab_size=tok.vocab_size)
    root.tokenizer = tok
    root.pos_scale = 1
    return root


@pytest.mark.parametrize("key,k", [("k1", 1), ("k4", 4)])
def test_reader_accepts_the_reference_map_exactly(key, k):
    m = MAP[key]
    cfg = DecoderConfig(vocab_size=m["vocab_size"])
    check_state_dict(m["params"], cfg)
    assert {n: list(s) for n, s in expected_shapes(cfg).items()} == m["params"]
    assert KmerTokenizer(k).vocab_size == m["vocab_size"]


@pytest.mark.parametrize("key,k", [("k1", 1), ("k4", 4)])
def test_own_model_has_the_reference_entries(key, k):
    from viktor_b200 import Basecaller
    model = Basecaller(KmerTokenizer(k))
    assert {n: list(t.shape) for n, t in model_state(model).items()} == MAP[key]["params"]
    ref_like = reference_like_model(MAP[key]["params"], k)
    assert {n: list(t.shape) for n, t in model_state(ref_like).items()} == MAP[key]["params"]


def test_reader_rejects_a_different_checkpoint():
    m = MAP["k1"]
    cfg = DecoderConfig(vocab_size=7)
    missing = dict(m["params"])
    del missing["decoder.layers.3.down.weight"]
    extra = dict(m["params"], **{"decoder.layers.8.down.weight": [512, 1536]})
    shaped = dict(m["params"], **{"decoder.layers.0.gate_up.weight": [2048, 512]})
    for bad in (missing, extra, shaped):
        with pytest.raises(ValueError):
            check_state_dict(bad, cfg)
