"""Host-side logic on CPU: the packed prefill plan and the tokenizer masks match the reference's definitions
(viktor/engine.py:145-159, :67-68; viktor/tokenizer.py:24-28)."""

import numpy as np
import torch

from viktor_b200.config import KmerTokenizer
from viktor_b200.engine import prefill_plan


def reference_plan(lens, row0, pos_scale):
    """The reference's torch construction, restated on CPU tensors."""
    n = len(lens)
    offsets = [0]
    for length in lens:
        offsets.append(offsets[-1] + length + 1)
    total, frames = offsets[-1], sum(lens)
    cu = torch.tensor(offsets, dtype=torch.int32)
    L = torch.tensor(lens)
    frame_seg = torch.repeat_interleave(torch.arange(n), L, output_size=frames)
    frame_idx = torch.arange(frames) + frame_seg
    last = cu[1:].long() - 1
    pos = (torch.arange(total) - torch.repeat_interleave(cu[:-1].long(), L + 1, output_size=total)).int()
    seq = torch.repeat_interleave(torch.arange(row0, row0 + n, dtype=torch.int32), L + 1, output_size=total)
    rpos = None if pos_scale == 1 else pos * pos_scale
    return cu, frame_idx, last, pos, seq, rpos


def test_prefill_plan_matches_reference():
    for lens, row0, s in [([5, 0, 17, 3], 0, 1), ([2048, 128, 1], 128, 1), ([9, 30], 2, 4)]:
        p = prefill_plan(lens, row0, s)
        cu, fi, last, pos, seq, rpos = reference_plan(lens, row0, s)
        assert np.array_equal(p["cu"], cu.numpy())
        assert np.array_equal(p["frame_idx"], fi.numpy())
        assert np.array_equal(p["last"], last.numpy())
        assert np.array_equal(p["pos"], pos.numpy())
        assert np.array_equal(p["seq"], seq.numpy())
        assert (p["rpos"] is None) == (rpos is None)
        if rpos is not None:
            assert np.array_equal(p["rpos"], rpos.numpy())
        assert p["total"] == int(cu[-1]) and p["max_len"] == max(lens) + 1
        assert np.array_equal(p["lengths"], np.asarray(lens) + 1)


def test_homopolymer_and_tail_masks():
    for k in (1, 4):
        tk = KmerTokenizer(k)
        homo = [i >= 3 and len(t) == tk.k and len(set(t)) == 1 for i, t in enumerate(tk.strings)]
        assert tk.homo_mask.tolist() == homo
        assert tk.tail_mask.sum() == (tk.vocab_size - 3 - 4 ** k)
