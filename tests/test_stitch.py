"""Host-side stitching (native vk_align / vk_overlap_cut / vk_stitch) against the pure-Python restatement in
oracle/stitch_py.py: exact equality of distances, locations, CIGAR paths, cuts and stitched reads; error-free
overlapping chunk calls stitch back to the read."""

import numpy as np
import pytest

from oracle import stitch_py as ref

BASES = np.array(list("ACGT"))


def _rand_seq(rng, n):
    return "".join(rng.choice(BASES, n))


def _mutate(rng, s, rate):
    out = []
    for ch in s:
        u = rng.random()
        if u < rate / 3:
            continue  # deletion
        if u < 2 * rate / 3:
            out.append(rng.choice(BASES))  # substitution
        elif u < rate:
            out.append(ch + rng.choice(BASES))  # insertion
        else:
            out.append(ch)
    return "".join(out)


def test_align_known_answers():
    from viktor_b200.stitch import HW, NW, SHW, align
    assert align("kitten", "sitting")["editDistance"] == 3
    r = align("GT", "AAGTAA", HW, path=True)
    assert r["editDistance"] == 0 and r["locations"] == [(2, 3)] and r["cigar"] == "=="
    assert align("AAAA", "TTTT", NW, 2)["editDistance"] == -1
    r = align("ACGT", "ACGTTTT", SHW, path=True)
    assert r["editDistance"] == 0 and r["locations"] == [(0, 3)] and r["cigar"] == "===="
    r = align("ACGAT", "TTACGTTT", HW, path=True)  # one deletion from the query: ACG-T
    assert r["editDistance"] == 1 and r["cigar"].count("I") == 1


def test_align_matches_oracle():
    from viktor_b200.stitch import align
    rng = np.random.default_rng(0)
    for _ in range(400):
        q = _rand_seq(rng, int(rng.integers(0, 25)))
        t = _mutate(rng, q, 0.3) if rng.random() < 0.7 else _rand_seq(rng, int(rng.integers(0, 30)))
        if rng.random() < 0.5:
            t = _rand_seq(rng, int(rng.integers(0, 6))) + t + _rand_seq(rng, int(rng.integers(0, 6)))
        mode = int(rng.integers(0, 3))
        k = int(rng.choice([-1, 2, 5]))
        got = align(q, t, mode, k, path=True)
        exp = ref.align(q, t, mode, k, path=True)
        assert got == exp, (q, t, mode, k, got, exp)


def test_align_distances_match_an_independent_matcher():
    """Edit distances of all three modes against the `regex` package's fuzzy matching (its own implementation,
    not derived from this code base or the oracle): the least k for which the query matches with at most k
    errors, anchored at both ends (NW), at the start (SHW) or anywhere (HW).  Distances up to 6 only: the fuzzy
    search grows exponentially in k."""
    regex = pytest.importorskip("regex")
    from viktor_b200.stitch import HW, NW, SHW, align

    def least_k(q, t, mode, kmax=6):
        find = {NW: regex.fullmatch, SHW: regex.match, HW: regex.search}[mode]
        for k in range(kmax + 1):
            if find("(?:%s){e<=%d}" % (q, k), t, timeout=5.0) is not None:
                return k
        return None

    rng = np.random.default_rng(1)
    checked = 0
    for _ in range(300):
        q = _rand_seq(rng, int(rng.integers(4, 24)))
        core = _mutate(rng, q, 0.15)
        for mode in (NW, SHW, HW):
            t = core
            if mode == SHW:
                t = core + _rand_seq(rng, int(rng.integers(0, 8)))
            elif mode == HW:
                t = _rand_seq(rng, int(rng.integers(0, 8))) + core + _rand_seq(rng, int(rng.integers(0, 8)))
            exp = least_k(q, t, mode)
            if exp is None:
                continue
            assert align(q, t, mode)["editDistance"] == exp, (q, t, mode)
            checked += 1
    assert checked > 800


def test_overlap_cut_matches_oracle():
    from viktor_b200.stitch import overlap_cut
    rng = np.random.default_rng(1)
    for i in range(60):
        read = _rand_seq(rng, 400)
        ov = int(rng.integers(20, 120))
        a = _mutate(rng, read[:250], 0.04 if i % 3 else 0.0)
        b = _mutate(rng, read[250 - ov:], 0.04 if i % 3 else 0.0)
        if i % 10 == 9:
            b = _rand_seq(rng, 150)  # no overlap at all: both kept whole
        frames, rate = ov // 2, 2.0 * float(rng.uniform(0.8, 1.2))
        assert overlap_cut(a, b, frames, rate) == ref.overlap_cut(a, b, frames, rate), i
    assert overlap_cut("ACGT", "ACGTACGTAC", 10, 1.0) == (4, 0)  # a chunk under 8 bases is kept whole


@pytest.mark.parametrize("errors", [0.0, 0.03])
def test_stitch_read(errors):
    """A read of 30000 samples at one base per 9 samples, cut into the reference's 12288-sample chunks with a
    600-sample overlap; each chunk call is the read's bases under its span (with sequencing errors or not)."""
    from viktor_b200.stitch import chunk_read, stitch
    rng = np.random.default_rng(2)
    n_samples, spb = 30000, 9
    read = _rand_seq(rng, n_samples // spb)
    spans = chunk_read(n_samples, 12288, 600)
    assert spans == ref.chunk_read(n_samples, 12288, 600) and len(spans) == 3
    calls = [_mutate(rng, read[a // spb:b // spb], errors) for a, b in spans]
    got = stitch(calls, spans, n_samples, 600)
    assert got == ref.stitch(calls, spans)
    if errors == 0.0:
        assert got == read
    else:
        d = ref.align(got[:400], read[:420], ref.SHW)["editDistance"]
        assert d <= 0.1 * 400


def test_trim_and_cap():
    from viktor_b200.stitch import ADAPTER, cap_homopolymers, trim_adapter
    tail = "ACGTTGCA" * 10
    assert trim_adapter("GG" + ADAPTER + tail) == tail
    assert trim_adapter(tail) == tail
    assert cap_homopolymers("C" + "A" * 70 + "G", 60) == "C" + "A" * 20 + "G"
    assert cap_homopolymers("A" * 59, 60) == "A" * 59
