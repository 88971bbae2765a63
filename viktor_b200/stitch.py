"""Whole-read assembly of chunk calls (the host side of scripts/basecall_viktor.py and viktor/chunking.py).

Chunking follows viktor/chunking.py:11-24 (chunk_read, repeat_pad).  Adjacent chunk calls overlap by the
encoder frames their signal windows share; each overlap is resolved by aligning the end of chunk i with the start
of chunk i + 1 and cutting both at the middle of the aligned overlap (scripts/basecall_viktor.py:31-108).  The
alignments and the cut search run in the native library (vk_align / vk_overlap_cut / vk_stitch, an edit-distance
aligner with edlib's semantics); the Python functions here keep the reference's names and arguments.
"""

from __future__ import annotations

import ctypes as C
import re

import numpy as np

from ._lib import call

STRIDE = 6  # samples per encoder frame (scripts/basecall_crf.py:30)
ADAPTER = "CCTGTACTTCGTTCAGTTACGTATTGCT"  # ligation adapter consensus (scripts/make_head_labels.py:34)
NW, SHW, HW = 0, 1, 2


def chunk_read(n, size, overlap):
    """(start, end) sample spans of a read of n samples: windows of `size` stepping by size - overlap, the
    remainder as a short last chunk (viktor/chunking.py:11-18)."""
    out, off = [], 0
    while off + size < n:
        out.append((off, off + size))
        off += size - overlap
    if off != n:
        out.append((off, n))
    return out


def repeat_pad(x, unit):
    """Pads x to a multiple of unit by repeating its head (viktor/chunking.py:21-24)."""
    while len(x) % unit:
        x = np.concatenate([x, x[:unit - len(x) % unit]])
    return x


def align(query: str, target: str, mode: int = NW, k: int = -1, path: bool = False):
    """Edit distance of query against target (NW global, SHW prefix, HW infix); k >= 0 caps it (-1 above).
    Returns dict(editDistance, locations=[(start, end)], cigar) shaped like the edlib results the reference
    reads."""
    q, t = query.encode(), target.encode()
    out = (C.c_int * 3)()
    cig = C.create_string_buffer(len(q) + len(t) + 1) if path else None
    call("vk_align", q, len(q), t, len(t), mode, k, out, cig, len(q) + len(t) + 1 if path else 0)
    d = out[0]
    return {"editDistance": d, "locations": [(out[1], out[2])] if d >= 0 else [],
            "cigar": cig.value.decode() if path and d >= 0 else None}


def overlap_cut(a: str, b: str, ov_frames: int, rate: float):
    """scripts/basecall_viktor.py:31-54: (cut_a, cut_b), keep a[:cut_a] + b[cut_b:]."""
    cut = (C.c_int * 2)()
    ab, bb = a.encode(), b.encode()
    call("vk_overlap_cut", ab, len(ab), bb, len(bb), int(ov_frames), float(rate), cut)
    return cut[0], cut[1]


def stitch(calls, spans, n_samples=None, overlap=None):
    """scripts/basecall_viktor.py:96-108: the read's sequence from its chunk calls and their sample spans."""
    raw = [c.encode() for c in calls]
    offsets = np.concatenate([[0], np.cumsum([len(r) for r in raw])]).astype(np.int64)
    sp = np.ascontiguousarray(np.asarray(spans, dtype=np.int64).reshape(len(raw), 2))
    cap = int(offsets[-1])
    buf = C.create_string_buffer(max(cap, 1))
    n_out = C.c_int64(0)
    call("vk_stitch", b"".join(raw), offsets.ctypes.data, sp.ctypes.data, len(raw), STRIDE, buf, cap,
         C.byref(n_out))
    return buf.raw[:n_out.value].decode()


def trim_adapter(seq: str, max_ed: int = 8, head: int = 120) -> str:
    """Cuts the ligation adapter (and anything before it) off the read start (scripts/basecall_viktor.py:73-77);
    no match within max_ed edits: the read is left as called."""
    r = align(ADAPTER, seq[:head], HW, max_ed)
    return seq[r["locations"][0][1] + 1:] if r["editDistance"] >= 0 else seq


def cap_homopolymers(seq: str, max_run: int, keep: int = 20) -> str:
    """Shortens every run of >= max_run identical bases to keep (scripts/basecall_viktor.py:80-83)."""
    return re.sub(rf"(.)\1{{{max_run - 1},}}", lambda m: m.group(1) * keep, seq)
