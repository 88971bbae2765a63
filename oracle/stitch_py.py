"""CPU oracle of the whole-read stitching (scripts/basecall_viktor.py:31-108, viktor/chunking.py:11-18).

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` to check the native stitching in ``viktor_b200``.

The reference resolves chunk overlaps with edlib (an unpinned dependency of the reference, not vendored and not
installed here).  ``align`` restates edlib's published semantics in pure Python over the full dynamic-programming
matrix (small inputs only): NW / SHW / HW modes with unit costs, a distance cap k, the first best end location
(the HW start being the smallest one that reaches the best distance there: the longest alignment), and the
alignment path as extended CIGAR operations traced back from the end preferring I, then D, then the diagonal.
Parity unpinned: without edlib here, equal-cost alignments may place an indel differently from edlib, which
can move a cut by a base; the functions above the aligner follow the reference line by line.
"""

from __future__ import annotations

NW, SHW, HW = 0, 1, 2
STRIDE = 6


def _matrix(q, t, free_start):
    n = len(t)
    D = [[0] * (n + 1) for _ in range(len(q) + 1)]
    D[0] = [0 if free_start else j for j in range(n + 1)]
    for i in range(1, len(q) + 1):
        row, up = D[i], D[i - 1]
        row[0] = i
        for j in range(1, n + 1):
            row[j] = min(up[j - 1] + (q[i - 1] != t[j - 1]), up[j] + 1, row[j - 1] + 1)
    return D


def align(q, t, mode=NW, k=-1, path=False):
    """edlib.align(q, t, mode, task="path" if path else "locations", k) as the reference reads it:
    dict(editDistance, locations=[(start, end)], cigar)."""
    D = _matrix(q, t, mode == HW)
    last, n = D[len(q)], len(t)
    if mode == NW:
        best, end = last[n], n - 1
    else:
        best, end = last[0], -1
        if n:
            bj = min(range(1, n + 1), key=lambda j: (last[j], j))
            if last[bj] <= best:
                best, end = last[bj], bj - 1
    if k >= 0 and best > k:
        return {"editDistance": -1, "locations": [], "cigar": None}
    start = 0
    if mode == HW and end >= 0:
        R = _matrix(q[::-1], t[:end + 1][::-1], False)
        jmax = max([j for j in range(end + 2) if R[len(q)][j] == best], default=0)
        start = end + 1 - jmax
    cigar = None
    if path:
        sub = t[start:end + 1]
        P = _matrix(q, sub, False)
        i, j, ops = len(q), len(sub), []
        while i > 0 or j > 0:
            cur = P[i][j]
            if i > 0 and P[i - 1][j] + 1 == cur:
                ops.append("I")
                i -= 1
            elif j > 0 and P[i][j - 1] + 1 == cur:
                ops.append("D")
                j -= 1
            else:
                ops.append("=" if q[i - 1] == sub[j - 1] else "X")
                i -= 1
                j -= 1
        cigar = "".join(reversed(ops))
    return {"editDistance": best, "locations": [(start, end)], "cigar": cigar}


def _mid_cut(a, b, p):
    """scripts/basecall_viktor.py:57-70."""
    q = a[p:]
    r = align(q, b[:int(len(q) * 1.4) + 16], SHW, max(len(q) // 3, 4), path=True)
    if r["editDistance"] < 0:
        return None
    half, ia, ib = len(q) // 2, 0, 0
    for op in r["cigar"]:
        if ia >= half and op in "=X":
            return p + ia, ib
        ia += op in "=XI"
        ib += op in "=XD"
    return p + half, ib


def overlap_cut(a, b, ov_frames, rate):
    """scripts/basecall_viktor.py:31-54."""
    if len(a) < 8 or len(b) < 8:
        return len(a), 0
    est = max(int(ov_frames * rate), 4)
    n_tail = min(len(a), int(est * 1.6) + 16)
    m = min(len(b), max(int(est * 0.5), 8))
    if n_tail >= m:
        r = align(b[:m], a[len(a) - n_tail:], HW, m // 3)
        if r["editDistance"] >= 0:
            cut = _mid_cut(a, b, len(a) - n_tail + r["locations"][0][0])
            if cut:
                return cut
    best = None
    for L in range(min(n_tail, len(b)), 9, -1):
        ed = align(a[-L:], b[:L], NW)["editDistance"]
        if ed <= L // 5 and (best is None or L - 4 * ed > best[0]):
            best = (L - 4 * ed, L)
    cut = best and _mid_cut(a, b, len(a) - best[1])
    return cut or (len(a), 0)


def stitch(calls, spans):
    """scripts/basecall_viktor.py:96-108."""
    out, cut_a_prev = [], 0
    for i, s in enumerate(calls):
        if i + 1 < len(calls):
            ov = (spans[i][1] - spans[i + 1][0]) // STRIDE
            rate = len(s) / max((spans[i][1] - spans[i][0]) // STRIDE, 1)
            ca, cb = overlap_cut(s, calls[i + 1], ov, rate)
            out.append(s[cut_a_prev:ca])
            cut_a_prev = cb
        else:
            out.append(s[cut_a_prev:])
    return "".join(out)


def chunk_read(n, size, overlap):
    """viktor/chunking.py:11-18."""
    out, off = [], 0
    while off + size < n:
        out.append((off, off + size))
        off += size - overlap
    if off != n:
        out.append((off, n))
    return out
