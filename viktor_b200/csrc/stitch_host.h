// Host-side assembly of chunk calls into read calls: the overlap resolution of scripts/basecall_viktor.py:31-108
// (overlap_cut, _mid_cut, stitch, trim_adapter) and the edit-distance alignments it asks of edlib (an unpinned
// Python dependency of the reference, not vendored).  The aligner restates edlib's published semantics
// (Sosic & Sikic, Bioinformatics 33(9), 2017) on a plain dynamic-programming matrix (the overlaps are a few
// hundred bases, so O(m n) per alignment is microseconds):
//  * modes: NW global; SHW the whole query against a prefix of the target; HW the whole query against any
//    infix of the target; unit costs for mismatch, insertion and deletion;
//  * k >= 0: a best distance above k is reported as -1;
//  * locations: the first (smallest) end position reaching the best distance; in HW mode its start is the
//    smallest one reaching the best distance at that end (the longest alignment); SHW starts at 0;
//  * path: the alignment of the query with target[start..end], as extended CIGAR operations ('=' match,
//    'X' mismatch, 'I' a query base absent from the target, 'D' a target base absent from the query), traced
//    back from the end cell preferring I, then D, then the diagonal.
#pragma once

#include <stdint.h>

#include <algorithm>
#include <string>
#include <vector>

namespace vk {
namespace stitch {

enum { kNW = 0, kSHW = 1, kHW = 2 };

struct Alignment {
  int dist = -1;  // -1: above k
  int start = 0;
  int end = -1;
  std::string ops;
};

// D[i][j] (row-major, n + 1 columns): cost of query[0, i) against target[., j); row 0 is 0 (free target start)
// or j.
inline void fill_matrix(const char* q, int m, const char* t, int n, bool free_start, std::vector<int>& D) {
  const size_t w = static_cast<size_t>(n) + 1;
  D.assign((static_cast<size_t>(m) + 1) * w, 0);
  for (int j = 0; j <= n; ++j) D[j] = free_start ? 0 : j;
  for (int i = 1; i <= m; ++i) {
    int* row = &D[i * w];
    const int* up = row - w;
    row[0] = i;
    const char qc = q[i - 1];
    for (int j = 1; j <= n; ++j)
      row[j] = std::min(up[j - 1] + (qc == t[j - 1] ? 0 : 1), std::min(up[j], row[j - 1]) + 1);
  }
}

// Global edit distance (two rows).
inline int nw_distance(const char* q, int m, const char* t, int n) {
  std::vector<int> a(n + 1), b(n + 1);
  for (int j = 0; j <= n; ++j) a[j] = j;
  for (int i = 1; i <= m; ++i) {
    b[0] = i;
    const char qc = q[i - 1];
    for (int j = 1; j <= n; ++j) b[j] = std::min(a[j - 1] + (qc == t[j - 1] ? 0 : 1), std::min(a[j], b[j - 1]) + 1);
    std::swap(a, b);
  }
  return a[n];
}

inline Alignment align(const char* q, int m, const char* t, int n, int mode, int k, bool path) {
  Alignment r;
  std::vector<int> D;
  fill_matrix(q, m, t, n, mode == kHW, D);
  const size_t w = static_cast<size_t>(n) + 1;
  const int* last = &D[static_cast<size_t>(m) * w];
  int best, end;
  if (mode == kNW) {
    best = last[n];
    end = n - 1;
  } else {  // first end j - 1 with the best distance; j = 0 (no target base used) only when strictly better
    best = last[0];
    end = -1;
    if (n > 0) {
      int bj = 1;
      for (int j = 2; j <= n; ++j)
        if (last[j] < last[bj]) bj = j;
      if (last[bj] <= best) {
        best = last[bj];
        end = bj - 1;
      }
    }
  }
  if (k >= 0 && best > k) return r;
  r.dist = best;
  r.end = end;
  r.start = 0;
  if (mode == kHW && end >= 0) {
    // smallest start reaching `best` at this end: the reversed query against target[end], target[end - 1], ...
    // with the start fixed (SHW), the largest reversed end with that distance
    std::string rq(q, q + m), rt(t, t + end + 1);
    std::reverse(rq.begin(), rq.end());
    std::reverse(rt.begin(), rt.end());
    std::vector<int> R;
    fill_matrix(rq.data(), m, rt.data(), end + 1, false, R);
    const int* rl = &R[static_cast<size_t>(m) * (end + 2)];
    int jmax = 0;
    for (int j = 1; j <= end + 1; ++j)
      if (rl[j] == best) jmax = j;
    r.start = end + 1 - jmax;
  }
  if (path) {
    const int s = r.start, len = r.end + 1 - r.start > 0 ? r.end + 1 - r.start : 0;
    std::vector<int> P;
    fill_matrix(q, m, t + s, len, false, P);
    const size_t pw = static_cast<size_t>(len) + 1;
    int i = m, j = len;
    while (i > 0 || j > 0) {
      const int cur = P[i * pw + j];
      if (i > 0 && P[(i - 1) * pw + j] + 1 == cur) {
        r.ops.push_back('I');
        --i;
      } else if (j > 0 && P[i * pw + j - 1] + 1 == cur) {
        r.ops.push_back('D');
        --j;
      } else {
        r.ops.push_back(q[i - 1] == t[s + j - 1] ? '=' : 'X');
        --i;
        --j;
      }
    }
    std::reverse(r.ops.begin(), r.ops.end());
  }
  return r;
}

struct Cut {
  bool ok;
  int a, b;
};

// scripts/basecall_viktor.py:57-70 _mid_cut: a[p:] overlaps the head of b; cut both at the middle of their
// alignment.
inline Cut mid_cut(const std::string& a, const std::string& b, int p) {
  const std::string q = a.substr(p);
  const int lq = static_cast<int>(q.size());
  const int tl = std::min(static_cast<int>(b.size()), static_cast<int>(lq * 1.4) + 16);
  const Alignment r = align(q.data(), lq, b.data(), tl, kSHW, std::max(lq / 3, 4), true);
  if (r.dist < 0) return Cut{false, 0, 0};
  const int half = lq / 2;
  int ia = 0, ib = 0;
  for (char op : r.ops) {
    if (ia >= half && (op == '=' || op == 'X')) return Cut{true, p + ia, ib};
    ia += (op == '=' || op == 'X' || op == 'I');
    ib += (op == '=' || op == 'X' || op == 'D');
  }
  return Cut{true, p + half, ib};
}

// scripts/basecall_viktor.py:31-54 overlap_cut: keep a[:cut.a] + b[cut.b:].
inline Cut overlap_cut(const std::string& a, const std::string& b, int ov_frames, double rate) {
  const int la = static_cast<int>(a.size()), lb = static_cast<int>(b.size());
  if (la < 8 || lb < 8) return Cut{true, la, 0};
  const int est = std::max(static_cast<int>(ov_frames * rate), 4);
  const int n_tail = std::min(la, static_cast<int>(est * 1.6) + 16);
  const int m = std::min(lb, std::max(static_cast<int>(est * 0.5), 8));
  if (n_tail >= m) {
    const Alignment r = align(b.data(), m, a.data() + la - n_tail, n_tail, kHW, m / 3, false);
    if (r.dist >= 0) {
      const Cut c = mid_cut(a, b, la - n_tail + r.start);  // a[p] aligns with b[0]
      if (c.ok) return c;
    }
  }
  // suffix(a) ~ prefix(b), at most one edit per 5 bases, score L - 4 x edits
  bool have = false;
  int best_score = 0, best_len = 0;
  for (int L = std::min(n_tail, lb); L > 9; --L) {
    const int ed = nw_distance(a.data() + la - L, L, b.data(), L);
    if (ed <= L / 5 && (!have || L - 4 * ed > best_score)) {
      have = true;
      best_score = L - 4 * ed;
      best_len = L;
    }
  }
  if (have) {
    const Cut c = mid_cut(a, b, la - best_len);
    if (c.ok) return c;
  }
  return Cut{true, la, 0};
}

inline int64_t floor_div(int64_t x, int64_t y) {
  int64_t q = x / y;
  if ((x % y != 0) && ((x < 0) != (y < 0))) --q;
  return q;
}

// Python slice s[lo:hi] for 0 <= lo, hi.
inline std::string py_slice(const std::string& s, int64_t lo, int64_t hi) {
  const int64_t n = static_cast<int64_t>(s.size());
  lo = std::min(lo, n);
  hi = std::min(hi, n);
  return hi > lo ? s.substr(lo, hi - lo) : std::string();
}

}  // namespace stitch
}  // namespace vk
