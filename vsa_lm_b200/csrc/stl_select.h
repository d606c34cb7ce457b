// Exact emulation of the CPU `torch.topk` result order (host + device).
//
// The reference ranks candidates with `torch.topk` on CPU tensors (vsa_lm/config/bolt3.py:133-134
// and :183). Among exactly equal values the order it returns is whatever its selection algorithm
// leaves behind: PyTorch's CPU top-k copies (value, index) pairs into a buffer and runs the C++
// standard library's selection on it — `partial_sort(first, first + k, last)` when k * 64 <= n,
// otherwise `nth_element(first, first + k - 1, last)` followed by `sort(first, first + k - 1)` —
// with a "NaN first, then strictly greater/less" comparator. Equal keys make the exact tie order a
// function of those algorithms' steps (GNU libstdc++'s introselect / introsort / heap routines).
//
// This header re-implements those published algorithms step for step so that ties come out in the
// same order, which matters for Bolt-3: at the first full-bank consolidation many attractor slots
// carry identical `keep` scores (equal utility, mutual nearest neighbours), and which slot is
// evicted first changes all later state. The CUDA kernels only call it when their counting-rank
// sort finds exactly equal values at a position that decides the result; the CPU test
// `test_topk_tie_order` checks it against `torch.topk`.
//
// All routines are iterative (no recursion) and every loop index is bounds-checked: an index that
// would leave [0, n) sets `*bad = 1` and the routine returns early instead of reading out of range.
#pragma once

#ifdef __CUDACC__
#define B3_HD __host__ __device__ __forceinline__
#else
#define B3_HD inline
#endif

namespace b3sel {

struct KV {
  float v;
  int i;
};

// "largest": NaN ranks first, then strictly greater. "smallest": NaN ranks last, then strictly less.
struct Cmp {
  bool largest;
  B3_HD bool operator()(const KV& a, const KV& b) const {
    const bool an = a.v != a.v, bn = b.v != b.v;
    if (largest) return (an && !bn) || (a.v > b.v);
    return (!an && bn) || (a.v < b.v);
  }
};

struct Ctx {
  KV* a;      // the buffer, positions [0, n)
  int n;
  int* bad;   // set to 1 on an out-of-range index
  Cmp comp;
  B3_HD bool ok(long p) const {
    if (p < 0 || p >= n) { *bad = 1; return false; }
    return true;
  }
  B3_HD void swap(long p, long q) {
    KV t = a[p]; a[p] = a[q]; a[q] = t;
  }
};

B3_HD int floor_log2(long n) {
  int k = 0;
  while (n > 1) { n >>= 1; ++k; }
  return k;
}

// Place the median of positions pa, pb, pc at position res.
B3_HD void median_to_first(Ctx& c, long res, long pa, long pb, long pc) {
  const KV& A = c.a[pa]; const KV& B = c.a[pb]; const KV& C = c.a[pc];
  if (c.comp(A, B)) {
    if (c.comp(B, C)) c.swap(res, pb);
    else if (c.comp(A, C)) c.swap(res, pc);
    else c.swap(res, pa);
  } else if (c.comp(A, C)) c.swap(res, pa);
  else if (c.comp(B, C)) c.swap(res, pc);
  else c.swap(res, pb);
}

// Hoare-style partition of [first, last) around the pivot at position `pivot` (outside the range).
B3_HD long partition(Ctx& c, long first, long last, long pivot) {
  for (int guard = 0; guard < 4 * c.n + 8; ++guard) {
    while (c.ok(first) && c.comp(c.a[first], c.a[pivot])) ++first;
    if (*c.bad) return first;
    --last;
    while (c.ok(last) && c.comp(c.a[pivot], c.a[last])) --last;
    if (*c.bad) return first;
    if (!(first < last)) return first;
    c.swap(first, last);
    ++first;
  }
  *c.bad = 1;
  return first;
}

B3_HD long partition_pivot(Ctx& c, long first, long last) {
  const long mid = first + (last - first) / 2;
  median_to_first(c, first, first + 1, mid, last - 1);
  return partition(c, first + 1, last, first);
}

// ---- heap routines (max-heap w.r.t. comp) on the sub-array starting at `base`
B3_HD void push_up(Ctx& c, long base, long hole, long top, KV val) {
  long parent = (hole - 1) / 2;
  while (hole > top && c.comp(c.a[base + parent], val)) {
    c.a[base + hole] = c.a[base + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  c.a[base + hole] = val;
}

B3_HD void adjust(Ctx& c, long base, long hole, long len, KV val) {
  const long top = hole;
  long child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (c.comp(c.a[base + child], c.a[base + child - 1])) child--;
    c.a[base + hole] = c.a[base + child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    c.a[base + hole] = c.a[base + child - 1];
    hole = child - 1;
  }
  push_up(c, base, hole, top, val);
}

B3_HD void make_heap(Ctx& c, long first, long last) {
  const long len = last - first;
  if (len < 2) return;
  long parent = (len - 2) / 2;
  while (true) {
    KV val = c.a[first + parent];
    adjust(c, first, parent, len, val);
    if (parent == 0) return;
    parent--;
  }
}

// Move the heap top of [first, last) to `result`, re-heapify with the old value of `result`.
B3_HD void pop_to(Ctx& c, long first, long last, long result) {
  KV val = c.a[result];
  c.a[result] = c.a[first];
  adjust(c, first, 0, last - first, val);
}

B3_HD void heap_select(Ctx& c, long first, long middle, long last) {
  make_heap(c, first, middle);
  for (long i = middle; i < last; ++i)
    if (c.comp(c.a[i], c.a[first])) pop_to(c, first, middle, i);
}

B3_HD void sort_heap(Ctx& c, long first, long last) {
  while (last - first > 1) {
    --last;
    pop_to(c, first, last, last);
  }
}

B3_HD void partial_sort(Ctx& c, long first, long middle, long last) {
  heap_select(c, first, middle, last);
  sort_heap(c, first, middle);
}

// ---- insertion sorts
// Shift `a[last]` left past every element it ranks before. The walk never goes below `lo`; reaching
// position -1 means the unguarded original would have read before the array, which is flagged.
B3_HD void linear_insert(Ctx& c, long last, long lo) {
  KV val = c.a[last];
  long next = last - 1;
  while (true) {
    if (next < lo) {
      if (next < 0) *c.bad = 1;
      break;
    }
    if (!c.comp(val, c.a[next])) break;
    c.a[last] = c.a[next];
    last = next;
    --next;
  }
  c.a[last] = val;
}

B3_HD void insertion_sort(Ctx& c, long first, long last) {
  if (first == last) return;
  for (long i = first + 1; i < last; ++i) {
    if (c.comp(c.a[i], c.a[first])) {
      KV val = c.a[i];
      for (long p = i; p > first; --p) c.a[p] = c.a[p - 1];
      c.a[first] = val;
    } else {
      linear_insert(c, i, first);
    }
  }
}

// The "unguarded" variant relies on a smaller element somewhere before `first`; the walk is
// bounded by 0 here and flags a violation instead of running off the array.
B3_HD void unguarded_insertion_sort(Ctx& c, long first, long last) {
  for (long i = first; i < last; ++i) linear_insert(c, i, 0);
}

B3_HD void final_insertion_sort(Ctx& c, long first, long last) {
  if (last - first > 16) {
    insertion_sort(c, first, first + 16);
    unguarded_insertion_sort(c, first + 16, last);
  } else {
    insertion_sort(c, first, last);
  }
}

// introsort loop with an explicit stack (the right part of each split is an independent range)
B3_HD void introsort_loop(Ctx& c, long first, long last, int depth) {
  // depth <= 2*log2(n) splits are pending at once; 40 covers n < 2^20
  int st_f[40], st_l[40];
  int st_d[40];
  int sp = 0;
  st_f[sp] = (int)first; st_l[sp] = (int)last; st_d[sp] = depth; ++sp;
  while (sp > 0 && !*c.bad) {
    --sp;
    long f = st_f[sp], l = st_l[sp];
    int d = st_d[sp];
    while (l - f > 16 && !*c.bad) {
      if (d == 0) {
        partial_sort(c, f, l, l);
        break;
      }
      --d;
      const long cut = partition_pivot(c, f, l);
      if (sp >= 40) { *c.bad = 1; return; }
      st_f[sp] = (int)cut; st_l[sp] = (int)l; st_d[sp] = d; ++sp;
      l = cut;
    }
  }
}

B3_HD void std_sort(Ctx& c, long first, long last) {
  if (first == last) return;
  introsort_loop(c, first, last, floor_log2(last - first) * 2);
  if (!*c.bad) final_insertion_sort(c, first, last);
}

B3_HD void nth_element(Ctx& c, long first, long nth, long last) {
  if (first == last || nth == last) return;
  int depth = floor_log2(last - first) * 2;
  while (last - first > 3 && !*c.bad) {
    if (depth == 0) {
      heap_select(c, first, nth + 1, last);
      c.swap(first, nth);
      return;
    }
    --depth;
    const long cut = partition_pivot(c, first, last);
    if (cut <= nth) first = cut;
    else last = cut;
  }
  insertion_sort(c, first, last);
}

// Reorder buf[0, n) so that buf[0, k) holds the top-k in the order CPU torch.topk(sorted=True)
// returns them. Returns 0 on success, 1 if a bounds check fired.
B3_HD int topk_order(KV* buf, int n, int k, bool largest) {
  int bad = 0;
  if (k <= 0 || n <= 0) return 0;
  Ctx c{buf, n, &bad, Cmp{largest}};
  if ((long)k * 64 <= n) {
    partial_sort(c, 0, k, n);
  } else {
    nth_element(c, 0, k - 1, n);
    if (!bad) std_sort(c, 0, k - 1);
  }
  return bad;
}

}  // namespace b3sel
