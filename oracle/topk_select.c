/*
 * CPU restatement of torch's CPU top-k order (TEST INFRASTRUCTURE ONLY).
 *
 * torch.topk on CPU (the op the reference's router calls, muserve/model/qwen35_layer_v2.py:570)
 * fills (value, index) pairs and runs, with a "greater, NaN first" comparator on the value:
 *   k*64 <= n : std::partial_sort(first, first+k, last)
 *   otherwise : std::nth_element(first, first+k-1, last); std::sort(first, first+k-1)
 * The order of tied values is whatever libstdc++'s algorithms leave.  This file restates those
 * published algorithms (libstdc++ bits/stl_algo.h, bits/stl_heap.h: __introselect with
 * median-of-three pivot and unguarded partition, __insertion_sort, __heap_select,
 * __sort_heap, __adjust_heap, __push_heap) step by step, so tests can pin the CUDA router's
 * replay against torch on the CPU.  Single-threaded, plain C.
 */
#include <math.h>
#include <stdint.h>

typedef struct { float v; int32_t i; } pair_t;

static int gt(float x, float y) { return (isnan(x) && !isnan(y)) || x > y; }
static void swp(pair_t* a, int x, int y) { pair_t t = a[x]; a[x] = a[y]; a[y] = t; }

static void insertion_sort(pair_t* a, int f, int l) {
  if (f == l) return;
  for (int i = f + 1; i < l; ++i) {
    pair_t val = a[i];
    if (gt(val.v, a[f].v)) {
      for (int j = i; j > f; --j) a[j] = a[j - 1];
      a[f] = val;
    } else {
      int j = i, n = i - 1;
      while (gt(val.v, a[n].v)) { a[j] = a[n]; j = n; --n; }
      a[j] = val;
    }
  }
}

static void move_median_to_first(pair_t* a, int r, int x, int y, int z) {
  if (gt(a[x].v, a[y].v)) {
    if (gt(a[y].v, a[z].v)) swp(a, r, y);
    else if (gt(a[x].v, a[z].v)) swp(a, r, z);
    else swp(a, r, x);
  } else if (gt(a[x].v, a[z].v)) swp(a, r, x);
  else if (gt(a[y].v, a[z].v)) swp(a, r, z);
  else swp(a, r, y);
}

static int unguarded_partition(pair_t* a, int f, int l, int p) {
  for (;;) {
    while (gt(a[f].v, a[p].v)) ++f;
    --l;
    while (gt(a[p].v, a[l].v)) --l;
    if (!(f < l)) return f;
    swp(a, f, l);
    ++f;
  }
}

static void push_heap(pair_t* a, int base, int hole, int top, pair_t val) {
  int parent = (hole - 1) / 2;
  while (hole > top && gt(a[base + parent].v, val.v)) {
    a[base + hole] = a[base + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a[base + hole] = val;
}

static void adjust_heap(pair_t* a, int base, int hole, int len, pair_t val) {
  const int top = hole;
  int sc = hole;
  while (sc < (len - 1) / 2) {
    sc = 2 * (sc + 1);
    if (gt(a[base + sc].v, a[base + sc - 1].v)) sc--;
    a[base + hole] = a[base + sc];
    hole = sc;
  }
  if ((len & 1) == 0 && sc == (len - 2) / 2) {
    sc = 2 * (sc + 1);
    a[base + hole] = a[base + sc - 1];
    hole = sc - 1;
  }
  push_heap(a, base, hole, top, val);
}

static void make_heap(pair_t* a, int f, int l) {
  int len = l - f;
  if (len < 2) return;
  for (int parent = (len - 2) / 2;; --parent) {
    adjust_heap(a, f, parent, len, a[f + parent]);
    if (parent == 0) return;
  }
}

static void pop_heap(pair_t* a, int f, int l, int r) {
  pair_t val = a[r];
  a[r] = a[f];
  adjust_heap(a, f, 0, l - f, val);
}

static void heap_select(pair_t* a, int f, int m, int l) {
  make_heap(a, f, m);
  for (int i = m; i < l; ++i)
    if (gt(a[i].v, a[f].v)) pop_heap(a, f, m, i);
}

static void sort_heap(pair_t* a, int f, int l) {
  while (l - f > 1) { --l; pop_heap(a, f, l, l); }
}

static int lg2(int n) { int r = 0; while (n >>= 1) ++r; return r; }

static void introselect(pair_t* a, int f, int nth, int l, int depth) {
  while (l - f > 3) {
    if (depth == 0) { heap_select(a, f, nth + 1, l); swp(a, f, nth); return; }
    --depth;
    int mid = f + (l - f) / 2;
    move_median_to_first(a, f, f + 1, mid, l - 1);
    int cut = unguarded_partition(a, f + 1, l, f);
    if (cut <= nth) f = cut; else l = cut;
  }
  insertion_sort(a, f, l);
}

static void introsort_loop(pair_t* a, int f, int l, int depth) {
  while (l - f > 16) {
    if (depth == 0) { heap_select(a, f, l, l); sort_heap(a, f, l); return; }
    --depth;
    int mid = f + (l - f) / 2;
    move_median_to_first(a, f, f + 1, mid, l - 1);
    int cut = unguarded_partition(a, f + 1, l, f);
    introsort_loop(a, cut, l, depth);
    l = cut;
  }
}

static void std_sort(pair_t* a, int f, int l) {
  if (l - f < 2) return;
  introsort_loop(a, f, l, 2 * lg2(l - f));
  if (l - f > 16) {
    insertion_sort(a, f, f + 16);
    for (int i = f + 16; i < l; ++i) {  /* unguarded linear insert */
      pair_t val = a[i];
      int j = i, n = i - 1;
      while (gt(val.v, a[n].v)) { a[j] = a[n]; j = n; --n; }
      a[j] = val;
    }
  } else {
    insertion_sort(a, f, l);
  }
}

/* rows [T, ld] of n values -> ids [T, k] int64 in torch CPU topk order. scratch: n pairs. */
void oracle_topk_rows(const float* vals, int64_t ld, int T, int n, int k, int64_t* ids, float* out_vals,
                      void* scratch) {
  pair_t* a = (pair_t*)scratch;
  for (int t = 0; t < T; ++t) {
    for (int i = 0; i < n; ++i) { a[i].v = vals[(int64_t)t * ld + i]; a[i].i = i; }
    if ((int64_t)k * 64 <= n) {
      heap_select(a, 0, k, n);
      sort_heap(a, 0, k);
    } else {
      introselect(a, 0, k - 1, n, 2 * lg2(n));
      std_sort(a, 0, k - 1);
    }
    for (int j = 0; j < k; ++j) {
      ids[(int64_t)t * k + j] = a[j].i;
      if (out_vals) out_vals[(int64_t)t * k + j] = a[j].v;
    }
  }
}
