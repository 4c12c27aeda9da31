// Router (softmax + top-k + renormalise) and dispatch bookkeeping (stable counting sort by
// local expert).  Reference: muserve/model/qwen35_layer_v2.py:568-605.
//
// Top-k order.  torch's CPU topk (the reference oracle) calls libstdc++
//   std::nth_element(q, q+k-1, q+E, greater) ; std::sort(q, q+k-1, greater)   when k*64 >  E
//   std::partial_sort(q, q+k, q+E, greater)                                   when k*64 <= E
// over (value, index) pairs compared by value only, so the order of tied values is an
// artefact of those algorithms (it is neither "lowest index first" nor stable).  The kernel
// below replays both algorithms step for step: libstdc++'s introselect (median-of-three
// pivot, unguarded Hoare partition, insertion sort below 4 elements, heap-select fallback
// when the depth budget runs out) and its heap routines.  The partition, the only O(E) step,
// runs warp-parallel: the left scan stops at every element !(x > p), the right scan at every
// element !(p > x); the m-th left stop swaps with the m-th right stop while it lies to the
// left of it, and the cut is min(next left stop, last swapped right stop).  That reproduces
// the sequential scan exactly (both scans only ever read positions the other has not
// swapped yet).  Comparisons use the logits: softmax is monotone, so the scores order and tie
// exactly like the logits except where two distinct logits round to the same fp32 score.
#pragma once
#include "common.cuh"

namespace msv {

// comparator of torch's CPU topk for largest=true: NaN sorts first
MSV_DEVICE bool gt(float x, float y) { return (x != x && y == y) || x > y; }

struct Arr {
  float* v;
  uint16_t* ix;
  MSV_DEVICE void swap(int a, int b) {
    float tv = v[a];
    v[a] = v[b];
    v[b] = tv;
    uint16_t ti = ix[a];
    ix[a] = ix[b];
    ix[b] = ti;
  }
};

// ---- sequential libstdc++ heap pieces (run by one lane) ------------------------------------

MSV_DEVICE void push_heap(Arr a, int base, int hole, int top, float val, uint16_t vix) {
  int parent = (hole - 1) / 2;
  while (hole > top && gt(a.v[base + parent], val)) {
    a.v[base + hole] = a.v[base + parent];
    a.ix[base + hole] = a.ix[base + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a.v[base + hole] = val;
  a.ix[base + hole] = vix;
}

MSV_DEVICE void adjust_heap(Arr a, int base, int hole, int len, float val, uint16_t vix) {
  const int top = hole;
  int sc = hole;
  while (sc < (len - 1) / 2) {
    sc = 2 * (sc + 1);
    if (gt(a.v[base + sc], a.v[base + sc - 1])) sc--;
    a.v[base + hole] = a.v[base + sc];
    a.ix[base + hole] = a.ix[base + sc];
    hole = sc;
  }
  if ((len & 1) == 0 && sc == (len - 2) / 2) {
    sc = 2 * (sc + 1);
    a.v[base + hole] = a.v[base + sc - 1];
    a.ix[base + hole] = a.ix[base + sc - 1];
    hole = sc - 1;
  }
  push_heap(a, base, hole, top, val, vix);
}

MSV_DEVICE void make_heap(Arr a, int f, int l) {
  const int len = l - f;
  if (len < 2) return;
  int parent = (len - 2) / 2;
  while (true) {
    adjust_heap(a, f, parent, len, a.v[f + parent], a.ix[f + parent]);
    if (parent == 0) return;
    parent--;
  }
}

MSV_DEVICE void pop_heap(Arr a, int f, int l, int r) {
  float val = a.v[r];
  uint16_t vix = a.ix[r];
  a.v[r] = a.v[f];
  a.ix[r] = a.ix[f];
  adjust_heap(a, f, 0, l - f, val, vix);
}

MSV_DEVICE void heap_select(Arr a, int f, int m, int l) {
  make_heap(a, f, m);
  for (int i = m; i < l; ++i)
    if (gt(a.v[i], a.v[f])) pop_heap(a, f, m, i);
}

MSV_DEVICE void sort_heap(Arr a, int f, int l) {
  while (l - f > 1) {
    --l;
    pop_heap(a, f, l, l);
  }
}

// ---- warp-parallel pieces -------------------------------------------------------------------

// libstdc++'s __insertion_sort over [f, l), l - f <= 32.  For a strict weak order it leaves a
// stable descending sort: an element moves left only past elements it compares greater than.
// So each lane takes one element and writes it at its rank: the elements greater than it, plus
// the equivalent ones before it.
MSV_DEVICE void warp_insertion_sort(Arr a, int f, int l) {
  const int lane = threadIdx.x & 31;
  const int n = l - f;
  if (n < 2) return;
  float x = 0.f;
  uint16_t xi = 0;
  if (lane < n) {
    x = a.v[f + lane];
    xi = a.ix[f + lane];
  }
  int rank = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float y = __shfl_sync(0xffffffffu, x, j);
    rank += j < n && (gt(y, x) || (j < lane && !gt(x, y)));
  }
  for (int j = 16; j < n; ++j) {
    const float y = __shfl_sync(0xffffffffu, x, j);
    rank += gt(y, x) || (j < lane && !gt(x, y));
  }
  __syncwarp();
  if (lane < n) {
    a.v[f + rank] = x;
    a.ix[f + rank] = xi;
  }
  __syncwarp();
}

// Unguarded partition of [lo, hi) around p, the pivot that the median step moved to lo-1 (the
// element it displaced, w, moved to position r; lane 0 stores that swap while this runs, so the
// sweep reads those two positions from registers).  One sweep over the range in 32-element
// chunks writes the left stops (positions >= lo holding !(x > p)) upward into lpos and the
// right stops (positions >= lo-1 holding !(p > x)) upward into rposr, so the m-th right stop
// counted from the top is rposr[nr-1-m].  A second loop swaps the m-th pairs while the left
// stop lies below the right one; the pairs are disjoint, one per lane.
MSV_DEVICE int warp_partition(Arr a, int lo, int hi, float p, int r, float w, uint16_t* lpos, uint16_t* rposr) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = lanemask_lt();
  const int b0 = lo - 1;
  const int nch = (hi - b0 + 31) >> 5;
  int nl = 0, nr = 0;
  // four chunks per step: their loads issue together, before any store of the step
  for (int c0 = 0; c0 < nch; c0 += 4) {
    float xs[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = b0 + 32 * (c0 + u) + lane;
      xs[u] = i < hi ? a.v[i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = b0 + 32 * (c0 + u) + lane;
      const bool in = i < hi;
      const float x = i == r ? w : (i == b0 ? p : xs[u]);
      const bool sl = in && i >= lo && !gt(x, p);
      const bool sr = in && !gt(p, x);
      const uint32_t bl = __ballot_sync(0xffffffffu, sl);
      const uint32_t br = __ballot_sync(0xffffffffu, sr);
      if (sl) lpos[nl + __popc(bl & lt)] = (uint16_t)i;
      if (sr) rposr[nr + __popc(br & lt)] = (uint16_t)i;
      nl += __popc(bl);
      nr += __popc(br);
    }
  }
  __syncwarp();
  // swaps happen for the prefix of m with lpos[m] < rpos[m] (monotone in m)
  const int mmax = min(nl, nr);
  int nsw = 0;
  int Ln = 0, Rn = 0;  // the next step's pair, loaded ahead of this step's swaps
  if (lane < mmax) {
    Ln = lpos[lane];
    Rn = rposr[nr - 1 - lane];
  }
  for (int base = 0; base < mmax; base += 32) {
    const int m = base + lane;
    const int L = Ln, R = Rn;
    if (m + 32 < mmax) {
      Ln = lpos[m + 32];
      Rn = rposr[nr - 33 - m];
    }
    const bool sw = m < mmax && L < R;
    const uint32_t bal = __ballot_sync(0xffffffffu, sw);
    if (sw) {
      const float lv = a.v[L], rv = a.v[R];
      const uint16_t li = a.ix[L], ri = a.ix[R];
      a.v[L] = rv;
      a.ix[L] = ri;
      a.v[R] = lv;
      a.ix[R] = li;
    }
    nsw += __popc(bal);
    if (bal != 0xffffffffu) break;
  }
  int cut = 0x7fffffff;
  if (nsw < nl) cut = lpos[nsw];
  if (nsw >= 1) cut = min(cut, (int)rposr[nr - nsw]);
  __syncwarp();
  return cut;
}

// Fast path: when the k+1 largest values of the row (the k largest when k == n) are all
// distinct, torch's result is unique, the k largest in descending order, whatever the
// algorithm's internal order.  For rows of up to 512 values a warp holds the row in registers
// (16 per lane) and selects in k+1 argmax rounds, stopping at the first tie; it writes the
// result to positions [0,k) and returns true, or returns false with the row untouched (the
// replay below then decides the order of the tied values).  Rows holding a NaN never come here.
constexpr int kFastTopkMax = 512;

// order-preserving map of a non-NaN float onto uint32 (larger float -> larger key; -0 and +0,
// which compare equal, share a key)
MSV_DEVICE uint32_t f32_order_key(float x) {
  const uint32_t u = x == 0.f ? 0u : __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __noinline__ bool warp_topk_distinct(Arr a, int n, int k) {
  if (n > kFastTopkMax) return false;
  const int lane = threadIdx.x & 31;
  const int rounds = k < n ? k + 1 : k;
  constexpr int NV = kFastTopkMax / 32;
  // order keys of the lane's values i = lane + 32 j; 0 marks taken or absent (no real key is 0)
  uint32_t kx[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    kx[j] = i < n ? f32_order_key(a.v[i]) : 0u;
  }
  // the lane's largest remaining key and its slot, by a pairwise tree (depth log2 NV)
  auto lane_best = [&](uint32_t& bk, int& bj) {
    uint32_t tk[NV];
    int tj[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      tk[j] = kx[j];
      tj[j] = j;
    }
#pragma unroll
    for (int w = NV / 2; w >= 1; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) {
        const bool hi = tk[j + w] > tk[j];
        tk[j] = hi ? tk[j + w] : tk[j];
        tj[j] = hi ? tj[j + w] : tj[j];
      }
    bk = tk[0];
    bj = tj[0];
  };
  uint32_t mk;
  int mj;
  lane_best(mk, mj);
  uint32_t prev = 0;
  int sel_i = 0;
  for (int r = 0; r < rounds; ++r) {
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, mk);
    const uint32_t holders = __ballot_sync(0xffffffffu, mk == kmax);
    // two lanes holding the maximum, or a maximum equal to the previous one, is a tie among
    // the k+1 largest (a tie found only in the last round lies below the selection)
    if ((r + 1 < rounds && __popc(holders) > 1) || (r > 0 && !(prev > kmax))) return false;
    prev = kmax;
    const int wl = __ffs(holders) - 1;
    const int bi = __shfl_sync(0xffffffffu, wl + 32 * mj, wl);
    if (lane == r) sel_i = bi;
    if (lane == wl) {
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (j == mj) kx[j] = 0u;
      lane_best(mk, mj);
    }
  }
  const float sel_v = lane < k ? a.v[sel_i] : 0.f;
  __syncwarp();
  if (lane < k) {
    a.v[lane] = sel_v;
    a.ix[lane] = (uint16_t)sel_i;
  }
  __syncwarp();
  return true;
}

// Full torch-CPU topk replay on one row held in shared memory.  On return positions
// [0,k) hold the result in torch's order.
MSV_DEVICE void warp_topk_torch_cpu(Arr a, int n, int k, uint16_t* lpos, uint16_t* rpos) {
  const int lane = threadIdx.x & 31;
  if (k * 64 <= n) {  // std::partial_sort
    if (lane == 0) {
      heap_select(a, 0, k, n);
      sort_heap(a, 0, k);
    }
    __syncwarp();
    return;
  }
  // std::nth_element(first, first + k - 1, last) == __introselect(depth = 2*floor(log2 n))
  int f = 0, l = n, nth = k - 1;
  int depth = 2 * (31 - __clz(n));
  bool done = false;
  while (l - f > 3) {
    if (depth == 0) {
      if (lane == 0) {
        heap_select(a, f, nth + 1, l);
        a.swap(f, nth);
      }
      done = true;
      break;
    }
    depth--;
    // libstdc++ __move_median_to_first(f, f+1, mid, l-1): every lane reads the candidates and
    // picks the same one, r; lane 0 swaps it with position f
    const int mid = f + (l - f) / 2;
    const float vf = a.v[f], vx = a.v[f + 1], vy = a.v[mid], vz = a.v[l - 1];
    const uint16_t jf = a.ix[f], jx = a.ix[f + 1], jy = a.ix[mid], jz = a.ix[l - 1];
    int r;
    float p;
    uint16_t jr;
    if (gt(vx, vy)) {
      if (gt(vy, vz)) r = mid, p = vy, jr = jy;
      else if (gt(vx, vz)) r = l - 1, p = vz, jr = jz;
      else r = f + 1, p = vx, jr = jx;
    } else if (gt(vx, vz)) r = f + 1, p = vx, jr = jx;
    else if (gt(vy, vz)) r = l - 1, p = vz, jr = jz;
    else r = mid, p = vy, jr = jy;
    __syncwarp();
    if (lane == 0) {
      a.v[f] = p;
      a.ix[f] = jr;
      a.v[r] = vf;
      a.ix[r] = jf;
    }
    const int cut = warp_partition(a, f + 1, l, p, r, vf, lpos, rpos);
    if (cut <= nth) f = cut;
    else l = cut;
  }
  __syncwarp();
  if (!done) warp_insertion_sort(a, f, l);  // l - f <= 3
  // std::sort(first, first + k - 1): k - 1 <= 16 elements, i.e. one insertion sort
  warp_insertion_sort(a, 0, k - 1);
}

constexpr int kRouteWarps = 4;
constexpr int kRouteMaxE = 1024;  // the host entry points reject larger rows

// One warp per token.  Shared memory per warp: n floats + 3n uint16.
__global__ void __launch_bounds__(kRouteWarps * 32) k_route_topk(const float* __restrict__ logits, int64_t ld,
                                                                  int T, int E, int k, int softmax, int renorm,
                                                                  void* __restrict__ out_w, int w_dtype,
                                                                  void* __restrict__ out_ids, int ids_dtype,
                                                                  float* __restrict__ out_vals,
                                                                  const float* __restrict__ logit_bias) {
  pdl_wait();
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kRouteWarps + warp;
  if (t >= T) return;  // whole warp exits together
  const int estride = (E + 7) & ~7;
  float* v = reinterpret_cast<float*>(sm) + warp * estride;
  uint16_t* ix = reinterpret_cast<uint16_t*>(reinterpret_cast<float*>(sm) + kRouteWarps * estride) + warp * 3 * estride;
  uint16_t* lpos = ix + estride;
  uint16_t* rpos = ix + 2 * estride;
  const float* row = logits + (int64_t)t * ld;
  float mx = -INFINITY;
  bool any_nan = false;
  uint32_t low_bits = 0;  // zero when every value of the row is a bf16 value
  float xr[kRouteMaxE / 32];  // the lane's values i = lane + 32 j (E <= kRouteMaxE)
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int i = lane + 32 * j;
    xr[j] = i < E ? row[i] : 0.f;
  }
  if (logit_bias) {  // an additive prior on the logits (fp32 add)
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j) {
      const int i = lane + 32 * j;
      if (i < E) xr[j] = __fadd_rn(xr[j], logit_bias[i]);
    }
  }
#pragma unroll
  for (int j = 0; j < kRouteMaxE / 32; ++j) {
    const int i = lane + 32 * j;
    if (i < E) {
      const float x = xr[j];
      v[i] = x;
      ix[i] = (uint16_t)i;
      mx = fmaxf(mx, x);
      any_nan |= (x != x);
      low_bits |= __float_as_uint(x) & 0xffffu;
    }
  }
  mx = warp_max(mx);
  any_nan = __any_sync(0xffffffffu, any_nan);
  // rows of bf16 logits (8-bit significands) usually hold ties among their largest values, so
  // they go straight to the replay; other rows try the distinct-values fast path first
  const bool bf16_row = !__any_sync(0xffffffffu, low_bits != 0);
  // torch's softmax turns a whole row into NaN when it holds a NaN or +inf logit; select on
  // that all-NaN row then, exactly as torch.topk sees it.
  const bool all_nan = softmax && (any_nan || mx == INFINITY);
  float sum = 0.f;
  if (softmax && !all_nan) {
#pragma unroll
    for (int j = 0; j < kRouteMaxE / 32; ++j)
      if (lane + 32 * j < E) sum += expf(xr[j] - mx);
    sum = warp_sum(sum);
  }
  if (all_nan)
    for (int i = lane; i < E; i += 32) v[i] = __int_as_float(0x7fffffff);
  __syncwarp();
  Arr a{v, ix};
  if (any_nan || all_nan || bf16_row || !warp_topk_distinct(a, E, k)) warp_topk_torch_cpu(a, E, k, lpos, rpos);
  // weights: score_j = exp(x_j - max) * (1/sum); optional renormalisation over the k
  float s = 0.f;
  uint16_t id = 0;
  if (lane < k) {
    id = ix[lane];
    float x = v[lane];
    s = softmax ? (all_nan ? x : expf(x - mx) * (1.0f / sum)) : x;
  }
  if (renorm) {
    float sj[16];  // k <= 16; all shuffles issue first, then the sum runs in slot order
#pragma unroll
    for (int j = 0; j < 16; ++j) sj[j] = __shfl_sync(0xffffffffu, s, j);
    float tot = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < k) tot += sj[j];
    s = __fdiv_rn(s, tot);
  }
  if (lane < k) {
    const int64_t o = (int64_t)t * k + lane;
    if (out_w) {
      if (w_dtype == MSV_BF16) reinterpret_cast<__nv_bfloat16*>(out_w)[o] = __float2bfloat16_rn(s);
      else reinterpret_cast<float*>(out_w)[o] = s;
    }
    if (out_vals) out_vals[o] = v[lane];
    if (ids_dtype == MSV_I64) reinterpret_cast<int64_t*>(out_ids)[o] = id;
    else reinterpret_cast<int32_t*>(out_ids)[o] = id;
  }
  pdl_trigger();
}

size_t route_smem_bytes(int E) {
  const int estride = (E + 7) & ~7;
  return (size_t)kRouteWarps * estride * (4 + 3 * 2);
}

// ── dispatch bookkeeping ────────────────────────────────────────────────────────────────

struct PermuteArgs {
  const void* ids;
  int ids_i64;
  int T, k, num_experts, placement, tp, rank, alignment;
  int e_local;
  int64_t* sort_order;
  int64_t* inverse_order;
  int32_t* sorted_expert_ids;
  int32_t* expert_counts;
  int32_t* num_local;
  int32_t* row_token;  // [T*k] token of each sorted row (internal)
  int32_t* slot_row;   // [T*k] sorted row of each slot, -1 when not local (internal)
  // grouped-GEMM tile lists (internal; nullptr to skip).  ntiles* point at two ints: the tile
  // count and the GEMM's tile-claim counter, which the builder zeroes.
  int4* tiles1;
  int* ntiles1;
  int bn1, nb1;
  int4* tiles2;
  int* ntiles2;
  int bn2, nb2;
  int shared_rows;    // > 0: append the shared-expert group (rows [row_base_shared, +shared_rows))
  int row_base_shared;
};

constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;
constexpr int kPermSingleMax = 8192;  // above this many slots the dispatch runs over many blocks

MSV_DEVICE int load_id(const PermuteArgs& p, int f) {
  return p.ids_i64 ? (int)reinterpret_cast<const int64_t*>(p.ids)[f] : reinterpret_cast<const int32_t*>(p.ids)[f];
}

// Block-wide exclusive scan of one int per thread (1024 threads); *total gets the sum.
// s_warp needs 33 ints.  Contains __syncthreads: every thread of the block must call it.
MSV_DEVICE int block_excl_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = s_warp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    s_warp[lane] = wi - w;
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  const int excl = s_warp[warp] + incl - v;
  *total = s_warp[32];
  __syncthreads();
  return excl;
}

// Tile list of one grouped GEMM: per local expert with c rows, ceil(c/bn) row chunks of
// near-equal size (multiples of 16) times nb weight n-blocks, ordered expert, n-block, chunk
// (chunks sharing a weight tile are adjacent).  The shared-expert group goes first.
MSV_DEVICE void build_tiles(const PermuteArgs& p, const int* counts, const int* offsets, int4* info, int* s_warp,
                            int4* tiles, int* ntiles, int bn, int nb) {
  const int tid = threadIdx.x;
  const int E = p.e_local;
  const int nsh_chunks = p.shared_rows > 0 ? (p.shared_rows + bn - 1) / bn : 0;
  const int nsh = nsh_chunks * nb;
  // per expert (one per thread, e_local <= 1024): chunk count and size, tile count -> scan
  const int c_mine = tid < E ? counts[tid] : 0;
  int nch = 0, cs = 0;
  if (c_mine > 0) {
    nch = (c_mine + bn - 1) / bn;
    cs = ((c_mine + nch - 1) / nch + 15) & ~15;
  }
  int total = 0;
  const int base_mine = block_excl_scan(nch * nb, s_warp, &total);
  if (tid < E) info[tid] = make_int4(nsh + base_mine, offsets[tid], c_mine, nch | (cs << 16));
  if (tid == 0) {
    ntiles[0] = nsh + total;
    ntiles[1] = 0;  // the GEMM's tile-claim counter
  }
  __syncthreads();
  // shared-expert tiles
  for (int i = tid; i < nsh; i += kPermThreads) {
    int nbi = i / nsh_chunks, ch = i % nsh_chunks;
    int scs = ((p.shared_rows + nsh_chunks - 1) / nsh_chunks + 15) & ~15;
    int r0 = ch * scs;
    int nr = min(scs, p.shared_rows - r0);
    tiles[i] = make_int4(p.row_base_shared + r0, nr, (1 << 24) | 0, nbi);
  }
  // one thread per (expert, n-block), so a warp writes an expert's consecutive tiles.
  // expert = item / nb as a multiply-high by ceil(2^32 / nb): exact while item * nb < 2^32.
  const uint32_t magic = nb > 1 ? 0xffffffffu / (uint32_t)nb + 1u : 0u;
  for (int item = tid; item < E * nb; item += kPermThreads) {
    const int e = nb > 1 ? (int)__umulhi((uint32_t)item, magic) : item;
    const int4 in = info[e];
    if (in.z == 0) continue;
    const int nbi = item - e * nb;
    const int enc = in.w & 0xffff, ecs = in.w >> 16;
    const int base = in.x + nbi * enc;
    for (int ch = 0; ch < enc; ++ch) {
      const int r0 = ch * ecs;
      int nr = min(ecs, in.z - r0);
      if (nr <= 0) nr = 0;
      tiles[base + ch] = make_int4(in.y + r0, nr, e, nbi);
    }
  }
  __syncthreads();
}

// One CTA.  Warp w owns the contiguous slot chunk [w*C, (w+1)*C): pass 1 counts local slots
// per (warp, expert); the scan turns the counts into each (warp, expert) base row; pass 2
// walks the chunk in order and ranks equal experts inside each 32-slot batch with
// __match_any_sync, which keeps the sort stable.
__global__ void __launch_bounds__(kPermThreads) k_permute(PermuteArgs p) {
  pdl_wait();
  extern __shared__ __align__(16) int hist[];  // [kPermWarps][e_local], counts, offsets
  __shared__ int s_nloc[kPermWarps];
  __shared__ int s_total;
  __shared__ int s_warp[33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.e_local;
  int* counts = hist + kPermWarps * E;   // [E]
  int* offsets = counts + E;             // [E+1]
  const int P = p.T * p.k;
  // counting warps: at least 64 slots each, so small batches sum few per-warp histograms
  const int HW = max(1, min(kPermWarps, (P + 63) / 64));
  const int C = (P + HW - 1) / HW;
  const int c0 = warp < HW ? min(P, warp * C) : P, c1 = warp < HW ? min(P, c0 + C) : P;
  for (int i = threadIdx.x; i < HW * E; i += kPermThreads) hist[i] = 0;
  __syncthreads();
  int nloc = 0;
  for (int f = c0 + lane; f < c1; f += 32) {
    int e = load_id(p, f);
    bool local = p.placement == 0 || (e % p.tp) == p.rank;
    int le = p.placement == 0 ? e : e / p.tp;
    if (local && le >= 0 && le < E) {
      atomicAdd(&hist[warp * E + le], 1);
      nloc++;
    }
  }
  for (int o = 16; o > 0; o >>= 1) nloc += __shfl_xor_sync(0xffffffffu, nloc, o);
  if (lane == 0) s_nloc[warp] = nloc;
  __syncthreads();
  // per-expert totals
  for (int e = threadIdx.x; e < E; e += kPermThreads) {
    int c = 0;
    for (int w = 0; w < HW; ++w) c += hist[w * E + e];
    counts[e] = c;
  }
  __syncthreads();
  {
    int total = 0;
    const int off = block_excl_scan(threadIdx.x < E ? counts[threadIdx.x] : 0, s_warp, &total);
    if (threadIdx.x < E) offsets[threadIdx.x] = off;
    if (threadIdx.x == 0) {
      offsets[E] = total;
      s_total = total;
      *p.num_local = total;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kPermThreads) {
    int run = offsets[e];
    for (int w = 0; w < HW; ++w) {
      int c = hist[w * E + e];
      hist[w * E + e] = run;
      run += c;
    }
    if (p.expert_counts) p.expert_counts[e] = counts[e];
  }
  int lpbase = 0;
  for (int w = 0; w < warp; ++w) lpbase += s_nloc[w];
  __syncthreads();
  for (int b0 = c0; b0 < c1; b0 += 32) {
    const int f = b0 + lane;
    const bool valid = f < c1;
    int e = valid ? load_id(p, f) : -1;
    int le = p.placement == 0 ? e : (e >= 0 ? e / p.tp : -1);
    bool local = valid && (p.placement == 0 || (e % p.tp) == p.rank) && le >= 0 && le < E;
    uint32_t bal = __ballot_sync(0xffffffffu, local);
    int lp = lpbase + __popc(bal & lanemask_lt());
    lpbase += __popc(bal);
    uint32_t key = local ? (uint32_t)le : 0xffffffffu;
    uint32_t peers = __match_any_sync(0xffffffffu, key);
    int r = 0;
    if (local) r = hist[warp * E + le] + __popc(peers & lanemask_lt());
    __syncwarp();
    if (local && (__ffs(peers) - 1) == lane) hist[warp * E + le] += __popc(peers);
    __syncwarp();
    if (valid) {
      if (p.slot_row) p.slot_row[f] = local ? r : -1;
      if (local) {
        if (p.row_token) p.row_token[r] = f / p.k;
        if (p.sort_order) p.sort_order[r] = lp;
        if (p.inverse_order) p.inverse_order[lp] = r;
        if (p.sorted_expert_ids) p.sorted_expert_ids[r] = le;
      }
    }
  }
  __syncthreads();
  if (p.sorted_expert_ids && p.alignment > 0) {
    const int nl = s_total;
    const int padded = ((nl + p.alignment - 1) / p.alignment) * p.alignment;
    for (int r = nl + threadIdx.x; r < padded; r += kPermThreads) p.sorted_expert_ids[r] = -1;
  }
  // the per-warp histogram is dead here: its first 4 * e_local ints hold the per-expert tile info
  int4* info = reinterpret_cast<int4*>(hist);
  if (p.tiles1) build_tiles(p, counts, offsets, info, s_warp, p.tiles1, p.ntiles1, p.bn1, p.nb1);
  if (p.tiles2) build_tiles(p, counts, offsets, info, s_warp, p.tiles2, p.ntiles2, p.bn2, p.nb2);
  pdl_trigger();
}

size_t permute_smem_bytes(int e_local) { return (size_t)(kPermWarps * e_local + 2 * e_local + 1) * sizeof(int); }

// ── multi-block dispatch (large T*k) ──────────────────────────────────────────────────────
// The same stable counting sort as k_permute, spread over blocks of kPermThreads slots:
//   k_perm_count:   per block, each slot's rank among the block's earlier slots of its expert
//                   (warp match + per-warp counts) and its index among the block's local slots;
//                   the block's per-expert counts and local count.
//   k_perm_scan:    one block: per-expert totals and offsets, every block's base per expert
//                   (offset + counts of earlier blocks), counts / num_local / tile lists.
//   k_perm_scatter: row = block base[expert] + rank; the slot <-> row maps.
// Slot f goes to block f / kPermThreads, warp (f % kPermThreads) / 32, lane f % 32, so the
// order (block, warp, lane) is slot order and the sort is stable as torch's argsort(stable).
struct PermuteScratch {
  int* blk_hist;  // [nblk][e_local] block counts, then block bases
  int* blk_nloc;  // [nblk] local slots per block, then their exclusive prefix
  int* lrank;     // [T*k] rank within (block, expert), -1 when not local
  int* lpos;      // [T*k] index among the block's local slots
  int nblk;
};

size_t perm_count_smem_bytes(int e_local) { return (size_t)(kPermWarps * e_local) * sizeof(int); }

__global__ void __launch_bounds__(kPermThreads) k_perm_count(PermuteArgs p, PermuteScratch s) {
  pdl_wait();
  extern __shared__ __align__(16) int wc[];  // [kPermWarps][e_local] per-warp counts, then bases
  __shared__ int s_wn[kPermWarps + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.e_local;
  const int P = p.T * p.k;
  const int f = blockIdx.x * kPermThreads + threadIdx.x;
  for (int i = threadIdx.x; i < kPermWarps * E; i += kPermThreads) wc[i] = 0;
  __syncthreads();
  const bool valid = f < P;
  const int e = valid ? load_id(p, f) : -1;
  const int le = p.placement == 0 ? e : (e >= 0 ? e / p.tp : -1);
  const bool local = valid && (p.placement == 0 || (e % p.tp) == p.rank) && le >= 0 && le < E;
  const uint32_t bal = __ballot_sync(0xffffffffu, local);
  const uint32_t peers = __match_any_sync(0xffffffffu, local ? (uint32_t)le : 0xffffffffu);
  const int rank_w = __popc(peers & lanemask_lt());
  if (local && (__ffs(peers) - 1) == lane) wc[warp * E + le] = __popc(peers);
  if (lane == 0) s_wn[warp] = __popc(bal);
  __syncthreads();
  // per expert: exclusive scan over the warps (slot order), block total
  for (int x = threadIdx.x; x < E; x += kPermThreads) {
    int run = 0;
    for (int w = 0; w < kPermWarps; ++w) {
      const int c = wc[w * E + x];
      wc[w * E + x] = run;
      run += c;
    }
    s.blk_hist[blockIdx.x * E + x] = run;
  }
  if (warp == 0) {
    const int v = s_wn[lane];
    int incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s_wn[lane] = incl - v;
    if (lane == 31) s.blk_nloc[blockIdx.x] = incl;
  }
  __syncthreads();
  if (valid) {
    s.lrank[f] = local ? wc[warp * E + le] + rank_w : -1;
    s.lpos[f] = local ? s_wn[warp] + __popc(bal & lanemask_lt()) : -1;
  }
  pdl_trigger();
}

__global__ void __launch_bounds__(kPermThreads) k_perm_scan(PermuteArgs p, PermuteScratch s) {
  pdl_wait();
  extern __shared__ __align__(16) int scan_sm[];  // tile info int4 [E], counts [E], offsets [E+1]
  __shared__ int s_warp[33];
  const int E = p.e_local;
  int4* info = reinterpret_cast<int4*>(scan_sm);
  int* counts = scan_sm + 4 * E;
  int* offsets = counts + E;
  // per-expert totals over the blocks, 16 blocks' counts in flight at a time
  constexpr int kB = 16;
  for (int x = threadIdx.x; x < E; x += kPermThreads) {
    int c = 0;
    for (int b0 = 0; b0 < s.nblk; b0 += kB) {
      int v[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) v[i] = b0 + i < s.nblk ? s.blk_hist[(b0 + i) * E + x] : 0;
#pragma unroll
      for (int i = 0; i < kB; ++i) c += v[i];
    }
    counts[x] = c;
  }
  __syncthreads();
  int total = 0;
  const int off = block_excl_scan(threadIdx.x < E ? counts[threadIdx.x] : 0, s_warp, &total);
  if (threadIdx.x < E) offsets[threadIdx.x] = off;
  if (threadIdx.x == 0) {
    offsets[E] = total;
    *p.num_local = total;
  }
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += kPermThreads) {
    int run = offsets[x];
    for (int b0 = 0; b0 < s.nblk; b0 += kB) {
      int v[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) v[i] = b0 + i < s.nblk ? s.blk_hist[(b0 + i) * E + x] : 0;
#pragma unroll
      for (int i = 0; i < kB; ++i)
        if (b0 + i < s.nblk) {
          s.blk_hist[(b0 + i) * E + x] = run;
          run += v[i];
        }
    }
    if (p.expert_counts) p.expert_counts[x] = counts[x];
  }
  // exclusive prefix of the blocks' local counts (at most kPermThreads blocks per pass)
  {
    int carry = 0;
    for (int b0 = 0; b0 < s.nblk; b0 += kPermThreads) {
      const int b = b0 + threadIdx.x;
      const int c = b < s.nblk ? s.blk_nloc[b] : 0;
      int tot = 0;
      const int ex = block_excl_scan(c, s_warp, &tot);
      if (b < s.nblk) s.blk_nloc[b] = carry + ex;
      carry += tot;
    }
  }
  if (p.sorted_expert_ids && p.alignment > 0) {
    const int padded = ((total + p.alignment - 1) / p.alignment) * p.alignment;
    for (int r = total + threadIdx.x; r < padded; r += kPermThreads) p.sorted_expert_ids[r] = -1;
  }
  __syncthreads();
  if (p.tiles1) build_tiles(p, counts, offsets, info, s_warp, p.tiles1, p.ntiles1, p.bn1, p.nb1);
  if (p.tiles2) build_tiles(p, counts, offsets, info, s_warp, p.tiles2, p.ntiles2, p.bn2, p.nb2);
  pdl_trigger();
}

size_t perm_scan_smem_bytes(int e_local) { return (size_t)(6 * e_local + 1) * sizeof(int); }

__global__ void __launch_bounds__(256) k_perm_scatter(PermuteArgs p, PermuteScratch s) {
  pdl_wait();
  const int P = p.T * p.k;
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= P) return;
  const int lr = s.lrank[f];
  if (lr < 0) {
    if (p.slot_row) p.slot_row[f] = -1;
    return;
  }
  const int e = load_id(p, f);
  const int le = p.placement == 0 ? e : e / p.tp;
  const int b = f / kPermThreads;
  const int r = s.blk_hist[b * p.e_local + le] + lr;
  const int lp = s.blk_nloc[b] + s.lpos[f];
  if (p.slot_row) p.slot_row[f] = r;
  if (p.row_token) p.row_token[r] = f / p.k;
  if (p.sort_order) p.sort_order[r] = lp;
  if (p.inverse_order) p.inverse_order[lp] = r;
  if (p.sorted_expert_ids) p.sorted_expert_ids[r] = le;
  pdl_trigger();
}

// Groups from an arbitrary per-row expert array (the ragged-GEMM shim): every maximal run
// of equal non-negative ids is one group, chunked by bn, times nb n-blocks.  One CTA.
__global__ void __launch_bounds__(1024) k_tiles_from_runs(const int32_t* __restrict__ m_indices, int M, int bn,
                                                          int nb, int4* __restrict__ tiles, int* __restrict__ ntiles,
                                                          int cap) {
  pdl_wait();
  __shared__ int s_base;
  __shared__ int s_warp[32];
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int b0 = 0; b0 < M; b0 += 1024) {
    const int m = b0 + threadIdx.x;
    int e = -1, len = 0;
    if (m < M) {
      e = m_indices[m];
      bool start = e >= 0 && (m == 0 || m_indices[m - 1] != e);
      if (start) {
        int j = m + 1;
        while (j < M && m_indices[j] == e) ++j;
        len = j - m;
      }
    }
    int nt = len > 0 ? ((len + bn - 1) / bn) * nb : 0;
    // block exclusive scan of nt
    int incl = nt;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = s_warp[lane];
      int vi = v;
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, vi, o);
        if (lane >= o) vi += y;
      }
      s_warp[lane] = vi - v;
    }
    __syncthreads();
    int pos = s_base + s_warp[warp] + incl - nt;
    if (len > 0) {
      int nch = (len + bn - 1) / bn;
      int cs = ((len + nch - 1) / nch + 15) & ~15;
      for (int nbi = 0; nbi < nb; ++nbi)
        for (int ch = 0; ch < nch; ++ch) {
          int r0 = ch * cs;
          int nr = min(cs, len - r0);
          int ti = pos + nbi * nch + ch;
          if (ti < cap) tiles[ti] = make_int4(m + r0, max(nr, 0), e, nbi);
        }
    }
    __syncthreads();
    if (threadIdx.x == 1023) s_base = pos + nt;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ntiles[0] = min(s_base, cap);
    ntiles[1] = 0;  // the GEMM's tile-claim counter
  }
  pdl_trigger();
}

}  // namespace msv

namespace msv {
// Tile list of a dense GEMM: one group of M rows chunked by bn, times nb n-blocks.
__global__ void k_tiles_dense(int M, int bn, int nb, int4* __restrict__ tiles, int* __restrict__ ntiles) {
  pdl_wait();
  const int nch = (M + bn - 1) / bn;
  const int n = nch * nb;
  const int cs = ((M + nch - 1) / nch + 15) & ~15;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int nbi = i / nch, ch = i % nch;
    const int r0 = ch * cs;
    tiles[i] = make_int4(r0, max(0, min(cs, M - r0)), 0, nbi);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    ntiles[0] = n;
    ntiles[1] = 0;  // the GEMM's tile-claim counter
  }
  pdl_trigger();
}
}  // namespace msv
