// Dispatch bookkeeping fused with the per-128 e4m3 quantisation, for batches of up to
// kPermSingleMax routed slots (decode).  References: muserve/model/qwen35_layer_v2.py:574-605
// (expand, local filter, stable argsort by expert, pad) and :71-86 / :612 (_fast_fp8_quantize of
// the gathered rows).
//
// One launch replaces the single-CTA dispatch and the quantise kernel.  Every CTA recounts the
// whole routing (at most 8192 slot ids, read once into shared memory) into per-warp expert
// histograms and their prefix, which gives the stable sorted row of any slot:
//   row(f) = offset[e] + (slots of expert e in earlier warp chunks) + (earlier slots of e in f's chunk)
// exactly the order of argsort(local ids, stable).  CTA 0 writes the per-expert counts and the
// gate_up GEMM's tile list, CTA 1 (CTA 0 when G == 1) the down GEMM's; with G > 2 those two take
// no tokens, and CTA 2 + j takes tokens j, j + (G - 2), ...: it places their k slots, quantises
// each token's row once and writes the e4m3 row and its scales to every sorted row that reads it
// (its local slots and its shared-expert row), and computes the shared-expert gate.  The first
// two tokens' activations are loaded before the recount, which hides their load latency.  The
// recount is redundant across CTAs but runs in parallel; the tile lists (a few microseconds in
// one CTA) and the token rows no longer wait for each other.
#pragma once
#include "quant_combine.cuh"
#include "route.cuh"

namespace msv {

constexpr int kDqThreads = kPermThreads;  // 1024: the tile-list builder's block size
constexpr int kDqMaxSlots = 256;          // slots of one CTA's tokens (the host sizes the grid for it)

size_t dispatch_quant_smem_bytes(int P, int e_local) {
  // per-warp histograms (reused for the tile builder's per-expert info), counts, offsets, slot ids
  return (size_t)(kPermWarps * e_local + 2 * e_local + 1 + P) * sizeof(int) + 64;
}

__global__ void __launch_bounds__(kDqThreads) k_dispatch_quant(PermuteArgs p, ScatterArgs q) {
  pdl_wait();
  extern __shared__ __align__(16) int dq_smem[];
  __shared__ int s_warp[33];
  __shared__ int s_rows[kDqMaxSlots];
  __shared__ float s_dot[kDqThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.e_local;
  const int P = p.T * p.k;
  // this CTA's tokens: tq, tq + Gq, ... (none for the tile-list CTAs 0 and 1 when G > 2)
  const int G = gridDim.x;
  const int tb = G > 2 ? 2 : 0;
  const int Gq = G - tb;
  const int tq = (int)blockIdx.x - tb;
  const int ntok = (tq >= 0 && tq < p.T) ? (p.T - tq + Gq - 1) / Gq : 0;
  // the first pass of the first two tokens (channels c0..c0+3) and of the gate weight: loaded
  // now, used after the recount
  const int c0 = threadIdx.x * 4;
  uint2 xpre0 = make_uint2(0u, 0u), xpre1 = make_uint2(0u, 0u), wpre = make_uint2(0u, 0u);
  if (c0 < q.K) {
    if (ntok > 0) xpre0 = *reinterpret_cast<const uint2*>(q.x + (int64_t)tq * q.ldx + c0);
    if (ntok > 1) xpre1 = *reinterpret_cast<const uint2*>(q.x + (int64_t)(tq + Gq) * q.ldx + c0);
    if (q.gate_w) wpre = *reinterpret_cast<const uint2*>(q.gate_w + c0);
  }
  // the per-warp histograms first: the tile builder reuses them as 16-byte int4 records
  int* hist = dq_smem;                     // [kPermWarps][E]: per-warp counts, then bases
  int* counts = hist + kPermWarps * E;     // [E]
  int* offsets = counts + E;               // [E + 1]
  int* le_of = offsets + E + 1;            // [P] local expert of each slot, -1 when not local
  // 1. the routing, once, as local expert ids
  for (int f = threadIdx.x; f < P; f += kDqThreads) {
    const int e = load_id(p, f);
    const bool local = p.placement == 0 || (e % p.tp) == p.rank;
    const int le = p.placement == 0 ? e : e / p.tp;
    le_of[f] = (local && le >= 0 && le < E) ? le : -1;
  }
  // counting warps: at least 64 slots each, warp w owns the slot chunk [w C, (w + 1) C)
  const int HW = max(1, min(kPermWarps, (P + 63) / 64));
  const int C = (P + HW - 1) / HW;
  for (int i = threadIdx.x; i < HW * E; i += kDqThreads) hist[i] = 0;
  __syncthreads();
  if (warp < HW) {
    const int c0 = min(P, warp * C), c1 = min(P, c0 + C);
    for (int f = c0 + lane; f < c1; f += 32) {
      const int le = le_of[f];
      if (le >= 0) atomicAdd(&hist[warp * E + le], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kDqThreads) {
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
      if (blockIdx.x == 0) *p.num_local = total;
    }
  }
  __syncthreads();
  // (warp, expert) bases: offset[e] + the counts of earlier chunks
  for (int e = threadIdx.x; e < E; e += kDqThreads) {
    int run = offsets[e];
    for (int w = 0; w < HW; ++w) {
      const int c = hist[w * E + e];
      hist[w * E + e] = run;
      run += c;
    }
    if (blockIdx.x == 0 && p.expert_counts) p.expert_counts[e] = counts[e];
  }
  __syncthreads();
  // 2. this CTA's tokens: sorted rows of their slots, one warp per slot
  for (int s = warp; s < ntok * p.k; s += kDqThreads / 32) {
    const int t = tq + (s / p.k) * Gq;
    const int f = t * p.k + s % p.k;
    const int le = le_of[f];
    int row = -1;
    if (le >= 0) {
      const int w = f / C;  // the chunk holding f
      int before = 0;
      for (int g = w * C + lane; g < f; g += 32) before += le_of[g] == le;
      before = __reduce_add_sync(0xffffffffu, before);
      row = hist[w * E + le] + before;
    }
    if (lane == 0) {
      s_rows[s] = row;
      p.slot_row[f] = row;
    }
  }
  __syncthreads();  // s_rows complete; the per-warp bases are dead from here
  // 3. the tile lists (their scans synchronise the whole CTA)
  int4* info = reinterpret_cast<int4*>(hist);
  if (blockIdx.x == 0 && p.tiles1) build_tiles(p, counts, offsets, info, s_warp, p.tiles1, p.ntiles1, p.bn1, p.nb1);
  if ((int)blockIdx.x == (G > 1 ? 1 : 0) && p.tiles2)
    build_tiles(p, counts, offsets, info, s_warp, p.tiles2, p.ntiles2, p.bn2, p.nb2);
  // 4. quantise each token once and write the e4m3 row and its scales to every row that reads
  // it: 4 channels per thread and pass, so a 128-channel block is one warp
  for (int i = 0; i < ntok; ++i) {
    const int t = tq + i * Gq;
    const __nv_bfloat16* __restrict__ xr = q.x + (int64_t)t * q.ldx;
    float dot = 0.f;
    for (int c = c0; c < q.K; c += kDqThreads * 4) {
      uint2 raw;
      if (c == c0 && i == 0) raw = xpre0;
      else if (c == c0 && i == 1) raw = xpre1;
      else raw = *reinterpret_cast<const uint2*>(xr + c);
      float f[4];
      f[0] = bf16_bits_to_f32(raw.x, 0);
      f[1] = bf16_bits_to_f32(raw.x, 1);
      f[2] = bf16_bits_to_f32(raw.y, 0);
      f[3] = bf16_bits_to_f32(raw.y, 1);
      float am = nanmax(nanmax(fabsf(f[0]), fabsf(f[1])), nanmax(fabsf(f[2]), fabsf(f[3])));
      if (q.gate_w) {
        const uint2 wraw = c == c0 ? wpre : *reinterpret_cast<const uint2*>(q.gate_w + c);
        dot = fmaf(f[0], bf16_bits_to_f32(wraw.x, 0), dot);
        dot = fmaf(f[1], bf16_bits_to_f32(wraw.x, 1), dot);
        dot = fmaf(f[2], bf16_bits_to_f32(wraw.y, 0), dot);
        dot = fmaf(f[3], bf16_bits_to_f32(wraw.y, 1), dot);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) am = nanmax(am, __shfl_xor_sync(0xffffffffu, am, o));
      // s = clamp(amax, min=1e-12) / 448 (NaN propagates as in torch.clamp)
      const float sc = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
      const uint32_t lo = f32x2_to_e4m3x2(clamp_pm(__fdiv_rn(f[0], sc), 448.0f), clamp_pm(__fdiv_rn(f[1], sc), 448.0f));
      const uint32_t hi = f32x2_to_e4m3x2(clamp_pm(__fdiv_rn(f[2], sc), 448.0f), clamp_pm(__fdiv_rn(f[3], sc), 448.0f));
      const uint32_t qv = lo | (hi << 16);
      for (int d = 0; d <= p.k; ++d) {
        const int r = d < p.k ? s_rows[i * p.k + d] : (q.shared_row0 >= 0 ? q.shared_row0 + t : -1);
        if (r < 0) continue;
        *reinterpret_cast<uint32_t*>(q.q + (int64_t)r * q.ldq + c) = qv;
        if (lane == 0) q.scale[(int64_t)(c / 128) * q.s_kb + r] = sc;
      }
    }
    if (q.gate_w) {  // uniform over the block
      dot = warp_sum(dot);
      if (lane == 0) s_dot[warp] = dot;
      __syncthreads();
      if (threadIdx.x == 0) {
        float d = 0.f;
        for (int w = 0; w < kDqThreads / 32; ++w) d += s_dot[w];
        const float lg = bf16_round(d);
        q.gate_val[t] = bf16_round(1.0f / (1.0f + expf(-lg)));
      }
      __syncthreads();
    }
  }
  pdl_trigger();
}

}  // namespace msv
