// Per-row per-128-channel e4m3 quantisation (with dispatch gather) and the weighted
// combine.  References: muserve/model/qwen35_layer_v2.py:71-86 (_fast_fp8_quantize),
// :649-673 (unsort, weighted sum, shared expert add), muserve/kernels/moe_dispatch.py:75-77,
// muserve/kernels/batched_moe.py:153-158.
#pragma once
#include "common.cuh"

namespace msv {

struct QuantArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  int K;
  // segment A: rows [0, rows_a) read x row idx_a[r] (idx_a == nullptr: identity); rows at or
  // beyond *nvalid_a (when given) are skipped
  int rows_a;
  const int32_t* idx_a;
  const int32_t* nvalid_a;
  // segment B: rows [rows_a, rows_a + rows_b) read x row (r - rows_a)
  int rows_b;
  uint8_t* q;
  int64_t ldq;
  float* scale;
  int64_t s_row, s_kb;
  // shared-expert gate: gv[t] = bf16(sigmoid(bf16(x[t] . wg))) for segment-B rows
  const __nv_bfloat16* gate_w;
  float* gate_val;
};

constexpr int kQuantWarps = 8;  // per CTA: kQuantWarps / kQuantSplit rows
constexpr int kQuantSplit = 4;  // warps per row
constexpr int kQuantRowsPerCta = kQuantWarps / kQuantSplit;

// kQuantSplit warps per output row; warp p of a row takes the row's 256-channel slabs p,
// p + kQuantSplit, ...  Each lane owns 8 consecutive channels (16 bytes) of a slab, so a
// 128-channel block is 16 lanes of one warp and its amax is a 4-step xor shuffle.  The shared
// gate's dot product is summed over the row's warps in warp order.
__global__ void __launch_bounds__(kQuantWarps * 32) k_quant_rows(QuantArgs a) {
  pdl_wait();
  __shared__ float s_dot[kQuantWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int part = warp % kQuantSplit;
  const int r = blockIdx.x * (kQuantWarps / kQuantSplit) + warp / kQuantSplit;
  bool active = r < a.rows_a + a.rows_b;
  int64_t src = 0;
  const bool seg_b = r >= a.rows_a;
  if (active) {
    if (!seg_b) {
      if (a.nvalid_a && r >= *a.nvalid_a) active = false;
      else src = a.idx_a ? a.idx_a[r] : r;
      if (src < 0) active = false;
    } else {
      src = r - a.rows_a;
    }
  }
  const bool want_gate = active && seg_b && a.gate_w != nullptr;
  float dot = 0.f;
  if (active) {
    const __nv_bfloat16* __restrict__ xr = a.x + src * a.ldx;
    uint8_t* __restrict__ qr = a.q + (int64_t)r * a.ldq;
    const int nslab = (a.K + 255) / 256;
    constexpr int kBatch = 4;  // slabs loaded before any is processed
    for (int s0 = part; s0 < nslab; s0 += kQuantSplit * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int c = (s0 + b * kQuantSplit) * 256 + lane * 8;
        raw[b] = c < a.K ? *reinterpret_cast<const uint4*>(xr + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int c = (s0 + b * kQuantSplit) * 256 + lane * 8;
        float f[8];
        const uint32_t w4[4] = {raw[b].x, raw[b].y, raw[b].z, raw[b].w};
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          f[i] = bf16_bits_to_f32(w4[i >> 1], i & 1);
          am = nanmax(am, fabsf(f[i]));
        }
        if (want_gate && c < a.K) {
          const uint4 wraw = *reinterpret_cast<const uint4*>(a.gate_w + c);
          const uint32_t g4[4] = {wraw.x, wraw.y, wraw.z, wraw.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) dot = fmaf(f[i], bf16_bits_to_f32(g4[i >> 1], i & 1), dot);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) am = nanmax(am, __shfl_xor_sync(0xffffffffu, am, o));
        // s = clamp(amax, min=1e-12) / 448 (NaN propagates as in torch.clamp)
        const float sc = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
        if (c < a.K) {
          uint32_t packed[2];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float lo = clamp_pm(__fdiv_rn(f[2 * i], sc), 448.0f);
            const float hi = clamp_pm(__fdiv_rn(f[2 * i + 1], sc), 448.0f);
            const uint16_t pr = f32x2_to_e4m3x2(lo, hi);
            if (i & 1) packed[i >> 1] |= (uint32_t)pr << 16;
            else packed[i >> 1] = pr;
          }
          *reinterpret_cast<uint2*>(qr + c) = make_uint2(packed[0], packed[1]);
          if ((lane & 15) == 0) a.scale[(int64_t)r * a.s_row + (int64_t)(c / 128) * a.s_kb] = sc;
        }
      }
    }
  }
  if (a.gate_w != nullptr) {  // uniform over the block
    dot = warp_sum(dot);
    if (lane == 0) s_dot[warp] = dot;
    __syncthreads();
    if (want_gate && part == 0 && lane == 0) {
      float d = s_dot[warp];
      for (int p = 1; p < kQuantSplit; ++p) d += s_dot[warp + p];
      const float lg = bf16_round(d);
      const float sg = bf16_round(1.0f / (1.0f + expf(-lg)));
      a.gate_val[src] = sg;
    }
  }
  pdl_trigger();
}

// Layer path: every token is quantised once and its e4m3 row and scales are written to each
// sorted row that reads it (its k routed slots, as the dispatch placed them, and its
// shared-expert row).  A token's 128-channel blocks quantise the same way in every expert it is
// routed to, so this equals quantising each gathered row (qwen35_layer_v2.py:578, :612), with one
// eleventh of the arithmetic and of the reads.  One CTA per token, 8 channels per thread and
// pass; a 128-channel block is 16 lanes, so its amax is a 4-step xor shuffle.
struct ScatterArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  int K, T, k;
  const int32_t* slot_row;  // [T*k] sorted row of each slot, -1 when the slot is not on this rank
  int shared_row0;          // >= 0: token t's shared-expert row is shared_row0 + t
  uint8_t* q;               // [rows, K] e4m3, sorted order
  int64_t ldq;
  float* scale;             // element (row, kb) at scale[kb * s_kb + row]
  int64_t s_kb;
  // shared-expert gate: gv[t] = bf16(sigmoid(bf16(x[t] . wg)))
  const __nv_bfloat16* gate_w;
  float* gate_val;
};

constexpr int kScatterThreads = 512;
constexpr int kScatterMaxDst = 17;  // k <= 16 routed slots + the shared-expert row

__global__ void __launch_bounds__(kScatterThreads) k_quant_scatter(ScatterArgs a) {
  pdl_wait();
  __shared__ int s_dst[kScatterMaxDst];
  __shared__ float s_dot[kScatterThreads / 32];
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x < kScatterMaxDst) {
    const int j = threadIdx.x;
    int r = -1;
    if (j < a.k) r = a.slot_row[(int64_t)t * a.k + j];
    else if (j == a.k && a.shared_row0 >= 0) r = a.shared_row0 + t;
    s_dst[j] = r;
  }
  __syncthreads();
  const int ndst = a.k + 1;
  const __nv_bfloat16* __restrict__ xr = a.x + (int64_t)t * a.ldx;
  float dot = 0.f;
  for (int c = threadIdx.x * 8; c < a.K; c += kScatterThreads * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
    float f[8];
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      f[i] = bf16_bits_to_f32(w4[i >> 1], i & 1);
      am = nanmax(am, fabsf(f[i]));
    }
    if (a.gate_w) {
      const uint4 wraw = *reinterpret_cast<const uint4*>(a.gate_w + c);
      const uint32_t g4[4] = {wraw.x, wraw.y, wraw.z, wraw.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(f[i], bf16_bits_to_f32(g4[i >> 1], i & 1), dot);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) am = nanmax(am, __shfl_xor_sync(0xffffffffu, am, o));
    // s = clamp(amax, min=1e-12) / 448 (NaN propagates as in torch.clamp)
    const float sc = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
    uint32_t packed[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = clamp_pm(__fdiv_rn(f[2 * i], sc), 448.0f);
      const float hi = clamp_pm(__fdiv_rn(f[2 * i + 1], sc), 448.0f);
      const uint16_t pr = f32x2_to_e4m3x2(lo, hi);
      if (i & 1) packed[i >> 1] |= (uint32_t)pr << 16;
      else packed[i >> 1] = pr;
    }
    const uint2 qv = make_uint2(packed[0], packed[1]);
    for (int d = 0; d < ndst; ++d) {
      const int r = s_dst[d];
      if (r < 0) continue;
      *reinterpret_cast<uint2*>(a.q + (int64_t)r * a.ldq + c) = qv;
      if ((lane & 15) == 0) a.scale[(int64_t)(c / 128) * a.s_kb + r] = sc;
    }
  }
  if (a.gate_w) {
    dot = warp_sum(dot);
    if (lane == 0) s_dot[warp] = dot;
    __syncthreads();
    if (threadIdx.x == 0) {
      float d = 0.f;
      for (int w = 0; w < kScatterThreads / 32; ++w) d += s_dot[w];
      const float lg = bf16_round(d);
      a.gate_val[t] = bf16_round(1.0f / (1.0f + expf(-lg)));
    }
  }
  pdl_trigger();
}

struct CombineArgs {
  const __nv_bfloat16* down;  // [rows, H] expert outputs in sorted-row order
  int64_t ld_down;
  const int32_t* slot_row;    // [T*k] row of each slot, -1 when not on this rank
  const int32_t* topk_ids;    // [T*k] (orders the DISPATCH / BATCHED modes)
  const void* topk_w;         // [T*k] bf16 or f32
  int w_f32;
  int T, H, k;
  int mode;                   // msv_combine_mode
  // shared expert: row (shared_row0 + t) of `down`, times gate_val[t] when gate_val != nullptr
  int add_shared;
  int shared_row0;
  const float* gate_val;
  __nv_bfloat16* out;
  int64_t ld_out;
};

constexpr int kCombineThreads = 512;  // most threads a CTA is launched with
constexpr int kCombineBatch = 8;  // slot rows loaded before any is summed

inline int combine_threads(int H) {
  const int t = ((H / 8 + 31) / 32) * 32;
  return t < kCombineThreads ? t : kCombineThreads;
}

// One token's combined row, by the whole CTA (s_row / s_w: the CTA's shared slots); each
// 8-channel piece goes to store(first channel, 4 words of packed bf16 pairs).  Each thread
// produces 8 consecutive channels per pass (one pass when H <= 4096).  Warp 0 reads the
// token's k slots in parallel (and orders them by expert id for the per-expert modes); the
// channel loop loads 8 slot rows before it sums them.
template <int MODE, class Store>
MSV_DEVICE void combine_token(const CombineArgs& a, int t, int* s_row, float* s_w, Store&& store, int c_begin = 0,
                              int c_end = -1) {
  if (c_end < 0) c_end = a.H;
  // the shared-expert gate loads first: its latency overlaps the slot setup below
  const float gv = (a.add_shared && a.gate_val) ? a.gate_val[t] : 1.0f;
  __syncthreads();  // the previous token's slots are no longer read
  if (threadIdx.x < 32) {
    const int j = threadIdx.x;
    int r = -1, id = 0x7fffffff;
    float w = 0.f;
    if (j < a.k) {
      const int64_t o = (int64_t)t * a.k + j;
      r = a.slot_row[o];
      w = a.w_f32 ? reinterpret_cast<const float*>(a.topk_w)[o]
                  : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.topk_w)[o]);
      id = a.topk_ids ? a.topk_ids[o] : j;
    }
    int pos = j;
    if (MODE != MSV_COMBINE_V2) {  // expert-ascending order of the per-expert loops
      pos = 0;
      for (int i = 0; i < a.k; ++i) {
        const int idi = __shfl_sync(0xffffffffu, id, i);
        pos += (idi < id) || (idi == id && i < j);
      }
    }
    if (j < a.k) {
      s_row[pos] = r;
      s_w[pos] = w;
    }
  }
  __syncthreads();
  for (int c = c_begin + threadIdx.x * 8; c < c_end; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    // kCombineBatch slot rows in flight at once (the shared-expert row with the first batch),
    // summed in slot order
    uint4 rsh = make_uint4(0, 0, 0, 0);
    for (int j0 = 0; j0 < a.k; j0 += kCombineBatch) {
      uint4 raw[kCombineBatch];
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        const int r = j0 + u < a.k ? s_row[j0 + u] : -1;
        raw[u] = r >= 0 ? *reinterpret_cast<const uint4*>(a.down + (int64_t)r * a.ld_down + c) : make_uint4(0, 0, 0, 0);
      }
      if (j0 == 0 && a.add_shared)
        rsh = *reinterpret_cast<const uint4*>(a.down + (int64_t)(a.shared_row0 + t) * a.ld_down + c);
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        const int j = j0 + u;
        if (j >= a.k) break;
        if (s_row[j] < 0) continue;
        const float w = s_w[j];
        const uint32_t wd[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float dv = bf16_bits_to_f32(wd[i >> 1], i & 1);
          if (MODE == MSV_COMBINE_V2) acc[i] += bf16_round(dv * w);
          // fp32 product and fp32 add rounded separately (no FMA contraction), then bf16
          else if (MODE == MSV_COMBINE_DISPATCH) acc[i] = bf16_round(__fadd_rn(acc[i], __fmul_rn(dv, w)));
          else acc[i] = bf16_round(acc[i] + bf16_round(dv * w));
        }
      }
    }
    if (a.add_shared) {
      const uint32_t wd[4] = {rsh.x, rsh.y, rsh.z, rsh.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float sd = bf16_bits_to_f32(wd[i >> 1], i & 1);
        if (a.gate_val) sd = bf16_round(sd * gv);
        acc[i] = bf16_round(bf16_round(acc[i]) + sd);
      }
    }
    uint32_t ow[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    store(c, ow);
  }
}

// One CTA per token and column slice: blockIdx.y of gridDim.y takes an equal share of the
// 8-column pieces, so small batches still spread their row loads over every SM (two CTAs per SM
// keep enough rows in flight at large batches).
template <int MODE>
__global__ void __launch_bounds__(kCombineThreads, 2) k_combine(CombineArgs a) {
  pdl_wait();
  __shared__ int s_row[16];
  __shared__ float s_w[16];
  const int t = blockIdx.x;
  __nv_bfloat16* dst = a.out + (int64_t)t * a.ld_out;
  const int pieces = a.H / 8, per = (pieces + gridDim.y - 1) / gridDim.y;
  const int c_begin = (int)blockIdx.y * per * 8;
  const int c_end = min(a.H, c_begin + per * 8);
  combine_token<MODE>(a, t, s_row, s_w, [&](int c, const uint32_t* ow) {
    *reinterpret_cast<uint4*>(dst + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }, c_begin, c_end);
  pdl_trigger();
}

// Column slices per token: enough CTAs for two per SM when the batch alone does not give them.
inline int combine_slices(int T, int H, int num_sms) {
  int s = T > 0 ? (2 * num_sms + T - 1) / T : 1;
  const int max_s = H / (8 * 32) > 0 ? H / (8 * 32) : 1;  // at least one warp of pieces per slice
  int p = 1;  // a power of two, so the slices split H / 8 pieces evenly
  while (p < s && p < 8 && p * 2 <= max_s) p *= 2;
  return p;
}

inline void launch_combine(const CombineArgs& a, cudaStream_t stream, int num_sms) {
  const int sl = combine_slices(a.T, a.H, num_sms);
  const int pieces_per = (a.H / 8 + sl - 1) / sl;
  const int th = ((pieces_per + 31) / 32) * 32;
  const dim3 grid(a.T, sl), block(th < kCombineThreads ? th : kCombineThreads);
  if (a.mode == MSV_COMBINE_V2) launch_k(k_combine<MSV_COMBINE_V2>, dim3(grid), dim3(block), 0, stream, a);
  else if (a.mode == MSV_COMBINE_DISPATCH) launch_k(k_combine<MSV_COMBINE_DISPATCH>, dim3(grid), dim3(block), 0, stream, a);
  else launch_k(k_combine<MSV_COMBINE_BATCHED>, dim3(grid), dim3(block), 0, stream, a);
}

}  // namespace msv
