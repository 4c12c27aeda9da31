// Weighted combine fused with the tensor-parallel all-reduce over NVLink peer memory.
// Reference: muserve/model/qwen35_layer_v2.py:657-662 (the per-rank [T,H] result, summed
// over the TP group by muserve/distributed.py:62-64 all_reduce).
//
// Every rank runs the same persistent grid of G CTAs (G <= SMs, so all of them are resident and
// a CTA never waits for one that cannot be scheduled).  CTA b owns tokens b, b + G, ...:
//   1. it combines its tokens into this rank's partial buffer (local stores);
//   2. round 1: it raises its flag in every rank's flag area and waits until every rank's CTA b
//      has raised its own (all partial rows of its tokens exist on every rank);
//   3. reduce-scatter + all-gather: this rank sums its H/W-column slice of those rows over the
//      W partial buffers (peer loads, rank order 0..W-1, fp32, one bf16 rounding: identical bits
//      on every rank) and stores the result into every rank's gather buffer (peer stores);
//   4. round 2: the same flag exchange (every slice of its tokens has arrived here);
//   5. it copies its tokens' rows from the gather buffer to the output.
// Flags carry a per-CTA call counter (epoch), kept in this rank's device memory and advanced by
// the CTA itself, so a captured CUDA graph replays correctly.  A rank can only reuse a buffer
// row after every rank has passed the round that ends all reads of it, so consecutive calls do
// not race.  Every wait gives up after kWaitTimeoutNs and raises MSV_ERR_TIMEOUT in the error
// word; the CTA then skips the rest of its work instead of hanging.
#pragma once
#include "common.cuh"
#include "quant_combine.cuh"

namespace msv {

constexpr int kMaxTpRanks = 8;
constexpr int kArMaxCtas = 1024;  // flag slots per rank and round

struct CombineArArgs {
  CombineArgs c;                          // combine inputs; c.out is the final output
  __nv_bfloat16* part[kMaxTpRanks];       // each rank's partial buffer [max_tokens, H]
  __nv_bfloat16* gath[kMaxTpRanks];       // each rank's gathered-result buffer [max_tokens, H]
  unsigned int* flags[kMaxTpRanks];       // each rank's flags [2][kMaxTpRanks][kArMaxCtas]
  unsigned int* epoch;                    // this rank's per-CTA call counters [kArMaxCtas]
  int world, rank;
  int* err;
};

MSV_DEVICE void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MSV_DEVICE unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Round `round` of CTA b: publish this CTA's flag on every rank, then wait for every rank's.
// Returns false (with the error word raised) when a wait ran out.  Called by the whole CTA.
MSV_DEVICE bool ar_exchange(const CombineArArgs& a, int round, unsigned int e, bool* s_ok) {
  __syncthreads();  // this CTA's stores (and, in round 2, its peer loads) are done
  if (threadIdx.x == 0) {
    bool ok = true;
    __threadfence_system();
    for (int p = 0; p < a.world; ++p)
      st_release_sys(a.flags[p] + (round * kMaxTpRanks + a.rank) * kArMaxCtas + blockIdx.x, e);
    const unsigned int* mine = a.flags[a.rank] + round * kMaxTpRanks * kArMaxCtas + blockIdx.x;
    const unsigned long long t0 = globaltimer();
    for (int p = 0; p < a.world && ok; ++p) {
      while (ld_acquire_sys(mine + p * kArMaxCtas) != e) {
        if (globaltimer() - t0 > kWaitTimeoutNs) {
          atomicExch(a.err, (int)MSV_ERR_TIMEOUT);
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok;
}

template <int MODE>
__global__ void __launch_bounds__(kCombineThreads, 1) k_combine_ar(CombineArArgs a) {
  pdl_wait();
  __shared__ int s_row[16];
  __shared__ float s_w[16];
  __shared__ bool s_ok;
  __shared__ unsigned int s_epoch;
  const CombineArgs& c = a.c;
  const int G = gridDim.x;
  if (threadIdx.x == 0) s_epoch = a.epoch[blockIdx.x] + 1u;
  // 1. combine this CTA's tokens into this rank's partial buffer
  __nv_bfloat16* mine = a.part[a.rank];
  for (int t = blockIdx.x; t < c.T; t += G) combine_token<MODE>(c, t, s_row, s_w, mine + (int64_t)t * c.H);
  __syncthreads();
  const unsigned int e = s_epoch;
  // 2. every rank's partial rows of these tokens are written
  if (!ar_exchange(a, 0, e, &s_ok)) return;
  // 3. this rank's column slice, summed over the ranks in rank order, sent to every rank
  const int hs = c.H / a.world;   // columns per rank, a multiple of 8
  const int c0 = a.rank * hs;
  const int vec_per_row = hs / 8;  // 16-byte vectors of the slice
  const int ntok = (c.T - blockIdx.x + G - 1) / G;
  for (int i = threadIdx.x; i < ntok * vec_per_row; i += blockDim.x) {
    const int t = blockIdx.x + (i / vec_per_row) * G;
    const int64_t off = (int64_t)t * c.H + c0 + (i % vec_per_row) * 8;
    uint4 raw[kMaxTpRanks];
#pragma unroll
    for (int p = 0; p < kMaxTpRanks; ++p)
      if (p < a.world) raw[p] = *reinterpret_cast<const uint4*>(a.part[p] + off);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxTpRanks; ++p) {
      if (p < a.world) {
        const uint32_t w4[4] = {raw[p].x, raw[p].y, raw[p].z, raw[p].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += bf16_bits_to_f32(w4[j >> 1], j & 1);
      }
    }
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 pr = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      ow[j] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    const uint4 o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
#pragma unroll
    for (int p = 0; p < kMaxTpRanks; ++p)
      if (p < a.world) *reinterpret_cast<uint4*>(a.gath[p] + off) = o;
  }
  // 4. every rank's slice of these tokens has arrived in this rank's gather buffer
  if (!ar_exchange(a, 1, e, &s_ok)) return;
  // 5. the gathered rows to the output
  const __nv_bfloat16* g = a.gath[a.rank];
  const int vec_row = c.H / 8;
  for (int i = threadIdx.x; i < ntok * vec_row; i += blockDim.x) {
    const int t = blockIdx.x + (i / vec_row) * G;
    const int v = i % vec_row;
    *reinterpret_cast<uint4*>(c.out + (int64_t)t * c.ld_out + v * 8) =
        *reinterpret_cast<const uint4*>(g + (int64_t)t * c.H + v * 8);
  }
  if (threadIdx.x == 0) a.epoch[blockIdx.x] = e;
  pdl_trigger();
}

}  // namespace msv
