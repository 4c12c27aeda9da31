// Weighted combine fused with the tensor-parallel all-reduce over NVLink peer memory.
// Reference: muserve/model/qwen35_layer_v2.py:657-662 (the per-rank [T,H] result, summed
// over the TP group by muserve/distributed.py:62-64 all_reduce).
//
// Data moves as self-validating 8-byte words: two bf16 values and a 32-bit flag, written and
// read as whole 64-bit elements, so a reader that sees the flag of this call sees its data, and
// no fence or separate flag exchange is needed.  Rank p owns the column slice
// [p*H/W, (p+1)*H/W).  Every rank runs the same persistent grid of G CTAs (at most what the
// SMs hold at once: all resident), and CTA b handles tokens b, b + G, ... on every rank:
//   A. it combines its tokens and pushes each 8-column piece to the piece's owner, into the
//      owner's receive area at (source rank, token, column) (peer stores);
//   B. for its tokens and this rank's slice, it waits for the W sources' words, sums them in
//      rank order 0..W-1 in fp32 with one bf16 rounding (identical bits on every rank), and
//      pushes the result to every rank's result area (peer stores);
//   C. it waits for its tokens' full rows in this rank's result area and writes the output.
// The flag is a per-CTA call counter (epoch) kept in this rank's device memory and advanced by
// the CTA itself, identical on all ranks, so a captured CUDA graph replays correctly.  This
// needs a fixed token-to-CTA mapping on a group: G = min(T, cap) with a cap that is the same
// for every call (the host takes the smallest occupancy over the three combine modes at the
// group's H), so token t is always handled by CTA t mod cap and every slot of token t only
// ever carries that CTA's counter values, whatever T or the combine mode of a call.  Reuse is
// ordered by the data: a rank writes a receive slot of call n+1 only after it has received the
// owner's call-n result, which the owner computed from that slot, and it writes a result slot of
// call n+1 only after every rank's call-n+1 pieces reached it, which each rank sends after
// reading its call-n result.  Every wait gives up after kWaitTimeoutNs, raises MSV_ERR_TIMEOUT
// in the error word and ends the CTA's work instead of hanging.
#pragma once
#include "common.cuh"
#include "quant_combine.cuh"

namespace msv {

constexpr int kMaxTpRanks = 8;
constexpr int kArMaxCtas = 1024;  // per-CTA epoch counters

struct CombineArArgs {
  CombineArgs c;                    // combine inputs; c.out is the final output
  uint64_t* recv[kMaxTpRanks];      // each rank's receive area [W][max_tokens][H/W/2] words
  uint64_t* res[kMaxTpRanks];       // each rank's result area [max_tokens][H/2] words
  unsigned int* epoch;              // this rank's per-CTA call counters [kArMaxCtas]
  int world, rank, max_tokens;
  int* err;
};

// two words {flag:data} as one 16-byte store of two 64-bit elements (each element atomic)
MSV_DEVICE void st_ll2(uint64_t* p, uint32_t d0, uint32_t d1, uint32_t f) {
  const uint64_t a = ((uint64_t)f << 32) | d0, b = ((uint64_t)f << 32) | d1;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

// Wait until both words at p carry flag f; their data in d0, d1.  False when the wait ran out
// (or another thread of the CTA gave up): the error word is raised once.
MSV_DEVICE bool ld_ll2(const uint64_t* p, uint32_t f, uint32_t& d0, uint32_t& d1, unsigned long long t0,
                       volatile int* s_abort, int* err) {
  uint64_t a, b;
  for (unsigned it = 0;; ++it) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    if ((uint32_t)(a >> 32) == f && (uint32_t)(b >> 32) == f) break;
    if ((it & 255) == 255) {
      if (*s_abort) return false;
      if (globaltimer() - t0 > kWaitTimeoutNs) {
        *s_abort = 1;
        atomicExch(err, (int)MSV_ERR_TIMEOUT);
        return false;
      }
    }
  }
  d0 = (uint32_t)a;
  d1 = (uint32_t)b;
  return true;
}

template <int MODE>
__global__ void __launch_bounds__(kCombineThreads, 2) k_combine_ar(CombineArArgs a) {
  pdl_wait();
  __shared__ int s_row[16];
  __shared__ float s_w[16];
  __shared__ unsigned int s_epoch;
  __shared__ int s_abort;
  const CombineArgs& c = a.c;
  const int G = gridDim.x, W = a.world, H = c.H;
  const int hs = H / W;  // columns per owner, a multiple of 8
  if (threadIdx.x == 0) {
    s_epoch = a.epoch[blockIdx.x] + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  // A. combine this CTA's tokens; each 8-column piece goes to its owner's receive area
  for (int t = blockIdx.x; t < c.T; t += G) {
    combine_token<MODE>(c, t, s_row, s_w, [&](int col, const uint32_t* ow) {
      const int s = col / hs, cc = col - s * hs;
      uint64_t* p = a.recv[s] + (((int64_t)a.rank * a.max_tokens + t) * hs + cc) / 2;
      st_ll2(p, ow[0], ow[1], e);
      st_ll2(p + 2, ow[2], ow[3], e);
    });
  }
  const unsigned long long t0 = globaltimer();
  // B. this rank's slice of these tokens: the W sources summed in rank order, sent to every rank
  const int ntok = (c.T - blockIdx.x + G - 1) / G;
  const int vps = hs / 8;  // 8-column pieces per slice
  bool ok = true;
  for (int i = threadIdx.x; i < ntok * vps && ok; i += blockDim.x) {
    const int t = blockIdx.x + (i / vps) * G;
    const int cc = (i % vps) * 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int p = 0; p < W && ok; ++p) {
      const uint64_t* src = a.recv[a.rank] + (((int64_t)p * a.max_tokens + t) * hs + cc) / 2;
      uint32_t d[4];
      ok = ld_ll2(src, e, d[0], d[1], t0, &s_abort, a.err) && ld_ll2(src + 2, e, d[2], d[3], t0, &s_abort, a.err);
      if (ok) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += bf16_bits_to_f32(d[j >> 1], j & 1);
      }
    }
    if (!ok) break;
    uint32_t ow[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 pr = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      ow[j] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    const int64_t w0 = ((int64_t)t * H + a.rank * hs + cc) / 2;
    for (int q = 0; q < W; ++q) {
      st_ll2(a.res[q] + w0, ow[0], ow[1], e);
      st_ll2(a.res[q] + w0 + 2, ow[2], ow[3], e);
    }
  }
  // C. these tokens' full rows from this rank's result area to the output
  const int vpr = H / 8;
  for (int i = threadIdx.x; i < ntok * vpr && ok; i += blockDim.x) {
    const int t = blockIdx.x + (i / vpr) * G;
    const int col = (i % vpr) * 8;
    const uint64_t* src = a.res[a.rank] + ((int64_t)t * H + col) / 2;
    uint32_t d[4];
    ok = ld_ll2(src, e, d[0], d[1], t0, &s_abort, a.err) && ld_ll2(src + 2, e, d[2], d[3], t0, &s_abort, a.err);
    if (ok) *reinterpret_cast<uint4*>(c.out + (int64_t)t * c.ld_out + col) = make_uint4(d[0], d[1], d[2], d[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0 && !s_abort) a.epoch[blockIdx.x] = e;
  pdl_trigger();
}

}  // namespace msv
