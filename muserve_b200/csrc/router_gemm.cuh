// Router logits on the tensor cores: partial[s][t][e] = sum over K split s of hidden[t,k] *
// gate_w[e,k], bf16 x bf16 -> fp32 (tcgen05 kind::f16, accumulators in TMEM).  The routing
// kernel (route.cuh) sums the splits in a fixed order, rounds to bf16 where the caller's
// reference does (qwen35_layer_v2.py:567-568, bf16_linear(...).float()), and runs softmax / top-k.
//
// Tile = 128 tokens (MMA M, TMEM lanes) x up to 256 experts (MMA N, TMEM columns) x one K split;
// grid (token tiles, expert tiles, splits).  Small batches split K so that the 4 MB gate weight is
// read by enough SMs (decode: 64 tokens, 2 expert tiles, 32 splits); large batches do not split.
// A K block is 64 bf16 (one 128-byte swizzle row): per stage a 16 KB token box and a 32 KB weight
// box, four K=16 MMAs.  Roles: warp 0 lane 0 TMA producer, warp 1 lane 0 MMA issuer (warp 1
// also owns TMEM); all four warps write the tile's fp32 partials (lane = token row).
// Every wait is bounded.
#pragma once
#include "common.cuh"
#include "grouped_gemm.cuh"

namespace msv {

struct RouterArgs {
  CUtensorMap tmA;  // hidden [T, H] bf16, box 64 x 128 rows, 128-byte swizzle
  CUtensorMap tmB;  // gate   [E, H] bf16, box 64 x 256 rows, 128-byte swizzle
  int T, H, E;
  int kb_per_split;  // 64-wide K blocks per split
  int round_bf16;    // one split: round to bf16 here (part is then the logits)
  float* part;       // [splits][T][E]
  int* err;
};

constexpr int kRtBM = 128, kRtBN = 256, kRtStages = 4;
constexpr int kRtABytes = kRtBM * 128, kRtBBytes = kRtBN * 128, kRtStageBytes = kRtABytes + kRtBBytes;
constexpr int kRtSmem = kRtStages * kRtStageBytes + 1024;

// tcgen05 instruction descriptor, kind::f16 with bf16 A and B, fp32 D, both K-major.
MSV_DEVICE uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

MSV_DEVICE void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__global__ void __launch_bounds__(128, 1) k_router_gemm(const __grid_constant__ RouterArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kRtStages], empty[kRtStages], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kRtBM, n0 = blockIdx.y * kRtBN, split = blockIdx.z;
  const int n = min(kRtBN, a.E - n0);  // multiple of 16
  const int nkb = a.H / 64;
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(nkb, kb0 + a.kb_per_split);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&a.tmA);
    tma_prefetch_desc(&a.tmB);
  }
  if (warp == 1) tmem_alloc(&s_tmem, kRtBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_wait();
  if (warp == 0) {
    if (lane == 0) {
      Ring<kRtStages> st;
      uint32_t issued = 0;
      for (int kb = kb0; kb < kb1; ++kb, st.next(), ++issued) {
        if (!mbar_wait(&empty[st.i], st.ph ^ 1, &s_abort)) break;
        uint8_t* sp = smem + st.i * kRtStageBytes;
        mbar_arrive_expect_tx(&full[st.i], kRtStageBytes);
        tma_load_2d(sp, &a.tmA, &full[st.i], kb * 64, m0);
        tma_load_2d(sp + kRtABytes, &a.tmB, &full[st.i], kb * 64, n0);
      }
      // no copy into this CTA's shared memory may outlive the CTA
      const uint32_t first = issued > (uint32_t)kRtStages ? issued - kRtStages : 0;
      for (uint32_t q = first; q < issued; ++q) wait_plain(&full[q % kRtStages], (q / kRtStages) & 1, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      Ring<kRtStages> st;
      const uint32_t idesc = umma_idesc_bf16(kRtBM, n);
      for (int kb = kb0; kb < kb1; ++kb, st.next()) {
        if (!mbar_wait(&full[st.i], st.ph, &s_abort)) break;
        tc_fence_after();
        uint8_t* sp = smem + st.i * kRtStageBytes;
        const uint64_t adesc = umma_desc_sw128(smem_u32(sp));
        const uint64_t bdesc = umma_desc_sw128(smem_u32(sp + kRtABytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[st.i]);
      }
      umma_commit(&done);  // also when the split is empty or aborted: nothing left in flight
    }
    __syncwarp();
  }
  // every warp: the tile's partials (lane = token row), 32 columns per TMEM load
  const bool waited = mbar_wait(&done, 0, &s_abort);
  // warp-uniform: tcgen05.ld is a warp-collective instruction
  const bool ok = __all_sync(0xffffffffu, waited && !s_abort && kb1 > kb0);
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  float* out = a.part + ((int64_t)split * a.T + row) * a.E + n0;
  for (int c = 0; c < n; c += 32) {
    float v[32];
    if (ok) {
      tmem_ld32(tl + (uint32_t)c, v);
      tmem_ld_wait();
      if (a.round_bf16)
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
    if (row < a.T) {
      // n - c is 16 or at least 32 (n is a multiple of 16)
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        if (c + j < n) *reinterpret_cast<float4*>(out + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kRtBN);
  }
  if (threadIdx.x == 0 && s_abort) atomicExch(a.err, (int)MSV_ERR_TIMEOUT);
  pdl_trigger();
}

// logits[t][e] = sum over splits s (in order) of part[s][t][e], rounded to bf16 when asked;
// four consecutive experts per thread, coalesced 16-byte loads, the split loads in flight
// together.  T * E is a multiple of 4 (E % 16 == 0).
__global__ void __launch_bounds__(256) k_router_sum_splits(const float* __restrict__ part, int nsplit, int64_t n4,
                                                           int round_bf16, float* __restrict__ logits) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4* p = reinterpret_cast<const float4*>(part) + i;
  float4 acc = p[0];
  int sp = 1;
  for (; sp + 4 <= nsplit; sp += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = p[(int64_t)(sp + u) * n4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc.x += v[u].x;
      acc.y += v[u].y;
      acc.z += v[u].z;
      acc.w += v[u].w;
    }
  }
  for (; sp < nsplit; ++sp) {
    const float4 v = p[(int64_t)sp * n4];
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  if (round_bf16) {
    acc.x = bf16_round(acc.x);
    acc.y = bf16_round(acc.y);
    acc.z = bf16_round(acc.z);
    acc.w = bf16_round(acc.w);
  }
  reinterpret_cast<float4*>(logits)[i] = acc;
  pdl_trigger();
}

}  // namespace msv
