// Gemma-style RMSNorm of the decoder's residual stream, with the residual add in front of it
// fused in.  Reference: muserve/model/qwen35_layer_v2.py:59-62 (rms_norm_gemma) as the decoder
// layer calls it at :713-715 (x2 = rms_norm_gemma(h, post_attention_layernorm.weight);
// h = h + moe_forward(x2)).
//
// torch's rms_norm on bf16 input computes in fp32 and rounds once:
//   w_eff = bf16(1 + float(weight)),  rstd = 1 / sqrt(sum(x^2) / H + eps),
//   out = bf16(x * rstd * float(w_eff)).
// The residual add is bf16(float(h) + float(add)).  sqrt and the division are the IEEE
// round-to-nearest forms, as on the host; the sum of squares runs in a different order than on
// the host, so rstd can differ from it by an ulp.
#pragma once
#include "common.cuh"

namespace msv {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;  // 8-element vectors per thread: H <= 8 * 8 * 256 = 16384

MSV_DEVICE float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
MSV_DEVICE float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
MSV_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// One CTA per row.  h <- bf16(h + add) when add != nullptr; out = rmsnorm(h) when out != nullptr.
__global__ void __launch_bounds__(kNormThreads) k_add_rms_norm(__nv_bfloat16* __restrict__ h,
                                                               const __nv_bfloat16* __restrict__ add,
                                                               const __nv_bfloat16* __restrict__ weight,
                                                               __nv_bfloat16* __restrict__ out, int H, float eps) {
  pdl_wait();
  __shared__ float s_part[kNormThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nv = H >> 3;
  const int64_t rbase = (int64_t)blockIdx.x * H;
  uint4* hrow = reinterpret_cast<uint4*>(h + rbase);
  const uint4* arow = add ? reinterpret_cast<const uint4*>(add + rbase) : nullptr;
  uint4 hv[kNormMaxVec];
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = tid + j * kNormThreads;
    hv[j] = c < nv ? hrow[c] : make_uint4(0, 0, 0, 0);
  }
  if (arow) {
    uint4 av[kNormMaxVec];
#pragma unroll
    for (int j = 0; j < kNormMaxVec; ++j) {
      const int c = tid + j * kNormThreads;
      av[j] = c < nv ? arow[c] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kNormMaxVec; ++j) {
      const int c = tid + j * kNormThreads;
      if (c < nv) {
        uint32_t* x = reinterpret_cast<uint32_t*>(&hv[j]);
        const uint32_t* y = reinterpret_cast<const uint32_t*>(&av[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          x[q] = pack_bf16x2(bf16_lo(x[q]) + bf16_lo(y[q]), bf16_hi(x[q]) + bf16_hi(y[q]));
        hrow[c] = hv[j];
      }
    }
  }
  if (!out) {
    pdl_trigger();
    return;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const uint32_t* x = reinterpret_cast<const uint32_t*>(&hv[j]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = bf16_lo(x[q]), b = bf16_hi(x[q]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) s_part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[w];
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
  const uint4* wrow = reinterpret_cast<const uint4*>(weight);
  uint4* orow = reinterpret_cast<uint4*>(out + rbase);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    const int c = tid + j * kNormThreads;
    if (c < nv) {
      const uint4 wv = wrow[c];
      const uint32_t* x = reinterpret_cast<const uint32_t*>(&hv[j]);
      const uint32_t* wq = reinterpret_cast<const uint32_t*>(&wv);
      uint4 ov;
      uint32_t* o = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // w_eff = bf16(1 + weight), then x * rstd * w_eff in fp32 with one rounding
        const float w0 = __bfloat162float(__float2bfloat16_rn(1.0f + bf16_lo(wq[q])));
        const float w1 = __bfloat162float(__float2bfloat16_rn(1.0f + bf16_hi(wq[q])));
        o[q] = pack_bf16x2(__fmul_rn(__fmul_rn(bf16_lo(x[q]), rstd), w0),
                           __fmul_rn(__fmul_rn(bf16_hi(x[q]), rstd), w1));
      }
      orow[c] = ov;
    }
  }
  pdl_trigger();
}

}  // namespace msv
