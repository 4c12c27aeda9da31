// Grouped (ragged-M) block-scaled e4m3 GEMM on 5th-generation tensor cores.
//
// Math (per output row m of group g, weight row n):
//   D[m, n] = sum_kb ( sum_{k in kb} A[m,k] W[e_g, n, k] ) * a_scale[m, kb] * w_scale[e_g, n/128, kb]
// which is mate.gemm.ragged_m_moe_gemm_8bit / gemm_fp8_nt_groupwise as called from
// muserve/model/qwen35_layer_v2.py:102-106, 613-618, 638-643.
//
// Shape of the work ("swap AB").  The 128 weight rows of an n-block fill the MMA's M=128
// side and a group's tokens form N (16..BN, multiple of 16), so an expert with 1 token
// (decode) or 160 tokens (prefill) pays no M padding and each weight tile is streamed from
// HBM once per token chunk.  A tile = (group, n-block, token chunk); the tile list is built
// on the device, the kernel is persistent (one CTA per SM, static round robin over tiles).
//
// Roles (warp-specialised, one CTA per SM):
//   warp 0      TMA producer: per 128-wide K block, NACC weight boxes [128 x 128 B] and one
//               token box [BN x 128 B], 128-byte swizzle, into an NSTAGE ring.
//   warp 1      MMA issuer: tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> fp32), 4 x K=32 per K
//               block, into a fresh TMEM buffer per K block (NBUF-deep ring); also stages the
//               K block's scales (a_scale[row] * w_scale) in shared memory; owns TMEM alloc.
//   warps 4..   epilogue warpgroups: per K block, tcgen05.ld the partial product, multiply by
//               the staged scales and accumulate in fp32 registers (the 128x128 fp32 scales
//               are arbitrary, so the scale cannot be folded into a UE8M0 block-scaled MMA);
//               at tile end write bf16 (EPI 0), or SwiGLU + per-128 e4m3 requant (EPI 1:
//               acc 0 = gate rows, acc 1 = up rows of the same 128 channels).
// Every wait is bounded (common.cuh); on timeout the CTA drains its copies and MMAs, frees
// TMEM and raises MSV_ERR_TIMEOUT in the error word.
#pragma once
#include "common.cuh"

namespace msv {

struct GemmArgs {
  CUtensorMap tmA[2][2];  // [weight set: 0 routed, 1 shared][acc]
  CUtensorMap tmB;        // activations [rows, K] e4m3
  int a_expert_rows[2];   // rows between consecutive experts in the A maps
  const float* ws[2][2];  // weight-scale base [set][acc]
  int64_t ws_expert_stride[2];
  int ws_nb_stride;       // floats between n-block rows of the scale matrix (= K/128)
  const float* as;        // activation scales: element (row, kb) at as[row*as_row + kb*as_kb]
  int64_t as_row, as_kb;
  const int4* tiles;      // {row0, rows, set<<24 | expert, n-block}
  const int* num_tiles;
  int num_kb;
  void* out;              // EPI 0: bf16 [rows, out_ld]; EPI 1: e4m3 [rows, out_ld]
  int64_t out_ld;
  float* out_scale;       // EPI 1: element (row, n-block) at out_scale[row*os_row + nb*os_kb]
  int64_t os_row, os_kb;
  int* err;
};

template <int BN_, int NACC_, int EPI_, int NWG_>
struct GemmCfg {
  static constexpr int BN = BN_, NACC = NACC_, EPI = EPI_, NWG = NWG_;
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = NACC * A_BYTES + B_BYTES;
  static constexpr int NBUF_RAW = 512 / (NACC * BN);
  static constexpr int NBUF = NBUF_RAW > 4 ? 4 : NBUF_RAW;
  static constexpr int COLS_USED = NBUF * NACC * BN;
  static constexpr int TMEM_COLS = COLS_USED <= 32 ? 32 : COLS_USED <= 64 ? 64 : COLS_USED <= 128 ? 128
                                   : COLS_USED <= 256 ? 256 : 512;
  static constexpr int CW = BN / NWG;
  static constexpr int THREADS = 128 + 128 * NWG;
  static constexpr int SCL_BYTES = NBUF * NACC * BN * 4;
  static constexpr int RED_BYTES = EPI == 1 ? NWG * 4 * CW * 4 : 0;
  static constexpr int TAIL_BYTES = SCL_BYTES + RED_BYTES + 64 * 8 + 64;
  static constexpr int SMEM_LIMIT = 232448 - 1024;  // 227 KB opt-in, minus alignment slack
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - TAIL_BYTES) / STAGE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > 12 ? 12 : NSTAGE_RAW;
  static constexpr int OFF_SCL = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_RED = OFF_SCL + SCL_BYTES;
  static constexpr int OFF_BAR = (OFF_RED + RED_BYTES + 7) & ~7;
  static constexpr int NBARS = 2 * NSTAGE + 2 * NBUF + 1 + NWG;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(CW % 16 == 0, "column slice must be whole 16-column TMEM loads");
  static_assert(NBUF >= 2, "need at least double-buffered TMEM partials");
  static_assert(NSTAGE >= 2, "pipeline too shallow");
  static_assert(SMEM_BYTES <= 232448, "shared memory over the sm_100 limit");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
};

MSV_DEVICE bool wait_plain(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
  unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > limit_ns) return false;
  return true;
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) k_grouped_gemm(const __grid_constant__ GemmArgs args) {
  constexpr int BN = C::BN, NACC = C::NACC, NSTAGE = C::NSTAGE, NBUF = C::NBUF, CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* scl = reinterpret_cast<float*>(smem + C::OFF_SCL);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + NBUF;
  uint64_t* drain = acce + NBUF;
  uint64_t* epib = drain + 1;  // per epilogue warpgroup: 4 warps meet here (bounded)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&accf[b], 2);           // MMA commit + scale staging
      mbar_init(&acce[b], 4 * C::NWG);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    for (int g = 0; g < C::NWG; ++g) mbar_init(&epib[g], 4);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tmB);
    tma_prefetch_desc(&args.tmA[0][0]);
  }
  if (warp == 1) tmem_alloc(s_tmem, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int ntiles = *args.num_tiles;
  const int nkb = args.num_kb;

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      uint32_t it = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
        const int4 td = args.tiles[tile];
        const int set = td.z >> 24, e = td.z & 0xFFFFFF;
        const int arow = e * args.a_expert_rows[set] + td.w * 128;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % NSTAGE;
          const uint32_t ph = (it / NSTAGE) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, s_abort)) {
            alive = false;
            break;
          }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
#pragma unroll
          for (int a = 0; a < NACC; ++a) tma_load_2d(st + a * C::A_BYTES, &args.tmA[set][a], &full[s], kb * 128, arow);
          tma_load_2d(st + NACC * C::A_BYTES, &args.tmB, &full[s], kb * 128, td.x);
          ++it;
        }
      }
      // no bulk copy into this CTA's shared memory may outlive the CTA
      const uint32_t first = it > (uint32_t)NSTAGE ? it - NSTAGE : 0;
      for (uint32_t j = first; j < it; ++j) wait_plain(&full[j % NSTAGE], (j / NSTAGE) & 1, kWaitTimeoutNs);
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer + scale staging ─────────────
    uint32_t it = 0, ait = 0;
    bool alive = true;
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      const int4 td = args.tiles[tile];
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      const int nr = td.y;
      int n_eff = (nr + 15) & ~15;
      n_eff = n_eff < 16 ? 16 : (n_eff > BN ? BN : n_eff);
      const uint32_t idesc = umma_idesc_e4m3(128, n_eff);
      const float* ws0 = args.ws[set][0] + e * args.ws_expert_stride[set] + td.w * args.ws_nb_stride;
      const float* ws1 = NACC > 1 ? args.ws[set][NACC - 1] + e * args.ws_expert_stride[set] + td.w * args.ws_nb_stride
                                  : ws0;
      for (int kb = 0; kb < nkb; ++kb) {
        float asv[BN / 32];
#pragma unroll
        for (int j = 0; j < BN / 32; ++j) {
          const int r = lane + 32 * j;
          asv[j] = r < nr ? __ldg(args.as + (int64_t)(td.x + r) * args.as_row + (int64_t)kb * args.as_kb) : 0.f;
        }
        const float wsv = lane == 0 ? __ldg(ws0 + kb) : (lane == 1 ? __ldg(ws1 + kb) : 0.f);
        const int b = ait % NBUF;
        const uint32_t aph = (ait / NBUF) & 1;
        if (!mbar_wait(&acce[b], aph ^ 1, s_abort)) {
          alive = false;
          break;
        }
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const float w = __shfl_sync(0xffffffffu, wsv, a);
#pragma unroll
          for (int j = 0; j < BN / 32; ++j) scl[(b * NACC + a) * BN + lane + 32 * j] = asv[j] * w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&accf[b]);
        const int s = it % NSTAGE;
        const uint32_t ph = (it / NSTAGE) & 1;
        if (!mbar_wait(&full[s], ph, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          uint8_t* st = smem + s * C::STAGE_BYTES;
          const uint64_t bdesc = umma_desc_sw128(smem_u32(st + NACC * C::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
              const uint64_t adesc = umma_desc_sw128(smem_u32(st + a * C::A_BYTES));
              umma_f8(tmem + (uint32_t)((b * NACC + a) * BN), adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
          umma_commit(&accf[b]);
        }
        __syncwarp();
        ++it;
        ++ait;
      }
    }
    // every MMA must have completed before TMEM is released
    if (lane == 0) {
      umma_commit(drain);
      wait_plain(drain, 0, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ───────────── epilogue warpgroups ─────────────
    const int ew = warp - 4, wg = ew >> 2, q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    uint32_t ait = 0, ephase = 0;
    bool alive = true;
    // the 4 warps of this warpgroup meet (bounded) before and after sharing the amax slots
    auto wg_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&epib[wg]);
      const bool ok = mbar_wait(&epib[wg], ephase, s_abort);
      ephase ^= 1;
      return ok;
    };
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      const int4 td = args.tiles[tile];
      const int nr = td.y;
      int n_eff = (nr + 15) & ~15;
      n_eff = n_eff < 16 ? 16 : (n_eff > BN ? BN : n_eff);
      float acc[NACC][CW];
#pragma unroll
      for (int a = 0; a < NACC; ++a)
#pragma unroll
        for (int c = 0; c < CW; ++c) acc[a][c] = 0.f;
      for (int kb = 0; kb < nkb; ++kb) {
        const int b = ait % NBUF;
        const uint32_t aph = (ait / NBUF) & 1;
        if (!mbar_wait(&accf[b], aph, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
#pragma unroll
          for (int cc = 0; cc < CW / 16; ++cc) {
            const int col = wg * CW + cc * 16;
            if (col < n_eff) {
              float pv[16];
              tmem_ld16(tmem + tlane + (uint32_t)((b * NACC + a) * BN + col), pv);
              tmem_ld_wait();
              const float4* sc4 = reinterpret_cast<const float4*>(scl + (b * NACC + a) * BN + col);
#pragma unroll
              for (int i4 = 0; i4 < 4; ++i4) {
                const float4 s4 = sc4[i4];
                acc[a][cc * 16 + i4 * 4 + 0] = fmaf(pv[i4 * 4 + 0], s4.x, acc[a][cc * 16 + i4 * 4 + 0]);
                acc[a][cc * 16 + i4 * 4 + 1] = fmaf(pv[i4 * 4 + 1], s4.y, acc[a][cc * 16 + i4 * 4 + 1]);
                acc[a][cc * 16 + i4 * 4 + 2] = fmaf(pv[i4 * 4 + 2], s4.z, acc[a][cc * 16 + i4 * 4 + 2]);
                acc[a][cc * 16 + i4 * 4 + 3] = fmaf(pv[i4 * 4 + 3], s4.w, acc[a][cc * 16 + i4 * 4 + 3]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[b]);
        ++ait;
      }
      if (!alive) break;
      const int64_t row0 = td.x;
      const int ncol = td.w * 128 + lrow;
      if constexpr (C::EPI == 0) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          const int t = wg * CW + c;
          if (t < nr) out[(row0 + t) * args.out_ld + ncol] = __float2bfloat16_rn(acc[0][c]);
        }
      } else {
        // SwiGLU exactly as the reference rounds it: gate/up GEMM outputs are bf16
        // (gate_up_out, :610-619), silu() rounds to bf16, the product rounds to bf16 (:624);
        // then _fast_fp8_quantize over these 128 channels (:637).
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          const float g = bf16_round(acc[0][c]);
          const float u = bf16_round(acc[NACC - 1][c]);
          const float sl = bf16_round(__fdiv_rn(g, 1.0f + expf(-g)));
          const float av = bf16_round(sl * u);
          acc[0][c] = av;
          const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(av)));
          if (lane == 0) red[(wg * 4 + q) * CW + c] = __uint_as_float(m);
        }
        if (!wg_sync()) break;
        uint8_t* outq = reinterpret_cast<uint8_t*>(args.out);
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          const int t = wg * CW + c;
          const float* rr = red + wg * 4 * CW + c;
          const float am = nanmax(nanmax(rr[0], rr[CW]), nanmax(rr[2 * CW], rr[3 * CW]));
          const float s = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
          if (t < nr) {
            const float qv = clamp_pm(__fdiv_rn(acc[0][c], s), 448.0f);
            outq[(row0 + t) * args.out_ld + ncol] = (uint8_t)(f32x2_to_e4m3x2(qv, 0.f) & 0xFF);
            if (lrow == 0) args.out_scale[(row0 + t) * args.os_row + (int64_t)td.w * args.os_kb] = s;
          }
        }
        if (!wg_sync()) break;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *s_abort) atomicExch(args.err, (int)MSV_ERR_TIMEOUT);
}

}  // namespace msv
