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
  static constexpr int SCL_BYTES = 0;
  static constexpr int RED_BYTES = EPI == 1 ? NWG * 4 * CW * 4 : 0;
  static constexpr int SLOT_FLOATS = BN + 4;  // per K-block step: a_scale of the chunk's rows, then w_scale per acc
  static constexpr int NSLOT_MAX = 20;
  static constexpr int TAIL_BYTES = SCL_BYTES + RED_BYTES + 128 * 8 + 64 + NSLOT_MAX * SLOT_FLOATS * 4;
  static constexpr int SMEM_LIMIT = 232448 - 1024;  // 227 KB opt-in, minus alignment slack
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - TAIL_BYTES) / STAGE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > 12 ? 12 : NSTAGE_RAW;
  static constexpr int OFF_SCL = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_RED = OFF_SCL + SCL_BYTES;
  // scale slots outlive their smem stage (the epilogue reads them after the MMA released the
  // stage), so they form their own ring with ready/free barriers
  static constexpr int NSLOT = NSTAGE + NBUF + 2 <= NSLOT_MAX ? NSTAGE + NBUF + 2 : NSLOT_MAX;
  static constexpr int OFF_SLOT = OFF_RED + RED_BYTES;
  static constexpr int OFF_BAR = (OFF_SLOT + NSLOT * SLOT_FLOATS * 4 + 7) & ~7;
  static constexpr int NISSUE = 2;  // MMA-issuing warps (1, 2), taking alternate K blocks
  static constexpr int NBARS = 2 * NSTAGE + 2 * NBUF + NISSUE + NWG + 2 * NSLOT;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(CW % 32 == 0, "column slice must be whole 32-column TMEM loads");
  static_assert(NBUF >= 2, "need at least double-buffered TMEM partials");
  static_assert(NSTAGE >= 2, "pipeline too shallow");
  static_assert(NSLOT > NSTAGE + NBUF, "scale ring must outlast the stage ring plus the TMEM ring");
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
  float* slots = reinterpret_cast<float*>(smem + C::OFF_SLOT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + NBUF;
  uint64_t* drain = acce + NBUF;      // one per issuing warp
  uint64_t* epib = drain + C::NISSUE;  // per epilogue warpgroup: 4 warps meet here (bounded)
  uint64_t* sready = epib + C::NWG;    // scale slot landed (one cp.async arrival per producer lane)
  uint64_t* sfree = sready + C::NSLOT; // scale slot consumed (one arrival per epilogue warp)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);  // TMA expect_tx
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&accf[b], 1);           // MMA commit
      mbar_init(&acce[b], 4 * C::NWG);  // one arrive per epilogue warp
    }
    for (int j = 0; j < C::NSLOT; ++j) {
      mbar_init(&sready[j], 32);
      mbar_init(&sfree[j], 4 * C::NWG);
    }
    for (int i = 0; i < C::NISSUE; ++i) mbar_init(&drain[i], 1);
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
    // ───────────── TMA producer (lane 0) + scale staging (all lanes, cp.async) ─────────────
    uint32_t it = 0;
    bool alive = true;
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      const int4 td = args.tiles[tile];
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      const int nr = td.y;
      const int arow = e * args.a_expert_rows[set] + td.w * 128;
      const float* wsp = args.ws[set][lane < NACC ? lane : 0] + e * args.ws_expert_stride[set] + td.w * args.ws_nb_stride;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = it % NSTAGE;
        const uint32_t ph = (it / NSTAGE) & 1;
        const int j = it % C::NSLOT;
        const uint32_t jph = (it / C::NSLOT) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, s_abort) || !mbar_wait(&sfree[j], jph ^ 1, s_abort)) {
          alive = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
#pragma unroll
          for (int a = 0; a < NACC; ++a) tma_load_2d(st + a * C::A_BYTES, &args.tmA[set][a], &full[s], kb * 128, arow);
          tma_load_2d(st + NACC * C::A_BYTES, &args.tmB, &full[s], kb * 128, td.x);
        }
        float* slot = slots + j * C::SLOT_FLOATS;
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) {
          const int r = lane + 32 * u;
          if (r < nr) cp_async_4(slot + r, args.as + (int64_t)(td.x + r) * args.as_row + (int64_t)kb * args.as_kb);
        }
        if (lane < NACC) cp_async_4(slot + BN + lane, wsp + kb);
        cp_async_mbar_arrive(&sready[j]);
        ++it;
      }
    }
    cp_async_wait_all();
    // no copy into this CTA's shared memory may outlive the CTA
    if (lane == 0) {
      const uint32_t first = it > (uint32_t)NSTAGE ? it - NSTAGE : 0;
      for (uint32_t q = first; q < it; ++q) wait_plain(&full[q % NSTAGE], (q / NSTAGE) & 1, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp >= 1 && warp <= C::NISSUE) {
    // ───────────── MMA issuers: warp 1+i takes K-block steps it % NISSUE == i ─────────────
    // A single thread sustains about one tcgen05.mma per 67 cycles, so two issuers keep the
    // tensor core fed at small N.  Every K-block step has its own stage and TMEM buffer, so the
    // issuers never touch the same accumulator and results do not depend on their interleaving.
    const int me = warp - 1;
    uint32_t it = 0, ait = 0;
    bool alive = true;
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      const int4 td = args.tiles[tile];
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      const int nr = td.y;
      int n_eff = (nr + 15) & ~15;
      n_eff = n_eff < 16 ? 16 : (n_eff > BN ? BN : n_eff);
      const uint32_t idesc = umma_idesc_e4m3(128, n_eff);
      for (int kb = 0; kb < nkb; ++kb) {
        if ((int)(it % C::NISSUE) != me) {
          ++it;
          ++ait;
          continue;
        }
        const int b = ait % NBUF;
        const uint32_t aph = (ait / NBUF) & 1;
        if (!mbar_wait(&acce[b], aph ^ 1, s_abort)) {
          alive = false;
          break;
        }
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
          uint64_t adesc[NACC];
#pragma unroll
          for (int a = 0; a < NACC; ++a) adesc[a] = umma_desc_sw128(smem_u32(st + a * C::A_BYTES));
          const uint32_t d0 = tmem + (uint32_t)(b * NACC * BN);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int a = 0; a < NACC; ++a)
              umma_f8(d0 + (uint32_t)(a * BN), adesc[a] + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
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
      umma_commit(&drain[me]);
      wait_plain(&drain[me], 0, kWaitTimeoutNs);
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
        // this K block's scales: a_scale per column (token row) and w_scale per accumulator
        const int j = ait % C::NSLOT;
        if (!mbar_wait(&sready[j], (ait / C::NSLOT) & 1, s_abort)) {
          alive = false;
          break;
        }
        const float* slot = slots + j * C::SLOT_FLOATS;
        // 32 columns per TMEM load; the buffer is handed back to the MMA warps as soon as the
        // last load of this K block has landed
        // 32-column groups of this warpgroup's slice that hold real columns
        const int span = n_eff - wg * CW;
        const int ngroups = span <= 0 ? 0 : (span >= CW ? CW / 32 : (span + 31) / 32);
        if (ngroups == 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[b]);
        }
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
#pragma unroll
          for (int g = 0; g < CW / 32; ++g) {
            const int col = wg * CW + g * 32;
            const bool last = (a == NACC - 1) && (g == ngroups - 1);
            if (g < ngroups) {
              float pv[32];
              const uint32_t ta = tmem + tlane + (uint32_t)((b * NACC + a) * BN + col);
              if (col + 32 <= n_eff) tmem_ld32(ta, pv);
              else tmem_ld16p(ta, pv);
              tmem_ld_wait();
              if (last) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acce[b]);
              }
              const float wsa = slot[BN + a];
              const float4* sc4 = reinterpret_cast<const float4*>(slot + col);
#pragma unroll
              for (int i4 = 0; i4 < 8; ++i4) {
                float4 s4 = sc4[i4];
                s4.x *= wsa;
                s4.y *= wsa;
                s4.z *= wsa;
                s4.w *= wsa;
                acc[a][g * 32 + i4 * 4 + 0] = fmaf(pv[i4 * 4 + 0], s4.x, acc[a][g * 32 + i4 * 4 + 0]);
                acc[a][g * 32 + i4 * 4 + 1] = fmaf(pv[i4 * 4 + 1], s4.y, acc[a][g * 32 + i4 * 4 + 1]);
                acc[a][g * 32 + i4 * 4 + 2] = fmaf(pv[i4 * 4 + 2], s4.z, acc[a][g * 32 + i4 * 4 + 2]);
                acc[a][g * 32 + i4 * 4 + 3] = fmaf(pv[i4 * 4 + 3], s4.w, acc[a][g * 32 + i4 * 4 + 3]);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[j]);
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
          if (t >= nr) break;
          out[(row0 + t) * args.out_ld + ncol] = __float2bfloat16_rn(acc[0][c]);
        }
      } else {
        // SwiGLU exactly as the reference rounds it: gate/up GEMM outputs are bf16
        // (gate_up_out, :610-619), silu() rounds to bf16, the product rounds to bf16 (:624);
        // then _fast_fp8_quantize over these 128 channels (:637).
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          if (wg * CW + c >= nr) break;  // warp-uniform
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
          if (t >= nr) break;
          const float* rr = red + wg * 4 * CW + c;
          const float am = nanmax(nanmax(rr[0], rr[CW]), nanmax(rr[2 * CW], rr[3 * CW]));
          const float s = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
          const float qv = clamp_pm(__fdiv_rn(acc[0][c], s), 448.0f);
          outq[(row0 + t) * args.out_ld + ncol] = (uint8_t)(f32x2_to_e4m3x2(qv, 0.f) & 0xFF);
          if (lrow == 0) args.out_scale[(row0 + t) * args.os_row + (int64_t)td.w * args.os_kb] = s;
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
