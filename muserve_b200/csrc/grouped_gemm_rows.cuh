// Grouped (ragged-M) block-scaled e4m3 GEMM with tokens on the MMA's M side: the large-batch
// form of grouped_gemm.cuh (same math, same tile list), for groups of about a hundred rows
// and more.
//
// Why a second layout.  With weight rows on M (grouped_gemm.cuh), every TMEM column is a token,
// so each K block's promotion acc += partial * a_scale[token] * w_scale needs a different
// scale per column.  Here a TMEM lane is a token: a thread promotes its columns with one
// scalar a_scale[token, kb] * w_scale[block, kb].  The price is the M granularity: a tile is
// 128 token rows, partly empty when a group is not a multiple of 128.
//
// Per-step fixed costs dominate this kernel (an mbarrier wait + arrive round is a few hundred
// cycles for one warp), so everything is batched: a pipeline stage carries two 128-wide K
// blocks, and the tile's activation and weight scales arrive once per tile by TMA into a
// double buffer instead of per K step.
//
// Tile = (group, n-block, token chunk of <= 128 rows).  Per K block four M=128 x N=128 x K=32
// MMAs into one TMEM buffer (two buffers per stage, two stages of buffers):
//   EPI 1 (gate_up): the tile's 128 channels run as two halves h = 0, 1; N = 64 gate rows +
//          64 up rows of channels [64h, 64h + 64).  Warpgroup w owns channels 16w..16w+15 of
//          each half (its gate and up columns), so SwiGLU needs no exchange, and the per-row
//          amax for the e4m3 requant is combined across the four warpgroups at tile end.
//   EPI 0 (plain -> bf16): N = the 128 weight rows of the n-block; warpgroup w owns 32 columns.
// Roles: warp 0 TMA producer of the operand stages; warps 1 and 2 MMA issuers on alternate
// stages (each owns one TMEM buffer pair, so one issuer's waits overlap the other's MMAs), warp 1
// also owns TMEM; warp 3 loads the tiles' scales into a ring of NSCB buffers, up to NSCB tiles
// ahead of the epilogue; warps 4..19 epilogue (warp w reads TMEM lanes 32 * (w % 4) .. +32).
// Every wait is bounded.
#pragma once
#include "grouped_gemm.cuh"

namespace msv {

struct RowsArgs {
  CUtensorMap tmTok;     // activations as 3-D [K/128][rows][128 B] e4m3, box 2 K blocks x 128 rows
  CUtensorMap tmW[2][2]; // weights [set][gate, up] (EPI 1: 2-D, box 64 rows) or [set][0] (EPI 0: 3-D like tmTok)
  CUtensorMap tmAS;      // activation scales, fp32 [K/128][srows] (K-block-major), box 132 x K/128
  CUtensorMap tmWS[2][2];// weight scales, fp32 [blocks][K/128], box K/128 x 1
  int w_rows[2];         // weight rows between consecutive experts, per set
  int ws_rows[2];        // weight-scale rows between consecutive experts, per set
  const int4* tiles;     // {row0, rows, set<<24 | expert, n-block}
  const int* num_tiles;
  int num_kb;
  void* out;             // EPI 0: bf16 [rows, out_ld]; EPI 1: e4m3 [rows, out_ld]
  int64_t out_ld;
  float* out_scale;      // EPI 1: element (row, n-block) at out_scale[row*os_row + nb*os_kb]
  int64_t os_row, os_kb;
  int* err;
};

template <int EPI_, int MAXKB_, int NSCB_>
struct RowsCfg {
  static constexpr int EPI = EPI_;
  static constexpr int MAXKB = MAXKB_;  // K <= 128 * MAXKB
  static constexpr int NSCB = NSCB_;    // scale buffers (tiles in flight between scale warp and epilogue)
  static constexpr int BM = 128;  // token rows per tile (TMEM lanes)
  static constexpr int BN = 128;  // weight rows per MMA (TMEM columns per buffer)
  static constexpr int KS = 2;    // 128-wide K blocks per pipeline stage
  static constexpr int NHALF = EPI == 1 ? 2 : 1;
  static constexpr int NWG = 4;
  static constexpr int NCTRL = 4;  // producer, two MMA issuers, scale loader
  static constexpr int THREADS = 32 * NCTRL + 128 * NWG;
  static constexpr int KB_BYTES = 128 * 128;  // one 128 x 128-byte operand tile
  static constexpr int STAGE_BYTES = KS * 2 * KB_BYTES;
  static constexpr int NPAIR = 2;             // TMEM buffer pairs (one pair per stage)
  static constexpr int TMEM_COLS = 512;
  static constexpr int SC_LD = BM + 4;        // activation-scale row: the chunk's rows from row0 & ~3
  static constexpr int SC_FLOATS = (SC_LD * MAXKB + 2 * MAXKB + 31) & ~31;  // + weight scales (gate, up); 128-byte multiple
  static constexpr int SC_BYTES = SC_FLOATS * 4;
  static constexpr int SMEM_LIMIT = 232448 - 1024;
  static constexpr int BAR_BYTES = 24 * 8;
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - NSCB * SC_BYTES - BAR_BYTES - 16) / STAGE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > 4 ? 4 : NSTAGE_RAW;
  static constexpr int OFF_SC = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_SC + NSCB * SC_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + BAR_BYTES;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(NSTAGE >= 3, "pipeline too shallow");
  static_assert(SMEM_BYTES <= 232448, "shared memory over the sm_100 limit");
  static_assert(NPAIR * KS * BN <= TMEM_COLS, "TMEM buffers");
  static_assert(2 * NSTAGE + 2 * NPAIR + 2 + 2 * NSCB + 1 <= BAR_BYTES / 8, "barrier area");
  static_assert(SC_BYTES % 128 == 0, "scale buffers are TMA destinations");
  static_assert(4 * BM * 4 <= SC_BYTES, "the amax exchange reuses a scale buffer");
};

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) k_grouped_gemm_rows(const __grid_constant__ RowsArgs args) {
  constexpr int NSTAGE = C::NSTAGE, NPAIR = C::NPAIR, BM = C::BM, BN = C::BN, KS = C::KS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* scb = reinterpret_cast<float*>(smem + C::OFF_SC);  // [NSCB][SC_FLOATS]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + NPAIR;
  uint64_t* drain = acce + NPAIR;   // [2] one per issuer
  uint64_t* sc_full = drain + 2;         // [NSCB] the tile's scales landed
  uint64_t* sc_free = sc_full + C::NSCB;  // [NSCB] the epilogue is done with them
  uint64_t* eall = sc_free + C::NSCB;     // EPI 1: all epilogue warps meet
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = args.num_kb;
  const int nsteps = nkb * C::NHALF / KS;  // stages per tile
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NPAIR; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4 * C::NWG);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&drain[b], 1);
    for (int b = 0; b < C::NSCB; ++b) {
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_free[b], 4 * C::NWG);
    }
    mbar_init(eall, 4 * C::NWG);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&args.tmTok);
    tma_prefetch_desc(&args.tmW[0][0]);
    tma_prefetch_desc(&args.tmAS);
  }
  if (warp == 1) tmem_alloc(s_tmem, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  const int ntiles = *args.num_tiles;

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    Ring<NSTAGE> st;
    uint32_t issued = 0;
    bool alive = true;
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      const int4 td = args.tiles[tile];
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      for (int s = 0; s < nsteps; ++s) {
        const int k0 = s * KS;
        const int h = k0 / nkb, kb = k0 - h * nkb;
        if (!mbar_wait(&empty[st.i], st.ph ^ 1, s_abort)) {
          alive = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sp = smem + st.i * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st.i], C::STAGE_BYTES);
          // KS token tiles in one 3-D box: [kb][row][128 B]
          tma_load_3d(sp, &args.tmTok, &full[st.i], 0, td.x, kb);
          uint8_t* wp = sp + KS * C::KB_BYTES;
          if constexpr (C::EPI == 1) {
            // per K block: 64 gate rows then 64 up rows of the same channels (one 128-row operand)
            const int r = e * args.w_rows[set] + td.w * 128 + h * 64;
#pragma unroll
            for (int j = 0; j < KS; ++j) {
              tma_load_2d(wp + j * C::KB_BYTES, &args.tmW[set][0], &full[st.i], (kb + j) * 128, r);
              tma_load_2d(wp + j * C::KB_BYTES + 64 * 128, &args.tmW[set][1], &full[st.i], (kb + j) * 128, r);
            }
          } else {
            tma_load_3d(wp, &args.tmW[set][0], &full[st.i], 0, e * args.w_rows[set] + td.w * 128, kb);
          }
        }
        __syncwarp();
        st.next();
        ++issued;
      }
    }
    // no copy into this CTA's shared memory may outlive the CTA
    if (lane == 0) {
      const uint32_t first = issued > (uint32_t)NSTAGE ? issued - NSTAGE : 0;
      for (uint32_t q = first; q < issued; ++q) wait_plain(&full[q % NSTAGE], (q / NSTAGE) & 1, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ───────────── MMA issuers: KS K blocks per stage into one TMEM buffer pair; issuer i
    // takes the stages that use pair i ─────────────
    const int me = warp - 1;
    Ring<NSTAGE> st;
    Ring<NPAIR> bp;
    bool alive = true;
    const uint32_t idesc = umma_idesc_e4m3(BM, BN);
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x) {
      for (int s = 0; s < nsteps; ++s, st.next(), bp.next()) {
        if (bp.i != me) continue;
        if (!mbar_wait(&acce[bp.i], bp.ph ^ 1, s_abort) || !mbar_wait(&full[st.i], st.ph, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          uint8_t* sp = smem + st.i * C::STAGE_BYTES;
#pragma unroll
          for (int j = 0; j < KS; ++j) {
            const uint64_t adesc = umma_desc_sw128(smem_u32(sp + j * C::KB_BYTES));
            const uint64_t bdesc = umma_desc_sw128(smem_u32(sp + (KS + j) * C::KB_BYTES));
            const uint32_t d = tmem + (uint32_t)((bp.i * KS + j) * BN);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) umma_f8(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty[st.i]);
          umma_commit(&accf[bp.i]);
        }
        __syncwarp();
      }
    }
    // every MMA of this issuer must have completed before TMEM is released
    if (lane == 0) {
      umma_commit(&drain[me]);
      wait_plain(&drain[me], 0, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ───────────── scales of each tile: activation scales of rows (row0 & ~3) .. +131 for
    // every K block, and the weight block's scale row(s) ─────────────
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tcount) {
      const int sb = tcount % C::NSCB;
      if (!mbar_wait(&sc_free[sb], ((tcount / C::NSCB) & 1) ^ 1, s_abort)) break;
      if (lane == 0) {
        const int4 td = args.tiles[tile];
        const int set = td.z >> 24, e = td.z & 0xFFFFFF;
        float* sc = scb + sb * C::SC_FLOATS;
        const uint32_t wbytes = (uint32_t)nkb * 4u;
        mbar_arrive_expect_tx(&sc_full[sb], (uint32_t)C::SC_LD * wbytes + (uint32_t)C::NHALF * wbytes);
        tma_load_2d(sc, &args.tmAS, &sc_full[sb], td.x & ~3, 0);
        const int wrow = e * args.ws_rows[set] + td.w;
        tma_load_2d(sc + C::SC_LD * C::MAXKB, &args.tmWS[set][0], &sc_full[sb], 0, wrow);
        if constexpr (C::EPI == 1)
          tma_load_2d(sc + C::SC_LD * C::MAXKB + C::MAXKB, &args.tmWS[set][1], &sc_full[sb], 0, wrow);
      }
      __syncwarp();
    }
    // no copy into this CTA's shared memory may outlive the CTA
    if (lane == 0)
      for (uint32_t t = tcount > (uint32_t)C::NSCB ? tcount - C::NSCB : 0; t < tcount; ++t)
        wait_plain(&sc_full[t % C::NSCB], (t / C::NSCB) & 1, kWaitTimeoutNs);
    __syncwarp();
  } else {
    // ───────────── epilogue: 16 warps, TMEM lane = token row ─────────────
    const int ew = warp - C::NCTRL, wg = ew >> 2, q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    Ring<NPAIR> bp;
    uint32_t tcount = 0, eph = 0;
    bool alive = true;
    auto all_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(eall);
      const bool ok = mbar_wait(eall, eph, s_abort);
      eph ^= 1;
      return ok;
    };
    for (int tile = blockIdx.x; tile < ntiles && alive; tile += gridDim.x, ++tcount) {
      const int4 td = args.tiles[tile];
      const int nr = td.y;
      const int64_t row0 = td.x;
      const int sb = tcount % C::NSCB;
      if (!mbar_wait(&sc_full[sb], (tcount / C::NSCB) & 1, s_abort)) break;
      float* sc = scb + sb * C::SC_FLOATS;
      const float* a_s = sc + (int)(row0 & 3) + lrow;  // a_s[kb * SC_LD]
      const float* w_s = sc + C::SC_LD * C::MAXKB;       // gate [0, MAXKB), up [MAXKB, 2 MAXKB)
      uint32_t act[C::NHALF][8];                          // EPI 1: SwiGLU output, bf16x2, 16 channels per half
      float mrow = 0.f;
      for (int h = 0; h < C::NHALF && alive; ++h) {
        float acc[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = 0.f;
        for (int s = h * (nkb / KS); s < (h + 1) * (nkb / KS); ++s, bp.next()) {
          if (!mbar_wait(&accf[bp.i], bp.ph, s_abort)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const int kb0 = s * KS - h * nkb;
          const uint32_t tb = tmem + tlane + (uint32_t)(bp.i * KS * BN);
          if constexpr (C::EPI == 0) {
            // both K blocks' loads in flight together
            float pv[KS][32];
#pragma unroll
            for (int j = 0; j < KS; ++j) tmem_ld32(tb + (uint32_t)(j * BN + wg * 32), pv[j]);
            float sj[KS];
#pragma unroll
            for (int j = 0; j < KS; ++j) sj[j] = a_s[(kb0 + j) * C::SC_LD] * w_s[kb0 + j];
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[bp.i]);
#pragma unroll
            for (int j = 0; j < KS; ++j)
#pragma unroll
              for (int c = 0; c < 32; c += 2) fma2(acc[c], acc[c + 1], pv[j][c], pv[j][c + 1], sj[j], sj[j]);
          } else {
            // one K block at a time (registers also hold the first half's SwiGLU output)
#pragma unroll
            for (int j = 0; j < KS; ++j) {
              float pv[32];
              tmem_ld16p(tb + (uint32_t)(j * BN + wg * 16), pv);
              tmem_ld16p(tb + (uint32_t)(j * BN + 64 + wg * 16), pv + 16);
              const float a = a_s[(kb0 + j) * C::SC_LD];
              const float sg = a * w_s[kb0 + j], su = a * w_s[C::MAXKB + kb0 + j];
              tmem_ld_wait();
#pragma unroll
              for (int c = 0; c < 16; c += 2) {
                fma2(acc[c], acc[c + 1], pv[c], pv[c + 1], sg, sg);
                fma2(acc[16 + c], acc[17 + c], pv[16 + c], pv[17 + c], su, su);
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[bp.i]);
          }
        }
        if (!alive) break;
        if constexpr (C::EPI == 0) {
          if (lrow < nr) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(args.out) + (row0 + lrow) * args.out_ld + td.w * 128 + wg * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
              uint4 v;
              __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
              for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(acc[c + 2 * i], acc[c + 2 * i + 1]);
              *reinterpret_cast<uint4*>(o + c) = v;
            }
          }
        } else {
          // SwiGLU as the reference rounds it: gate and up GEMM outputs in bf16
          // (gate_up_out, qwen35_layer_v2.py:610-619), silu() rounded to bf16, the product
          // rounded to bf16 (:624)
#pragma unroll
          for (int c = 0; c < 16; c += 2) {
            float av[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float g = bf16_round(acc[c + i]);
              const float u = bf16_round(acc[16 + c + i]);
              const float sgl = bf16_round(__fdiv_rn(g, 1.0f + expf(-g)));
              av[i] = bf16_round(sgl * u);
              mrow = nanmax(mrow, fabsf(av[i]));
            }
            const __nv_bfloat162 v = __floats2bfloat162_rn(av[0], av[1]);
            act[h][c / 2] = *reinterpret_cast<const uint32_t*>(&v);
          }
        }
      }
      if (!alive) break;
      if constexpr (C::EPI == 1) {
        // _fast_fp8_quantize (qwen35_layer_v2.py:71-86, :637) over the tile's 128 channels:
        // the row's amax is the max over the four warpgroups; the amax exchange reuses this
        // tile's scale buffer once every warp has read its last scale from it
        if (!all_sync()) break;
        float* red = sc;  // [4][BM]
        red[wg * BM + lrow] = mrow;
        if (!all_sync()) break;
        const float am = nanmax(nanmax(red[lrow], red[BM + lrow]), nanmax(red[2 * BM + lrow], red[3 * BM + lrow]));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[sb]);
        if (lrow < nr) {
          const float s = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
          uint8_t* o = reinterpret_cast<uint8_t*>(args.out) + (row0 + lrow) * args.out_ld + td.w * 128 + wg * 16;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 v;
            uint16_t* p = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&act[h][i]);
              const float q0 = clamp_pm(__fdiv_rn(__low2float(b), s), 448.0f);
              const float q1 = clamp_pm(__fdiv_rn(__high2float(b), s), 448.0f);
              p[i] = f32x2_to_e4m3x2(q0, q1);
            }
            *reinterpret_cast<uint4*>(o + h * 64) = v;
          }
          if (wg == 0) args.out_scale[(row0 + lrow) * args.os_row + (int64_t)td.w * args.os_kb] = s;
        }
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[sb]);
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
  pdl_trigger();
}

}  // namespace msv
