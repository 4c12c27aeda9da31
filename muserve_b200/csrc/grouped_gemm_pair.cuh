// The gate_up GEMM of large batches on CTA pairs: tokens on the MMA's M side, M = 256 token rows
// per pair (tcgen05 cta_group::2), N = 256 weight rows (the gate and up rows of 128 channels) per
// MMA, SwiGLU and the per-128 e4m3 requant in the epilogue.  Same math and tile list as
// grouped_gemm.cuh / grouped_gemm_rows.cuh:
//   D[m, n] = sum_kb ( sum_{k in kb} A[m,k] W[e, n, k] ) * a_scale[m, kb] * w_scale[e, n/128, kb]
// (mate.gemm.ragged_m_moe_gemm_8bit as called from muserve/model/qwen35_layer_v2.py:613-618).
//
// Why pairs.  The single-CTA token-rows kernel (grouped_gemm_rows.cuh) runs a 128-channel block
// as two halves and loads the token tile once per half: 128 B of operands per SM cycle at the
// tensor rate.  Here each CTA of a pair loads its own 128 token rows (A) and one of the two
// 128-row weight halves (rank 0 the gate rows, rank 1 the up rows); rank 0 issues M=256 x N=256
// MMAs that read both CTAs' operands and write each SM's 128 rows of D (128 lanes x 256
// columns) into that SM's TMEM: 64 B per SM cycle, and the token tile is read once per block.
// Measured on B200, the kernel is bound by the operand stream: with the MMAs and the TMEM reads
// taken out it still needs ~1.05 ms at prefill_c2, because each SM keeps six 32 KB stages in
// flight and a TMA load then takes ~3.4 us (a latency that did not change with L2 prefetch of
// the weights, with the tokens forced to hit L2, or with 3-D, 64- or 128-row boxes).
//
// TMEM: two 256-column buffers, one per K block in flight.  The fp32 scales differ per row and
// per K block, so every K block accumulates into a fresh buffer that the epilogue promotes into
// registers (acc += partial * a_scale * w_scale) and hands back once its last load landed.
//
// Tile = (group, 128-channel block, chunk of <= 256 rows), rows [row0, row0 + rows); rank r
// takes rows row0 + 128 r .. +127.  Token rows are loaded in 64-row boxes and a box that starts
// beyond the chunk is skipped.  D columns 0-127 are the gate of channels 0-127, 128-255 their up.
// Roles (both CTAs): warp 0 TMA producer (its loads complete on rank 0's stage barrier); warp 1
// MMA issuer (rank 0; warp 1 of each CTA owns TMEM); warp 3 loads each tile's scales by TMA into a
// ring; warps 4..19 epilogue (warp w reads TMEM lanes 32 (w % 4) .. +31, channel group
// (w - 4) / 4).  Every wait is bounded; no TMA load here uses multicast, and MMA completions are
// committed to each CTA's barrier separately.  Barriers use CTA-scope semantics (release and
// acquire at cluster scope on these hot barriers cost microseconds per K block).
#pragma once
#include "grouped_gemm_rows.cuh"

namespace msv {

// ── CTA pairs (2-CTA clusters sharing one tcgen05 MMA) ──────────────────────────────────

MSV_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same shared-memory offset in CTA `rank` of this cluster.
MSV_DEVICE uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Every thread of both CTAs (orders barrier initialisation and teardown across the pair).
MSV_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on a barrier of either CTA of the pair.  The barriers below hand over TMEM columns and
// shared-memory stages ordered by tcgen05 fences and TMA completion, so CTA-scope semantics
// suffice; cluster-scope release/acquire on these hot barriers cost microseconds per K block.
MSV_DEVICE void mbar_arrive_cl(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Bounded spinning wait (no suspend: a peer's arrival must be seen at once).
MSV_DEVICE bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15) == 0) {
      if (*abort) return false;
      if (clock64() - t0 > kWaitTimeoutCycles) {
        *abort = 1;
        return false;
      }
    }
  }
}
// 2-D tiled load into this CTA's shared memory, completing on the barrier at `bar_cl` (a
// shared::cluster address, here always rank 0's stage barrier).  No multicast.
MSV_DEVICE void tma_load_2d_cg2(void* dst, const CUtensorMap* m, uint32_t bar_cl, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cl), "r"(x), "r"(y)
      : "memory");
}
// M = 256 MMA over the pair, issued by rank 0: A rows 0-127 from rank 0's tile and 128-255 from
// rank 1's (same shared-memory offset), B columns 0..N/2-1 from rank 0 and N/2..N-1 from rank 1;
// each SM's 128 rows of D land in its own TMEM at the same address.
MSV_DEVICE void umma_f8_cg2(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u));
}
// Arrive once on the barrier at `bar_cl` (either CTA) when the pair MMAs this thread issued so
// far have completed.
MSV_DEVICE void umma_commit_cg2(uint32_t bar_cl) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cl)
               : "memory");
}
// Warp-wide, warp 1 of both CTAs together: TMEM columns for the pair MMAs.
MSV_DEVICE void tmem_alloc_cg2(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
MSV_DEVICE void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <int MAXKB_, int NSCB_>
struct PairCfg {
  static constexpr int MAXKB = MAXKB_;  // K <= 128 * MAXKB
  static constexpr int NSCB = NSCB_;    // scale buffers (tiles in flight between scale warp and epilogue)
  static constexpr int BM = 128;        // token rows per CTA (TMEM lanes); 256 per pair
  static constexpr int BN = 256;        // MMA N: weight rows per pair tile (TMEM columns per K block)
  static constexpr int NBUF = 2;        // K blocks in flight in TMEM
  static constexpr int NWG = 4;
  static constexpr int NCTRL = 4;       // producer, MMA issuer, (idle), scale loader
  static constexpr int THREADS = 32 * NCTRL + 128 * NWG;
  // 96 registers per thread (65536 / 640, rounded down to 8): an epilogue thread holds 64 fp32
  // accumulators and loads its TMEM columns 16 at a time.
  static constexpr int NREG_LAUNCH = 96;
  static constexpr int A_BYTES = 128 * 128;   // this CTA's 128 token rows x 128 B
  static constexpr int B_BYTES = 128 * 128;   // this CTA's 128 of the 256 weight rows x 128 B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SC_LD = BM + 4;  // activation-scale row: the CTA's rows from (row & ~3)
  static constexpr int SC_FLOATS = (SC_LD * MAXKB + 2 * MAXKB + 31) & ~31;
  static constexpr int SC_BYTES = SC_FLOATS * 4;
  static constexpr int SMEM_LIMIT = 232448 - 1024;
  static constexpr int BAR_BYTES = 40 * 8;
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - NSCB * SC_BYTES - BAR_BYTES - 16) / STAGE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > 8 ? 8 : NSTAGE_RAW;
  static constexpr int OFF_SC = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_SC + NSCB * SC_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + BAR_BYTES;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(NSTAGE >= 4, "pipeline too shallow");
  static_assert(SMEM_BYTES <= 232448, "shared memory over the sm_100 limit");
  static_assert(NBUF * BN <= TMEM_COLS, "TMEM buffers");
  static_assert(2 * NSTAGE + 2 * NBUF + 1 + 2 * NSCB + 1 <= BAR_BYTES / 8, "barrier area");
  static_assert(SC_BYTES % 128 == 0, "scale buffers are TMA destinations");
  static_assert(4 * BM * 4 <= SC_BYTES, "the amax exchange reuses a scale buffer");
};

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) __maxnreg__(C::NREG_LAUNCH)
    k_grouped_gemm_pair(const __grid_constant__ RowsArgs args) {
  constexpr int NSTAGE = C::NSTAGE, BM = C::BM, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  // the same offsets in both CTAs (one descriptor addresses both halves of an operand)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* scb = reinterpret_cast<float*>(smem + C::OFF_SC);  // [NSCB][SC_FLOATS]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);  // rank 0: both CTAs' stage loads
  uint64_t* empty = full + NSTAGE;                                   // each CTA: its stage is free
  uint64_t* accf = empty + NSTAGE;                                   // each CTA: a K block's MMAs completed
  uint64_t* acce = accf + C::NBUF;                                   // rank 0: both epilogues released it
  uint64_t* drain = acce + C::NBUF;                                  // rank 0's issuer
  uint64_t* sc_full = drain + 1;                                     // [NSCB] the tile's scales landed
  uint64_t* sc_free = sc_full + C::NSCB;                             // [NSCB] the epilogue is done with them
  uint64_t* eall = sc_free + C::NSCB;                                // all epilogue warps meet (amax exchange)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nkb = args.num_kb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 2 * 4 * C::NWG);
    }
    mbar_init(drain, 1);
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
  if (warp == 1) tmem_alloc_cg2(s_tmem, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival or load
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  const int ntiles = *args.num_tiles;

  if (warp == 0) {
    // ───────────── TMA producer: this CTA's token rows and its 128 weight rows ─────────────
    Ring<NSTAGE> st;
    uint32_t issued = 0;
    bool alive = true;
    for (int tile = pair; tile < ntiles && alive; tile += npairs) {
      const int4 td = args.tiles[tile];
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      const int arow = td.x + BM * (int)rank;
      // token rows come in 64-row boxes, and a box that starts beyond the chunk is not loaded:
      // its shared memory keeps stale rows whose results the epilogue never stores
      auto nbox = [&](int r) { return (td.y > BM * r) + (td.y > BM * r + 64); };
      const int my_boxes = nbox((int)rank);
      const uint32_t stage_tx = (uint32_t)(nbox(0) + nbox(1)) * (64u * 128u) + 2u * C::B_BYTES;
      // rank 0 loads the gate rows, rank 1 the up rows of the block's 128 channels
      const int wrow = e * args.w_rows[set] + td.w * 128;
      const CUtensorMap* wmap = &args.tmW[set][rank];
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait_spin(&empty[st.i], st.ph ^ 1, s_abort)) {
          alive = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sp = smem + st.i * C::STAGE_BYTES;
          const uint32_t full_cl = mapa_shared(smem_u32(&full[st.i]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[st.i], stage_tx);  // both CTAs' bytes
          for (int bx = 0; bx < my_boxes; ++bx) tma_load_2d_cg2(sp + bx * 64 * 128, &args.tmTok, full_cl, kb * 128, arow + 64 * bx);
          tma_load_2d_cg2(sp + C::A_BYTES, wmap, full_cl, kb * 128, wrow);
          tma_load_2d_cg2(sp + C::A_BYTES + 64 * 128, wmap, full_cl, kb * 128, wrow + 64);
        }
        __syncwarp();
        st.next();
        ++issued;
      }
    }
    // no copy into either CTA's shared memory may outlive it: rank 0 waits for the last stages
    // (their barrier counts both CTAs' bytes); the final cluster barrier holds rank 1 until then
    if (rank == 0 && lane == 0) {
      const uint32_t first = issued > (uint32_t)NSTAGE ? issued - NSTAGE : 0;
      for (uint32_t q = first; q < issued; ++q) wait_plain(&full[q % NSTAGE], (q / NSTAGE) & 1, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ───────────── MMA issuer (rank 0): per K block four M=256 x N=256 x K=32 MMAs into
    // TMEM buffer kbg % 2, completion committed to both CTAs ─────────────
    if (rank == 0) {
      Ring<NSTAGE> st;
      uint32_t kbg = 0;
      bool alive = true;
      const uint32_t idesc = umma_idesc_e4m3(256, BN);
      for (int tile = pair; tile < ntiles && alive; tile += npairs) {
        for (int kb = 0; kb < nkb; ++kb, st.next(), ++kbg) {
          const int b = (int)(kbg & 1);
          if (!mbar_wait_spin(&full[st.i], st.ph, s_abort) ||
              !mbar_wait_spin(&acce[b], ((kbg >> 1) & 1) ^ 1, s_abort)) {
            alive = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            uint8_t* sp = smem + st.i * C::STAGE_BYTES;
            const uint64_t adesc = umma_desc_sw128(smem_u32(sp));
            const uint64_t bdesc = umma_desc_sw128(smem_u32(sp + C::A_BYTES));
            const uint32_t d = tmem + (uint32_t)(b * BN);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) umma_f8_cg2(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
            umma_commit_cg2(mapa_shared(smem_u32(&accf[b]), 0));
            umma_commit_cg2(mapa_shared(smem_u32(&accf[b]), 1));
            umma_commit_cg2(mapa_shared(smem_u32(&empty[st.i]), 0));
            umma_commit_cg2(mapa_shared(smem_u32(&empty[st.i]), 1));
          }
          __syncwarp();
        }
      }
      // every MMA has completed before TMEM is released
      if (lane == 0) {
        umma_commit_cg2(mapa_shared(smem_u32(drain), 0));
        wait_plain(drain, 0, kWaitTimeoutNs);
      }
      __syncwarp();
    }
  } else if (warp == 3) {
    // ───────────── scales of each tile for this CTA's rows: activation scales of rows
    // (row & ~3) .. +131 for every K block, and the weight blocks' scale rows ─────────────
    uint32_t tcount = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++tcount) {
      const int sb = tcount % C::NSCB;
      if (!mbar_wait(&sc_free[sb], ((tcount / C::NSCB) & 1) ^ 1, s_abort)) break;
      if (lane == 0) {
        const int4 td = args.tiles[tile];
        const int set = td.z >> 24, e = td.z & 0xFFFFFF;
        float* sc = scb + sb * C::SC_FLOATS;
        const uint32_t wbytes = (uint32_t)nkb * 4u;
        mbar_arrive_expect_tx(&sc_full[sb], (uint32_t)C::SC_LD * wbytes + 2u * wbytes);
        tma_load_2d(sc, &args.tmAS, &sc_full[sb], (td.x + BM * (int)rank) & ~3, 0);
        const int wrow = e * args.ws_rows[set] + td.w;
        tma_load_2d(sc + C::SC_LD * C::MAXKB, &args.tmWS[set][0], &sc_full[sb], 0, wrow);           // gate
        tma_load_2d(sc + C::SC_LD * C::MAXKB + C::MAXKB, &args.tmWS[set][1], &sc_full[sb], 0, wrow);  // up
      }
      __syncwarp();
    }
    // no copy into this CTA's shared memory may outlive the CTA
    if (lane == 0)
      for (uint32_t t = tcount > (uint32_t)C::NSCB ? tcount - C::NSCB : 0; t < tcount; ++t)
        wait_plain(&sc_full[t % C::NSCB], (t / C::NSCB) & 1, kWaitTimeoutNs);
    __syncwarp();
  } else if (warp >= C::NCTRL) {
    // ───────────── epilogue: 16 warps, TMEM lane = token row; channel group j takes TMEM
    // columns 32j .. +31 (gate of channels 32j ..) and 128 + 32j .. +31 (their up) ─────────
    const int j = (warp - C::NCTRL) >> 2, q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    uint32_t tcount = 0, eph = 0, kbg = 0;
    bool alive = true;
    auto all_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(eall);
      const bool ok = mbar_wait(eall, eph, s_abort);
      eph ^= 1;
      return ok;
    };
    const uint32_t acce_cl = mapa_shared(smem_u32(acce), 0);  // rank 0's buffer-release barriers
    const uint32_t tcol = tmem + tlane + (uint32_t)(32 * j);
    for (int tile = pair; tile < ntiles && alive; tile += npairs, ++tcount) {
      const int sb = tcount % C::NSCB;
      float* sc = scb + sb * C::SC_FLOATS;
      const float* a_s;
      {
        const int row0 = args.tiles[tile].x;
        a_s = sc + ((row0 + BM * (int)rank) & 3) + lrow;  // a_s[kb * SC_LD]
      }
      if (!mbar_wait(&sc_full[sb], (tcount / C::NSCB) & 1, s_abort)) break;
      const float* w_s0 = sc + C::SC_LD * C::MAXKB;
      const int w_s1 = C::MAXKB;  // the up scales follow the gate scales
      float acc[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) acc[c] = 0.f;
      for (int kb = 0; kb < nkb; ++kb, ++kbg) {
        const int b = (int)(kbg & 1);
        const float a = a_s[kb * C::SC_LD];
        const float s0 = a * w_s0[kb], s1 = a * w_s0[w_s1 + kb];
        if (!mbar_wait_spin(&accf[b], (kbg >> 1) & 1, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tcol + (uint32_t)(b * BN);
        // four rounds of 16 columns (the registers hold 64 accumulators besides); the buffer
        // goes back to the issuer once the last load landed
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float p[16];
          tmem_ld16p(tb + (uint32_t)((r >> 1) * 128 + (r & 1) * 16), p);
          tmem_ld_wait();
          if (r == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cl(acce_cl + (uint32_t)(b * 8));
          }
          const float sv = r < 2 ? s0 : s1;
#pragma unroll
          for (int c = 0; c < 16; c += 2) fma2(acc[16 * r + c], acc[16 * r + c + 1], p[c], p[c + 1], sv, sv);
        }
      }
      if (!alive) break;
      const int4 td = args.tiles[tile];
      const int prow = BM * (int)rank + lrow;  // row within the pair tile
      const int64_t grow = (int64_t)td.x + prow;
      const bool valid = prow < td.y;
      {
        // SwiGLU as the reference rounds it: gate and up GEMM outputs in bf16
        // (gate_up_out, qwen35_layer_v2.py:610-619), silu() rounded to bf16, the product
        // rounded to bf16 (:624); then _fast_fp8_quantize over the tile's 128 channels (:637)
        uint32_t act[16];
        float mrow = 0.f;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float av[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float g = bf16_round(acc[c + i]);
            const float up = bf16_round(acc[32 + c + i]);
            const float sgl = bf16_round(__fdiv_rn(g, 1.0f + expf(-g)));
            av[i] = bf16_round(sgl * up);
            mrow = nanmax(mrow, fabsf(av[i]));
          }
          const __nv_bfloat162 v = __floats2bfloat162_rn(av[0], av[1]);
          act[c / 2] = *reinterpret_cast<const uint32_t*>(&v);
        }
        // the row's amax is the max over the four column groups; the exchange reuses this
        // tile's scale buffer once every warp has read its last scale from it
        if (!all_sync()) break;
        float* red = sc;  // [4][BM]
        red[j * BM + lrow] = mrow;
        if (!all_sync()) break;
        const float am = nanmax(nanmax(red[lrow], red[BM + lrow]), nanmax(red[2 * BM + lrow], red[3 * BM + lrow]));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[sb]);
        if (valid) {
          const float s = (am != am) ? am : __fdiv_rn(fmaxf(am, 1e-12f), 448.0f);
          uint8_t* o = reinterpret_cast<uint8_t*>(args.out) + grow * args.out_ld + td.w * 128 + 32 * j;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 v;
            uint16_t* pk = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const __nv_bfloat162 bv = *reinterpret_cast<const __nv_bfloat162*>(&act[8 * h + i]);
              const float q0 = clamp_pm(__fdiv_rn(__low2float(bv), s), 448.0f);
              const float q1 = clamp_pm(__fdiv_rn(__high2float(bv), s), 448.0f);
              pk[i] = f32x2_to_e4m3x2(q0, q1);
            }
            *reinterpret_cast<uint4*>(o + 16 * h) = v;
          }
          if (j == 0) args.out_scale[grow * args.os_row + (int64_t)td.w * args.os_kb] = s;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs, loads or arrivals may touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *s_abort) atomicExch(args.err, (int)MSV_ERR_TIMEOUT);
  pdl_trigger();
}

}  // namespace msv
