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
// on the device, the kernel is persistent (one CTA per SM; tile order below).
//
// The 128x128 fp32 weight scales and per-row x 128 activation scales are arbitrary fp32
// values, so they cannot be folded into a UE8M0 block-scaled MMA: every 128-wide K block
// ("K step") is accumulated into its own TMEM buffer and promoted into fp32 registers with
// its scale (as the reference's block-wise scaling defines it).
//
// Roles (warp-specialised, one CTA per SM):
//   warp 0      TMA producer: per K step, NACC weight boxes [128 x 128 B] and one token box
//               [BN x 128 B] (128-byte swizzle) into an NSTAGE ring; its 32 lanes also copy
//               the step's activation and weight scales into a scale-slot ring (cp.async).
//   warps 1, 2  MMA issuers, alternate K steps: tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> fp32),
//               4 x K=32 per step per accumulator, into the step's TMEM buffer (NBUF ring).
//               A single thread issues about one MMA per 67 cycles, so two share the work;
//               every step has its own stage and buffer, so the order they run in is free.
//   warp 3      scale warp: per K step, combined scale a_scale[row] * w_scale[acc] for every
//               column of the tile, computed once into shared memory.
//   warps 4..   epilogue warpgroups: per K step, tcgen05.ld 32 (or 16) columns at a time,
//               hand the TMEM buffer back as soon as the last load landed, then
//               acc += partial * scale with paired fp32 FMAs.  Each warpgroup takes a column
//               slice of every accumulator, or (plain bf16 output, one warpgroup per
//               accumulator) all columns of its own accumulator: tiles of one K step are
//               epilogue-bound, and this halves the work a warpgroup does per tile.  A 16-column
//               slice loads TMEM 16 columns at a time (gate_up with two warpgroups: the SwiGLU
//               finish of a 32-token tile, one chain per column, runs on eight warps instead of
//               four).  At tile end: bf16 out (EPI 0), or SwiGLU + per-128 e4m3 requant (EPI 1:
//               acc 0 = gate rows, acc 1 = up rows of the same channels).
// Tile order: CTA b starts with tile b; every later tile is claimed from a global counter
// (GemmArgs::tile_next, zeroed by the tile-list builder) when the producer starts issuing the
// loads of its current tile.  SMs do not stream at the same rate (measured per CTA: 19 to
// 28 us for the same 1 MB tile), so a static round robin left the last ~20 % of a launch on a
// shrinking set of slow SMs.  Tiles of fewer than 4 K steps keep the static order (null
// tile_next): there a claim per tile costs more than the imbalance it removes.  Either way the
// producer alone reads the tile list, one tile ahead, and hands each descriptor to the other
// roles through a shared-memory ring: a global load costs about a microsecond under load, as
// long as a whole one-K-step tile, which every role would otherwise pay per tile.
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
  int* tile_next;         // claim counter of the tiles after the first round (0 at launch), or
                          // null: static round robin
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
  // EPI 0 with one warpgroup per accumulator (NWG == NACC): each warpgroup promotes all BN
  // columns of its own accumulator; otherwise each takes a BN / NWG column slice of every one
  static constexpr bool ASPLIT = EPI == 0 && NACC > 1 && NWG == NACC;
  static constexpr int NA = ASPLIT ? 1 : NACC;  // accumulators per epilogue thread
  static constexpr int CW = ASPLIT ? BN : BN / NWG;
  static constexpr int THREADS = 128 + 128 * NWG;
  static constexpr int NISSUE = 2;
  static constexpr int NSLOT = 8;                       // scale-slot ring depth (K steps)
  static constexpr int TRING = 16;                      // tile-descriptor ring depth (tiles the producer may lead by)
  static constexpr int NCONS = NISSUE + 1 + 4 * NWG;    // warps that read each descriptor
  static constexpr int RAW_FLOATS = BN + 4;             // per slot: a_scale of the chunk's rows, w_scale per acc
  static constexpr int SCL_FLOATS = NACC * BN;          // per slot: combined scales
  static constexpr int RED_BYTES = EPI == 1 ? NWG * 4 * CW * 4 : 0;
  static constexpr int TAIL_BYTES = NSLOT * (RAW_FLOATS + SCL_FLOATS) * 4 + RED_BYTES + 128 * 8 + TRING * 16 + 64;
  static constexpr int SMEM_LIMIT = 232448 - 1024;  // 227 KB opt-in, minus alignment slack
  static constexpr int NSTAGE_RAW = (SMEM_LIMIT - TAIL_BYTES) / STAGE_BYTES;
  static constexpr int NSTAGE = NSTAGE_RAW > 12 ? 12 : NSTAGE_RAW;
  static constexpr int OFF_RAW = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_SCL = OFF_RAW + NSLOT * RAW_FLOATS * 4;
  static constexpr int OFF_RED = OFF_SCL + NSLOT * SCL_FLOATS * 4;
  static constexpr int OFF_BAR = (OFF_RED + RED_BYTES + 7) & ~7;
  static constexpr int NBARS = 2 * NSTAGE + 2 * NBUF + NISSUE + NWG + 3 * NSLOT + 2 * TRING;
  static constexpr int OFF_TILE = (OFF_BAR + NBARS * 8 + 15) & ~15;
  static constexpr int OFF_MISC = OFF_TILE + TRING * 16;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int LW = CW < 32 ? CW : 32;  // columns per TMEM load (16 or 32)
  static_assert(CW % 16 == 0 && CW % LW == 0, "column slice must be whole 16- or 32-column TMEM loads");
  static_assert(NBUF >= 2, "need at least double-buffered TMEM partials");
  static_assert(NSTAGE >= 2, "pipeline too shallow");
  static_assert(NBARS <= 128, "barrier area");
  static_assert(SMEM_BYTES <= 232448, "shared memory over the sm_100 limit");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
};

MSV_DEVICE bool wait_plain(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
  unsigned long long t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, kSuspendNs))
    if (globaltimer() - t0 > limit_ns) return false;
  return true;
}

// Ring position: index and phase parity advanced without division.
template <int N>
struct Ring {
  int i = 0;
  uint32_t ph = 0;
  MSV_DEVICE void next() {
    if (++i == N) {
      i = 0;
      ph ^= 1;
    }
  }
};

// acc[0..1] += p[0..1] * s[0..1] as one paired fp32 FMA.
MSV_DEVICE void fma2(float& a0, float& a1, float p0, float p1, float s0, float s1) {
  uint64_t a, p, s, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(p) : "f"(p0), "f"(p1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(s) : "f"(s0), "f"(s1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(p), "l"(s), "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(d));
}

// CLAIM: tiles after the first round come from args.tile_next (false: static round robin).
// The two orders are separate instantiations so that neither carries the other's code.
template <class C, bool CLAIM>
__global__ void __launch_bounds__(C::THREADS, 1) k_grouped_gemm(const __grid_constant__ GemmArgs args) {
  constexpr int BN = C::BN, NACC = C::NACC, NSTAGE = C::NSTAGE, NBUF = C::NBUF, CW = C::CW, NSLOT = C::NSLOT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* raw = reinterpret_cast<float*>(smem + C::OFF_RAW);
  float* scl = reinterpret_cast<float*>(smem + C::OFF_SCL);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + NSTAGE;
  uint64_t* accf = empty + NSTAGE;
  uint64_t* acce = accf + NBUF;
  uint64_t* drain = acce + NBUF;         // one per issuing warp
  uint64_t* epib = drain + C::NISSUE;    // per epilogue warpgroup: 4 warps meet here (bounded)
  uint64_t* sready = epib + C::NWG;      // raw scales landed (one cp.async arrival per producer lane)
  uint64_t* cready = sready + NSLOT;     // combined scales written by the scale warp
  uint64_t* sfree = cready + NSLOT;      // slot consumed (one arrival per epilogue warp)
  uint64_t* tfull = sfree + NSLOT;       // tile descriptor published (producer)
  uint64_t* tfree = tfull + C::TRING;    // tile descriptor read (every consumer warp)
  int4* s_tile = reinterpret_cast<int4*>(smem + C::OFF_TILE);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4 * C::NWG);
    }
    for (int i = 0; i < C::NISSUE; ++i) mbar_init(&drain[i], 1);
    for (int g = 0; g < C::NWG; ++g) mbar_init(&epib[g], 4);
    for (int j = 0; j < NSLOT; ++j) {
      mbar_init(&sready[j], 32);
      mbar_init(&cready[j], 1);
      mbar_init(&sfree[j], 4 * C::NWG);
    }
    for (int j = 0; j < C::TRING; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tfree[j], C::NCONS);
    }
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
  pdl_wait();
  const int ntiles = *args.num_tiles;
  const int nkb = args.num_kb;
  constexpr bool dyn = CLAIM;
  const int4 kEnd = make_int4(-1, 0, 0, 0);  // ring entry after the last tile (row0 < 0)
  // this CTA's next tile descriptor from the ring (x < 0: none left); false on timeout or abort
  auto next_tile = [&](Ring<C::TRING>& tr, int4& td) -> bool {
    if (!mbar_wait(&tfull[tr.i], tr.ph, s_abort)) return false;
    td = s_tile[tr.i];
    __syncwarp();
    if (lane == 0) mbar_arrive(&tfree[tr.i]);
    tr.next();
    return true;
  };

  if (warp == 0) {
    // ───────────── TMA producer (lane 0) + raw scale copies (all lanes) ─────────────
    Ring<NSTAGE> st;
    Ring<NSLOT> sl;
    uint32_t issued = 0;
    bool alive = true;
    Ring<C::TRING> tr;
    int tile = blockIdx.x;
    int4 td = tile < ntiles ? args.tiles[tile] : kEnd;
    for (;;) {
      if (!mbar_wait(&tfree[tr.i], tr.ph ^ 1, s_abort)) break;
      if (lane == 0) {
        s_tile[tr.i] = td;
        mbar_arrive(&tfull[tr.i]);
      }
      tr.next();
      if (td.x < 0) break;
      // the next tile, claimed or known now; its descriptor is loaded at once in the static
      // order, and two K steps into this tile (the claim has returned by then) when claimed,
      // so both round trips overlap this tile's loads
      int nt = tile + (int)gridDim.x;
      if (dyn && lane == 0) nt = atomicAdd(args.tile_next, 1) + (int)gridDim.x;
      int4 ntd = kEnd;
      if (!dyn && nt < ntiles) ntd = args.tiles[nt];
      const int kb_fetch = dyn ? min(2, nkb - 1) : -1;
      const int set = td.z >> 24, e = td.z & 0xFFFFFF;
      const int nr = td.y;
      // EPI 0 with NACC accumulators: a tile covers NACC consecutive 128-row weight blocks of one
      // matrix (accumulator a: rows + 128 a, scale row + a); EPI 1: one block of gate and of up
      constexpr int NBLK = C::EPI == 0 ? NACC : 1;
      const int arow = e * args.a_expert_rows[set] + td.w * 128 * NBLK;
      const int acc_l = lane < NACC ? lane : 0;
      const float* wsp = C::EPI == 0
                             ? args.ws[set][0] + e * args.ws_expert_stride[set] + (td.w * NBLK + acc_l) * args.ws_nb_stride
                             : args.ws[set][acc_l] + e * args.ws_expert_stride[set] + td.w * args.ws_nb_stride;
      const float* asp = args.as + (int64_t)td.x * args.as_row;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&empty[st.i], st.ph ^ 1, s_abort) || !mbar_wait(&sfree[sl.i], sl.ph ^ 1, s_abort)) {
          alive = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sp = smem + st.i * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st.i], C::STAGE_BYTES);
#pragma unroll
          for (int a = 0; a < NACC; ++a)
            tma_load_2d(sp + a * C::A_BYTES, &args.tmA[set][C::EPI == 0 ? 0 : a], &full[st.i], kb * 128,
                        arow + (C::EPI == 0 ? a * 128 : 0));
          tma_load_2d(sp + NACC * C::A_BYTES, &args.tmB, &full[st.i], kb * 128, td.x);
        }
        float* slot = raw + sl.i * C::RAW_FLOATS;
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) {
          const int r = lane + 32 * u;
          if (r < nr) cp_async_4(slot + r, asp + (int64_t)r * args.as_row + (int64_t)kb * args.as_kb);
        }
        if (lane < NACC) cp_async_4(slot + BN + lane, wsp + kb);
        cp_async_mbar_arrive(&sready[sl.i]);
        st.next();
        sl.next();
        ++issued;
        if (kb == kb_fetch) {
          nt = __shfl_sync(0xffffffffu, nt, 0);
          if (nt < ntiles) ntd = args.tiles[nt];
        }
      }
      if (!alive) break;
      tile = nt;
      td = ntd;
    }
    cp_async_wait_all();
    // no copy into this CTA's shared memory may outlive the CTA
    if (lane == 0) {
      const uint32_t first = issued > (uint32_t)NSTAGE ? issued - NSTAGE : 0;
      for (uint32_t q = first; q < issued; ++q) wait_plain(&full[q % NSTAGE], (q / NSTAGE) & 1, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ───────────── MMA issuers: warp 1 takes even K steps, warp 2 odd ones ─────────────
    const int me = warp - 1;
    Ring<NSTAGE> st;
    Ring<NBUF> bf;
    uint32_t step = 0;
    bool alive = true;
    Ring<C::TRING> tr;
    for (;;) {
      int4 td;
      if (!next_tile(tr, td) || td.x < 0) break;
      const int nr = td.y;
      int n_eff = (nr + 15) & ~15;
      n_eff = n_eff < 16 ? 16 : (n_eff > BN ? BN : n_eff);
      const uint32_t idesc = umma_idesc_e4m3(128, n_eff);
      for (int kb = 0; kb < nkb; ++kb, ++step, st.next(), bf.next()) {
        if ((int)(step & 1) != me) continue;
        if (!mbar_wait(&acce[bf.i], bf.ph ^ 1, s_abort) || !mbar_wait(&full[st.i], st.ph, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          uint8_t* sp = smem + st.i * C::STAGE_BYTES;
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sp + NACC * C::A_BYTES));
          uint64_t adesc[NACC];
#pragma unroll
          for (int a = 0; a < NACC; ++a) adesc[a] = umma_desc_sw128(smem_u32(sp + a * C::A_BYTES));
          const uint32_t d0 = tmem + (uint32_t)(bf.i * NACC * BN);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int a = 0; a < NACC; ++a)
              umma_f8(d0 + (uint32_t)(a * BN), adesc[a] + 2 * kk, bdesc + 2 * kk, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty[st.i]);
          umma_commit(&accf[bf.i]);
        }
        __syncwarp();
      }
      if (!alive) break;
    }
    // every MMA must have completed before TMEM is released
    if (lane == 0) {
      umma_commit(&drain[me]);
      wait_plain(&drain[me], 0, kWaitTimeoutNs);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ───────────── scale warp: combined scale per column and accumulator, once per K step ─────────────
    Ring<NSLOT> sl;
    bool alive = true;
    Ring<C::TRING> tr;
    for (;;) {
      int4 td;
      if (!next_tile(tr, td) || td.x < 0) break;
      const int nr = td.y;
      for (int kb = 0; kb < nkb; ++kb, sl.next()) {
        if (!mbar_wait(&sready[sl.i], sl.ph, s_abort)) {
          alive = false;
          break;
        }
        const float* slot = raw + sl.i * C::RAW_FLOATS;
        float* sc = scl + sl.i * C::SCL_FLOATS;
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const float w = slot[BN + a];
#pragma unroll
          for (int u = 0; u < BN / 32; ++u) {
            const int r = lane + 32 * u;
            sc[a * BN + r] = r < nr ? slot[r] * w : 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&cready[sl.i]);
      }
      if (!alive) break;
    }
  } else {
    // ───────────── epilogue warpgroups ─────────────
    const int ew = warp - 4, wg = ew >> 2, q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    Ring<NBUF> bf;
    Ring<NSLOT> sl;
    uint32_t ephase = 0;
    bool alive = true;
    // the 4 warps of this warpgroup meet (bounded) before and after sharing the amax slots
    auto wg_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&epib[wg]);
      const bool ok = mbar_wait(&epib[wg], ephase, s_abort);
      ephase ^= 1;
      return ok;
    };
    Ring<C::TRING> tr;
    for (;;) {
      int4 td;
      if (!next_tile(tr, td) || td.x < 0) break;
      const int nr = td.y;
      int n_eff = (nr + 15) & ~15;
      n_eff = n_eff < 16 ? 16 : (n_eff > BN ? BN : n_eff);
      // this warpgroup's accumulators [a0, a0 + NA) and columns [cb, cb + CW); the 32-column
      // groups of them that hold real columns
      constexpr int NA = C::NA;
      const int a0 = C::ASPLIT ? wg : 0;
      const int cb = C::ASPLIT ? 0 : wg * CW;
      const int span = n_eff - cb;
      constexpr int LW = C::LW;
      const int ngroups = span <= 0 ? 0 : (span >= CW ? CW / LW : (span + LW - 1) / LW);
      float acc[NA][CW];
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int c = 0; c < CW; ++c) acc[a][c] = 0.f;
      for (int kb = 0; kb < nkb; ++kb, bf.next(), sl.next()) {
        if (!mbar_wait(&accf[bf.i], bf.ph, s_abort) || !mbar_wait(&cready[sl.i], sl.ph, s_abort)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const float* sc = scl + sl.i * C::SCL_FLOATS;
        if (ngroups == 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[bf.i]);
        }
#pragma unroll
        for (int aa = 0; aa < NA; ++aa) {
          const int a = a0 + aa;
#pragma unroll
          for (int g = 0; g < CW / LW; ++g) {
            const int col = cb + g * LW;
            if (g < ngroups) {
              float pv[LW];
              const uint32_t ta = tmem + tlane + (uint32_t)((bf.i * NACC + a) * BN + col);
              if constexpr (LW == 32) {
                if (col + 32 <= n_eff) tmem_ld32(ta, pv);
                else tmem_ld16p(ta, pv);
              } else {
                tmem_ld16p(ta, pv);
              }
              tmem_ld_wait();
              if (aa == NA - 1 && g == ngroups - 1) {  // last load of this step: buffer back to the MMA warps
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acce[bf.i]);
              }
              const float4* s4p = reinterpret_cast<const float4*>(sc + a * BN + col);
#pragma unroll
              for (int i4 = 0; i4 < LW / 4; ++i4) {
                const float4 s4 = s4p[i4];
                float* ac = &acc[aa][g * LW + i4 * 4];
                fma2(ac[0], ac[1], pv[i4 * 4 + 0], pv[i4 * 4 + 1], s4.x, s4.y);
                fma2(ac[2], ac[3], pv[i4 * 4 + 2], pv[i4 * 4 + 3], s4.z, s4.w);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[sl.i]);
      }
      if (!alive) break;
      const int64_t row0 = td.x;
      const int ncol = td.w * 128 + lrow;
      if constexpr (C::EPI == 0) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
#pragma unroll
        for (int aa = 0; aa < NA; ++aa) {
          const int col = (td.w * NACC + a0 + aa) * 128 + lrow;
#pragma unroll
          for (int c = 0; c < CW; ++c) {
            const int t = cb + c;
            if (t >= nr) break;
            out[(row0 + t) * args.out_ld + col] = __float2bfloat16_rn(acc[aa][c]);
          }
        }
      } else {
        // SwiGLU exactly as the reference rounds it: gate/up GEMM outputs are bf16
        // (gate_up_out, :610-619), silu() rounds to bf16, the product rounds to bf16 (:624);
        // then _fast_fp8_quantize over these 128 channels (:637).
#pragma unroll
        for (int c = 0; c < CW; ++c) {
          if (wg * CW + c >= nr) break;  // warp-uniform
          const float g = bf16_round(acc[0][c]);
          const float u = bf16_round(acc[NA - 1][c]);
          const float sg = bf16_round(__fdiv_rn(g, 1.0f + expf(-g)));
          const float av = bf16_round(sg * u);
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
  pdl_trigger();
}

}  // namespace msv
