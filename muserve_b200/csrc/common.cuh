// Device helpers shared by the MoE kernels: bf16/e4m3 conversions, warp reductions,
// mbarriers with bounded waits, TMA tile loads, and the tcgen05 (5th-gen tensor core /
// tensor memory) instructions used by the grouped GEMM.  sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/muserve_moe.h"

#define MSV_DEVICE __device__ __forceinline__

namespace msv {

// element `hi` (0: low half, 1: high half) of two packed bf16 values, widened exactly to f32
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t w, int hi) {
  return __uint_as_float(hi ? (w & 0xffff0000u) : (w << 16));
}

// Programmatic dependent launch.  Every kernel of this library is launched (launch_k) so that it
// may start while the previous kernel on its stream is finishing.  pdl_wait() blocks until that
// kernel has completed and its writes are visible; each kernel calls it before touching any
// global memory another kernel of the stream reads or writes (only its own set-up of shared
// memory, barriers and TMEM comes first).  pdl_trigger() lets the next kernel start launching;
// kernels call it once their main work is done.
MSV_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MSV_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host-side count of the kernels this library has launched (msv_launch_count).
inline std::atomic<unsigned long long> g_launch_count{0};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args&&... args) {
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Every device-side wait gives up after this long and reports MSV_ERR_TIMEOUT through the
// kernel's error word; nothing in these kernels can spin forever.  Hot-path waits count SM
// cycles (clock64, cheap to read); 4e9 cycles is about 2 s at the B200's 1.97 GHz.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s
constexpr long long kWaitTimeoutCycles = 4000000000ll;

// ── numerics ────────────────────────────────────────────────────────────────────────────

MSV_DEVICE float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Reference clamp semantics (torch.clamp): NaN propagates, unlike fminf/fmaxf.
MSV_DEVICE float clamp_pm(float v, float lim) {
  v = (v > lim) ? lim : v;
  v = (v < -lim) ? -lim : v;
  return v;
}

// e4m3 (fn) round-to-nearest-even with saturation; inputs are already clamped to ±448.
MSV_DEVICE uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// torch's amax propagates NaN; fmaxf does not.  |x| values are >= 0 so NaN is the only
// special case.
MSV_DEVICE float nanmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fffffff) : fmaxf(a, b);
}

MSV_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
MSV_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

MSV_DEVICE uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

MSV_DEVICE unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MSV_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ── mbarrier ────────────────────────────────────────────────────────────────────────────

MSV_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
MSV_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
MSV_DEVICE void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

MSV_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MSV_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
MSV_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that suspends the thread until the phase completes or `ns` nanoseconds pass, so a
// waiting warp takes no issue slots from the warps sharing its scheduler.
constexpr uint32_t kSuspendNs = 200000;  // 0.2 ms: how often a sleeping waiter re-checks abort/timeout
MSV_DEVICE bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false (and raises
// *abort) when the wait runs out or another role of the CTA already aborted.
MSV_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, kSuspendNs)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitTimeoutCycles) {
      *abort = 1;
      return false;
    }
  }
}

// ── TMA ─────────────────────────────────────────────────────────────────────────────────

MSV_DEVICE void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled load (no multicast).  x = innermost coordinate in elements (multiple of 16 bytes
// here: always a multiple of 128 fp8 elements), y = row.
MSV_DEVICE void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load (no multicast): coordinates {x, y, z}, x a multiple of 16 bytes.
MSV_DEVICE void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ── tcgen05 ─────────────────────────────────────────────────────────────────────────────

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle that TMA's SWIZZLE_128B writes: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start>>4 [0,14), leading byte offset>>4 [16,30) (unused for this layout, 1),
// stride byte offset>>4 [32,46) = 1024>>4, descriptor version 1 [46,48), layout 2 =
// SWIZZLE_128B [61,64).  The tile base must be 1024-byte aligned.
MSV_DEVICE uint64_t umma_desc_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f8f6f4: D fp32 [4,6)=1, A=B=e4m3 (0), both K-major,
// N>>3 at [17,23), M>>4 at [24,29).
MSV_DEVICE uint32_t umma_idesc_e4m3(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

MSV_DEVICE void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread has completed.
MSV_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

MSV_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MSV_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-wide: allocate ncols (power of two >= 32) TMEM columns; the address lands in *dst.
MSV_DEVICE void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MSV_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Warp-wide load of 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
MSV_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp-wide load of 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
MSV_DEVICE void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
MSV_DEVICE void tmem_ld16p(uint32_t taddr, float* v) {
  float t[16];
  tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(t));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = t[i];
}
MSV_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

MSV_DEVICE void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

MSV_DEVICE void cp_async_4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Arrive on `bar` once this thread's earlier cp.async copies have landed (the barrier's
// expected count includes this arrival).
MSV_DEVICE void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MSV_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

}  // namespace msv
