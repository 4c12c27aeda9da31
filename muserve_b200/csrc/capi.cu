// Host side of the C ABI declared in include/muserve_moe.h: argument checks, tensor-map
// cache, kernel-variant choice and the launch sequence of the MoE layer.  Nothing here
// allocates device memory or synchronises a stream (msv_check_device_error excepted).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "combine_ar.cuh"
#include "dispatch_quant.cuh"
#include "common.cuh"
#include "grouped_gemm.cuh"
#include "grouped_gemm_rows.cuh"
#include "grouped_gemm_pair.cuh"
#include "quant_combine.cuh"
#include "route.cuh"
#include "norm.cuh"
#include "router_gemm.cuh"

namespace msv {

// Error word raised by device-side bounded waits (MSV_ERR_TIMEOUT); one per device.
__device__ int g_dev_err;

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MSV_OK;
  return fail(MSV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  int num_sms = 0;
  int* err_word = nullptr;
};

std::mutex g_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(MSV_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.num_sms == 0) {
    int major = 0;
    if (int rc = cuda_check(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "attr"))
      return rc;
    if (major != 10) return fail(MSV_ERR_UNSUPPORTED, "device %d is sm_%d0; this library is built for sm_100a", dev, major);
    if (int rc = cuda_check(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev), "attr"))
      return rc;
    void* p = nullptr;
    if (int rc = cuda_check(cudaGetSymbolAddress(&p, g_dev_err), "cudaGetSymbolAddress(g_dev_err)")) return rc;
    d.err_word = static_cast<int*>(p);
  }
  *out = &d;
  return MSV_OK;
}

// ── tensor maps ───────────────────────────────────────────────────────────────────────────

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

// pointers msv_ipc_import returned -> the mapped allocation's base (for msv_ipc_close)
std::mutex g_ipc_mu;
std::unordered_map<uintptr_t, void*> g_ipc_bases;

// one rank's shared buffer: the receive area and the result area, each max_tokens x H values
// as 8-byte words of two bf16 values and a flag
size_t tp_area_bytes(int max_tokens, int hidden) {
  return (((size_t)max_tokens * (size_t)hidden * 4) + 255) & ~(size_t)255;
}

struct MapKey {
  uintptr_t base;
  uint64_t rows, cols, stride;
  uint32_t box_rows, box_cols, f32;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && stride == o.stride && box_rows == o.box_rows &&
           box_cols == o.box_cols && f32 == o.f32;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = k.base * 0x9E3779B97F4A7C15ull;
    h ^= (k.rows + 0x632BE59BD9B4E019ull) + (h << 6) + (h >> 2);
    h ^= (k.cols * 31 + k.stride * 131 + k.box_rows + ((uint64_t)k.box_cols << 20) + ((uint64_t)k.f32 << 40)) + (h << 6) +
         (h >> 2);
    return h;
  }
};
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D e4m3 (byte) matrix [rows, cols] with row stride `stride` bytes, box [box_rows x 128 B],
// 128-byte swizzle, zero fill out of bounds.  Cached: a map only encodes addresses and sizes.
int tensor_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t stride, uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(MSV_ERR_INVALID, "operand not 16-byte aligned");
  if (stride % 16 != 0 || cols % 128 != 0) return fail(MSV_ERR_INVALID, "operand row stride / width not multiple of 16/128");
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride, box_rows, 128, 0};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MSV_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSV_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu", (int)r,
                                     (unsigned long long)rows, (unsigned long long)cols);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return MSV_OK;
}

// 2-D bf16 matrix [rows, cols] with row stride `stride` bytes, box [box_rows x 64 elements]
// (128 bytes), 128-byte swizzle, zero fill out of bounds.  Cached like tensor_map.
int tensor_map_bf16(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t stride, uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(MSV_ERR_INVALID, "bf16 operand not 16-byte aligned");
  if (stride % 16 != 0 || cols % 64 != 0) return fail(MSV_ERR_INVALID, "bf16 operand row stride / width not multiple of 16 B / 64");
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride, box_rows, 64, 3};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MSV_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSV_ERR_INVALID, "cuTensorMapEncodeTiled (bf16) failed (%d) rows=%llu cols=%llu", (int)r,
                                     (unsigned long long)rows, (unsigned long long)cols);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return MSV_OK;
}

// 3-D view of an e4m3 (byte) matrix [rows, cols] as [cols/128][rows][128 B]: box [nkb blocks x
// box_rows x 128 B], 128-byte swizzle, zero fill; one load brings nkb consecutive K blocks.
int tensor_map_kblocks(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t stride,
                       uint32_t box_rows, uint32_t nkb) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(MSV_ERR_INVALID, "operand not 16-byte aligned");
  if (stride % 16 != 0 || cols % 128 != 0) return fail(MSV_ERR_INVALID, "operand row stride / width not multiple of 16/128");
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride, box_rows, nkb, 2};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MSV_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  CUtensorMap m;
  cuuint64_t dims[3] = {128, rows, cols / 128};
  cuuint64_t strides[2] = {stride, 128};
  cuuint32_t box[3] = {128, box_rows, nkb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSV_ERR_INVALID, "cuTensorMapEncodeTiled (3-D) failed (%d) rows=%llu cols=%llu", (int)r,
                                     (unsigned long long)rows, (unsigned long long)cols);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return MSV_OK;
}

// 2-D fp32 matrix [rows, cols] with row stride `stride` bytes (a multiple of 16), box
// [box_rows x box_cols] (box_cols * 4 a multiple of 16), no swizzle, zero fill out of bounds.
int tensor_map_f32(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t stride, uint32_t box_cols,
                   uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || stride % 16 != 0 || (box_cols * 4) % 16 != 0)
    return fail(MSV_ERR_INVALID, "fp32 scale matrix not 16-byte aligned (base, row stride or box width)");
  MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride, box_rows, box_cols, 1};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MSV_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSV_ERR_INVALID, "cuTensorMapEncodeTiled (fp32) failed (%d) rows=%llu cols=%llu", (int)r,
                                     (unsigned long long)rows, (unsigned long long)cols);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return MSV_OK;
}

// ── grouped GEMM variants ────────────────────────────────────────────────────────────────

using G1Small = GemmCfg<32, 2, 1, 2>;   // gate+up -> SwiGLU -> e4m3, <= 32 rows per chunk, two epilogue
                                        // warpgroups of 16 token columns each
using G2Small = GemmCfg<32, 1, 0, 1>;   // plain -> bf16, <= 32 rows per chunk
using G2Pair = GemmCfg<32, 2, 0, 2>;    // plain -> bf16, two 128-row blocks per tile (32 KB of weights per stage),
                                        // one epilogue warpgroup per block
using G2Large = GemmCfg<192, 1, 0, 3>;  // plain -> bf16, <= 192 rows per chunk
using R1 = RowsCfg<1, 32, 2>;          // tokens on M: gate+up halves -> SwiGLU -> e4m3 (K <= 4096)
using R2 = RowsCfg<0, 8, 4>;           // tokens on M: plain -> bf16 (K <= 1024)
using P1 = PairCfg<32, 2>;             // CTA pairs, 256 tokens x 128 channels: gate+up -> SwiGLU -> e4m3 (K <= 4096)

// The grouped GEMM claims its tiles after the first round from the counter the tile-list
// builder zeroed (ntiles[1]) when a tile has at least 4 K steps; shorter tiles keep the static
// round robin, where a claim per tile costs more than the balance it buys.
int* claim_counter(int* ntiles, int nkb) { return nkb >= 4 ? ntiles + 1 : nullptr; }

template <class C>
int launch_gemm(const GemmArgs& a, cudaStream_t st, int num_sms) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    for (auto fn : {k_grouped_gemm<C, false>, k_grouped_gemm<C, true>})
      if (int rc = cuda_check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES),
                              "cudaFuncSetAttribute(grouped_gemm)"))
        return rc;
    configured[dev] = true;
  }
  if (a.tile_next)
    launch_k(k_grouped_gemm<C, true>, dim3(num_sms), dim3(C::THREADS), C::SMEM_BYTES, st, a);
  else
    launch_k(k_grouped_gemm<C, false>, dim3(num_sms), dim3(C::THREADS), C::SMEM_BYTES, st, a);
  return cuda_check(cudaGetLastError(), "launch grouped_gemm");
}

template <class C>
int launch_gemm_rows(const RowsArgs& a, cudaStream_t st, int num_sms) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    if (int rc = cuda_check(cudaFuncSetAttribute(k_grouped_gemm_rows<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::SMEM_BYTES),
                            "cudaFuncSetAttribute(grouped_gemm_rows)"))
      return rc;
    configured[dev] = true;
  }
  launch_k(k_grouped_gemm_rows<C>, dim3(num_sms), dim3(C::THREADS), C::SMEM_BYTES, st, a);
  return cuda_check(cudaGetLastError(), "launch grouped_gemm_rows");
}

// Grid cap of the fused combine + all-reduce for blocks of `threads` threads: the smallest
// per-SM occupancy over the three combine-mode instances times the SMs, at most kArMaxCtas.
// Independent of the mode, so a group's token-to-CTA mapping never changes between calls.
int combine_ar_grid_cap(int threads, int num_sms, int* cap) {
  void (*kerns[3])(CombineArArgs) = {k_combine_ar<MSV_COMBINE_V2>, k_combine_ar<MSV_COMBINE_DISPATCH>,
                                     k_combine_ar<MSV_COMBINE_BATCHED>};
  int per_sm = 1 << 30;
  for (auto* k : kerns) {
    int n = 0;
    if (int rc = cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, 0),
                            "cudaOccupancyMaxActiveBlocksPerMultiprocessor"))
      return rc;
    per_sm = n < per_sm ? n : per_sm;
  }
  per_sm = per_sm < 1 ? 1 : per_sm;
  const int g = per_sm * num_sms;
  *cap = g < kArMaxCtas ? g : kArMaxCtas;
  return MSV_OK;
}

// CTA-pair kernels: 2-CTA clusters, as many as can be resident at once (persistent).
template <class C>
int launch_gemm_pair(const RowsArgs& a, cudaStream_t st, int num_sms) {
  static int npairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!npairs[dev]) {
    if (int rc = cuda_check(cudaFuncSetAttribute(k_grouped_gemm_pair<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::SMEM_BYTES),
                            "cudaFuncSetAttribute(grouped_gemm_pair)"))
      return rc;
    cfg.gridDim = dim3((unsigned)(num_sms & ~1));
    int n = 0;
    if (int rc = cuda_check(cudaOccupancyMaxActiveClusters(&n, k_grouped_gemm_pair<C>, &cfg),
                            "cudaOccupancyMaxActiveClusters(grouped_gemm_pair)"))
      return rc;
    if (n < 1) return fail(MSV_ERR_UNSUPPORTED, "grouped_gemm_pair: no 2-CTA cluster fits on this device");
    npairs[dev] = n < num_sms / 2 ? n : num_sms / 2;
  }
  cfg.gridDim = dim3((unsigned)(2 * npairs[dev]));
  cfg.numAttrs = 2;
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, k_grouped_gemm_pair<C>, a), "launch grouped_gemm_pair")) return rc;
  return cuda_check(cudaGetLastError(), "launch grouped_gemm_pair");
}

int launch_gemm_variant(bool small, const GemmArgs& a, cudaStream_t st, int nsm) {
  return small ? launch_gemm<G2Small>(a, st, nsm) : launch_gemm<G2Large>(a, st, nsm);
}
int variant_bn(bool small) { return small ? G2Small::BN : G2Large::BN; }

// ── workspace carving ────────────────────────────────────────────────────────────────────

struct Carver {
  uint8_t* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

size_t tile_cap(int groups, int rows, int bn, int nb) {
  return (size_t)nb * ((size_t)groups + (size_t)(rows + bn - 1) / bn + 1);
}

bool is_pow2_aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace msv

// ── static scratch of msv_ragged_moe_gemm_fp8_noalloc ────────────────────────────────────
// The allocation-free ragged GEMM keeps its tile list here instead of in a caller workspace.
// Layout: the int tile count at byte 0, the int4 tile list from byte 256.  Each device's
// context holds its own copy; on one device every call shares it.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
constexpr size_t kNoAllocTileOffset = 256;
constexpr size_t kNoAllocMaxTiles = (kNoAllocScratchBytes - kNoAllocTileOffset) / sizeof(int4);  // 262128
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace msv {
namespace {

uint8_t* g_noalloc_ptr[64];  // device address of g_noalloc_scratch per device, guarded by g_mu

// Set-up, once per device, with that device current: look up the array's device address.
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(MSV_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (int rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(g_noalloc_scratch)"))
      return rc;
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MSV_OK;
}

// Same map as tensor_map() but encoded on every call, outside the host-side cache, so that
// the allocation-free entry point does not grow a host container either.
int tensor_map_uncached(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t stride,
                        uint32_t box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(MSV_ERR_INVALID, "operand not 16-byte aligned");
  if (stride % 16 != 0 || cols % 128 != 0) return fail(MSV_ERR_INVALID, "operand row stride / width not multiple of 16/128");
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSV_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu", (int)r,
                                     (unsigned long long)rows, (unsigned long long)cols);
  return MSV_OK;
}

}  // namespace
}  // namespace msv

using namespace msv;

// ═════════════════════════════════════════════════════════════════════════════════════════
extern "C" {

const char* msv_last_error(void) { return t_err.c_str(); }
int msv_version(void) { return 100; }

int msv_check_device_error(msv_stream_t stream) {
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (int rc = cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize")) return rc;
  int v = 0;
  if (int rc = cuda_check(cudaMemcpy(&v, d->err_word, sizeof(int), cudaMemcpyDeviceToHost), "read error word")) return rc;
  int z = 0;
  if (int rc = cuda_check(cudaMemcpy(d->err_word, &z, sizeof(int), cudaMemcpyHostToDevice), "clear error word")) return rc;
  if (v != 0) return fail(MSV_ERR_TIMEOUT, "a bounded device-side wait gave up (code %d)", v);
  return MSV_OK;
}

unsigned long long msv_launch_count(void) { return g_launch_count.load(std::memory_order_relaxed); }

int msv_route_topk(const float* logits, int64_t ld, int T, int E, int k, int renormalize, void* topk_w, int w_dtype,
                   void* topk_ids, int ids_dtype, msv_stream_t stream) {
  if (!logits || !topk_ids || T < 0 || E < 1 || E > 1024 || k < 1 || k > 16 || k > E || ld < E)
    return fail(MSV_ERR_INVALID, "msv_route_topk: bad arguments (T=%d E=%d k=%d ld=%lld)", T, E, k, (long long)ld);
  if ((w_dtype != MSV_F32 && w_dtype != MSV_BF16) || (ids_dtype != MSV_I32 && ids_dtype != MSV_I64))
    return fail(MSV_ERR_INVALID, "msv_route_topk: dtype codes");
  if (T == 0) return MSV_OK;
  const size_t sm = route_smem_bytes(E);
  launch_k(k_route_topk, dim3((T + kRouteWarps - 1) / kRouteWarps), dim3(kRouteWarps * 32), sm, stream, 
      logits, ld, T, E, k, 1, renormalize, topk_w, w_dtype, topk_ids, ids_dtype, nullptr, nullptr);
  return cuda_check(cudaGetLastError(), "launch route_topk");
}

namespace {
// K splits of the router GEMM: enough CTAs to cover the SMs when the token and expert tiles
// alone do not, at least two 64-wide K blocks per split, at most 32 splits.
int router_splits(int T, int H, int E, int num_sms) {
  const int base = ((T + kRtBM - 1) / kRtBM) * ((E + kRtBN - 1) / kRtBN);
  const int nkb = H / 64;
  int s = base > 0 ? num_sms / base : 1;
  s = s < 1 ? 1 : s;
  const int cap = nkb / 2 < 32 ? nkb / 2 : 32;
  s = s > cap ? cap : s;
  s = s < 1 ? 1 : s;
  const int kps = (nkb + s - 1) / s;
  return (nkb + kps - 1) / kps;  // every split non-empty
}
}  // namespace

size_t msv_router_workspace_size(int T, int H, int E) {
  if (T < 0 || H <= 0 || H % 64 || E < 16 || E % 16 || E > 1024) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int nsm = 148;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  // the splits' partial sums, then the summed logits
  return ((size_t)router_splits(T, H, E, nsm) + 1) * (size_t)(T > 0 ? T : 1) * (size_t)E * sizeof(float) + 512;
}

namespace {
int router_from_hidden_impl(const void* hidden, const void* gate_w, int T, int H, int E, int k, int renormalize,
                            int round_logits_bf16, const float* logit_bias, void* topk_w, int w_dtype, void* topk_ids,
                            int ids_dtype, float* logits_out, void* workspace, size_t workspace_bytes,
                            msv_stream_t stream) {
  if (!hidden || !gate_w || !topk_ids || T < 0 || H <= 0 || H % 64 || E < 16 || E % 16 || E > 1024 || k < 1 ||
      k > 16 || k > E)
    return fail(MSV_ERR_INVALID,
                "msv_router_from_hidden: bad arguments (T=%d H=%d E=%d k=%d; H %% 64 == 0, 16 <= E <= 1024, E %% 16 == 0)",
                T, H, E, k);
  if ((w_dtype != MSV_F32 && w_dtype != MSV_BF16) || (ids_dtype != MSV_I32 && ids_dtype != MSV_I64))
    return fail(MSV_ERR_INVALID, "msv_router_from_hidden: dtype codes");
  if (logits_out && !is_pow2_aligned(logits_out, 16))
    return fail(MSV_ERR_INVALID, "msv_router_from_hidden: logits_out must be 16-byte aligned");
  if (T == 0) return MSV_OK;
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  const int nsplit = router_splits(T, H, E, d->num_sms);
  const size_t part_bytes = (((size_t)nsplit * T * E * sizeof(float)) + 255) & ~(size_t)255;
  const size_t need = part_bytes + (size_t)T * E * sizeof(float);
  if (!workspace || workspace_bytes < need || !is_pow2_aligned(workspace, 256))
    return fail(MSV_ERR_INVALID, "msv_router_from_hidden: workspace %zu < %zu bytes or not 256-byte aligned",
                workspace_bytes, need);
  static bool configured[64] = {};
  if (!configured[dev]) {
    if (int rc = cuda_check(cudaFuncSetAttribute(k_router_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmem),
                            "cudaFuncSetAttribute(router_gemm)"))
      return rc;
    configured[dev] = true;
  }
  RouterArgs a{};
  if (int rc = tensor_map_bf16(&a.tmA, hidden, (uint64_t)T, (uint64_t)H, (uint64_t)H * 2, kRtBM)) return rc;
  if (int rc = tensor_map_bf16(&a.tmB, gate_w, (uint64_t)E, (uint64_t)H, (uint64_t)H * 2, kRtBN)) return rc;
  a.T = T;
  a.H = H;
  a.E = E;
  const int nkb = H / 64;
  a.kb_per_split = (nkb + nsplit - 1) / nsplit;
  float* logits = logits_out ? logits_out : static_cast<float*>(workspace);
  // one split: the GEMM writes the (rounded) logits itself; several: partial sums, then a sum
  a.round_bf16 = nsplit == 1 && round_logits_bf16;
  a.part = nsplit == 1 ? logits : static_cast<float*>(workspace);
  a.err = d->err_word;
  const dim3 grid((T + kRtBM - 1) / kRtBM, (E + kRtBN - 1) / kRtBN, nsplit);
  launch_k(k_router_gemm, dim3(grid), dim3(128), kRtSmem, stream, a);
  if (int rc = cuda_check(cudaGetLastError(), "launch router_gemm")) return rc;
  if (nsplit > 1) {
    // the splits summed in order (and rounded) into the logits the routing reads
    if (!logits_out) logits = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + part_bytes);
    const int64_t n4 = (int64_t)T * E / 4;
    launch_k(k_router_sum_splits, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0, stream, a.part, nsplit, n4, round_logits_bf16 ? 1 : 0,
                                                                            logits);
    if (int rc = cuda_check(cudaGetLastError(), "launch router_sum_splits")) return rc;
  }
  launch_k(k_route_topk, dim3((T + kRouteWarps - 1) / kRouteWarps), dim3(kRouteWarps * 32), route_smem_bytes(E), stream, 
      logits, E, T, E, k, 1, renormalize, topk_w, w_dtype, topk_ids, ids_dtype, nullptr, logit_bias);
  return cuda_check(cudaGetLastError(), "launch route_topk");
}
}  // namespace

int msv_router_from_hidden(const void* hidden, const void* gate_w, int T, int H, int E, int k, int renormalize,
                           int round_logits_bf16, void* topk_w, int w_dtype, void* topk_ids, int ids_dtype,
                           float* logits_out, void* workspace, size_t workspace_bytes, msv_stream_t stream) {
  return router_from_hidden_impl(hidden, gate_w, T, H, E, k, renormalize, round_logits_bf16, nullptr, topk_w, w_dtype,
                                 topk_ids, ids_dtype, logits_out, workspace, workspace_bytes, stream);
}

int msv_router_from_hidden_bias(const void* hidden, const void* gate_w, int T, int H, int E, int k, int renormalize,
                                int round_logits_bf16, const float* logit_bias, void* topk_w, int w_dtype,
                                void* topk_ids, int ids_dtype, float* logits_out, void* workspace,
                                size_t workspace_bytes, msv_stream_t stream) {
  if (!logit_bias) return fail(MSV_ERR_INVALID, "msv_router_from_hidden_bias: null logit_bias");
  return router_from_hidden_impl(hidden, gate_w, T, H, E, k, renormalize, round_logits_bf16, logit_bias, topk_w,
                                 w_dtype, topk_ids, ids_dtype, logits_out, workspace, workspace_bytes, stream);
}

int msv_add_rms_norm_gemma(void* h, const void* add, const void* weight, int T, int H, float eps, void* out,
                           msv_stream_t stream) {
  if (!h || T < 0 || H <= 0 || H % 8 || H > 8 * kNormMaxVec * kNormThreads || (out && !weight) || (!out && !add))
    return fail(MSV_ERR_INVALID, "msv_add_rms_norm_gemma: bad arguments (T=%d H=%d; H %% 8 == 0, H <= %d)", T, H,
                8 * kNormMaxVec * kNormThreads);
  if (!is_pow2_aligned(h, 16) || (add && !is_pow2_aligned(add, 16)) || (weight && !is_pow2_aligned(weight, 16)) ||
      (out && !is_pow2_aligned(out, 16)))
    return fail(MSV_ERR_INVALID, "msv_add_rms_norm_gemma: pointers must be 16-byte aligned");
  if (T == 0) return MSV_OK;
  launch_k(k_add_rms_norm, dim3(T), dim3(kNormThreads), 0, stream, static_cast<__nv_bfloat16*>(h),
           static_cast<const __nv_bfloat16*>(add), static_cast<const __nv_bfloat16*>(weight),
           static_cast<__nv_bfloat16*>(out), H, eps);
  return cuda_check(cudaGetLastError(), "launch add_rms_norm");
}

int msv_topk_select(const float* values, int64_t ld, int T, int E, int k, void* topk_ids, int ids_dtype,
                    float* out_values, msv_stream_t stream) {
  if (!values || !topk_ids || T < 0 || E < 1 || E > 1024 || k < 1 || k > 16 || k > E || ld < E)
    return fail(MSV_ERR_INVALID, "msv_topk_select: bad arguments");
  if (ids_dtype != MSV_I32 && ids_dtype != MSV_I64) return fail(MSV_ERR_INVALID, "msv_topk_select: ids dtype");
  if (T == 0) return MSV_OK;
  launch_k(k_route_topk, dim3((T + kRouteWarps - 1) / kRouteWarps), dim3(kRouteWarps * 32), route_smem_bytes(E), stream, 
      values, ld, T, E, k, 0, 0, nullptr, MSV_F32, topk_ids, ids_dtype, out_values, nullptr);
  return cuda_check(cudaGetLastError(), "launch topk_select");
}

int msv_moe_permute(const void* topk_ids, int ids_dtype, int T, int k, int num_experts, int placement, int tp, int rank,
                    int alignment, int64_t* sort_order, int64_t* inverse_order, int32_t* sorted_expert_ids,
                    int32_t* expert_counts, int32_t* num_local, msv_stream_t stream) {
  if (!topk_ids || !num_local || T < 0 || k < 1 || num_experts < 1 || (ids_dtype != MSV_I32 && ids_dtype != MSV_I64))
    return fail(MSV_ERR_INVALID, "msv_moe_permute: bad arguments");
  if (placement && (tp < 1 || rank < 0 || rank >= tp)) return fail(MSV_ERR_INVALID, "msv_moe_permute: tp/rank");
  const int e_local = placement ? (num_experts + tp - 1) / tp : num_experts;
  if (e_local > 1024) return fail(MSV_ERR_UNSUPPORTED, "msv_moe_permute: more than 1024 local experts");
  PermuteArgs p{};
  p.ids = topk_ids;
  p.ids_i64 = ids_dtype == MSV_I64;
  p.T = T;
  p.k = k;
  p.num_experts = num_experts;
  p.placement = placement;
  p.tp = placement ? tp : 1;
  p.rank = placement ? rank : 0;
  p.alignment = alignment;
  p.e_local = e_local;
  p.sort_order = sort_order;
  p.inverse_order = inverse_order;
  p.sorted_expert_ids = sorted_expert_ids;
  p.expert_counts = expert_counts;
  p.num_local = num_local;
  const size_t sm = permute_smem_bytes(e_local);
  if (sm > 48 * 1024)
    if (int rc = cuda_check(cudaFuncSetAttribute(k_permute, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                            "cudaFuncSetAttribute(permute)"))
      return rc;
  launch_k(k_permute, dim3(1), dim3(kPermThreads), sm, stream, p);
  return cuda_check(cudaGetLastError(), "launch permute");
}

int msv_fp8_quant_128(const void* x, int64_t ldx, int M, int K, const int32_t* row_index, uint8_t* q, int64_t ldq,
                      float* scale, int64_t s_row, int64_t s_kb, msv_stream_t stream) {
  if (!x || !q || !scale || M < 0 || K <= 0 || K % 128 != 0 || ldx < K || ldq < K)
    return fail(MSV_ERR_INVALID, "msv_fp8_quant_128: bad arguments (M=%d K=%d)", M, K);
  if (!is_pow2_aligned(x, 16) || (ldx * 2) % 16 != 0 || !is_pow2_aligned(q, 8) || ldq % 8 != 0)
    return fail(MSV_ERR_INVALID, "msv_fp8_quant_128: x rows must be 16-byte aligned, q rows 8-byte aligned");
  if (M == 0) return MSV_OK;
  QuantArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.K = K;
  a.rows_a = M;
  a.idx_a = row_index;
  a.q = q;
  a.ldq = ldq;
  a.scale = scale;
  a.s_row = s_row;
  a.s_kb = s_kb;
  launch_k(k_quant_rows, dim3((M + kQuantRowsPerCta - 1) / kQuantRowsPerCta), dim3(kQuantWarps * 32), 0, stream, a);
  return cuda_check(cudaGetLastError(), "launch quant");
}

size_t msv_ragged_gemm_workspace_size(int M, int N) {
  Carver c{nullptr};
  c.take<int4>(tile_cap(M, M, 32, N / 128));
  c.take<int>(2);
  return c.off + 256;
}

int msv_ragged_moe_gemm_fp8(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* w, const float* w_scale,
                            int E, int N, const int32_t* m_indices, void* out, void* workspace, size_t ws_bytes,
                            msv_stream_t stream) {
  if (!a || !a_scale || !w || !w_scale || !m_indices || !out || M < 0 || K <= 0 || N <= 0 || E <= 0 ||
      K % 128 != 0 || N % 128 != 0)
    return fail(MSV_ERR_INVALID, "msv_ragged_moe_gemm_fp8: bad arguments (M=%d K=%d N=%d E=%d)", M, K, N, E);
  if (M == 0) return MSV_OK;
  if (!workspace || ws_bytes < msv_ragged_gemm_workspace_size(M, N) || !is_pow2_aligned(workspace, 256))
    return fail(MSV_ERR_INVALID, "msv_ragged_moe_gemm_fp8: workspace too small or not 256-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const bool small = (M / E) <= 24;
  const int bn = variant_bn(small), nb = N / 128;
  const size_t cap = tile_cap(M, M, 32, nb);
  Carver c{static_cast<uint8_t*>(workspace)};
  int4* tiles = c.take<int4>(cap);
  int* ntiles = c.take<int>(2);  // tile count, claim counter
  launch_k(k_tiles_from_runs, dim3(1), dim3(1024), 0, stream, m_indices, M, bn, nb, tiles, ntiles, (int)cap);
  if (int rc = cuda_check(cudaGetLastError(), "launch tiles_from_runs")) return rc;
  GemmArgs g{};
  if (int rc = tensor_map(&g.tmA[0][0], w, (uint64_t)E * N, K, K, 128)) return rc;
  g.tmA[1][0] = g.tmA[0][0];
  if (int rc = tensor_map(&g.tmB, a, M, K, K, bn)) return rc;
  g.a_expert_rows[0] = g.a_expert_rows[1] = N;
  g.ws[0][0] = g.ws[1][0] = w_scale;
  g.ws[0][1] = g.ws[1][1] = w_scale;
  g.ws_expert_stride[0] = g.ws_expert_stride[1] = (int64_t)(N / 128) * (K / 128);
  g.ws_nb_stride = K / 128;
  g.as = a_scale;
  g.as_row = K / 128;
  g.as_kb = 1;
  g.tiles = tiles;
  g.num_tiles = ntiles;
  g.tile_next = claim_counter(ntiles, K / 128);
  g.num_kb = K / 128;
  g.out = out;
  g.out_ld = N;
  g.err = d->err_word;
  return launch_gemm_variant(small, g, stream, d->num_sms);
}

// The kernels and results are those of msv_ragged_moe_gemm_fp8; only the tile list moves from
// the caller's workspace to g_noalloc_scratch.  Nothing in the scratch has to start at zero:
// k_tiles_from_runs writes the tile count and every tile below it before the GEMM reads them,
// so stale contents from an earlier call are never read.  The capacity check uses M * N/128
// tiles, an upper bound of what k_tiles_from_runs emits (each run of r rows gives at most r
// row chunks per n-block), so the builder never truncates the list.
int msv_ragged_moe_gemm_fp8_noalloc(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* w,
                                    const float* w_scale, int E, int N, const int32_t* m_indices, void* out,
                                    msv_stream_t stream) {
  if (!a || !a_scale || !w || !w_scale || !m_indices || !out || M < 0 || K <= 0 || N <= 0 || E <= 0 ||
      K % 128 != 0 || N % 128 != 0)
    return fail(MSV_ERR_INVALID, "msv_ragged_moe_gemm_fp8_noalloc: bad arguments (M=%d K=%d N=%d E=%d)", M, K, N, E);
  const long long need = (long long)M * (N / 128);
  if (need > (long long)kNoAllocMaxTiles)
    return fail(MSV_ERR_INVALID,
                "msv_ragged_moe_gemm_fp8_noalloc: M * N/128 = %lld tiles exceeds the static scratch limit of %lld "
                "tiles (%zu bytes); use msv_ragged_moe_gemm_fp8 with a workspace",
                need, (long long)kNoAllocMaxTiles, kNoAllocScratchBytes);
  uint8_t* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (M == 0) return MSV_OK;
  const bool small = (M / E) <= 24;
  const int bn = variant_bn(small), nb = N / 128;
  int* ntiles = reinterpret_cast<int*>(scratch);
  int4* tiles = reinterpret_cast<int4*>(scratch + kNoAllocTileOffset);
  launch_k(k_tiles_from_runs, dim3(1), dim3(1024), 0, stream, m_indices, M, bn, nb, tiles, ntiles, (int)need);
  if (int rc = cuda_check(cudaGetLastError(), "launch tiles_from_runs")) return rc;
  GemmArgs g{};
  if (int rc = tensor_map_uncached(&g.tmA[0][0], w, (uint64_t)E * N, K, K, 128)) return rc;
  g.tmA[1][0] = g.tmA[0][0];
  if (int rc = tensor_map_uncached(&g.tmB, a, M, K, K, bn)) return rc;
  g.a_expert_rows[0] = g.a_expert_rows[1] = N;
  g.ws[0][0] = g.ws[1][0] = w_scale;
  g.ws[0][1] = g.ws[1][1] = w_scale;
  g.ws_expert_stride[0] = g.ws_expert_stride[1] = (int64_t)(N / 128) * (K / 128);
  g.ws_nb_stride = K / 128;
  g.as = a_scale;
  g.as_row = K / 128;
  g.as_kb = 1;
  g.tiles = tiles;
  g.num_tiles = ntiles;
  g.tile_next = claim_counter(ntiles, K / 128);
  g.num_kb = K / 128;
  g.out = out;
  g.out_ld = N;
  g.err = d->err_word;
  return launch_gemm_variant(small, g, stream, d->num_sms);
}

size_t msv_gemm_fp8_workspace_size(int M, int N) {
  Carver c{nullptr};
  c.take<int4>(tile_cap(1, M, 32, N / 128));
  c.take<int>(2);
  return c.off + 256;
}

int msv_gemm_fp8_nt_groupwise(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* b,
                              const float* b_scale, int N, void* out, void* workspace, size_t ws_bytes,
                              msv_stream_t stream) {
  if (!a || !a_scale || !b || !b_scale || !out || M < 0 || K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(MSV_ERR_INVALID, "msv_gemm_fp8_nt_groupwise: bad arguments (M=%d K=%d N=%d)", M, K, N);
  if (M == 0) return MSV_OK;
  if (!workspace || ws_bytes < msv_gemm_fp8_workspace_size(M, N) || !is_pow2_aligned(workspace, 256))
    return fail(MSV_ERR_INVALID, "msv_gemm_fp8_nt_groupwise: workspace too small or not 256-byte aligned");
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const bool small = M <= 32;
  const int bn = variant_bn(small), nb = N / 128;
  Carver c{static_cast<uint8_t*>(workspace)};
  int4* tiles = c.take<int4>(tile_cap(1, M, 32, nb));
  int* ntiles = c.take<int>(2);  // tile count, claim counter
  launch_k(k_tiles_dense, dim3(64), dim3(256), 0, stream, M, bn, nb, tiles, ntiles);
  if (int rc = cuda_check(cudaGetLastError(), "launch tiles_dense")) return rc;
  GemmArgs g{};
  if (int rc = tensor_map(&g.tmA[0][0], b, N, K, K, 128)) return rc;
  g.tmA[1][0] = g.tmA[0][0];
  if (int rc = tensor_map(&g.tmB, a, M, K, K, bn)) return rc;
  g.a_expert_rows[0] = g.a_expert_rows[1] = 0;
  g.ws[0][0] = g.ws[1][0] = g.ws[0][1] = g.ws[1][1] = b_scale;
  g.ws_expert_stride[0] = g.ws_expert_stride[1] = 0;
  g.ws_nb_stride = K / 128;
  g.as = a_scale;
  g.as_row = K / 128;
  g.as_kb = 1;
  g.tiles = tiles;
  g.num_tiles = ntiles;
  g.tile_next = claim_counter(ntiles, K / 128);
  g.num_kb = K / 128;
  g.out = out;
  g.out_ld = N;
  g.err = d->err_word;
  return launch_gemm_variant(small, g, stream, d->num_sms);
}

// ── whole layer ──────────────────────────────────────────────────────────────────────────

namespace {
struct LayerPlan {
  int T, H, E, k, I, Is, P, rows, e_local;
  bool shared, small1, small2, rows1, rows2, cg2, pair2;
  int bn1, bn2, nb1, nb2, srows;
  size_t cap1, cap2;
};

int plan_layer(const msv_moe_shape* s, LayerPlan* L) {
  if (!s) return fail(MSV_ERR_INVALID, "msv_moe_forward: null shape");
  L->T = s->tokens;
  L->H = s->hidden;
  L->E = s->num_experts;
  L->k = s->top_k;
  L->I = s->inter;
  L->Is = s->shared_inter;
  if (L->T < 0 || L->H <= 0 || L->H % 128 || L->E <= 0 || L->k < 1 || L->k > 16 || L->k > L->E || L->I <= 0 ||
      L->I % 128 || L->Is < 0 || L->Is % 128)
    return fail(MSV_ERR_INVALID, "msv_moe_forward: bad shape (T=%d H=%d E=%d k=%d I=%d Is=%d)", L->T, L->H, L->E,
                L->k, L->I, L->Is);
  if (s->placement && (s->tp < 1 || s->rank < 0 || s->rank >= s->tp || L->E % s->tp))
    return fail(MSV_ERR_INVALID, "msv_moe_forward: placement 1 needs E %% tp == 0 and 0 <= rank < tp");
  L->shared = L->Is > 0;
  if (L->shared && L->Is != L->I)
    return fail(MSV_ERR_UNSUPPORTED, "msv_moe_forward: shared intermediate (%d) must equal routed (%d)", L->Is, L->I);
  L->e_local = s->placement ? L->E / s->tp : L->E;
  if (L->e_local > 1024) return fail(MSV_ERR_UNSUPPORTED, "msv_moe_forward: more than 1024 local experts");
  L->P = L->T * L->k;
  L->rows = L->P + (L->shared ? L->T : 0);
  const double avg = (double)L->P / (s->placement ? (double)s->tp : 1.0) / (double)L->e_local;
  L->small1 = avg <= 24.0;
  L->small2 = avg <= 24.0;
  // large batches: tokens on the MMA's M side (128-row token chunks).  That kernel loads the
  // tile's K blocks in pairs and its scales as one box, so it needs K/128 a multiple of 4 and
  // at most 32; other large shapes use the weight-rows kernels.
  L->rows1 = !L->small1 && (L->H / 128) % 4 == 0 && L->H / 128 <= R1::MAXKB;
  L->rows2 = !L->small2 && (L->I / 128) % 4 == 0 && L->I / 128 <= R2::MAXKB;
  // the gate_up GEMM of those shapes runs on CTA pairs (256-row chunks); the down GEMM keeps
  // the single-CTA token-rows kernel, which measured faster than a pair form at K = 1024
  L->cg2 = L->rows1 && L->H / 128 <= P1::MAXKB;
  L->bn1 = L->cg2 ? 2 * P1::BM : L->rows1 ? R1::BM : G1Small::BN;
  L->bn2 = L->rows2 ? R2::BM : (L->small2 ? G2Small::BN : G2Large::BN);
  // small-batch down GEMM: two 128-row blocks of H per tile, so each pipeline stage carries as
  // many weight bytes as the gate_up GEMM's (gate + up)
  L->pair2 = !L->rows2 && L->small2 && L->H % 256 == 0;
  L->nb1 = L->I / 128;
  L->nb2 = L->pair2 ? L->H / 256 : L->H / 128;
  L->srows = (L->rows + 3) & ~3;  // K-block stride of the activation scales (16-byte rows)
  L->cap1 = tile_cap(L->e_local, L->P, L->bn1, L->nb1) + (size_t)L->nb1 * ((L->T + L->bn1 - 1) / L->bn1 + 1);
  L->cap2 = tile_cap(L->e_local, L->P, L->bn2, L->nb2) + (size_t)L->nb2 * ((L->T + L->bn2 - 1) / L->bn2 + 1);
  return MSV_OK;
}

struct LayerWs {
  int32_t *ids, *counts, *num_local, *slot_row, *row_token;
  void* w;
  int4 *tiles1, *tiles2;
  int *blk_hist, *blk_nloc, *lrank, *lpos;  // multi-block dispatch scratch
  int *ntiles1, *ntiles2;
  uint8_t *xq, *aq;
  float *xs, *as, *gate_val;
  __nv_bfloat16* down;
};

size_t carve_layer(const LayerPlan& L, uint8_t* base, LayerWs* w) {
  Carver c{base};
  w->ids = c.take<int32_t>(L.P);
  w->w = c.take<float>(L.P);
  w->counts = c.take<int32_t>(L.e_local);
  w->num_local = c.take<int32_t>(1);
  w->slot_row = c.take<int32_t>(L.P);
  w->row_token = c.take<int32_t>(L.P);
  w->tiles1 = c.take<int4>(L.cap1);
  w->ntiles1 = c.take<int>(2);  // tile count, claim counter
  w->tiles2 = c.take<int4>(L.cap2);
  w->ntiles2 = c.take<int>(2);
  w->xq = c.take<uint8_t>((size_t)L.rows * L.H);
  w->xs = c.take<float>((size_t)L.srows * (L.H / 128));
  w->aq = c.take<uint8_t>((size_t)L.rows * L.I);
  w->as = c.take<float>((size_t)L.srows * (L.I / 128));
  w->down = c.take<__nv_bfloat16>((size_t)L.rows * L.H);
  w->gate_val = c.take<float>((size_t)(L.T > 0 ? L.T : 1));
  const int nblk = (L.P + kPermThreads - 1) / kPermThreads;
  w->blk_hist = c.take<int>((size_t)(nblk > 0 ? nblk : 1) * L.e_local);
  w->blk_nloc = c.take<int>((size_t)(nblk > 0 ? nblk : 1));
  w->lrank = c.take<int>((size_t)(L.P > 0 ? L.P : 1));
  w->lpos = c.take<int>((size_t)(L.P > 0 ? L.P : 1));
  return c.off + 256;
}
}  // namespace

size_t msv_moe_forward_workspace_size(const msv_moe_shape* shape) {
  LayerPlan L;
  if (plan_layer(shape, &L) != MSV_OK) return 0;
  LayerWs w;
  return carve_layer(L, nullptr, &w);
}

namespace {
int moe_forward_impl(const msv_moe_shape* s, const msv_moe_weights* W, const void* hidden, const float* logits,
                     void* topk_w, int32_t* topk_ids, void* out, int flags, void* workspace, size_t ws_bytes,
                     cudaStream_t stream, cudaEvent_t* ev, const msv_tp_comm* comm = nullptr) {
  auto mark = [&](int i) -> int {
    return (ev && ev[i]) ? cuda_check(cudaEventRecord(ev[i], stream), "cudaEventRecord") : (int)MSV_OK;
  };
  LayerPlan L;
  if (int rc = plan_layer(s, &L)) return rc;
  if (!W || !hidden || !out) return fail(MSV_ERR_INVALID, "msv_moe_forward: null weights/hidden/out");
  const bool given = flags & MSV_FWD_ROUTING_GIVEN;
  if (given && (!topk_w || !topk_ids)) return fail(MSV_ERR_INVALID, "msv_moe_forward: routing given but null");
  if (!given && !logits) return fail(MSV_ERR_INVALID, "msv_moe_forward: null router logits");
  if (!given && L.E > 1024)
    return fail(MSV_ERR_UNSUPPORTED, "msv_moe_forward: the router takes at most 1024 experts (E=%d)", L.E);
  if (!W->gate_w || !W->up_w || !W->gate_s || !W->up_s || !W->down_w || !W->down_s)
    return fail(MSV_ERR_INVALID, "msv_moe_forward: null routed-expert weight");
  if (L.shared && (!W->sh_gate_w || !W->sh_up_w || !W->sh_down_w || !W->sh_gate_s || !W->sh_up_s || !W->sh_down_s))
    return fail(MSV_ERR_INVALID, "msv_moe_forward: null shared-expert weight");
  if (s->weights_dtype != MSV_BF16 && s->weights_dtype != MSV_F32)
    return fail(MSV_ERR_INVALID, "msv_moe_forward: weights_dtype");
  if (s->combine_mode < 0 || s->combine_mode > 2) return fail(MSV_ERR_INVALID, "msv_moe_forward: combine_mode");
  if (!is_pow2_aligned(hidden, 16) || !is_pow2_aligned(out, 16))
    return fail(MSV_ERR_INVALID, "msv_moe_forward: hidden/out must be 16-byte aligned");
  if (W->sh_gate_logit_w && !is_pow2_aligned(W->sh_gate_logit_w, 16))
    return fail(MSV_ERR_INVALID, "msv_moe_forward: the shared-expert gate weight must be 16-byte aligned");
  if (L.T == 0) return MSV_OK;
  LayerWs w;
  const size_t need = carve_layer(L, nullptr, &w);
  if (!workspace || ws_bytes < need || !is_pow2_aligned(workspace, 256))
    return fail(MSV_ERR_INVALID, "msv_moe_forward: workspace %zu < %zu bytes or not 256-byte aligned", ws_bytes, need);
  carve_layer(L, static_cast<uint8_t*>(workspace), &w);
  DeviceInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;

  // 1. router
  int32_t* ids = topk_ids ? topk_ids : w.ids;
  void* rw = topk_w ? topk_w : w.w;
  if (int rc = mark(0)) return rc;
  if (!given) {
    launch_k(k_route_topk, dim3((L.T + kRouteWarps - 1) / kRouteWarps), dim3(kRouteWarps * 32), route_smem_bytes(L.E), stream, 
        logits, L.E, L.T, L.E, L.k, 1, 1, rw, s->weights_dtype, ids, MSV_I32, nullptr, nullptr);
    if (int rc = cuda_check(cudaGetLastError(), "launch route_topk")) return rc;
  }
  // 2. dispatch bookkeeping + tile lists
  PermuteArgs p{};
  p.ids = ids;
  p.ids_i64 = 0;
  p.T = L.T;
  p.k = L.k;
  p.num_experts = L.E;
  p.placement = s->placement;
  p.tp = s->placement ? s->tp : 1;
  p.rank = s->placement ? s->rank : 0;
  p.alignment = 0;
  p.e_local = L.e_local;
  p.expert_counts = w.counts;
  p.num_local = w.num_local;
  p.row_token = w.row_token;
  p.slot_row = w.slot_row;
  p.tiles1 = w.tiles1;
  p.ntiles1 = w.ntiles1;
  p.bn1 = L.bn1;
  p.nb1 = L.nb1;
  p.tiles2 = w.tiles2;
  p.ntiles2 = w.ntiles2;
  p.bn2 = L.bn2;
  p.nb2 = L.nb2;
  const bool do_shared = L.shared && s->add_shared;  // ranks that do not add it skip its GEMMs
  p.shared_rows = do_shared ? L.T : 0;
  p.row_base_shared = L.P;
  if (int rc = mark(1)) return rc;
  // 3. quantisation: each token once, its e4m3 row and scales written to every sorted row that
  //    reads it (the routed slots the dispatch placed, then the shared expert's row)
  ScatterArgs q{};
  q.x = static_cast<const __nv_bfloat16*>(hidden);
  q.ldx = L.H;
  q.K = L.H;
  q.T = L.T;
  q.k = L.k;
  q.slot_row = w.slot_row;
  q.shared_row0 = do_shared ? L.P : -1;
  q.q = w.xq;
  q.ldq = L.H;
  q.scale = w.xs;
  q.s_kb = L.srows;
  q.gate_w = (do_shared && W->sh_gate_logit_w) ? static_cast<const __nv_bfloat16*>(W->sh_gate_logit_w) : nullptr;
  q.gate_val = w.gate_val;
  if (L.P <= kPermSingleMax) {
    // decode-sized batches: dispatch and quantisation in one launch; every CTA recounts the
    // routing and places its own tokens (at most kDqMaxSlots slots per CTA)
    const size_t dsm = dispatch_quant_smem_bytes(L.P, L.e_local);
    if (int rc = cuda_check(cudaFuncSetAttribute(k_dispatch_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm),
                            "cudaFuncSetAttribute(dispatch_quant)"))
      return rc;
    // CTAs 0 and 1 build the tile lists and take no tokens; the others take at most per_cta
    const int per_cta = kDqMaxSlots / L.k;
    int g = L.T + 2 < d->num_sms ? L.T + 2 : d->num_sms;
    const int need = (L.T + per_cta - 1) / per_cta + 2;
    g = g > need ? g : need;
    launch_k(k_dispatch_quant, dim3(g), dim3(kDqThreads), dsm, stream, p, q);
    if (int rc = cuda_check(cudaGetLastError(), "launch dispatch_quant")) return rc;
    if (int rc = mark(2)) return rc;
  } else {
    // the same stable counting sort over blocks of slots: counts, one scan block (+ tile
    // lists), scatter; then the quantisation
    PermuteScratch ps{w.blk_hist, w.blk_nloc, w.lrank, w.lpos, (L.P + kPermThreads - 1) / kPermThreads};
    const size_t csm = perm_count_smem_bytes(L.e_local);
    if (csm > 48 * 1024)
      if (int rc = cuda_check(cudaFuncSetAttribute(k_perm_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm),
                              "cudaFuncSetAttribute(perm_count)"))
        return rc;
    launch_k(k_perm_count, dim3(ps.nblk), dim3(kPermThreads), csm, stream, p, ps);
    if (int rc = cuda_check(cudaGetLastError(), "launch perm_count")) return rc;
    launch_k(k_perm_scan, dim3(1), dim3(kPermThreads), perm_scan_smem_bytes(L.e_local), stream, p, ps);
    if (int rc = cuda_check(cudaGetLastError(), "launch perm_scan")) return rc;
    launch_k(k_perm_scatter, dim3((L.P + 255) / 256), dim3(256), 0, stream, p, ps);
    if (int rc = cuda_check(cudaGetLastError(), "launch perm_scatter")) return rc;
    if (int rc = mark(2)) return rc;
    launch_k(k_quant_scatter, dim3(L.T), dim3(kScatterThreads), 0, stream, q);
    if (int rc = cuda_check(cudaGetLastError(), "launch quant_scatter")) return rc;
  }
  if (int rc = mark(3)) return rc;
  // 4. gate_up GEMM with SwiGLU + requant epilogue
  const uint64_t gu_rows = (uint64_t)(L.e_local - 1) * W->gu_expert_rows + L.I;
  const int nkb1 = L.H / 128, nkb2 = L.I / 128;
  if (L.cg2) {
    RowsArgs r{};
    if (int rc = tensor_map(&r.tmTok, w.xq, L.rows, L.H, L.H, 64)) return rc;  // 64-row token boxes
    if (int rc = tensor_map(&r.tmW[0][0], W->gate_w, gu_rows, L.H, L.H, 64)) return rc;
    if (int rc = tensor_map(&r.tmW[0][1], W->up_w, gu_rows, L.H, L.H, 64)) return rc;
    const int64_t rpe = W->gu_scale_expert_stride / nkb1;  // scale rows between experts
    const uint64_t gs_rows = (uint64_t)(L.e_local - 1) * rpe + L.I / 128;
    if (int rc = tensor_map_f32(&r.tmWS[0][0], W->gate_s, gs_rows, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    if (int rc = tensor_map_f32(&r.tmWS[0][1], W->up_s, gs_rows, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    if (L.shared) {
      if (int rc = tensor_map(&r.tmW[1][0], W->sh_gate_w, L.Is, L.H, L.H, 64)) return rc;
      if (int rc = tensor_map(&r.tmW[1][1], W->sh_up_w, L.Is, L.H, L.H, 64)) return rc;
      if (int rc = tensor_map_f32(&r.tmWS[1][0], W->sh_gate_s, L.Is / 128, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
      if (int rc = tensor_map_f32(&r.tmWS[1][1], W->sh_up_s, L.Is / 128, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    } else {
      r.tmW[1][0] = r.tmW[0][0];
      r.tmW[1][1] = r.tmW[0][1];
      r.tmWS[1][0] = r.tmWS[0][0];
      r.tmWS[1][1] = r.tmWS[0][1];
    }
    if (int rc = tensor_map_f32(&r.tmAS, w.xs, nkb1, L.srows, (uint64_t)L.srows * 4, P1::SC_LD, nkb1)) return rc;
    r.w_rows[0] = (int)W->gu_expert_rows;
    r.w_rows[1] = 0;
    r.ws_rows[0] = (int)rpe;
    r.ws_rows[1] = 0;
    r.tiles = w.tiles1;
    r.num_tiles = w.ntiles1;
    r.num_kb = nkb1;
    r.out = w.aq;
    r.out_ld = L.I;
    r.out_scale = w.as;
    r.os_row = 1;
    r.os_kb = L.srows;
    r.err = d->err_word;
    if (int rc = launch_gemm_pair<P1>(r, stream, d->num_sms)) return rc;
  } else if (L.rows1) {
    RowsArgs r{};
    if (int rc = tensor_map_kblocks(&r.tmTok, w.xq, L.rows, L.H, L.H, R1::BM, R1::KS)) return rc;
    if (int rc = tensor_map(&r.tmW[0][0], W->gate_w, gu_rows, L.H, L.H, 64)) return rc;
    if (int rc = tensor_map(&r.tmW[0][1], W->up_w, gu_rows, L.H, L.H, 64)) return rc;
    const int64_t rpe = W->gu_scale_expert_stride / nkb1;  // scale rows between experts
    const uint64_t gs_rows = (uint64_t)(L.e_local - 1) * rpe + L.I / 128;
    if (int rc = tensor_map_f32(&r.tmWS[0][0], W->gate_s, gs_rows, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    if (int rc = tensor_map_f32(&r.tmWS[0][1], W->up_s, gs_rows, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    if (L.shared) {
      if (int rc = tensor_map(&r.tmW[1][0], W->sh_gate_w, L.Is, L.H, L.H, 64)) return rc;
      if (int rc = tensor_map(&r.tmW[1][1], W->sh_up_w, L.Is, L.H, L.H, 64)) return rc;
      if (int rc = tensor_map_f32(&r.tmWS[1][0], W->sh_gate_s, L.Is / 128, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
      if (int rc = tensor_map_f32(&r.tmWS[1][1], W->sh_up_s, L.Is / 128, nkb1, (uint64_t)nkb1 * 4, nkb1, 1)) return rc;
    } else {
      r.tmW[1][0] = r.tmW[0][0];
      r.tmW[1][1] = r.tmW[0][1];
      r.tmWS[1][0] = r.tmWS[0][0];
      r.tmWS[1][1] = r.tmWS[0][1];
    }
    if (int rc = tensor_map_f32(&r.tmAS, w.xs, nkb1, L.srows, (uint64_t)L.srows * 4, R1::SC_LD, nkb1)) return rc;
    r.w_rows[0] = (int)W->gu_expert_rows;
    r.w_rows[1] = 0;
    r.ws_rows[0] = (int)rpe;
    r.ws_rows[1] = 0;
    r.tiles = w.tiles1;
    r.num_tiles = w.ntiles1;
    r.num_kb = nkb1;
    r.out = w.aq;
    r.out_ld = L.I;
    r.out_scale = w.as;
    r.os_row = 1;
    r.os_kb = L.srows;
    r.err = d->err_word;
    if (int rc = launch_gemm_rows<R1>(r, stream, d->num_sms)) return rc;
  } else {
    GemmArgs g1{};
    if (int rc = tensor_map(&g1.tmA[0][0], W->gate_w, gu_rows, L.H, L.H, 128)) return rc;
    if (int rc = tensor_map(&g1.tmA[0][1], W->up_w, gu_rows, L.H, L.H, 128)) return rc;
    if (L.shared) {
      if (int rc = tensor_map(&g1.tmA[1][0], W->sh_gate_w, L.Is, L.H, L.H, 128)) return rc;
      if (int rc = tensor_map(&g1.tmA[1][1], W->sh_up_w, L.Is, L.H, L.H, 128)) return rc;
    } else {
      g1.tmA[1][0] = g1.tmA[0][0];
      g1.tmA[1][1] = g1.tmA[0][1];
    }
    if (int rc = tensor_map(&g1.tmB, w.xq, L.rows, L.H, L.H, L.bn1)) return rc;
    g1.a_expert_rows[0] = (int)W->gu_expert_rows;
    g1.a_expert_rows[1] = 0;
    g1.ws[0][0] = W->gate_s;
    g1.ws[0][1] = W->up_s;
    g1.ws[1][0] = L.shared ? W->sh_gate_s : W->gate_s;
    g1.ws[1][1] = L.shared ? W->sh_up_s : W->up_s;
    g1.ws_expert_stride[0] = W->gu_scale_expert_stride;
    g1.ws_expert_stride[1] = 0;
    g1.ws_nb_stride = nkb1;
    g1.as = w.xs;
    g1.as_row = 1;
    g1.as_kb = L.srows;
    g1.tiles = w.tiles1;
    g1.num_tiles = w.ntiles1;
    g1.tile_next = claim_counter(w.ntiles1, nkb1);
    g1.num_kb = nkb1;
    g1.out = w.aq;
    g1.out_ld = L.I;
    g1.out_scale = w.as;
    g1.os_row = 1;
    g1.os_kb = L.srows;
    g1.err = d->err_word;
    if (int rc = launch_gemm<G1Small>(g1, stream, d->num_sms)) return rc;
  }
  if (int rc = mark(4)) return rc;
  // 5. down GEMM
  if (L.rows2) {
    RowsArgs r{};
    if (int rc = tensor_map_kblocks(&r.tmTok, w.aq, L.rows, L.I, L.I, R2::BM, R2::KS)) return rc;
    if (int rc = tensor_map_kblocks(&r.tmW[0][0], W->down_w, (uint64_t)L.e_local * L.H, L.I, L.I, 128, R2::KS)) return rc;
    if (int rc = tensor_map_f32(&r.tmWS[0][0], W->down_s, (uint64_t)L.e_local * (L.H / 128), nkb2, (uint64_t)nkb2 * 4,
                                nkb2, 1))
      return rc;
    if (L.shared) {
      if (int rc = tensor_map_kblocks(&r.tmW[1][0], W->sh_down_w, L.H, L.Is, L.Is, 128, R2::KS)) return rc;
      if (int rc = tensor_map_f32(&r.tmWS[1][0], W->sh_down_s, L.H / 128, nkb2, (uint64_t)nkb2 * 4, nkb2, 1)) return rc;
    } else {
      r.tmW[1][0] = r.tmW[0][0];
      r.tmWS[1][0] = r.tmWS[0][0];
    }
    r.tmW[0][1] = r.tmW[0][0];
    r.tmW[1][1] = r.tmW[1][0];
    r.tmWS[0][1] = r.tmWS[0][0];
    r.tmWS[1][1] = r.tmWS[1][0];
    if (int rc = tensor_map_f32(&r.tmAS, w.as, nkb2, L.srows, (uint64_t)L.srows * 4, R2::SC_LD, nkb2)) return rc;
    r.w_rows[0] = L.H;
    r.w_rows[1] = 0;
    r.ws_rows[0] = L.H / 128;
    r.ws_rows[1] = 0;
    r.tiles = w.tiles2;
    r.num_tiles = w.ntiles2;
    r.num_kb = nkb2;
    r.out = w.down;
    r.out_ld = L.H;
    r.err = d->err_word;
    if (int rc = launch_gemm_rows<R2>(r, stream, d->num_sms)) return rc;
  } else {
    GemmArgs g2{};
    if (int rc = tensor_map(&g2.tmA[0][0], W->down_w, (uint64_t)L.e_local * L.H, L.I, L.I, 128)) return rc;
    if (L.shared) {
      if (int rc = tensor_map(&g2.tmA[1][0], W->sh_down_w, L.H, L.Is, L.Is, 128)) return rc;
    } else {
      g2.tmA[1][0] = g2.tmA[0][0];
    }
    g2.tmA[0][1] = g2.tmA[0][0];
    g2.tmA[1][1] = g2.tmA[1][0];
    if (int rc = tensor_map(&g2.tmB, w.aq, L.rows, L.I, L.I, L.bn2)) return rc;
    g2.a_expert_rows[0] = L.H;
    g2.a_expert_rows[1] = 0;
    g2.ws[0][0] = g2.ws[0][1] = W->down_s;
    g2.ws[1][0] = g2.ws[1][1] = L.shared ? W->sh_down_s : W->down_s;
    g2.ws_expert_stride[0] = (int64_t)(L.H / 128) * nkb2;
    g2.ws_expert_stride[1] = 0;
    g2.ws_nb_stride = nkb2;
    g2.as = w.as;
    g2.as_row = 1;
    g2.as_kb = L.srows;
    g2.tiles = w.tiles2;
    g2.num_tiles = w.ntiles2;
    g2.tile_next = claim_counter(w.ntiles2, nkb2);
    g2.num_kb = nkb2;
    g2.out = w.down;
    g2.out_ld = L.H;
    g2.err = d->err_word;
    if (L.pair2) {
      if (int rc = launch_gemm<G2Pair>(g2, stream, d->num_sms)) return rc;
    } else {
      if (int rc = launch_gemm_variant(L.small2, g2, stream, d->num_sms)) return rc;
    }
  }
  if (int rc = mark(5)) return rc;
  // 6. weighted combine (+ shared expert)
  CombineArgs cb{};
  cb.down = w.down;
  cb.ld_down = L.H;
  cb.slot_row = w.slot_row;
  cb.topk_ids = ids;
  cb.topk_w = rw;
  cb.w_f32 = s->weights_dtype == MSV_F32;
  cb.T = L.T;
  cb.H = L.H;
  cb.k = L.k;
  cb.mode = s->combine_mode;
  cb.add_shared = do_shared;
  cb.shared_row0 = L.P;
  cb.gate_val = (do_shared && W->sh_gate_logit_w) ? w.gate_val : nullptr;
  cb.out = static_cast<__nv_bfloat16*>(out);
  cb.ld_out = L.H;
  if (comm) {
    // combine fused with the sum over the TP group (peer memory; a group of one exchanges
    // flags with itself)
    CombineArArgs ar{};
    ar.c = cb;
    const size_t rb = tp_area_bytes(comm->max_tokens, comm->hidden);
    for (int p = 0; p < comm->world; ++p) {
      uint8_t* base = static_cast<uint8_t*>(comm->shared[p]);
      ar.recv[p] = reinterpret_cast<uint64_t*>(base);
      ar.res[p] = reinterpret_cast<uint64_t*>(base + rb);
    }
    ar.epoch = comm->epoch;
    ar.world = comm->world;
    ar.rank = comm->rank;
    ar.max_tokens = comm->max_tokens;
    ar.err = d->err_word;
    // The grid is at most what the SMs hold at once, so every CTA is resident and none waits
    // for one that cannot be scheduled.  The cap must be the same for every call on a group
    // (token t is always handled by CTA t mod cap, whose epoch flags its slots): it is the
    // smallest occupancy of the three combine-mode instances at this H, which depends only on
    // the device and the group's hidden size, never on the call's mode or token count.
    const int threads = combine_threads(L.H);
    void (*kern)(CombineArArgs) = cb.mode == MSV_COMBINE_V2          ? k_combine_ar<MSV_COMBINE_V2>
                                  : cb.mode == MSV_COMBINE_DISPATCH ? k_combine_ar<MSV_COMBINE_DISPATCH>
                                                                    : k_combine_ar<MSV_COMBINE_BATCHED>;
    int cap = 0;
    if (int rc = combine_ar_grid_cap(threads, d->num_sms, &cap)) return rc;
    const int g = L.T < cap ? L.T : cap;
    launch_k(kern, dim3(g), dim3(threads), 0, stream, ar);
    if (int rc = cuda_check(cudaGetLastError(), "launch combine_ar")) return rc;
    return mark(6);
  }
  launch_combine(cb, stream, d->num_sms);
  if (int rc = cuda_check(cudaGetLastError(), "launch combine")) return rc;
  return mark(6);
}

int check_tp_comm(const msv_tp_comm* c, const msv_moe_shape* s) {
  if (!c) return fail(MSV_ERR_INVALID, "msv_moe_forward_tp: null comm");
  if (c->world < 1 || c->world > MSV_MAX_TP || c->rank < 0 || c->rank >= c->world || !c->epoch)
    return fail(MSV_ERR_INVALID, "msv_moe_forward_tp: bad group (world=%d rank=%d)", c->world, c->rank);
  if (!s || s->tokens > c->max_tokens || s->hidden != c->hidden || s->hidden % (8 * c->world))
    return fail(MSV_ERR_INVALID,
                "msv_moe_forward_tp: T=%d must be <= max_tokens=%d, H=%d == hidden=%d and a multiple of 8*world",
                s ? s->tokens : -1, c->max_tokens, s ? s->hidden : -1, c->hidden);
  for (int p = 0; p < c->world; ++p)
    if (!c->shared[p] || !is_pow2_aligned(c->shared[p], 256))
      return fail(MSV_ERR_INVALID, "msv_moe_forward_tp: shared[%d] null or not 256-byte aligned", p);
  if (!is_pow2_aligned(c->epoch, 16)) return fail(MSV_ERR_INVALID, "msv_moe_forward_tp: epoch not 16-byte aligned");
  return MSV_OK;
}
}  // namespace

int msv_moe_forward(const msv_moe_shape* s, const msv_moe_weights* W, const void* hidden, const float* logits,
                    void* topk_w, int32_t* topk_ids, void* out, int flags, void* workspace, size_t ws_bytes,
                    msv_stream_t stream) {
  return moe_forward_impl(s, W, hidden, logits, topk_w, topk_ids, out, flags, workspace, ws_bytes, stream, nullptr);
}

int msv_moe_forward_profiled(const msv_moe_shape* s, const msv_moe_weights* W, const void* hidden,
                             const float* logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                             void* workspace, size_t ws_bytes, msv_stream_t stream, void* const* events) {
  if (!events) return fail(MSV_ERR_INVALID, "msv_moe_forward_profiled: null events");
  cudaEvent_t ev[7];
  for (int i = 0; i < 7; ++i) ev[i] = static_cast<cudaEvent_t>(events[i]);
  return moe_forward_impl(s, W, hidden, logits, topk_w, topk_ids, out, flags, workspace, ws_bytes, stream, ev);
}

size_t msv_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int msv_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return fail(MSV_ERR_INVALID, "msv_ipc_export: null argument");
  AddressRangeFn fn = address_range_fn();
  if (!fn) return fail(MSV_ERR_CUDA, "cuMemGetAddressRange unavailable from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MSV_ERR_INVALID, "msv_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  if (int rc = cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle")) return rc;
  std::memcpy(handle_out, &h, sizeof h);
  *offset_out = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return MSV_OK;
}

int msv_ipc_import(const void* handle, uint64_t offset, void** ptr_out) {
  if (!handle || !ptr_out) return fail(MSV_ERR_INVALID, "msv_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  if (int rc = cuda_check(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
    return rc;
  void* p = static_cast<uint8_t*>(base) + offset;
  {
    std::lock_guard<std::mutex> g(g_ipc_mu);
    g_ipc_bases[reinterpret_cast<uintptr_t>(p)] = base;
  }
  *ptr_out = p;
  return MSV_OK;
}

int msv_ipc_close(void* ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> g(g_ipc_mu);
    auto it = g_ipc_bases.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == g_ipc_bases.end()) return fail(MSV_ERR_INVALID, "msv_ipc_close: not a pointer msv_ipc_import returned");
    base = it->second;
    g_ipc_bases.erase(it);
  }
  return cuda_check(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

size_t msv_tp_shared_bytes(int max_tokens, int hidden) {
  if (max_tokens <= 0 || hidden <= 0) return 0;
  return 2 * tp_area_bytes(max_tokens, hidden);
}

size_t msv_tp_epoch_bytes(void) { return (size_t)kArMaxCtas * sizeof(unsigned int); }

int msv_moe_forward_tp(const msv_moe_shape* s, const msv_moe_weights* W, const void* hidden, const float* logits,
                       void* topk_w, int32_t* topk_ids, void* out, int flags, void* workspace, size_t ws_bytes,
                       const msv_tp_comm* comm, msv_stream_t stream) {
  if (int rc = check_tp_comm(comm, s)) return rc;
  return moe_forward_impl(s, W, hidden, logits, topk_w, topk_ids, out, flags, workspace, ws_bytes, stream, nullptr,
                          comm);
}

int msv_moe_forward_tp_profiled(const msv_moe_shape* s, const msv_moe_weights* W, const void* hidden,
                                const float* logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                                void* workspace, size_t ws_bytes, const msv_tp_comm* comm, msv_stream_t stream,
                                void* const* events) {
  if (!events) return fail(MSV_ERR_INVALID, "msv_moe_forward_tp_profiled: null events");
  if (int rc = check_tp_comm(comm, s)) return rc;
  cudaEvent_t ev[7];
  for (int i = 0; i < 7; ++i) ev[i] = static_cast<cudaEvent_t>(events[i]);
  return moe_forward_impl(s, W, hidden, logits, topk_w, topk_ids, out, flags, workspace, ws_bytes, stream, ev, comm);
}

}  // extern "C"
