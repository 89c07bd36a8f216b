// Library-wide C-ABI plumbing: error reporting, the device error word and TMA
// descriptor encoding (through the driver entry point, so the library links only the
// CUDA runtime).
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "ltx_common.cuh"
#include "ltx_internal.h"

namespace ltx {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }
void clear_error() { t_last_error.clear(); }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct TmapKey {
  const void* ptr;
  uint64_t inner, outer, ld;
  uint32_t box_inner, box_outer;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && ld == o.ld && box_inner == o.box_inner &&
           box_outer == o.box_outer;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.ptr);
    for (uint64_t v : {k.inner, k.outer, k.ld, uint64_t(k.box_inner) << 32 | k.box_outer})
      h = (h ^ v) * 0x100000001b3ull + (h >> 29);
    return size_t(h);
  }
};
struct TmapCache {
  std::mutex mu;
  std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> maps;
};
static thread_local TmapCache* t_tmap_cache = nullptr;

TmapCache* tmap_cache_new() { return new TmapCache(); }
void tmap_cache_delete(TmapCache* c) { delete c; }
TmapScope::TmapScope(TmapCache* c) : prev_(t_tmap_cache) { t_tmap_cache = c; }
TmapScope::~TmapScope() { t_tmap_cache = prev_; }

static CUtensorMap encode_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                                       uint32_t box_inner, uint32_t box_outer);

CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                              uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    throw ApiError{LTX_ERR_INVALID, "TMA operand must be 16-byte aligned"};
  if ((ld * 2) % 16 != 0) throw ApiError{LTX_ERR_INVALID, "TMA row stride must be a multiple of 16 bytes"};
  if (box_inner * 2 > 128 || box_outer > 256 || box_inner == 0 || box_outer == 0)
    throw ApiError{LTX_ERR_INVALID, "TMA box out of range"};
  TmapCache* cache = t_tmap_cache;
  if (cache == nullptr) return encode_tmap_bf16_2d(ptr, inner, outer, ld, box_inner, box_outer);
  const TmapKey key{ptr, inner, outer, ld, box_inner, box_outer};
  {
    std::lock_guard<std::mutex> lock(cache->mu);
    auto it = cache->maps.find(key);
    if (it != cache->maps.end()) return it->second;
  }
  const CUtensorMap m = encode_tmap_bf16_2d(ptr, inner, outer, ld, box_inner, box_outer);
  std::lock_guard<std::mutex> lock(cache->mu);
  if (cache->maps.size() >= 8192) cache->maps.clear();
  cache->maps.emplace(key, m);
  return m;
}

static CUtensorMap encode_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                                       uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) throw ApiError{LTX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable"};
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw ApiError{LTX_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r))};
  return m;
}

CUtensorMap make_tmap_bf16_4d(const void* ptr, const uint64_t (&dims)[4], const uint64_t (&strides)[3],
                              const uint32_t (&box)[4]) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    throw ApiError{LTX_ERR_INVALID, "TMA operand must be 16-byte aligned"};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0) throw ApiError{LTX_ERR_INVALID, "TMA strides must be multiples of 16 bytes"};
  if (box[0] * 2 > 128 || box[0] == 0)
    throw ApiError{LTX_ERR_INVALID, "TMA box out of range"};
  for (int i = 1; i < 4; ++i)
    if (box[i] == 0 || box[i] > 256) throw ApiError{LTX_ERR_INVALID, "TMA box out of range"};
  auto fn = encode_fn();
  if (fn == nullptr) throw ApiError{LTX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable"};
  CUtensorMap m;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), d, st, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw ApiError{LTX_ERR_CUDA, "cuTensorMapEncodeTiled (4-D) failed with code " + std::to_string(int(r))};
  return m;
}

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int num_sms() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

void ensure_smem_limit(std::atomic<uint64_t>& done, const void* kern, int bytes) {
  int dev = 0;
  LTX_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return;
  LTX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (bit != 0) done.fetch_or(bit, std::memory_order_release);
}

}  // namespace ltx

extern "C" const char* ltx_last_error(void) { return ltx::t_last_error.c_str(); }

extern "C" int ltx_abi_version(void) { return 1; }

extern "C" uint64_t ltx_launch_count(void) { return ltx::g_launches.load(std::memory_order_relaxed); }

extern "C" int ltx_device_error_flags(int* flags, int clear, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(flags != nullptr, "flags is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int value = 0;
  LTX_CUDA(cudaMemcpyFromSymbolAsync(&value, g_ltx_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  LTX_CUDA(cudaStreamSynchronize(s));
  *flags = value;
  if (clear) {
    const int zero = 0;
    LTX_CUDA(cudaMemcpyToSymbolAsync(g_ltx_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    LTX_CUDA(cudaStreamSynchronize(s));
  }
  LTX_API_END
}

// ---------------------------------------------------------------------------------
// Test hook (include/ltxb200_testing.h): one thread waits on an mbarrier that nothing
// ever arrives on, through the same bounded wait the tcgen05 kernels use, with a short
// limit; it must give up, set the device error word and return.
// ---------------------------------------------------------------------------------
namespace ltx {
namespace detail {
__global__ void bounded_wait_probe_kernel(unsigned long long limit_cycles, int* returned) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait_limit(&bar, 0, &abort_flag, limit_cycles, 1000u);
    *returned = ok ? 2 : 1;
  }
}
}  // namespace detail
}  // namespace ltx

extern "C" int ltx_test_bounded_wait(unsigned long long limit_cycles, int* returned, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(returned != nullptr, "returned is NULL");
  LTX_REQUIRE(limit_cycles > 0 && limit_cycles <= 100000000ull, "limit must be in (0, 1e8] cycles");
  ltx::detail::bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_cycles, returned),
      ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
