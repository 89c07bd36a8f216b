// Host-side plumbing shared by the C-ABI entry points: status codes, the thread-local
// error message, argument checks and TMA descriptor encoding.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <string>

#include "../../include/ltxb200.h"

namespace ltx {

void set_error(const std::string& msg);
void clear_error();

struct ApiError {
  int code;
  std::string msg;
};

// Encode a 2-D, 128-byte-swizzled bf16 tensor map over a row-major matrix.
// inner = elements per row (contiguous), outer = rows, ld = elements between rows,
// box = (box_inner x box_outer) elements; box_inner * 2 must be <= 128.
// Throws ApiError on invalid input.
// Encode a 4-D, 128-byte-swizzled bf16 tensor map: dims[0] contiguous, strides in bytes
// for dims 1..3, box[0] * 2 <= 128 bytes. Throws ApiError on invalid input.
CUtensorMap make_tmap_bf16_4d(const void* ptr, const uint64_t (&dims)[4], const uint64_t (&strides)[3],
                              const uint32_t (&box)[4]);
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                              uint32_t box_outer);

// Cache of encoded tensor maps, keyed by everything a 2-D map encodes (address,
// extents, row stride, box), so a hit is always the descriptor a fresh encoding would
// give. While a TmapScope is alive on a thread, make_tmap_bf16_2d consults the scope's
// cache before encoding (the ltx_ctx of the whole-step entry point owns one).
struct TmapCache;
TmapCache* tmap_cache_new();
void tmap_cache_delete(TmapCache* c);
class TmapScope {
 public:
  explicit TmapScope(TmapCache* c);
  ~TmapScope();
  TmapScope(const TmapScope&) = delete;
  TmapScope& operator=(const TmapScope&) = delete;

 private:
  TmapCache* prev_;
};

// Number of SMs of the current device (cached per device).
int num_sms();

// Process-wide count of kernels this library has launched (ltx_launch_count).
void note_launch();

// Raises the dynamic shared-memory limit of `kern` to `bytes` on the current device the
// first time a call site launches it there. `done` is the call site's static bitmask of
// devices already configured (thread-safe; devices >= 64 are configured on every call).
void ensure_smem_limit(std::atomic<uint64_t>& done, const void* kern, int bytes);
template <class K>
inline void ensure_smem_limit(std::atomic<uint64_t>& done, K* kern, int bytes) {
  ensure_smem_limit(done, reinterpret_cast<const void*>(kern), bytes);
}

}  // namespace ltx

#define LTX_API_BEGIN \
  try {               \
    ltx::clear_error();
#define LTX_API_END                                              \
  return LTX_OK;                                                 \
  }                                                              \
  catch (const ltx::ApiError& e) {                               \
    ltx::set_error(e.msg);                                       \
    return e.code;                                               \
  }                                                              \
  catch (...) {                                                  \
    ltx::set_error("unexpected C++ exception");                  \
    return LTX_ERR_INVALID;                                      \
  }

#define LTX_REQUIRE(cond, msg)                                                   \
  do {                                                                           \
    if (!(cond)) throw ltx::ApiError{LTX_ERR_INVALID, std::string(__func__) + ": " + (msg)}; \
  } while (0)

#define LTX_UNSUPPORTED(cond, msg)                                                   \
  do {                                                                               \
    if (!(cond)) throw ltx::ApiError{LTX_ERR_UNSUPPORTED, std::string(__func__) + ": " + (msg)}; \
  } while (0)

#define LTX_CUDA(call)                                                                                  \
  do {                                                                                                  \
    cudaError_t err_ = (call);                                                                          \
    if (err_ != cudaSuccess)                                                                            \
      throw ltx::ApiError{LTX_ERR_CUDA, std::string(__func__) + ": " #call ": " + cudaGetErrorString(err_)}; \
  } while (0)
