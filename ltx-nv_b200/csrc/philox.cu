// Initial-noise generation: torch-compatible Philox4x32-10 normal fill.
//
// Stream definition (reference: cuda_c_standalone/common/philox.cu:19-35, the
// re-statement of torch's distribution_elementwise_grid_stride_kernel): thread
// idx < threads = 256*grid owns Philox subsequence idx starting at `offset`; each round
// yields four normals that land at out[base + ii*threads + idx], ii = 0..3, with base
// advancing by 4*threads per round. The per-thread normals come from the CUDA toolkit's
// curand device API (curand_init / curand_normal4), the same calls torch makes, so the
// values are bit-identical to torch.randn for the same seed, offset and grid.
//
// B200 launch design: each block stages its 4x256 normals in shared memory and writes
// them back as 4 contiguous 1 KiB segments with 16-byte (fp32) / 8-byte (bf16) stores,
// instead of 4 strided scalar stores per thread.
#include <curand_kernel.h>
#include "ltx_common.cuh"
#include "ltx_internal.h"

namespace ltx {
namespace detail {

template <typename T>
__global__ void __launch_bounds__(256) philox_randn_kernel(T* __restrict__ out, int64_t n, uint64_t seed,
                                                           uint64_t offset) {
  const int tid = threadIdx.x;
  const int64_t threads = int64_t(gridDim.x) * 256;
  const int64_t idx = int64_t(blockIdx.x) * 256 + tid;
  curandStatePhilox4_32_10_t st;
  curand_init(seed, idx, offset, &st);
  const int64_t step = threads * 4;
  const int64_t rounded = ((n - 1) / step + 1) * step;
  __shared__ float buf[4][256 + 4];
  // Store phase: thread tid writes elements j..j+3 of segment ii.
  const int ii = tid >> 6;
  const int j = (tid & 63) * 4;
  for (int64_t base = 0; base < rounded; base += step) {
    float4 r = curand_normal4(&st);
    buf[0][tid] = r.x;
    buf[1][tid] = r.y;
    buf[2][tid] = r.z;
    buf[3][tid] = r.w;
    __syncthreads();
    const int64_t o = base + ii * threads + int64_t(blockIdx.x) * 256 + j;
    const float v0 = buf[ii][j], v1 = buf[ii][j + 1], v2 = buf[ii][j + 2], v3 = buf[ii][j + 3];
    if (o + 3 < n) {
      if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(out + o) = make_float4(v0, v1, v2, v3);
      } else {
        uint2 u;
        u.x = pack_bf16x2(v0, v1);
        u.y = pack_bf16x2(v2, v3);
        *reinterpret_cast<uint2*>(out + o) = u;
      }
    } else {
      const float vv[4] = {v0, v1, v2, v3};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (o + e < n) st_elem<T>(out + o + e, vv[e]);
    }
    __syncthreads();
  }
}

__global__ void philox_raw_kernel(uint32_t* __restrict__ out, int64_t threads, int64_t rounds, uint64_t seed,
                                  uint64_t offset) {
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= threads) return;
  curandStatePhilox4_32_10_t st;
  curand_init(seed, t, offset, &st);
  for (int64_t r = 0; r < rounds; ++r) {
    uint4 v = curand4(&st);
    uint32_t* o = out + (r * threads + t) * 4;
    o[0] = v.x;
    o[1] = v.y;
    o[2] = v.z;
    o[3] = v.w;
  }
}

}  // namespace detail
}  // namespace ltx

using namespace ltx::detail;

extern "C" int ltx_philox_grid(int device, int64_t n, int* grid) {
  LTX_API_BEGIN
  LTX_REQUIRE(grid != nullptr, "grid is NULL");
  LTX_REQUIRE(n > 0, "n must be positive");
  cudaDeviceProp prop;
  LTX_CUDA(cudaGetDeviceProperties(&prop, device));
  const int64_t cap = int64_t(prop.multiProcessorCount) * (prop.maxThreadsPerMultiProcessor / 256);
  int64_t g = (n + 255) / 256;
  if (g > cap) g = cap;
  *grid = int(g);
  LTX_API_END
}

extern "C" int64_t ltx_philox_offset_increment(int64_t n, int grid) {
  if (n <= 0 || grid <= 0) return 0;
  return ((n - 1) / (int64_t(256) * grid * 4) + 1) * 4;
}

extern "C" int ltx_philox_randn(void* out, int64_t n, int dtype, uint64_t seed, uint64_t offset, int grid,
                                void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(out != nullptr, "out is NULL");
  LTX_REQUIRE(n > 0, "n must be positive");
  LTX_REQUIRE(grid > 0 && grid <= (1 << 24), "grid out of range");
  LTX_REQUIRE(dtype == LTX_F32 || dtype == LTX_BF16, "dtype must be F32 or BF16");
  LTX_REQUIRE(reinterpret_cast<uintptr_t>(out) % 16 == 0, "out must be 16-byte aligned");
  LTX_REQUIRE(offset % 4 == 0, "offset must be a multiple of 4 (torch advances it in 4s)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_F32)
    philox_randn_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(out), n, seed, offset), ltx::note_launch();
  else
    philox_randn_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out), n, seed, offset), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_philox_raw(uint32_t* out, int64_t threads, int64_t rounds, uint64_t seed, uint64_t offset,
                              void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(out != nullptr, "out is NULL");
  LTX_REQUIRE(threads > 0 && rounds > 0, "threads and rounds must be positive");
  LTX_REQUIRE(threads <= (int64_t(1) << 30), "threads out of range");
  const int64_t blocks = (threads + 255) / 256;
  philox_raw_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, threads, rounds, seed,
                                                                                     offset), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
