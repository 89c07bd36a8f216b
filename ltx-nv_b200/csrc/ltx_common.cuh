// Shared device helpers for the sm_100a kernels: bf16 conversion, bounded mbarrier
// waits, TMA (cp.async.bulk.tensor) and tcgen05 (TMEM / UMMA) wrappers in inline PTX.
//
// Every spin-wait is bounded: after LTX_WAIT_LIMIT_CYCLES of SM clock it records an
// error code in g_ltx_device_error (read by ltx_device_error_flags on the host) and
// returns false so the caller can unwind instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#define LTX_DEVICE __device__ __forceinline__

// ~4 s at the B200 boost clock: far above any legitimate wait inside one launch.
#define LTX_WAIT_LIMIT_CYCLES (8000000000ull)

// Device-side error word (bit flags, sticky until the host clears it).
enum : int {
  LTX_DEVERR_MBAR_TIMEOUT = 1,
  LTX_DEVERR_BAD_SHAPE = 2,
};
// Defined here: the library is built as one translation unit (csrc/ltxb200.cu).
__device__ int g_ltx_device_error = 0;

LTX_DEVICE void ltx_flag_error(int bit) { atomicOr(&g_ltx_device_error, bit); }

// ---------------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------------
LTX_DEVICE float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
LTX_DEVICE __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }
// Round an fp32 value to the nearest bf16 and widen it again (models a torch .to(bf16)).
LTX_DEVICE float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Round two fp32 values to bf16 and widen them again with one packed conversion.
LTX_DEVICE void round_bf16_pair(float& a, float& b) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  a = __low2float(p);
  b = __high2float(p);
}
LTX_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}
LTX_DEVICE void unpack_bf16x2(uint32_t w, float& lo, float& hi) {
  __nv_bfloat162 p = *reinterpret_cast<__nv_bfloat162*>(&w);
  lo = __low2float(p);
  hi = __high2float(p);
}

// Generic element load/store for the dtype-templated kernels (float or bf16 storage,
// fp32 arithmetic).
template <typename T> LTX_DEVICE float ld_elem(const T* p);
template <> LTX_DEVICE float ld_elem<float>(const float* p) { return *p; }
template <> LTX_DEVICE float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T> LTX_DEVICE void st_elem(T* p, float v);
template <> LTX_DEVICE void st_elem<float>(float* p, float v) { *p = v; }
template <> LTX_DEVICE void st_elem<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
// Round to the storage type's precision (identity for fp32).
template <typename T> LTX_DEVICE float round_to(float v);
template <> LTX_DEVICE float round_to<float>(float v) { return v; }
template <> LTX_DEVICE float round_to<__nv_bfloat16>(float v) { return round_bf16(v); }

// Load / store 8 consecutive elements (16 bytes of bf16, 32 bytes of fp32).
template <typename T> LTX_DEVICE void ld8(const T* p, float (&v)[8]);
template <> LTX_DEVICE void ld8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  unpack_bf16x2(u.x, v[0], v[1]);
  unpack_bf16x2(u.y, v[2], v[3]);
  unpack_bf16x2(u.z, v[4], v[5]);
  unpack_bf16x2(u.w, v[6], v[7]);
}
template <> LTX_DEVICE void ld8<float>(const float* p, float (&v)[8]) {
  float4 a = reinterpret_cast<const float4*>(p)[0];
  float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T> LTX_DEVICE void st8(T* p, const float (&v)[8]);
template <> LTX_DEVICE void st8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <> LTX_DEVICE void st8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Warp / block reductions.
LTX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
LTX_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over the whole block; `red` must hold >= 32 floats. All threads get the result.
LTX_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : 0.f;
  return warp_sum(t);
}

// ---------------------------------------------------------------------------------
// Shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------------
LTX_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

LTX_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
LTX_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
LTX_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
LTX_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
LTX_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same with a suspend-time hint (ns): the thread sleeps until the phase completes
// or the hint expires instead of polling, leaving the issue slots of its SM
// sub-partition to the warps that do the work.
LTX_DEVICE bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Non-blocking probe (test_wait returns at once; try_wait may suspend the thread for
// a while before reporting "not yet", which stalls a warp that polls several barriers).
LTX_DEVICE bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete. Returns false (and flags the
// device error word) if the wait exceeds the cycle budget; `abort` is a shared flag
// that lets the other roles of the CTA give up promptly once one of them timed out.
LTX_DEVICE bool mbar_wait_limit(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned long long limit,
                                uint32_t sleep_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, sleep_ns)) return true;
    if (abort != nullptr && *abort) return false;
    if (clock64() - t0 > limit) {
      ltx_flag_error(LTX_DEVERR_MBAR_TIMEOUT);
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}
LTX_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  return mbar_wait_limit(bar, parity, abort, LTX_WAIT_LIMIT_CYCLES, 100000u);
}

// ---------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------------
LTX_DEVICE void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
LTX_DEVICE void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 4-D tiled load (box x fastest); coordinates other than x may be negative or past the
// end (zero fill); x times the element size must be a multiple of 16 bytes.
LTX_DEVICE void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM loads / stores
// ---------------------------------------------------------------------------------
// ---------------------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2). No TMA multicast: each CTA loads its
// own operand halves and signals the even ("leader") CTA's barrier.
// ---------------------------------------------------------------------------------
LTX_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs (call from converged warps).
LTX_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
LTX_DEVICE uint32_t mapa_shared(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier given by its shared::cluster address (possibly in the peer CTA).
LTX_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2D tiled TMA load into this CTA's shared memory whose completion bytes are counted on
// the barrier at `bar_cluster_addr` (the leader CTA's barrier for a CTA pair).
LTX_DEVICE void tma_load_2d_pair(void* dst, const void* tmap, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
// TMEM allocation shared by a CTA pair: issued by the same warp of both CTAs.
LTX_DEVICE void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
LTX_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
LTX_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LTX_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
LTX_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
LTX_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LTX_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LTX_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate).
LTX_DEVICE void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same with the A operand read from TMEM (used for P*V in attention).
LTX_DEVICE void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Pair MMA (M = 256 over the two CTAs' shared memory and TMEM), issued by the leader.
LTX_DEVICE void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at the same offset in every CTA of `cta_mask` once all earlier
// pair MMAs of this thread complete.
LTX_DEVICE void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
LTX_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both operands K-major
// unless b_mn_major is set (B stored with N contiguous).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int b_mn_major) {
  return (1u << 4)                          // D format: f32
         | (1u << 7)                        // A format: bf16
         | (1u << 10)                       // B format: bf16
         | (uint32_t(b_mn_major & 1) << 16)  // B major-ness
         | (uint32_t(N >> 3) << 17)         // N / 8
         | (uint32_t(M >> 4) << 24);        // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B). `lbo`/`sbo` are byte offsets.
LTX_DEVICE uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr & 0x3FFFF) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  d |= uint64_t(2) << 61;  // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 columns of 32-bit TMEM words -> 32 registers per thread.
LTX_DEVICE void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 columns.
LTX_DEVICE void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 16 columns store (registers -> TMEM).
LTX_DEVICE void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 32 lanes x 32 columns store.
LTX_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
LTX_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Programmatic dependent launch (see launch_pdl): wait until the kernels ahead of this
// one in the stream have completed and their memory is visible; then let the next
// kernel of the stream be scheduled.
LTX_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LTX_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Barrier `id` (1..15; 0 is __syncthreads) over the first `threads` threads' warps.
LTX_DEVICE void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 2^x on the special-function unit (approximate, flushes subnormals; exact 0 for -inf).
LTX_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic (two lanes per instruction on sm_100).
LTX_DEVICE uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
LTX_DEVICE void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
LTX_DEVICE uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
LTX_DEVICE uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
LTX_DEVICE uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
LTX_DEVICE uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// max of three fp32 values in one instruction.
LTX_DEVICE float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the FMA / integer pipes, to take load off the special-function unit:
// Cody-Waite range reduction x = n + f, n = round(x) (by the 1.5*2^23 shifter trick),
// f in [-1/2, 1/2], 2^f by a cubic whose coefficients were fitted to minimise the
// relative error on that interval (max relative error 7.6e-5), and 2^n added into the
// exponent field. Valid for -126 <= x <= 127; callers pass finite x <= 8.
// The shifted sum t = x + 1.5*2^23 has the bit pattern 0x4B400000 + n, and
// 0x4B400000 << 23 wraps to 0 in 32 bits, so (bits(t) << 23) == (n << 23).
LTX_DEVICE float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.0551708005f, f, 0.242609262f), f, 0.693260968f), f, 0.999928176f);
  return __int_as_float(__float_as_int(p) + int(uint32_t(__float_as_int(t)) << 23));
}

// The same for two values with packed fp32x2 arithmetic.
LTX_DEVICE void ex2_poly2(float x0, float x1, float& y0, float& y1) {
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  const uint64_t shifter = f2_pack(12582912.f, 12582912.f);
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t t = f2_add(x, shifter);
  const uint64_t f = f2_sub(x, f2_sub(t, shifter));
  uint64_t p = f2_fma(f2_pack(0.0551708005f, 0.0551708005f), f, f2_pack(0.242609262f, 0.242609262f));
  p = f2_fma(p, f, f2_pack(0.693260968f, 0.693260968f));
  p = f2_fma(p, f, f2_pack(0.999928176f, 0.999928176f));
  float t0, t1, p0, p1;
  f2_unpack(t, t0, t1);
  f2_unpack(p, p0, p1);
  y0 = __int_as_float(__float_as_int(p0) + int(uint32_t(__float_as_int(t0)) << 23));
  y1 = __int_as_float(__float_as_int(p1) + int(uint32_t(__float_as_int(t1)) << 23));
}
LTX_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

LTX_DEVICE int lane_id() { return threadIdx.x & 31; }
LTX_DEVICE int warp_id() { return threadIdx.x >> 5; }
