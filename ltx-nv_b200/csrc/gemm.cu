// Linear layers C = epilogue(A * W^T + bias), A (M, K) and W (N, K) both K-major
// (nn.Linear's weight layout), for every projection of the DiT step.
//
// bf16, M >= 32: persistent, warp-specialised tcgen05 kernel.
//   * 128 x BN output tiles (BN = 128 or 256), K consumed in 64-element (128-byte)
//     slabs that TMA writes into a STAGES-deep ring of 128B-swizzled shared buffers.
//   * warp 0 / lane 0: TMA producer. warp 1 / lane 0: issues tcgen05.mma (M=128,
//     N=BN, K=16 per instruction) into a double-buffered fp32 accumulator in TMEM, and
//     commits each slab back to the producer. warps 2-5: epilogue; each thread owns one
//     accumulator row (TMEM lane), pulls 32 columns at a time with tcgen05.ld, applies
//     bias / activation / gate / residual and stores bf16 with 16-byte stores while the
//     MMA warp already accumulates the next tile into the other TMEM buffer.
//   * Grid = min(#tiles, #SMs); tiles are visited N-fastest so the A row block stays
//     in L2 while its N tiles are produced.
// bf16 or fp32, M < 32: weight-streaming kernel (the per-sample adaLN / timestep MLPs,
//   where the problem is reading W once from HBM).
// fp32, M >= 32: CUDA-core tiled kernel (the accuracy mode).
#include <algorithm>

#include "ltx_kernels.cuh"

namespace ltx {
namespace detail {

constexpr int kBM = 128;
constexpr int kBK = 64;

// PAIR: a cluster of two CTAs on neighbouring SMs computes a 256 x BN tile with
// tcgen05 cta_group::2 MMAs (M = 256): each CTA loads its 128 rows of A and half of
// the BN rows of B, so a stage holds 16 + 16 KB per SM instead of 16 + 32 KB and the
// ring is six stages deep.
template <int BN, bool PAIR = false>
struct TcCfg {
  static constexpr int STAGES = PAIR ? 6 : (BN == 256 ? 4 : 6);
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // B rows loaded by one CTA
  static constexpr int B_BYTES = B_ROWS * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int VEC_BYTES = 3 * BN * 2;  // bias, gate table, row_vec of one tile
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + VEC_BYTES + 1024;
};

// Named barrier 1 over the 8 epilogue warps (256 threads) of gemm_tc_kernel.
LTX_DEVICE void epi_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

LTX_DEVICE uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int BN, bool PAIR>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   __nv_bfloat16* __restrict__ C, int64_t ldc, int M, int N, int K, Epi<__nv_bfloat16> epi) {
  using Cfg = TcCfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  // CTA pair: rank 0 (leader) issues the MMAs and owns full[] and tempty[]; tiles are
  // 256 rows, rank r takes rows [128 r, 128 r + 128) and B rows [BN/2 r, BN/2 r + BN/2).
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  constexpr int TM = PAIR ? 2 * kBM : kBM;
  const int m_tiles = (M + TM - 1) / TM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (K + kBK - 1) / kBK;
  const int tile0 = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int tile_step = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 16 : 8);  // one arrival per epilogue warp (of both CTAs)
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
    __syncwarp();
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = tile0; tile < num_tiles; tile += tile_step) {
        const int m0 = (tile / n_tiles) * TM + int(rank) * kBM;
        const int n0 = (tile % n_tiles) * BN + int(rank) * Cfg::B_ROWS;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % Cfg::STAGES;
          const uint32_t r = uint32_t(it / Cfg::STAGES);
          if (!mbar_wait(&empty[s], (r & 1) ^ 1, abort_flag)) goto done;
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's full[s]
            const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
            tma_load_2d_pair(sa, &tmA, fb, kb * kBK, m0);
            tma_load_2d_pair(sb, &tmB, fb, kb * kBK, n0);
          } else {
            mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
            tma_load_2d(sa, &tmA, &full[s], kb * kBK, m0);
            tma_load_2d(sb, &tmB, &full[s], kb * kBK, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_bf16(TM, BN, 0);
      int it = 0, local = 0;
      for (int tile = tile0; tile < num_tiles; tile += tile_step, ++local) {
        const int acc = local & 1;
        const uint32_t u = uint32_t(local >> 1);
        if (!mbar_wait(&tempty[acc], (u & 1) ^ 1, abort_flag)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < k_blocks; kb += 2) {
          // two k-blocks per round: both waits first, then 8 MMAs, each stage released
          // right after its own MMAs
          const int nb = (kb + 1 < k_blocks) ? 2 : 1;
          const int s0 = it % Cfg::STAGES;
          const int s1 = (it + 1) % Cfg::STAGES;
          if (!mbar_wait(&full[s0], uint32_t(it / Cfg::STAGES) & 1, abort_flag)) goto done;
          if (nb == 2 && !mbar_wait(&full[s1], uint32_t((it + 1) / Cfg::STAGES) & 1, abort_flag)) goto done;
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (j < nb) {
              const int s = j ? s1 : s0;
              const uint32_t a_addr = smem_u32(smem + s * Cfg::STAGE_BYTES);
              const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
                const uint64_t bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
                if constexpr (PAIR)
                  umma_ss_pair(d_tmem, ad, bd, idesc, (kb + j > 0 || k > 0) ? 1u : 0u);
                else
                  umma_ss(d_tmem, ad, bd, idesc, (kb + j > 0 || k > 0) ? 1u : 0u);
              }
              if constexpr (PAIR)
                umma_commit_pair(&empty[s], 3);
              else
                umma_commit(&empty[s]);
            }
          }
          it += nb;
        }
        if constexpr (PAIR)
          umma_commit_pair(&tfull[acc], 3);
        else
          umma_commit(&tfull[acc]);
      }
    }
  } else {
    // Epilogue warps 2..9: warp w reads TMEM lane quadrant w % 4 (one accumulator row
    // per thread) and column half (w - 2) / 4 of the tile, so two warps share each SM
    // sub-partition and hide each other's latencies.
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const int c_lo = ((warp - 2) >> 2) * (BN / 2), c_hi = c_lo + BN / 2;
    const int et = threadIdx.x - 64;  // 0..255 among the epilogue threads
    // Per-column vectors of the epilogue (bias, gate table, row_vec), staged per tile.
    __nv_bfloat16* s_vec = reinterpret_cast<__nv_bfloat16*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES);
    const bool gres = epi.kind == LTX_EPI_GATE_RESIDUAL;
    const __nv_bfloat16* gtab = (gres && epi.gate.table != nullptr) ? epi.gate.table + epi.gate.toff : nullptr;
    const __nv_bfloat16* vsrc0 = epi.bias;
    const __nv_bfloat16* vsrc2 = epi.kind == LTX_EPI_ROW_MASK_ADD ? epi.row_vec : nullptr;
    // A thread whose wait failed keeps iterating (skipping the work) so that every
    // epilogue thread reaches the same named barriers.
    bool ok = true;
    int local = 0;
    // this warp's arrival on tempty (the leader's barrier for a CTA pair)
    auto release_acc = [&](int acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        else
          mbar_arrive(&tempty[acc]);
      }
    };
    for (int tile = tile0; tile < num_tiles; tile += tile_step, ++local) {
      const int acc = local & 1;
      const uint32_t u = uint32_t(local >> 1);
      const int m0 = (tile / n_tiles) * TM + int(rank) * kBM;
      const int n0 = (tile % n_tiles) * BN;
      const int64_t m = int64_t(m0) + row_in_tile;
      // sample / token of this row, once per tile (32-bit division; M < 2^31)
      const int64_t sb = int64_t(int(m) / int(epi.rows_per_batch));
      const int64_t stok = m - sb * epi.rows_per_batch;
      if (n0 + BN <= N) {
        // Full-width tile. The per-column vectors go to shared memory once per tile;
        // the per-row operands (residual, per-token gate) do not depend on the
        // accumulator and are loaded one 32-column slab ahead of their use, the first
        // slab before waiting for the MMAs. No global load is left between the TMEM
        // read and the store of a slab.
        epi_bar_sync();
        for (int i = et; i < 3 * (BN / 8); i += 256) {
          const int w = i / (BN / 8), c = (i - w * (BN / 8)) * 8;
          const __nv_bfloat16* src = w == 0 ? vsrc0 : (w == 1 ? gtab : vsrc2);
          if (src != nullptr)
            *reinterpret_cast<uint4*>(s_vec + w * BN + c) = *reinterpret_cast<const uint4*>(src + n0 + c);
        }
        epi_bar_sync();
        const bool live = m < M;
        const __nv_bfloat16* resp = (gres && live) ? epi.residual + m * epi.ld_res + n0 : nullptr;
        const __nv_bfloat16* gmod = (gres && live && epi.gate.mod != nullptr)
                                        ? epi.gate.mod + sb * epi.gate.ldb + stok * epi.gate.ldt + epi.gate.moff + n0
                                        : nullptr;
        const float rmask = (epi.kind == LTX_EPI_ROW_MASK_ADD && live) ? epi.row_mask[m] : 0.f;
        auto load_row = [&](int c0, uint4 (&r)[4], uint4 (&g)[4]) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            r[j] = resp != nullptr ? *reinterpret_cast<const uint4*>(resp + c0 + j * 8) : make_uint4(0, 0, 0, 0);
            g[j] = gmod != nullptr ? *reinterpret_cast<const uint4*>(gmod + c0 + j * 8) : make_uint4(0, 0, 0, 0);
          }
        };
        uint4 rc[4], gc[4];
        load_row(c_lo, rc, gc);
        if (ok && !mbar_wait(&tfull[acc], u & 1, abort_flag)) ok = false;
        if (!ok) continue;
        tc_fence_after();
        const uint32_t tbase = tmem_base + uint32_t(acc * BN) + (uint32_t(q * 32) << 16);
        __nv_bfloat16* crow = C + m * ldc + n0;
#pragma unroll 1
        for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(tbase + uint32_t(c0), rr);
          uint4 rn[4], gn[4];
          if (c0 + 32 < c_hi) load_row(c0 + 32, rn, gn);
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int cl = c0 + j * 8;
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(rr[j * 8 + e]);
              if (vsrc0 != nullptr) {
                float b[8];
                ld8<__nv_bfloat16>(s_vec + cl, b);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += b[e];
              }
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = round_bf16(v[e]);
              if (epi.kind == LTX_EPI_GELU_TANH) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = gelu_act<__nv_bfloat16>(v[e]);
              } else if (epi.kind == LTX_EPI_SILU) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = silu_f(v[e]);
              } else if (gres) {
                // ltx_kernels.cuh epilogue8: residual + round(round(acc + bias) * gate),
                // gate = round(table + mod).
                float g[8], r[8];
                if (epi.gate.on) {
#pragma unroll
                  for (int e = 0; e < 8; ++e) g[e] = 0.f;
                  if (gtab != nullptr) {
                    float a[8];
                    ld8<__nv_bfloat16>(s_vec + BN + cl, a);
#pragma unroll
                    for (int e = 0; e < 8; ++e) g[e] += a[e];
                  }
                  if (gmod != nullptr) {
                    unpack_bf16x2(gc[j].x, r[0], r[1]);
                    unpack_bf16x2(gc[j].y, r[2], r[3]);
                    unpack_bf16x2(gc[j].z, r[4], r[5]);
                    unpack_bf16x2(gc[j].w, r[6], r[7]);
#pragma unroll
                    for (int e = 0; e < 8; ++e) g[e] += r[e];
                  }
#pragma unroll
                  for (int e = 0; e < 8; ++e) g[e] = round_bf16(g[e]);
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e) g[e] = 1.f;
                }
                unpack_bf16x2(rc[j].x, r[0], r[1]);
                unpack_bf16x2(rc[j].y, r[2], r[3]);
                unpack_bf16x2(rc[j].z, r[4], r[5]);
                unpack_bf16x2(rc[j].w, r[6], r[7]);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = r[e] + round_bf16(v[e] * g[e]);
              } else if (epi.kind == LTX_EPI_ROW_MASK_ADD && rmask > 0.f) {
                float a[8];
                ld8<__nv_bfloat16>(s_vec + 2 * BN + cl, a);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += a[e];
              }
              st8<__nv_bfloat16>(crow + cl, v);
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            rc[j] = rn[j];
            gc[j] = gn[j];
          }
        }
        release_acc(acc);
        continue;
      }
      // Ragged last column tile (N not a multiple of BN): generic epilogue per 8 columns.
      if (ok && !mbar_wait(&tfull[acc], u & 1, abort_flag)) ok = false;
      if (!ok) continue;
      tc_fence_after();
      {
        const uint32_t tbase = tmem_base + uint32_t(acc * BN) + (uint32_t(q * 32) << 16);
#pragma unroll 1
        for (int c0 = c_lo; c0 < c_hi && n0 + c0 < N; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(tbase + uint32_t(c0), rr);
          tmem_wait_ld();
          if (m < M) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int64_t col = int64_t(n0) + c0 + g * 8;
              if (col + 8 <= N) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(rr[g * 8 + e]);
                epilogue8<__nv_bfloat16>(epi, m, col, v, nullptr, sb, stok);
                st8<__nv_bfloat16>(C + m * ldc + col, v);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (col + e < N)
                    C[m * ldc + col + e] =
                        __float2bfloat16_rn(epilogue1<__nv_bfloat16>(epi, m, col + e, __uint_as_float(rr[g * 8 + e])));
              }
            }
          }
        }
      }
      release_acc(acc);
    }
  }
done:
  __syncwarp();
  if constexpr (PAIR) {
    // no CTA of the pair leaves while the other may still signal its barriers
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
  }
}

// ---------------------------------------------------------------------------------
// CUDA-core tiled GEMM (fp32 accuracy mode): 64x64 tile, BK = 16, 4x4 per thread.
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, int64_t lda, const T* __restrict__ W,
                                                        int64_t ldw, T* __restrict__ C, int64_t ldc, int M, int N,
                                                        int K, Epi<T> epi) {
  __shared__ float As[16][64 + 4];
  __shared__ float Ws[16][64 + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = int64_t(blockIdx.y) * 64, n0 = int64_t(blockIdx.x) * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      const int r = e >> 4, kk = e & 15;
      As[kk][r] = (m0 + r < M && k0 + kk < K) ? ld_elem<T>(A + (m0 + r) * lda + k0 + kk) : 0.f;
      Ws[kk][r] = (n0 + r < N && k0 + kk < K) ? ld_elem<T>(W + (n0 + r) * ldw + k0 + kk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n < N) st_elem<T>(C + m * ldc + n, epilogue1<T>(epi, m, n, acc[i][j]));
    }
  }
}

// ---------------------------------------------------------------------------------
// Weight-streaming GEMM for M < 32: A rows (optionally SiLU'd) staged in shared memory
// as fp32, one warp per output column, W read once with 16-byte loads.
// ---------------------------------------------------------------------------------
template <typename T, int MR>
__global__ void __launch_bounds__(256) gemm_skinny_kernel(const T* __restrict__ A, int64_t lda,
                                                          const T* __restrict__ W, int64_t ldw, T* __restrict__ C,
                                                          int64_t ldc, int M, int N, int K, Epi<T> epi, int silu_in,
                                                          int64_t row0) {
  extern __shared__ float As[];  // MR x K
  for (int i = threadIdx.x; i < MR * K; i += blockDim.x) {
    const int m = i / K, k = i - m * K;
    float v = 0.f;
    if (m < M) {
      v = ld_elem<T>(A + int64_t(m) * lda + k);
      if (silu_in) v = round_to<T>(silu_f(v));
    }
    As[i] = v;
  }
  __syncthreads();
  const int lane = lane_id();
  const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + warp_id();
  const int64_t nw = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t n = gw; n < N; n += nw) {
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    const T* wr = W + n * ldw;
    for (int k = lane * 8; k < K; k += 256) {
      float w[8];
      ld8<T>(wr + k, w);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[m * K + k]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[m * K + k + 4]);
        acc[m] = fmaf(a0.x, w[0], acc[m]);
        acc[m] = fmaf(a0.y, w[1], acc[m]);
        acc[m] = fmaf(a0.z, w[2], acc[m]);
        acc[m] = fmaf(a0.w, w[3], acc[m]);
        acc[m] = fmaf(a1.x, w[4], acc[m]);
        acc[m] = fmaf(a1.y, w[5], acc[m]);
        acc[m] = fmaf(a1.z, w[6], acc[m]);
        acc[m] = fmaf(a1.w, w[7], acc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = warp_sum(acc[m]);
    if (lane < MR && lane < M) {
      float v = 0.f;
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m == lane) v = acc[m];
      st_elem<T>(C + int64_t(lane) * ldc + n, epilogue1<T>(epi, row0 + lane, n, v));
    }
  }
}

template <typename T>
void launch_skinny(const T* A, int64_t lda, const T* W, int64_t ldw, T* C, int64_t ldc, int64_t M, int64_t N,
                   int64_t K, Epi<T> epi, int silu_in, cudaStream_t s) {
  int mr = 8;
  while (mr > 1 && int64_t(mr) * K * 4 > 96 * 1024) mr >>= 1;
  LTX_UNSUPPORTED(int64_t(mr) * K * 4 <= 200 * 1024, "K too large for the weight-streaming path");
  const size_t smem = size_t(mr) * K * 4;
  int64_t blocks = (N + 7) / 8;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  for (int64_t r0 = 0; r0 < M; r0 += mr) {
    const int mm = int(M - r0 < mr ? M - r0 : mr);
    // Epilogue row indices stay absolute (row0 + lane); only A and C are shifted.
    Epi<T> e = epi;
    auto run = [&](auto mr_const) {
      constexpr int MRC = decltype(mr_const)::value;
      auto kern = gemm_skinny_kernel<T, MRC>;
      if (smem > 48 * 1024) LTX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      kern<<<unsigned(blocks), 256, smem, s>>>(A + r0 * lda, lda, W, ldw, C + r0 * ldc, ldc, mm, int(N), int(K), e,
                                               silu_in, r0), ltx::note_launch();
    };
    switch (mr) {
      case 8: run(std::integral_constant<int, 8>{}); break;
      case 4: run(std::integral_constant<int, 4>{}); break;
      case 2: run(std::integral_constant<int, 2>{}); break;
      default: run(std::integral_constant<int, 1>{}); break;
    }
  }
}

template <int BN, bool PAIR>
void launch_tc(const void* A, int64_t lda, const void* W, int64_t ldw, void* C, int64_t ldc, int64_t M, int64_t N,
               int64_t K, const Epi<__nv_bfloat16>& epi, cudaStream_t s) {
  using Cfg = TcCfg<BN, PAIR>;
  const CUtensorMap ta = make_tmap_bf16_2d(A, uint64_t(K), uint64_t(M), uint64_t(lda), kBK, kBM);
  const CUtensorMap tb = make_tmap_bf16_2d(W, uint64_t(K), uint64_t(N), uint64_t(ldw), kBK, Cfg::B_ROWS);
  constexpr int64_t TM = PAIR ? 2 * kBM : kBM;
  const int64_t tiles = ((M + TM - 1) / TM) * ((N + BN - 1) / BN);
  auto kern = gemm_tc_kernel<BN, PAIR>;
  static std::atomic<uint64_t> smem_done{0};
  ensure_smem_limit(smem_done, kern, Cfg::SMEM);
  auto Cp = static_cast<__nv_bfloat16*>(C);
  if constexpr (PAIR) {
    // one CTA pair per two SMs, persistent over the 256-row tiles
    const int64_t pairs = std::min<int64_t>(num_sms() / 2, tiles);
    launch_pdl(kern, dim3(unsigned(2 * pairs)), dim3(320), Cfg::SMEM, s, 2, ta, tb, Cp, ldc, int(M), int(N), int(K),
               epi);
  } else {
    int64_t grid = num_sms();
    if (tiles < grid) grid = tiles;
    launch_pdl(kern, dim3(unsigned(grid)), dim3(320), Cfg::SMEM, s, 1, ta, tb, Cp, ldc, int(M), int(N), int(K), epi);
  }
}


// ---------------------------------------------------------------------------------
// Output projection fused with X0 + CFG + Euler (ltx_dit.py:378, 591-593, 551-562,
// 602-606). Each CTA owns 128 tokens: the cond rows [t0, t0+128) and the uncond rows
// [T+t0, T+t0+128) of the head-modulated hidden state are multiplied by the same
// W (C = 128 output channels) into two TMEM accumulators, so the epilogue sees the
// cond / uncond velocity of a latent element side by side and writes the next latent.
// ---------------------------------------------------------------------------------
struct HeadCfg {
  static constexpr int STAGES = 4;
  static constexpr int A_BYTES = kBM * kBK * 2;     // one 128-row slab
  static constexpr int B_BYTES = 128 * kBK * 2;     // W slab (128 channels)
  static constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 256 + 1024;
};

__global__ void __launch_bounds__(192, 1)
    head_cfg_euler_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int T,
                          int K, const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ latent,
                          const float* __restrict__ ts, float cfg_m1, float sigma, float dt,
                          __nv_bfloat16* __restrict__ vel_out, __nv_bfloat16* __restrict__ denoised,
                          __nv_bfloat16* __restrict__ new_latent) {
  using Cfg = HeadCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  const int t0 = blockIdx.x * kBM;
  const int k_blocks = (K + kBK - 1) / kBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % Cfg::STAGES;
        const uint32_t r = uint32_t(kb / Cfg::STAGES);
        if (!mbar_wait(&empty[s], (r & 1) ^ 1, abort_flag)) break;
        uint8_t* base = smem + s * Cfg::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
        tma_load_2d(base, &tmA, &full[s], kb * kBK, t0);
        tma_load_2d(base + Cfg::A_BYTES, &tmA, &full[s], kb * kBK, T + t0);
        tma_load_2d(base + 2 * Cfg::A_BYTES, &tmB, &full[s], kb * kBK, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, 128, 0);
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        const int s = kb % Cfg::STAGES;
        const uint32_t r = uint32_t(kb / Cfg::STAGES);
        if (!mbar_wait(&full[s], r & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_c = smem_u32(smem + s * Cfg::STAGE_BYTES);
        const uint32_t a_u = a_c + Cfg::A_BYTES;
        const uint32_t b_w = a_c + 2 * Cfg::A_BYTES;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t bd = umma_desc_sw128(b_w + k * 32, 16, 1024);
          const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
          umma_ss(tmem_base, umma_desc_sw128(a_c + k * 32, 16, 1024), bd, idesc, acc);
          umma_ss(tmem_base + 128, umma_desc_sw128(a_u + k * 32, 16, 1024), bd, idesc, acc);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
    }
  } else {
    const int q = warp & 3;
    const int t = t0 + q * 32 + lane;
    if (mbar_wait(tfull, 0, abort_flag)) {
      tc_fence_after();
      const uint32_t lane_off = uint32_t(q * 32) << 16;
      const float tsc = t < T ? ts[t] : 0.f, tsu = t < T ? ts[T + t] : 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t rc[32], ru[32];
        tmem_ld32(tmem_base + lane_off + uint32_t(c0), rc);
        tmem_ld32(tmem_base + lane_off + 128u + uint32_t(c0), ru);
        tmem_wait_ld();
        if (t < T) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = c0 + g * 8;
            float bb[8], lat[8], vc[8], vu[8], den[8], nxt[8];
            ld8<__nv_bfloat16>(bias + col, bb);
            ld8<__nv_bfloat16>(latent + int64_t(t) * 128 + col, lat);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              vc[e] = round_bf16(__uint_as_float(rc[g * 8 + e]) + bb[e]);
              vu[e] = round_bf16(__uint_as_float(ru[g * 8 + e]) + bb[e]);
              cfg_euler_point<__nv_bfloat16>(vc[e], vu[e], lat[e], tsc, tsu, cfg_m1, sigma, dt, den[e], nxt[e]);
            }
            if (vel_out) {
              st8<__nv_bfloat16>(vel_out + int64_t(t) * 128 + col, vc);
              st8<__nv_bfloat16>(vel_out + (int64_t(T) + t) * 128 + col, vu);
            }
            if (denoised) st8<__nv_bfloat16>(denoised + int64_t(t) * 128 + col, den);
            st8<__nv_bfloat16>(new_latent + int64_t(t) * 128 + col, nxt);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace detail

// Tile-width override for tests: 0 = automatic (256-column tiles on CTA pairs when
// N >= 512 and M >= 256, else 128), 128 or 256 force single-CTA tiles of that width.
// Thread-local, so it changes only the calling thread's GEMMs.
static thread_local int g_gemm_bn_override = 0;

}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

extern "C" int ltx_gemm_set_tile_n(int bn) {
  LTX_API_BEGIN
  LTX_REQUIRE(bn == 0 || bn == 128 || bn == 256, "tile N must be 0, 128 or 256");
  g_gemm_bn_override = bn;
  LTX_API_END
}

extern "C" int ltx_linear(const void* A, int64_t lda, const void* W, int64_t ldw, void* C, int64_t ldc, int64_t M,
                          int64_t N, int64_t K, const ltx_epilogue* epi, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_F32 || dtype == LTX_BF16, "dtype must be F32 or BF16");
  LTX_REQUIRE(A && W && C, "A, W and C must be non-NULL");
  LTX_REQUIRE(M > 0 && N > 0 && K > 0, "M, N, K must be positive");
  LTX_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31), "size out of range");
  LTX_REQUIRE(lda >= K && ldw >= K && ldc >= N, "leading dimensions too small");
  const int silu_in = epi ? epi->silu_input : 0;
  const bool skinny = M < 32 || silu_in;
  const bool simt = dtype == LTX_F32 && !skinny;
  if (!simt) {
    // Weight-streaming path: 16-byte W loads. tcgen05 path: TMA on A and W, 16-byte
    // stores of C.
    LTX_REQUIRE(K % 8 == 0 && ldw % 8 == 0, "K and ldw must be multiples of 8");
    check_vec_ptr(W, "W");
    if (!skinny) {
      LTX_REQUIRE(lda % 8 == 0 && ldc % 8 == 0, "lda and ldc must be multiples of 8");
      check_vec_ptr(A, "A");
      check_vec_ptr(C, "C");
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_F32) {
    Epi<float> e = make_epi<float>(epi);
    if (M < 32 || silu_in) {
      launch_skinny<float>(static_cast<const float*>(A), lda, static_cast<const float*>(W), ldw,
                           static_cast<float*>(C), ldc, M, N, K, e, silu_in, s);
    } else {
      dim3 grid(unsigned((N + 63) / 64), unsigned((M + 63) / 64));
      gemm_simt_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(A), lda, static_cast<const float*>(W),
                                                   ldw, static_cast<float*>(C), ldc, int(M), int(N), int(K), e), ltx::note_launch();
    }
  } else {
    Epi<__nv_bfloat16> e = make_epi<__nv_bfloat16>(epi);
    if (M < 32 || silu_in) {
      launch_skinny<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(W),
                                   ldw, static_cast<__nv_bfloat16*>(C), ldc, M, N, K, e, silu_in, s);
    } else {
      int bn = g_gemm_bn_override;
      if (bn == 0) bn = (N >= 512) ? 256 : 128;
      if (bn == 256 && M >= 2 * kBM && g_gemm_bn_override == 0)
        launch_tc<256, true>(A, lda, W, ldw, C, ldc, M, N, K, e, s);
      else if (bn == 256)
        launch_tc<256, false>(A, lda, W, ldw, C, ldc, M, N, K, e, s);
      else
        launch_tc<128, false>(A, lda, W, ldw, C, ldc, M, N, K, e, s);
    }
  }
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_proj_out_cfg_euler(const void* x, int64_t ldx, const void* W, const void* bias, int64_t T, int C,
                                      int64_t K, const void* latent, const float* timesteps, float cfg_scale,
                                      float sigma, float sigma_next, void* vel_out, void* denoised, void* new_latent,
                                      int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_F32 || dtype == LTX_BF16, "dtype must be F32 or BF16");
  LTX_REQUIRE(x && W && bias && latent && timesteps && new_latent, "NULL argument");
  LTX_REQUIRE(T > 0 && K > 0 && C > 0, "bad sizes");
  LTX_REQUIRE(sigma != 0.f, "sigma must be non-zero (Euler divides by it)");
  LTX_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldx >= K, "K and ldx must be multiples of 8, ldx >= K");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_F32) {
    // Accuracy mode: CUDA-core projection into vel_out, then the element-wise update.
    LTX_REQUIRE(vel_out != nullptr, "fp32 mode needs vel_out (2*T*C) for the projection");
    ltx_epilogue e{};
    e.kind = LTX_EPI_NONE;
    e.bias = bias;
    Epi<float> ef = make_epi<float>(&e);
    dim3 grid(unsigned((C + 63) / 64), unsigned((2 * T + 63) / 64));
    gemm_simt_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, static_cast<const float*>(W), K,
                                                 static_cast<float*>(vel_out), C, int(2 * T), C, int(K), ef), ltx::note_launch();
    LTX_CUDA(cudaGetLastError());
    const int64_t n = T * C;
    cfg_euler_kernel<float><<<unsigned((n + 255) / 256), 256, 0, s>>>(
        static_cast<const float*>(vel_out), static_cast<const float*>(latent), timesteps, T, C, cfg_scale - 1.f,
        sigma, sigma_next - sigma, static_cast<float*>(denoised), static_cast<float*>(new_latent)), ltx::note_launch();
  } else {
    LTX_UNSUPPORTED(C == 128, "the fused bf16 head supports 128 output channels");
    check_vec_ptr(x, "x");
    check_vec_ptr(W, "W");
    check_vec_ptr(bias, "bias");
    check_vec_ptr(latent, "latent");
    check_vec_ptr(new_latent, "new_latent");
    check_vec_ptr(denoised, "denoised");
    check_vec_ptr(vel_out, "vel_out");
    const CUtensorMap ta = make_tmap_bf16_2d(x, uint64_t(K), uint64_t(2 * T), uint64_t(ldx), kBK, kBM);
    const CUtensorMap tb = make_tmap_bf16_2d(W, uint64_t(K), 128, uint64_t(K), kBK, 128);
    static std::atomic<uint64_t> smem_done{0};
    ensure_smem_limit(smem_done, head_cfg_euler_kernel, HeadCfg::SMEM);
    head_cfg_euler_kernel<<<unsigned((T + kBM - 1) / kBM), 192, HeadCfg::SMEM, s>>>(
        ta, tb, int(T), int(K), static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(latent),
        timesteps, cfg_scale - 1.f, sigma, sigma_next - sigma, static_cast<__nv_bfloat16*>(vel_out),
        static_cast<__nv_bfloat16*>(denoised), static_cast<__nv_bfloat16*>(new_latent)), ltx::note_launch();
  }
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
