// Attention core softmax(Q K^T * scale) V with the per-(token, head) output gate
// 2*sigmoid(logit) fused in (ltx_nn.py:22-26 sdpa, 227-235 gating).
//
// bf16 path: one CTA per (256 queries, head, sample) = two 128-row Q tiles, 11 warps:
//   warps 0-3   softmax of Q tile 0 (one query row per thread = TMEM lane)
//   warps 4-7   softmax of Q tile 1
//   warp 8      TMA producer: both Q tiles once, then K and V tiles of 128 keys into a
//               STAGES-deep ring
//   warp 9      tcgen05.mma issuer of Q tile 0, TMEM owner
//   warp 10     tcgen05.mma issuer of Q tile 1 (on another SM sub-partition, so the
//               two issue streams and their waits overlap); head_dim 128 has no warp
//               10: warp 9 issues both tiles' MMAs in a fixed alternation (below)
// S_i = Q_i K^T lands in TMEM as fp32; the softmax of tile i writes P_i as packed bf16;
// O_i accumulates P_i V over all key tiles in TMEM (A operand read from TMEM, V as an
// MN-major 128B-swizzled smem operand).
//
// TMEM (512 columns):
//   head_dim 64:  S_0, S_1 at [0,128), [128,256); P_0, P_1 at [256,320), [320,384);
//                 O_0, O_1 at [384,448), [448,512). P has its own columns, so the softmax
//                 releases S_i as soon as it has loaded it and the issuer computes
//                 S_i(t+2) = Q_i K_{t+2}^T right after P_i V_t, while the softmax of key
//                 tile t+1 runs: the MMA round trip is off the softmax's critical path.
//   head_dim 128: S_i at [128 i, 128 i + 128) with P_i written over its first 64 columns,
//                 O_i at [256 + 128 i, ...); S_i(t+1) is issued after P_i V_t.
// Lazy rescaling: each row keeps a reference max m_ref and only moves it (rescaling its
// O row and l) when the tile max exceeds it by more than 8 (log2 units); P = 2^(s - m_ref)
// then stays <= 256, and O / l is unchanged by the choice of reference.
// Keys at or beyond Tk are masked to -inf (last tile only); rows at or beyond Tq are not
// stored.
//
// fp32 path: CUDA-core online-softmax kernel, one query per thread (accuracy mode).
#include <algorithm>
#include <type_traits>

#include "ltx_kernels.cuh"

namespace ltx {
namespace detail {

template <int D>
struct FaCfg {
  static constexpr int BM = 128;                    // rows per Q tile
  static constexpr int BN = 128;                    // keys per K/V tile
  static constexpr int SUB = D / 64;                // 64-column (128-byte) sub-tiles per row
  static constexpr int TILE_BYTES = 128 * D * 2;    // one Q, K or V tile
  static constexpr int STAGES = D == 64 ? 5 : 2;  // d 64: K is needed two tiles ahead
  static constexpr int SMEM = TILE_BYTES * (2 + 2 * STAGES) + 512 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr bool SEP_P = D == 64;            // P in its own TMEM columns
  // d 64: one MMA-issuing warp per Q tile (warps 9, 10); d 128: one issuer for both
  // tiles (warp 9), so 10 warps.
  static constexpr int THREADS = SEP_P ? 352 : 320;
  static constexpr uint32_t s_col(int i) { return uint32_t(128 * i); }
  static constexpr uint32_t p_col(int i) { return SEP_P ? uint32_t(256 + 64 * i) : uint32_t(128 * i); }
  static constexpr uint32_t o_col(int i) { return SEP_P ? uint32_t(384 + 64 * i) : uint32_t(256 + D * i); }
  static constexpr float RESCALE_THRESHOLD = 8.f;
};

LTX_DEVICE uint8_t* fa_align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Split of one attention call. A unit is (sample b, head h, 256 queries), numbered
// u = x + nq2 (h + H b) in grid order, so neighbouring units share K and V in L2.
// fmha_tc_kernel runs units [0, n_full) whole, one CTA each, in full waves of the SMs.
// The n_split units after them would only partly fill a last wave; fmha_part_kernel
// runs each of them as split_k parts over contiguous key ranges, CTA p = su * split_k + j
// being part j of unit n_full + su. A part writes fp32 O / l and the row's log2-sum-exp
// to slot p of part_o / part_lse; the last part of a unit to finish (arrival counter
// counters[su], reset by that CTA) merges the split_k parts in part order, applies the
// gate and writes O.
struct FaSched {
  int B, H, nq2, n_full, n_split, split_k;
  float* part_o;    // [n_split * split_k][256][D]
  float* part_lse;  // [n_split * split_k][256]
  int* counters;    // [n_split], zero before the first launch, left at zero
  // Output scatter (sequence-parallel exchange), when out_rows > 0: row qi of sample b goes
  // to row b * out_rows + qi % out_rows of owner qi / out_rows's buffer out[owner] (row
  // stride out_ld), columns from out_col0 + h * D on; O is not written.
  __nv_bfloat16* out[8];
  int64_t out_rows, out_ld;
  int out_col0;
};

constexpr int kFaMaxSplit = 8;

// Output row qi of sample b, head h: in O, or scattered to its token owner's buffer.
template <int D>
LTX_DEVICE __nv_bfloat16* fa_out_row(__nv_bfloat16* O, int64_t ldo, int Tq, int b, int h, int64_t qi,
                                     const FaSched& sch) {
  if (sch.out_rows > 0) {
    const int64_t owner = qi / sch.out_rows;
    return sch.out[owner] + (int64_t(b) * sch.out_rows + (qi - owner * sch.out_rows)) * sch.out_ld + sch.out_col0 +
           int64_t(h) * D;
  }
  return O + (int64_t(b) * Tq + qi) * ldo + int64_t(h) * D;
}

// Exponential pairs (of the 64 in a 128-key row of S) computed on the FMA pipe by the
// cubic of ex2_poly2 instead of the special-function unit, bit j = pair j.
#ifndef LTX_FA_POLY_PAIRS
#define LTX_FA_POLY_PAIRS 0x888888888a8a8888ull
#endif
constexpr uint64_t kFaPolyPairs = LTX_FA_POLY_PAIRS;

// One CTA's work. PART = false: a whole unit (all keys); PART = true: tk_part keys from
// key tile kv0 on, of unit n_full + su, merged as above (Tk is a multiple of the key
// tile and every part has the same tk_part keys). The two run in separate kernels,
// each with its own register allocation.
template <int D, bool PART>
__device__ __forceinline__ void fmha_body(const CUtensorMap* tmQ_, const CUtensorMap* tmK_,
                                          const CUtensorMap* tmV_, __nv_bfloat16* __restrict__ O, int64_t ldo,
                                          int Tq, int Tk, float scale_log2, const __nv_bfloat16* __restrict__ gate,
                                          int64_t ld_gate, float* __restrict__ o32, float* __restrict__ lse,
                                          int64_t ld_lse, const int h, const int b, const int q0, const int kv0,
                                          const int tk_part, const int su, const int part, const FaSched& sch) {
  using Cfg = FaCfg<D>;
  const CUtensorMap& tmQ = *tmQ_;
  const CUtensorMap& tmK = *tmK_;
  const CUtensorMap& tmV = *tmV_;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = fa_align1024(smem_raw);
  uint8_t* sQ = smem;                          // Q tile i at sQ + i * TILE
  uint8_t* sKV = smem + 2 * Cfg::TILE_BYTES;  // stage s: K at sKV + 2s*TILE, V at +TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::TILE_BYTES * (2 + 2 * Cfg::STAGES));
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;               // [STAGES]
  uint64_t* v_full = k_full + Cfg::STAGES;   // [STAGES]
  uint64_t* kv_empty = v_full + Cfg::STAGES; // [STAGES] released by both tiles' P V
  uint64_t* s_full = kv_empty + Cfg::STAGES; // [2] S_i(t) computed
  uint64_t* s_free = s_full + 2;             // [2] S_i(t) loaded by the softmax (SEP_P only)
  uint64_t* p_full = s_free + 2;             // [2] P_i(t) stored
  uint64_t* o_done = p_full + 2;             // [2] P_i V_t completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* merge_flag = abort_flag + 1;  // PART: this CTA merges its unit

  const int warp = warp_id(), lane = lane_id();
  // A part's keys are tk_part keys from tile kv0 on, tk_part a kernel parameter like Tk:
  // the key count that bounds the loops and decides full tiles must stay a launch
  // constant (computed per CTA, it made the softmax loop a third slower).
  const int tk_eff = PART ? tk_part : Tk;
  const int n_kv = (tk_eff + Cfg::BN - 1) / Cfg::BN;  // key tiles of this CTA

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if constexpr (!PART) {
    // the kernels ahead in the stream (which write q, k, v) complete before any access;
    // only then may the next kernel (the split units' parts among them) be scheduled
    pdl_wait();
    pdl_trigger();
  }

  if (warp == 8) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int col0 = h * D;
      mbar_arrive_expect_tx(q_full, 2 * Cfg::TILE_BYTES);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < Cfg::SUB; ++j)
          tma_load_2d(sQ + i * Cfg::TILE_BYTES + j * (Cfg::TILE_BYTES / Cfg::SUB), &tmQ, q_full, col0 + 64 * j,
                      b * Tq + q0 + i * Cfg::BM);
      for (int t = 0; t < n_kv; ++t) {
        const int s = t % Cfg::STAGES;
        const uint32_t r = uint32_t(t / Cfg::STAGES);
        if (!mbar_wait(&kv_empty[s], (r & 1) ^ 1, abort_flag)) break;
        uint8_t* sk = sKV + (2 * s) * Cfg::TILE_BYTES;
        uint8_t* sv = sk + Cfg::TILE_BYTES;
        const int row = b * Tk + (PART ? kv0 * Cfg::BN : 0) + t * Cfg::BN;
        mbar_arrive_expect_tx(&k_full[s], Cfg::TILE_BYTES);
#pragma unroll
        for (int j = 0; j < Cfg::SUB; ++j)
          tma_load_2d(sk + j * (Cfg::TILE_BYTES / Cfg::SUB), &tmK, &k_full[s], col0 + 64 * j, row);
        mbar_arrive_expect_tx(&v_full[s], Cfg::TILE_BYTES);
#pragma unroll
        for (int j = 0; j < Cfg::SUB; ++j)
          tma_load_2d(sv + j * (Cfg::TILE_BYTES / Cfg::SUB), &tmV, &v_full[s], col0 + 64 * j, row);
      }
    }
  } else if (warp == 9 || warp == 10) {
    if constexpr (!Cfg::SEP_P) {
      // ---------------- one MMA issuer for both Q tiles (head_dim 128) ----------------
      // P_i aliases S_i, so S_i(t+1) can only be issued after P_i V_t. Per key tile the
      // issuer keeps the order  P_0 V_t, Q_0 K_{t+1}, P_1 V_t, Q_1 K_{t+1}:  the tensor
      // pipe runs one tile's pair of MMAs while the other tile's softmax computes, and
      // the two softmaxes fall into alternation instead of competing for the
      // special-function unit at the same time (two independent issuers let the tiles
      // run in phase: 1.45 ms against 1.13 ms at B=2, H=32, T=6144).
      if (warp == 9 && lane == 0) {
        constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0);
        constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 1);
        auto issue_qk = [&](int i, int t) {
          const uint32_t qa = smem_u32(sQ) + uint32_t(i * Cfg::TILE_BYTES);
          const uint32_t s_tmem = tmem + Cfg::s_col(i);
          const uint32_t k_addr = smem_u32(sKV + (2 * (t % Cfg::STAGES)) * Cfg::TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int j = kk >> 2, k4 = kk & 3;
            const uint32_t off = uint32_t(j * (Cfg::TILE_BYTES / Cfg::SUB) + k4 * 32);
            umma_ss(s_tmem, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024), idesc_s,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[i]);
        };
        auto issue_pv = [&](int i, int t) {
          const uint32_t p_tmem = tmem + Cfg::p_col(i);
          const uint32_t o_tmem = tmem + Cfg::o_col(i);
          const int st = t % Cfg::STAGES;
          const uint32_t v_addr = smem_u32(sKV + (2 * st + 1) * Cfg::TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < Cfg::BN / 16; ++kk) {
            const uint64_t vd = umma_desc_sw128(v_addr + uint32_t(kk * 2048), Cfg::TILE_BYTES / Cfg::SUB, 1024);
            umma_ts(o_tmem, p_tmem + uint32_t(kk * 8), vd, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_done[i]);
          umma_commit(&kv_empty[st]);  // count 2: both Q tiles' P V of this stage
        };
        bool ok = mbar_wait(q_full, 0, abort_flag) && mbar_wait(&k_full[0], 0, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_qk(0, 0);
          issue_qk(1, 0);
        }
        for (int t = 0; ok && t < n_kv; ++t) {
          const int tn = t + 1;
          ok = mbar_wait(&v_full[t % Cfg::STAGES], uint32_t(t / Cfg::STAGES) & 1, abort_flag);
          if (ok && tn < n_kv)
            ok = mbar_wait(&k_full[tn % Cfg::STAGES], uint32_t(tn / Cfg::STAGES) & 1, abort_flag);
          for (int i = 0; ok && i < 2; ++i) {
            if (!mbar_wait(&p_full[i], uint32_t(t) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(i, t);
            if (tn < n_kv) issue_qk(i, tn);
          }
        }
      }
    } else {
    // ------------------- MMA issuers, one per Q tile (head_dim 64) -------------------
    // Warp 9 issues every MMA of Q tile 0, warp 10 every MMA of Q tile 1: the two
    // chains interleave in the tensor pipe, so one issuer's waits and bookkeeping
    // overlap the other's MMAs.
    const int i = warp - 9;
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 1);
      const uint32_t qa = smem_u32(sQ) + uint32_t(i * Cfg::TILE_BYTES);
      const uint32_t s_tmem = tmem + Cfg::s_col(i);
      const uint32_t p_tmem = tmem + Cfg::p_col(i);
      const uint32_t o_tmem = tmem + Cfg::o_col(i);
      auto issue_qk = [&](int t) {
        const int s = t % Cfg::STAGES;
        const uint32_t k_addr = smem_u32(sKV + (2 * s) * Cfg::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int j = kk >> 2, k4 = kk & 3;
          const uint32_t off = uint32_t(j * (Cfg::TILE_BYTES / Cfg::SUB) + k4 * 32);
          umma_ss(s_tmem, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[i]);
      };
      auto issue_pv = [&](int t) {
        const int s = t % Cfg::STAGES;
        const uint32_t v_addr = smem_u32(sKV + (2 * s + 1) * Cfg::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < Cfg::BN / 16; ++kk) {
          // 16 keys per step: P columns [8kk, 8kk+8) (two bf16 per column), V rows
          // [16kk, 16kk+16) = two 8-row swizzle atoms of 1024 bytes.
          const uint64_t vd = umma_desc_sw128(v_addr + uint32_t(kk * 2048), Cfg::TILE_BYTES / Cfg::SUB, 1024);
          umma_ts(o_tmem, p_tmem + uint32_t(kk * 8), vd, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[i]);
        umma_commit(&kv_empty[s]);  // count 2: both Q tiles' P V of this stage
      };
      bool ok = mbar_wait(q_full, 0, abort_flag) && mbar_wait(&k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      // Order per key tile t: P_i V_t, then Q_i K_{t+2}^T. S_i is computed two tiles
      // ahead (S_i is free as soon as the softmax has loaded it), so the softmax never
      // waits for its next S, and P_i V_t runs while the softmax of tile t+1 computes
      // its exponentials.
      if (ok && n_kv > 1) {
        ok = mbar_wait(&k_full[1 % Cfg::STAGES], uint32_t(1 / Cfg::STAGES) & 1, abort_flag) &&
             mbar_wait(&s_free[i], 0, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_qk(1);
        }
      }
      for (int t = 0; ok && t < n_kv; ++t) {
        const int t2 = t + 2;
        if (!mbar_wait(&v_full[t % Cfg::STAGES], uint32_t(t / Cfg::STAGES) & 1, abort_flag) ||
            !mbar_wait(&p_full[i], uint32_t(t) & 1, abort_flag))
          break;
        tc_fence_after();
        issue_pv(t);
        if (t2 < n_kv) {
          if (!mbar_wait(&k_full[t2 % Cfg::STAGES], uint32_t(t2 / Cfg::STAGES) & 1, abort_flag) ||
              !mbar_wait(&s_free[i], uint32_t(t + 1) & 1, abort_flag))
            break;
          tc_fence_after();
          issue_qk(t2);
        }
      }
    }
    }
  } else {
    // --------------------- softmax / correction / epilogue ---------------------
    const int qt = warp >> 2;                  // Q tile of this warpgroup
    const int row = (warp & 3) * 32 + lane;    // row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_tmem = tmem + Cfg::s_col(qt) + lane_off;
    const uint32_t p_tmem = tmem + Cfg::p_col(qt) + lane_off;
    const uint32_t o_tmem = tmem + Cfg::o_col(qt) + lane_off;
    float m_ref = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < n_kv; ++t) {
      if (!mbar_wait(&s_full[qt], uint32_t(t) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + uint32_t(c * 32), *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_wait_ld();
      if constexpr (Cfg::SEP_P) {
        // S_i is in registers: let the MMA warp compute the next S_i now.
        tc_fence_before();
        mbar_arrive(&s_free[qt]);
      }
      const int valid = tk_eff - t * Cfg::BN;
      if (valid < Cfg::BN) {
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e >= valid) sv[e] = -INFINITY;
      }
      // row max: 3-input max, 8 independent chains
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = sv[e];
#pragma unroll
      for (int e = 8; e < 128; e += 16)
#pragma unroll
        for (int j = 0; j < 8; ++j) m8[j] = fmax3(m8[j], sv[e + j], sv[e + 8 + j]);
      const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      const float m_cand = mx * scale_log2;
      const bool need = (t == 0) || (m_cand > m_ref + Cfg::RESCALE_THRESHOLD);
      float alpha = 1.f;
      if (need) {
        const float m_new = fmaxf(m_ref, m_cand);
        alpha = (t == 0) ? 0.f : ex2_approx(m_ref - m_new);
        m_ref = m_new;
      }
      // x = s * scale_log2 - m_ref and the row sum in packed fp32x2 (two lanes per
      // instruction); on full tiles the pairs set in kFaPolyPairs take the FMA-pipe
      // exponential, the others the special-function unit.
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = f2_pack(-m_ref, -m_ref);
      uint64_t rs2[4] = {0, 0, 0, 0};  // bit pattern of (0.f, 0.f)
      uint32_t pk[64];
      const bool full = valid >= Cfg::BN;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0, x1, p0, p1;
          f2_unpack(f2_fma(f2_pack(sv[c * 32 + e], sv[c * 32 + e + 1]), sc2, nm2), x0, x1);
          if (full && ((kFaPolyPairs >> (c * 16 + (e >> 1))) & 1u)) {
            ex2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          rs2[(e >> 1) & 3] = f2_add(rs2[(e >> 1) & 3], f2_pack(p0, p1));
          pk[c * 16 + (e >> 1)] = pack_bf16x2(p0, p1);
        }
        // Aliased P: S_i(t) is in registers and P_i V_{t-1} completed before Q_i K_t^T
        // wrote S_i, so each chunk is stored at once.
        if constexpr (!Cfg::SEP_P) tmem_st16(p_tmem + uint32_t(c * 16), *reinterpret_cast<uint32_t(*)[16]>(&pk[c * 16]));
      }
      if constexpr (Cfg::SEP_P) {
        // Separate P: P_i V_{t-1} must be complete before P_i(t) overwrites P_i. Waiting
        // only now, after the exponentials, leaves that MMA the whole softmax to finish.
        if (t > 0) {
          if (!mbar_wait(&o_done[qt], uint32_t(t - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tmem_st16(p_tmem + uint32_t(c * 16), *reinterpret_cast<uint32_t(*)[16]>(&pk[c * 16]));
      }
      float r0, r1;
      f2_unpack(f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3])), r0, r1);
      // Rescale this row's O accumulator when its reference max moved (warp-collective
      // TMEM access: the whole warp takes the branch, rows that did not move use 1).
      // Done after the P store so that the S registers are dead.
      if (t > 0 && __any_sync(0xffffffffu, need)) {
        if (!Cfg::SEP_P) {
          if (!mbar_wait(&o_done[qt], uint32_t(t - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
          tmem_st32(o_tmem + uint32_t(c0), rr);
        }
      }
      l_run = l_run * alpha + (r0 + r1);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[qt]);
    }
    const bool have = ok && mbar_wait(&o_done[qt], uint32_t(n_kv - 1) & 1, abort_flag);
    if constexpr (PART) {
      // fp32 O / l and the log2-sum-exp of this key range to slot su * split_k + part;
      // every part CTA counts itself in exactly once (also after an abort, so the counter
      // always returns to zero) and the last one merges all parts in part order.
      const int r = qt * Cfg::BM + row;
      const int qi = q0 + r;
      const int64_t slot = int64_t(su) * sch.split_k + part;
      if (have) {
        tc_fence_after();
        const float inv_l = 1.f / l_run;
        float* dst = sch.part_o + (slot * 256 + r) * D;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
          if (qi < Tq) {
#pragma unroll
            for (int e4 = 0; e4 < 32; e4 += 4)
              __stcg(reinterpret_cast<float4*>(dst + c0 + e4),
                     make_float4(__uint_as_float(rr[e4]) * inv_l, __uint_as_float(rr[e4 + 1]) * inv_l,
                                 __uint_as_float(rr[e4 + 2]) * inv_l, __uint_as_float(rr[e4 + 3]) * inv_l));
          }
        }
        if (qi < Tq) __stcg(sch.part_lse + slot * 256 + r, m_ref + log2f(l_run));
      }
      __threadfence();
      named_bar_sync(1, 2 * Cfg::BM);  // the 8 softmax warps
      if (threadIdx.x == 0) {
        const int last = atomicAdd(&sch.counters[su], 1) == sch.split_k - 1;
        if (last) atomicExch(&sch.counters[su], 0);
        *merge_flag = last;
      }
      named_bar_sync(1, 2 * Cfg::BM);
      if (*merge_flag) {
        // All MMAs and loads of this CTA are complete (every softmax thread waited for its
        // tile's last P V before the barrier above), so shared memory is free: stage the
        // per-row part weights 2^(lse_j - max), 1 / sum and the gate there, then merge with
        // whole warps reading contiguous rows of the parts, many loads in flight.
        __threadfence();
        float* mw = reinterpret_cast<float*>(smem);  // [kFaMaxSplit][256]
        float* minv = mw + kFaMaxSplit * 256;        // [256]
        float* mg = minv + 256;                      // [256]
        const int64_t slot0 = int64_t(su) * sch.split_k;
        {
          float w[kFaMaxSplit];
          float lmax = -INFINITY;
#pragma unroll
          for (int j = 0; j < kFaMaxSplit; ++j) {
            w[j] = (j < sch.split_k && qi < Tq) ? __ldcg(sch.part_lse + (slot0 + j) * 256 + r) : -INFINITY;
            lmax = fmaxf(lmax, w[j]);
          }
          float wsum = 0.f;
#pragma unroll
          for (int j = 0; j < kFaMaxSplit; ++j) {
            w[j] = (j < sch.split_k && qi < Tq) ? exp2f(w[j] - lmax) : 0.f;
            wsum += w[j];
            mw[j * 256 + r] = w[j];
          }
          minv[r] = qi < Tq ? 1.f / wsum : 0.f;
          float g = 1.f;
          if (gate != nullptr && qi < Tq) {
            const float lg = __bfloat162float(gate[(int64_t(b) * Tq + qi) * ld_gate + h]);
            const float sg = round_bf16(1.f / (1.f + expf(-lg)));
            g = round_bf16(2.f * sg);
          }
          mg[r] = g;
        }
        named_bar_sync(1, 2 * Cfg::BM);
        constexpr int C4 = D / 4;  // float4 chunks per row; 256 * C4 is a multiple of 1024
        const float* src = sch.part_o + slot0 * 256 * D;
        const int tid = int(threadIdx.x);
        for (int c = tid; c < 256 * C4; c += 4 * 256) {
          float4 acc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int cc = c + u * 256, rr = cc / C4, col = (cc % C4) * 4;
            acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kFaMaxSplit; ++j) {
              if (j < sch.split_k) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(src + (int64_t(j) * 256 + rr) * D + col));
                const float wj = mw[j * 256 + rr];
                acc[u].x += wj * a.x;
                acc[u].y += wj * a.y;
                acc[u].z += wj * a.z;
                acc[u].w += wj * a.w;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int cc = c + u * 256, rr = cc / C4, col = (cc % C4) * 4;
            const int qr = q0 + rr;
            if (qr < Tq) {
              const float inv = minv[rr], g = mg[rr];
              float o0 = round_bf16(acc[u].x * inv), o1 = round_bf16(acc[u].y * inv);
              float o2 = round_bf16(acc[u].z * inv), o3 = round_bf16(acc[u].w * inv);
              if (gate != nullptr) {
                o0 *= g;
                o1 *= g;
                o2 *= g;
                o3 *= g;
              }
              *reinterpret_cast<uint2*>(fa_out_row<D>(O, ldo, Tq, b, h, qr, sch) + col) =
                  make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
            }
          }
        }
      }
    } else if (have) {
      tc_fence_after();
      const int qi = q0 + qt * Cfg::BM + row;
      const float inv_l = 1.f / l_run;
      float g = 1.f;
      const int64_t orow = int64_t(b) * Tq + qi;
      if (o32 != nullptr) {
        // partial attention over a part of the keys (split-KV): fp32 O / l and the
        // row's log2-sum-exp of the scaled scores, log2(sum_j 2^(s_j * scale * log2 e)),
        // for a later merge; no gate
        float* op32 = o32 + orow * ldo + int64_t(h) * D;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
          if (qi < Tq) {
#pragma unroll
            for (int e4 = 0; e4 < 32; e4 += 4)
              *reinterpret_cast<float4*>(op32 + c0 + e4) =
                  make_float4(__uint_as_float(rr[e4]) * inv_l, __uint_as_float(rr[e4 + 1]) * inv_l,
                              __uint_as_float(rr[e4 + 2]) * inv_l, __uint_as_float(rr[e4 + 3]) * inv_l);
          }
        }
        if (qi < Tq) lse[orow * ld_lse + h] = m_ref + log2f(l_run);
      } else {
        if (gate != nullptr && qi < Tq) {
          const float lg = __bfloat162float(gate[orow * ld_gate + h]);
          const float sg = round_bf16(1.f / (1.f + expf(-lg)));
          g = round_bf16(2.f * sg);
        }
        __nv_bfloat16* op = fa_out_row<D>(O, ldo, Tq, b, h, qi < Tq ? qi : 0, sch);  // stored only if qi < Tq
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
          if (qi < Tq) {
#pragma unroll
            for (int e8 = 0; e8 < 32; e8 += 8) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float o = round_bf16(__uint_as_float(rr[e8 + e]) * inv_l);
                v[e] = gate != nullptr ? o * g : o;
              }
              st8<__nv_bfloat16>(op + c0 + e8, v);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int D>
// d 64: 11 warps, three share one SM sub-partition's 16K registers, so <= 168 per
// thread; d 128: 10 warps (registers are allocated for 12, so also <= 168).
__global__ void __launch_bounds__(FaCfg<D>::THREADS, 1)
    fmha_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo, int Tq,
                   int Tk, float scale_log2, const __nv_bfloat16* __restrict__ gate, int64_t ld_gate,
                   float* __restrict__ o32, float* __restrict__ lse, int64_t ld_lse, const FaSched sch) {
  // Whole units only: the units from n_full on run as parts (fmha_part_kernel). A CTA
  // that leaves still waits for the kernels ahead of it: fmha_part_kernel is scheduled
  // once every CTA here has passed that wait or exited, and it reads q, k, v without a
  // wait of its own (with n_full = 0 every CTA leaves here).
  if (int(blockIdx.x) + int(gridDim.x) * (int(blockIdx.y) + int(gridDim.y) * int(blockIdx.z)) >= sch.n_full) {
    pdl_wait();
    return;
  }
  fmha_body<D, false>(&tmQ, &tmK, &tmV, O, ldo, Tq, Tk, scale_log2, gate, ld_gate, o32, lse, ld_lse,
                      int(blockIdx.y), int(blockIdx.z), int(blockIdx.x) * 2 * FaCfg<D>::BM, 0, 0, -1, -1, sch);
}

// The split units' parts, one CTA each (CTA p = part p % split_k of unit n_full + p /
// split_k), launched after fmha_tc_kernel has run the whole units in full waves.
template <int D>
__global__ void __launch_bounds__(FaCfg<D>::THREADS, 1)
    fmha_part_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo, int Tq,
                     int Tk, float scale_log2, const __nv_bfloat16* __restrict__ gate, int64_t ld_gate,
                     const int tk_part, const FaSched sch) {
  // Launched after fmha_tc_kernel, whose CTAs let it be scheduled only once the kernels
  // writing q, k and v have completed; it needs nothing that grid writes, so it starts
  // at once, and it lets the next kernel be scheduled (which waits for its completion).
  pdl_trigger();
  const int p = int(blockIdx.x);
  const int su = p / sch.split_k, part = p % sch.split_k;
  const int unit = sch.n_full + su;
  const int kv0 = part * (tk_part / FaCfg<D>::BN);
  fmha_body<D, true>(&tmQ, &tmK, &tmV, O, ldo, Tq, Tk, scale_log2, gate, ld_gate, nullptr, nullptr, 0,
                     (unit / sch.nq2) % sch.H, unit / (sch.nq2 * sch.H), (unit % sch.nq2) * 2 * FaCfg<D>::BM, kv0,
                     tk_part, su, part, sch);
  // Complete only after the whole-unit grid has: work queued behind this launch then
  // sees both grids' outputs.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// Short-context attention (Tk <= 128: all keys in one tile), the cross-attention to the
// text context. Persistent CTAs walk a contiguous range of tasks (sample, head, 128-row
// Q tile), ordered so that consecutive tasks share (sample, head): K and V of a
// (sample, head) are loaded once per run of tasks (two generations double-buffered),
// Q tiles are double-buffered, and the two softmax warpgroups take alternate tasks, so
// the output of task j is normalised and stored while task j+1 is in its softmax and
// the tensor core and TMA work ahead. Same roles as fmha_tc_kernel: warps 0-3 and 4-7
// softmax + epilogue, warp 8 TMA, warp 9 MMA.
// TMEM: S_w at [128 w, 128 w + 128) with P_w written over its first 64 columns,
// O_w at [256 + D w, 256 + D w + D).
// ---------------------------------------------------------------------------------
template <int D>
struct Kv1Cfg {
  static constexpr int TILE = 128 * D * 2;
  static constexpr int SUB = D / 64;
  static constexpr int SMEM = TILE * 2 + TILE * 4 + 512 + 1024;  // Q x 2, (K, V) x 2
  static constexpr uint32_t TMEM_COLS = 512;
};

template <int D>
__global__ void __launch_bounds__(320, 1)
    fmha_kv1_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo, int Tq,
                    int Tk, int H, int n_qt, int64_t n_tasks, float scale_log2,
                    const __nv_bfloat16* __restrict__ gate, int64_t ld_gate) {
  using Cfg = Kv1Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = fa_align1024(smem_raw);
  uint8_t* sQ = smem;                        // slot w at sQ + w * TILE
  uint8_t* sKV = smem + 2 * Cfg::TILE;       // generation buffer g: K at sKV + 2g*TILE, V at +TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * Cfg::TILE);
  uint64_t* q_full = bars;          // [2]
  uint64_t* q_empty = bars + 2;     // [2]
  uint64_t* kv_full = bars + 4;     // [2]
  uint64_t* kv_empty = bars + 6;    // [2]
  uint64_t* s_full = bars + 8;      // [2]
  uint64_t* p_full = bars + 10;     // [2]
  uint64_t* o_full = bars + 12;     // [2]
  uint64_t* slot_free = bars + 14;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int64_t t0 = int64_t(blockIdx.x) * n_tasks / gridDim.x;
  const int n_local = int(int64_t(blockIdx.x + 1) * n_tasks / gridDim.x - t0);
  // task -> (sample, head, Q tile); bh = sample * H + head
  auto task_bh = [&](int j) { return int((t0 + j) / n_qt); };
  auto task_qt = [&](int j) { return int((t0 + j) % n_qt); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&slot_free[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == 8) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int gen = -1, prev_bh = -1;
      for (int j = 0; j < n_local; ++j) {
        const int bh = task_bh(j);
        const int b = bh / H, h = bh - b * H;
        if (bh != prev_bh) {
          ++gen;
          prev_bh = bh;
          const int kb = gen & 1;
          if (gen >= 2 && !mbar_wait(&kv_empty[kb], uint32_t((gen >> 1) - 1) & 1, abort_flag)) break;
          uint8_t* sk = sKV + (2 * kb) * Cfg::TILE;
          mbar_arrive_expect_tx(&kv_full[kb], 2 * Cfg::TILE);
#pragma unroll
          for (int jj = 0; jj < Cfg::SUB; ++jj) {
            tma_load_2d(sk + jj * (Cfg::TILE / Cfg::SUB), &tmK, &kv_full[kb], h * D + 64 * jj, b * Tk);
            tma_load_2d(sk + Cfg::TILE + jj * (Cfg::TILE / Cfg::SUB), &tmV, &kv_full[kb], h * D + 64 * jj, b * Tk);
          }
        }
        const int w = j & 1;
        if (j >= 2 && !mbar_wait(&q_empty[w], uint32_t((j >> 1) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[w], Cfg::TILE);
#pragma unroll
        for (int jj = 0; jj < Cfg::SUB; ++jj)
          tma_load_2d(sQ + w * Cfg::TILE + jj * (Cfg::TILE / Cfg::SUB), &tmQ, &q_full[w], h * D + 64 * jj,
                      b * Tq + task_qt(j) * 128);
      }
    }
  } else if (warp == 9) {
    // ------------------------------ MMA issuer ---------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 1);
      int gen = -1, prev_bh = -1;
      bool ok = true;
      for (int j = 0; ok && j <= n_local; ++j) {
        const int gen_prev = gen;  // generation of task j - 1
        if (j < n_local) {
          const int bh = task_bh(j);
          const int w = j & 1;
          if (bh != prev_bh) {
            ++gen;
            prev_bh = bh;
            if (!mbar_wait(&kv_full[gen & 1], uint32_t(gen >> 1) & 1, abort_flag)) break;
          }
          if (!mbar_wait(&q_full[w], uint32_t(j >> 1) & 1, abort_flag)) break;
          // S_w / P_w / O_w are free once the softmax warpgroup finished task j - 2.
          if (j >= 2 && !mbar_wait(&slot_free[w], uint32_t((j >> 1) - 1) & 1, abort_flag)) break;
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ + w * Cfg::TILE);
          const uint32_t ka = smem_u32(sKV + (2 * (gen & 1)) * Cfg::TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = uint32_t((kk >> 2) * (Cfg::TILE / Cfg::SUB) + (kk & 3) * 32);
            umma_ss(tmem + uint32_t(128 * w), umma_desc_sw128(qa + off, 16, 1024),
                    umma_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[w]);
          umma_commit(&q_empty[w]);
        }
        if (j >= 1) {
          const int jp = j - 1, wp = jp & 1;
          if (!mbar_wait(&p_full[wp], uint32_t(jp >> 1) & 1, abort_flag)) break;
          tc_fence_after();
          const uint32_t va = smem_u32(sKV + (2 * (gen_prev & 1) + 1) * Cfg::TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t vd = umma_desc_sw128(va + uint32_t(kk * 2048), Cfg::TILE / Cfg::SUB, 1024);
            umma_ts(tmem + uint32_t(256 + D * wp), tmem + uint32_t(128 * wp + kk * 8), vd, idesc_o, kk > 0 ? 1u : 0u);
          }
          umma_commit(&o_full[wp]);
          // last task of its generation: K / V buffer free once this completes
          if (j == n_local || gen != gen_prev) umma_commit(&kv_empty[gen_prev & 1]);
        }
      }
    }
  } else {
    // --------------------- softmax / normalisation / store ---------------------
    const int w = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_tmem = tmem + uint32_t(128 * w) + lane_off;
    const uint32_t o_tmem = tmem + uint32_t(256 + D * w) + lane_off;
    for (int j = w; j < n_local; j += 2) {
      const int bh = task_bh(j);
      const int b = bh / H, h = bh - b * H;
      const uint32_t par = uint32_t(j >> 1) & 1;
      if (!mbar_wait(&s_full[w], par, abort_flag)) break;
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + uint32_t(c * 32), *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tmem_wait_ld();
      if (Tk < 128) {
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e >= Tk) sv[e] = -INFINITY;
      }
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = sv[e];
#pragma unroll
      for (int e = 8; e < 128; e += 16)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) m8[jj] = fmax3(m8[jj], sv[e + jj], sv[e + 8 + jj]);
      const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      const float m_ref = mx * scale_log2;
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = f2_pack(-m_ref, -m_ref);
      uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(sv[c * 32 + e], sv[c * 32 + e + 1]), sc2, nm2), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          rs2[(e >> 1) & 3] = f2_add(rs2[(e >> 1) & 3], f2_pack(p0, p1));
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st16(s_tmem + uint32_t(c * 16), pk);
      }
      float r0, r1;
      f2_unpack(f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3])), r0, r1);
      const float l_run = r0 + r1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[w]);
      // gate logit load overlaps the P V MMA
      const int qi = task_qt(j) * 128 + row;
      const int64_t orow = int64_t(b) * Tq + qi;
      float g = 1.f;
      if (gate != nullptr && qi < Tq) {
        const float lg = __bfloat162float(gate[orow * ld_gate + h]);
        const float sg = round_bf16(1.f / (1.f + expf(-lg)));
        g = round_bf16(2.f * sg);
      }
      const float inv_l = 1.f / l_run;
      if (!mbar_wait(&o_full[w], par, abort_flag)) break;
      tc_fence_after();
      __nv_bfloat16* op = O + orow * ldo + int64_t(h) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(o_tmem + uint32_t(c0), rr);
        tmem_wait_ld();
        if (qi < Tq) {
#pragma unroll
          for (int e8 = 0; e8 < 32; e8 += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float o = round_bf16(__uint_as_float(rr[e8 + e]) * inv_l);
              v[e] = gate != nullptr ? o * g : o;
            }
            st8<__nv_bfloat16>(op + c0 + e8, v);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&slot_free[w]);
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// fp32 attention on CUDA cores: one query per thread, K/V tiles of 32 keys in smem.
// ---------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) attn_simt_kernel(const float* __restrict__ Q, int64_t ldq,
                                                        const float* __restrict__ K, int64_t ldk,
                                                        const float* __restrict__ V, int64_t ldv,
                                                        float* __restrict__ O, int64_t ldo, int Tq, int Tk,
                                                        float scale, const float* __restrict__ gate,
                                                        int64_t ld_gate) {
  constexpr int KT = 32;
  __shared__ float sk[KT][D];
  __shared__ float sv[KT][D];
  const int h = blockIdx.y, b = blockIdx.z;
  const int qi = blockIdx.x * 128 + threadIdx.x;
  const bool active = qi < Tq;
  float q[D], acc[D];
  const float* qp = Q + (int64_t(b) * Tq + (active ? qi : 0)) * ldq + int64_t(h) * D;
#pragma unroll
  for (int c = 0; c < D; ++c) {
    q[c] = active ? qp[c] : 0.f;
    acc[c] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < Tk; k0 += KT) {
    __syncthreads();
    for (int i = threadIdx.x; i < KT * D; i += blockDim.x) {
      const int r = i / D, c = i - r * D;
      const bool in = k0 + r < Tk;
      const int64_t row = int64_t(b) * Tk + k0 + r;
      sk[r][c] = in ? K[row * ldk + int64_t(h) * D + c] : 0.f;
      sv[r][c] = in ? V[row * ldv + int64_t(h) * D + c] : 0.f;
    }
    __syncthreads();
    const int nk = Tk - k0 < KT ? Tk - k0 : KT;
    for (int r = 0; r < nk; ++r) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < D; ++c) s = fmaf(q[c], sk[r][c], s);
      s *= scale;
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int c = 0; c < D; ++c) acc[c] = fmaf(acc[c], corr, p * sv[r][c]);
      m = mn;
    }
  }
  if (!active) return;
  const int64_t orow = int64_t(b) * Tq + qi;
  float g = 1.f;
  if (gate != nullptr) g = 2.f / (1.f + expf(-gate[orow * ld_gate + h]));
  float* op = O + orow * ldo + int64_t(h) * D;
#pragma unroll
  for (int c = 0; c < D; ++c) op[c] = (acc[c] / l) * g;
}

// Split plan of one launch. The R = units mod SMs units beyond the last whole wave
// are split into k parts of n/k key tiles each (k divides the n key tiles; Tk a multiple
// of the key tile) when that ends sooner. Measured on the B200, in key-tile times: a
// whole unit costs about kFaWholeFixedTiles + n, a part kFaPartFixedTiles + n/k (the
// part's extra launch, partial stores and merge); the tail costs one round of whole
// units without the split and ceil(R k / SMs) rounds of parts with it.
struct FaPlan {
  int n_full = 0, split_k = 1, n_split = 0;
  int64_t slots() const { return int64_t(n_split) * split_k; }
};
// Attention workspace: [counters: kFaCounterBytes][part_lse: slots x 256 fp32]
// [part_o: slots x 256 x D fp32]. The counters sit at offset 0 for every shape and every
// launch leaves them at zero, so one zero-filled workspace serves any sequence of calls
// on one stream.
constexpr size_t kFaCounterBytes = 4096;
constexpr int kFaMinTilesPerPart = 3;
constexpr int kFaMaxSlotsPerSm = 4;  // bounds the workspace
constexpr double kFaWholeFixedTiles = 11.0, kFaPartFixedTiles = 16.0;

inline FaPlan fa_plan(int64_t units, int64_t Tk, int sms) {
  FaPlan p;
  p.n_full = int(units);
  const int64_t R = units % sms;
  const int n = int(Tk / 128);
  if (R == 0 || Tk % 128 != 0 || R > int64_t(kFaCounterBytes / sizeof(int))) return p;
  double best = kFaWholeFixedTiles + n;
  int best_k = 1;
  for (int k = 2; k <= kFaMaxSplit && k * kFaMinTilesPerPart <= n; ++k) {
    if (n % k != 0 || R * k > int64_t(kFaMaxSlotsPerSm) * sms) continue;
    const double cost = double((R * k + sms - 1) / sms) * (kFaPartFixedTiles + double(n / k));
    if (cost < best - 1e-9) {
      best = cost;
      best_k = k;
    }
  }
  if (best_k > 1) {
    p.n_full = int(units - R);
    p.split_k = best_k;
    p.n_split = int(R);
  }
  return p;
}

// Test hook (ltx_test_attention_force_split): > 0 runs every unit as that many parts,
// < 0 never splits.
static thread_local int g_fa_force_split = 0;

inline FaPlan fa_plan_for(int B, int64_t Tq, int64_t Tk, int H) {
  const int64_t units = int64_t(B) * H * ((Tq + 255) / 256);
  const int k = g_fa_force_split;
  if (k < 0) {
    FaPlan p;
    p.n_full = int(units);
    return p;
  }
  if (k > 0) {
    FaPlan p;
    if (Tk % 128 == 0 && (Tk / 128) % k == 0 && units <= int64_t(kFaCounterBytes / sizeof(int))) {
      p.n_full = 0;
      p.n_split = int(units);
      p.split_k = k;
    } else {
      p.n_full = int(units);
    }
    return p;
  }
  return fa_plan(units, Tk, num_sms());
}

inline size_t fa_workspace_bytes(const FaPlan& p, int D) {
  if (p.n_split == 0) return 0;
  return kFaCounterBytes + size_t(p.slots()) * 256 * 4 + size_t(p.slots()) * 256 * size_t(D) * 4;
}

template <int D>
void launch_fmha_tc(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                    int64_t ldo, int B, int64_t Tq, int64_t Tk, int H, float scale, const void* gate,
                    int64_t ld_gate, cudaStream_t s, float* o32 = nullptr, float* lse = nullptr,
                    int64_t ld_lse = 0, void* workspace = nullptr, size_t ws_bytes = 0,
                    void* const* out_parts = nullptr, int parts = 0, int64_t out_rows = 0, int64_t out_ld = 0,
                    int out_col0 = 0) {
  using Cfg = FaCfg<D>;
  const uint64_t cols = uint64_t(H) * D;
  const CUtensorMap tq = make_tmap_bf16_2d(q, cols, uint64_t(B) * Tq, uint64_t(ldq), 64, 128);
  const CUtensorMap tk = make_tmap_bf16_2d(k, cols, uint64_t(B) * Tk, uint64_t(ldk), 64, 128);
  const CUtensorMap tv = make_tmap_bf16_2d(v, cols, uint64_t(B) * Tk, uint64_t(ldv), 64, 128);
  auto kern = fmha_tc_kernel<D>;
  static std::atomic<uint64_t> smem_done{0};
  ensure_smem_limit(smem_done, kern, Cfg::SMEM);
  const int nq2 = int((Tq + 2 * Cfg::BM - 1) / (2 * Cfg::BM));
  FaSched sch{};
  sch.B = B;
  sch.H = H;
  sch.nq2 = nq2;
  sch.n_full = int(int64_t(B) * H * nq2);
  sch.split_k = 1;
  if (out_parts != nullptr) {
    for (int j = 0; j < parts; ++j) sch.out[j] = static_cast<__nv_bfloat16*>(out_parts[j]);
    sch.out_rows = out_rows;
    sch.out_ld = out_ld;
    sch.out_col0 = out_col0;
  }
  if (o32 == nullptr && workspace != nullptr) {
    const FaPlan p = fa_plan_for(B, Tq, Tk, H);
    if (p.n_split > 0 && ws_bytes >= fa_workspace_bytes(p, D)) {
      char* w = static_cast<char*>(workspace);
      sch.n_full = p.n_full;
      sch.n_split = p.n_split;
      sch.split_k = p.split_k;
      sch.counters = reinterpret_cast<int*>(w);
      sch.part_lse = reinterpret_cast<float*>(w + kFaCounterBytes);
      sch.part_o = reinterpret_cast<float*>(w + kFaCounterBytes + size_t(p.slots()) * 256 * 4);
    }
  }
  const dim3 grid{unsigned(nq2), unsigned(H), unsigned(B)};
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_pdl(kern, grid, dim3(Cfg::THREADS), Cfg::SMEM, s, 1, tq, tk, tv, static_cast<__nv_bfloat16*>(o), ldo,
             int(Tq), int(Tk), scale_log2, static_cast<const __nv_bfloat16*>(gate), ld_gate, o32, lse, ld_lse, sch);
  if (sch.n_split > 0) {
    auto pk = fmha_part_kernel<D>;
    static std::atomic<uint64_t> smem_done_p{0};
    ensure_smem_limit(smem_done_p, pk, Cfg::SMEM);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(unsigned(sch.n_split * sch.split_k));
    lc.blockDim = dim3(Cfg::THREADS);
    lc.dynamicSmemBytes = Cfg::SMEM;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LTX_CUDA(cudaLaunchKernelEx(&lc, pk, tq, tk, tv, static_cast<__nv_bfloat16*>(o), ldo, int(Tq), int(Tk),
                                scale_log2, static_cast<const __nv_bfloat16*>(gate), ld_gate,
                                int(Tk / sch.split_k), sch));
    ltx::note_launch();
  }
}

template <int D>
void launch_fmha_kv1(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                     int64_t ldo, int B, int64_t Tq, int64_t Tk, int H, float scale, const void* gate,
                     int64_t ld_gate, cudaStream_t s) {
  using Cfg = Kv1Cfg<D>;
  const uint64_t cols = uint64_t(H) * D;
  const CUtensorMap tq = make_tmap_bf16_2d(q, cols, uint64_t(B) * Tq, uint64_t(ldq), 64, 128);
  const CUtensorMap tk = make_tmap_bf16_2d(k, cols, uint64_t(B) * Tk, uint64_t(ldk), 64, 128);
  const CUtensorMap tv = make_tmap_bf16_2d(v, cols, uint64_t(B) * Tk, uint64_t(ldv), 64, 128);
  auto kern = fmha_kv1_kernel<D>;
  static std::atomic<uint64_t> smem_done{0};
  ensure_smem_limit(smem_done, kern, Cfg::SMEM);
  const int n_qt = int((Tq + 127) / 128);
  const int64_t n_tasks = int64_t(B) * H * n_qt;
  const int grid = int(std::min<int64_t>(n_tasks, num_sms()));
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_pdl(kern, dim3(unsigned(grid)), dim3(320), Cfg::SMEM, s, 1, tq, tk, tv, static_cast<__nv_bfloat16*>(o), ldo,
             int(Tq), int(Tk), H, n_qt, n_tasks, scale_log2, static_cast<const __nv_bfloat16*>(gate), ld_gate);
}

// ---------------------------------------------------------------------------------
// Perturbed self-attention (STG): the attention output is replaced by V
// (ltx_nn.py:209-210, and the blend at 229-230 with a 0/1 per-sample mask), then the
// per-(token, head) gate 2*sigmoid(logit) applies as for a real attention output
// (231-235). One thread per 8 consecutive elements of one head.
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void value_gate_kernel(const T* __restrict__ v, int64_t ldv, const T* __restrict__ gate, int64_t ld_gate,
                                  T* __restrict__ o, int64_t ldo, int64_t rows, int heads, int d) {
  const int per_row = heads * d / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * per_row) return;
  const int64_t r = i / per_row;
  const int c = int(i - r * per_row) * 8;
  float x[8];
  ld8<T>(v + r * ldv + c, x);
  if (gate != nullptr) {
    const float lg = ld_elem<T>(gate + r * ld_gate + c / d);
    float g;
    if constexpr (std::is_same<T, float>::value) {
      g = 2.f / (1.f + expf(-lg));
    } else {
      const float sg = round_bf16(1.f / (1.f + expf(-lg)));
      g = round_bf16(2.f * sg);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] *= g;
  }
  st8<T>(o + r * ldo + c, x);
}

}  // namespace detail
}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

extern "C" int ltx_value_gate(const void* v, int64_t ldv, const void* gate_logits, int64_t ld_gate, void* o,
                              int64_t ldo, int64_t rows, int heads, int head_dim, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_F32 || dtype == LTX_BF16, "dtype must be F32 or BF16");
  LTX_REQUIRE(v && o, "v and o must be non-NULL");
  LTX_REQUIRE(rows > 0 && heads > 0 && head_dim > 0 && head_dim % 8 == 0, "bad shape (head_dim % 8 == 0)");
  const int64_t inner = int64_t(heads) * head_dim;
  LTX_REQUIRE(ldv >= inner && ldo >= inner && ldv % 8 == 0 && ldo % 8 == 0,
              "ldv / ldo must be multiples of 8 and >= heads*head_dim");
  if (gate_logits) LTX_REQUIRE(ld_gate >= heads, "ld_gate must be >= heads");
  check_vec_ptr(v, "v");
  check_vec_ptr(o, "o");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = rows * (inner / 8);
  const unsigned blocks = unsigned((n + 255) / 256);
  if (dtype == LTX_F32)
    value_gate_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(v), ldv,
                                                    static_cast<const float*>(gate_logits), ld_gate,
                                                    static_cast<float*>(o), ldo, rows, heads, head_dim),
        ltx::note_launch();
  else
    value_gate_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(v), ldv, static_cast<const __nv_bfloat16*>(gate_logits), ld_gate,
        static_cast<__nv_bfloat16*>(o), ldo, rows, heads, head_dim),
        ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" size_t ltx_attention_workspace_bytes(int B, int64_t Tq, int64_t Tk, int heads, int head_dim) {
  if (B <= 0 || Tq <= 0 || Tk <= 128 || heads <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  return fa_workspace_bytes(fa_plan_for(B, Tq, Tk, heads), head_dim);
}

extern "C" int ltx_attention_ws(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                void* o, int64_t ldo, int B, int64_t Tq, int64_t Tk, int heads, int head_dim,
                                float scale, const void* gate_logits, int64_t ld_gate, void* workspace,
                                size_t workspace_bytes, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_F32 || dtype == LTX_BF16, "dtype must be F32 or BF16");
  LTX_REQUIRE(q && k && v && o, "q, k, v and o must be non-NULL");
  LTX_REQUIRE(B > 0 && Tq > 0 && Tk > 0 && heads > 0, "B, Tq, Tk and heads must be positive");
  LTX_REQUIRE(int64_t(B) * Tq < (int64_t(1) << 31) && int64_t(B) * Tk < (int64_t(1) << 31), "too many rows");
  const int64_t inner = int64_t(heads) * head_dim;
  LTX_REQUIRE(ldq >= inner && ldk >= inner && ldv >= inner && ldo >= inner, "leading dimensions too small");
  if (gate_logits) LTX_REQUIRE(ld_gate >= heads, "ld_gate must be >= heads");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_BF16) {
    LTX_UNSUPPORTED(head_dim == 64 || head_dim == 128, "bf16 attention supports head_dim 64 and 128");
    LTX_REQUIRE(ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && ldo % 8 == 0, "leading dims must be multiples of 8");
    check_vec_ptr(q, "q");
    check_vec_ptr(k, "k");
    check_vec_ptr(v, "v");
    check_vec_ptr(o, "o");
    // one key tile (the text context): persistent short-context kernel
    if (Tk <= 128 && head_dim == 64)
      launch_fmha_kv1<64>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s);
    else if (Tk <= 128)
      launch_fmha_kv1<128>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s);
    else if (head_dim == 64)
      launch_fmha_tc<64>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s, nullptr,
                         nullptr, 0, workspace, workspace_bytes);
    else
      launch_fmha_tc<128>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s, nullptr,
                          nullptr, 0, workspace, workspace_bytes);
  } else {
    dim3 grid(unsigned((Tq + 127) / 128), unsigned(heads), unsigned(B));
    auto Qp = static_cast<const float*>(q);
    auto Kp = static_cast<const float*>(k);
    auto Vp = static_cast<const float*>(v);
    auto Op = static_cast<float*>(o);
    auto Gp = static_cast<const float*>(gate_logits);
    switch (head_dim) {
      case 32: attn_simt_kernel<32><<<grid, 128, 0, s>>>(Qp, ldq, Kp, ldk, Vp, ldv, Op, ldo, int(Tq), int(Tk), scale, Gp, ld_gate), ltx::note_launch(); break;
      case 64: attn_simt_kernel<64><<<grid, 128, 0, s>>>(Qp, ldq, Kp, ldk, Vp, ldv, Op, ldo, int(Tq), int(Tk), scale, Gp, ld_gate), ltx::note_launch(); break;
      case 128: attn_simt_kernel<128><<<grid, 128, 0, s>>>(Qp, ldq, Kp, ldk, Vp, ldv, Op, ldo, int(Tq), int(Tk), scale, Gp, ld_gate), ltx::note_launch(); break;
      default: LTX_UNSUPPORTED(false, "fp32 attention supports head_dim 32, 64 and 128");
    }
  }
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                             void* o, int64_t ldo, int B, int64_t Tq, int64_t Tk, int heads, int head_dim,
                             float scale, const void* gate_logits, int64_t ld_gate, int dtype, void* stream) {
  return ltx_attention_ws(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, head_dim, scale, gate_logits, ld_gate,
                          nullptr, 0, dtype, stream);
}

extern "C" int ltx_test_attention_force_split(int parts) {
  LTX_API_BEGIN
  LTX_REQUIRE(parts >= -1 && parts <= kFaMaxSplit, "parts must be in [-1, 8]");
  g_fa_force_split = parts;
  LTX_API_END
}

extern "C" int ltx_attention_scatter(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                     int64_t ldv, int B, int64_t T, int heads, int head_dim, float scale,
                                     const void* gate_logits, int64_t ld_gate, void* workspace, size_t workspace_bytes,
                                     int parts, void* const* out, int64_t out_ld, int out_col0, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(q && k && v && out, "q, k, v and out must be non-NULL");
  LTX_REQUIRE(B > 0 && T > 128 && heads > 0, "B and heads must be positive, T > 128");
  LTX_UNSUPPORTED(head_dim == 64 || head_dim == 128, "bf16 attention supports head_dim 64 and 128");
  LTX_REQUIRE(parts >= 1 && parts <= 8 && T % parts == 0, "parts must be 1..8 and divide T");
  LTX_REQUIRE(int64_t(B) * T < (int64_t(1) << 31), "too many rows");
  const int64_t inner = int64_t(heads) * head_dim;
  LTX_REQUIRE(ldq >= inner && ldk >= inner && ldv >= inner, "leading dimensions too small");
  LTX_REQUIRE(ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && out_ld % 8 == 0 && out_col0 % 8 == 0,
              "leading dims and out_col0 must be multiples of 8");
  LTX_REQUIRE(out_ld >= out_col0 + inner, "out_ld too small");
  if (gate_logits) LTX_REQUIRE(ld_gate >= heads, "ld_gate must be >= heads");
  check_vec_ptr(q, "q");
  check_vec_ptr(k, "k");
  check_vec_ptr(v, "v");
  for (int j = 0; j < parts; ++j) {
    LTX_REQUIRE(out[j] != nullptr, "out[j] is NULL");
    check_vec_ptr(out[j], "out[j]");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    launch_fmha_tc<64>(q, ldq, k, ldk, v, ldv, nullptr, 0, B, T, T, heads, scale, gate_logits, ld_gate, s, nullptr,
                       nullptr, 0, workspace, workspace_bytes, out, parts, T / parts, out_ld, out_col0);
  else
    launch_fmha_tc<128>(q, ldq, k, ldk, v, ldv, nullptr, 0, B, T, T, heads, scale, gate_logits, ld_gate, s, nullptr,
                        nullptr, 0, workspace, workspace_bytes, out, parts, T / parts, out_ld, out_col0);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_test_attention_plan(int64_t units, int64_t Tk, int sms, int* n_full, int* split_k) {
  LTX_API_BEGIN
  LTX_REQUIRE(units > 0 && Tk > 0 && sms > 0 && n_full != nullptr && split_k != nullptr, "bad argument");
  const FaPlan p = fa_plan(units, Tk, sms);
  *n_full = p.n_full;
  *split_k = p.n_split > 0 ? p.split_k : 1;
  LTX_API_END
}
