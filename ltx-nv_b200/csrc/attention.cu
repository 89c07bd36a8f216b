// Attention core softmax(Q K^T * scale) V with the per-(token, head) output gate
// 2*sigmoid(logit) fused in (ltx_nn.py:22-26 sdpa, 227-235 gating).
//
// bf16 path, one CTA per (128 queries, head, sample), 6 warps:
//   warps 0-3  softmax / correction / epilogue, one query row per thread (TMEM lane)
//   warp 4     TMA producer: Q once, then K and V tiles of 128 keys into a ring
//   warp 5     tcgen05.mma issuer (and TMEM owner)
// TMEM (512 columns): S/P buffers 0,1 at [0,128) and [128,256): S = Q K^T lands there
// as fp32, the softmax overwrites it in place with P as packed bf16 (P chunk c goes to
// columns [16c, 16c+16), all of which it has already read). O_part buffers 0,1 at
// [256, 256+D) and [256+D, 256+2D) receive P V (A operand read from TMEM, V as an
// MN-major 128B-swizzled smem operand). The softmax threads keep the running output
// in registers: O = (O + O_part[j-1]) * exp2(m[j-1] - m[j]) while P V of tile j runs.
// Keys at or beyond Tk are masked to -inf, query rows at or beyond Tq are not stored.
//
// fp32 path: CUDA-core online-softmax kernel, one query per thread (accuracy mode).
#include "ltx_kernels.cuh"

namespace ltx {
namespace detail {

template <int D>
struct FaCfg {
  static constexpr int BM = 128;
  static constexpr int BN = 128;
  static constexpr int SUB = D / 64;                // 64-column (128-byte) sub-tiles per row
  static constexpr int TILE_BYTES = 128 * D * 2;    // Q, K or V tile
  static constexpr int STAGES = D == 64 ? 3 : 2;
  static constexpr int SMEM = TILE_BYTES * (1 + 2 * STAGES) + 512 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
};

LTX_DEVICE uint8_t* fa_align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int D>
__global__ void __launch_bounds__(192, 1)
    fmha_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo, int Tq,
                   int Tk, float scale_log2, const __nv_bfloat16* __restrict__ gate, int64_t ld_gate) {
  using Cfg = FaCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = fa_align1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + Cfg::TILE_BYTES;  // stage s: K at sKV + 2s*TILE, V at +TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::TILE_BYTES * (1 + 2 * Cfg::STAGES));
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                      // [STAGES]
  uint64_t* v_full = k_full + Cfg::STAGES;          // [STAGES]
  uint64_t* kv_empty = v_full + Cfg::STAGES;        // [STAGES]
  uint64_t* s_full = kv_empty + Cfg::STAGES;        // [2]
  uint64_t* p_full = s_full + 2;                    // [2]
  uint64_t* o_full = p_full + 2;                    // [2]
  uint64_t* o_empty = o_full + 2;                   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * Cfg::BM;
  const int n_kv = (Tk + Cfg::BN - 1) / Cfg::BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int col0 = h * D;
      mbar_arrive_expect_tx(q_full, Cfg::TILE_BYTES);
#pragma unroll
      for (int j = 0; j < Cfg::SUB; ++j)
        tma_load_2d(sQ + j * (Cfg::TILE_BYTES / Cfg::SUB), &tmQ, q_full, col0 + 64 * j, b * Tq + q0);
      for (int t = 0; t < n_kv; ++t) {
        const int s = t % Cfg::STAGES;
        const uint32_t r = uint32_t(t / Cfg::STAGES);
        if (!mbar_wait(&kv_empty[s], (r & 1) ^ 1, abort_flag)) break;
        uint8_t* sk = sKV + (2 * s) * Cfg::TILE_BYTES;
        uint8_t* sv = sk + Cfg::TILE_BYTES;
        const int row = b * Tk + t * Cfg::BN;
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
  } else if (warp == 5) {
    // ------------------------------ MMA issuer ---------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 1);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag);
      // S[t%2] = Q K_t^T
      auto issue_qk = [&](int t) -> bool {
        const int s = t % Cfg::STAGES;
        const uint32_t r = uint32_t(t / Cfg::STAGES);
        if (!mbar_wait(&k_full[s], r & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + (2 * s) * Cfg::TILE_BYTES);
        const uint32_t d_tmem = tmem + uint32_t((t & 1) * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int j = kk >> 2, k4 = kk & 3;
          const uint32_t off = uint32_t(j * (Cfg::TILE_BYTES / Cfg::SUB) + k4 * 32);
          umma_ss(d_tmem, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t & 1]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_kv > 1) ok = issue_qk(1);
      for (int t = 0; ok && t < n_kv; ++t) {
        const int buf = t & 1;
        const uint32_t u = uint32_t(t >> 1);
        const int s = t % Cfg::STAGES;
        const uint32_t r = uint32_t(t / Cfg::STAGES);
        if (!mbar_wait(&p_full[buf], u & 1, abort_flag)) break;
        if (!mbar_wait(&o_empty[buf], (u & 1) ^ 1, abort_flag)) break;
        if (!mbar_wait(&v_full[s], r & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sKV + (2 * s + 1) * Cfg::TILE_BYTES);
        const uint32_t p_tmem = tmem + uint32_t(buf * 128);
        const uint32_t o_tmem = tmem + Cfg::O_COL + uint32_t(buf * D);
#pragma unroll
        for (int kk = 0; kk < Cfg::BN / 16; ++kk) {
          // 16 keys per step: P columns [8kk, 8kk+8) (two bf16 per column), V rows
          // [16kk, 16kk+16) = two 8-row swizzle atoms of 1024 bytes.
          const uint64_t vd = umma_desc_sw128(v_addr + uint32_t(kk * 2048), Cfg::TILE_BYTES / Cfg::SUB, 1024);
          umma_ts(o_tmem, p_tmem + uint32_t(kk * 8), vd, idesc_o, kk > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[buf]);
        umma_commit(&kv_empty[s]);
        if (t + 2 < n_kv) {
          // S/P buffer `buf` is reused by Q K_{t+2}^T: wait until P V_t has read it.
          if (!mbar_wait(&o_full[buf], u & 1, abort_flag)) break;
          ok = issue_qk(t + 2);
        }
      }
    }
  } else {
    // --------------------- softmax / correction / epilogue ---------------------
    const int row = warp * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    float o_acc[D];
#pragma unroll
    for (int c = 0; c < D; ++c) o_acc[c] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < n_kv; ++t) {
      const int buf = t & 1;
      const uint32_t u = uint32_t(t >> 1);
      if (!mbar_wait(&s_full[buf], u & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_tmem = tmem + uint32_t(buf * 128) + lane_off;
      const int key0 = t * Cfg::BN;
      const int valid = Tk - key0;  // keys in this tile that exist (may exceed 128)
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(s_tmem + uint32_t(c0), rr);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < valid) mx = fmaxf(mx, __uint_as_float(rr[e]));
      }
      const float m_new = fmaxf(m_run, mx * scale_log2);
      // pass 2: P = exp2(S*scale_log2 - m_new), packed to bf16 in place
      float rs = 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(s_tmem + uint32_t(c0), rr);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = (c0 + e < valid) ? exp2f(fmaf(__uint_as_float(rr[e]), scale_log2, -m_new)) : 0.f;
          float p1 = (c0 + e + 1 < valid) ? exp2f(fmaf(__uint_as_float(rr[e + 1]), scale_log2, -m_new)) : 0.f;
          rs += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st16(s_tmem + uint32_t(c0 >> 1), pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[buf]);
      const float alpha = (t == 0) ? 0.f : exp2f(m_run - m_new);
      if (t > 0) {
        const int pb = (t - 1) & 1;
        const uint32_t pu = uint32_t((t - 1) >> 1);
        if (!mbar_wait(&o_full[pb], pu & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t o_tmem = tmem + Cfg::O_COL + uint32_t(pb * D) + lane_off;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o_acc[c0 + e] = (o_acc[c0 + e] + __uint_as_float(rr[e])) * alpha;
        }
        tc_fence_before();
        mbar_arrive(&o_empty[pb]);
      }
      l_run = l_run * alpha + rs;
      m_run = m_new;
    }
    if (ok) {
      const int pb = (n_kv - 1) & 1;
      const uint32_t pu = uint32_t((n_kv - 1) >> 1);
      if (mbar_wait(&o_full[pb], pu & 1, abort_flag)) {
        tc_fence_after();
        const uint32_t o_tmem = tmem + Cfg::O_COL + uint32_t(pb * D) + lane_off;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + uint32_t(c0), rr);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o_acc[c0 + e] += __uint_as_float(rr[e]);
        }
        const int qi = q0 + row;
        if (qi < Tq) {
          const int64_t orow = int64_t(b) * Tq + qi;
          float g = 1.f;
          if (gate != nullptr) {
            const float lg = __bfloat162float(gate[orow * ld_gate + h]);
            const float sg = round_bf16(1.f / (1.f + expf(-lg)));
            g = round_bf16(2.f * sg);
          }
          const float inv_l = 1.f / l_run;
          __nv_bfloat16* op = O + orow * ldo + int64_t(h) * D;
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float o = round_bf16(o_acc[c0 + e] * inv_l);
              v[e] = gate != nullptr ? o * g : o;
            }
            st8<__nv_bfloat16>(op + c0, v);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 5) {
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

template <int D>
void launch_fmha_tc(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                    int64_t ldo, int B, int64_t Tq, int64_t Tk, int H, float scale, const void* gate,
                    int64_t ld_gate, cudaStream_t s) {
  using Cfg = FaCfg<D>;
  const uint64_t cols = uint64_t(H) * D;
  const CUtensorMap tq = make_tmap_bf16_2d(q, cols, uint64_t(B) * Tq, uint64_t(ldq), 64, 128);
  const CUtensorMap tk = make_tmap_bf16_2d(k, cols, uint64_t(B) * Tk, uint64_t(ldk), 64, 128);
  const CUtensorMap tv = make_tmap_bf16_2d(v, cols, uint64_t(B) * Tk, uint64_t(ldv), 64, 128);
  auto kern = fmha_tc_kernel<D>;
  static int attr_dev = -1;
  int dev = 0;
  LTX_CUDA(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    LTX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr_dev = dev;
  }
  dim3 grid(unsigned((Tq + 127) / 128), unsigned(H), unsigned(B));
  const float scale_log2 = scale * 1.4426950408889634f;
  kern<<<grid, 192, Cfg::SMEM, s>>>(tq, tk, tv, static_cast<__nv_bfloat16*>(o), ldo, int(Tq), int(Tk), scale_log2,
                                    static_cast<const __nv_bfloat16*>(gate), ld_gate), ltx::note_launch();
}

}  // namespace detail
}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

extern "C" int ltx_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                             void* o, int64_t ldo, int B, int64_t Tq, int64_t Tk, int heads, int head_dim,
                             float scale, const void* gate_logits, int64_t ld_gate, int dtype, void* stream) {
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
    if (head_dim == 64)
      launch_fmha_tc<64>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s);
    else
      launch_fmha_tc<128>(q, ldq, k, ldk, v, ldv, o, ldo, B, Tq, Tk, heads, scale, gate_logits, ld_gate, s);
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
