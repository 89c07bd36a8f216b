// Single-pass element-wise kernels of the DiT block: fused norm + adaLN modulation,
// q/k RMSNorm + split RoPE, GELU-tanh, gated residual, timestep sinusoid, RoPE tables
// and the X0 + CFG + Euler update.
//
// Each kernel reads its inputs once and writes its output once with 16-byte vector
// accesses (8 bf16 / 2x4 fp32 per access); row reductions stay in registers + one
// shared-memory exchange. Arithmetic is fp32; the storage dtype's rounding is applied
// at the points where the reference's op-by-op PyTorch code rounds (each torch op on a
// bf16 tensor returns a rounded bf16 tensor).
#include <algorithm>
#include <mutex>
#include <string>
#include <type_traits>

#include "ltx_kernels.cuh"

namespace ltx {
namespace detail {

constexpr int kMaxVecPerThread = 4;

// ---------------------------------------------------------------------------------
// y = norm(x) * (1 + scale) + shift          (ltx_dit.py:261,273,290,311,314,376-377)
// ---------------------------------------------------------------------------------
template <typename T, int NV>
__global__ void __launch_bounds__(1024) norm_modulate_kernel(const T* __restrict__ x, int64_t ldx, T* __restrict__ y,
                                                             int64_t ldy, int64_t rows_per_batch, int D, int kind,
                                                             float eps, ModVec<T> shift, ModVec<T> scale) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / rows_per_batch, t = row - b * rows_per_batch;
  const T* xr = x + row * ldx;
  T* yr = y + row * ldy;
  const int nvec = D >> 3;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      ld8<T>(xr + c * 8, v[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) s += (kind == LTX_NORM_LAYER) ? v[i][k] : v[i][k] * v[i][k];
    }
  }
  float mean = 0.f, rstd;
  if (kind == LTX_NORM_NONE) {
    rstd = 1.f;
  } else if (kind == LTX_NORM_LAYER) {
    mean = block_sum(s, red) / float(D);
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nvec) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = v[i][k] - mean;
          s2 += d * d;
        }
      }
    }
    rstd = rsqrtf(block_sum(s2, red) / float(D) + eps);
  } else {
    rstd = rsqrtf(block_sum(s, red) / float(D) + eps);
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      float o[8], sc[8], sh[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = round_to<T>((v[i][k] - mean) * rstd);
      if (scale.on) {
        scale.at8(b, t, c * 8, sc);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = round_to<T>(o[k] * round_to<T>(1.f + sc[k]));
      }
      if (shift.on) {
        shift.at8(b, t, c * 8, sh);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = o[k] + sh[k];
      }
      st8<T>(yr + c * 8, o);
    }
  }
}

// Fast path of the same op for bf16 rows of D = 256 * NC with per-sample (or no)
// modulation: one warp per row, no block-wide reduction. A CTA's rows all belong to
// one sample, so round(1 + scale) and round(shift) are built once per CTA in shared
// memory; a row then costs its load, its store and three bf16 roundings per element
// (two of them packed two to an instruction). Same rounding sequence as
// norm_modulate_kernel. KIND (ltx_norm_kind) is a template parameter so that RMSNorm
// carries no mean and LTX_NORM_NONE no normalisation; the products run as packed
// fp32x2 operations.
template <int NC, int KIND>
__global__ void __launch_bounds__(256) norm_rows_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                             __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                             int64_t rows, int64_t rows_per_batch,
                                                             int chunks_per_sample, int rows_per_chunk, float eps,
                                                             ModVec<__nv_bfloat16> shift, ModVec<__nv_bfloat16> scale) {
  constexpr int D = 256 * NC;
  __shared__ float s1p[D];  // round(1 + scale)
  __shared__ float shf[D];  // round(shift)
  const int64_t b = blockIdx.x / chunks_per_sample;
  const int chunk = int(blockIdx.x - b * chunks_per_sample);
  const int64_t r0 = b * rows_per_batch + int64_t(chunk) * rows_per_chunk;
  const int64_t r1 = min(min(r0 + rows_per_chunk, (b + 1) * rows_per_batch), rows);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  // The first row of each warp is loaded before the vectors are built, and every
  // later row one row ahead of its use.
  uint4 raw[NC];
  auto load_row = [&](int64_t r) {
    const __nv_bfloat16* xr = x + r * ldx;
#pragma unroll
    for (int i = 0; i < NC; ++i) raw[i] = *reinterpret_cast<const uint4*>(xr + (i * 32 + lane) * 8);
  };
  if (r0 + warp < r1) load_row(r0 + warp);
  for (int c8 = threadIdx.x; c8 < D / 8; c8 += blockDim.x) {
    float a[8];
    if (scale.on) {
      scale.at8(b, 0, c8 * 8, a);
#pragma unroll
      for (int k = 0; k < 8; ++k) s1p[c8 * 8 + k] = round_bf16(1.f + a[k]);
    }
    if (shift.on) {
      shift.at8(b, 0, c8 * 8, a);
#pragma unroll
      for (int k = 0; k < 8; ++k) shf[c8 * 8 + k] = a[k];
    }
  }
  __syncthreads();
  for (int64_t r = r0 + warp; r < r1; r += 8) {
    float v[NC][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      unpack_bf16x2(raw[i].x, v[i][0], v[i][1]);
      unpack_bf16x2(raw[i].y, v[i][2], v[i][3]);
      unpack_bf16x2(raw[i].z, v[i][4], v[i][5]);
      unpack_bf16x2(raw[i].w, v[i][6], v[i][7]);
#pragma unroll
      for (int k = 0; k < 8; ++k) s += (KIND == LTX_NORM_LAYER) ? v[i][k] : v[i][k] * v[i][k];
    }
    if (r + 8 < r1) load_row(r + 8);
    float mean = 0.f, rstd = 1.f;
    if constexpr (KIND == LTX_NORM_LAYER) {
      mean = warp_sum(s) / float(D);
      float s2 = 0.f;
#pragma unroll
      for (int i = 0; i < NC; ++i)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = v[i][k] - mean;
          s2 += d * d;
        }
      rstd = rsqrtf(warp_sum(s2) / float(D) + eps);
    } else if constexpr (KIND == LTX_NORM_RMS) {
      rstd = rsqrtf(warp_sum(s) / float(D) + eps);
    }
    const uint64_t r2 = f2_pack(rstd, rstd), m2 = f2_pack(mean, mean);
    __nv_bfloat16* yr = y + r * ldy;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = (i * 32 + lane) * 8;
      float o[8];
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        if constexpr (KIND == LTX_NORM_NONE) {
          o[k] = v[i][k];  // (v - 0) * 1, already bf16
          o[k + 1] = v[i][k + 1];
        } else {
          uint64_t t = f2_pack(v[i][k], v[i][k + 1]);
          if constexpr (KIND == LTX_NORM_LAYER) t = f2_sub(t, m2);
          f2_unpack(f2_mul(t, r2), o[k], o[k + 1]);
          round_bf16_pair(o[k], o[k + 1]);
        }
      }
      if (scale.on) {
        const float4 sa = *reinterpret_cast<const float4*>(&s1p[c]);
        const float4 sb = *reinterpret_cast<const float4*>(&s1p[c + 4]);
        const uint64_t s2v[4] = {f2_pack(sa.x, sa.y), f2_pack(sa.z, sa.w), f2_pack(sb.x, sb.y), f2_pack(sb.z, sb.w)};
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          f2_unpack(f2_mul(f2_pack(o[k], o[k + 1]), s2v[k >> 1]), o[k], o[k + 1]);
          round_bf16_pair(o[k], o[k + 1]);
        }
      }
      if (shift.on) {
        const float4 ha = *reinterpret_cast<const float4*>(&shf[c]);
        const float4 hb = *reinterpret_cast<const float4*>(&shf[c + 4]);
        const uint64_t h2v[4] = {f2_pack(ha.x, ha.y), f2_pack(ha.z, ha.w), f2_pack(hb.x, hb.y), f2_pack(hb.z, hb.w)};
#pragma unroll
        for (int k = 0; k < 8; k += 2) f2_unpack(f2_add(f2_pack(o[k], o[k + 1]), h2v[k >> 1]), o[k], o[k + 1]);
      }
      st8<__nv_bfloat16>(yr + c, o);
    }
  }
}

// ---------------------------------------------------------------------------------
// q/k RMSNorm over the whole inner dim (with weight) + split RoPE, in place
// (ltx_nn.py:186-187,214-218 and 99-115). Thread -> (head h, 8 pair indices j0..j0+7):
// it owns x[h*d + j] and its rotation partner x[h*d + d/2 + j].
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(1024) qk_norm_rope_kernel(T* __restrict__ x, int64_t ldx, int64_t rows_per_batch,
                                                            int heads, int d, const T* __restrict__ w, float eps,
                                                            const T* __restrict__ cos_t,
                                                            const T* __restrict__ sin_t, int64_t ld_rope,
                                                            int64_t rope_ld_batch) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / rows_per_batch, t = row - b * rows_per_batch;
  const int per_head = d >> 4;  // threads per head
  const int nthr = heads * per_head;
  const int D = heads * d;
  const bool active = threadIdx.x < nthr;
  const int h = threadIdx.x / per_head;
  const int j0 = (threadIdx.x % per_head) * 8;
  const int c1 = h * d + j0, c2 = c1 + (d >> 1);
  T* xr = x + row * ldx;
  float a[8], bb[8];
  float s = 0.f;
  if (active) {
    ld8<T>(xr + c1, a);
    ld8<T>(xr + c2, bb);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += a[k] * a[k] + bb[k] * bb[k];
  }
  const float ss = block_sum(s, red);
  if (!active) return;
  if (w != nullptr) {  // NULL weight: rotation only
    const float rstd = rsqrtf(ss / float(D) + eps);
    float w1[8], w2[8];
    ld8<T>(w + c1, w1);
    ld8<T>(w + c2, w2);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      a[k] = round_to<T>(a[k] * rstd * w1[k]);
      bb[k] = round_to<T>(bb[k] * rstd * w2[k]);
    }
  }
  if (cos_t != nullptr) {
    const int64_t ro = b * rope_ld_batch + t * ld_rope + h * (d >> 1) + j0;
    float cs[8], sn[8];
    ld8<T>(cos_t + ro, cs);
    ld8<T>(sin_t + ro, sn);
    float o1[8], o2[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // first*c - second*s ; second*c + first*s, each product rounded like the
      // reference's separate torch ops (no fused multiply-add).
      o1[k] = round_to<T>(__fsub_rn(round_to<T>(__fmul_rn(a[k], cs[k])), round_to<T>(__fmul_rn(bb[k], sn[k]))));
      o2[k] = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(bb[k], cs[k])), round_to<T>(__fmul_rn(a[k], sn[k]))));
    }
    st8<T>(xr + c1, o1);
    st8<T>(xr + c2, o2);
  } else {
    st8<T>(xr + c1, a);
    st8<T>(xr + c2, bb);
  }
}

// Destinations of the sequence-parallel exchange fused into the self-attention q/k pass
// (ltx_qk_norm_rope_scatter): row t of sample b of this rank's tokens goes to row
// b * t_full + row0 + t of every SP rank's receive buffer, which holds
// [q | k | v | gate logits] of that rank's hp heads (widths dp, dp, dp, hp).
struct SpScatter {
  __nv_bfloat16* dst[8];  // receive buffer of SP rank j, as mapped in this process
  int64_t ld, t_full, row0;
  int hp, dp, v_off, gate_off;  // gate_off < 0: no gate logits
};

// Fast path of the same op for bf16: one warp per row, NI slots of (head, 8 pairs) per
// lane, no block-wide reduction, the roundings done two to a packed conversion. Same
// rounding sequence as above. Rows stay packed in registers between the sum-of-squares
// pass and the output pass, which keeps enough warps resident to cover the load
// latency. SCATTER: the rows are not written back but sent, with the row's v and gate
// logits, to the SP ranks' receive buffers (SpScatter).
template <int NI, bool SCATTER = false>
__global__ void __launch_bounds__(256, 2) qk_rows_bf16_kernel(__nv_bfloat16* __restrict__ x, int64_t ldx, int64_t rows,
                                                           int64_t rows_per_batch, int rows_per_cta, int d,
                                                           const __nv_bfloat16* __restrict__ w, float eps,
                                                           const __nv_bfloat16* __restrict__ cos_t,
                                                           const __nv_bfloat16* __restrict__ sin_t, int64_t ld_rope,
                                                           int64_t rope_ld_batch, const __nv_bfloat16* __restrict__ w2,
                                                           int64_t off2, const SpScatter sc) {
  // w2 != nullptr: a second column block at off2 (self-attention k) is normalised with
  // w2 and rotated with the same RoPE entries, which are loaded once per row.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = int64_t(blockIdx.x) * rows_per_cta;
  const int64_t r1 = min(r0 + rows_per_cta, rows);
  const int per_head = d >> 4;
  const float inv_D = 1.f / float(32 * NI * 16);
  const int n_parts = w2 != nullptr ? 2 : 1;
  pdl_wait();
  pdl_trigger();
  for (int64_t r = r0 + warp; r < r1; r += 8) {
    const int64_t b = r / rows_per_batch, t = r - b * rows_per_batch;
    const int64_t ro = b * rope_ld_batch + t * ld_rope;
    uint4 ra[NI], rb[NI], rc[NI], rs[NI];
    if (cos_t != nullptr) {
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int u = i * 32 + lane;
        const int h = u / per_head, j0 = (u - h * per_head) * 8;
        rc[i] = *reinterpret_cast<const uint4*>(cos_t + ro + h * (d >> 1) + j0);
        rs[i] = *reinterpret_cast<const uint4*>(sin_t + ro + h * (d >> 1) + j0);
      }
    }
    const int64_t drow = SCATTER ? b * sc.t_full + sc.row0 + t : 0;  // row in the receive buffers
    // destination of (head h, column c within the head) of column block `part`
    auto dst_of = [&](int part, int h, int c) -> __nv_bfloat16* {
      const int j = h / sc.hp;
      return sc.dst[j] + drow * sc.ld + part * sc.dp + (h - j * sc.hp) * d + c;
    };
    for (int part = 0; part < n_parts; ++part) {
    __nv_bfloat16* xr = x + r * ldx + (part ? off2 : 0);
    const __nv_bfloat16* wp = part ? w2 : w;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int u = i * 32 + lane;
      const int h = u / per_head, j0 = (u - h * per_head) * 8;
      ra[i] = *reinterpret_cast<const uint4*>(xr + h * d + j0);
      rb[i] = *reinterpret_cast<const uint4*>(xr + h * d + j0 + (d >> 1));
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&ra[i]);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&rb[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a0, a1, b0, b1;
        unpack_bf16x2(pa[k], a0, a1);
        unpack_bf16x2(pb[k], b0, b1);
        s += a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1;
      }
    }
    const float rstd = rsqrtf(warp_sum(s) * inv_D + eps);
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int u = i * 32 + lane;
      const int h = u / per_head, j0 = (u - h * per_head) * 8;
      const int c1 = h * d + j0;
      float a[8], bb[8];
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&ra[i]);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&rb[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        unpack_bf16x2(pa[k], a[2 * k], a[2 * k + 1]);
        unpack_bf16x2(pb[k], bb[2 * k], bb[2 * k + 1]);
      }
      if (wp != nullptr) {
        float wa[8], wb[8];
        ld8<__nv_bfloat16>(wp + c1, wa);
        ld8<__nv_bfloat16>(wp + c1 + (d >> 1), wb);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          a[k] = a[k] * rstd * wa[k];
          bb[k] = bb[k] * rstd * wb[k];
          round_bf16_pair(a[k], bb[k]);
        }
      }
      if (cos_t != nullptr) {
        float cs[8], sn[8], o1[8], o2[8];
        const uint32_t* pc = reinterpret_cast<const uint32_t*>(&rc[i]);
        const uint32_t* ps = reinterpret_cast<const uint32_t*>(&rs[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          unpack_bf16x2(pc[k], cs[2 * k], cs[2 * k + 1]);
          unpack_bf16x2(ps[k], sn[2 * k], sn[2 * k + 1]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // first*c - second*s ; second*c + first*s, each product rounded (no FMA)
          float p1 = __fmul_rn(a[k], cs[k]), p2 = __fmul_rn(bb[k], sn[k]);
          float p3 = __fmul_rn(bb[k], cs[k]), p4 = __fmul_rn(a[k], sn[k]);
          round_bf16_pair(p1, p2);
          round_bf16_pair(p3, p4);
          o1[k] = __fsub_rn(p1, p2);
          o2[k] = __fadd_rn(p3, p4);
        }
        if constexpr (SCATTER) {
          st8<__nv_bfloat16>(dst_of(part, h, j0), o1);
          st8<__nv_bfloat16>(dst_of(part, h, j0 + (d >> 1)), o2);
        } else {
          st8<__nv_bfloat16>(xr + c1, o1);
          st8<__nv_bfloat16>(xr + c1 + (d >> 1), o2);
        }
      } else {
        if constexpr (SCATTER) {
          st8<__nv_bfloat16>(dst_of(part, h, j0), a);
          st8<__nv_bfloat16>(dst_of(part, h, j0 + (d >> 1)), bb);
        } else {
          st8<__nv_bfloat16>(xr + c1, a);
          st8<__nv_bfloat16>(xr + c1 + (d >> 1), bb);
        }
      }
    }
    }
    if constexpr (SCATTER) {
      // v and the gate logits of the row, unchanged, to the owners of their heads
      const int D = 32 * NI * 16;
      const __nv_bfloat16* xv = x + r * ldx + sc.v_off;
      for (int u = lane; u < D / 8; u += 32) {
        const int h = (u * 8) / d, c = u * 8 - h * d;
        *reinterpret_cast<uint4*>(dst_of(2, h, c)) = *reinterpret_cast<const uint4*>(xv + u * 8);
      }
      if (sc.gate_off >= 0) {
        const int heads = D / d;
        for (int h = lane; h < heads; h += 32) {
          const int j = h / sc.hp;
          sc.dst[j][drow * sc.ld + 3 * sc.dp + (h - j * sc.hp)] = x[r * ldx + sc.gate_off + h];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// RoPE tables (ltx_nn.py:80-96): column c of (T, dim/2): c < pad -> (1, 0); else
// k = c - pad, f = k / n_axes, axis = k % n_axes, mid = (start + end) / 2 of the
// token's bounds on that axis, angle = freqs[f] * ((mid / max_pos[axis]) * 2 - 1).
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void rope_tables_kernel(const float* __restrict__ bounds, int n_axes, int64_t T_, const float* __restrict__ freqs,
                                   int n_freq, const float* __restrict__ max_pos, int half, T* __restrict__ cos_o,
                                   T* __restrict__ sin_o) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T_ * half) return;
  const int64_t t = i / half;
  const int c = int(i - t * half);
  const int pad = half - n_freq * n_axes;
  float cv = 1.f, sv = 0.f;
  if (c >= pad) {
    const int k = c - pad;
    const int f = k / n_axes, axis = k - (k / n_axes) * n_axes;
    const float* bt = bounds + (int64_t(axis) * T_ + t) * 2;
    const float mid = __fdiv_rn(__fadd_rn(bt[0], bt[1]), 2.f);
    const float frac = __fdiv_rn(mid, max_pos[axis]);
    const float ang = __fmul_rn(freqs[f], __fsub_rn(__fmul_rn(frac, 2.f), 1.f));
    cv = cosf(ang);
    sv = sinf(ang);
  }
  st_elem<T>(cos_o + i, cv);
  st_elem<T>(sin_o + i, sv);
}

// ---------------------------------------------------------------------------------
// GELU-tanh (ltx_nn.py:248)
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void gelu_tanh_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  const int64_t nv = n >> 3;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float v[8];
    ld8<T>(x + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = gelu_tanh_f(v[k]);
    st8<T>(y + i * 8, v);
  }
  // tail (n % 8)
  const int64_t tail0 = nv * 8;
  const int64_t i = tail0 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n && i < tail0 + 8) st_elem<T>(y + i, gelu_tanh_f(ld_elem<T>(x + i)));
}

// ---------------------------------------------------------------------------------
// out = x + round(y * gate)              (ltx_dit.py:265,277,311,314)
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void gate_residual_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ y, int64_t ldy,
                                     T* __restrict__ out, int64_t ldo, int64_t rows, int64_t rows_per_batch, int D,
                                     ModVec<T> gate) {
  const int nvr = D >> 3;
  const int64_t total = rows * nvr;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t row = i / nvr;
    const int c = int(i - row * nvr) * 8;
    const int64_t b = row / rows_per_batch, t = row - b * rows_per_batch;
    float xv[8], yv[8], g[8];
    ld8<T>(x + row * ldx + c, xv);
    ld8<T>(y + row * ldy + c, yv);
    if (gate.on) {
      gate.at8(b, t, c, g);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) g[k] = 1.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) xv[k] = xv[k] + round_to<T>(yv[k] * g[k]);
    st8<T>(out + row * ldo + c, xv);
  }
}

// ---------------------------------------------------------------------------------
// Timestep sinusoid [cos, sin] (standalone/common.py:138-148), argument t*scale.
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void timestep_embedding_kernel(const float* __restrict__ tv, int64_t n, float scale, int dim,
                                          float log_max_period, T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * dim) return;
  const int64_t r = i / dim;
  const int c = int(i - r * dim);
  const int half = dim >> 1;
  float v = 0.f;  // odd-dim pad column
  if (c < 2 * half) {
    const int j = c < half ? c : c - half;
    const float f = expf(__fdiv_rn(__fmul_rn(-log_max_period, float(j)), float(half)));
    const float arg = __fmul_rn(__fmul_rn(tv[r], scale), f);
    v = c < half ? cosf(arg) : sinf(arg);
  }
  st_elem<T>(out + i, v);
}

// ---------------------------------------------------------------------------------
// X0 + CFG guide + Euler (ltx_dit.py:591-593, 551-562 with rescale 0, 602-606).
// vel rows [0, T) are the cond pass, [T, 2T) the uncond pass of the same latent.
// ---------------------------------------------------------------------------------
template <typename T>
LTX_DEVICE void cfg_euler_point(float vc, float vu, float lat, float tsc, float tsu, float cfg_m1, float sigma,
                                float dt, float& den, float& nxt) {
  // x0 = (latent - v * timesteps).to(dtype)
  const float x0c = round_to<T>(__fsub_rn(lat, __fmul_rn(vc, tsc)));
  const float x0u = round_to<T>(__fsub_rn(lat, __fmul_rn(vu, tsu)));
  // pred = cond + (cfg - 1) * (cond - uncond), then .to(dtype)
  den = round_to<T>(__fadd_rn(x0c, __fmul_rn(cfg_m1, __fsub_rn(x0c, x0u))));
  // velocity = ((sample - denoised) / sigma).to(dtype); sample + velocity * dt
  const float vel = round_to<T>(__fdiv_rn(__fsub_rn(lat, den), sigma));
  nxt = round_to<T>(__fadd_rn(lat, __fmul_rn(vel, dt)));
}

template <typename T>
__global__ void cfg_euler_kernel(const T* __restrict__ vel, const T* __restrict__ latent, const float* __restrict__ ts,
                                 int64_t T_, int C, float cfg_m1, float sigma, float dt, T* __restrict__ denoised,
                                 T* __restrict__ new_latent) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n = T_ * C;
  if (i >= n) return;
  const int64_t t = i / C;
  float den, nxt;
  cfg_euler_point<T>(ld_elem<T>(vel + i), ld_elem<T>(vel + n + i), ld_elem<T>(latent + i), ts[t], ts[T_ + t], cfg_m1,
                     sigma, dt, den, nxt);
  if (denoised) st_elem<T>(denoised + i, den);
  st_elem<T>(new_latent + i, nxt);
}

// pred = c + (cfg-1)(c-u) + stg(c-p) + (mod-1)(c-m), evaluated left to right in fp32 and
// rounded once, like the reference's fp32 tensor expression (ltx_dit.py:552-557).
template <typename T>
__global__ void guide_kernel(const T* __restrict__ c, const T* __restrict__ u, const T* __restrict__ p,
                             const T* __restrict__ m, int64_t n, float cfg_m1, float stg, float mod_m1,
                             T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float cv = ld_elem<T>(c + i);
  float r = __fadd_rn(cv, __fmul_rn(cfg_m1, __fsub_rn(cv, ld_elem<T>(u + i))));
  r = __fadd_rn(r, __fmul_rn(stg, __fsub_rn(cv, ld_elem<T>(p + i))));
  r = __fadd_rn(r, __fmul_rn(mod_m1, __fsub_rn(cv, ld_elem<T>(m + i))));
  st_elem<T>(out + i, r);
}

// Guidance with std rescale (ltx_dit.py:558-561): factor = rescale * std(cond) / std(pred)
// + (1 - rescale) over all n elements (unbiased), out = round(pred * factor).
// Pass 1 (guide_stats_kernel): each block accumulates sum and sum of squares of cond
// and pred in double and writes them to its slot of the workspace; the last block to
// finish (completion counter in the workspace) adds the slots in block order, so the
// result does not depend on scheduling, stores the factor and resets the counter to 0.
// Pass 2 (guide_scale_kernel) recomputes pred and scales it.
struct GuideWs {
  unsigned int counter;  // blocks of pass 1 finished; 0 between calls
  float factor;
  double pad;            // keeps the partials 16-byte aligned
  // double partials[blocks][4] follow
};
constexpr int kGuideThreads = 256;
constexpr int64_t kGuideElemsPerBlock = 4096;
constexpr int kGuideMaxBlocks = 1024;

inline int guide_rescale_blocks(int64_t n) {
  return int(std::min<int64_t>(kGuideMaxBlocks, std::max<int64_t>(1, (n + kGuideElemsPerBlock - 1) / kGuideElemsPerBlock)));
}
inline size_t guide_rescale_ws_bytes(int64_t n) {
  return sizeof(GuideWs) + size_t(guide_rescale_blocks(n)) * 4 * sizeof(double);
}

template <typename T>
LTX_DEVICE float guide_pred(const T* c, const T* u, const T* p, const T* m, int64_t i, float cfg_m1, float stg,
                            float mod_m1, float& cv) {
  cv = ld_elem<T>(c + i);
  float r = __fadd_rn(cv, __fmul_rn(cfg_m1, __fsub_rn(cv, ld_elem<T>(u + i))));
  r = __fadd_rn(r, __fmul_rn(stg, __fsub_rn(cv, ld_elem<T>(p + i))));
  return __fadd_rn(r, __fmul_rn(mod_m1, __fsub_rn(cv, ld_elem<T>(m + i))));
}

LTX_DEVICE double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = (lane < int(blockDim.x >> 5)) ? red[lane] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

template <typename T>
__global__ void __launch_bounds__(kGuideThreads) guide_stats_kernel(const T* __restrict__ c, const T* __restrict__ u,
                                                                    const T* __restrict__ p, const T* __restrict__ m,
                                                                    int64_t n, float cfg_m1, float stg, float mod_m1,
                                                                    float rescale, GuideWs* __restrict__ ws) {
  __shared__ double red[kGuideThreads / 32];
  __shared__ bool last;
  double* parts = reinterpret_cast<double*>(ws + 1);
  double a[4] = {0.0, 0.0, 0.0, 0.0};  // sum c, sum c^2, sum pred, sum pred^2
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    float cv;
    const float pv = guide_pred<T>(c, u, p, m, i, cfg_m1, stg, mod_m1, cv);
    a[0] += double(cv);
    a[1] += double(cv) * double(cv);
    a[2] += double(pv);
    a[3] += double(pv) * double(pv);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const double t = block_sum_d(a[k], red);
    if (threadIdx.x == 0) parts[blockIdx.x * 4 + k] = t;
  }
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(&ws->counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double s[4] = {0.0, 0.0, 0.0, 0.0};
    for (unsigned b = 0; b < gridDim.x; ++b)
#pragma unroll
      for (int k = 0; k < 4; ++k) s[k] += reinterpret_cast<volatile double*>(parts)[b * 4 + k];
    const double nn = double(n);
    const double var_c = (s[1] - s[0] * s[0] / nn) / (nn - 1.0);
    const double var_p = (s[3] - s[2] * s[2] / nn) / (nn - 1.0);
    const float ratio = float(sqrt(fmax(var_c, 0.0)) / sqrt(fmax(var_p, 0.0)));
    ws->factor = __fadd_rn(__fmul_rn(rescale, ratio), 1.f - rescale);
    ws->counter = 0u;
  }
}

template <typename T>
__global__ void guide_scale_kernel(const T* __restrict__ c, const T* __restrict__ u, const T* __restrict__ p,
                                   const T* __restrict__ m, int64_t n, float cfg_m1, float stg, float mod_m1,
                                   const GuideWs* __restrict__ ws, T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float cv;
  const float pv = guide_pred<T>(c, u, p, m, i, cfg_m1, stg, mod_m1, cv);
  st_elem<T>(out + i, __fmul_rn(pv, ws->factor));
}

template <typename T>
void launch_guide_rescale(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n,
                          float cfg_m1, float stg, float mod_m1, float rescale, void* out, GuideWs* ws,
                          cudaStream_t s) {
  auto c = static_cast<const T*>(cond);
  auto u = static_cast<const T*>(uncond);
  auto p = static_cast<const T*>(ptb);
  auto m = static_cast<const T*>(mod);
  guide_stats_kernel<T><<<unsigned(guide_rescale_blocks(n)), kGuideThreads, 0, s>>>(c, u, p, m, n, cfg_m1, stg,
                                                                                   mod_m1, rescale, ws),
      ltx::note_launch();
  guide_scale_kernel<T><<<unsigned((n + 255) / 256), 256, 0, s>>>(c, u, p, m, n, cfg_m1, stg, mod_m1, ws,
                                                                  static_cast<T*>(out)),
      ltx::note_launch();
}

// Learnable-register fill of the text connector (ltx_te.py:218-223): a token whose
// additive mask is negative (padding) is replaced by register row (token % R); the
// reference's blend binary*h + (1-binary)*regs with binary in {0, 1} is this selection.
template <typename T>
__global__ void register_fill_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ mask,
                                     const T* __restrict__ regs, int R, int64_t rows, int64_t S, int D,
                                     T* __restrict__ out, int64_t ldo) {
  const int per_row = D / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * per_row) return;
  const int64_t r = i / per_row;
  const int c = int(i - r * per_row) * 8;
  const bool keep = ld_elem<T>(mask + r) >= 0.f;
  const T* src = keep ? x + r * ldx + c : regs + int64_t((r % S) % R) * D + c;
  float v[8];
  ld8<T>(src, v);
  st8<T>(out + r * ldo + c, v);
}

// X0 from a velocity (ltx_dit.py:591-593): out = round(latent - v * timesteps[row]).
template <typename T>
__global__ void x0_kernel(const T* __restrict__ latent, const T* __restrict__ vel, const float* __restrict__ ts,
                          int64_t rows, int C, T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * C) return;
  st_elem<T>(out + i, __fsub_rn(ld_elem<T>(latent + i), __fmul_rn(ld_elem<T>(vel + i), ts[i / C])));
}

// velocity = round((sample - denoised) / sigma); out = round(sample + velocity * dt).
template <typename T>
__global__ void euler_kernel(const T* __restrict__ s, const T* __restrict__ d, int64_t n, float sigma, float dt,
                             T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float sv = ld_elem<T>(s + i);
  const float vel = round_to<T>(__fdiv_rn(__fsub_rn(sv, ld_elem<T>(d + i)), sigma));
  st_elem<T>(out + i, __fadd_rn(sv, __fmul_rn(vel, dt)));
}

// ---------------------------------------------------------------------------------
// Sequence-parallel exchange layouts (all-to-all send / receive buffers).
// pack:   dst[j][r][:] = concat over segments s of src[r][off_s + j*w_s : off_s + (j+1)*w_s]
// unpack: dst[r][j*w : (j+1)*w] = src[j][r][:]
// One thread moves 8 consecutive elements (16 bytes of bf16).
// ---------------------------------------------------------------------------------
struct SpSegments {
  int n;
  int off[4];
  int w[4];
  int W;  // sum of w
};

__global__ void sp_pack_kernel(const uint4* __restrict__ src, int64_t ld_src8, int64_t rows, int parts, SpSegments seg,
                               uint4* __restrict__ dst) {
  const int W8 = seg.W >> 3;
  const int64_t total = int64_t(parts) * rows * W8;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  pdl_wait();
  pdl_trigger();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t j = i / (rows * W8);
    const int64_t rem = i - j * rows * W8;
    const int64_t r = rem / W8;
    int c8 = int(rem - r * W8);
    int s = 0;
    while (c8 >= (seg.w[s] >> 3)) {
      c8 -= seg.w[s] >> 3;
      ++s;
    }
    dst[i] = src[r * ld_src8 + ((seg.off[s] + int(j) * seg.w[s]) >> 3) + c8];
  }
}

__global__ void sp_unpack_kernel(const uint4* __restrict__ src, int64_t rows, int parts, int w8,
                                 uint4* __restrict__ dst, int64_t ld_dst8) {
  const int64_t total = int64_t(parts) * rows * w8;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  pdl_wait();
  pdl_trigger();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / (int64_t(parts) * w8);
    const int64_t rem = i - r * parts * w8;
    const int64_t j = rem / w8;
    const int64_t c8 = rem - j * w8;
    dst[r * ld_dst8 + j * w8 + c8] = src[(j * rows + r) * w8 + c8];
  }
}

inline unsigned grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return unsigned(g);
}

template <typename T>
void launch_norm_modulate(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int64_t rpb, int D, int kind,
                          float eps, const ltx_modulation* m, cudaStream_t s) {
  const int nvec = D / 8;
  int threads = ((nvec + 31) / 32) * 32;
  int nv = 1;
  while (threads > 1024 && nv < kMaxVecPerThread) {
    ++nv;
    threads = (((nvec + nv - 1) / nv + 31) / 32) * 32;
  }
  LTX_UNSUPPORTED(threads <= 1024, "D too large for norm_modulate");
  ModVec<T> sh = make_modvec<T>(m, 0), sc = make_modvec<T>(m, 1);
  auto xp = static_cast<const T*>(x);
  auto yp = static_cast<T*>(y);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const bool per_sample = (!sh.on || sh.mod == nullptr || sh.ldt == 0) && (!sc.on || sc.mod == nullptr || sc.ldt == 0);
    const int nc = D / 256;
    if (per_sample && D % 256 == 0 && nc >= 1 && nc <= 8 && (rows % rpb == 0 || rows <= rpb)) {
      // two resident CTAs per SM, each streaming an even share of one sample's rows
      const int64_t target = int64_t(num_sms()) * 2;
      const int64_t n_samples = (rows + rpb - 1) / rpb;
      int64_t per = std::max<int64_t>(8, (rows + target - 1) / target);
      per = std::min<int64_t>(per, std::min<int64_t>(rpb, rows));
      const int64_t chunks = (std::min<int64_t>(rpb, rows) + per - 1) / per;
      const unsigned grid = unsigned(n_samples * chunks);
#define LTX_NORM_ROWS_K(NCV, KV)                                                                             \
  launch_pdl(norm_rows_bf16_kernel<NCV, KV>, dim3(grid), dim3(256), 0, s, 1, xp, ldx, yp, ldy, rows, rpb, int(chunks), \
             int(per), eps, sh, sc)
#define LTX_NORM_ROWS(NCV)                                                                 \
  (kind == LTX_NORM_LAYER ? LTX_NORM_ROWS_K(NCV, LTX_NORM_LAYER)                           \
                          : kind == LTX_NORM_NONE ? LTX_NORM_ROWS_K(NCV, LTX_NORM_NONE)     \
                                                  : LTX_NORM_ROWS_K(NCV, LTX_NORM_RMS))
      switch (nc) {
        case 1: LTX_NORM_ROWS(1); break;
        case 2: LTX_NORM_ROWS(2); break;
        case 3: LTX_NORM_ROWS(3); break;
        case 4: LTX_NORM_ROWS(4); break;
        case 5: LTX_NORM_ROWS(5); break;
        case 6: LTX_NORM_ROWS(6); break;
        case 7: LTX_NORM_ROWS(7); break;
        default: LTX_NORM_ROWS(8); break;
      }
#undef LTX_NORM_ROWS
#undef LTX_NORM_ROWS_K
      return;
    }
  }
  switch (nv) {
    case 1: norm_modulate_kernel<T, 1><<<unsigned(rows), threads, 0, s>>>(xp, ldx, yp, ldy, rpb, D, kind, eps, sh, sc), ltx::note_launch(); break;
    case 2: norm_modulate_kernel<T, 2><<<unsigned(rows), threads, 0, s>>>(xp, ldx, yp, ldy, rpb, D, kind, eps, sh, sc), ltx::note_launch(); break;
    case 3: norm_modulate_kernel<T, 3><<<unsigned(rows), threads, 0, s>>>(xp, ldx, yp, ldy, rpb, D, kind, eps, sh, sc), ltx::note_launch(); break;
    default: norm_modulate_kernel<T, 4><<<unsigned(rows), threads, 0, s>>>(xp, ldx, yp, ldy, rpb, D, kind, eps, sh, sc), ltx::note_launch(); break;
  }
}

}  // namespace detail
}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

#define LTX_CHECK_DTYPE(dt) LTX_REQUIRE((dt) == LTX_F32 || (dt) == LTX_BF16, "dtype must be F32 or BF16")

extern "C" int ltx_norm_modulate(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows,
                                 int64_t rows_per_batch, int D, int norm_kind, float eps, const ltx_modulation* mod,
                                 int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(x && y, "x and y must be non-NULL");
  LTX_REQUIRE(rows > 0 && rows < (int64_t(1) << 31), "rows out of range");
  LTX_REQUIRE(D > 0 && D % 8 == 0, "D must be a positive multiple of 8");
  LTX_REQUIRE(ldx % 8 == 0 && ldy % 8 == 0 && ldx >= D && ldy >= D, "ldx/ldy must be multiples of 8 and >= D");
  LTX_REQUIRE(rows_per_batch > 0, "rows_per_batch must be positive");
  LTX_REQUIRE(norm_kind == LTX_NORM_RMS || norm_kind == LTX_NORM_LAYER || norm_kind == LTX_NORM_NONE, "bad norm_kind");
  check_vec_ptr(x, "x");
  check_vec_ptr(y, "y");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_F32)
    launch_norm_modulate<float>(x, ldx, y, ldy, rows, rows_per_batch, D, norm_kind, eps, mod, s);
  else
    launch_norm_modulate<__nv_bfloat16>(x, ldx, y, ldy, rows, rows_per_batch, D, norm_kind, eps, mod, s);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_qk_norm_rope(void* x, int64_t ldx, int64_t rows, int64_t rows_per_batch, int heads, int head_dim,
                                const void* weight, float eps, const void* cos_tab, const void* sin_tab,
                                int64_t ld_rope, int64_t rope_ld_batch, int dtype, void* stream);

extern "C" int ltx_qk_norm_rope_pair(void* x, int64_t ldx, int64_t k_offset, int64_t rows, int64_t rows_per_batch,
                                     int heads, int head_dim, const void* q_weight, const void* k_weight, float eps,
                                     const void* cos_tab, const void* sin_tab, int64_t ld_rope, int64_t rope_ld_batch,
                                     int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x != nullptr && q_weight != nullptr && k_weight != nullptr, "x and both weights must be non-NULL");
  LTX_REQUIRE(k_offset % 8 == 0 && k_offset >= int64_t(heads) * head_dim, "k_offset must be a multiple of 8 past q");
  LTX_REQUIRE(ldx >= k_offset + int64_t(heads) * head_dim, "ldx too small for the k block");
  const int nthr = heads * (head_dim / 16);
  const bool fast = dtype == LTX_BF16 && head_dim % 16 == 0 && (nthr % 32) == 0 && nthr / 32 <= 4 && ldx % 8 == 0 &&
                    rows > 0 && rows_per_batch > 0 && (cos_tab == nullptr) == (sin_tab == nullptr) &&
                    (cos_tab == nullptr || (ld_rope % 8 == 0 && rope_ld_batch % 8 == 0));
  if (!fast) {
    // generic: the two blocks one after the other
    char* xb = static_cast<char*>(x);
    const size_t es = dtype == LTX_F32 ? 4 : 2;
    int st = ltx_qk_norm_rope(x, ldx, rows, rows_per_batch, heads, head_dim, q_weight, eps, cos_tab, sin_tab, ld_rope,
                              rope_ld_batch, dtype, stream);
    if (st != LTX_OK) return st;
    return ltx_qk_norm_rope(xb + k_offset * es, ldx, rows, rows_per_batch, heads, head_dim, k_weight, eps, cos_tab,
                            sin_tab, ld_rope, rope_ld_batch, dtype, stream);
  }
  check_vec_ptr(x, "x");
  check_vec_ptr(q_weight, "q_weight");
  check_vec_ptr(k_weight, "k_weight");
  check_vec_ptr(cos_tab, "cos");
  check_vec_ptr(sin_tab, "sin");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ni = nthr / 32;
  const int64_t target = int64_t(num_sms()) * 2;
  const int per = int(std::max<int64_t>(8, (rows + target - 1) / target));
  const unsigned grid = unsigned((rows + per - 1) / per);
  auto xb = static_cast<__nv_bfloat16*>(x);
  auto wq = static_cast<const __nv_bfloat16*>(q_weight);
  auto wk = static_cast<const __nv_bfloat16*>(k_weight);
  auto cb = static_cast<const __nv_bfloat16*>(cos_tab);
  auto sb = static_cast<const __nv_bfloat16*>(sin_tab);
#define LTX_QK_PAIR(NIV)                                                                                           \
  launch_pdl(qk_rows_bf16_kernel<NIV, false>, dim3(grid), dim3(256), 0, s, 1, xb, ldx, rows, rows_per_batch, per, \
             head_dim, wq, eps, cb, sb, ld_rope, rope_ld_batch, wk, k_offset, SpScatter{})
  switch (ni) {
    case 1: LTX_QK_PAIR(1); break;
    case 2: LTX_QK_PAIR(2); break;
    case 3: LTX_QK_PAIR(3); break;
    default: LTX_QK_PAIR(4); break;
  }
#undef LTX_QK_PAIR
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_qk_norm_rope_scatter(const void* x, int64_t ldx, int64_t rows, int64_t rows_per_batch, int heads,
                                        int head_dim, const void* q_weight, const void* k_weight, float eps,
                                        const void* cos_tab, const void* sin_tab, int64_t ld_rope,
                                        int64_t rope_ld_batch, int gated, int parts, int sp_rank,
                                        void* const* dst, int64_t ld_dst, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x != nullptr && q_weight != nullptr && k_weight != nullptr && dst != nullptr, "NULL argument");
  LTX_REQUIRE(parts >= 1 && parts <= 8 && sp_rank >= 0 && sp_rank < parts, "parts must be 1..8 and sp_rank < parts");
  LTX_REQUIRE(heads % parts == 0, "heads must split evenly over the SP ranks");
  const int nthr = heads * (head_dim / 16);
  LTX_UNSUPPORTED(head_dim % 16 == 0 && nthr % 32 == 0 && nthr / 32 <= 4,
                  "the fused exchange needs heads * head_dim / 16 a multiple of 32, at most 128");
  LTX_REQUIRE(rows > 0 && rows_per_batch > 0 && rows % rows_per_batch == 0, "rows must be whole samples");
  LTX_REQUIRE((cos_tab == nullptr) == (sin_tab == nullptr), "cos and sin go together");
  const int64_t D = int64_t(heads) * head_dim;
  const int hp = heads / parts, dp = hp * head_dim;
  LTX_REQUIRE(ldx % 8 == 0 && ldx >= 3 * D + (gated ? heads : 0), "ldx too small for q, k, v (and gate logits)");
  LTX_REQUIRE(dp % 8 == 0 && ld_dst % 8 == 0 && ld_dst >= 3 * dp + (gated ? hp : 0), "bad receive-buffer row");
  LTX_REQUIRE(cos_tab == nullptr || (ld_rope % 8 == 0 && rope_ld_batch % 8 == 0), "RoPE strides must be multiples of 8");
  check_vec_ptr(x, "x");
  check_vec_ptr(q_weight, "q_weight");
  check_vec_ptr(k_weight, "k_weight");
  check_vec_ptr(cos_tab, "cos");
  check_vec_ptr(sin_tab, "sin");
  SpScatter sc{};
  for (int j = 0; j < parts; ++j) {
    LTX_REQUIRE(dst[j] != nullptr, "dst[j] is NULL");
    check_vec_ptr(dst[j], "dst[j]");
    sc.dst[j] = static_cast<__nv_bfloat16*>(dst[j]);
  }
  sc.ld = ld_dst;
  sc.t_full = rows_per_batch * parts;
  sc.row0 = int64_t(sp_rank) * rows_per_batch;
  sc.hp = hp;
  sc.dp = dp;
  sc.v_off = int(2 * D);
  sc.gate_off = gated ? int(3 * D) : -1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ni = nthr / 32;
  const int64_t target = int64_t(num_sms()) * 2;
  const int per = int(std::max<int64_t>(8, (rows + target - 1) / target));
  const unsigned grid = unsigned((rows + per - 1) / per);
  auto xb = static_cast<__nv_bfloat16*>(const_cast<void*>(x));
  auto wq = static_cast<const __nv_bfloat16*>(q_weight);
  auto wk = static_cast<const __nv_bfloat16*>(k_weight);
  auto cb = static_cast<const __nv_bfloat16*>(cos_tab);
  auto sb = static_cast<const __nv_bfloat16*>(sin_tab);
#define LTX_QK_SCATTER(NIV)                                                                                      \
  launch_pdl(qk_rows_bf16_kernel<NIV, true>, dim3(grid), dim3(256), 0, s, 1, xb, ldx, rows, rows_per_batch, per, \
             head_dim, wq, eps, cb, sb, ld_rope, rope_ld_batch, wk, D, sc)
  switch (ni) {
    case 1: LTX_QK_SCATTER(1); break;
    case 2: LTX_QK_SCATTER(2); break;
    case 3: LTX_QK_SCATTER(3); break;
    default: LTX_QK_SCATTER(4); break;
  }
#undef LTX_QK_SCATTER
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_qk_norm_rope(void* x, int64_t ldx, int64_t rows, int64_t rows_per_batch, int heads, int head_dim,
                                const void* weight, float eps, const void* cos_tab, const void* sin_tab,
                                int64_t ld_rope, int64_t rope_ld_batch, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(x != nullptr, "x must be non-NULL");
  LTX_REQUIRE(weight != nullptr || cos_tab != nullptr, "nothing to do: no weight and no RoPE tables");
  LTX_REQUIRE(rows > 0 && rows < (int64_t(1) << 31), "rows out of range");
  LTX_REQUIRE(heads > 0 && head_dim > 0 && head_dim % 16 == 0, "head_dim must be a positive multiple of 16");
  const int nthr = heads * (head_dim / 16);
  LTX_UNSUPPORTED(nthr <= 1024, "heads*head_dim too large (max 16384)");
  LTX_REQUIRE(ldx % 8 == 0 && ldx >= int64_t(heads) * head_dim, "ldx must be a multiple of 8 and >= heads*head_dim");
  LTX_REQUIRE(rows_per_batch > 0, "rows_per_batch must be positive");
  LTX_REQUIRE((cos_tab == nullptr) == (sin_tab == nullptr), "cos and sin must both be given or both be NULL");
  if (cos_tab) LTX_REQUIRE(ld_rope % 8 == 0 && rope_ld_batch % 8 == 0, "rope strides must be multiples of 8");
  check_vec_ptr(x, "x");
  check_vec_ptr(weight, "weight");
  check_vec_ptr(cos_tab, "cos");
  check_vec_ptr(sin_tab, "sin");
  const int threads = ((nthr + 31) / 32) * 32;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LTX_F32)
    qk_norm_rope_kernel<float><<<unsigned(rows), threads, 0, s>>>(
        static_cast<float*>(x), ldx, rows_per_batch, heads, head_dim, static_cast<const float*>(weight), eps,
        static_cast<const float*>(cos_tab), static_cast<const float*>(sin_tab), ld_rope, rope_ld_batch), ltx::note_launch();
  else if ((nthr % 32) == 0 && nthr / 32 <= 4) {
    // one warp per row; 2 CTAs of 8 warps per SM, an even share of rows each
    const int ni = nthr / 32;
    const int64_t target = int64_t(num_sms()) * 2;
    const int per = int(std::max<int64_t>(8, (rows + target - 1) / target));
    const unsigned grid = unsigned((rows + per - 1) / per);
    auto xb = static_cast<__nv_bfloat16*>(x);
    auto wb = static_cast<const __nv_bfloat16*>(weight);
    auto cb = static_cast<const __nv_bfloat16*>(cos_tab);
    auto sb = static_cast<const __nv_bfloat16*>(sin_tab);
#define LTX_QK_ROWS(NIV)                                                                                    \
  launch_pdl(qk_rows_bf16_kernel<NIV, false>, dim3(grid), dim3(256), 0, s, 1, xb, ldx, rows, rows_per_batch, per, \
             head_dim, wb, eps, cb, sb, ld_rope, rope_ld_batch, static_cast<const __nv_bfloat16*>(nullptr), int64_t(0), \
             SpScatter{})
    switch (ni) {
      case 1: LTX_QK_ROWS(1); break;
      case 2: LTX_QK_ROWS(2); break;
      case 3: LTX_QK_ROWS(3); break;
      default: LTX_QK_ROWS(4); break;
    }
#undef LTX_QK_ROWS
  } else
    qk_norm_rope_kernel<__nv_bfloat16><<<unsigned(rows), threads, 0, s>>>(
        static_cast<__nv_bfloat16*>(x), ldx, rows_per_batch, heads, head_dim,
        static_cast<const __nv_bfloat16*>(weight), eps, static_cast<const __nv_bfloat16*>(cos_tab),
        static_cast<const __nv_bfloat16*>(sin_tab), ld_rope, rope_ld_batch), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_rope_tables(const float* bounds, int n_axes, int64_t T, const float* freqs, int n_freq,
                               const float* max_pos, int dim, void* cos_out, void* sin_out, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(bounds && freqs && max_pos && cos_out && sin_out, "NULL argument");
  LTX_REQUIRE(n_axes > 0 && T > 0 && n_freq > 0 && dim > 0 && dim % 2 == 0, "bad sizes");
  const int half = dim / 2;
  LTX_REQUIRE(n_freq * n_axes <= half, "n_freq * n_axes must be <= dim/2");
  const int64_t n = T * half;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = unsigned((n + 255) / 256);
  if (dtype == LTX_F32)
    rope_tables_kernel<float><<<blocks, 256, 0, s>>>(bounds, n_axes, T, freqs, n_freq, max_pos, half,
                                                     static_cast<float*>(cos_out), static_cast<float*>(sin_out)), ltx::note_launch();
  else
    rope_tables_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(bounds, n_axes, T, freqs, n_freq, max_pos, half,
                                                             static_cast<__nv_bfloat16*>(cos_out),
                                                             static_cast<__nv_bfloat16*>(sin_out)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_gelu_tanh(const void* x, void* y, int64_t n, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(x && y, "NULL argument");
  LTX_REQUIRE(n > 0, "n must be positive");
  check_vec_ptr(x, "x");
  check_vec_ptr(y, "y");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(n / 8 + 8, 256);
  if (dtype == LTX_F32)
    gelu_tanh_kernel<float><<<g, 256, 0, s>>>(static_cast<const float*>(x), static_cast<float*>(y), n), ltx::note_launch();
  else
    gelu_tanh_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                       static_cast<__nv_bfloat16*>(y), n), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_gate_residual(const void* x, int64_t ldx, const void* y, int64_t ldy, void* out, int64_t ldo,
                                 int64_t rows, int64_t rows_per_batch, int D, const ltx_modulation* gate, int dtype,
                                 void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(x && y && out, "NULL argument");
  LTX_REQUIRE(rows > 0 && D > 0 && D % 8 == 0, "rows must be positive and D a multiple of 8");
  LTX_REQUIRE(ldx % 8 == 0 && ldy % 8 == 0 && ldo % 8 == 0, "leading dimensions must be multiples of 8");
  LTX_REQUIRE(rows_per_batch > 0, "rows_per_batch must be positive");
  check_vec_ptr(x, "x");
  check_vec_ptr(y, "y");
  check_vec_ptr(out, "out");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(rows * (D / 8), 256);
  if (dtype == LTX_F32)
    gate_residual_kernel<float><<<g, 256, 0, s>>>(static_cast<const float*>(x), ldx, static_cast<const float*>(y), ldy,
                                                  static_cast<float*>(out), ldo, rows, rows_per_batch, D,
                                                  make_modvec<float>(gate, 1)), ltx::note_launch();
  else
    gate_residual_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(y), ldy,
        static_cast<__nv_bfloat16*>(out), ldo, rows, rows_per_batch, D, make_modvec<__nv_bfloat16>(gate, 1)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_timestep_embedding(const float* t, int64_t n, float scale, int dim, float max_period, void* out,
                                      int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(t && out, "NULL argument");
  LTX_REQUIRE(n > 0 && dim > 1 && max_period > 0.f, "bad sizes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = n * dim;
  const unsigned blocks = unsigned((total + 255) / 256);
  const float lmp = logf(max_period);
  if (dtype == LTX_F32)
    timestep_embedding_kernel<float><<<blocks, 256, 0, s>>>(t, n, scale, dim, lmp, static_cast<float*>(out)), ltx::note_launch();
  else
    timestep_embedding_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(t, n, scale, dim, lmp,
                                                                    static_cast<__nv_bfloat16*>(out)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_cfg_euler(const void* vel, const void* latent, const float* timesteps, int64_t T, int C,
                             float cfg_scale, float sigma, float sigma_next, void* denoised, void* new_latent,
                             int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(vel && latent && timesteps && new_latent, "NULL argument");
  LTX_REQUIRE(T > 0 && C > 0, "bad sizes");
  LTX_REQUIRE(sigma != 0.f, "sigma must be non-zero (Euler divides by it)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = T * C;
  const unsigned blocks = unsigned((n + 255) / 256);
  const float cfg_m1 = cfg_scale - 1.f;
  const float dt = sigma_next - sigma;
  if (dtype == LTX_F32)
    cfg_euler_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(vel), static_cast<const float*>(latent),
                                                   timesteps, T, C, cfg_m1, sigma, dt, static_cast<float*>(denoised),
                                                   static_cast<float*>(new_latent)), ltx::note_launch();
  else
    cfg_euler_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(vel), static_cast<const __nv_bfloat16*>(latent), timesteps, T, C, cfg_m1,
        sigma, dt, static_cast<__nv_bfloat16*>(denoised), static_cast<__nv_bfloat16*>(new_latent)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_guide(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n,
                         float cfg_scale, float stg_scale, float modality_scale, void* out, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(cond && uncond && ptb && mod && out, "NULL argument");
  LTX_REQUIRE(n > 0, "n must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = unsigned((n + 255) / 256);
  if (dtype == LTX_F32)
    guide_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(cond), static_cast<const float*>(uncond),
                                               static_cast<const float*>(ptb), static_cast<const float*>(mod), n,
                                               cfg_scale - 1.f, stg_scale, modality_scale - 1.f,
                                               static_cast<float*>(out)), ltx::note_launch();
  else
    guide_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(cond), static_cast<const __nv_bfloat16*>(uncond),
        static_cast<const __nv_bfloat16*>(ptb), static_cast<const __nv_bfloat16*>(mod), n, cfg_scale - 1.f,
        stg_scale, modality_scale - 1.f, static_cast<__nv_bfloat16*>(out)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" size_t ltx_guide_rescale_workspace_bytes(int64_t n) { return n > 0 ? guide_rescale_ws_bytes(n) : 0; }

extern "C" int ltx_guide_rescale(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n,
                                 float cfg_scale, float stg_scale, float modality_scale, float rescale_scale,
                                 void* out, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(cond && uncond && ptb && mod && out && workspace, "NULL argument");
  LTX_REQUIRE(n > 1, "n must be at least 2 (unbiased std)");
  LTX_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
  LTX_REQUIRE(workspace_bytes >= guide_rescale_ws_bytes(n), "workspace too small (ltx_guide_rescale_workspace_bytes)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto ws = static_cast<GuideWs*>(workspace);
  if (dtype == LTX_F32)
    launch_guide_rescale<float>(cond, uncond, ptb, mod, n, cfg_scale - 1.f, stg_scale, modality_scale - 1.f,
                                rescale_scale, out, ws, s);
  else
    launch_guide_rescale<__nv_bfloat16>(cond, uncond, ptb, mod, n, cfg_scale - 1.f, stg_scale,
                                        modality_scale - 1.f, rescale_scale, out, ws, s);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

// Allocation-free variant: the scratch is a file-scope device array. Static device
// memory starts zeroed at module load, so the completion counter starts at zero and each
// call leaves it at zero. One scratch per device: overlapping calls race on it.
constexpr int kGuideStaticBlocks = 256;  // n <= 256 * kGuideElemsPerBlock = 1,048,576
constexpr size_t kGuideStaticBytes = sizeof(GuideWs) + size_t(kGuideStaticBlocks) * 4 * sizeof(double);
static __device__ __align__(256) unsigned char g_guide_scratch[kGuideStaticBytes];

extern "C" int ltx_guide_rescale_noalloc(const void* cond, const void* uncond, const void* ptb, const void* mod,
                                         int64_t n, float cfg_scale, float stg_scale, float modality_scale,
                                         float rescale_scale, void* out, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(cond && uncond && ptb && mod && out, "NULL argument");
  LTX_REQUIRE(n > 1, "n must be at least 2 (unbiased std)");
  if (guide_rescale_ws_bytes(n) > kGuideStaticBytes)
    throw ApiError{LTX_ERR_INVALID, "n = " + std::to_string(n) + " exceeds the static scratch of " +
                                        std::to_string(kGuideStaticBytes) + " bytes (at most " +
                                        std::to_string(int64_t(kGuideStaticBlocks) * kGuideElemsPerBlock) +
                                        " elements); use ltx_guide_rescale with a workspace"};
  // Device address of the scratch, looked up once per device with that device current.
  // std::call_once makes the first call thread-safe; a lookup that fails leaves the flag
  // unset, so the next call retries it.
  static std::once_flag scratch_once[64];
  static void* scratch_ptr[64] = {};
  int dev = 0;
  LTX_CUDA(cudaGetDevice(&dev));
  LTX_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range");
  std::call_once(scratch_once[dev], [dev] {
    void* ptr = nullptr;
    LTX_CUDA(cudaGetSymbolAddress(&ptr, g_guide_scratch));
    scratch_ptr[dev] = ptr;
  });
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto ws = static_cast<GuideWs*>(scratch_ptr[dev]);
  if (dtype == LTX_F32)
    launch_guide_rescale<float>(cond, uncond, ptb, mod, n, cfg_scale - 1.f, stg_scale, modality_scale - 1.f,
                                rescale_scale, out, ws, s);
  else
    launch_guide_rescale<__nv_bfloat16>(cond, uncond, ptb, mod, n, cfg_scale - 1.f, stg_scale,
                                        modality_scale - 1.f, rescale_scale, out, ws, s);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_register_fill(const void* x, int64_t ldx, const void* additive_mask, const void* registers,
                                 int num_registers, int64_t rows, int64_t rows_per_batch, int D, void* out,
                                 int64_t ldo, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(x && additive_mask && registers && out, "NULL argument");
  LTX_REQUIRE(rows > 0 && rows_per_batch > 0 && num_registers > 0 && D > 0 && D % 8 == 0,
              "bad shape (D must be a positive multiple of 8)");
  LTX_REQUIRE(ldx % 8 == 0 && ldo % 8 == 0 && ldx >= D && ldo >= D, "ldx / ldo must be multiples of 8 and >= D");
  check_vec_ptr(x, "x");
  check_vec_ptr(registers, "registers");
  check_vec_ptr(out, "out");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = unsigned((rows * (D / 8) + 255) / 256);
  if (dtype == LTX_F32)
    register_fill_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), ldx,
                                                       static_cast<const float*>(additive_mask),
                                                       static_cast<const float*>(registers), num_registers, rows,
                                                       rows_per_batch, D, static_cast<float*>(out), ldo),
        ltx::note_launch();
  else
    register_fill_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(additive_mask),
        static_cast<const __nv_bfloat16*>(registers), num_registers, rows, rows_per_batch, D,
        static_cast<__nv_bfloat16*>(out), ldo),
        ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_x0(const void* latent, const void* velocity, const float* timesteps, int64_t rows, int C,
                      void* out, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(latent && velocity && timesteps && out, "NULL argument");
  LTX_REQUIRE(rows > 0 && C > 0, "rows and C must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = unsigned((rows * C + 255) / 256);
  if (dtype == LTX_F32)
    x0_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(latent), static_cast<const float*>(velocity),
                                            timesteps, rows, C, static_cast<float*>(out)), ltx::note_launch();
  else
    x0_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(latent),
                                                    static_cast<const __nv_bfloat16*>(velocity), timesteps, rows, C,
                                                    static_cast<__nv_bfloat16*>(out)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_euler(const void* sample, const void* denoised, int64_t n, float sigma, float sigma_next,
                         void* out, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_CHECK_DTYPE(dtype);
  LTX_REQUIRE(sample && denoised && out, "NULL argument");
  LTX_REQUIRE(n > 0, "n must be positive");
  LTX_REQUIRE(sigma != 0.f, "sigma must be non-zero (Euler divides by it)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = unsigned((n + 255) / 256);
  if (dtype == LTX_F32)
    euler_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(sample), static_cast<const float*>(denoised),
                                               n, sigma, sigma_next - sigma, static_cast<float*>(out)), ltx::note_launch();
  else
    euler_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(sample),
                                                       static_cast<const __nv_bfloat16*>(denoised), n, sigma,
                                                       sigma_next - sigma, static_cast<__nv_bfloat16*>(out)), ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
