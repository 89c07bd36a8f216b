// Device-side views of the C-ABI parameter structs, shared by the element-wise, GEMM
// and denoise kernels.
#pragma once
#include "ltx_common.cuh"
#include "ltx_internal.h"

#include <utility>

namespace ltx {

// Launch with programmatic stream serialisation: the grid may be scheduled while the
// previous kernel of the stream is still running (once all of that kernel's CTAs have
// executed pdl_trigger or exited). Every kernel launched this way calls pdl_wait (all
// threads) after its on-chip prologue and before its first global-memory access, and
// pdl_trigger after that wait, so a kernel never reads or writes global memory before
// the kernels ahead of it in the stream have completed.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  LTX_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  note_launch();
}

// One adaLN vector: v[c] = round(table[toff + c] + mod[b*ldb + t*ldt + moff + c]).
// Mirrors get_ada_values (ltx_dit.py:192-198): the table row and the timestep
// modulation are added in the activation dtype, so the sum is rounded to it.
template <typename T>
struct ModVec {
  const T* table = nullptr;
  const T* mod = nullptr;
  int64_t ldb = 0, ldt = 0, toff = 0, moff = 0;
  int on = 0;

  LTX_DEVICE float at(int64_t b, int64_t t, int64_t c) const {
    float v = 0.f;
    if (table) v += ld_elem<T>(table + toff + c);
    if (mod) v += ld_elem<T>(mod + b * ldb + t * ldt + moff + c);
    return round_to<T>(v);
  }
  LTX_DEVICE void at8(int64_t b, int64_t t, int64_t c, float (&v)[8]) const {
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (table) {
      ld8<T>(table + toff + c, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] += a[i];
    }
    if (mod) {
      ld8<T>(mod + b * ldb + t * ldt + moff + c, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] += a[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = round_to<T>(v[i]);
  }
};

inline void check_vec_ptr(const void* p, const char* what) {
  if (p != nullptr && reinterpret_cast<uintptr_t>(p) % 16 != 0)
    throw ApiError{LTX_ERR_INVALID, std::string(what) + " must be 16-byte aligned"};
}

// Build the shift (which = 0) or scale/gate (which = 1) vector of an ltx_modulation.
template <typename T>
ModVec<T> make_modvec(const ltx_modulation* m, int which) {
  ModVec<T> v;
  if (m == nullptr) return v;
  const int has = which == 0 ? m->has_shift : m->has_scale;
  if (!has) return v;
  v.table = static_cast<const T*>(m->table);
  v.mod = static_cast<const T*>(m->mod);
  v.ldb = m->mod_ld_batch;
  v.ldt = m->mod_ld_tok;
  v.toff = which == 0 ? m->shift_table_off : m->scale_table_off;
  v.moff = which == 0 ? m->shift_mod_off : m->scale_mod_off;
  v.on = (v.table != nullptr || v.mod != nullptr) ? 1 : 0;
  check_vec_ptr(v.table, "modulation table");
  check_vec_ptr(v.mod, "modulation tensor");
  if ((v.ldb % 8) || (v.ldt % 8) || (v.toff % 8) || (v.moff % 8))
    throw ApiError{LTX_ERR_INVALID, "modulation strides and offsets must be multiples of 8 elements"};
  return v;
}

// GEMM epilogue parameters (device view of ltx_epilogue).
template <typename T>
struct Epi {
  int kind = LTX_EPI_NONE;
  const T* bias = nullptr;
  const T* residual = nullptr;
  int64_t ld_res = 0;
  ModVec<T> gate;
  int64_t rows_per_batch = 1;
  const float* row_mask = nullptr;
  const T* row_vec = nullptr;
};

LTX_DEVICE float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}
LTX_DEVICE float silu_f(float x) { return x / (1.f + expf(-x)); }

// GELU-tanh with the hardware tanh approximation (relative error ~2^-11, below the
// 2^-8 rounding of the bf16 result); the fp32 accuracy mode uses gelu_tanh_f.
LTX_DEVICE float gelu_tanh_fast(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(inner));
  return 0.5f * x * (1.f + t);
}
template <typename T> LTX_DEVICE float gelu_act(float x);
template <> LTX_DEVICE float gelu_act<float>(float x) { return gelu_tanh_f(x); }
template <> LTX_DEVICE float gelu_act<__nv_bfloat16>(float x) { return gelu_tanh_fast(x); }

// Apply the epilogue to 8 consecutive accumulator columns [col, col+8) of row `row`.
// Rounding follows the reference's op-by-op dtype: the Linear result is rounded to
// the activation dtype before the activation / gate / residual is applied.
// `sb` / `st` are the row's sample and token index (row = sb * rows_per_batch + st);
// pass sb < 0 to have them computed here (a 64-bit division: hoist it out of loops).
template <typename T>
LTX_DEVICE void epilogue8(const Epi<T>& e, int64_t row, int64_t col, float (&v)[8], const float* res_pre = nullptr,
                          int64_t sb = -1, int64_t st = 0) {
  if (e.bias) {
    float b[8];
    ld8<T>(e.bias + col, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += b[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = round_to<T>(v[i]);
  switch (e.kind) {
    case LTX_EPI_GELU_TANH:
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = gelu_act<T>(v[i]);
      break;
    case LTX_EPI_SILU:
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = silu_f(v[i]);
      break;
    case LTX_EPI_GATE_RESIDUAL: {
      float g[8], r[8];
      if (e.gate.on) {
        if (sb < 0) {
          sb = row / e.rows_per_batch;
          st = row - sb * e.rows_per_batch;
        }
        e.gate.at8(sb, st, col, g);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = 1.f;
      }
      if (res_pre != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = res_pre[i];
      } else {
        ld8<T>(e.residual + row * e.ld_res + col, r);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = r[i] + round_to<T>(v[i] * g[i]);
      break;
    }
    case LTX_EPI_ROW_MASK_ADD: {
      if (e.row_mask[row] > 0.f) {
        float a[8];
        ld8<T>(e.row_vec + col, a);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] += a[i];
      }
      break;
    }
    default:
      break;
  }
}

// Scalar form of the same epilogue (tails and the CUDA-core GEMM).
template <typename T>
LTX_DEVICE float epilogue1(const Epi<T>& e, int64_t row, int64_t col, float v) {
  if (e.bias) v += ld_elem<T>(e.bias + col);
  v = round_to<T>(v);
  switch (e.kind) {
    case LTX_EPI_GELU_TANH:
      return gelu_act<T>(v);
    case LTX_EPI_SILU:
      return silu_f(v);
    case LTX_EPI_GATE_RESIDUAL: {
      const int64_t b = row / e.rows_per_batch, t = row - b * e.rows_per_batch;
      const float g = e.gate.on ? e.gate.at(b, t, col) : 1.f;
      return ld_elem<T>(e.residual + row * e.ld_res + col) + round_to<T>(v * g);
    }
    case LTX_EPI_ROW_MASK_ADD:
      return e.row_mask[row] > 0.f ? v + ld_elem<T>(e.row_vec + col) : v;
    default:
      return v;
  }
}

template <typename T>
Epi<T> make_epi(const ltx_epilogue* p) {
  Epi<T> e;
  if (p == nullptr) return e;
  e.kind = p->kind;
  e.bias = static_cast<const T*>(p->bias);
  e.residual = static_cast<const T*>(p->residual);
  e.ld_res = p->ld_residual;
  e.rows_per_batch = p->rows_per_batch > 0 ? p->rows_per_batch : 1;
  e.row_mask = p->row_mask;
  e.row_vec = static_cast<const T*>(p->row_vec);
  if (e.kind < LTX_EPI_NONE || e.kind > LTX_EPI_ROW_MASK_ADD)
    throw ApiError{LTX_ERR_INVALID, "unknown epilogue kind"};
  if (e.kind == LTX_EPI_GATE_RESIDUAL) {
    if (e.residual == nullptr) throw ApiError{LTX_ERR_INVALID, "GATE_RESIDUAL needs a residual"};
    if (e.ld_res % 8) throw ApiError{LTX_ERR_INVALID, "ld_residual must be a multiple of 8"};
    check_vec_ptr(e.residual, "residual");
    e.gate = make_modvec<T>(&p->gate, 1);
  }
  if (e.kind == LTX_EPI_ROW_MASK_ADD && (e.row_mask == nullptr || e.row_vec == nullptr))
    throw ApiError{LTX_ERR_INVALID, "ROW_MASK_ADD needs row_mask and row_vec"};
  check_vec_ptr(e.bias, "bias");
  check_vec_ptr(e.row_vec, "row_vec");
  return e;
}

}  // namespace ltx
