// Whole CFG denoise step of the video DiT behind one C entry point (ltx_dit_step), for
// callers that drive the library from C or C++ without Python. It issues the same
// kernels, with the same arguments and in the same order, as the Python drop-in
// (ltx_dit.cfg_denoise_step: LTXModel.prepare -> run_blocks -> head_hidden ->
// proj_out_cfg_euler), so both produce bit-identical latents.
//
// The step orchestrates ltx_dit.py:354-378 (forward) and :551-606 (X0, guide, Euler) of
// lipaul/ltx-nv for the B = 2 [cond, uncond] batch; every operation is one of the
// library's own entry points (tcgen05 GEMMs, FMHA, row kernels).
#include <cmath>
#include <cstring>
#include <vector>

#include "ltx_kernels.cuh"

struct ltx_ctx {
  int device = 0;
  ltx::TmapCache* tmaps = nullptr;
  void* ws = nullptr;  // device workspace (cudaMalloc'd by ltx_dit_reserve)
  size_t ws_bytes = 0;
  // sizes the workspace and the uploaded tables were made for
  ltx_dit_config cfg{};
  int64_t T = 0, S = 0;
  bool rope_valid = false;    // RoPE tables of the last step's positions
  bool text_kv_valid = false; // text K/V of the last step's contexts
};

namespace ltx {
namespace detail {

__global__ void fill_f32_kernel(float* out, int64_t n, float v) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = v;
}

constexpr double kPi = 3.141592653589793;
inline int64_t pad8(int64_t n) { return (n + 7) / 8 * 8; }
inline size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// Workspace layout of one step (offsets in bytes from the workspace base).
struct StepLayout {
  size_t x, h, big, o, kv, ctx2, cos, sin, tmod, emb, tproj, th, ts, tin, freqs, maxpos, attn, attn_bytes, total;
  int64_t rows1, rows2, big_cols, n_freq;
};

inline StepLayout step_layout(const ltx_dit_config& c, int64_t T, int64_t S) {
  StepLayout L{};
  const int64_t D = int64_t(c.heads) * c.head_dim;
  const int64_t H = c.gated_attention ? c.heads : 0;
  const size_t es = c.dtype == LTX_BF16 ? 2 : 4;
  L.rows1 = pad8(3 * D + H);
  L.rows2 = pad8(D + H);
  L.big_cols = std::max<int64_t>(std::max<int64_t>(L.rows1, L.rows2), c.ffn_dim);
  L.n_freq = D / (2 * 3);
  size_t off = 0;
  auto take = [&off](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  L.x = take(size_t(2 * T * D) * es);
  L.h = take(size_t(2 * T * D) * es);
  L.big = take(size_t(2 * T * L.big_cols) * es);
  L.o = take(size_t(2 * T * D) * es);
  L.kv = take(size_t(c.num_layers) * size_t(2 * S * 2 * D) * es);
  L.ctx2 = take(size_t(2 * S) * size_t(c.cross_dim) * es);
  L.cos = take(size_t(T * D / 2) * es);
  L.sin = take(size_t(T * D / 2) * es);
  L.tmod = take(size_t(2 * 6 * D) * es);
  L.emb = take(size_t(2 * D) * es);
  L.tproj = take(size_t(2 * 256) * es);
  L.th = take(size_t(2 * D) * es);
  L.ts = take(size_t(2 * T) * sizeof(float));
  L.tin = take(2 * sizeof(float));
  L.freqs = take(size_t(L.n_freq) * sizeof(float));
  L.maxpos = take(3 * sizeof(float));
  // self-attention's split-tail workspace (zero-filled by ltx_dit_reserve)
  L.attn_bytes = c.dtype == LTX_BF16 ? ltx_attention_workspace_bytes(2, T, T, c.heads, c.head_dim) : 0;
  L.attn = take(L.attn_bytes);
  L.total = off;
  return L;
}

inline void check_config(const ltx_dit_config* c) {
  LTX_REQUIRE(c != nullptr, "NULL config");
  LTX_REQUIRE(c->dtype == LTX_BF16 || c->dtype == LTX_F32, "dtype must be LTX_BF16 or LTX_F32");
  LTX_REQUIRE(c->num_layers > 0 && c->heads > 0 && c->head_dim > 0, "bad model sizes");
  LTX_REQUIRE(c->in_channels > 0 && c->out_channels > 0 && c->cross_dim > 0 && c->ffn_dim > 0, "bad model sizes");
  LTX_REQUIRE(int64_t(c->heads) * c->head_dim >= 6 && (int64_t(c->heads) * c->head_dim) % 8 == 0,
              "hidden size must be a multiple of 8 (and hold the 3-axis RoPE grid)");
  LTX_REQUIRE(c->timestep_scale_multiplier > 0.f && c->theta > 1.0, "bad timestep scale / theta");
}

// ltx_modulation of rows (shift_row, scale_row) of a (n, D) adaLN table plus the matching
// slices of a per-sample (B, n*D) modulation (st.mod of ltx_dit.py's _Stream).
inline ltx_modulation table_mod(const void* table, const void* tmod, int64_t D, int n, int shift_row, int scale_row) {
  ltx_modulation m{};
  m.table = table;
  m.mod = tmod;
  m.mod_ld_batch = int64_t(n) * D;
  m.mod_ld_tok = 0;
  if (shift_row >= 0) {
    m.has_shift = 1;
    m.shift_table_off = m.shift_mod_off = int64_t(shift_row) * D;
  }
  if (scale_row >= 0) {
    m.has_scale = 1;
    m.scale_table_off = m.scale_mod_off = int64_t(scale_row) * D;
  }
  return m;
}

inline ltx_epilogue epi_bias(const void* bias) {
  ltx_epilogue e{};
  e.kind = LTX_EPI_NONE;
  e.bias = bias;
  e.rows_per_batch = 1;
  return e;
}

inline ltx_epilogue epi_gate_residual(const void* bias, void* x, int64_t ldx, const ltx_modulation* gate,
                                      int64_t rows_per_batch) {
  ltx_epilogue e{};
  e.kind = LTX_EPI_GATE_RESIDUAL;
  e.bias = bias;
  e.residual = x;
  e.ld_residual = ldx;
  if (gate) e.gate = *gate;
  e.rows_per_batch = rows_per_batch;
  return e;
}

// Re-raises a failed library call as the step's own error, naming the operation.
inline void ok(int status, const char* what) {
  if (status != LTX_OK) throw ApiError{status, std::string("ltx_dit_step: ") + what + ": " + ltx_last_error()};
}

}  // namespace detail
}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

extern "C" int ltx_ctx_create(int device, ltx_ctx** ctx) {
  LTX_API_BEGIN
  LTX_REQUIRE(ctx != nullptr, "ctx is NULL");
  int n = 0;
  LTX_CUDA(cudaGetDeviceCount(&n));
  LTX_REQUIRE(device >= 0 && device < n, "device ordinal out of range");
  auto* c = new ltx_ctx();
  c->device = device;
  c->tmaps = tmap_cache_new();
  *ctx = c;
  LTX_API_END
}

extern "C" int ltx_ctx_destroy(ltx_ctx* ctx) {
  LTX_API_BEGIN
  if (ctx == nullptr) return LTX_OK;
  if (ctx->ws != nullptr) {
    int prev = 0;
    LTX_CUDA(cudaGetDevice(&prev));
    LTX_CUDA(cudaSetDevice(ctx->device));
    const cudaError_t e = cudaFree(ctx->ws);
    cudaSetDevice(prev);
    ctx->ws = nullptr;
    if (e != cudaSuccess) throw ApiError{LTX_ERR_CUDA, std::string("cudaFree: ") + cudaGetErrorString(e)};
  }
  tmap_cache_delete(ctx->tmaps);
  delete ctx;
  LTX_API_END
}

extern "C" size_t ltx_dit_workspace_bytes(const ltx_dit_config* cfg, int64_t T, int64_t S) {
  if (cfg == nullptr || T <= 0 || S <= 0 || cfg->heads <= 0 || cfg->head_dim <= 0) return 0;
  return step_layout(*cfg, T, S).total;
}

extern "C" int ltx_dit_reserve(ltx_ctx* ctx, const ltx_dit_config* cfg, int64_t T, int64_t S) {
  LTX_API_BEGIN
  LTX_REQUIRE(ctx != nullptr, "ctx is NULL");
  check_config(cfg);
  LTX_REQUIRE(T > 0 && S > 0, "T and S must be positive");
  const StepLayout L = step_layout(*cfg, T, S);
  int prev = 0;
  LTX_CUDA(cudaGetDevice(&prev));
  LTX_CUDA(cudaSetDevice(ctx->device));
  struct Restore {
    int dev;
    ~Restore() { cudaSetDevice(dev); }
  } restore{prev};
  if (ctx->ws_bytes < L.total) {
    if (ctx->ws != nullptr) LTX_CUDA(cudaFree(ctx->ws));
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    LTX_CUDA(cudaMalloc(&ctx->ws, L.total));
    ctx->ws_bytes = L.total;
  }
  // RoPE frequency grid theta^linspace(0, 1, n) * pi / 2 in float64, then float32
  // (generate_freq_grid_np, ltx_nn.py:34-46), and the per-axis max positions.
  std::vector<float> freqs(size_t(L.n_freq));
  const double step = L.n_freq > 1 ? 1.0 / double(L.n_freq - 1) : 0.0;
  for (int64_t i = 0; i < L.n_freq; ++i) {
    const double x = (i == L.n_freq - 1 && L.n_freq > 1) ? 1.0 : double(i) * step;
    freqs[size_t(i)] = float(std::pow(cfg->theta, x) * kPi / 2.0);
  }
  char* base = static_cast<char*>(ctx->ws);
  LTX_CUDA(cudaMemcpy(base + L.freqs, freqs.data(), freqs.size() * sizeof(float), cudaMemcpyHostToDevice));
  LTX_CUDA(cudaMemcpy(base + L.maxpos, cfg->max_pos, 3 * sizeof(float), cudaMemcpyHostToDevice));
  if (L.attn_bytes > 0) LTX_CUDA(cudaMemset(base + L.attn, 0, L.attn_bytes));
  ctx->cfg = *cfg;
  ctx->T = T;
  ctx->S = S;
  ctx->rope_valid = false;
  ctx->text_kv_valid = false;
  LTX_API_END
}

extern "C" int ltx_dit_step(ltx_ctx* ctx, const ltx_dit_config* cfg, const ltx_dit_weights* w,
                            const ltx_dit_step_args* a, void* velocity, void* denoised, void* new_latent,
                            void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(ctx != nullptr && w != nullptr && a != nullptr, "NULL argument");
  check_config(cfg);
  LTX_REQUIRE(ctx->ws != nullptr, "call ltx_dit_reserve before ltx_dit_step");
  LTX_REQUIRE(a->latent && a->positions && a->context_pos && a->context_neg && new_latent, "NULL argument");
  LTX_REQUIRE(w->blocks != nullptr, "weights->blocks is NULL");
  LTX_REQUIRE(a->sigma != 0.f, "sigma must be non-zero (the Euler step divides by it)");
  const int64_t T = a->T, S = a->S;
  LTX_REQUIRE(T > 0 && S > 0, "T and S must be positive");
  const StepLayout L = step_layout(*cfg, T, S);
  LTX_REQUIRE(L.total <= ctx->ws_bytes, "workspace too small for this step: call ltx_dit_reserve with its sizes");
  LTX_REQUIRE(cfg->dtype == LTX_BF16 || (velocity != nullptr && denoised != nullptr),
              "fp32 mode needs velocity and denoised buffers");
  int dev = 0;
  LTX_CUDA(cudaGetDevice(&dev));
  LTX_REQUIRE(dev == ctx->device, "the context's device must be current");
  // reuse of step-invariant tables only within the sizes they were computed for
  const bool same_shape = ctx->T == T && ctx->S == S && std::memcmp(&ctx->cfg, cfg, sizeof(*cfg)) == 0;
  if (!same_shape) {
    ctx->cfg = *cfg;
    ctx->T = T;
    ctx->S = S;
    ctx->rope_valid = ctx->text_kv_valid = false;
  }
  TmapScope scope(ctx->tmaps);

  const int dt = cfg->dtype;
  const size_t es = dt == LTX_BF16 ? 2 : 4;
  const int64_t D = int64_t(cfg->heads) * cfg->head_dim;
  const int64_t H = cfg->heads, hd = cfg->head_dim, C = cfg->cross_dim, F = cfg->ffn_dim;
  const int64_t M = 2 * T;  // the [cond, uncond] batch, sample-major rows
  const float eps = cfg->norm_eps;
  const float attn_scale = float(std::pow(double(hd), -0.5));  // dim_head ** -0.5, rounded once
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(ctx->ws);
  void* x = base + L.x;
  void* h = base + L.h;
  void* big = base + L.big;
  void* o = base + L.o;
  char* kv_all = base + L.kv;
  void* ctx2 = base + L.ctx2;
  void* cosb = base + L.cos;
  void* sinb = base + L.sin;
  void* tmod = base + L.tmod;
  void* emb = base + L.emb;
  void* tproj = base + L.tproj;
  void* th = base + L.th;
  float* ts = reinterpret_cast<float*>(base + L.ts);
  float* tin = reinterpret_cast<float*>(base + L.tin);
  const float* freqs = reinterpret_cast<const float*>(base + L.freqs);
  const float* maxpos = reinterpret_cast<const float*>(base + L.maxpos);
  auto el = [es](void* p, int64_t elems) { return static_cast<void*>(static_cast<char*>(p) + elems * es); };

  // ---- timesteps: sigma for every token of both samples (fp32) --------------------
  fill_f32_kernel<<<unsigned(std::min<int64_t>((M + 255) / 256, 4096)), 256, 0, s>>>(ts, M, a->sigma),
      note_launch();
  fill_f32_kernel<<<1, 32, 0, s>>>(tin, 2, a->sigma), note_launch();
  LTX_CUDA(cudaGetLastError());

  // ---- patchify (+ keyframe embedding) of both samples' copy of the latent ---------
  {
    ltx_epilogue e = epi_bias(w->patchify_b);
    if (a->keyframes_mask != nullptr && w->keyframes_emb != nullptr) {
      e.kind = LTX_EPI_ROW_MASK_ADD;
      e.row_mask = a->keyframes_mask;
      e.row_vec = w->keyframes_emb;
    }
    for (int b = 0; b < 2; ++b)
      ok(ltx_linear(a->latent, cfg->in_channels, w->patchify_w, cfg->in_channels, el(x, b * T * D), D, T, D,
                    cfg->in_channels, &e, dt, stream),
         "patchify");
  }

  // ---- adaLN-single: sinusoid -> linear_1 + SiLU -> linear_2 -> linear(SiLU(.)) ----
  ok(ltx_timestep_embedding(tin, 2, cfg->timestep_scale_multiplier, 256, 10000.f, tproj, dt, stream),
     "timestep embedding");
  {
    ltx_epilogue e1 = epi_bias(w->t_linear_1_b);
    e1.kind = LTX_EPI_SILU;
    ok(ltx_linear(tproj, 256, w->t_linear_1_w, 256, th, D, 2, D, 256, &e1, dt, stream), "timestep linear_1");
    ltx_epilogue e2 = epi_bias(w->t_linear_2_b);
    ok(ltx_linear(th, D, w->t_linear_2_w, D, emb, D, 2, D, D, &e2, dt, stream), "timestep linear_2");
    ltx_epilogue e3 = epi_bias(w->adaln_b);
    e3.silu_input = 1;
    ok(ltx_linear(emb, D, w->adaln_w, D, tmod, 6 * D, 2, 6 * D, D, &e3, dt, stream), "adaLN linear");
  }

  // ---- RoPE tables of the positions (shared by both samples) -----------------------
  if (!(a->flags & LTX_STEP_REUSE_ROPE) || !ctx->rope_valid) {
    ok(ltx_rope_tables(a->positions, 3, T, freqs, int(L.n_freq), maxpos, int(D), cosb, sinb, dt, stream),
       "RoPE tables");
    ctx->rope_valid = true;
  }

  // ---- text-context K/V of every block (k RMS-normalised, no RoPE) -----------------
  const bool kv_fresh = !(a->flags & LTX_STEP_REUSE_TEXT_KV) || !ctx->text_kv_valid;
  if (kv_fresh) {
    LTX_CUDA(cudaMemcpyAsync(ctx2, a->context_pos, size_t(S * C) * es, cudaMemcpyDeviceToDevice, s));
    LTX_CUDA(cudaMemcpyAsync(el(ctx2, S * C), a->context_neg, size_t(S * C) * es, cudaMemcpyDeviceToDevice, s));
  }

  const int64_t rows1 = L.rows1, rows2 = L.rows2;
  for (int i = 0; i < cfg->num_layers; ++i) {
    const ltx_dit_block_weights& bw = w->blocks[i];
    void* kv = kv_all + size_t(i) * size_t(2 * S * 2 * D) * es;
    // self-attention (ltx_dit.py:259-266)
    ltx_modulation m01 = table_mod(bw.scale_shift_table, tmod, D, 6, 0, 1);
    ok(ltx_norm_modulate(x, D, h, D, M, T, int(D), LTX_NORM_RMS, eps, &m01, dt, stream), "norm1");
    {
      ltx_epilogue e = epi_bias(bw.attn1_qkvg_b);
      ok(ltx_linear(h, D, bw.attn1_qkvg_w, D, big, rows1, M, rows1, D, &e, dt, stream), "QKV");
    }
    ok(ltx_qk_norm_rope_pair(big, rows1, D, M, T, int(H), int(hd), bw.attn1_q_norm, bw.attn1_k_norm, eps, cosb, sinb,
                             D / 2, 0, dt, stream),
       "q/k norm + RoPE");
    ok(ltx_attention_ws(big, rows1, el(big, D), rows1, el(big, 2 * D), rows1, o, D, 2, T, T, int(H), int(hd),
                        attn_scale, cfg->gated_attention ? el(big, 3 * D) : nullptr, rows1,
                        L.attn_bytes > 0 ? base + L.attn : nullptr, L.attn_bytes, dt, stream),
       "self-attention");
    {
      ltx_modulation g2 = table_mod(bw.scale_shift_table, tmod, D, 6, -1, 2);
      ltx_epilogue e = epi_gate_residual(bw.attn1_out_b, x, D, &g2, T);
      ok(ltx_linear(o, D, bw.attn1_out_w, D, x, D, M, D, D, &e, dt, stream), "attention out");
    }
    // text cross-attention without cross-adaLN (ltx_dit.py:237-248, 267-282)
    ok(ltx_norm_modulate(x, D, h, D, M, T, int(D), LTX_NORM_RMS, eps, nullptr, dt, stream), "norm2");
    {
      ltx_epilogue e = epi_bias(bw.attn2_qg_b);
      ok(ltx_linear(h, D, bw.attn2_qg_w, D, big, rows2, M, rows2, D, &e, dt, stream), "text q");
    }
    ok(ltx_qk_norm_rope(big, rows2, M, T, int(H), int(hd), bw.attn2_q_norm, eps, nullptr, nullptr, 0, 0, dt, stream),
       "text q norm");
    if (kv_fresh) {
      ltx_epilogue e = epi_bias(bw.attn2_kv_b);
      ok(ltx_linear(ctx2, C, bw.attn2_kv_w, C, kv, 2 * D, 2 * S, 2 * D, C, &e, dt, stream), "text K/V");
      ok(ltx_qk_norm_rope(kv, 2 * D, 2 * S, S, int(H), int(hd), bw.attn2_k_norm, eps, nullptr, nullptr, 0, 0, dt,
                          stream),
         "text k norm");
    }
    ok(ltx_attention(big, rows2, kv, 2 * D, el(kv, D), 2 * D, o, D, 2, T, S, int(H), int(hd), attn_scale,
                     cfg->gated_attention ? el(big, D) : nullptr, rows2, dt, stream),
       "text cross-attention");
    {
      ltx_epilogue e = epi_gate_residual(bw.attn2_out_b, x, D, nullptr, T);
      ok(ltx_linear(o, D, bw.attn2_out_w, D, x, D, M, D, D, &e, dt, stream), "text out");
    }
    // feed-forward (ltx_dit.py:309-314)
    ltx_modulation m34 = table_mod(bw.scale_shift_table, tmod, D, 6, 3, 4);
    ok(ltx_norm_modulate(x, D, h, D, M, T, int(D), LTX_NORM_RMS, eps, &m34, dt, stream), "norm3");
    {
      ltx_epilogue e = epi_bias(bw.ff_in_b);
      e.kind = LTX_EPI_GELU_TANH;
      ok(ltx_linear(h, D, bw.ff_in_w, D, big, F, M, F, D, &e, dt, stream), "FFN in");
      ltx_modulation g5 = table_mod(bw.scale_shift_table, tmod, D, 6, -1, 5);
      ltx_epilogue e2 = epi_gate_residual(bw.ff_out_b, x, D, &g5, T);
      ok(ltx_linear(big, F, bw.ff_out_w, F, x, D, M, D, F, &e2, dt, stream), "FFN out");
    }
  }
  if (kv_fresh) ctx->text_kv_valid = true;

  // ---- head: LayerNorm * (1 + scale) + shift with (table + embedded), then proj_out
  //      with X0 + CFG + Euler in its epilogue (ltx_dit.py:371-378, 591-606) ---------
  {
    ltx_modulation m{};
    m.table = w->scale_shift_table;
    m.mod = emb;
    m.mod_ld_batch = D;
    m.has_shift = 1;
    m.shift_table_off = 0;
    m.shift_mod_off = 0;
    m.has_scale = 1;
    m.scale_table_off = D;
    m.scale_mod_off = 0;
    ok(ltx_norm_modulate(x, D, h, D, M, T, int(D), LTX_NORM_LAYER, eps, &m, dt, stream), "head norm");
  }
  ok(ltx_proj_out_cfg_euler(h, D, w->proj_out_w, w->proj_out_b, T, cfg->out_channels, D, a->latent, ts, a->cfg_scale,
                            a->sigma, a->sigma_next, velocity, denoised, new_latent, dt, stream),
     "proj_out + CFG + Euler");
  LTX_API_END
}
