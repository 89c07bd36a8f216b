/*
 * ltxb200.h - C ABI of libltxb200.so, the B200 (sm_100a) kernels behind the LTX-2.5 DiT
 * denoising step.
 *
 * Conventions
 *  - Every pointer argument is a device pointer owned by the caller. The library
 *    allocates device memory in two places only: ltx_dit_reserve sizes the workspace an
 *    ltx_ctx owns for the whole-step entry point (freed by ltx_ctx_destroy), and
 *    ltx_peer_alloc allocates a buffer that other processes map (ltx_peer_free).
 *  - `stream` is a cudaStream_t passed as void*; every call is asynchronous on it and
 *    performs no device synchronisation.
 *  - Every entry point returns LTX_OK (0) or an ltx_status error code; ltx_last_error()
 *    returns a message for the calling thread's last failure. Nothing throws or exits.
 *  - `dtype` selects the storage type of activations: LTX_F32 (the accuracy mode) or
 *    LTX_BF16. Arithmetic is fp32 in both; bf16 results are rounded to nearest-even.
 *  - Row-major matrices are described by (pointer, leading dimension in elements).
 *  - "rows_per_batch" maps a flattened row index r to its sample b = r / rows_per_batch
 *    (the reference's (B, T, D) activations flattened to (B*T, D)).
 *
 * Reference interface each entry replaces is cited as lipaul/ltx-nv file:line.
 */
#ifndef LTXB200_H
#define LTXB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LTX_OK = 0,
  LTX_ERR_INVALID = 1,     /* bad argument: null pointer, size, alignment, stride */
  LTX_ERR_CUDA = 2,        /* a CUDA runtime / driver call failed */
  LTX_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
  LTX_ERR_DEVICE = 4       /* a kernel reported an error through the device error word */
} ltx_status;

typedef enum { LTX_F32 = 0, LTX_BF16 = 1 } ltx_dtype;

/* Message for the calling thread's last failed call ("" if none). */
const char* ltx_last_error(void);
/* ABI version of this library (bumped on any signature change). */
int ltx_abi_version(void);
/* Number of kernels this library has launched in this process (all devices, all
 * streams; CUDA-graph replays are not counted). Instrumentation, no reference
 * counterpart. */
uint64_t ltx_launch_count(void);
/* Read (and clear when `clear` != 0) the device error word that bounded waits set when
 * they give up (1 = mbarrier wait timed out, 2 = sequence-parallel peer barrier timed
 * out). Synchronises `stream`. */
int ltx_device_error_flags(int* flags, int clear, void* stream);

/* ---------------------------------------------------------------------------------- */
/* Initial noise: torch-compatible Philox4x32-10 normal fill.                          */
/* Replaces cuda_c_standalone/common/philox.cu:19-45 (randn_kernel / randn_dispatch),  */
/* the engine behind torch.randn(generator=cuda) in standalone/ltx_dit.py:502,513.     */
/* ---------------------------------------------------------------------------------- */

/* Grid that torch's launch policy picks for `n` elements on `device`
 * (philox.cu:6-17: min(ceil(n/256), SMs * maxThreadsPerSM / 256)). */
int ltx_philox_grid(int device, int64_t n, int* grid);
/* Generator offset advance for one fill of `n` elements at `grid` blocks of 256
 * threads (philox.cu:16): ((n-1)/(256*grid*4)+1)*4. */
int64_t ltx_philox_offset_increment(int64_t n, int grid);
/* out[i] = N(0,1) sample i of the stream (seed, offset) laid out exactly as torch's
 * grid-stride kernel with `grid` blocks writes it (philox.cu:24-33). dtype F32/BF16. */
int ltx_philox_randn(void* out, int64_t n, int dtype, uint64_t seed, uint64_t offset, int grid, void* stream);
/* Raw Philox4x32-10 words: for thread t < threads and round r < rounds, writes the four
 * 32-bit outputs of counter (offset/4 + r, subsequence t) under key `seed` to
 * out[(r*threads + t)*4 + 0..3]. Test hook for the CPU restatement of the cipher. */
int ltx_philox_raw(uint32_t* out, int64_t threads, int64_t rounds, uint64_t seed, uint64_t offset, void* stream);

/* ---------------------------------------------------------------------------------- */
/* Fused normalisation + adaLN modulation.                                             */
/* Replaces rms_norm (standalone/ltx_nn.py:18) + get_ada_values (ltx_dit.py:192-198)   */
/* + "norm(x) * (1 + scale) + shift" (ltx_dit.py:261,273,290,311,314) and the output   */
/* head LayerNorm + modulation (ltx_dit.py:371-377).                                   */
/* ---------------------------------------------------------------------------------- */
/* LTX_NORM_NONE skips the normalisation: y = x * (1 + scale) + shift (the cross-adaLN
 * text-context modulation, ltx_dit.py:246). */
typedef enum { LTX_NORM_RMS = 0, LTX_NORM_LAYER = 1, LTX_NORM_NONE = 2 } ltx_norm_kind;

/* Per-sample (or per-token) modulation vector v = table[toff + c] + mod[b*ld_b + t*ld_t
 * + moff + c], rounded to the storage dtype the way the reference's bf16 add rounds. A
 * NULL table or mod drops that term; off < 0 disables the vector. */
typedef struct {
  const void* table;   /* (n, D) adaLN scale-shift table, or NULL */
  const void* mod;     /* (B, T?, n*D) timestep modulation, or NULL */
  int64_t mod_ld_batch; /* elements between samples in `mod` */
  int64_t mod_ld_tok;   /* elements between tokens in `mod` (0: per-sample) */
  int64_t shift_table_off, shift_mod_off; /* element offsets of the shift vector */
  int64_t scale_table_off, scale_mod_off; /* element offsets of the scale vector */
  int has_shift, has_scale;
} ltx_modulation;

/* y[r, :] = norm(x[r, :]) * (1 + scale_b) + shift_b over `rows` rows of width D. */
int ltx_norm_modulate(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t rows, int64_t rows_per_batch,
                      int D, int norm_kind, float eps, const ltx_modulation* mod, int dtype, void* stream);

/* ---------------------------------------------------------------------------------- */
/* q/k RMSNorm (learned weight, over the whole inner dim) + split RoPE, in place.      */
/* Replaces Attention.q_norm/k_norm (ltx_nn.py:186-187,214-215) and                    */
/* apply_split_rotary_emb (ltx_nn.py:99-115).                                          */
/* cos/sin: (rows_per_batch, heads*head_dim/2) tables, token stride ld_rope, sample    */
/* stride rope_ld_batch (0 when all samples share positions). NULL cos: no RoPE;       */
/* NULL weight: no normalisation (rotation only, apply_split_rotary_emb).              */
/* ---------------------------------------------------------------------------------- */
int ltx_qk_norm_rope(void* x, int64_t ldx, int64_t rows, int64_t rows_per_batch, int heads, int head_dim,
                     const void* weight, float eps, const void* cos_tab, const void* sin_tab, int64_t ld_rope,
                     int64_t rope_ld_batch, int dtype, void* stream);

/* Self-attention q and k in one pass (ltx_nn.py:186-187, 214-218): the q block at column 0
 * and the k block at column k_offset of the same rows are each RMS-normalised over the
 * inner dim with their own weight and rotated with the same RoPE tables (read once per
 * row). Same arithmetic as two ltx_qk_norm_rope calls. */
int ltx_qk_norm_rope_pair(void* x, int64_t ldx, int64_t k_offset, int64_t rows, int64_t rows_per_batch, int heads,
                          int head_dim, const void* q_weight, const void* k_weight, float eps, const void* cos_tab,
                          const void* sin_tab, int64_t ld_rope, int64_t rope_ld_batch, int dtype, void* stream);
/* RoPE tables from token positions (precompute_freqs_cis, ltx_nn.py:63-96): `bounds`
 * (n_axes, T, 2) fp32 [start, end) positions of one sample (the reference's
 * positions[b]), `freqs` (F) fp32 frequency grid (computed in float64 by the caller,
 * ltx_nn.py:34-46), max_pos per axis; writes cos/sin (T, dim/2) in `dtype` with the
 * front padding of ltx_nn.py:88-92. */
int ltx_rope_tables(const float* bounds, int n_axes, int64_t T, const float* freqs, int n_freq,
                    const float* max_pos, int dim, void* cos_out, void* sin_out, int dtype, void* stream);

/* ---------------------------------------------------------------------------------- */
/* Element-wise kernels (FeedForward GELU ltx_nn.py:248, residual gate                */
/* ltx_dit.py:265,311, timestep sinusoid standalone/common.py:138-148).                */
/* ---------------------------------------------------------------------------------- */
int ltx_gelu_tanh(const void* x, void* y, int64_t n, int dtype, void* stream);
/* out[r, :] = x[r, :] + y[r, :] * gate_b, gate from `mod` (shift fields unused; the gate
 * vector is described by scale_* fields). NULL mod: gate = 1. */
int ltx_gate_residual(const void* x, int64_t ldx, const void* y, int64_t ldy, void* out, int64_t ldo,
                      int64_t rows, int64_t rows_per_batch, int D, const ltx_modulation* gate, int dtype,
                      void* stream);
/* out[i, :] = [cos(t_i*scale*f_j), sin(t_i*scale*f_j)], f_j = exp(-ln(max_period) j/half). */
int ltx_timestep_embedding(const float* t, int64_t n, float scale, int dim, float max_period, void* out, int dtype,
                           void* stream);

/* ---------------------------------------------------------------------------------- */
/* Linear layers: C = epilogue(A * W^T + bias) with A (M, K) and W (N, K) K-major.     */
/* Replaces every nn.Linear on the path (ltx_nn.py:126-158,188-192,244-245,            */
/* ltx_dit.py:331-347) and cuda_c_standalone/common/gemm.cu:36-73 (linear()).          */
/* bf16: TMA-fed tcgen05/TMEM kernel (M >= 32) or a weight-streaming kernel (M < 32);  */
/* fp32: CUDA-core kernel.                                                             */
/* ---------------------------------------------------------------------------------- */
typedef enum {
  LTX_EPI_NONE = 0,          /* C = acc (+ bias) */
  LTX_EPI_GELU_TANH = 1,     /* C = gelu_tanh(acc + bias) */
  LTX_EPI_SILU = 2,          /* C = silu(acc + bias) */
  LTX_EPI_GATE_RESIDUAL = 3, /* C = residual + round(acc + bias) * gate_b */
  LTX_EPI_ROW_MASK_ADD = 4   /* C = round(acc + bias) + (row_mask[r] > 0) * row_vec */
} ltx_epilogue_kind;

typedef struct {
  int kind;
  const void* bias;         /* (N,) or NULL */
  const void* residual;     /* GATE_RESIDUAL: (M, N) with ld_residual; may alias C */
  int64_t ld_residual;
  ltx_modulation gate;      /* GATE_RESIDUAL: gate vector in the scale_* fields */
  int64_t rows_per_batch;   /* row -> sample map for the gate */
  const float* row_mask;    /* ROW_MASK_ADD: (M,) */
  const void* row_vec;      /* ROW_MASK_ADD: (N,) */
  int silu_input;           /* apply SiLU to A while loading it (weight-streaming path only) */
} ltx_epilogue;

int ltx_linear(const void* A, int64_t lda, const void* W, int64_t ldw, void* C, int64_t ldc, int64_t M, int64_t N,
               int64_t K, const ltx_epilogue* epi, int dtype, void* stream);

/* ---------------------------------------------------------------------------------- */
/* Attention: softmax(Q K^T * scale) V per (sample, head), non-causal, no mask, with   */
/* the per-(token, head) output gate 2*sigmoid(logit) fused in.                        */
/* Replaces sdpa (ltx_nn.py:22-26) + the gating of Attention.forward (ltx_nn.py:231-235)*/
/* and cuda_c_standalone/common/gemm.cu:17-34 (the unfused QK^T / PV plan).            */
/* Q rows of sample b start at q + b*Tq*ldq; head h occupies columns [h*d, (h+1)*d).    */
/* gate_logits: (B*Tq, H) with ld_gate, or NULL for no gate.                           */
/* bf16: tcgen05 FMHA (head_dim 64 or 128); fp32: CUDA-core kernel.                    */
/* ---------------------------------------------------------------------------------- */
int ltx_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                  int64_t ldo, int B, int64_t Tq, int64_t Tk, int heads, int head_dim, float scale,
                  const void* gate_logits, int64_t ld_gate, int dtype, void* stream);
/* ltx_attention with a workspace; same operands, and results equal up to bf16 rounding
 * of P within the split rows. The bf16 kernel runs one CTA per (sample, head, 256
 * queries); when these units leave the last wave of SMs partly filled, the units of that
 * wave are split over 2-8 key ranges whose fp32 partials the last CTA of each unit merges
 * (same as ltx_attention otherwise). The workspace (device memory,
 * ltx_attention_workspace_bytes bytes, 16-byte aligned) must be zero-filled before its
 * first use; every call leaves its counters at zero, so one workspace serves any sequence
 * of calls issued to one stream (calls that may run concurrently need one each). NULL,
 * or fewer bytes than the shape needs, runs without the split. Same reference as
 * ltx_attention. ltx_attention_workspace_bytes returns 0 when the shape has nothing to
 * split (then the two calls are the same). */
size_t ltx_attention_workspace_bytes(int B, int64_t Tq, int64_t Tk, int heads, int head_dim);
int ltx_attention_ws(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                     int64_t ldo, int B, int64_t Tq, int64_t Tk, int heads, int head_dim, float scale,
                     const void* gate_logits, int64_t ld_gate, void* workspace, size_t workspace_bytes, int dtype,
                     void* stream);

/* ---------------------------------------------------------------------------------- */
/* Denoise update: X0 conversion + CFG guidance + Euler step.                          */
/* Replaces guided_denoise_step's X0 (ltx_dit.py:591-593), guide (ltx_dit.py:551-562,  */
/* with rescale_scale = 0) and euler_step (ltx_dit.py:602-606).                        */
/* ---------------------------------------------------------------------------------- */
/* Element-wise form: vel (2, T, C) = model output for [cond, uncond] of one latent,
 * latent/new_latent (T, C), timesteps (2, T) per-token sigma. Writes new_latent and
 * (optionally) denoised (T, C). */
int ltx_cfg_euler(const void* vel, const void* latent, const float* timesteps, int64_t T, int C, float cfg_scale,
                  float sigma, float sigma_next, void* denoised, void* new_latent, int dtype, void* stream);

/* Perturbed self-attention (STG, ltx_nn.py:209-210 and the 0/1 blend at 229-230): the
 * attention output of `rows` rows is V itself, then gated per (token, head) by
 * 2*sigmoid(logit) like a real attention output (231-235; gate_logits may be NULL). The
 * caller passes the rows of the perturbed samples. */
int ltx_value_gate(const void* v, int64_t ldv, const void* gate_logits, int64_t ld_gate, void* o, int64_t ldo,
                   int64_t rows, int heads, int head_dim, int dtype, void* stream);

/* Guidance blend of four x0 predictions (ltx_dit.py:551-557, rescale_scale = 0):
 * out = cond + (cfg-1)(cond-uncond) + stg(cond-ptb) + (modality-1)(cond-mod). */
int ltx_guide(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n, float cfg_scale,
              float stg_scale, float modality_scale, void* out, int dtype, void* stream);
/* Guidance blend with std rescale (ltx_dit.py:551-562, rescale_scale != 0): pred as in
 * ltx_guide (fp32), factor = rescale*std(cond)/std(pred) + (1-rescale) with the unbiased
 * std over all n elements, out = round(pred*factor). Two kernels on `stream`. The
 * workspace (ltx_guide_rescale_workspace_bytes(n) bytes, 16-byte aligned, device memory
 * owned by the caller) holds per-block partial sums and a completion counter that must
 * be zero before the first call; every call leaves it zero again. Calls that share a
 * workspace must not run concurrently. */
size_t ltx_guide_rescale_workspace_bytes(int64_t n);
int ltx_guide_rescale(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n,
                      float cfg_scale, float stg_scale, float modality_scale, float rescale_scale, void* out,
                      void* workspace, size_t workspace_bytes, int dtype, void* stream);
/* ltx_guide_rescale without a caller workspace: the same two kernels, same results, with
 * the scratch in a static device array of 8208 bytes, so the call allocates nothing. It
 * takes n <= 1,048,576 elements (one video latent of the benchmark configurations is
 * 786,432) and rejects larger n with an error. The scratch's completion counter starts
 * at zero at module load and every call leaves it zero. One scratch per device: calls
 * that overlap in time on the same device (several streams or threads) race on it. The
 * first call on a device looks up the scratch's address (cudaGetSymbolAddress, once per
 * device and thread-safe); make that first call before any stream capture. The address
 * is kept for the life of the process, so after a cudaDeviceReset of a device this entry
 * point must not be called on it again. No counterpart in the reference. */
int ltx_guide_rescale_noalloc(const void* cond, const void* uncond, const void* ptb, const void* mod, int64_t n,
                              float cfg_scale, float stg_scale, float modality_scale, float rescale_scale, void* out,
                              int dtype, void* stream);
/* Text-connector register fill (ltx_te.py:218-223): out row r = x row r where the
 * additive mask of token r is >= 0, else registers row ((r % rows_per_batch) %
 * num_registers). x / out (rows, D) row-major, mask (rows) and registers
 * (num_registers, D) in the same dtype. */
int ltx_register_fill(const void* x, int64_t ldx, const void* additive_mask, const void* registers, int num_registers,
                      int64_t rows, int64_t rows_per_batch, int D, void* out, int64_t ldo, int dtype, void* stream);
/* X0 of a velocity prediction (ltx_dit.py:591-593, X0Model): out = round(latent - v *
 * timesteps[row]) with fp32 math; latent, velocity and out are (rows, C), timesteps fp32 (rows). */
int ltx_x0(const void* latent, const void* velocity, const float* timesteps, int64_t rows, int C, void* out,
           int dtype, void* stream);
/* Euler step (ltx_dit.py:602-606): v = round((sample-denoised)/sigma);
 * out = sample + v*(sigma_next - sigma). */
int ltx_euler(const void* sample, const void* denoised, int64_t n, float sigma, float sigma_next, void* out,
              int dtype, void* stream);

/* Fused form: the output projection (proj_out, ltx_dit.py:378) of the head-modulated
 * hidden state x (2*T, K) with weight W (C, K) and bias, followed in its epilogue by the
 * same X0 + CFG + Euler update. vel_out (2, T, C) (optional) receives the projection. */
int ltx_proj_out_cfg_euler(const void* x, int64_t ldx, const void* W, const void* bias, int64_t T, int C, int64_t K,
                           const void* latent, const float* timesteps, float cfg_scale, float sigma,
                           float sigma_next, void* vel_out, void* denoised, void* new_latent, int dtype,
                           void* stream);

/* ---------------------------------------------------------------------------------- */
/* Sequence-parallel (Ulysses) exchange layouts around NCCL all-to-all. No counterpart */
/* in the reference, which runs the whole sequence on one GPU (full-sequence sdpa,     */
/* ltx_nn.py:227).                                                                     */
/* ---------------------------------------------------------------------------------- */
/* dst[j][r][:] = concat over segments s of src[r][off_s + j*w_s, off_s + (j+1)*w_s),
 * for j < parts, r < rows (1..4 segments, 16-byte aligned widths and offsets). */
int ltx_sp_pack(const void* src, int64_t ld_src, int64_t rows, int parts, int n_seg, const int* seg_off,
                const int* seg_w, void* dst, int dtype, void* stream);
/* dst[r][j*w, (j+1)*w) = src[j][r][:] for j < parts, r < rows. */
int ltx_sp_unpack(const void* src, int64_t rows, int parts, int w, void* dst, int64_t ld_dst, int dtype,
                  void* stream);

/* The same exchange fused into the kernels on either side of it, over NVLink peer memory
 * (no counterpart in the reference, which runs on one GPU). Every SP rank owns one
 * buffer from ltx_peer_alloc (cudaMalloc'd and zero-filled, with a 64-byte CUDA IPC
 * handle that the other ranks of the node pass to ltx_peer_open to map it); kernels only
 * store to peer memory and load local memory.
 *
 * ltx_qk_norm_rope_scatter: ltx_qk_norm_rope_pair on x = (rows, [q | k | v | gate])
 * rows of this rank (rows_per_batch tokens per sample, D = heads * head_dim wide blocks,
 * gate logits when gated), except that the rows are not written back: the q, k, v
 * columns and gate logits of the heads of SP rank j (heads / parts of them) go to row
 * b * rows_per_batch * parts + sp_rank * rows_per_batch + t of dst[j], laid out
 * [q | k | v | gate] of width 3 * D / parts (+ heads / parts): the receive buffer that
 * pack + all-to-all would fill. bf16 only.
 * ltx_attention_scatter: self-attention over the B x T tokens of the receive buffer
 * (as ltx_attention_ws, with the same workspace), each output row written to the rank
 * that owns its token: row t of sample b to row b * (T / parts) + t % (T / parts) of
 * out[t / (T / parts)], columns out_col0 .. out_col0 + heads * head_dim (what
 * all-to-all + unpack would deliver). bf16 only, T > 128.
 * ltx_sp_barrier: every rank of the SP group calls it in the same order; it returns
 * (asynchronously, on `stream`) once every rank's preceding kernels have completed their
 * stores. flags[j] is rank j's flag array (`parts` ints, zero-filled) as mapped in this
 * process, counter a zero-filled int of this rank. A wait that lasts limit_cycles SM
 * cycles gives up: bit 2 of the device error word (ltx_device_error_flags). */
int ltx_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int ltx_peer_open(const void* ipc_handle, void** ptr);
int ltx_peer_close(void* ptr);
int ltx_peer_free(void* ptr);
int ltx_qk_norm_rope_scatter(const void* x, int64_t ldx, int64_t rows, int64_t rows_per_batch, int heads,
                             int head_dim, const void* q_weight, const void* k_weight, float eps, const void* cos_tab,
                             const void* sin_tab, int64_t ld_rope, int64_t rope_ld_batch, int gated, int parts,
                             int sp_rank, void* const* dst, int64_t ld_dst, void* stream);
int ltx_attention_scatter(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, int B,
                          int64_t T, int heads, int head_dim, float scale, const void* gate_logits, int64_t ld_gate,
                          void* workspace, size_t workspace_bytes, int parts, void* const* out, int64_t out_ld,
                          int out_col0, void* stream);
int ltx_sp_barrier(int* const* flags, int* counter, int parts, int rank, unsigned long long limit_cycles,
                   void* stream);

/* Split-KV attention across ranks (the audio queries of the video-to-audio attention,
 * ltx_dit.py:299-307, against video keys sharded by sequence parallelism). No counterpart
 * in the reference, which attends over all keys on one GPU (ltx_nn.py:227).
 * ltx_attention_partial: softmax(Q K^T * scale) V over this part of the keys, bf16
 * inputs as ltx_attention (head_dim 64 or 128), no gate; writes o_part (B*Tq, ldo) fp32 =
 * O / l and lse (B*Tq, ld_lse) fp32 = log2(sum_j 2^(s_j * scale * log2(e))) per head. */
int ltx_attention_partial(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                          float* o_part, int64_t ldo, float* lse, int64_t ld_lse, int B, int64_t Tq, int64_t Tk,
                          int heads, int head_dim, float scale, void* stream);
/* Merge of `parts` partials into the attention over all keys: o_parts (parts, rows,
 * heads*head_dim) and lse_parts (parts, rows, heads) contiguous fp32 (what an all-gather
 * of ltx_attention_partial outputs holds); out (rows, ldo) bf16 = the merged output with
 * the gate 2*sigmoid(logit) of gate_logits (rows, ld_gate) applied as ltx_attention does
 * (NULL: no gate). */
int ltx_attention_merge(const float* o_parts, const float* lse_parts, int parts, int64_t rows, int heads,
                        int head_dim, const void* gate_logits, int64_t ld_gate, void* out, int64_t ldo,
                        void* stream);

/* ---------------------------------------------------------------------------------- */
/* Video VAE decoder (ConvVideoDecoder, ltx_vae.py:167-222). Activations are           */
/* channels-last (B, F, H, W, C) bf16; the reference's tensors are (B, C, F, H, W).    */
/* ---------------------------------------------------------------------------------- */
/* CausalConv3d (ltx_vae.py:31-57) with stride 1: ksize 3 -> 3x3x3 taps, zero padding of
 * one voxel in H and W, frames padded by repeating the edge frames (causal = 0: one
 * copy at each end; causal = 1: two copies of the first frame in front); ksize 1 -> the
 * 1x1x1 Conv3d shortcut (ltx_vae.py:100). weight (cout, taps, cin) bf16, i.e. the
 * reference's (cout, cin, kt, kh, kw) permuted to tap-major K; bias (cout).
 * out = round(conv + bias), then + residual (same layout as out, may equal out) when
 * residual is not NULL. cin a multiple of 64, cout of 8; out must not alias x. */
int ltx_conv3d(const void* x, int B, int F, int H, int W, int cin, const void* weight, const void* bias, int cout,
               int ksize, int causal, const void* residual, void* out, void* stream);
/* The same with norm_silu = 1: out = silu(PixelNorm_eps(round(conv + bias))) over each
 * voxel's cout channels (ResnetBlock3D's conv1 followed by norm2 and the nonlinearity,
 * ltx_vae.py:107-110), computed in the epilogue. Needs cout <= 256 and no residual. */
int ltx_conv3d_norm(const void* x, int B, int F, int H, int W, int cin, const void* weight, const void* bias,
                    int cout, int ksize, int causal, const void* residual, int norm_silu, float eps, void* out,
                    void* stream);
/* PixelNorm (ltx_vae.py:20-28) over the C channels of each of `rows` voxels, followed by
 * SiLU when silu != 0 (ResnetBlock3D.nonlin, ltx_vae.py:111-115; the decoder's final
 * norm + SiLU, :209-210). x may equal y. */
int ltx_pixel_norm(const void* x, void* y, int64_t rows, int C, float eps, int silu, void* stream);
/* GroupNorm(1, C, eps) with affine weight / bias (ResnetBlock3D.norm3, ltx_vae.py:99):
 * per sample, mean and variance over its n_per_sample = F*H*W*C values. Two passes;
 * workspace of ltx_group_norm1_workspace_bytes(B) bytes (caller-owned, no init). */
int64_t ltx_group_norm1_workspace_bytes(int B);
int ltx_group_norm1(const void* x, int B, int64_t n_per_sample, int C, const void* weight, const void* bias, float eps,
                    void* workspace, int64_t ws_bytes, void* y, void* stream);
/* DepthToSpaceUpsample's rearrange (ltx_vae.py:135-143): x (B, F, H, W, c*p1*p2*p3) ->
 * y (B, F*p1 - drop_first, H*p2, W*p3, c); drop_first = 1 drops the first frame (the
 * reference does so when p1 == 2). c a multiple of 8. */
int ltx_depth_to_space(const void* x, int B, int F, int H, int W, int c, int p1, int p2, int p3, int drop_first,
                       void* y, void* stream);
/* PerChannelStatistics.un_normalize (ltx_vae.py:83-87) of the (B, C, F, H, W) latent into
 * the channels-last layout: y = round(round(x * bf16(std)) + bf16(mean)); std / mean fp32. */
int ltx_vae_latent_in(const void* latent, int B, int C, int F, int H, int W, const float* std_of_means,
                      const float* mean_of_means, void* y, void* stream);
/* Output unpatchify (ltx_vae.py:212-216) of x (B, F, H, W, c*p*p): mode 0 -> the
 * reference's (B, c, F, H*p, W*p) bf16 tensor; mode 1 -> decode_video's (F, H*p, W*p, c)
 * float frames of sample 0, (v + 1) / 2 clamped to [0, 1] (ltx_vae.py:218-222). */
int ltx_vae_unpatchify(const void* x, int B, int F, int H, int W, int c, int p, int mode, void* out, void* stream);

/* ---------------------------------------------------------------------------------- */
/* Whole denoise step: one CFG step of the video DiT (3 and 5) for   */
/* a C or C++ caller that links this library without Python.                           */
/* Replaces LTXModel.forward (standalone/ltx_dit.py:354-378) on the B=2 [cond, uncond] */
/* batch followed by X0 + guide + euler_step (ltx_dit.py:551-606, CFG-only guidance),   */
/* the sequence the reference's native port leaves unbuilt (cuda_c_standalone/Makefile: */
/* the dit/ and runner/ targets, 11,21-27).                                             */
/* ---------------------------------------------------------------------------------- */

/* Opaque per-device context: the cache of encoded TMA descriptors (keyed by pointer,
 * extents, row stride and box, so a hit is always valid), the step workspace and the
 * step-invariant tables (RoPE tables, text-context K/V) of the last step. One context
 * per device and thread; calls on one context must not overlap. */
typedef struct ltx_ctx ltx_ctx;

int ltx_ctx_create(int device, ltx_ctx** ctx);
/* Frees the workspace (on the context's device) and the context. NULL is a no-op. */
int ltx_ctx_destroy(ltx_ctx* ctx);

/* Video-only DiT configuration (DiTConfig of ltx_dit.py:28-82 with cross-adaLN off and
 * no audio stream: the text context keeps its own width cross_dim). */
typedef struct {
  int num_layers;
  int heads, head_dim;             /* hidden D = heads * head_dim */
  int in_channels, out_channels;   /* latent channels (128, 128) */
  int cross_dim;                   /* text context width C */
  int ffn_dim;                     /* FeedForward inner width (4 * D) */
  int gated_attention;             /* to_gate_logits present in both attentions */
  float norm_eps;                  /* 1e-6 */
  double theta;                    /* RoPE theta (10000) */
  float max_pos[3];                /* (20, 2048, 2048) */
  float timestep_scale_multiplier; /* 1000 */
  int dtype;                       /* LTX_BF16 or LTX_F32 */
} ltx_dit_config;

/* Device pointers of one block, in the storage dtype. Packed weights are row blocks of
 * the reference's nn.Linear weights, each packed matrix zero-padded to a multiple of 8
 * rows (its bias to the same length):
 *   attn1_qkvg = [attn1.to_q; to_k; to_v; to_gate_logits]   (3D + H (+pad), D)
 *   attn2_qg   = [attn2.to_q; to_gate_logits]               (D + H (+pad), D)
 *   attn2_kv   = [attn2.to_k; to_v]                          (2D, C)
 * (without gated attention the gate rows are absent). ff biases may be NULL
 * (ff_bias = False). Names follow BasicAVTransformerBlock (ltx_dit.py:209-235). */
typedef struct {
  const void* scale_shift_table; /* (6, D) */
  const void* attn1_qkvg_w;
  const void* attn1_qkvg_b;
  const void* attn1_q_norm;      /* (D) RMSNorm gains */
  const void* attn1_k_norm;
  const void* attn1_out_w;       /* (D, D) */
  const void* attn1_out_b;
  const void* attn2_qg_w;
  const void* attn2_qg_b;
  const void* attn2_kv_w;
  const void* attn2_kv_b;
  const void* attn2_q_norm;
  const void* attn2_k_norm;
  const void* attn2_out_w;
  const void* attn2_out_b;
  const void* ff_in_w;           /* (F, D) */
  const void* ff_in_b;
  const void* ff_out_w;          /* (D, F) */
  const void* ff_out_b;
} ltx_dit_block_weights;

/* Model-level device pointers (LTXModel, ltx_dit.py:325-352) and the host array of the
 * num_layers blocks. */
typedef struct {
  const void* patchify_w;        /* (D, in_channels) */
  const void* patchify_b;        /* (D) */
  const void* keyframes_emb;     /* (D) keyframes_abs_pos_embedding, or NULL */
  const void* t_linear_1_w;      /* adaln_single.emb.timestep_embedder.linear_1 (D, 256) */
  const void* t_linear_1_b;
  const void* t_linear_2_w;      /* ... linear_2 (D, D) */
  const void* t_linear_2_b;
  const void* adaln_w;           /* adaln_single.linear (6D, D) */
  const void* adaln_b;
  const void* scale_shift_table; /* (2, D) output head */
  const void* proj_out_w;        /* (out_channels, D) */
  const void* proj_out_b;
  const ltx_dit_block_weights* blocks;
} ltx_dit_weights;

/* Step flags. REUSE_TEXT_KV: use the text-context K/V projections of the previous step
 * on this context (the caller asserts that the contexts and weights are unchanged: they
 * are constant over a denoise loop, ltx_dit.py:609-621). REUSE_ROPE: use the previous
 * step's RoPE tables (same positions). Without a previous step they are computed. */
enum { LTX_STEP_REUSE_TEXT_KV = 1, LTX_STEP_REUSE_ROPE = 2 };

typedef struct {
  const void* latent;          /* (T, in_channels) current latent of the video */
  const float* positions;      /* (3, T, 2) fp32 [start, end) bounds (video_positions of one sample) */
  const void* context_pos;     /* (S, C) conditional text context */
  const void* context_neg;     /* (S, C) unconditional text context */
  const float* keyframes_mask; /* (T) fp32, > 0 on conditioned tokens, or NULL */
  int64_t T, S;
  float sigma, sigma_next, cfg_scale;
  int flags;
} ltx_dit_step_args;

/* Device bytes the context needs for steps of T latent tokens and S text tokens. */
size_t ltx_dit_workspace_bytes(const ltx_dit_config* cfg, int64_t T, int64_t S);
/* Sizes the context's workspace for (cfg, T, S): the one call of this library that
 * allocates device memory (cudaMalloc on the context's device; freed by
 * ltx_ctx_destroy). It also uploads the RoPE frequency grid (computed in float64 on the
 * host, ltx_nn.py:34-46). Synchronous. ltx_dit_step itself allocates nothing, so it can
 * be captured in a CUDA graph once reserved. */
int ltx_dit_reserve(ltx_ctx* ctx, const ltx_dit_config* cfg, int64_t T, int64_t S);
/* One CFG denoise step on `stream`: velocity (2, T, out) [cond; uncond] (may be NULL in
 * bf16), denoised (T, out) (may be NULL in bf16) and new_latent (T, out). The same
 * kernels with the same arguments as ltx_dit.cfg_denoise_step, so the results are
 * bit-identical. Calls on one context must not overlap in time. */
int ltx_dit_step(ltx_ctx* ctx, const ltx_dit_config* cfg, const ltx_dit_weights* weights, const ltx_dit_step_args* args,
                 void* velocity, void* denoised, void* new_latent, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LTXB200_H */
