// C-ABI of the sequence-parallel exchange layouts (kernels in elementwise.cu).
//
// Ulysses attention over P ranks: each rank holds T/P tokens with every head. Before
// attention, rank r sends to rank j the q/k/v/gate columns of j's heads for its own
// tokens (pack), so after NCCL's all-to-all rank j holds all T tokens of its heads in
// token order: exactly the (T, W) row-major operand the attention kernel reads. After
// attention the (T, D/P) output goes back the same way and unpack rebuilds the
// (T/P, D) rows the out-projection GEMM consumes.
#include <cstring>

#include "ltx_kernels.cuh"

using namespace ltx;
using namespace ltx::detail;

extern "C" int ltx_sp_pack(const void* src, int64_t ld_src, int64_t rows, int parts, int n_seg, const int* seg_off,
                           const int* seg_w, void* dst, int dtype, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_BF16 || dtype == LTX_F32, "dtype must be F32 or BF16");
  LTX_REQUIRE(src && dst && seg_off && seg_w, "NULL argument");
  LTX_REQUIRE(rows > 0 && parts > 0 && n_seg > 0 && n_seg <= 4, "bad sizes (1..4 segments)");
  const int esz = dtype == LTX_BF16 ? 2 : 4;
  const int vec = 16 / esz;  // elements per 16-byte move
  SpSegments seg{};
  seg.n = n_seg;
  int W = 0;
  for (int s = 0; s < n_seg; ++s) {
    LTX_REQUIRE(seg_w[s] > 0 && seg_off[s] >= 0, "segment widths must be positive, offsets non-negative");
    LTX_REQUIRE((seg_w[s] * esz) % 16 == 0 && (seg_off[s] * esz) % 16 == 0,
                "segment widths and offsets must be multiples of 16 bytes");
    LTX_REQUIRE(int64_t(seg_off[s]) + int64_t(parts) * seg_w[s] <= ld_src, "segment exceeds the source row");
    // the kernel counts in 8-element units of 16 bytes: express widths in bf16-equivalent elements
    seg.off[s] = seg_off[s] * esz / 2;
    seg.w[s] = seg_w[s] * esz / 2;
    W += seg.w[s];
  }
  seg.W = W;
  LTX_REQUIRE((ld_src * esz) % 16 == 0, "ld_src must be a multiple of 16 bytes");
  check_vec_ptr(src, "src");
  check_vec_ptr(dst, "dst");
  (void)vec;
  const int64_t total = int64_t(parts) * rows * (W / 8);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  launch_pdl(sp_pack_kernel, dim3(unsigned(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
             static_cast<const uint4*>(src), ld_src * esz / 16, rows, parts, seg, static_cast<uint4*>(dst));
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_sp_unpack(const void* src, int64_t rows, int parts, int w, void* dst, int64_t ld_dst, int dtype,
                             void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(dtype == LTX_BF16 || dtype == LTX_F32, "dtype must be F32 or BF16");
  LTX_REQUIRE(src && dst, "NULL argument");
  LTX_REQUIRE(rows > 0 && parts > 0 && w > 0, "bad sizes");
  const int esz = dtype == LTX_BF16 ? 2 : 4;
  LTX_REQUIRE((int64_t(w) * esz) % 16 == 0 && (ld_dst * esz) % 16 == 0, "w and ld_dst must be multiples of 16 bytes");
  LTX_REQUIRE(ld_dst >= int64_t(parts) * w, "ld_dst too small");
  check_vec_ptr(src, "src");
  check_vec_ptr(dst, "dst");
  const int w8 = int(int64_t(w) * esz / 16);
  const int64_t total = int64_t(parts) * rows * w8;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  launch_pdl(sp_unpack_kernel, dim3(unsigned(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
             static_cast<const uint4*>(src), rows, parts, w8, static_cast<uint4*>(dst), ld_dst * esz / 16);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

// ---------------------------------------------------------------------------------
// Split-KV attention across ranks (the video-to-audio attention under sequence
// parallelism: the audio queries attend to video keys that are sharded over the ranks).
// Each rank computes a partial attention over its keys (fp32 O / l and the log2-sum-exp
// of the scaled scores per (row, head)); after an all-gather every rank merges the R
// partials exactly as one softmax over all keys would weigh them:
//   M = max_r lse_r,  w_r = 2^(lse_r - M),  O = sum_r w_r O_r / sum_r w_r,
// then applies the output gate 2 * sigmoid(logit) with the roundings of the fused
// attention epilogue.
// ---------------------------------------------------------------------------------
namespace ltx {
namespace detail {

// One thread per (row, head, 8-column group).
__global__ void attn_merge_kernel(const float* __restrict__ o_parts, const float* __restrict__ lse_parts, int R,
                                  int64_t rows, int H, int D, const __nv_bfloat16* __restrict__ gate,
                                  int64_t ld_gate, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int g8 = D / 8;
  const int64_t total = rows * H * g8;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c8 = int(i % g8);
    const int64_t rh = i / g8;
    const int h = int(rh % H);
    const int64_t r = rh / H;
    float m = -INFINITY;
    for (int p = 0; p < R; ++p) m = fmaxf(m, lse_parts[(int64_t(p) * rows + r) * H + h]);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}, wsum = 0.f;
    for (int p = 0; p < R; ++p) {
      const float w = exp2f(lse_parts[(int64_t(p) * rows + r) * H + h] - m);
      const float* src = o_parts + (int64_t(p) * rows + r) * (int64_t(H) * D) + int64_t(h) * D + c8 * 8;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      acc[0] += w * a.x, acc[1] += w * a.y, acc[2] += w * a.z, acc[3] += w * a.w;
      acc[4] += w * b.x, acc[5] += w * b.y, acc[6] += w * b.z, acc[7] += w * b.w;
      wsum += w;
    }
    float g = 1.f;
    if (gate != nullptr) {
      const float sg = round_bf16(1.f / (1.f + expf(-__bfloat162float(gate[r * ld_gate + h]))));
      g = round_bf16(2.f * sg);
    }
    const float inv = 1.f / wsum;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float o = round_bf16(acc[e] * inv);
      v[e] = gate != nullptr ? o * g : o;
    }
    st8<__nv_bfloat16>(out + r * ldo + int64_t(h) * D + c8 * 8, v);
  }
}

}  // namespace detail
}  // namespace ltx

extern "C" int ltx_attention_partial(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                     float* o_part, int64_t ldo, float* lse, int64_t ld_lse, int B, int64_t Tq,
                                     int64_t Tk, int heads, int head_dim, float scale, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(q && k && v && o_part && lse, "NULL argument");
  LTX_REQUIRE(B > 0 && Tq > 0 && Tk > 0 && heads > 0, "B, Tq, Tk and heads must be positive");
  LTX_REQUIRE(int64_t(B) * Tq < (int64_t(1) << 31) && int64_t(B) * Tk < (int64_t(1) << 31), "too many rows");
  LTX_UNSUPPORTED(head_dim == 64 || head_dim == 128, "partial attention supports head_dim 64 and 128 (bf16)");
  const int64_t inner = int64_t(heads) * head_dim;
  LTX_REQUIRE(ldq >= inner && ldk >= inner && ldv >= inner && ldo >= inner, "leading dimensions too small");
  LTX_REQUIRE(ld_lse >= heads, "ld_lse must be >= heads");
  LTX_REQUIRE(ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && ldo % 4 == 0,
              "leading dims must be multiples of 8 (q, k, v) and 4 (o_part)");
  check_vec_ptr(q, "q");
  check_vec_ptr(k, "k");
  check_vec_ptr(v, "v");
  check_vec_ptr(o_part, "o_part");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    launch_fmha_tc<64>(q, ldq, k, ldk, v, ldv, nullptr, ldo, B, Tq, Tk, heads, scale, nullptr, 0, s, o_part, lse,
                       ld_lse);
  else
    launch_fmha_tc<128>(q, ldq, k, ldk, v, ldv, nullptr, ldo, B, Tq, Tk, heads, scale, nullptr, 0, s, o_part, lse,
                        ld_lse);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_attention_merge(const float* o_parts, const float* lse_parts, int parts, int64_t rows, int heads,
                                   int head_dim, const void* gate_logits, int64_t ld_gate, void* out, int64_t ldo,
                                   void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(o_parts && lse_parts && out, "NULL argument");
  LTX_REQUIRE(parts > 0 && rows > 0 && heads > 0 && head_dim > 0 && head_dim % 8 == 0, "bad sizes");
  LTX_REQUIRE(ldo >= int64_t(heads) * head_dim && ldo % 8 == 0, "ldo too small or not a multiple of 8");
  if (gate_logits) LTX_REQUIRE(ld_gate >= heads, "ld_gate must be >= heads");
  check_vec_ptr(o_parts, "o_parts");
  check_vec_ptr(out, "out");
  const int64_t total = rows * heads * (head_dim / 8);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  attn_merge_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      o_parts, lse_parts, parts, rows, heads, head_dim, static_cast<const __nv_bfloat16*>(gate_logits), ld_gate,
      static_cast<__nv_bfloat16*>(out), ldo),
      ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

// ---------------------------------------------------------------------------------
// Ulysses exchange over NVLink peer memory. Each SP rank owns one buffer (ltx_peer_alloc,
// shared through a CUDA IPC handle): the q/k pass writes every row's head blocks straight
// into the receive buffer of the rank that owns the heads, the attention epilogue writes
// every output row straight into the buffer of the rank that owns the token, and a flag
// barrier (ltx_sp_barrier) separates writers from readers. Kernels only store to peer
// memory; every load is local.
// ---------------------------------------------------------------------------------
namespace ltx {
namespace detail {

struct SpFlags {
  int* flag[8];  // flag[j]: SP rank j's flag array (one int per rank), as mapped here
};

LTX_DEVICE void st_release_sys(int* p, int v) { asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory"); }
LTX_DEVICE int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: count this barrier on this rank, publish the count in this rank's slot of
// every peer's flag array, then wait until every peer has published at least the same
// count here. All ranks pass the same sequence of barriers, so their counts agree; the
// count lives in device memory, so a captured graph replays correctly. The wait gives up
// after limit SM cycles: device error bit 2, and the kernel returns.
__global__ void sp_barrier_kernel(SpFlags f, int* counter, int parts, int rank, unsigned long long limit) {
  if (threadIdx.x != 0) return;
  const int epoch = *counter + 1;
  *counter = epoch;
  __threadfence_system();
  for (int j = 0; j < parts; ++j)
    if (j != rank) st_release_sys(f.flag[j] + rank, epoch);
  const unsigned long long t0 = clock64();
  for (int j = 0; j < parts; ++j) {
    if (j == rank) continue;
    while (ld_acquire_sys(f.flag[rank] + j) < epoch) {
      if (clock64() - t0 > limit) {
        ltx_flag_error(2);
        return;
      }
      __nanosleep(128);
    }
  }
  __threadfence_system();
}

}  // namespace detail
}  // namespace ltx

extern "C" int ltx_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  LTX_API_BEGIN
  LTX_REQUIRE(ptr != nullptr && ipc_handle != nullptr && bytes > 0, "bad argument");
  void* p = nullptr;
  LTX_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    LTX_CUDA(e);
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  LTX_API_END
}

extern "C" int ltx_peer_open(const void* ipc_handle, void** ptr) {
  LTX_API_BEGIN
  LTX_REQUIRE(ptr != nullptr && ipc_handle != nullptr, "bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  LTX_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  LTX_API_END
}

extern "C" int ltx_peer_close(void* ptr) {
  LTX_API_BEGIN
  if (ptr != nullptr) LTX_CUDA(cudaIpcCloseMemHandle(ptr));
  LTX_API_END
}

extern "C" int ltx_peer_free(void* ptr) {
  LTX_API_BEGIN
  if (ptr != nullptr) LTX_CUDA(cudaFree(ptr));
  LTX_API_END
}

extern "C" int ltx_sp_barrier(int* const* flags, int* counter, int parts, int rank, unsigned long long limit_cycles,
                              void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(flags != nullptr && counter != nullptr, "NULL argument");
  LTX_REQUIRE(parts >= 1 && parts <= 8 && rank >= 0 && rank < parts, "parts must be 1..8 and rank < parts");
  LTX_REQUIRE(limit_cycles > 0 && limit_cycles <= 20000000000ull, "limit must be in (0, 2e10] cycles");
  SpFlags f{};
  for (int j = 0; j < parts; ++j) {
    LTX_REQUIRE(flags[j] != nullptr, "flags[j] is NULL");
    f.flag[j] = flags[j];
  }
  sp_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, counter, parts, rank, limit_cycles),
      note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
