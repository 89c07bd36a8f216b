// C-ABI of the sequence-parallel exchange layouts (kernels in elementwise.cu).
//
// Ulysses attention over P ranks: each rank holds T/P tokens with every head. Before
// attention, rank r sends to rank j the q/k/v/gate columns of j's heads for its own
// tokens (pack), so after NCCL's all-to-all rank j holds all T tokens of its heads in
// token order: exactly the (T, W) row-major operand the attention kernel reads. After
// attention the (T, D/P) output goes back the same way and unpack rebuilds the
// (T/P, D) rows the out-projection GEMM consumes.
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
  sp_pack_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), ld_src * esz / 16, rows, parts, seg, static_cast<uint4*>(dst)),
      ltx::note_launch();
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
  sp_unpack_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), rows, parts, w8, static_cast<uint4*>(dst), ld_dst * esz / 16),
      ltx::note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
