// Video VAE decoder kernels (lipaul/ltx-nv standalone/ltx_vae.py:20-222): the 3x3x3 /
// 1x1x1 convolution as an implicit GEMM on the tcgen05 tensor cores, and the
// channels-last element-wise stages around it (PixelNorm + SiLU, GroupNorm(1),
// depth-to-space, latent un-normalisation, output unpatchify).
//
// Activations are channels-last (B, F, H, W, C) bf16 so that the C input channels of a
// voxel are one contiguous row: the convolution's K dimension is (tap, channel) and an
// A-operand row of 64 channels is one 128-byte line.
#include <algorithm>

#include "ltx_kernels.cuh"

namespace ltx {
namespace detail {

struct ConvShape {
  int F, H, W;  // spatial size of input and output (stride 1, 'same' padding)
  int cin, cout;
  int taps;     // 27 (3x3x3) or 1 (1x1x1)
  int t_off;    // input frame of tap dt: clamp(f + dt + t_off, 0, F - 1)
  int bf;       // B * F frames
  int hb, wb;   // spatial block of one M tile: hb rows x wb columns of one frame, hb * wb = 128 * MH
  int th, tw;   // blocks per frame: ceil(H / hb) x ceil(W / wb)
  int norm_silu;  // 1: write silu(PixelNorm(conv + bias)) (all Cout channels in one tile)
  float eps;      // PixelNorm eps
};

// MH = 128-row halves of an M tile: 2 for BN <= 128 (256 voxels share each weight block,
// two M=128 accumulators), 1 for BN = 256 (TMEM holds 2 x 256 columns).
template <int BN, int MH>
struct ConvCfg {
  static constexpr int A_BYTES = MH * 128 * 64 * 2;  // 128 * MH voxels x 64 channels
  static constexpr int B_BYTES = BN * 64 * 2;        // BN output channels x 64 channels
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * MH * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
};

// Implicit-GEMM convolution, one CTA per SM, persistent over output tiles of 128 * MH
// voxels (an hb x wb block of one frame) by BN output channels. K = (tap, 64-channel
// block).
// The A operand of a k-block is the input block shifted by the tap, (64 channels, wb,
// hb, 1 frame), loaded by one 4-D TMA from the channels-last activation: the hardware
// zero-fills rows and columns outside the frame, and the frame coordinate is clamped
// (edge-frame padding). The box lands as 128 rows of 128 bytes in the 128B-swizzled
// K-major layout the MMA reads.
//   warp 0     TMA of the input block and of the weight block [BN x 64]
//   warp 1     TMEM allocation and the single-thread tcgen05.mma issue (MH x M=128, N=BN)
//   warps 2-5  epilogue: one TMEM lane quadrant each, + bias (+ residual), bf16 stores
// The TMEM accumulator is double-buffered so the epilogue of one tile overlaps the
// MMAs of the next.
template <int BN, int MH>
__global__ void __launch_bounds__(192, 1)
    conv3d_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* residual, __nv_bfloat16* out,
                     ConvShape cs) {
  using Cfg = ConvCfg<BN, MH>;
  constexpr int S = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::STAGE_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int cchunks = cs.cin / 64;
  const int k_blocks = cs.taps * cchunks;
  const int n_tiles = (cs.cout + BN - 1) / BN;
  const int per_frame = cs.th * cs.tw;
  const int num_tiles = cs.bf * per_frame * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mt = tile / n_tiles, n0 = (tile - mt * n_tiles) * BN;
        const int bf = mt / per_frame, rem = mt - bf * per_frame;
        const int h0 = (rem / cs.tw) * cs.hb, w0 = (rem % cs.tw) * cs.wb;
        const int f = bf % cs.F, fbase = bf - f;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], (uint32_t(it / S) & 1u) ^ 1u, abort_flag)) goto done;
          const int tap = kb / cchunks, cc = kb - tap * cchunks;
          int fi = f, dh = 0, dw = 0;
          if (cs.taps == 27) {
            fi = min(max(f + tap / 9 + cs.t_off, 0), cs.F - 1);
            dh = (tap / 3) % 3 - 1;
            dw = tap % 3 - 1;
          }
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          tma_load_4d(sa, &tmX, &full[s], cc * 64, w0 + dw, h0 + dh, fbase + fi);
          tma_load_2d(sa + Cfg::A_BYTES, &tmW, &full[s], kb * 64, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN, 0);
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t u = uint32_t(local >> 1);
        if (!mbar_wait(&tempty[acc], (u & 1u) ^ 1u, abort_flag)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * MH * BN);
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], uint32_t(it / S) & 1u, abort_flag)) goto done;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int h = 0; h < MH; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_ss(d_tmem + uint32_t(h * BN), umma_desc_sw128(a_addr + h * 16384 + k * 32, 16, 1024),
                      umma_desc_sw128(b_addr + k * 32, 16, 1024), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else {
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t u = uint32_t(local >> 1);
      const int mt = tile / n_tiles, n0 = (tile - mt * n_tiles) * BN;
      const int bf = mt / per_frame, rem = mt - bf * per_frame;
      if (!mbar_wait(&tfull[acc], u & 1u, abort_flag)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
      const int row = h * 128 + q * 32 + lane;
      const int rh = row / cs.wb, rw = row - rh * cs.wb;
      const int hh = (rem / cs.tw) * cs.hb + rh, ww = (rem % cs.tw) * cs.wb + rw;
      const bool live = hh < cs.H && ww < cs.W;
      const int64_t m = (int64_t(bf) * cs.H + hh) * cs.W + ww;
      const uint32_t tbase = tmem_base + uint32_t((acc * MH + h) * BN) + (uint32_t(q * 32) << 16);
      // PixelNorm of the voxel's Cout outputs (ltx_vae.py:20-28, then SiLU): a first pass
      // over the accumulator sums round(v^2) of v = round(conv + bias), as the reference's
      // x**2 and mean over the stored output do.
      float rden = 0.f;
      if (cs.norm_silu) {
        float ss = 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < BN && c0 < cs.cout; c0 += 32) {
          uint32_t rr[32];
          tmem_ld32(tbase + uint32_t(c0), rr);
          tmem_wait_ld();
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = c0 + g * 8;
            if (col < cs.cout) {
              float bb[8];
              ld8<__nv_bfloat16>(bias + col, bb);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float v = round_bf16(__uint_as_float(rr[g * 8 + e]) + bb[e]);
                ss += round_bf16(v * v);
              }
            }
          }
        }
        const float mean = round_bf16(ss / float(cs.cout));
        rden = 1.f / round_bf16(sqrtf(round_bf16(mean + cs.eps)));
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN && n0 + c0 < cs.cout; c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(tbase + uint32_t(c0), rr);
        tmem_wait_ld();
        if (live && cs.norm_silu) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = c0 + g * 8;
            if (col < cs.cout) {
              float v[8], bb[8];
              ld8<__nv_bfloat16>(bias + col, bb);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float a = round_bf16(round_bf16(__uint_as_float(rr[g * 8 + e]) + bb[e]) * rden);
                v[e] = __fdividef(a, 1.f + __expf(-a));
              }
              st8<__nv_bfloat16>(out + m * cs.cout + col, v);
            }
          }
        } else if (live) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = n0 + c0 + g * 8;
            if (col < cs.cout) {
              float v[8], bb[8];
              ld8<__nv_bfloat16>(bias + col, bb);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = round_bf16(__uint_as_float(rr[g * 8 + e]) + bb[e]);
              if (residual != nullptr) {
                float rs[8];
                ld8<__nv_bfloat16>(residual + m * cs.cout + col, rs);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += rs[e];
              }
              st8<__nv_bfloat16>(out + m * cs.cout + col, v);
            }
          }
        }
      }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
done:
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Spatial block of an M tile of `rows` voxels for an H x W frame: the (hb, wb) with
// hb * wb = rows whose blocks cover the frame with the fewest padded voxels (ties: the
// wider block).
void conv_block_shape(int H, int W, int rows, int& hb, int& wb) {
  int64_t best = -1;
  for (int w = rows; w >= 1; w >>= 1) {
    const int h = rows / w;
    const int64_t cover = int64_t((H + h - 1) / h) * h * (int64_t((W + w - 1) / w) * w);
    if (best < 0 || cover < best) {
      best = cover;
      hb = h;
      wb = w;
    }
  }
}

template <int BN, int MH>
void launch_conv(const void* x, int B, const void* w, const void* bias, const void* residual, void* out,
                 ConvShape cs, cudaStream_t s) {
  using Cfg = ConvCfg<BN, MH>;
  conv_block_shape(cs.H, cs.W, 128 * MH, cs.hb, cs.wb);
  cs.th = (cs.H + cs.hb - 1) / cs.hb;
  cs.tw = (cs.W + cs.wb - 1) / cs.wb;
  if (int64_t(cs.bf) * cs.th * cs.tw * ((cs.cout + BN - 1) / BN) >= (int64_t(1) << 31))
    throw ApiError{LTX_ERR_INVALID, "tensor too large"};
  const uint64_t k = uint64_t(cs.taps) * uint64_t(cs.cin);
  const CUtensorMap tw = make_tmap_bf16_2d(w, k, uint64_t(cs.cout), k, 64, BN);
  const uint64_t c2 = uint64_t(cs.cin) * 2;
  const uint64_t dims[4] = {uint64_t(cs.cin), uint64_t(cs.W), uint64_t(cs.H), uint64_t(B) * cs.F};
  // byte strides of W, H and frame
  const uint64_t strides[3] = {c2, c2 * cs.W, c2 * cs.W * cs.H};
  const uint32_t box[4] = {64, uint32_t(cs.wb), uint32_t(cs.hb), 1};
  const CUtensorMap tx = make_tmap_bf16_4d(x, dims, strides, box);
  auto kern = conv3d_tc_kernel<BN, MH>;
  static std::atomic<uint64_t> smem_done{0};
  ensure_smem_limit(smem_done, kern, Cfg::SMEM);
  const int64_t tiles = int64_t(cs.bf) * cs.th * cs.tw * ((cs.cout + BN - 1) / BN);
  const int grid = int(std::min<int64_t>(tiles, num_sms()));
  kern<<<grid, 192, Cfg::SMEM, s>>>(tx, tw, static_cast<const __nv_bfloat16*>(bias),
                                     static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), cs),
      ltx::note_launch();
}

// ---------------------------------------------------------------------------------
// Element-wise stages (channels-last rows of C channels)
// ---------------------------------------------------------------------------------

// PixelNorm (ltx_vae.py:20-28) over the C channels of each voxel, optionally followed by
// SiLU, with the bf16 roundings of the reference's tensor ops: x^2, mean, + eps, sqrt,
// division and SiLU each round to bf16. G lanes share a voxel and each holds V 16-byte
// chunks (8 channels) of it in registers: C = 8 * G * V, one read and one write per
// element.
template <int G, int V>
__global__ void __launch_bounds__(256) pixel_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                         __nv_bfloat16* __restrict__ y, int64_t rows, float eps,
                                                         int silu) {
  constexpr int C = 8 * G * V;
  constexpr int PER_WARP = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane / G, li = lane % G;
  const int64_t step = int64_t(gridDim.x) * 8 * PER_WARP;
  for (int64_t r0 = (int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5)) * PER_WARP; r0 < rows; r0 += step) {
    const int64_t r = r0 + sub;
    const bool live = r < rows;
    uint4 u[V];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      u[v] = live ? *reinterpret_cast<const uint4*>(x + r * C + (v * G + li) * 8) : make_uint4(0, 0, 0, 0);
      float a[8];
      unpack_bf16x2(u[v].x, a[0], a[1]);
      unpack_bf16x2(u[v].y, a[2], a[3]);
      unpack_bf16x2(u[v].z, a[4], a[5]);
      unpack_bf16x2(u[v].w, a[6], a[7]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += round_bf16(a[e] * a[e]);
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean = round_bf16(ss / float(C));
    const float den = round_bf16(sqrtf(round_bf16(mean + eps)));
    // x / den as x * (1 / den): within one fp32 ulp of the division, before the bf16
    // rounding; SiLU with the fast exponential and divide intrinsics
    const float rden = 1.f / den;
    if (!live) continue;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float a[8];
      unpack_bf16x2(u[v].x, a[0], a[1]);
      unpack_bf16x2(u[v].y, a[2], a[3]);
      unpack_bf16x2(u[v].z, a[4], a[5]);
      unpack_bf16x2(u[v].w, a[6], a[7]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a[e] = round_bf16(a[e] * rden);
        if (silu) a[e] = __fdividef(a[e], 1.f + __expf(-a[e]));
      }
      st8<__nv_bfloat16>(y + r * C + (v * G + li) * 8, a);
    }
  }
}

// Any other even C: one warp per voxel, two channels per lane step (two reads per element).
__global__ void __launch_bounds__(256) pixel_norm_generic_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 __nv_bfloat16* __restrict__ y, int64_t rows, int C,
                                                                 float eps, int silu) {
  const int64_t warps = int64_t(gridDim.x) * 8;
  for (int64_t r = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5); r < rows; r += warps) {
    const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + r * C);
    __nv_bfloat162* yr = reinterpret_cast<__nv_bfloat162*>(y + r * C);
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
    for (int j = lane; j < C / 2; j += 32) {
      const float2 v = __bfloat1622float2(xr[j]);
      ss += round_bf16(v.x * v.x) + round_bf16(v.y * v.y);
    }
    ss = warp_sum(ss);
    const float mean = round_bf16(ss / float(C));
    const float den = round_bf16(sqrtf(round_bf16(mean + eps)));
    for (int j = lane; j < C / 2; j += 32) {
      const float2 v = __bfloat1622float2(xr[j]);
      float a = round_bf16(v.x / den), b = round_bf16(v.y / den);
      if (silu) {
        a = a / (1.f + expf(-a));
        b = b / (1.f + expf(-b));
      }
      yr[j] = __floats2bfloat162_rn(a, b);
    }
  }
}

// GroupNorm with one group (ltx_vae.py:96, torch.nn.GroupNorm(1, C, eps=1e-6)): per sample
// the mean and variance of all F*H*W*C values. Pass 1: per-block partial sums (fp64) of
// value and square; pass 2: every block combines its sample's partials in block order
// (deterministic) and writes (x - mean) * rstd * w[c] + b[c], rounded once.
constexpr int kGnBlocks = 128;  // partial-sum blocks per sample

__global__ void __launch_bounds__(256) group_norm_stats_kernel(const __nv_bfloat16* __restrict__ x, int64_t n,
                                                               double* __restrict__ part) {
  const int b = blockIdx.y;
  const __nv_bfloat16* xs = x + int64_t(b) * n;
  double s = 0.0, s2 = 0.0;
  for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += int64_t(kGnBlocks) * 256) {
    const double v = double(__bfloat162float(xs[i]));
    s += v;
    s2 += v * v;
  }
  __shared__ double red[2][256];
  red[0][threadIdx.x] = s;
  red[1][threadIdx.x] = s2;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      red[0][threadIdx.x] += red[0][threadIdx.x + o];
      red[1][threadIdx.x] += red[1][threadIdx.x + o];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    part[(int64_t(b) * kGnBlocks + blockIdx.x) * 2] = red[0][0];
    part[(int64_t(b) * kGnBlocks + blockIdx.x) * 2 + 1] = red[1][0];
  }
}

__global__ void __launch_bounds__(256) group_norm_apply_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, int C,
                                                               const __nv_bfloat16* __restrict__ wt,
                                                               const __nv_bfloat16* __restrict__ bs, float eps,
                                                               const double* __restrict__ part,
                                                               __nv_bfloat16* __restrict__ y) {
  const int b = blockIdx.y;
  __shared__ float stat[2];
  if (threadIdx.x == 0) {
    double s = 0.0, s2 = 0.0;
    for (int i = 0; i < kGnBlocks; ++i) {
      s += part[(int64_t(b) * kGnBlocks + i) * 2];
      s2 += part[(int64_t(b) * kGnBlocks + i) * 2 + 1];
    }
    const double mean = s / double(n);
    const double var = std::max(s2 / double(n) - mean * mean, 0.0);
    stat[0] = float(mean);
    stat[1] = float(1.0 / sqrt(var + double(eps)));
  }
  __syncthreads();
  const float mean = stat[0], rstd = stat[1];
  const __nv_bfloat16* xs = x + int64_t(b) * n;
  __nv_bfloat16* ys = y + int64_t(b) * n;
  for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += int64_t(gridDim.x) * 256) {
    const int c = int(i % C);
    const float v = (__bfloat162float(xs[i]) - mean) * rstd * __bfloat162float(wt[c]) + __bfloat162float(bs[c]);
    ys[i] = __float2bfloat16_rn(v);
  }
}

// DepthToSpaceUpsample's rearrange (ltx_vae.py:135-143): input channel ((c*p1 + i)*p2 + j)*p3
// + k of voxel (d, h, w) goes to channel c of voxel (d*p1 + i - drop, h*p2 + j, w*p3 + k);
// with drop = 1 the first output frame is dropped. One thread per output (voxel, 8
// channels).
__global__ void __launch_bounds__(256) depth_to_space_kernel(const __nv_bfloat16* __restrict__ x,
                                                             __nv_bfloat16* __restrict__ y, int B, int F, int H,
                                                             int W, int c, int p1, int p2, int p3, int drop) {
  const int Fo = F * p1 - drop, Ho = H * p2, Wo = W * p3;
  const int cg = c / 8;
  const int64_t total = int64_t(B) * Fo * Ho * Wo * cg;
  const int cin = c * p1 * p2 * p3;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int g = int(i % cg);
    int64_t t = i / cg;
    const int wo = int(t % Wo);
    t /= Wo;
    const int ho = int(t % Ho);
    t /= Ho;
    const int fo = int(t % Fo);
    const int b = int(t / Fo);
    const int fd = fo + drop;
    const int d = fd / p1, ii = fd - d * p1, h = ho / p2, jj = ho - h * p2, w = wo / p3, kk = wo - w * p3;
    const __nv_bfloat16* src = x + (((int64_t(b) * F + d) * H + h) * W + w) * cin + (ii * p2 + jj) * p3 + kk;
    const int step = p1 * p2 * p3;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __bfloat162float(src[int64_t(g * 8 + e) * step]);
    st8<__nv_bfloat16>(y + i * 8, v);
  }
}

// The same rearrange read per input voxel: thread (voxel, g) loads the 8 * P contiguous
// input channels of output channels 8g..8g+7 (P = p1 * p2 * p3 subpositions, P 16-byte
// loads), transposes them in registers and stores 8 channels to each of the P output
// voxels (one 16-byte store each; 16-byte aligned output, c a multiple of 8).
template <int P>
__global__ void __launch_bounds__(256) depth_to_space_vox_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 __nv_bfloat16* __restrict__ y, int B, int F, int H,
                                                                 int W, int c, int p1, int p2, int p3, int drop) {
  const int Fo = F * p1 - drop, Ho = H * p2, Wo = W * p3;
  const int cg = c / 8;
  const int64_t total = int64_t(B) * F * H * W * cg;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int g = int(i % cg);
    const int64_t vox = i / cg;  // ((b * F + d) * H + h) * W + w
    const int w = int(vox % W);
    int64_t t = vox / W;
    const int h = int(t % H);
    t /= H;
    const int d = int(t % F);
    const int b = int(t / F);
    // in[e * P + s] = channel (8g + e) * P + s of the voxel: P chunks of 16 bytes
    uint32_t in[4 * P];
    const uint4* src = reinterpret_cast<const uint4*>(x + vox * (int64_t(c) * P) + int64_t(g) * 8 * P);
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const uint4 u = src[k];
      in[4 * k] = u.x;
      in[4 * k + 1] = u.y;
      in[4 * k + 2] = u.z;
      in[4 * k + 3] = u.w;
    }
    const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(in);
#pragma unroll
    for (int sidx = 0; sidx < P; ++sidx) {
      const int ii = sidx / (p2 * p3), jj = (sidx / p3) % p2, kk = sidx % p3;
      const int fo = d * p1 + ii - drop;
      if (fo < 0) continue;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __bfloat162float(hv[e * P + sidx]);
      st8<__nv_bfloat16>(y + (((int64_t(b) * Fo + fo) * Ho + h * p2 + jj) * Wo + w * p3 + kk) * c + g * 8, v);
    }
  }
}

// PerChannelStatistics.un_normalize (ltx_vae.py:83-87) and the NCDHW -> channels-last
// transpose of the latent: y[b,f,h,w,c] = round(round(x[b,c,f,h,w] * std[c]) + mean[c]), std
// and mean rounded to bf16 first (the reference's .to(x)).
__global__ void __launch_bounds__(256) vae_latent_in_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ stdv,
                                                            const float* __restrict__ meanv,
                                                            __nv_bfloat16* __restrict__ y, int B, int C,
                                                            int64_t fhw) {
  const int64_t total = int64_t(B) * C * fhw;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % C);
    const int64_t t = i / C;  // b * fhw + voxel
    const int64_t b = t / fhw, vox = t - b * fhw;
    const float v = __bfloat162float(x[(b * C + c) * fhw + vox]);
    y[i] = __float2bfloat16_rn(round_bf16(v * round_bf16(stdv[c])) + round_bf16(meanv[c]));
  }
}

// Output unpatchify (ltx_vae.py:212-216): channel ((c*p + r)*p + q) of voxel (f, h, w), q
// fastest, goes to pixel (h*p + q, w*p + r) of channel c. mode 0 writes the reference's
// (B, c, F, H*p, W*p) bf16 tensor; mode 1 writes decode_video's float (F, H*p, W*p, c)
// frames of sample 0 in [0, 1] ((v + 1) / 2, clamped).
__global__ void __launch_bounds__(256) vae_unpatchify_kernel(const __nv_bfloat16* __restrict__ x, void* out, int B,
                                                             int F, int H, int W, int c, int p, int mode) {
  const int Ho = H * p, Wo = W * p;
  const int64_t total = (mode == 0 ? int64_t(B) : 1) * c * F * Ho * Wo;
  const int cin = c * p * p;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int b, ch, f, ho, wo;
    int64_t t = i;
    if (mode == 0) {  // (B, c, F, Ho, Wo)
      wo = int(t % Wo);
      t /= Wo;
      ho = int(t % Ho);
      t /= Ho;
      f = int(t % F);
      t /= F;
      ch = int(t % c);
      b = int(t / c);
    } else {  // (F, Ho, Wo, c) of sample 0
      ch = int(t % c);
      t /= c;
      wo = int(t % Wo);
      t /= Wo;
      ho = int(t % Ho);
      f = int(t / Ho);
      b = 0;
    }
    const int h = ho / p, q = ho - h * p, w = wo / p, r = wo - w * p;
    const float v = __bfloat162float(x[(((int64_t(b) * F + f) * H + h) * W + w) * cin + (ch * p + r) * p + q]);
    if (mode == 0)
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else
      static_cast<float*>(out)[i] = fminf(fmaxf((v + 1.f) * 0.5f, 0.f), 1.f);
  }
}

// Mode 0 of the unpatchify with 8 consecutive output columns per thread (one 16-byte
// store): (W * p) % 8 == 0 and p dividing 8.
__global__ void __launch_bounds__(256) vae_unpatchify8_kernel(const __nv_bfloat16* __restrict__ x,
                                                              __nv_bfloat16* __restrict__ out, int B, int F, int H,
                                                              int W, int c, int p) {
  const int Ho = H * p, Wo = W * p, Wg = Wo / 8;
  const int64_t total = int64_t(B) * c * F * Ho * Wg;
  const int cin = c * p * p;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t t = i;
    const int wg = int(t % Wg);
    t /= Wg;
    const int ho = int(t % Ho);
    t /= Ho;
    const int f = int(t % F);
    t /= F;
    const int ch = int(t % c);
    const int b = int(t / c);
    const int h = ho / p, q = ho - h * p;
    const __nv_bfloat16* row = x + ((int64_t(b) * F + f) * H + h) * int64_t(W) * cin + (ch * p) * p + q;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int wo = wg * 8 + e, w = wo / p, r = wo - w * p;
      v[e] = __bfloat162float(row[int64_t(w) * cin + r * p]);
    }
    st8<__nv_bfloat16>(out + i * 8, v);
  }
}

int ew_grid(int64_t work, int per_block = 256) {
  const int64_t cap = int64_t(num_sms()) * 16;
  return int(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, cap)));
}

}  // namespace detail
}  // namespace ltx

using namespace ltx;
using namespace ltx::detail;

static void check16(const void* p, const char* what) {
  if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
    throw ApiError{LTX_ERR_INVALID, std::string(what) + " must be 16-byte aligned"};
}

extern "C" int ltx_conv3d(const void* x, int B, int F, int H, int W, int cin, const void* weight, const void* bias,
                          int cout, int ksize, int causal, const void* residual, void* out, void* stream) {
  return ltx_conv3d_norm(x, B, F, H, W, cin, weight, bias, cout, ksize, causal, residual, 0, 0.f, out, stream);
}

extern "C" int ltx_conv3d_norm(const void* x, int B, int F, int H, int W, int cin, const void* weight,
                               const void* bias, int cout, int ksize, int causal, const void* residual,
                               int norm_silu, float eps, void* out, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x && weight && bias && out, "x, weight, bias and out must be non-NULL");
  LTX_REQUIRE(ksize == 1 || ksize == 3, "ksize must be 1 or 3");
  LTX_REQUIRE(B > 0 && F > 0 && H > 0 && W > 0, "sizes must be positive");
  LTX_REQUIRE(cin > 0 && cin % 64 == 0, "cin must be a positive multiple of 64");
  LTX_REQUIRE(cout > 0 && cout % 8 == 0, "cout must be a positive multiple of 8");
  const int64_t m = int64_t(B) * F * H * W;
  LTX_REQUIRE(m < (int64_t(1) << 31) && m * std::max(cin, cout) < (int64_t(1) << 46), "tensor too large");
  LTX_REQUIRE(x != out && (residual == nullptr || residual != x), "out and residual must not alias x");
  check16(x, "x");
  check16(weight, "weight");
  check16(bias, "bias");
  check16(out, "out");
  if (residual) check16(residual, "residual");
  ConvShape cs;
  cs.F = F;
  cs.H = H;
  cs.W = W;
  cs.cin = cin;
  cs.cout = cout;
  cs.taps = ksize == 3 ? 27 : 1;
  cs.t_off = causal ? -2 : -1;
  cs.bf = B * F;
  cs.norm_silu = norm_silu ? 1 : 0;
  cs.eps = eps;
  LTX_REQUIRE(!norm_silu || (cout <= 256 && residual == nullptr),
              "the fused PixelNorm needs cout <= 256 (one tile per voxel row) and no residual");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cout <= 64)
    launch_conv<64, 2>(x, B, weight, bias, residual, out, cs, s);
  else if (cout <= 128)
    launch_conv<128, 2>(x, B, weight, bias, residual, out, cs, s);
  else
    launch_conv<256, 1>(x, B, weight, bias, residual, out, cs, s);
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_pixel_norm(const void* x, void* y, int64_t rows, int C, float eps, int silu, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x && y, "x and y must be non-NULL");
  LTX_REQUIRE(rows > 0 && C > 0 && C % 2 == 0, "rows must be positive and C even");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto xp = static_cast<const __nv_bfloat16*>(x);
  auto yp = static_cast<__nv_bfloat16*>(y);
  const int sl = silu ? 1 : 0;
  const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
  // voxels per 256-thread block: 8 warps x (32 / G)
  if (vec && C == 64)
    pixel_norm_kernel<8, 1><<<ew_grid(rows, 32), 256, 0, s>>>(xp, yp, rows, eps, sl), note_launch();
  else if (vec && C == 128)
    pixel_norm_kernel<16, 1><<<ew_grid(rows, 16), 256, 0, s>>>(xp, yp, rows, eps, sl), note_launch();
  else if (vec && C == 256)
    pixel_norm_kernel<32, 1><<<ew_grid(rows, 8), 256, 0, s>>>(xp, yp, rows, eps, sl), note_launch();
  else if (vec && C == 512)
    pixel_norm_kernel<32, 2><<<ew_grid(rows, 8), 256, 0, s>>>(xp, yp, rows, eps, sl), note_launch();
  else if (vec && C == 1024)
    pixel_norm_kernel<32, 4><<<ew_grid(rows, 8), 256, 0, s>>>(xp, yp, rows, eps, sl), note_launch();
  else
    pixel_norm_generic_kernel<<<ew_grid(rows, 8), 256, 0, s>>>(xp, yp, rows, C, eps, sl), note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int64_t ltx_group_norm1_workspace_bytes(int B) { return B > 0 ? int64_t(B) * kGnBlocks * 2 * 8 : -1; }

extern "C" int ltx_group_norm1(const void* x, int B, int64_t n_per_sample, int C, const void* weight,
                               const void* bias, float eps, void* workspace, int64_t ws_bytes, void* y,
                               void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x && weight && bias && workspace && y, "NULL argument");
  LTX_REQUIRE(B > 0 && C > 0 && n_per_sample > 0 && n_per_sample % C == 0, "bad sizes");
  LTX_REQUIRE(ws_bytes >= ltx_group_norm1_workspace_bytes(B), "workspace smaller than ltx_group_norm1_workspace_bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto part = static_cast<double*>(workspace);
  group_norm_stats_kernel<<<dim3(kGnBlocks, B), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n_per_sample,
                                                             part),
      note_launch();
  const int gx = std::max(1, std::min(ew_grid(n_per_sample), 1024));
  group_norm_apply_kernel<<<dim3(gx, B), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), n_per_sample, C, static_cast<const __nv_bfloat16*>(weight),
      static_cast<const __nv_bfloat16*>(bias), eps, part, static_cast<__nv_bfloat16*>(y)),
      note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_depth_to_space(const void* x, int B, int F, int H, int W, int c, int p1, int p2, int p3,
                                  int drop_first, void* y, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x && y && x != y, "x and y must be non-NULL and distinct");
  LTX_REQUIRE(B > 0 && F > 0 && H > 0 && W > 0 && c > 0 && c % 8 == 0, "bad sizes (c must be a multiple of 8)");
  LTX_REQUIRE(p1 >= 1 && p2 >= 1 && p3 >= 1 && p1 <= 4 && p2 <= 4 && p3 <= 4, "strides must be 1..4");
  LTX_REQUIRE(drop_first == 0 || (drop_first == 1 && F * p1 > 1), "drop_first must be 0 or 1");
  check16(y, "y");
  const int64_t work = int64_t(B) * (int64_t(F) * p1 - drop_first) * H * p2 * W * p3 * (c / 8);
  const int P = p1 * p2 * p3;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto xp = static_cast<const __nv_bfloat16*>(x);
  auto yp = static_cast<__nv_bfloat16*>(y);
  const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0;
  const int64_t vwork = int64_t(B) * F * H * W * (c / 8);
  if (vec && P == 8)
    depth_to_space_vox_kernel<8><<<ew_grid(vwork), 256, 0, s>>>(xp, yp, B, F, H, W, c, p1, p2, p3, drop_first),
        note_launch();
  else if (vec && P == 4)
    depth_to_space_vox_kernel<4><<<ew_grid(vwork), 256, 0, s>>>(xp, yp, B, F, H, W, c, p1, p2, p3, drop_first),
        note_launch();
  else if (vec && P == 2)
    depth_to_space_vox_kernel<2><<<ew_grid(vwork), 256, 0, s>>>(xp, yp, B, F, H, W, c, p1, p2, p3, drop_first),
        note_launch();
  else
    depth_to_space_kernel<<<ew_grid(work), 256, 0, s>>>(xp, yp, B, F, H, W, c, p1, p2, p3, drop_first),
        note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_vae_latent_in(const void* latent, int B, int C, int F, int H, int W, const float* std_of_means,
                                 const float* mean_of_means, void* y, void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(latent && std_of_means && mean_of_means && y, "NULL argument");
  LTX_REQUIRE(B > 0 && C > 0 && F > 0 && H > 0 && W > 0, "bad sizes");
  const int64_t fhw = int64_t(F) * H * W;
  vae_latent_in_kernel<<<ew_grid(int64_t(B) * C * fhw), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(latent), std_of_means, mean_of_means, static_cast<__nv_bfloat16*>(y), B, C,
      fhw),
      note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}

extern "C" int ltx_vae_unpatchify(const void* x, int B, int F, int H, int W, int c, int p, int mode, void* out,
                                  void* stream) {
  LTX_API_BEGIN
  LTX_REQUIRE(x && out, "NULL argument");
  LTX_REQUIRE(B > 0 && F > 0 && H > 0 && W > 0 && c > 0 && p > 0, "bad sizes");
  LTX_REQUIRE(mode == 0 || mode == 1, "mode must be 0 (bf16 NCDHW) or 1 (float frames of sample 0)");
  const int64_t work = (mode == 0 ? int64_t(B) : 1) * c * F * int64_t(H) * p * W * p;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mode == 0 && (int64_t(W) * p) % 8 == 0 && 8 % p == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0)
    vae_unpatchify8_kernel<<<ew_grid(work / 8), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                            static_cast<__nv_bfloat16*>(out), B, F, H, W, c, p),
        note_launch();
  else
    vae_unpatchify_kernel<<<ew_grid(work), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), out, B, F, H, W, c, p,
                                                        mode),
        note_launch();
  LTX_CUDA(cudaGetLastError());
  LTX_API_END
}
