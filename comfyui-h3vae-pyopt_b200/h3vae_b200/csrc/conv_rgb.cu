// Decoder output conv: 3x3x3 fp16 conv from C (multiple of 64) channels to
// the 3 RGB channels, fp32 accumulate on tcgen05 (kind::f16).
//
// A 3-wide N tile would spend the whole kernel re-reading the 27 shifted
// input taps for almost no MMA work, so the taps are packed into N instead:
// for input row slab (kd, r) (128 consecutive padded columns w' of padded
// row r of frame t + kd),
//     Y_r[w', kh*9 + kw*3 + o] += sum_c in[w', c] * W[o, c, kd, kh, kw]
// with N = 32 (27 used): each slab is loaded once per kd and read once by
// its 4 MMAs.  The epilogue then forms, for output row i of the tile,
//     out[i][w] = sum_kh sum_kw Y_{i+kh}[w + kw, kh*9 + kw*3 + o] + bias[o]
// walking the input rows once with a sliding window of partial sums; the kw
// shift is a shift across TMEM lanes, done through shared memory.
//
// Tile = 6 output rows x 126 output columns of one (b, t): 8 input rows per
// kd, 128 A rows (126 outputs + the 2 columns the last ones reach).  Warps:
// 0 TMA (weights once, then A slabs through a ring of up to 12 stages), 1 TMEM owner +
// MMA issuer, 2..5 epilogue (one TMEM lane quadrant each).  Double-buffered
// TMEM accumulators (2 x 8 input rows x 32 columns).  Output: planar fp16
// [B, 3, T, H, W] (the layout of the decoder's result).
#include "common.cuh"

namespace h3b {

constexpr int kRgbRows = 6;                      // output rows per tile
constexpr int kRgbInRows = kRgbRows + 2;         // input rows per kd
constexpr int kRgbCols = 126;                    // output columns per tile
constexpr int kRgbN = 32;                        // MMA N: (kh, kw, o) packed, 27 used
constexpr int kRgbMaxStages = 12;
constexpr int kRgbEpiWarps = 4;
constexpr int kRgbThreads = 64 + 32 * kRgbEpiWarps;
constexpr uint32_t kRgbABytes = 128 * 128;       // 128 rows x 64 fp16 channels
constexpr uint32_t kRgbBBytes = kRgbN * 128;     // 32 rows x 64 fp16 channels
constexpr int kRgbMaxChunks = 4;                 // C <= 256

struct RgbParams {
  int B, T, H, W, C, c_chunks;
  int stages;           // A ring depth (as many 16 KB slabs as shared memory holds)
  int h_tiles, w_tiles, num_tiles;
  const __half* bias;   // [3] or nullptr
  __half* out;          // planar [B, 3, T, H, W]
};

__global__ void __launch_bounds__(kRgbThreads, 1)
    conv_rgb_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                    const RgbParams p) {
  constexpr uint32_t kIdesc = make_idesc_f16(128, kRgbN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_wtiles = 3 * p.c_chunks;           // (kd, chunk)
  uint8_t* smem_w = smem;                         // [kd][chunk] x 4 KB
  uint8_t* smem_a = smem + 3 * p.c_chunks * kRgbBBytes;
  float* xbuf = reinterpret_cast<float*>(smem_a + p.stages * kRgbABytes);   // [2][128][6]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xbuf + 2 * 128 * 6);
  uint64_t* w_full = bars;
  uint64_t* full = bars + 1;
  uint64_t* empty = full + kRgbMaxStages;
  uint64_t* t_full = empty + kRgbMaxStages;
  uint64_t* t_empty = t_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(t_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slabs = 3 * kRgbInRows * p.c_chunks;  // A loads per tile

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&t_full[a], 1);
      mbar_init(&t_empty[a], 32 * kRgbEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto tile_coords = [&](int tile, int& b, int& t, int& h0, int& w0) {
    int q = tile;
    const int wt = q % p.w_tiles; q /= p.w_tiles;
    const int ht = q % p.h_tiles; q /= p.h_tiles;
    t = q % p.T;
    b = q / p.T;
    h0 = ht * kRgbRows;
    w0 = wt * kRgbCols;
  };

  if (warp == 0) {
    // ---------------------------------- TMA ----------------------------------
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(w_full, n_wtiles * kRgbBBytes);
      for (int k = 0; k < n_wtiles; ++k)
        tma_load_2d(smem_w + k * kRgbBBytes, &map_w, w_full, (k % p.c_chunks) * 64, (k / p.c_chunks) * kRgbN);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int b, t, h0, w0;
        tile_coords(tile, b, t, h0, w0);
        for (int k = 0; k < slabs; ++k, ++it) {
          const int cc = k % p.c_chunks;
          const int r = (k / p.c_chunks) % kRgbInRows;
          const int kd = k / (p.c_chunks * kRgbInRows);
          const uint32_t s = it % p.stages;
          if (!mbar_poll(&empty[s], ((it / p.stages) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], kRgbABytes);
          tma_load_5d(smem_a + s * kRgbABytes, &map_x, &full[s], cc * 64, w0, h0 + r, t + kd, b);
        }
      }
      mbar_wait(w_full, 0, nullptr);
      for (uint32_t s = 0; s < p.stages && s < it; ++s) {
        const uint32_t last = it - 1 - ((it - 1 - s) % p.stages);
        mbar_wait(&full[s], (last / p.stages) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      bool ok = mbar_poll(w_full, 0, abort_flag);
      uint32_t it = 0, local = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const uint32_t acc = local & 1u;
        if (!mbar_poll(&t_empty[acc], ((local >> 1) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * (kRgbInRows * kRgbN);
        for (int k = 0; k < slabs && ok; ++k, ++it) {
          const int cc = k % p.c_chunks;
          const int r = (k / p.c_chunks) % kRgbInRows;
          const int kd = k / (p.c_chunks * kRgbInRows);
          const uint32_t s = it % p.stages;
          if (!mbar_poll(&full[s], (it / p.stages) & 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(smem_a + s * kRgbABytes));
          const uint64_t bdesc = make_sw128_desc(smem_u32(smem_w + (kd * p.c_chunks + cc) * kRgbBBytes));
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_f16(d0 + r * kRgbN, adesc + 2 * ks, bdesc + 2 * ks, kIdesc, (kd > 0 || cc > 0 || ks > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&t_full[acc]);
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;   // A row w' == TMEM lane
    const float b0 = p.bias != nullptr ? __half2float(p.bias[0]) : 0.0f;
    const float b1 = p.bias != nullptr ? __half2float(p.bias[1]) : 0.0f;
    const float b2 = p.bias != nullptr ? __half2float(p.bias[2]) : 0.0f;
    auto epi_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"r"(32 * kRgbEpiWarps) : "memory"); };
    const int64_t plane = static_cast<int64_t>(p.T) * p.H * p.W;
    uint32_t local = 0;
    int parity = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const uint32_t acc = local & 1u;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&t_full[acc], (local >> 1) & 1u, abort_flag));
      int b, t, h0, w0;
      tile_coords(tile, b, t, h0, w0);
      if (ok) tc_fence_after();
      const uint32_t t_row = tmem_base + acc * (kRgbInRows * kRgbN) + (static_cast<uint32_t>(quad * 32) << 16);
      // part[q][n]: running sum for output row (r - 2 + q) of this column, n = kw*3 + o
      float part[3][9];
#pragma unroll
      for (int q = 0; q < 3; ++q)
#pragma unroll
        for (int n = 0; n < 9; ++n) part[q][n] = 0.0f;
#pragma unroll 1
      for (int r = 0; r < kRgbInRows; ++r) {
        uint32_t y[32];
        if (ok) {
          tmem_ld32(t_row + r * kRgbN, y);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) y[k] = 0u;
        }
        // input row r feeds output rows r (kh = 0), r - 1 (kh = 1), r - 2 (kh = 2)
#pragma unroll
        for (int n = 0; n < 9; ++n) {
          part[0][n] = __fadd_rn(part[0][n], __uint_as_float(y[18 + n]));   // output row r - 2, now complete
          part[1][n] = __fadd_rn(part[1][n], __uint_as_float(y[9 + n]));    // output row r - 1
          part[2][n] = __fadd_rn(part[2][n], __uint_as_float(y[n]));        // output row r
        }
        if (r >= 2) {
          const int i = r - 2;
          float* xb = xbuf + parity * 128 * 6;
#pragma unroll
          for (int k = 0; k < 6; ++k) xb[row * 6 + k] = part[0][3 + k];
          epi_sync();
          const int w = w0 + row;
          const int h = h0 + i;
          if (row < kRgbCols && w < p.W && h < p.H && ok) {
            const float* n1 = xb + (row + 1) * 6;   // kw = 1 of column w+1
            const float* n2 = xb + (row + 2) * 6;   // kw = 2 of column w+2
            const float o0 = __fadd_rn(__fadd_rn(__fadd_rn(part[0][0], n1[0]), n2[3]), b0);
            const float o1 = __fadd_rn(__fadd_rn(__fadd_rn(part[0][1], n1[1]), n2[4]), b1);
            const float o2 = __fadd_rn(__fadd_rn(__fadd_rn(part[0][2], n1[2]), n2[5]), b2);
            __half* dst = p.out + ((static_cast<int64_t>(b) * 3 * p.T + t) * p.H + h) * p.W + w;
            dst[0] = __float2half_rn(o0);
            dst[plane] = __float2half_rn(o1);
            dst[2 * plane] = __float2half_rn(o2);
          }
          parity ^= 1;
        }
        // slide the window: row r - 1 becomes the oldest
#pragma unroll
        for (int n = 0; n < 9; ++n) {
          part[0][n] = part[1][n];
          part[1][n] = part[2][n];
          part[2][n] = 0.0f;
        }
      }
      tc_fence_before();
      mbar_arrive(&t_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace h3b

extern "C" int h3b_conv3d_rgb_f16(const void* x, const int64_t* x_dims, const void* w_packed, const void* bias,
                                  void* out, h3b_stream_t stream) {
  using namespace h3b;
  const char* name = "h3b_conv3d_rgb_f16";
  if (!x || !x_dims || !w_packed || !out) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  const int64_t B = x_dims[0], Dp = x_dims[1], Hp = x_dims[2], Wp = x_dims[3], C = x_dims[4];
  if (B <= 0 || Dp < 3 || Hp < 3 || Wp < 3 || C <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: bad input shape", name);
  if (C % 64 != 0 || C > 64 * kRgbMaxChunks)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: C=%lld must be a multiple of 64 up to 256", name, (long long)C);
  if (B * Dp * Hp * Wp * C >= (int64_t(1) << 40)) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: too large", name);
  if ((reinterpret_cast<uintptr_t>(out) & 1u) || (bias && (reinterpret_cast<uintptr_t>(bias) & 1u)))
    return h3b_host::set_error(H3B_EINVAL, "%s: misaligned output", name);
  RgbParams p{};
  p.B = (int)B; p.T = (int)(Dp - 2); p.H = (int)(Hp - 2); p.W = (int)(Wp - 2); p.C = (int)C;
  p.c_chunks = (int)(C / 64);
  p.h_tiles = (p.H + kRgbRows - 1) / kRgbRows;
  p.w_tiles = (p.W + kRgbCols - 1) / kRgbCols;
  const int64_t tiles = B * p.T * p.h_tiles * p.w_tiles;
  if (tiles >= (int64_t(1) << 31)) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: too many tiles", name);
  p.num_tiles = (int)tiles;
  p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(out);
  CUtensorMap mx, mw;
  uint64_t xdims[5] = {(uint64_t)C, (uint64_t)Wp, (uint64_t)Hp, (uint64_t)Dp, (uint64_t)B};
  uint64_t xstr[4] = {(uint64_t)(C * 2), (uint64_t)(C * Wp * 2), (uint64_t)(C * Wp * Hp * 2),
                      (uint64_t)(C * Wp * Hp * Dp * 2)};
  uint32_t xbox[5] = {64, 128, 1, 1, 1};
  uint32_t es5[5] = {1, 1, 1, 1, 1};
  int rc = h3b_host::encode_tiled(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, x, xdims, xstr, xbox, es5,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t wdims[2] = {(uint64_t)C, (uint64_t)(3 * kRgbN)};
  uint64_t wstr[1] = {(uint64_t)(C * 2)};
  uint32_t wbox[2] = {64, (uint32_t)kRgbN};
  uint32_t es2[2] = {1, 1};
  rc = h3b_host::encode_tiled(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w_packed, wdims, wstr, wbox, es2,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // Deep A ring: each 16 KB slab feeds only ~100 cycles of MMAs, so many loads
  // must be in flight to cover the L2 latency.
  constexpr size_t kFixed = 2 * 128 * 6 * 4 + (2 * kRgbMaxStages + 6) * 8 + 16 + 1024;
  const size_t wbytes = 3 * static_cast<size_t>(p.c_chunks) * kRgbBBytes;
  p.stages = static_cast<int>(std::min<size_t>(kRgbMaxStages, (232448 - kFixed - wbytes) / kRgbABytes));
  const size_t smem = wbytes + static_cast<size_t>(p.stages) * kRgbABytes + kFixed;
  cudaError_t e = cudaFuncSetAttribute(conv_rgb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int grid = (int)std::min<int64_t>(tiles, h3b_host::num_sms());
  conv_rgb_kernel<<<grid, kRgbThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mx, mw, p);
  return h3b_host::check_launch(name);
}
