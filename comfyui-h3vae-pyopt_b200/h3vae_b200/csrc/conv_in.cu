// Encoder input conv: pixel normalization + causal/reflect padding + the
// 3x3x3 conv from the few pixel channels to the first stage width, on the
// tcgen05 tensor cores (kind::f16, fp32 accumulate).
//
// A channel count of 3 does not fit a 128-byte TMA/MMA K row, so the im2col
// tile is built by threads instead of TMA:
//   1. pixel_pad_kernel writes the normalized, padded input once as
//      P[b][t+2][h+2][w+2][4] fp16 (channel 3 and the two causal frames are
//      zero): 8 bytes per padded pixel, a few tens of MB that stay in L2.
//   2. conv_in_kernel (persistent, two CTAs per SM): for each tile of 128
//      consecutive output pixels of one (b, t, h) row, 256 threads gather the
//      27 taps x 4 channels = 108 K values of each row (two taps per 16-byte
//      chunk) straight into a 128-byte-swizzled K-major A tile, one warp
//      issues 7 MMAs (K = 112) against the weight tile held in shared memory
//      for the whole kernel, and the same 256 threads run the epilogue of the
//      previous tile (tcgen05.ld, + bias, fp16 NDHWC store) while the MMA of
//      the current one runs.  Double-buffered A tiles and TMEM accumulators.
#include "common.cuh"

namespace h3b {

constexpr int kCinPad = 4;            // channels per padded pixel (8 bytes)
constexpr int kCinTaps = 27;
constexpr int kCinK = 112;            // 27 taps * 4 channels = 108, padded to 7 MMAs of K=16
constexpr int kCinChunks = kCinK / 8; // 16-byte chunks per A row
constexpr int kCinO = 128;            // output channels (the first stage width)
constexpr int kCinWorkers = 8;        // build + epilogue warps
constexpr int kCinThreads = 32 * (kCinWorkers + 1);
constexpr uint32_t kCinKBlockBytes = 128 * 128;   // 128 rows x 128 bytes
constexpr uint32_t kCinATileBytes = 2 * kCinKBlockBytes;
constexpr uint32_t kCinBTileBytes = 2 * kCinKBlockBytes;
constexpr uint32_t kCinStageBytes = 1024;   // per build/epilogue warp: 16 rows x 64 B of output staging
constexpr uint32_t kCinSmemBytes = 2 * kCinATileBytes + kCinBTileBytes + 1024 + 1024 + kCinWorkers * kCinStageBytes;

// 32 output rows (lane r = row r) x 32 fp16 channels to dst0 + r * row_stride
// through this warp's 1 KB staging buffer, 16 rows per pass: the rows' 16-byte
// chunks are XOR-swizzled so the shared accesses are conflict free, and each
// global store instruction writes 8 rows x 64 contiguous bytes (instead of 32
// rows x 16 B).  Warp-collective; rows >= valid_rows are not written.
__device__ __forceinline__ void cin_store_chunk32(uint32_t stage, const uint4 (&row)[4], __half* dst0,
                                                  int64_t row_stride, int valid_rows) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    if ((lane >> 4) == pass) {
      const int rl = lane & 15;
#pragma unroll
      for (int k = 0; k < 4; ++k) st_shared_v4(stage + rl * 64 + ((k ^ ((rl >> 1) & 3)) << 4), row[k]);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int rl = (lane >> 2) + 8 * i;
      const int k = lane & 3;
      const uint4 v = ld_shared_v4(stage + rl * 64 + ((k ^ ((rl >> 1) & 3)) << 4));
      const int r = pass * 16 + rl;
      if (r < valid_rows) *reinterpret_cast<uint4*>(dst0 + r * row_stride + k * 8) = v;
    }
    __syncwarp();
  }
}

// Byte offset of 16-byte chunk j (0..15) of row r (0..127) in a two-K-block,
// 128-byte-swizzled K-major tile (the layout TMA SWIZZLE_128B produces).
__device__ __forceinline__ uint32_t sw128_chunk_offset(int r, int j) {
  return static_cast<uint32_t>(j >> 3) * kCinKBlockBytes + static_cast<uint32_t>(r >> 3) * 1024u +
         static_cast<uint32_t>(r & 7) * 128u + static_cast<uint32_t>(((j & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ int reflect_index(int i, int n) {
  // PyTorch 'reflect' padding by one: -1 -> 1, n -> n - 2.
  if (i < 0) return -i;
  if (i >= n) return 2 * n - 2 - i;
  return i;
}

// One thread per padded pixel: normalize ((x + 1) * 0.5 - mean) / std in fp32,
// round to fp16 (the order of the host-side normalization), reflect / causal pad.
__global__ void pixel_pad_kernel(const __half* __restrict__ x, int B, int cin, int T, int H, int W, int64_t sB,
                                 int64_t sC, int64_t sT, int64_t sH, int64_t sW, const float* __restrict__ mean,
                                 const float* __restrict__ stdv, int reflect, uint2* __restrict__ P) {
  const int Hp = H + 2, Wp = W + 2, Tp = T + 2;
  const int64_t total = static_cast<int64_t>(B) * Tp * Hp * Wp;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t t = idx;
    const int wp = static_cast<int>(t % Wp); t /= Wp;
    const int hp = static_cast<int>(t % Hp); t /= Hp;
    const int tp = static_cast<int>(t % Tp);
    const int b = static_cast<int>(t / Tp);
    __align__(8) __half v[kCinPad] = {__float2half_rn(0.f), __float2half_rn(0.f), __float2half_rn(0.f),
                                      __float2half_rn(0.f)};
    int h = hp - 1, w = wp - 1;
    bool inside = tp >= 2;
    if (reflect) {
      h = reflect_index(h, H);
      w = reflect_index(w, W);
    } else {
      inside = inside && h >= 0 && h < H && w >= 0 && w < W;
    }
    if (inside) {
      const __half* src = x + b * sB + (tp - 2) * sT + h * sH + w * sW;
#pragma unroll
      for (int c = 0; c < kCinPad; ++c) {
        if (c < cin) {
          float f = __half2float(src[c * sC]);
          if (mean != nullptr) f = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(f, 1.0f), 0.5f), mean[c]), stdv[c]);
          v[c] = __float2half_rn(f);
        }
      }
    }
    P[idx] = *reinterpret_cast<const uint2*>(v);
  }
}

__global__ void __launch_bounds__(kCinThreads, 2)
    conv_in_kernel(const uint2* __restrict__ P, int B, int T, int H, int W, const __half* __restrict__ wgt,
                   int cin, const __half* __restrict__ bias, __half* __restrict__ out) {
  constexpr uint32_t kIdesc = make_idesc_f16(128, kCinO);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;                              // 2 stages
  uint8_t* smem_b = smem + 2 * kCinATileBytes;
  float* s_bias = reinterpret_cast<float*>(smem_b + kCinBTileBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_bias + kCinO);
  uint64_t* a_full = bars;        // [2], count = worker threads
  uint64_t* a_empty = bars + 2;   // [2], tcgen05.commit
  uint64_t* t_full = bars + 4;    // [2], tcgen05.commit
  uint64_t* t_empty = bars + 6;   // [2], count = worker threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Hp = H + 2, Wp = W + 2;
  const int w_tiles = (W + 127) / 128;
  const int num_tiles = B * T * H * w_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 32 * kCinWorkers);
      mbar_init(&a_empty[i], 1);
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 32 * kCinWorkers);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Weight tile: row o, K index k = tap * 4 + c, zero for c >= cin and k >= 108.
  for (int idx = threadIdx.x; idx < kCinO * kCinChunks; idx += blockDim.x) {
    const int o = idx / kCinChunks;
    const int j = idx - o * kCinChunks;
    __align__(16) __half v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int tap = 2 * j + (e >> 2);
      const int c = e & 3;
      v[e] = (tap < kCinTaps && c < cin) ? wgt[(static_cast<int64_t>(o) * kCinTaps + tap) * cin + c]
                                         : __float2half_rn(0.f);
    }
    *reinterpret_cast<uint4*>(smem_b + sw128_chunk_offset(o, j)) = *reinterpret_cast<const uint4*>(v);
  }
  for (int o = threadIdx.x; o < kCinO; o += blockDim.x) s_bias[o] = bias != nullptr ? __half2float(bias[o]) : 0.f;
  fence_proxy_async_smem();
  if (warp == kCinWorkers) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kCinWorkers) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      uint32_t i = 0;
      const uint64_t b0 = make_sw128_desc(smem_u32(smem_b));
      const uint64_t b1 = make_sw128_desc(smem_u32(smem_b + kCinKBlockBytes));
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
        const uint32_t s = i & 1u;
        const uint32_t ph = (i >> 1) & 1u;
        if (!mbar_wait(&a_full[s], ph, abort_flag)) break;
        if (!mbar_wait(&t_empty[s], ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint64_t a0 = make_sw128_desc(smem_u32(smem_a + s * kCinATileBytes));
        const uint64_t a1 = make_sw128_desc(smem_u32(smem_a + s * kCinATileBytes + kCinKBlockBytes));
        const uint32_t d = tmem_base + s * kCinO;
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16(d, a0 + 2 * k, b0 + 2 * k, kIdesc, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 3; ++k) mma_f16(d, a1 + 2 * k, b1 + 2 * k, kIdesc, 1u);
        tc_commit(&a_empty[s]);
        tc_commit(&t_full[s]);
      }
    }
  } else {
    // ---------------------- im2col build + epilogue warps ---------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;   // A row == TMEM lane == output pixel of the tile
    const int half = warp >> 2;         // chunks 0..6 / 7..13 while building; columns 0..63 / 64..127 after
    const uint32_t stage = smem_u32(smem_b + kCinBTileBytes + 2048) + warp * kCinStageBytes;
    auto epilogue = [&](int tile, uint32_t i) -> bool {
      const uint32_t s = i & 1u;
      // tcgen05.ld is warp-collective: leave together if any lane's wait gave up
      if (!__all_sync(0xffffffffu, mbar_wait(&t_full[s], (i >> 1) & 1u, abort_flag))) return false;
      tc_fence_after();
      int t = tile;
      const int wt = t % w_tiles; t /= w_tiles;
      const int h = t % H; t /= H;
      const int tt = t % T;
      const int b = t / T;
      const int w0 = wt * 128 + quad * 32;   // output column of lane 0 of this warp
      const uint32_t t_row = tmem_base + s * kCinO + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
      // the warp's 32 rows are consecutive pixels of one output row; those with w < W are stored
      __half* dst0 = out + ((((static_cast<int64_t>(b) * T + tt) * H + h) * W + w0) * kCinO) + half * 64;
      const int valid_rows = W - w0 < 32 ? W - w0 : 32;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);
        tmem_ld_wait();
        uint4 rowv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __align__(16) __half2 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = half * 64 + c * 32 + q * 8 + 2 * e;
            hv[e] = __floats2half2_rn(__fadd_rn(__uint_as_float(r[q * 8 + 2 * e]), s_bias[col]),
                                      __fadd_rn(__uint_as_float(r[q * 8 + 2 * e + 1]), s_bias[col + 1]));
          }
          rowv[q] = *reinterpret_cast<const uint4*>(hv);
        }
        if (valid_rows > 0) cin_store_chunk32(stage, rowv, dst0 + c * 32, kCinO, valid_rows);
      }
      tc_fence_before();
      mbar_arrive(&t_empty[s]);
      return true;
    };

    uint32_t i = 0;
    int prev_tile = -1;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++i) {
      const uint32_t s = i & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[s], ((i >> 1) & 1u) ^ 1u, abort_flag))) { ok = false; break; }
      int t = tile;
      const int wt = t % w_tiles; t /= w_tiles;
      const int h = t % H; t /= H;
      const int tt = t % T;
      const int b = t / T;
      const int w = min(wt * 128 + row, W - 1);   // rows past W gather valid pixels; their outputs are dropped
      // Padded input origin of this output pixel: frame tt (causal pad in front), row h, column w.
      const uint2* base = P + ((static_cast<int64_t>(b) * (T + 2) + tt) * Hp + h) * Wp + w;
      uint8_t* a_tile = smem_a + s * kCinATileBytes;
      const int j0 = half * 7;
#pragma unroll
      for (int jj = 0; jj < 7; ++jj) {
        const int j = j0 + jj;
        uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
        const int t0 = 2 * j, t1 = 2 * j + 1;
        // tap = kd * 9 + kh * 3 + kw
        lo = __ldg(base + ((t0 / 9) * Hp + (t0 / 3) % 3) * Wp + t0 % 3);
        if (t1 < kCinTaps) hi = __ldg(base + ((t1 / 9) * Hp + (t1 / 3) % 3) * Wp + t1 % 3);
        *reinterpret_cast<uint4*>(a_tile + sw128_chunk_offset(row, j)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
      fence_proxy_async_smem();
      mbar_arrive(&a_full[s]);
      if (prev_tile >= 0) ok = epilogue(prev_tile, i - 1);
      prev_tile = tile;
    }
    if (ok && prev_tile >= 0) epilogue(prev_tile, i - 1);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kCinWorkers) tmem_dealloc(tmem_base, 256);
}


// Rows of the causal 3x3x3 conv as a GEMM operand (the decoder's latent conv-in:
// 16 channels are narrower than one 128-byte K row of the implicit-GEMM conv,
// so its input is unrolled and multiplied by the library's fp16 GEMM).  Thread
// i -> (position m = i / 27, tap = i % 27): out[m, tap*C .. tap*C + C) holds
// the C channels of input frame t + kd - 2 (zero before frame 0: the two causal
// zero frames), row y + kh - 1 and column x + kw - 1, reflected at the edges
// (zero-padded instead when H or W is 1), exactly the padded tensor the conv
// reads.  Column order (kd, kh, kw, c) matches a [N, 3, 3, 3, C] weight.
__global__ void im2col_causal_kernel(const __half* __restrict__ x, int B, int C, int T, int H, int W, int64_t sB,
                                     int64_t sC, int64_t sT, int64_t sH, int64_t sW, int reflect, __half* out) {
  const int64_t total = static_cast<int64_t>(B) * T * H * W * 27;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int tap = static_cast<int>(i % 27);
    int64_t m = i / 27;
    const int xw = static_cast<int>(m % W);
    int64_t r = m / W;
    const int y = static_cast<int>(r % H);
    r /= H;
    const int t = static_cast<int>(r % T);
    const int b = static_cast<int>(r / T);
    const int kd = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
    const int ts = t + kd - 2;
    int ys = y + kh - 1, xs = xw + kw - 1;
    bool in = ts >= 0;
    if (reflect) {
      ys = ys < 0 ? -ys : (ys >= H ? 2 * H - 2 - ys : ys);
      xs = xs < 0 ? -xs : (xs >= W ? 2 * W - 2 - xs : xs);
    } else {
      in = in && ys >= 0 && ys < H && xs >= 0 && xs < W;
    }
    __half* dst = out + m * (27 * static_cast<int64_t>(C)) + tap * C;
    const __half* src = x + b * sB + static_cast<int64_t>(ts) * sT + static_cast<int64_t>(ys) * sH +
                        static_cast<int64_t>(xs) * sW;
    for (int c0 = 0; c0 < C; c0 += 8) {
      __align__(16) __half v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = in ? src[(c0 + k) * sC] : __float2half_rn(0.0f);
      *reinterpret_cast<uint4*>(dst + c0) = *reinterpret_cast<const uint4*>(v);
    }
  }
}

}  // namespace h3b

extern "C" {

int h3b_im2col_causal_f16(const void* x, const int64_t* dims5, const int64_t* strides5, void* out,
                          h3b_stream_t stream) {
  const char* name = "h3b_im2col_causal_f16";
  if (!x || !dims5 || !strides5 || !out) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  const int64_t B = dims5[0], C = dims5[1], T = dims5[2], H = dims5[3], W = dims5[4];
  if (B <= 0 || C <= 0 || T <= 0 || H <= 0 || W <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: empty input", name);
  if (C % 8 != 0) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: channels must be a multiple of 8, got %lld", name,
                                             (long long)C);
  if (B * T * H * W * 27 >= (int64_t(1) << 40) || C > 4096 || B > (int64_t(1) << 30) || T > (int64_t(1) << 30) ||
      H > (int64_t(1) << 30) || W > (int64_t(1) << 30))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: input too large", name);
  if (reinterpret_cast<uintptr_t>(out) & 15u) return h3b_host::set_error(H3B_EINVAL, "%s: out must be 16-byte aligned", name);
  const int reflect = (H > 1 && W > 1) ? 1 : 0;
  const int64_t total = B * T * H * W * 27;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(h3b_host::num_sms()) * 16);
  h3b::im2col_causal_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), (int)B, (int)C, (int)T, (int)H, (int)W, strides5[0], strides5[1], strides5[2],
      strides5[3], strides5[4], reflect, static_cast<__half*>(out));
  return h3b_host::check_launch(name);
}

size_t h3b_conv_in_workspace_size(int64_t B, int64_t T, int64_t H, int64_t W) {
  if (B <= 0 || T <= 0 || H <= 0 || W <= 0) return 0;
  return static_cast<size_t>(B * (T + 2) * (H + 2) * (W + 2)) * sizeof(uint2);
}

int h3b_conv_in_f16(const void* x, const int64_t* dims5, const int64_t* strides5, const float* norm_mean,
                    const float* norm_std, const void* w, int64_t out_channels, const void* bias, void* out,
                    void* workspace, size_t workspace_bytes, h3b_stream_t stream) {
  const char* name = "h3b_conv_in_f16";
  if (!x || !dims5 || !strides5 || !w || !out || !workspace) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  const int64_t B = dims5[0], cin = dims5[1], T = dims5[2], H = dims5[3], W = dims5[4];
  if (B <= 0 || T <= 0 || H <= 0 || W <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: empty input", name);
  if (cin < 1 || cin > h3b::kCinPad)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: 1..4 input channels supported, got %lld", name, (long long)cin);
  if (out_channels != h3b::kCinO)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: %d output channels supported, got %lld", name, h3b::kCinO,
                               (long long)out_channels);
  if ((norm_mean == nullptr) != (norm_std == nullptr))
    return h3b_host::set_error(H3B_EINVAL, "%s: pass both normalization vectors or neither", name);
  if (B * (T + 2) * (H + 2) * (W + 2) >= (int64_t(1) << 40) || B * T * H * ((W + 127) / 128) >= (int64_t(1) << 31))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: input too large", name);
  if (workspace_bytes < h3b_conv_in_workspace_size(B, T, H, W))
    return h3b_host::set_error(H3B_EINVAL, "%s: workspace too small", name);
  if ((reinterpret_cast<uintptr_t>(out) & 15u) || (reinterpret_cast<uintptr_t>(workspace) & 7u))
    return h3b_host::set_error(H3B_EINVAL, "%s: out must be 16-byte and workspace 8-byte aligned", name);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint2* P = static_cast<uint2*>(workspace);
  const int reflect = (H > 1 && W > 1) ? 1 : 0;
  const int64_t total = B * (T + 2) * (H + 2) * (W + 2);
  const int sms = h3b_host::num_sms();
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(sms) * 16);
  h3b::pixel_pad_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __half*>(x), (int)B, (int)cin, (int)T, (int)H, (int)W, strides5[0], strides5[1], strides5[2],
      strides5[3], strides5[4], norm_mean, norm_std, reflect, P);
  int rc = h3b_host::check_launch(name);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(h3b::conv_in_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(h3b::kCinSmemBytes));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int64_t tiles = B * T * H * ((W + 127) / 128);
  // ~98 KB of shared memory and 256 TMEM columns: two CTAs per SM hide the gather latency.
  const int grid = static_cast<int>(std::min<int64_t>(tiles, 2 * static_cast<int64_t>(sms)));
  h3b::conv_in_kernel<<<grid, h3b::kCinThreads, h3b::kCinSmemBytes, st>>>(
      P, (int)B, (int)T, (int)H, (int)W, static_cast<const __half*>(w), (int)cin, static_cast<const __half*>(bias),
      static_cast<__half*>(out));
  return h3b_host::check_launch(name);
}

}  // extern "C"
