// tcgen05 kind::i8 mainloop shared by the implicit-GEMM causal conv3d and the
// decoder INT8 linears.
//
// Structure (one persistent CTA per SM, 10 warps):
//   warp 0      TMA producer: A tile (128 rows x 128 int8 of K) and B tile
//               (BN rows x 128 int8 of K) per k-block into a STAGES-deep ring
//               of 128-byte-swizzled shared-memory buffers.
//   warp 1      TMEM owner + MMA issuer: 4 x tcgen05.mma (K=32 each) per
//               k-block into one of two TMEM accumulators (2 x BN int32 columns).
//   warps 2..9  epilogue: tcgen05.ld of the finished accumulator (one TMEM
//               lane = one output row per thread; the two warps of a lane
//               quadrant take alternate 32-column chunks), dequantize, fused
//               op, store.
// The double-buffered accumulator lets the epilogue of tile i overlap the
// mainloop of tile i+1.
//
// Conv mode: the A operand of output tile (b, od, rows oh0.., cols ow0..) for
// tap (kd, kh, kw) and channel chunk c0 is one 5-D TMA box
// {128 channels, bw, bh, 1, 1} at (c0, ow0+kw, oh0+kh, od+kd, b) of the padded
// NDHWC int8 input -- the im2col tile is never materialized.  Output frames
// od < 2 start at tap kd = 2 - od when the producer guarantees two zero causal
// frames (integer zero products are skipped, the sum is unchanged).
#include "common.cuh"

namespace h3b {

enum class AMode : int { kGemm2D = 0, kConv5D = 1 };
enum class Epi : int { kLinear = 0, kConv = 1, kSwiGLU = 2, kQkvRope = 3 };

struct MmaParams {
  int M, N, K;          // GEMM view (conv: N = out channels)
  int m_tiles, n_tiles;
  int k_blocks;         // GEMM: ceil(K / 128); conv: taps * c_chunks
  // conv geometry
  int B, Do, Ho, Wo;
  int kd, kh, kw, taps, c_chunks, C;
  int bw, bh, w_tiles, h_tiles;
  int causal;
  // epilogue operands
  const float* a_scale;  // GEMM: [M] per row; conv: scalar
  const float* w_scale;  // [N] (SwiGLU: [2F])
  const __half* bias;    // [N] or nullptr
  __half* out;
  int64_t ldo;           // GEMM row stride of out
  int64_t osB, osD, osH, osW;
  int32_t* acc_out;
  const __half* residual;  // conv: optional fp16 tensor added after the fp16 rounding (same strides as out)
  // SwiGLU
  int F;
  // QKV + RoPE
  int heads, tokens, R;
  float eps;
  const __half* cos_t;
  const __half* sin_t;
  __half* q_out;
  __half* k_out;
  __half* v_out;
};

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage = 4 MMAs of K=32
constexpr int kEpiWarps = 8;   // two warps per TMEM lane quadrant, splitting the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kATileBytes = kBM * kBK;

// Column stride between the two TMEM accumulators (kept a power of two) and
// the power-of-two allocation that holds both.
template <int BN>
struct TmemLayout {
  static constexpr uint32_t acc_stride = (BN <= 32) ? 32 : (BN <= 64) ? 64 : (BN <= 128) ? 128 : 256;
  static constexpr uint32_t cols = 2 * acc_stride;
};

// ---------------------------------------------------------------------------
// Epilogue helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float dequant(uint32_t acc_bits, float sx, float ws, const __half* bias, int n) {
  float v = __fmul_rn(static_cast<float>(static_cast<int32_t>(acc_bits)), sx);
  if (bias != nullptr) return __fmaf_rn(v, ws, __half2float(bias[n]));
  return __fmul_rn(v, ws);
}

__device__ __forceinline__ void store_row_chunk(__half* dst, const float (&v)[32], int valid_cols, bool vec_ok) {
  if (valid_cols >= 32 && vec_ok) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __align__(16) __half2 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
      *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<uint4*>(h);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid_cols) dst[j] = __float2half_rn(v[j]);
  }
}

__device__ __forceinline__ void store_acc_chunk(int32_t* dst, const uint32_t (&r)[32], int valid_cols) {
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < valid_cols) dst[j] = static_cast<int32_t>(r[j]);
}

// v = fp16(fp16(v) + residual): the residual block's `x + h` on fp16 tensors.
__device__ __forceinline__ void add_residual_chunk(float (&v)[32], const __half* res, int valid_cols, bool vec_ok) {
  if (valid_cols >= 32 && vec_ok) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 raw = *reinterpret_cast<const uint4*>(res + q * 8);
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[q * 8 + 2 * j] = __fadd_rn(round_fp16(v[q * 8 + 2 * j]), f.x);
        v[q * 8 + 2 * j + 1] = __fadd_rn(round_fp16(v[q * 8 + 2 * j + 1]), f.y);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid_cols) v[j] = __fadd_rn(round_fp16(v[j]), __half2float(res[j]));
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES, AMode AM, Epi EP>
__global__ void __launch_bounds__(kThreads, 1)
    mma_i8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const MmaParams p) {
  constexpr uint32_t kBTileBytes = BN * kBK;
  constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  constexpr uint32_t kTmemCols = TmemLayout<BN>::cols;
  constexpr uint32_t kAccStride = TmemLayout<BN>::acc_stride;
  constexpr uint32_t kIdesc = make_idesc_i8(kBM, BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * kATileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one_sync()) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_tile = tile / p.n_tiles;
        const int n_tile = tile - m_tile * p.n_tiles;
        int kb_begin = 0, kb_end = p.k_blocks;
        int b = 0, od = 0, oh0 = 0, ow0 = 0;
        if constexpr (AM == AMode::kConv5D) {
          int t = m_tile;
          const int tw = t % p.w_tiles; t /= p.w_tiles;
          const int th = t % p.h_tiles; t /= p.h_tiles;
          od = t % p.Do;
          b = t / p.Do;
          oh0 = th * p.bh;
          ow0 = tw * p.bw;
          if (p.causal && od < 2) kb_begin = (2 - od) * p.kh * p.kw * p.c_chunks;
        }
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
          uint8_t* sa = smem_a + s * kATileBytes;
          uint8_t* sb = smem_b + s * kBTileBytes;
          if constexpr (AM == AMode::kConv5D) {
            const int tap = kb / p.c_chunks;
            const int cc = kb - tap * p.c_chunks;
            const int tkw = tap % p.kw;
            const int tkh = (tap / p.kw) % p.kh;
            const int tkd = tap / (p.kw * p.kh);
            tma_load_5d(sa, &map_a, &full_bar[s], cc * kBK, ow0 + tkw, oh0 + tkh, od + tkd, b);
            tma_load_2d(sb, &map_b, &full_bar[s], kb * kBK, n_tile * BN);
          } else {
            tma_load_2d(sa, &map_a, &full_bar[s], kb * kBK, m_tile * kBM);
            if constexpr (EP == Epi::kSwiGLU) {
              const int j0 = n_tile * (BN / 2);
              tma_load_2d(sb, &map_b, &full_bar[s], kb * kBK, j0);
              tma_load_2d(sb + (BN / 2) * kBK, &map_b, &full_bar[s], kb * kBK, p.F + j0);
            } else {
              tma_load_2d(sb, &map_b, &full_bar[s], kb * kBK, n_tile * BN);
            }
          }
        }
      }
      // Drain: make sure no TMA write into this CTA's shared memory is still in
      // flight before the CTA can exit (bounded).
      for (uint32_t s = 0; s < STAGES && s < it; ++s) {
        const uint32_t last = it - 1 - ((it - 1 - s) % STAGES);
        mbar_wait(&full_bar[s], (last / STAGES) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      uint32_t it = 0;
      uint32_t local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        int kb_begin = 0;
        if constexpr (AM == AMode::kConv5D) {
          if (p.causal) {
            const int m_tile = tile / p.n_tiles;
            const int od = (m_tile / (p.w_tiles * p.h_tiles)) % p.Do;
            if (od < 2) kb_begin = (2 - od) * p.kh * p.kw * p.c_chunks;
          }
        }
        const uint32_t acc = local & 1u;
        const uint32_t aph = (local >> 1) & 1u;
        if (!mbar_wait(&tempty_bar[acc], aph ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccStride;
        for (int kb = kb_begin; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(smem_a + s * kATileBytes));
          const uint64_t bdesc = make_sw128_desc(smem_u32(smem_b + s * kBTileBytes));
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            // Advance the start address by 32 bytes (2 x 16 B) per K=32 step.
            mma_i8(d_tmem, adesc + 2 * k, bdesc + 2 * k, kIdesc, (kb > kb_begin || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[s]);
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int quad = warp & 3;          // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;   // tile row == TMEM lane
    const int half = (warp - 2) >> 2;   // 0 / 1: which alternate column chunks this warp owns
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int m_tile = tile / p.n_tiles;
      const int n_tile = tile - m_tile * p.n_tiles;
      const uint32_t acc = local & 1u;
      const uint32_t aph = (local >> 1) & 1u;
      if (!mbar_wait(&tfull_bar[acc], aph, abort_flag)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * kAccStride + (static_cast<uint32_t>(quad * 32) << 16);

      if constexpr (EP == Epi::kLinear) {
        const int64_t m = static_cast<int64_t>(m_tile) * kBM + row;
        const bool valid = m < p.M;
        const float sx = valid ? p.a_scale[m] : 0.0f;
        const bool vec_ok = (p.ldo % 8) == 0;
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait();
          const int n0 = n_tile * BN + c * 32;
          const int valid_cols = p.N - n0;
          if (valid && valid_cols > 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = min(n0 + j, p.N - 1);
              v[j] = dequant(r[j], sx, p.w_scale[n], p.bias, n);
            }
            store_row_chunk(p.out + m * p.ldo + n0, v, valid_cols, vec_ok);
            if (p.acc_out != nullptr) store_acc_chunk(p.acc_out + m * p.N + n0, r, valid_cols);
          }
        }
      } else if constexpr (EP == Epi::kConv) {
        int t = m_tile;
        const int tw = t % p.w_tiles; t /= p.w_tiles;
        const int th = t % p.h_tiles; t /= p.h_tiles;
        const int od = t % p.Do;
        const int b = t / p.Do;
        const int oh = th * p.bh + row / p.bw;
        const int ow = tw * p.bw + row % p.bw;
        const bool valid = (oh < p.Ho) && (ow < p.Wo);
        const float sx = *p.a_scale;
        const int64_t obase = b * p.osB + od * p.osD + static_cast<int64_t>(oh) * p.osH + static_cast<int64_t>(ow) * p.osW;
        const int64_t pos = ((static_cast<int64_t>(b) * p.Do + od) * p.Ho + oh) * p.Wo + ow;
        const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && (p.osW % 8 == 0) &&
                            (p.osH % 8 == 0) && (p.osD % 8 == 0) && (p.osB % 8 == 0);
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait();
          const int n0 = n_tile * BN + c * 32;
          const int valid_cols = p.N - n0;
          if (valid && valid_cols > 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = min(n0 + j, p.N - 1);
              v[j] = dequant(r[j], sx, p.w_scale[n], p.bias, n);
            }
            if (p.residual != nullptr) add_residual_chunk(v, p.residual + obase + n0, valid_cols, vec_ok);
            store_row_chunk(p.out + obase + n0, v, valid_cols, vec_ok);
            if (p.acc_out != nullptr) store_acc_chunk(p.acc_out + pos * p.N + n0, r, valid_cols);
          }
        }
      } else if constexpr (EP == Epi::kSwiGLU) {
        const int64_t m = static_cast<int64_t>(m_tile) * kBM + row;
        const bool valid = m < p.M;
        const float sx = valid ? p.a_scale[m] : 0.0f;
        const bool vec_ok = (p.F % 8) == 0;
#pragma unroll 1
        for (int c = half; c < BN / 64; c += 2) {
          uint32_t rg[32], ru[32];
          tmem_ld32(t_row + c * 32, rg);
          tmem_ld32(t_row + BN / 2 + c * 32, ru);
          tmem_ld_wait();
          const int j0 = n_tile * (BN / 2) + c * 32;
          const int valid_cols = p.F - j0;
          if (valid && valid_cols > 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int jj = min(j0 + j, p.F - 1);
              const float g = round_fp16(dequant(rg[j], sx, p.w_scale[jj], p.bias, jj));
              const float u = round_fp16(dequant(ru[j], sx, p.w_scale[p.F + jj], p.bias, p.F + jj));
              const float sg = __fdividef(g, __fadd_rn(1.0f, expf(-g)));
              v[j] = __fmul_rn(sg, u);
            }
            store_row_chunk(p.out + m * p.F + j0, v, valid_cols, vec_ok);
          }
        }
      } else if constexpr (EP == Epi::kQkvRope) {
        // BN == 192: this tile is one head's [q | k | v] for 128 tokens.
        const int64_t m = static_cast<int64_t>(m_tile) * kBM + row;
        const bool valid = m < p.M;
        const float sx = valid ? p.a_scale[m] : 0.0f;
        const int h = n_tile;
        const int64_t bb = valid ? m / p.tokens : 0;
        const int64_t tt = valid ? m - bb * p.tokens : 0;
        const int64_t dst_off = ((bb * p.heads + h) * p.tokens + tt) * 64;
#pragma unroll 1
        for (int part = half; part < 3; part += 2) {
          float x[64];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld32(t_row + part * 64 + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = h * 192 + part * 64 + c * 32 + j;
              x[c * 32 + j] = valid ? round_fp16(dequant(r[j], sx, p.w_scale[n], p.bias, n)) : 0.0f;
            }
          }
          if (valid) {
            if (part < 2) {
              qk_norm_rope_store(x, p.eps, p.R, p.cos_t + m * p.R, p.sin_t + m * p.R,
                                 (part == 0 ? p.q_out : p.k_out) + dst_off);
            } else {
              __align__(16) __half outv[64];
#pragma unroll
              for (int d = 0; d < 64; ++d) outv[d] = __float2half_rn(x[d]);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                reinterpret_cast<uint4*>(p.v_out + dst_off)[q] = reinterpret_cast<const uint4*>(outv)[q];
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// ---------------------------------------------------------------------------
// Generic SIMT fallback for conv geometries outside the TMA contract
// (channel counts not a multiple of 128, stride 2, 1-wide temporal kernels
// mixed with strides).  Exact int32 accumulation, same epilogue.
// ---------------------------------------------------------------------------
__global__ void conv3d_i8_simt_kernel(const int8_t* __restrict__ qx, int B, int D, int H, int W, int C,
                                      const int8_t* __restrict__ qw, int O, int kd, int kh, int kw, int sd,
                                      int sh, int sw, int Do, int Ho, int Wo, const float* x_scale,
                                      const float* __restrict__ w_scale, const __half* __restrict__ bias,
                                      __half* out, int64_t osB, int64_t osD, int64_t osH, int64_t osW,
                                      int32_t* acc_out, const __half* residual) {
  const int64_t total = static_cast<int64_t>(B) * Do * Ho * Wo * O;
  const int64_t ktot = static_cast<int64_t>(kd) * kh * kw * C;
  const float sx = *x_scale;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(idx % O);
    int64_t pos = idx / O;
    const int ow = static_cast<int>(pos % Wo);
    int64_t t = pos / Wo;
    const int oh = static_cast<int>(t % Ho);
    t /= Ho;
    const int od = static_cast<int>(t % Do);
    const int b = static_cast<int>(t / Do);
    int32_t acc = 0;
    for (int a = 0; a < kd; ++a)
      for (int bh = 0; bh < kh; ++bh)
        for (int cw = 0; cw < kw; ++cw) {
          const int64_t in_off =
              ((((static_cast<int64_t>(b) * D + od * sd + a) * H + oh * sh + bh) * W) + ow * sw + cw) * C;
          const int64_t w_off = n * ktot + ((static_cast<int64_t>(a) * kh + bh) * kw + cw) * C;
          for (int c = 0; c < C; ++c) acc += static_cast<int32_t>(qx[in_off + c]) * static_cast<int32_t>(qw[w_off + c]);
        }
    float v = __fmul_rn(static_cast<float>(acc), sx);
    v = (bias != nullptr) ? __fmaf_rn(v, w_scale[n], __half2float(bias[n])) : __fmul_rn(v, w_scale[n]);
    const int64_t o_off = b * osB + od * osD + oh * osH + ow * osW + n;
    if (residual != nullptr) v = __fadd_rn(round_fp16(v), __half2float(residual[o_off]));
    out[o_off] = __float2half_rn(v);
    if (acc_out != nullptr) acc_out[pos * O + n] = acc;
  }
}

}  // namespace h3b

// ===========================================================================
// Host launchers
// ===========================================================================
namespace {

using namespace h3b;

template <int BN, int STAGES, AMode AM, Epi EP>
int launch_mma(const CUtensorMap& ma, const CUtensorMap& mb, const MmaParams& p, cudaStream_t stream,
               const char* name) {
  constexpr size_t smem = STAGES * (kATileBytes + BN * kBK) + 1024 + 256;
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = mma_i8_kernel<BN, STAGES, AM, EP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int tiles = p.m_tiles * p.n_tiles;
  if (tiles <= 0) return H3B_OK;
  const int grid = tiles < h3b_host::num_sms() ? tiles : h3b_host::num_sms();
  kern<<<grid, kThreads, smem, stream>>>(ma, mb, p);
  return h3b_host::check_launch(name);
}

int make_gemm_maps(CUtensorMap* ma, CUtensorMap* mb, const int8_t* qa, int64_t M, int64_t K, const int8_t* qw,
                   int64_t w_rows, int b_box_rows) {
  uint64_t adims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  uint64_t astr[1] = {static_cast<uint64_t>(K)};
  uint32_t abox[2] = {kBK, kBM};
  uint32_t es[2] = {1, 1};
  int rc = h3b_host::encode_tiled(ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qa, adims, astr, abox, es,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t bdims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(w_rows)};
  uint64_t bstr[1] = {static_cast<uint64_t>(K)};
  uint32_t bbox[2] = {kBK, static_cast<uint32_t>(b_box_rows)};
  return h3b_host::encode_tiled(mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw, bdims, bstr, bbox, es,
                                CU_TENSOR_MAP_SWIZZLE_128B);
}

int check_gemm_common(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale, int64_t M,
                      int64_t N, int64_t K, const char* name) {
  if (!qa || !a_scale || !qw || !w_scale) return h3b_host::set_error(H3B_EINVAL, "%s: NULL operand", name);
  if (M <= 0 || N <= 0 || K <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: empty problem M=%lld N=%lld K=%lld", name,
                                                              (long long)M, (long long)N, (long long)K);
  if (K % 16 != 0) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: K=%lld must be a multiple of 16", name, (long long)K);
  if (M > (int64_t(1) << 30) || N > (int64_t(1) << 30) || K > (int64_t(1) << 24))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: problem too large for 32-bit tile indexing", name);
  if (K * 127 * 127 >= (int64_t(1) << 31))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: K=%lld can overflow the int32 accumulator", name, (long long)K);
  return H3B_OK;
}

}  // namespace

extern "C" {

int h3b_conv3d_i8(const int8_t* qx, const int64_t* x_dims, const int8_t* qw, int64_t out_channels, int kd, int kh,
                  int kw, int sd, int sh, int sw, const float* x_scale, const float* w_scale, const void* bias,
                  void* out, const int64_t* out_strides, const void* residual, int32_t* acc_out,
                  int causal_zero_frames, h3b_stream_t stream) {
  const char* name = "h3b_conv3d_i8";
  if (!qx || !x_dims || !qw || !x_scale || !w_scale || !out || !out_strides)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  const int64_t B = x_dims[0], D = x_dims[1], H = x_dims[2], W = x_dims[3], C = x_dims[4];
  const int64_t O = out_channels;
  if (B <= 0 || D <= 0 || H <= 0 || W <= 0 || C <= 0 || O <= 0)
    return h3b_host::set_error(H3B_EINVAL, "%s: empty tensor", name);
  for (int k : {kd, kh, kw})
    if (k != 1 && k != 3) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: kernel dims must be 1 or 3", name);
  for (int s : {sd, sh, sw})
    if (s != 1 && s != 2) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: strides must be 1 or 2", name);
  if (causal_zero_frames != 0 && causal_zero_frames != 2)
    return h3b_host::set_error(H3B_EINVAL, "%s: causal_zero_frames must be 0 or 2", name);
  const int64_t Do = (D - kd) / sd + 1, Ho = (H - kh) / sh + 1, Wo = (W - kw) / sw + 1;
  if (D < kd || H < kh || W < kw) return h3b_host::set_error(H3B_EINVAL, "%s: input too small for valid conv", name);
  const int64_t taps = static_cast<int64_t>(kd) * kh * kw;
  if (taps * C * 127 * 127 >= (int64_t(1) << 31))
    return h3b_host::set_error(H3B_EINVAL, "%s: INT32 accumulator bound exceeds signed INT32 range", name);
  if (B * D * H * W * C >= (int64_t(1) << 40) || B * Do * Ho * Wo * O >= (int64_t(1) << 40))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: tensor too large", name);

  const __half* bias_h = static_cast<const __half*>(bias);
  __half* out_h = static_cast<__half*>(out);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  const bool tma_path = (C % kBK == 0) && sd == 1 && sh == 1 && sw == 1 && B * Do <= (int64_t(1) << 30);
  if (!tma_path) {
    const int64_t total = B * Do * Ho * Wo * O;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    conv3d_i8_simt_kernel<<<static_cast<unsigned>(blocks), threads, 0, st>>>(
        qx, (int)B, (int)D, (int)H, (int)W, (int)C, qw, (int)O, kd, kh, kw, sd, sh, sw, (int)Do, (int)Ho, (int)Wo,
        x_scale, w_scale, bias_h, out_h, out_strides[0], out_strides[1], out_strides[2], out_strides[3], acc_out,
        static_cast<const __half*>(residual));
    return h3b_host::check_launch(name);
  }

  MmaParams p{};
  int bw = 1;
  while (bw < Wo && bw < kBM) bw <<= 1;
  const int bh = kBM / bw;
  p.B = (int)B; p.Do = (int)Do; p.Ho = (int)Ho; p.Wo = (int)Wo;
  p.kd = kd; p.kh = kh; p.kw = kw; p.taps = (int)taps; p.C = (int)C; p.c_chunks = (int)(C / kBK);
  p.bw = bw; p.bh = bh;
  p.w_tiles = (int)((Wo + bw - 1) / bw);
  p.h_tiles = (int)((Ho + bh - 1) / bh);
  p.causal = (causal_zero_frames == 2 && kd == 3) ? 1 : 0;
  p.N = (int)O;
  p.K = (int)(taps * C);
  p.k_blocks = p.taps * p.c_chunks;
  p.m_tiles = (int)(B * Do) * p.h_tiles * p.w_tiles;
  p.a_scale = x_scale; p.w_scale = w_scale; p.bias = bias_h;
  p.out = out_h;
  p.osB = out_strides[0]; p.osD = out_strides[1]; p.osH = out_strides[2]; p.osW = out_strides[3];
  p.acc_out = acc_out;
  p.residual = static_cast<const __half*>(residual);
  if (residual != nullptr && (reinterpret_cast<uintptr_t>(residual) & 15u) != (reinterpret_cast<uintptr_t>(out) & 15u))
    return h3b_host::set_error(H3B_EINVAL, "%s: residual and out must share 16-byte alignment", name);

  CUtensorMap ma, mb;
  uint64_t adims[5] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)D, (uint64_t)B};
  uint64_t astr[4] = {(uint64_t)C, (uint64_t)(C * W), (uint64_t)(C * W * H), (uint64_t)(C * W * H * D)};
  uint32_t abox[5] = {kBK, (uint32_t)bw, (uint32_t)bh, 1, 1};
  uint32_t es[5] = {1, 1, 1, 1, 1};
  int rc = h3b_host::encode_tiled(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, qx, adims, astr, abox, es,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (O <= 128) {
    p.n_tiles = 1;
    uint64_t bdims[2] = {(uint64_t)(taps * C), (uint64_t)O};
    uint64_t bstr[1] = {(uint64_t)(taps * C)};
    uint32_t bbox[2] = {kBK, 128};
    rc = h3b_host::encode_tiled(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw, bdims, bstr, bbox, es, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    return launch_mma<128, 6, AMode::kConv5D, Epi::kConv>(ma, mb, p, st, name);
  }
  p.n_tiles = (int)((O + 255) / 256);
  uint64_t bdims[2] = {(uint64_t)(taps * C), (uint64_t)O};
  uint64_t bstr[1] = {(uint64_t)(taps * C)};
  uint32_t bbox[2] = {kBK, 256};
  rc = h3b_host::encode_tiled(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw, bdims, bstr, bbox, es, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return launch_mma<256, 4, AMode::kConv5D, Epi::kConv>(ma, mb, p, st, name);
}

int h3b_gemm_i8(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale, const void* bias,
                int64_t M, int64_t N, int64_t K, void* out, int64_t ldo, int32_t* acc_out, h3b_stream_t stream) {
  const char* name = "h3b_gemm_i8";
  int rc = check_gemm_common(qa, a_scale, qw, w_scale, M, N, K, name);
  if (rc) return rc;
  if (!out || ldo < N) return h3b_host::set_error(H3B_EINVAL, "%s: bad output", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.k_blocks = (int)((K + kBK - 1) / kBK);
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.a_scale = a_scale; p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(out); p.ldo = ldo; p.acc_out = acc_out;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap ma, mb;
  // Wide N fills the SMs with 128x256 tiles; narrow problems use 128x128.
  const int64_t tiles256 = p.m_tiles * ((N + 255) / 256);
  if (N > 128 && tiles256 >= h3b_host::num_sms()) {
    p.n_tiles = (int)((N + 255) / 256);
    rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, N, 256);
    if (rc) return rc;
    return launch_mma<256, 4, AMode::kGemm2D, Epi::kLinear>(ma, mb, p, st, name);
  }
  p.n_tiles = (int)((N + 127) / 128);
  rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, N, 128);
  if (rc) return rc;
  return launch_mma<128, 6, AMode::kGemm2D, Epi::kLinear>(ma, mb, p, st, name);
}

int h3b_gemm_i8_swiglu(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                       const void* bias, int64_t M, int64_t F, int64_t K, void* act, h3b_stream_t stream) {
  const char* name = "h3b_gemm_i8_swiglu";
  int rc = check_gemm_common(qa, a_scale, qw, w_scale, M, 2 * F, K, name);
  if (rc) return rc;
  if (!act) return h3b_host::set_error(H3B_EINVAL, "%s: NULL output", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)(2 * F); p.K = (int)K; p.F = (int)F;
  p.k_blocks = (int)((K + kBK - 1) / kBK);
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.n_tiles = (int)((F + 127) / 128);
  p.a_scale = a_scale; p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(act);
  CUtensorMap ma, mb;
  rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, 2 * F, 128);
  if (rc) return rc;
  return launch_mma<256, 4, AMode::kGemm2D, Epi::kSwiGLU>(ma, mb, p, reinterpret_cast<cudaStream_t>(stream), name);
}

int h3b_gemm_i8_qkv_rope(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                         const void* bias, int64_t batch, int64_t tokens, int64_t heads, int64_t K, const void* cos_t,
                         const void* sin_t, int64_t rot_dims, float eps, void* q_out, void* k_out, void* v_out,
                         h3b_stream_t stream) {
  const char* name = "h3b_gemm_i8_qkv_rope";
  const int64_t M = batch * tokens, N = heads * 192;
  int rc = check_gemm_common(qa, a_scale, qw, w_scale, M, N, K, name);
  if (rc) return rc;
  if (!q_out || !k_out || !v_out || (rot_dims > 0 && (!cos_t || !sin_t)))
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (rot_dims != 0 && rot_dims != 16 && rot_dims != 32 && rot_dims != 48 && rot_dims != 64)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: rotary dims must be one of 0, 16, 32, 48, 64", name);
  if (rot_dims > 0 && ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t)) & 15u))
    return h3b_host::set_error(H3B_EINVAL, "%s: cos/sin tables must be 16-byte aligned", name);
  for (const void* ptr : std::initializer_list<const void*>{q_out, k_out, v_out})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return h3b_host::set_error(H3B_EINVAL, "%s: q/k/v must be 16-byte aligned", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.k_blocks = (int)((K + kBK - 1) / kBK);
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.n_tiles = (int)heads;
  p.heads = (int)heads; p.tokens = (int)tokens; p.R = (int)rot_dims; p.eps = eps;
  p.cos_t = static_cast<const __half*>(cos_t); p.sin_t = static_cast<const __half*>(sin_t);
  p.q_out = static_cast<__half*>(q_out); p.k_out = static_cast<__half*>(k_out); p.v_out = static_cast<__half*>(v_out);
  p.a_scale = a_scale; p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  CUtensorMap ma, mb;
  rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, N, 192);
  if (rc) return rc;
  return launch_mma<192, 5, AMode::kGemm2D, Epi::kQkvRope>(ma, mb, p, reinterpret_cast<cudaStream_t>(stream), name);
}

}  // extern "C"
