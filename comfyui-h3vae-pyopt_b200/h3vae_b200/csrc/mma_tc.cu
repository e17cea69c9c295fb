// tcgen05 mainloop shared by the implicit-GEMM causal conv3d (INT8 and fp16
// operands) and the decoder linears (INT8; fp16 for the fp16 decoder profile).
//
// Structure (one persistent CTA per SM, 10 warps):
//   warp 0      TMA producer: MT A tiles (128 rows x 128 bytes of K each) and
//               one B tile (BN rows x 128 bytes of K) per k-block into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory buffers.
//   warp 1      TMEM owner + MMA issuer: 4 x tcgen05.mma per k-block and A
//               tile (kind::i8 K=32 or kind::f16 K=16: 32 bytes of K each)
//               into one of two TMEM accumulators (MT x BN 32-bit columns).
//               MT = 2 lets two 128-row M tiles share each B tile, which
//               halves the B traffic per MMA for narrow (BN = 128) outputs.
//   warps 2..9  epilogue: tcgen05.ld of the finished accumulator (one TMEM
//               lane = one output row per thread; the two warps of a lane
//               quadrant take alternate 32-column chunks), dequantize with
//               the tile's column constants staged in shared memory, fused
//               op, store -- through a per-warp shared staging buffer when
//               the warp's 32 rows are evenly strided, so each global store
//               instruction writes 8 rows x 64 contiguous bytes.
// The double-buffered accumulator lets the epilogue of tile i overlap the
// mainloop of tile i+1.
//
// Conv mode: the A operand of output tile (b, od, rows oh0.., cols ow0..) for
// tap (kd, kh, kw) and channel chunk c0 is one 5-D TMA box
// {128 bytes of channels, bw*sw, bh*sh, 1, 1} at
// (c0, ow0*sw+kw, oh0*sh+kh, od*sd+kd, b) of the padded NDHWC input, with TMA
// element strides {1, sw, sh, 1, 1} so a stride-2 conv reads every other
// pixel -- the im2col tile is never materialized.  Taps that only read the
// two zero causal frames (od*sd + kd < 2) are skipped when the producer
// guarantees those frames (zero products, the sum is unchanged).
#include "common.cuh"

namespace h3b {

enum class AMode : int { kGemm2D = 0, kConv5D = 1 };
enum class Epi : int { kLinear = 0, kConv = 1, kSwiGLU = 2, kQkvRope = 3, kResidual = 4 };

// fp32 column constants staged per tile: weight scale and bias, plus the
// residual gate for the residual epilogue.
__host__ __device__ constexpr int cst_arrays(Epi ep) { return ep == Epi::kResidual ? 3 : 2; }

struct MmaParams {
  int M, N, K;          // GEMM view (conv: N = out channels)
  int m_tiles, n_tiles;
  int k_blocks;         // GEMM: ceil(K / 128); conv: taps * c_chunks
  int m_groups;         // ceil(m_tiles / MT): CTA tiles along M
  // conv geometry
  int B, Do, Ho, Wo;
  int kd, kh, kw, taps, c_chunks, C;
  int sd, sh, sw;
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
  const __half* residual;  // conv: optional fp16 tensor added after the fp16 rounding (same strides as out);
                           // residual GEMM: the block input x [M, ldo]
  // residual GEMM (attention-out + residual + RMS statistics)
  const __half* gate;      // per-column residual gate g [N]
  float* row_sumsq;        // [M, 2 * n_tiles] per-row partial sums of raw^2 (or h^2 with round_stats)
  int round_stats;
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
// the power-of-two allocation that holds both; W = MT * BN columns each.
template <int W>
struct TmemLayout {
  static_assert(W <= 256, "two accumulators must fit the 512 TMEM columns");
  static constexpr uint32_t acc_stride = (W <= 32) ? 32 : (W <= 64) ? 64 : (W <= 128) ? 128 : 256;
  static constexpr uint32_t cols = 2 * acc_stride;
};

// ---------------------------------------------------------------------------
// Epilogue helpers
// ---------------------------------------------------------------------------
// Column constants of the tile being finished: the epilogue warps stage the
// per-column weight scale and bias (as fp32) of the current N tile in shared
// memory, so the per-element dequantization reads them with broadcast 16-byte
// shared loads instead of one global load per element and column.
//
// 32 output columns of one row: INT8 dequantization fp32(acc) * sx * ws + b
// (the CK contract's fma(acc * sx, ws, b); b = 0 without a bias), or the fp32
// accumulator of an fp16 conv plus its bias.
template <bool F16>
__device__ __forceinline__ void dequant_chunk(const uint32_t (&r)[32], float sx, const float* ws, const float* bs,
                                              float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 b4 = reinterpret_cast<const float4*>(bs)[q];
    const float b[4] = {b4.x, b4.y, b4.z, b4.w};
    if constexpr (F16) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * q + j] = __fadd_rn(__uint_as_float(r[4 * q + j]), b[j]);
    } else {
      // packed fp32 pairs: the same two roundings per element
      const float4 w4 = reinterpret_cast<const float4*>(ws)[q];
      const float2 s2 = make_float2(sx, sx);
      const float2 lo = f2x_fma(f2x_mul(make_float2(static_cast<float>(static_cast<int32_t>(r[4 * q])),
                                                    static_cast<float>(static_cast<int32_t>(r[4 * q + 1]))), s2),
                                make_float2(w4.x, w4.y), make_float2(b4.x, b4.y));
      const float2 hi = f2x_fma(f2x_mul(make_float2(static_cast<float>(static_cast<int32_t>(r[4 * q + 2])),
                                                    static_cast<float>(static_cast<int32_t>(r[4 * q + 3]))), s2),
                                make_float2(w4.z, w4.w), make_float2(b4.z, b4.w));
      v[4 * q] = lo.x;
      v[4 * q + 1] = lo.y;
      v[4 * q + 2] = hi.x;
      v[4 * q + 3] = hi.y;
    }
  }
}

// Barrier over the epilogue warps (named barrier 1) that also ANDs a predicate
// across them: every epilogue warp leaves the tile loop at the same tile when
// any of their bounded waits gave up, and the shared-memory column constants
// written before it are visible after it.
__device__ __forceinline__ bool epi_barrier_and(bool pred, int threads) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(threads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float ex2_approx_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// 32 fp32 values as fp16 in four 16-byte vectors.
__device__ __forceinline__ void pack_row32(const float (&v)[32], uint4 (&o)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __align__(16) __half2 h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[k * 8 + 2 * j], v[k * 8 + 2 * j + 1]);
    o[k] = *reinterpret_cast<const uint4*>(h);
  }
}

// Stores a 32-row x 32-column fp16 chunk (row r = lane r's four vectors) to
// dst0 + r * row_stride through this warp's 2 KB shared staging buffer: the
// lanes write their rows (16-byte chunks XOR-swizzled by row, so both the
// shared stores and loads are bank-conflict free), then each global store
// instruction writes 8 rows x 64 contiguous bytes instead of 32 rows x 16 B.
// Warp-collective; rows >= valid_rows are not written.  dst0 and row_stride
// must keep every row 16-byte aligned.
__device__ __forceinline__ void store_chunk32_staged(uint32_t stage, const uint4 (&row)[4], __half* dst0,
                                                     int64_t row_stride, int valid_rows) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k) st_shared_v4(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4), row[k]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (lane >> 2) + 8 * i;
    const int k = lane & 3;
    const uint4 val = ld_shared_v4(stage + r * 64 + ((k ^ ((r >> 1) & 3)) << 4));
    if (r < valid_rows) *reinterpret_cast<uint4*>(dst0 + r * row_stride + k * 8) = val;
  }
  __syncwarp();
}

// The counterpart of store_chunk32_staged for loads: rows src0 + r * row_stride
// (r < valid_rows) are read 8 rows x 64 B per instruction into the warp's
// staging buffer, then each lane takes its own row's four 16-byte vectors
// (rows >= valid_rows read as zeros).  Warp-collective.
__device__ __forceinline__ void load_chunk32_staged(uint32_t stage, const __half* src0, int64_t row_stride,
                                                    int valid_rows, uint4 (&row)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (lane >> 2) + 8 * i;
    const int k = lane & 3;
    const uint4 val = r < valid_rows ? __ldg(reinterpret_cast<const uint4*>(src0 + r * row_stride + k * 8))
                                     : make_uint4(0, 0, 0, 0);
    st_shared_v4(stage + r * 64 + ((k ^ ((r >> 1) & 3)) << 4), val);
  }
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k) row[k] = ld_shared_v4(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4));
  __syncwarp();
}

// v = fp16(fp16(v) + residual) for 32 values with the residual row in registers.
__device__ __forceinline__ void add_residual_row(float (&v)[32], const uint4 (&res)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half2* h = reinterpret_cast<const __half2*>(&res[k]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      v[k * 8 + 2 * j] = __fadd_rn(round_fp16(v[k * 8 + 2 * j]), f.x);
      v[k * 8 + 2 * j + 1] = __fadd_rn(round_fp16(v[k * 8 + 2 * j + 1]), f.y);
    }
  }
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
template <int BN, int STAGES, AMode AM, Epi EP, int MT, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    mma_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const MmaParams p) {
  static_assert(MT == 1 || MT == 2, "one or two M tiles per CTA tile");
  static_assert(MT == 1 || EP == Epi::kConv || EP == Epi::kLinear, "paired M tiles: conv / linear epilogues only");
  static_assert(!F16 || (EP != Epi::kQkvRope && EP != Epi::kResidual), "fp16 operands: conv, linear and SwiGLU epilogues");
  static_assert(EP != Epi::kResidual || (MT == 1 && AM == AMode::kGemm2D), "residual epilogue: GEMM, one M tile");
  constexpr int kCstArrays = cst_arrays(EP);
  constexpr int kKE = F16 ? 64 : 128;   // K elements per 128-byte k-block
  constexpr uint32_t kBTileBytes = BN * kBK;
  constexpr uint32_t kAStageBytes = MT * kATileBytes;
  constexpr uint32_t kStageBytes = kAStageBytes + kBTileBytes;
  constexpr uint32_t kTmemCols = TmemLayout<MT * BN>::cols;
  constexpr uint32_t kAccStride = TmemLayout<MT * BN>::acc_stride;
  constexpr uint32_t kIdesc = F16 ? make_idesc_f16(kBM, BN) : make_idesc_i8(kBM, BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * kAStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [2 buffers][scale | bias (| gate)][BN] fp32 column constants of the
  // epilogue, then one 2 KB load/store staging buffer per epilogue warp
  float* cst = reinterpret_cast<float*>(smem + STAGES * kStageBytes + 256);
  const uint32_t stage_base = smem_u32(cst + 2 * kCstArrays * BN);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_groups * p.n_tiles;

  // Conv: output tile m_tile -> (b, od, oh0, ow0); first k-block that does not
  // only read the two zero causal frames.
  auto conv_tile = [&](int m_tile, int& b, int& od, int& oh0, int& ow0) {
    int t = m_tile;
    const int tw = t % p.w_tiles; t /= p.w_tiles;
    const int th = t % p.h_tiles; t /= p.h_tiles;
    od = t % p.Do;
    b = t / p.Do;
    oh0 = th * p.bh;
    ow0 = tw * p.bw;
  };
  auto first_kblock = [&](int m_group) {
    int kb = 0;
    if constexpr (AM == AMode::kConv5D) {
      if (p.causal) {
        kb = p.k_blocks;
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const int mt = m_group * MT + i;
          if (mt >= p.m_tiles) break;
          const int od = (mt / (p.w_tiles * p.h_tiles)) % p.Do;
          const int kd0 = max(0, 2 - od * p.sd);
          kb = min(kb, kd0 * p.kh * p.kw * p.c_chunks);
        }
      }
    }
    return kb;
  };

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
        const int m_group = tile / p.n_tiles;
        const int n_tile = tile - m_group * p.n_tiles;
        const int kb_begin = first_kblock(m_group);
        int cb[MT], cd[MT], chh[MT], cw[MT];
        if constexpr (AM == AMode::kConv5D) {
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            // A tile past the last M tile decodes to b >= B: the TMA box is
            // entirely out of range and loads zeros.
            conv_tile(m_group * MT + i, cb[i], cd[i], chh[i], cw[i]);
            cd[i] *= p.sd;
            chh[i] *= p.sh;
            cw[i] *= p.sw;
          }
        }
        for (int kb = kb_begin; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
          uint8_t* sa = smem_a + s * kAStageBytes;
          uint8_t* sb = smem_b + s * kBTileBytes;
          if constexpr (AM == AMode::kConv5D) {
            const int tap = kb / p.c_chunks;
            const int cc = kb - tap * p.c_chunks;
            const int tkw = tap % p.kw;
            const int tkh = (tap / p.kw) % p.kh;
            const int tkd = tap / (p.kw * p.kh);
#pragma unroll
            for (int i = 0; i < MT; ++i)
              tma_load_5d(sa + i * kATileBytes, &map_a, &full_bar[s], cc * kKE, cw[i] + tkw, chh[i] + tkh,
                          cd[i] + tkd, cb[i]);
            tma_load_2d(sb, &map_b, &full_bar[s], kb * kKE, n_tile * BN);
          } else {
#pragma unroll
            for (int i = 0; i < MT; ++i)
              tma_load_2d(sa + i * kATileBytes, &map_a, &full_bar[s], kb * kKE, (m_group * MT + i) * kBM);
            if constexpr (EP == Epi::kSwiGLU) {
              const int j0 = n_tile * (BN / 2);
              tma_load_2d(sb, &map_b, &full_bar[s], kb * kKE, j0);
              tma_load_2d(sb + (BN / 2) * kBK, &map_b, &full_bar[s], kb * kKE, p.F + j0);
            } else {
              tma_load_2d(sb, &map_b, &full_bar[s], kb * kKE, n_tile * BN);
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
        const int kb_begin = first_kblock(tile / p.n_tiles);
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
          const uint64_t bdesc = make_sw128_desc(smem_u32(smem_b + s * kBTileBytes));
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            const uint64_t adesc = make_sw128_desc(smem_u32(smem_a + s * kAStageBytes + i * kATileBytes));
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k) {
              // Advance the start address by 32 bytes (2 x 16 B) per MMA K step.
              const uint32_t accumulate = (kb > kb_begin || k > 0) ? 1u : 0u;
              if constexpr (F16)
                mma_f16(d_tmem + i * BN, adesc + 2 * k, bdesc + 2 * k, kIdesc, accumulate);
              else
                mma_i8(d_tmem + i * BN, adesc + 2 * k, bdesc + 2 * k, kIdesc, accumulate);
            }
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
    const int etid = threadIdx.x - 64;  // 0 .. 255 over the epilogue warps
    const uint32_t stage = stage_base + (warp - 2) * 2048;
    // Column constants of a tile, one column per epilogue thread (BN <= 256):
    // weight scale and bias of column etid of the tile's N range (SwiGLU: gate
    // columns in [0, BN/2), the matching up columns in [BN/2, BN)).  They are
    // loaded one tile ahead so the global-load latency hides behind a tile.
    auto load_column = [&](int tile, float& w, float& bv, float& gv) {
      w = 1.0f;
      bv = 0.0f;
      gv = 0.0f;
      if (tile >= num_tiles || etid >= BN) return;
      const int n_tile = tile % p.n_tiles;
      int col;
      bool in;
      if constexpr (EP == Epi::kSwiGLU) {
        const int j = n_tile * (BN / 2) + (etid < BN / 2 ? etid : etid - BN / 2);
        in = j < p.F;
        col = etid < BN / 2 ? j : p.F + j;
      } else {
        col = n_tile * BN + etid;
        in = col < p.N;
      }
      if (!in) return;
      if constexpr (!F16) w = __ldg(p.w_scale + col);
      if (p.bias != nullptr) bv = __half2float(p.bias[col]);
      if constexpr (EP == Epi::kResidual) gv = __half2float(p.gate[col]);
    };
    float next_w, next_b, next_g;
    load_column(blockIdx.x, next_w, next_b, next_g);
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int m_group = tile / p.n_tiles;
      const int n_tile = tile - m_group * p.n_tiles;
      const uint32_t acc = local & 1u;
      const uint32_t aph = (local >> 1) & 1u;
      // Double-buffered constants: every epilogue warp has passed the barrier
      // of tile local-1, hence finished tile local-2, before buffer local&1 is
      // rewritten here.
      float* cw = cst + (local & 1u) * (kCstArrays * BN);
      float* cb = cw + BN;
      float* cg = cb + BN;   // residual gate (residual epilogue only)
      if (etid < BN) {
        cw[etid] = next_w;
        cb[etid] = next_b;
        if constexpr (EP == Epi::kResidual) cg[etid] = next_g;
      }
      load_column(tile + gridDim.x, next_w, next_b, next_g);
      // Row data that does not come from the MMA is fetched before the wait.
      float sx_pre = 0.0f;
      int64_t m_pre = 0;
      if constexpr (EP == Epi::kLinear || EP == Epi::kSwiGLU || EP == Epi::kQkvRope || EP == Epi::kResidual) {
        m_pre = static_cast<int64_t>(m_group * MT) * kBM + row;
        if (!F16 && MT == 1 && m_pre < p.M) sx_pre = __ldg(p.a_scale + m_pre);
      }
      // tcgen05.ld is warp-collective and the barrier spans all epilogue warps:
      // they leave together if any thread's bounded wait gave up.
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&tfull_bar[acc], aph, abort_flag));
      if (!epi_barrier_and(ready, 32 * kEpiWarps)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + acc * kAccStride + (static_cast<uint32_t>(quad * 32) << 16);

      if constexpr (EP == Epi::kLinear) {
#pragma unroll 1
        for (int i = 0; i < MT; ++i) {
          const uint32_t t_row = t_acc + i * BN;
          const int64_t m = static_cast<int64_t>(m_group * MT + i) * kBM + row;
          const bool valid = m < p.M;
          const float sx = (F16 || MT == 1) ? sx_pre : (valid ? p.a_scale[m] : 0.0f);
          const bool vec_ok = (p.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0;
          const int64_t m_warp = m - lane;
          const int valid_rows = static_cast<int>(p.M - m_warp < 32 ? p.M - m_warp : 32);
#pragma unroll 1
          for (int c = half; c < BN / 32; c += 2) {
            uint32_t r[32];
            tmem_ld32(t_row + c * 32, r);
            tmem_ld_wait();
            const int n0 = n_tile * BN + c * 32;
            const int valid_cols = p.N - n0;
            if (valid_cols >= 32 && vec_ok && valid_rows > 0) {
              float v[32];
              dequant_chunk<F16>(r, sx, cw + c * 32, cb + c * 32, v);
              uint4 row[4];
              pack_row32(v, row);
              store_chunk32_staged(stage, row, p.out + m_warp * p.ldo + n0, p.ldo, valid_rows);
              if (!F16 && valid && p.acc_out != nullptr) store_acc_chunk(p.acc_out + m * p.N + n0, r, valid_cols);
            } else if (valid && valid_cols > 0) {
              float v[32];
              dequant_chunk<F16>(r, sx, cw + c * 32, cb + c * 32, v);
              store_row_chunk(p.out + m * p.ldo + n0, v, valid_cols, vec_ok);
              if (!F16 && p.acc_out != nullptr) store_acc_chunk(p.acc_out + m * p.N + n0, r, valid_cols);
            }
          }
        }
      } else if constexpr (EP == Epi::kConv) {
        const float sx = F16 ? 0.0f : *p.a_scale;
        const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && (p.osW % 8 == 0) &&
                            (p.osH % 8 == 0) && (p.osD % 8 == 0) && (p.osB % 8 == 0);
#pragma unroll 1
        for (int i = 0; i < MT; ++i) {
          const uint32_t t_row = t_acc + i * BN;
          const int mt = m_group * MT + i;
          int b, od, oh0, ow0;
          conv_tile(mt, b, od, oh0, ow0);
          const int oh = oh0 + row / p.bw;
          const int ow = ow0 + row % p.bw;
          const bool valid = (mt < p.m_tiles) && (oh < p.Ho) && (ow < p.Wo);
          const int64_t obase =
              b * p.osB + od * p.osD + static_cast<int64_t>(oh) * p.osH + static_cast<int64_t>(ow) * p.osW;
          const int64_t pos = ((static_cast<int64_t>(b) * p.Do + od) * p.Ho + oh) * p.Wo + ow;
          // With output tiles at least 32 columns wide a warp's 32 rows are
          // consecutive positions of one output row (the valid ones a prefix):
          // residual loads and output stores then go through the staging buffer.
          const int valid_rows = __popc(__ballot_sync(0xffffffffu, valid));
          const int64_t obase0 = __shfl_sync(0xffffffffu, obase, 0);
#pragma unroll 1
          for (int c = half; c < BN / 32; c += 2) {
            uint32_t r[32];
            tmem_ld32(t_row + c * 32, r);
            tmem_ld_wait();
            const int n0 = n_tile * BN + c * 32;
            const int valid_cols = p.N - n0;
            if (p.bw >= 32 && vec_ok && valid_cols >= 32 && valid_rows > 0) {
              float v[32];
              dequant_chunk<F16>(r, sx, cw + c * 32, cb + c * 32, v);
              if (p.residual != nullptr) {
                uint4 res[4];
                load_chunk32_staged(stage, p.residual + obase0 + n0, p.osW, valid_rows, res);
                add_residual_row(v, res);
              }
              uint4 row[4];
              pack_row32(v, row);
              store_chunk32_staged(stage, row, p.out + obase0 + n0, p.osW, valid_rows);
              if (valid && !F16 && p.acc_out != nullptr) store_acc_chunk(p.acc_out + pos * p.N + n0, r, valid_cols);
            } else if (valid && valid_cols > 0) {
              float v[32];
              dequant_chunk<F16>(r, sx, cw + c * 32, cb + c * 32, v);
              if (p.residual != nullptr) add_residual_chunk(v, p.residual + obase + n0, valid_cols, vec_ok);
              store_row_chunk(p.out + obase + n0, v, valid_cols, vec_ok);
              if (!F16 && p.acc_out != nullptr) store_acc_chunk(p.acc_out + pos * p.N + n0, r, valid_cols);
            }
          }
        }
      } else if constexpr (EP == Epi::kResidual) {
        // Attention-out + residual: a = fp16(fma(acc * sx, ws, b)) (the linear's
        // fp16 output), raw = fma(a, g, x), h = fp16(raw) is written in place of
        // a, and the row's sum of raw^2 over the columns this warp handles goes
        // to row_sumsq[m, 2 * n_tile + half]; the RMSNorm + row quantization
        // kernel adds the row's partials in a fixed order.
        const uint32_t t_row = t_acc;
        const int64_t m = m_pre;
        const bool valid = m < p.M;
        const float sx = sx_pre;
        const bool vec_ok = (p.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0 &&
                            (reinterpret_cast<uintptr_t>(p.residual) & 15u) == 0;
        const int64_t m_warp = m - lane;
        const int valid_rows = static_cast<int>(p.M - m_warp < 32 ? p.M - m_warp : 32);
        float ss = 0.0f;
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait();
          const int n0 = n_tile * BN + c * 32;
          const int valid_cols = p.N - n0;
          if (valid_cols >= 32 && vec_ok && valid_rows > 0) {
            float v[32];
            dequant_chunk<false>(r, sx, cw + c * 32, cb + c * 32, v);
            uint4 xr[4];
            load_chunk32_staged(stage, p.residual + m_warp * p.ldo + n0, p.ldo, valid_rows, xr);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const __half2* xh = reinterpret_cast<const __half2*>(&xr[k]);
              const float4 g0 = *reinterpret_cast<const float4*>(cg + c * 32 + k * 8);
              const float4 g1 = *reinterpret_cast<const float4*>(cg + c * 32 + k * 8 + 4);
              const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 xf = __half22float2(xh[j]);
                const float2 raw = f2x_fma(make_float2(round_fp16(v[k * 8 + 2 * j]), round_fp16(v[k * 8 + 2 * j + 1])),
                                           make_float2(gg[2 * j], gg[2 * j + 1]), xf);
                const float2 hf = __half22float2(__floats2half2_rn(raw.x, raw.y));
                const float2 st = p.round_stats ? hf : raw;
                ss = __fmaf_rn(st.x, st.x, ss);
                ss = __fmaf_rn(st.y, st.y, ss);
                v[k * 8 + 2 * j] = hf.x;
                v[k * 8 + 2 * j + 1] = hf.y;
              }
            }
            uint4 row[4];
            pack_row32(v, row);
            store_chunk32_staged(stage, row, p.out + m_warp * p.ldo + n0, p.ldo, valid_rows);
          } else if (valid && valid_cols > 0) {
            float v[32];
            dequant_chunk<false>(r, sx, cw + c * 32, cb + c * 32, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < valid_cols) {
                const float raw = __fmaf_rn(round_fp16(v[j]), cg[c * 32 + j], __half2float(p.residual[m * p.ldo + n0 + j]));
                const float hf = round_fp16(raw);
                const float st = p.round_stats ? hf : raw;
                ss = __fmaf_rn(st, st, ss);
                p.out[m * p.ldo + n0 + j] = __float2half_rn(hf);
              }
            }
          }
        }
        if (valid) p.row_sumsq[m * (2 * p.n_tiles) + 2 * n_tile + half] = ss;
      } else if constexpr (EP == Epi::kSwiGLU) {
        const uint32_t t_row = t_acc;
        const int64_t m = m_pre;
        const bool valid = m < p.M;
        const float sx = sx_pre;
        const bool vec_ok = (p.F % 8) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0;
        const int64_t m_warp = m - lane;
        const int valid_rows = static_cast<int>(p.M - m_warp < 32 ? p.M - m_warp : 32);
        constexpr float kNegLog2e = -1.4426950408889634f;
#pragma unroll 1
        for (int c = half; c < BN / 64; c += 2) {
          uint32_t rg[32], ru[32];
          tmem_ld32(t_row + c * 32, rg);
          tmem_ld32(t_row + BN / 2 + c * 32, ru);
          tmem_ld_wait();
          const int j0 = n_tile * (BN / 2) + c * 32;
          const int valid_cols = p.F - j0;
          const bool staged = valid_cols >= 32 && vec_ok && valid_rows > 0;
          if (staged || (valid && valid_cols > 0)) {
            float g[32], u[32];
            dequant_chunk<F16>(rg, sx, cw + c * 32, cb + c * 32, g);
            dequant_chunk<F16>(ru, sx, cw + BN / 2 + c * 32, cb + BN / 2 + c * 32, u);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              // gate and up rounded to fp16 (the linear's fp16 output), then
              // silu(g) * u = g / (1 + 2^(-g log2 e)) * u in fp32
              const float2 gg = __half22float2(__floats2half2_rn(g[j], g[j + 1]));
              const float2 uu = __half22float2(__floats2half2_rn(u[j], u[j + 1]));
              const float e0 = ex2_approx_ftz(__fmul_rn(gg.x, kNegLog2e));
              const float e1 = ex2_approx_ftz(__fmul_rn(gg.y, kNegLog2e));
              g[j] = __fmul_rn(__fmul_rn(gg.x, rcp_approx_ftz(__fadd_rn(1.0f, e0))), uu.x);
              g[j + 1] = __fmul_rn(__fmul_rn(gg.y, rcp_approx_ftz(__fadd_rn(1.0f, e1))), uu.y);
            }
            if (staged) {
              uint4 row[4];
              pack_row32(g, row);
              store_chunk32_staged(stage, row, p.out + m_warp * p.F + j0, p.F, valid_rows);
            } else {
              store_row_chunk(p.out + m * p.F + j0, g, valid_cols, vec_ok);
            }
          }
        }
      } else if constexpr (EP == Epi::kQkvRope) {
        // BN == 192: this tile is one head's [q | k | v] for 128 tokens.  Half
        // 0 finishes q and v columns 0..31, half 1 k and v columns 32..63.
        const uint32_t t_row = t_acc;
        const int64_t m = m_pre;
        const bool valid = m < p.M;
        const float sx = sx_pre;
        const int h = n_tile;
        const int64_t bb = valid ? m / p.tokens : 0;
        const int64_t tt = valid ? m - bb * p.tokens : 0;
        const int64_t dst_off = ((bb * p.heads + h) * p.tokens + tt) * 64;
        // The warp's 32 rows are consecutive tokens of one batch entry (the
        // common case): then their q / k / v rows are consecutive 128-byte rows
        // of [B, H, n, 64] and the stores go through the staging buffer.
        const int64_t dst_off0 = __shfl_sync(0xffffffffu, dst_off, 0);
        const int64_t bb0 = __shfl_sync(0xffffffffu, bb, 0);
        const bool staged = __all_sync(0xffffffffu, !valid || (bb == bb0 && dst_off == dst_off0 + lane * 64));
        const int valid_rows = static_cast<int>(p.M - (m - lane) < 32 ? p.M - (m - lane) : 32);
        uint4 rc[8], rs[8];
        {
          uint32_t r[32];
          tmem_ld32(t_row + 128 + half * 32, r);
          tmem_ld_wait();
          float v[32];
          dequant_chunk<false>(r, sx, cw + 128 + half * 32, cb + 128 + half * 32, v);
          if (staged) {
            uint4 row[4];
            pack_row32(v, row);
            store_chunk32_staged(stage, row, p.v_out + dst_off0 + half * 32, 64, valid_rows);
          } else if (valid) {
            store_row_chunk(p.v_out + dst_off + half * 32, v, 32, true);
          }
        }
        // the token's rope tables, in flight while q (or k) is dequantized
        if (valid) {
          load_rope_row(p.cos_t + m * p.R, p.sin_t + m * p.R, p.R, rc, rs);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) rc[q] = rs[q] = make_uint4(0, 0, 0, 0);
        }
        __half2 x[32];   // the 64 fp16-rounded q (or k) outputs of this row
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(t_row + half * 64 + c * 32, r);
          tmem_ld_wait();
          const float* ws = cw + half * 64 + c * 32;
          const float* bs = cb + half * 64 + c * 32;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 w4 = reinterpret_cast<const float4*>(ws)[q];
            const float4 b4 = reinterpret_cast<const float4*>(bs)[q];
            const float2 s2 = make_float2(sx, sx);
            const auto dq = [&](int j, float w0, float w1, float b0, float b1) {
              const float2 a = make_float2(static_cast<float>(static_cast<int32_t>(r[4 * q + j])),
                                           static_cast<float>(static_cast<int32_t>(r[4 * q + j + 1])));
              const float2 v2 = f2x_fma(f2x_mul(a, s2), make_float2(w0, w1), make_float2(b0, b1));
              return __floats2half2_rn(v2.x, v2.y);
            };
            x[c * 16 + 2 * q] = dq(0, w4.x, w4.y, b4.x, b4.y);
            x[c * 16 + 2 * q + 1] = dq(2, w4.z, w4.w, b4.z, b4.w);
          }
        }
        uint4 o[8];
        qk_norm_rope_regs(x, p.eps, p.R, rc, rs, o);
        __half* qk = half == 0 ? p.q_out : p.k_out;
        if (staged) {
          const uint4 lo[4] = {o[0], o[1], o[2], o[3]}, hi[4] = {o[4], o[5], o[6], o[7]};
          store_chunk32_staged(stage, lo, qk + dst_off0, 64, valid_rows);
          store_chunk32_staged(stage, hi, qk + dst_off0 + 32, 64, valid_rows);
        } else if (valid) {
#pragma unroll
          for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(qk + dst_off)[q] = o[q];
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
// INT8 conv with per-token activation scales (one fp32 scale per padded input
// position).  The scale is not constant along a row of the im2col matrix --
// every tap reads a different input position -- so it cannot be applied after
// the int32 reduction.  The MMA warp therefore closes the accumulation after
// every 128-channel k-block (|partial| <= 128*127*127 < 2^22) into one of two
// TMEM buffers, and the epilogue warps fold each partial into fp32 registers
// as acc += float(P) * s_x[input position of that tap] (int32 -> fp32 through
// the 1.5 * 2^23 magic constant, exact below 2^22), then write
// fp16(fma(acc, s_w[n], bias[n])) (+ residual) once per tile.  BN = 128; each
// epilogue thread keeps one row x 64 columns.
// ---------------------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    conv_i8_token_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const MmaParams p, const float* __restrict__ x_scales, int Dp, int Hp, int Wp) {
  constexpr int BN = 128;
  constexpr uint32_t kBTileBytes = BN * kBK;
  constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  constexpr uint32_t kIdesc = make_idesc_i8(kBM, BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * kATileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* pfull_bar = bars + 2 * STAGES;        // [2] partial accumulator ready
  uint64_t* pempty_bar = bars + 2 * STAGES + 2;   // [2] partial consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;

  auto conv_tile = [&](int m_tile, int& b, int& od, int& oh0, int& ow0) {
    int t = m_tile;
    const int tw = t % p.w_tiles; t /= p.w_tiles;
    const int th = t % p.h_tiles; t /= p.h_tiles;
    od = t % p.Do;
    b = t / p.Do;
    oh0 = th * p.bh;
    ow0 = tw * p.bw;
  };
  auto first_kblock = [&](int m_tile) {
    if (!p.causal) return 0;
    const int od = (m_tile / (p.w_tiles * p.h_tiles)) % p.Do;
    return max(0, 2 - od * p.sd) * p.kh * p.kw * p.c_chunks;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&pfull_bar[a], 1);
      mbar_init(&pempty_bar[a], 32 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
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
        int b, od, oh0, ow0;
        conv_tile(m_tile, b, od, oh0, ow0);
        for (int kb = first_kblock(m_tile); kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % STAGES;
          if (!mbar_poll(&empty_bar[s], ((it / STAGES) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
          const int tap = kb / p.c_chunks;
          const int cc = kb - tap * p.c_chunks;
          const int tkw = tap % p.kw, tkh = (tap / p.kw) % p.kh, tkd = tap / (p.kw * p.kh);
          tma_load_5d(smem_a + s * kATileBytes, &map_a, &full_bar[s], cc * kBK, ow0 * p.sw + tkw, oh0 * p.sh + tkh,
                      od * p.sd + tkd, b);
          tma_load_2d(smem_b + s * kBTileBytes, &map_b, &full_bar[s], kb * kBK, n_tile * BN);
        }
      }
      for (uint32_t s = 0; s < STAGES && s < it; ++s) {
        const uint32_t last = it - 1 - ((it - 1 - s) % STAGES);
        mbar_wait(&full_bar[s], (last / STAGES) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      uint32_t it = 0, part = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = first_kblock(tile / p.n_tiles); kb < p.k_blocks && ok; ++kb, ++it, ++part) {
          const uint32_t buf = part & 1u;
          if (!mbar_poll(&pempty_bar[buf], ((part >> 1) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t s = it % STAGES;
          if (!mbar_poll(&full_bar[s], (it / STAGES) & 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_desc(smem_u32(smem_a + s * kATileBytes));
          const uint64_t bdesc = make_sw128_desc(smem_u32(smem_b + s * kBTileBytes));
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_i8(tmem_base + buf * BN, adesc + 2 * k, bdesc + 2 * k, kIdesc, k > 0 ? 1u : 0u);
          tc_commit(&empty_bar[s]);
          tc_commit(&pfull_bar[buf]);
        }
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int half = (warp - 2) >> 2;   // columns half*64 .. +64
    constexpr float kMagic = 12582912.0f;
    uint32_t part = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_tile = tile / p.n_tiles;
      const int n_tile = tile - m_tile * p.n_tiles;
      int b, od, oh0, ow0;
      conv_tile(m_tile, b, od, oh0, ow0);
      const int oh = oh0 + row / p.bw;
      const int ow = ow0 + row % p.bw;
      const bool valid = (oh < p.Ho) && (ow < p.Wo);
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
      bool ok = true;
      for (int kb = first_kblock(m_tile); kb < p.k_blocks; ++kb, ++part) {
        const uint32_t buf = part & 1u;
        ok = __all_sync(0xffffffffu, ok && mbar_wait(&pfull_bar[buf], (part >> 1) & 1u, abort_flag));
        const int tap = kb / p.c_chunks;
        const int tkw = tap % p.kw, tkh = (tap / p.kw) % p.kh, tkd = tap / (p.kw * p.kh);
        float sx = 0.0f;
        if (valid) {
          const int64_t ip = ((static_cast<int64_t>(b) * Dp + od * p.sd + tkd) * Hp + oh * p.sh + tkh) * Wp +
                             ow * p.sw + tkw;
          sx = __ldg(x_scales + ip);
        }
        if (ok) {
          tc_fence_after();
          const uint32_t t_row = tmem_base + buf * BN + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld32(t_row + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              // exact int32 -> fp32 below 2^22: (M + P) - M
              const float2 f = f2x_sub(make_float2(__int_as_float(0x4B400000 + static_cast<int>(r[j])),
                                                   __int_as_float(0x4B400000 + static_cast<int>(r[j + 1]))),
                                       make_float2(kMagic, kMagic));
              const float2 v = f2x_fma(f, make_float2(sx, sx), make_float2(acc[c * 32 + j], acc[c * 32 + j + 1]));
              acc[c * 32 + j] = v.x;
              acc[c * 32 + j + 1] = v.y;
            }
          }
          tc_fence_before();
        }
        mbar_arrive(&pempty_bar[buf]);
      }
      if (!ok || !valid) continue;
      const int64_t obase = b * p.osB + od * p.osD + static_cast<int64_t>(oh) * p.osH + static_cast<int64_t>(ow) * p.osW;
      const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && (p.osW % 8 == 0) &&
                          (p.osH % 8 == 0) && (p.osD % 8 == 0) && (p.osB % 8 == 0);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int n0 = n_tile * BN + half * 64 + c * 32;
        const int valid_cols = p.N - n0;
        if (valid_cols <= 0) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = min(n0 + j, p.N - 1);
          v[j] = p.bias != nullptr ? __fmaf_rn(acc[c * 32 + j], p.w_scale[n], __half2float(p.bias[n]))
                                   : __fmul_rn(acc[c * 32 + j], p.w_scale[n]);
        }
        if (p.residual != nullptr) add_residual_chunk(v, p.residual + obase + n0, valid_cols, vec_ok);
        store_row_chunk(p.out + obase + n0, v, valid_cols, vec_ok);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 256);
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

// The INT8 conv variant that reads the three kw taps from one input strip.
#include "conv_kw.cu"

// ===========================================================================
// Host launchers
// ===========================================================================
namespace {

using namespace h3b;

template <int BN, int STAGES, AMode AM, Epi EP, int MT = 1, bool F16 = false>
int launch_mma(const CUtensorMap& ma, const CUtensorMap& mb, const MmaParams& p, cudaStream_t stream,
               const char* name) {
  constexpr size_t smem = STAGES * (MT * kATileBytes + BN * kBK) + 1024 + 256 +
                         2 * cst_arrays(EP) * BN * sizeof(float) + kEpiWarps * 2048;
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = mma_tc_kernel<BN, STAGES, AM, EP, MT, F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int tiles = p.m_groups * p.n_tiles;
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

// fp16 operands: K elements of 2 bytes, the same 128-byte k-block boxes.
int make_gemm_maps_f16(CUtensorMap* ma, CUtensorMap* mb, const void* a, int64_t M, int64_t K, const void* w,
                       int64_t w_rows, int b_box_rows) {
  uint64_t adims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  uint64_t astr[1] = {static_cast<uint64_t>(K) * 2};
  uint32_t abox[2] = {kBK / 2, kBM};
  uint32_t es[2] = {1, 1};
  int rc = h3b_host::encode_tiled(ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, adims, astr, abox, es,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t bdims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(w_rows)};
  uint64_t bstr[1] = {static_cast<uint64_t>(K) * 2};
  uint32_t bbox[2] = {kBK / 2, static_cast<uint32_t>(b_box_rows)};
  return h3b_host::encode_tiled(mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w, bdims, bstr, bbox, es,
                                CU_TENSOR_MAP_SWIZZLE_128B);
}

int check_gemm_f16(const void* a, const void* w, int64_t M, int64_t N, int64_t K, const char* name) {
  if (!a || !w) return h3b_host::set_error(H3B_EINVAL, "%s: NULL operand", name);
  if (M <= 0 || N <= 0 || K <= 0)
    return h3b_host::set_error(H3B_EINVAL, "%s: empty problem M=%lld N=%lld K=%lld", name, (long long)M,
                               (long long)N, (long long)K);
  if (K % 8 != 0) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: K=%lld must be a multiple of 8", name, (long long)K);
  if ((reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u))
    return h3b_host::set_error(H3B_EINVAL, "%s: operands must be 16-byte aligned", name);
  if (M > (int64_t(1) << 30) || N > (int64_t(1) << 30) || K > (int64_t(1) << 24))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: problem too large for 32-bit tile indexing", name);
  return H3B_OK;
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

// Shared host side of the INT8 and fp16 implicit-GEMM convs: geometry checks,
// tile shape, tensor maps (5-D im2col boxes with element strides for the
// conv stride), kernel choice.  elt = operand bytes (1 or 2).
struct ConvArgs {
  const void* x;
  const int64_t* x_dims;
  const void* w;
  int64_t O;
  int kd, kh, kw, sd, sh, sw;
  const float* x_scale;
  const float* w_scale;
  const void* bias;
  void* out;
  const int64_t* out_strides;
  const void* residual;
  int32_t* acc_out;
  int causal_zero_frames;
  cudaStream_t stream;
};

int check_conv_geometry(const ConvArgs& a, const char* name, int64_t* dims6) {
  if (!a.x || !a.x_dims || !a.w || !a.out || !a.out_strides)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  const int64_t B = a.x_dims[0], D = a.x_dims[1], H = a.x_dims[2], W = a.x_dims[3], C = a.x_dims[4];
  if (B <= 0 || D <= 0 || H <= 0 || W <= 0 || C <= 0 || a.O <= 0)
    return h3b_host::set_error(H3B_EINVAL, "%s: empty tensor", name);
  for (int k : {a.kd, a.kh, a.kw})
    if (k != 1 && k != 3) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: kernel dims must be 1 or 3", name);
  for (int s : {a.sd, a.sh, a.sw})
    if (s != 1 && s != 2) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: strides must be 1 or 2", name);
  if (a.causal_zero_frames != 0 && a.causal_zero_frames != 2)
    return h3b_host::set_error(H3B_EINVAL, "%s: causal_zero_frames must be 0 or 2", name);
  if (D < a.kd || H < a.kh || W < a.kw) return h3b_host::set_error(H3B_EINVAL, "%s: input too small for valid conv", name);
  const int64_t Do = (D - a.kd) / a.sd + 1, Ho = (H - a.kh) / a.sh + 1, Wo = (W - a.kw) / a.sw + 1;
  if (B * D * H * W * C >= (int64_t(1) << 40) || B * Do * Ho * Wo * a.O >= (int64_t(1) << 40))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: tensor too large", name);
  if (a.residual != nullptr &&
      (reinterpret_cast<uintptr_t>(a.residual) & 15u) != (reinterpret_cast<uintptr_t>(a.out) & 15u))
    return h3b_host::set_error(H3B_EINVAL, "%s: residual and out must share 16-byte alignment", name);
  dims6[0] = Do; dims6[1] = Ho; dims6[2] = Wo;
  return H3B_OK;
}

template <bool F16>
int conv3d_tc(const ConvArgs& a, int64_t Do, int64_t Ho, int64_t Wo, const char* name) {
  constexpr int kElt = F16 ? 2 : 1;
  constexpr int kKE = kBK / kElt;
  const int64_t B = a.x_dims[0], D = a.x_dims[1], H = a.x_dims[2], W = a.x_dims[3], C = a.x_dims[4];
  const int64_t taps = static_cast<int64_t>(a.kd) * a.kh * a.kw;
  MmaParams p{};
  int bw = 1;
  while (bw < Wo && bw < kBM) bw <<= 1;
  const int bh = kBM / bw;
  p.B = (int)B; p.Do = (int)Do; p.Ho = (int)Ho; p.Wo = (int)Wo;
  p.kd = a.kd; p.kh = a.kh; p.kw = a.kw; p.sd = a.sd; p.sh = a.sh; p.sw = a.sw;
  p.taps = (int)taps; p.C = (int)C; p.c_chunks = (int)(C / kKE);
  p.bw = bw; p.bh = bh;
  p.w_tiles = (int)((Wo + bw - 1) / bw);
  p.h_tiles = (int)((Ho + bh - 1) / bh);
  p.causal = (a.causal_zero_frames == 2 && a.kd == 3) ? 1 : 0;
  p.N = (int)a.O;
  p.K = (int)(taps * C);
  p.k_blocks = p.taps * p.c_chunks;
  p.m_tiles = (int)(B * Do) * p.h_tiles * p.w_tiles;
  p.a_scale = a.x_scale; p.w_scale = a.w_scale; p.bias = static_cast<const __half*>(a.bias);
  p.out = static_cast<__half*>(a.out);
  p.osB = a.out_strides[0]; p.osD = a.out_strides[1]; p.osH = a.out_strides[2]; p.osW = a.out_strides[3];
  p.acc_out = a.acc_out;
  p.residual = static_cast<const __half*>(a.residual);

  const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap ma, mb;
  uint64_t adims[5] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)D, (uint64_t)B};
  uint64_t astr[4] = {(uint64_t)(C * kElt), (uint64_t)(C * W * kElt), (uint64_t)(C * W * H * kElt),
                      (uint64_t)(C * W * H * D * kElt)};
  // With element strides {1, sw, sh} the box spans bw*sw x bh*sh pixels and
  // loads every sw-th / sh-th one: bw x bh rows of 128 bytes.
  uint32_t abox[5] = {(uint32_t)kKE, (uint32_t)(bw * a.sw), (uint32_t)(bh * a.sh), 1, 1};
  uint32_t aes[5] = {1, (uint32_t)a.sw, (uint32_t)a.sh, 1, 1};
  int rc = h3b_host::encode_tiled(&ma, dt, 5, a.x, adims, astr, abox, aes, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint32_t es[2] = {1, 1};
  uint64_t bdims[2] = {(uint64_t)(taps * C), (uint64_t)a.O};
  uint64_t bstr[1] = {(uint64_t)(taps * C * kElt)};
  auto b_map = [&](uint32_t rows) {
    uint32_t bbox[2] = {(uint32_t)kKE, rows};
    return h3b_host::encode_tiled(&mb, dt, 2, a.w, bdims, bstr, bbox, es, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  const int sms = h3b_host::num_sms();
  // 3x3x3 stride-1 convs over rows of >= 128 output columns: the kw-strip mainloop
  if (a.kd == 3 && a.kh == 3 && a.kw == 3 && a.sd == 1 && a.sh == 1 && a.sw == 1 && bw == kBM && C % kKE == 0) {
    if (a.O <= 128 && (p.m_tiles + 1) / 2 >= sms)
      return launch_conv_kw<128, 2, 3, 6, F16>(a.x, a.x_dims, a.w, a.O, (int)taps, p, a.stream, name);
    if (a.O > 128 && a.O <= 256 && p.m_tiles >= sms)
      return launch_conv_kw<256, 1, 2, 5, F16>(a.x, a.x_dims, a.w, a.O, (int)taps, p, a.stream, name);
  }
  if (a.O <= 64) {
    p.n_tiles = 1;
    p.m_groups = (p.m_tiles + 1) / 2;
    if ((rc = b_map(64))) return rc;
    return launch_mma<64, 5, AMode::kConv5D, Epi::kConv, 2, F16>(ma, mb, p, a.stream, name);
  }
  if (a.O <= 128) {
    p.n_tiles = 1;
    if ((rc = b_map(128))) return rc;
    // Two M tiles per CTA share the B tile when there is enough work to fill the SMs.
    if ((p.m_tiles + 1) / 2 >= sms) {
      p.m_groups = (p.m_tiles + 1) / 2;
      return launch_mma<128, 4, AMode::kConv5D, Epi::kConv, 2, F16>(ma, mb, p, a.stream, name);
    }
    p.m_groups = p.m_tiles;
    return launch_mma<128, 6, AMode::kConv5D, Epi::kConv, 1, F16>(ma, mb, p, a.stream, name);
  }
  p.n_tiles = (int)((a.O + 255) / 256);
  p.m_groups = p.m_tiles;
  if ((rc = b_map(256))) return rc;
  return launch_mma<256, 4, AMode::kConv5D, Epi::kConv, 1, F16>(ma, mb, p, a.stream, name);
}

}  // namespace

extern "C" {

int h3b_conv3d_i8(const int8_t* qx, const int64_t* x_dims, const int8_t* qw, int64_t out_channels, int kd, int kh,
                  int kw, int sd, int sh, int sw, const float* x_scale, const float* w_scale, const void* bias,
                  void* out, const int64_t* out_strides, const void* residual, int32_t* acc_out,
                  int causal_zero_frames, h3b_stream_t stream) {
  const char* name = "h3b_conv3d_i8";
  ConvArgs a{qx, x_dims, qw, out_channels, kd, kh, kw, sd, sh, sw, x_scale, w_scale, bias, out, out_strides,
             residual, acc_out, causal_zero_frames, reinterpret_cast<cudaStream_t>(stream)};
  if (!x_scale || !w_scale) return h3b_host::set_error(H3B_EINVAL, "%s: NULL scale", name);
  int64_t o3[3];
  int rc = check_conv_geometry(a, name, o3);
  if (rc) return rc;
  const int64_t B = x_dims[0], D = x_dims[1], H = x_dims[2], W = x_dims[3], C = x_dims[4];
  const int64_t Do = o3[0], Ho = o3[1], Wo = o3[2], O = out_channels;
  const int64_t taps = static_cast<int64_t>(kd) * kh * kw;
  if (taps * C * 127 * 127 >= (int64_t(1) << 31))
    return h3b_host::set_error(H3B_EINVAL, "%s: INT32 accumulator bound exceeds signed INT32 range", name);
  const bool tma_path = (C % kBK == 0) && B * Do <= (int64_t(1) << 30);
  if (!tma_path) {
    const int64_t total = B * Do * Ho * Wo * O;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    conv3d_i8_simt_kernel<<<static_cast<unsigned>(blocks), threads, 0, a.stream>>>(
        qx, (int)B, (int)D, (int)H, (int)W, (int)C, qw, (int)O, kd, kh, kw, sd, sh, sw, (int)Do, (int)Ho, (int)Wo,
        x_scale, w_scale, static_cast<const __half*>(bias), static_cast<__half*>(out), out_strides[0],
        out_strides[1], out_strides[2], out_strides[3], acc_out, static_cast<const __half*>(residual));
    return h3b_host::check_launch(name);
  }
  return conv3d_tc<false>(a, Do, Ho, Wo, name);
}

int h3b_conv3d_i8_token(const int8_t* qx, const int64_t* x_dims, const int8_t* qw, int64_t out_channels, int kd,
                        int kh, int kw, int sd, int sh, int sw, const float* x_scales, const float* w_scale,
                        const void* bias, void* out, const int64_t* out_strides, const void* residual,
                        int causal_zero_frames, h3b_stream_t stream) {
  const char* name = "h3b_conv3d_i8_token";
  ConvArgs a{qx, x_dims, qw, out_channels, kd, kh, kw, sd, sh, sw, x_scales, w_scale, bias, out, out_strides,
             residual, nullptr, causal_zero_frames, reinterpret_cast<cudaStream_t>(stream)};
  if (!x_scales || !w_scale) return h3b_host::set_error(H3B_EINVAL, "%s: NULL scale", name);
  int64_t o3[3];
  int rc = check_conv_geometry(a, name, o3);
  if (rc) return rc;
  const int64_t B = x_dims[0], D = x_dims[1], H = x_dims[2], W = x_dims[3], C = x_dims[4];
  if (C % kBK != 0) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: C=%lld must be a multiple of 128", name, (long long)C);
  if (B * o3[0] > (int64_t(1) << 30)) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: too many frames", name);
  const int64_t Do = o3[0], Ho = o3[1], Wo = o3[2];
  const int64_t taps = static_cast<int64_t>(kd) * kh * kw;
  MmaParams p{};
  int bw = 1;
  while (bw < Wo && bw < kBM) bw <<= 1;
  const int bh = kBM / bw;
  p.B = (int)B; p.Do = (int)Do; p.Ho = (int)Ho; p.Wo = (int)Wo;
  p.kd = kd; p.kh = kh; p.kw = kw; p.sd = sd; p.sh = sh; p.sw = sw;
  p.taps = (int)taps; p.C = (int)C; p.c_chunks = (int)(C / kBK);
  p.bw = bw; p.bh = bh;
  p.w_tiles = (int)((Wo + bw - 1) / bw);
  p.h_tiles = (int)((Ho + bh - 1) / bh);
  p.causal = (causal_zero_frames == 2 && kd == 3) ? 1 : 0;
  p.N = (int)out_channels;
  p.K = (int)(taps * C);
  p.k_blocks = p.taps * p.c_chunks;
  p.m_tiles = (int)(B * Do) * p.h_tiles * p.w_tiles;
  p.m_groups = p.m_tiles;
  p.n_tiles = (int)((out_channels + 127) / 128);
  p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(out);
  p.osB = out_strides[0]; p.osD = out_strides[1]; p.osH = out_strides[2]; p.osW = out_strides[3];
  p.residual = static_cast<const __half*>(residual);
  CUtensorMap ma, mb;
  uint64_t adims[5] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)D, (uint64_t)B};
  uint64_t astr[4] = {(uint64_t)C, (uint64_t)(C * W), (uint64_t)(C * W * H), (uint64_t)(C * W * H * D)};
  uint32_t abox[5] = {kBK, (uint32_t)(bw * sw), (uint32_t)(bh * sh), 1, 1};
  uint32_t aes[5] = {1, (uint32_t)sw, (uint32_t)sh, 1, 1};
  rc = h3b_host::encode_tiled(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, qx, adims, astr, abox, aes, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t bdims[2] = {(uint64_t)(taps * C), (uint64_t)out_channels};
  uint64_t bstr[1] = {(uint64_t)(taps * C)};
  uint32_t bbox[2] = {kBK, 128};
  uint32_t es[2] = {1, 1};
  rc = h3b_host::encode_tiled(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, qw, bdims, bstr, bbox, es, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  constexpr int kStages = 6;
  constexpr size_t smem = kStages * (kATileBytes + 128 * kBK) + 1024 + 256;
  auto kern = conv_i8_token_kernel<kStages>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < h3b_host::num_sms() ? tiles : h3b_host::num_sms();
  kern<<<grid, kThreads, smem, a.stream>>>(ma, mb, p, x_scales, (int)D, (int)H, (int)W);
  return h3b_host::check_launch(name);
}

int h3b_conv3d_f16(const void* x, const int64_t* x_dims, const void* w, int64_t out_channels, int kd, int kh, int kw,
                   int sd, int sh, int sw, const void* bias, void* out, const int64_t* out_strides,
                   const void* residual, int causal_zero_frames, h3b_stream_t stream) {
  const char* name = "h3b_conv3d_f16";
  ConvArgs a{x, x_dims, w, out_channels, kd, kh, kw, sd, sh, sw, nullptr, nullptr, bias, out, out_strides,
             residual, nullptr, causal_zero_frames, reinterpret_cast<cudaStream_t>(stream)};
  int64_t o3[3];
  int rc = check_conv_geometry(a, name, o3);
  if (rc) return rc;
  const int64_t C = x_dims[4];
  if (C % 64 != 0)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: C=%lld must be a multiple of 64", name, (long long)C);
  if (x_dims[0] * o3[0] > (int64_t(1) << 30)) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: too many frames", name);
  return conv3d_tc<true>(a, o3[0], o3[1], o3[2], name);
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
  p.m_groups = p.m_tiles;
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

int64_t h3b_gemm_i8_residual_parts(int64_t N) { return N > 0 ? 2 * ((N + 127) / 128) : 0; }

int h3b_gemm_i8_residual(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                         const void* bias, int64_t M, int64_t N, int64_t K, const void* x, const void* gate,
                         int round_stats, void* h, int64_t ldh, float* row_sumsq, h3b_stream_t stream) {
  const char* name = "h3b_gemm_i8_residual";
  int rc = check_gemm_common(qa, a_scale, qw, w_scale, M, N, K, name);
  if (rc) return rc;
  if (!x || !gate || !h || !row_sumsq || ldh < N) return h3b_host::set_error(H3B_EINVAL, "%s: bad x / gate / h", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.k_blocks = (int)((K + kBK - 1) / kBK);
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.m_groups = p.m_tiles;
  p.n_tiles = (int)((N + 127) / 128);
  p.a_scale = a_scale; p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(h); p.ldo = ldh;
  p.residual = static_cast<const __half*>(x);
  p.gate = static_cast<const __half*>(gate);
  p.row_sumsq = row_sumsq;
  p.round_stats = round_stats ? 1 : 0;
  CUtensorMap ma, mb;
  rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, N, 128);
  if (rc) return rc;
  return launch_mma<128, 6, AMode::kGemm2D, Epi::kResidual>(ma, mb, p, reinterpret_cast<cudaStream_t>(stream), name);
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
  p.m_groups = p.m_tiles;
  p.n_tiles = (int)((F + 127) / 128);
  p.a_scale = a_scale; p.w_scale = w_scale; p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(act);
  CUtensorMap ma, mb;
  rc = make_gemm_maps(&ma, &mb, qa, M, K, qw, 2 * F, 128);
  if (rc) return rc;
  return launch_mma<256, 4, AMode::kGemm2D, Epi::kSwiGLU>(ma, mb, p, reinterpret_cast<cudaStream_t>(stream), name);
}

int h3b_gemm_f16(const void* a, const void* w, const void* bias, int64_t M, int64_t N, int64_t K, void* out,
                 int64_t ldo, h3b_stream_t stream) {
  const char* name = "h3b_gemm_f16";
  int rc = check_gemm_f16(a, w, M, N, K, name);
  if (rc) return rc;
  if (!out || ldo < N) return h3b_host::set_error(H3B_EINVAL, "%s: bad output", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.k_blocks = (int)((K + kBK / 2 - 1) / (kBK / 2));
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.m_groups = p.m_tiles;
  p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(out); p.ldo = ldo;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap ma, mb;
  const int64_t tiles256 = p.m_tiles * ((N + 255) / 256);
  if (N > 128 && tiles256 >= h3b_host::num_sms()) {
    p.n_tiles = (int)((N + 255) / 256);
    rc = make_gemm_maps_f16(&ma, &mb, a, M, K, w, N, 256);
    if (rc) return rc;
    return launch_mma<256, 4, AMode::kGemm2D, Epi::kLinear, 1, true>(ma, mb, p, st, name);
  }
  p.n_tiles = (int)((N + 127) / 128);
  rc = make_gemm_maps_f16(&ma, &mb, a, M, K, w, N, 128);
  if (rc) return rc;
  return launch_mma<128, 6, AMode::kGemm2D, Epi::kLinear, 1, true>(ma, mb, p, st, name);
}

int h3b_gemm_f16_swiglu(const void* a, const void* w, const void* bias, int64_t M, int64_t F, int64_t K, void* act,
                        h3b_stream_t stream) {
  const char* name = "h3b_gemm_f16_swiglu";
  int rc = check_gemm_f16(a, w, M, 2 * F, K, name);
  if (rc) return rc;
  if (!act) return h3b_host::set_error(H3B_EINVAL, "%s: NULL output", name);
  MmaParams p{};
  p.M = (int)M; p.N = (int)(2 * F); p.K = (int)K; p.F = (int)F;
  p.k_blocks = (int)((K + kBK / 2 - 1) / (kBK / 2));
  p.m_tiles = (int)((M + kBM - 1) / kBM);
  p.m_groups = p.m_tiles;
  p.n_tiles = (int)((F + 127) / 128);
  p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(act);
  CUtensorMap ma, mb;
  rc = make_gemm_maps_f16(&ma, &mb, a, M, K, w, 2 * F, 128);
  if (rc) return rc;
  return launch_mma<256, 4, AMode::kGemm2D, Epi::kSwiGLU, 1, true>(ma, mb, p, reinterpret_cast<cudaStream_t>(stream),
                                                                   name);
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
  p.m_groups = p.m_tiles;
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
