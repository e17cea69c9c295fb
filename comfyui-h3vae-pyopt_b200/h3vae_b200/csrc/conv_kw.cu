// Implicit-GEMM causal conv3d (INT8, or fp16 operands with fp32 accumulation)
// with the three kw taps read from one input strip (stride 1, kernel width 3,
// 128 output columns per M tile; C_out <= 128 with two M tiles per CTA, or
// C_out <= 256 with one).
//
// In the mma_tc conv mainloop every k-block (tap, channel chunk) loads its own
// 128-row A box, so each input row is fetched from L2 once per kw tap.  Here
// one k-group is (kd, kh, channel chunk): the producer loads, per M tile, a
// strip of 136 consecutive input columns (128 outputs + the 2 columns the
// last ones reach, rounded up to a multiple of 8 rows) and the three B tiles
// of taps kw = 0, 1, 2; the MMA warp reads the A operand of tap kw as the
// strip's rows kw .. kw+127 by starting the shared-memory descriptor kw
// 128-byte rows into it (the 128-byte swizzle phase follows the row address).
// A traffic drops from 3 x 16 KB to 17 KB per M tile and (kd, kh, chunk).
//
// Two rings: strips (AST stages x MT tiles x 17 KB) and B tiles (BST stages
// x BN rows x 128 B), each with full / empty mbarriers.  Epilogue as the mma_tc conv
// epilogue (per-tensor scale, column constants in shared memory, fused bias
// and residual).  Taps that only read the two zero causal frames are skipped.
#include "common.cuh"

namespace h3b {

constexpr int kKwStripRows = 136;
constexpr uint32_t kKwStripBytes = kKwStripRows * kBK;   // 17408 = 17 x 1024

template <int BN, int MT, int AST, int BST>
struct KwCfg {
  static constexpr uint32_t a_stage = MT * kKwStripBytes;
  static constexpr uint32_t b_stage = BN * kBK;
  static constexpr size_t smem = AST * a_stage + BST * b_stage + 1024 + 256 + 2 * BN * sizeof(float) +
                                 kEpiWarps * 2048;   // + one 2 KB load/store staging buffer per epilogue warp
};

template <int kKwBN, int kKwMT, int kKwAStages, int kKwBStages, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    conv_kw_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                      const MmaParams p) {
  constexpr uint32_t kKwAStageBytes = KwCfg<kKwBN, kKwMT, kKwAStages, kKwBStages>::a_stage;
  constexpr uint32_t kKwBStageBytes = KwCfg<kKwBN, kKwMT, kKwAStages, kKwBStages>::b_stage;
  constexpr uint32_t kTmemCols = TmemLayout<kKwMT * kKwBN>::cols;
  constexpr uint32_t kAccStride = TmemLayout<kKwMT * kKwBN>::acc_stride;
  constexpr uint32_t kIdesc = F16 ? make_idesc_f16(kBM, kKwBN) : make_idesc_i8(kBM, kKwBN);
  constexpr int kKE = F16 ? 64 : 128;   // K elements per 128-byte chunk

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kKwAStages * kKwAStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_b + kKwBStages * kKwBStageBytes);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + kKwAStages;
  uint64_t* b_full = a_empty + kKwAStages;
  uint64_t* b_empty = b_full + kKwBStages;
  uint64_t* tfull_bar = b_empty + kKwBStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* cst = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_groups;                 // n_tiles == 1
  const int groups_per_kd = 3 * p.c_chunks;         // (kh, chunk) per kd

  auto conv_tile = [&](int m_tile, int& b, int& od, int& oh0, int& ow0) {
    int t = m_tile;
    const int tw = t % p.w_tiles; t /= p.w_tiles;
    const int th = t % p.h_tiles; t /= p.h_tiles;
    od = t % p.Do;
    b = t / p.Do;
    oh0 = th * p.bh;
    ow0 = tw * p.bw;
  };
  // first (kd, kh, chunk) group that does not only read the two zero causal frames
  auto first_group = [&](int m_group) {
    if (!p.causal) return 0;
    int kd0 = 3;
#pragma unroll
    for (int i = 0; i < kKwMT; ++i) {
      const int mt = m_group * kKwMT + i;
      if (mt >= p.m_tiles) break;
      const int od = (mt / (p.w_tiles * p.h_tiles)) % p.Do;
      kd0 = min(kd0, max(0, 2 - od));
    }
    return kd0 * groups_per_kd;
  };
  const int n_groups = 3 * groups_per_kd;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKwAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kKwBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
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
      uint32_t ia = 0, ib = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int cb[kKwMT], cd[kKwMT], chh[kKwMT], cw[kKwMT];
#pragma unroll
        for (int i = 0; i < kKwMT; ++i) conv_tile(tile * kKwMT + i, cb[i], cd[i], chh[i], cw[i]);
        for (int g = first_group(tile); g < n_groups && ok; ++g, ++ia) {
          const int kd = g / groups_per_kd;
          const int kh = (g / p.c_chunks) % 3;
          const int cc = g % p.c_chunks;
          const uint32_t sa = ia % kKwAStages;
          if (!mbar_wait(&a_empty[sa], ((ia / kKwAStages) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&a_full[sa], kKwAStageBytes);
#pragma unroll
          for (int i = 0; i < kKwMT; ++i)
            // An M tile past the last one decodes to b >= B: the box is out of range and loads zeros.
            tma_load_5d(smem_a + sa * kKwAStageBytes + i * kKwStripBytes, &map_a, &a_full[sa], cc * kKE, cw[i],
                        chh[i] + kh, cd[i] + kd, cb[i]);
          for (int kw = 0; kw < 3; ++kw, ++ib) {
            const uint32_t sb = ib % kKwBStages;
            if (!mbar_wait(&b_empty[sb], ((ib / kKwBStages) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&b_full[sb], kKwBStageBytes);
            tma_load_2d(smem_b + sb * kKwBStageBytes, &map_b, &b_full[sb], ((kd * 3 + kh) * 3 + kw) * p.C + cc * kKE,
                        0);
          }
        }
      }
      // Drain: no TMA write into this CTA's shared memory may be in flight at exit (bounded).
      for (uint32_t s = 0; s < kKwAStages && s < ia; ++s) {
        const uint32_t last = ia - 1 - ((ia - 1 - s) % kKwAStages);
        mbar_wait(&a_full[s], (last / kKwAStages) & 1u, nullptr);
      }
      for (uint32_t s = 0; s < kKwBStages && s < ib; ++s) {
        const uint32_t last = ib - 1 - ((ib - 1 - s) % kKwBStages);
        mbar_wait(&b_full[s], (last / kKwBStages) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      uint32_t ia = 0, ib = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int g0 = first_group(tile);
        const uint32_t acc = local & 1u;
        if (!mbar_wait(&tempty_bar[acc], (((local >> 1) & 1u) ^ 1u), abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccStride;
        for (int g = g0; g < n_groups && ok; ++g, ++ia) {
          const uint32_t sa = ia % kKwAStages;
          if (!mbar_wait(&a_full[sa], (ia / kKwAStages) & 1u, abort_flag)) { ok = false; break; }
          const uint32_t a_base = smem_u32(smem_a + sa * kKwAStageBytes);
          for (int kw = 0; kw < 3; ++kw, ++ib) {
            const uint32_t sb = ib % kKwBStages;
            if (!mbar_wait(&b_full[sb], (ib / kKwBStages) & 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint64_t bdesc = make_sw128_desc(smem_u32(smem_b + sb * kKwBStageBytes));
#pragma unroll
            for (int i = 0; i < kKwMT; ++i) {
              // Tap kw reads strip rows kw .. kw+127: the descriptor starts kw
              // 128-byte rows in, with base offset 0 -- the MMA derives the
              // 128-byte swizzle phase of each row from its shared-memory
              // address, as the TMA did when it wrote the strip (verified
              // bit-exactly against an exact conv).
              const uint64_t adesc = make_sw128_desc(a_base + i * kKwStripBytes + kw * kBK);
#pragma unroll
              for (int k = 0; k < kBK / 32; ++k) {   // 32 bytes of K per MMA
                const uint32_t accumulate = (g > g0 || kw > 0 || k > 0) ? 1u : 0u;
                if constexpr (F16)
                  mma_f16(d_tmem + i * kKwBN, adesc + 2 * k, bdesc + 2 * k, kIdesc, accumulate);
                else
                  mma_i8(d_tmem + i * kKwBN, adesc + 2 * k, bdesc + 2 * k, kIdesc, accumulate);
              }
            }
            tc_commit(&b_empty[sb]);
          }
          if (!ok) break;
          tc_commit(&a_empty[sa]);
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int half = (warp - 2) >> 2;
    const int etid = threadIdx.x - 64;
    const uint32_t stage = smem_u32(cst + 2 * kKwBN) + (warp - 2) * 2048;
    // column constants (weight scale, bias) of the single N tile, staged once
    if (etid < kKwBN) {
      const bool in = etid < p.N;
      cst[etid] = (in && !F16) ? __ldg(p.w_scale + etid) : 1.0f;
      cst[kKwBN + etid] = (in && p.bias != nullptr) ? __half2float(p.bias[etid]) : 0.0f;
    }
    const float* cw = cst;
    const float* cb = cst + kKwBN;
    const float sx = F16 ? 0.0f : *p.a_scale;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.out) & 15u) == 0) && (p.osW % 8 == 0) &&
                        (p.osH % 8 == 0) && (p.osD % 8 == 0) && (p.osB % 8 == 0);
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const uint32_t acc = local & 1u;
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&tfull_bar[acc], (local >> 1) & 1u, abort_flag));
      if (!epi_barrier_and(ready, 32 * kEpiWarps)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + acc * kAccStride + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
      for (int i = 0; i < kKwMT; ++i) {
        const uint32_t t_row = t_acc + i * kKwBN;
        const int mt = tile * kKwMT + i;
        int b, od, oh0, ow0;
        conv_tile(mt, b, od, oh0, ow0);
        const int oh = oh0 + row / p.bw;
        const int ow = ow0 + row % p.bw;
        const bool valid = (mt < p.m_tiles) && (oh < p.Ho) && (ow < p.Wo);
        const int64_t obase =
            b * p.osB + od * p.osD + static_cast<int64_t>(oh) * p.osH + static_cast<int64_t>(ow) * p.osW;
        const int64_t pos = ((static_cast<int64_t>(b) * p.Do + od) * p.Ho + oh) * p.Wo + ow;
        // a warp's 32 rows are consecutive positions of one output row (the
        // valid ones a prefix): staged residual loads and output stores
        const int valid_rows = __popc(__ballot_sync(0xffffffffu, valid));
        const int64_t obase0 = __shfl_sync(0xffffffffu, obase, 0);
#pragma unroll 1
        for (int c = half; c < kKwBN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait();
          const int n0 = c * 32;
          const int valid_cols = p.N - n0;
          if (vec_ok && valid_cols >= 32 && valid_rows > 0) {
            float v[32];
            dequant_chunk<F16>(r, sx, cw + n0, cb + n0, v);
            if (p.residual != nullptr) {
              uint4 res[4];
              load_chunk32_staged(stage, p.residual + obase0 + n0, p.osW, valid_rows, res);
              add_residual_row(v, res);
            }
            uint4 row[4];
            pack_row32(v, row);
            store_chunk32_staged(stage, row, p.out + obase0 + n0, p.osW, valid_rows);
            if (!F16 && valid && p.acc_out != nullptr) store_acc_chunk(p.acc_out + pos * p.N + n0, r, valid_cols);
          } else if (valid && valid_cols > 0) {
            float v[32];
            dequant_chunk<F16>(r, sx, cw + n0, cb + n0, v);
            if (p.residual != nullptr) add_residual_chunk(v, p.residual + obase + n0, valid_cols, vec_ok);
            store_row_chunk(p.out + obase + n0, v, valid_cols, vec_ok);
            if (!F16 && p.acc_out != nullptr) store_acc_chunk(p.acc_out + pos * p.N + n0, r, valid_cols);
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

}  // namespace h3b

namespace {

// Launch of the kw-strip conv for an INT8 conv whose geometry conv3d_tc has
// already validated and described in p (C % 128 == 0, 3x3x3 kernel, stride 1,
// bw = 128 so one M tile is 128 columns of one output row, C_out <= BN).
template <int BN, int MT, int AST, int BST, bool F16>
int launch_conv_kw(const void* x, const int64_t* x_dims, const void* w, int64_t O, int taps, h3b::MmaParams p,
                   cudaStream_t stream, const char* name) {
  using namespace h3b;
  using Cfg = KwCfg<BN, MT, AST, BST>;
  const int64_t B = x_dims[0], D = x_dims[1], H = x_dims[2], W = x_dims[3], C = x_dims[4];
  CUtensorMap ma, mb;
  uint64_t adims[5] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)D, (uint64_t)B};
  uint64_t astr[4] = {(uint64_t)C, (uint64_t)(C * W), (uint64_t)(C * W * H), (uint64_t)(C * W * H * D)};
  constexpr int kElt = F16 ? 2 : 1;
  constexpr int kKE = kBK / kElt;
  const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  for (auto& v : astr) v *= kElt;
  uint32_t abox[5] = {(uint32_t)kKE, (uint32_t)kKwStripRows, 1, 1, 1};
  uint32_t aes[5] = {1, 1, 1, 1, 1};
  int rc = h3b_host::encode_tiled(&ma, dt, 5, x, adims, astr, abox, aes, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t bdims[2] = {(uint64_t)(taps * C), (uint64_t)O};
  uint64_t bstr[1] = {(uint64_t)(taps * C * kElt)};
  uint32_t bbox[2] = {(uint32_t)kKE, (uint32_t)BN};
  uint32_t es[2] = {1, 1};
  rc = h3b_host::encode_tiled(&mb, dt, 2, w, bdims, bstr, bbox, es, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  p.n_tiles = 1;
  p.m_groups = (p.m_tiles + MT - 1) / MT;
  static_assert(Cfg::smem <= 232448, "shared memory budget");
  auto kern = conv_kw_kernel<BN, MT, AST, BST, F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Cfg::smem));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  const int grid = p.m_groups < h3b_host::num_sms() ? p.m_groups : h3b_host::num_sms();
  kern<<<grid, kThreads, Cfg::smem, stream>>>(ma, mb, p);
  return h3b_host::check_launch(name);
}

}  // namespace
