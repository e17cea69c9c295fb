// Non-causal fp16 attention (head dim 64) on the tcgen05 tensor cores.
//
// One CTA = one (batch, head) and two 128-query tiles; 10 warps:
//   warp 0      TMA: both Q tiles once, then K and V tiles of 128 keys through
//               a 3-stage ring
//   warp 1      TMEM owner + MMA issuer.  Per key block j and query tile t:
//               S_j(t) = Q_t K_j^T (M128 N128 K64, fp32 in TMEM), then, once the
//               softmax of tile t has written P_j(t) to shared memory,
//               O(t) += P_j(t) V_j (M128 N64 K128, V as the MN-major B operand
//               straight from its TMA tile).  S_{j+1}(t) is issued as soon as
//               the softmax has copied S_j(t) out of TMEM.
//   warps 2..9  softmax, four warps per query tile, one query row per thread
//               (its TMEM lane).  The row's 128 scores come out of TMEM in one
//               round trip, after which the S columns are released so the MMA
//               warp computes S_{j+1} while this block is exponentiated.
//               P_j = exp2(S_j * scale*log2e - m) (score pairs scaled by
//               one packed f32x2 FMA) is rounded to fp16 into 128-byte-swizzled
//               shared memory.  O accumulates in TMEM across key blocks; V is
//               extended by a shared-memory block of fp16 ones (P V at N = 80),
//               so O's column 64 accumulates the row sum of the rounded P in
//               fp32 and the exponential loop carries no additions.  The
//               reference max m only moves when a block's max exceeds it by
//               more than 8 (log2 units; P stays <= 256, well inside fp16);
//               then the rows' O and row sums in TMEM are rescaled by
//               exp2(m_old - m_new) before the next P V accumulates.  One
//               division by the row sum at the end.
// The base-2 exponentials (16K per tile and key block, one SFU op each) are
// the bound; the two tiles take turns on the SFU (named-barrier ping-pong) so
// one tile's exponentials overlap the other's TMEM reads, maximum and waits.
// Every mbarrier wait is bounded (see common.cuh); its outcome is made
// warp-uniform before any warp-collective TMEM access.
#include "common.cuh"

namespace h3b {

// Packed fp32 pairs (Blackwell f32x2 arithmetic) and the single-instruction
// base-2 exponential of the softmax.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Base-2 exponentials of a pair of scores on the FMA pipe (packed f32x2), for
// the share of the softmax that does not go to the SFU: Cody-Waite reduction
// x = j + f with j = rint(x) (the 1.5 * 2^23 addition), f in [-1/2, 1/2], then
// 2^f by a degree-3 polynomial and 2^j added into the exponent field.  The
// coefficients are a minimax fit (Lawson's iteratively reweighted least
// squares, relative error) of 2^f on [-1/2, 1/2] made for this kernel: max
// relative error 7.5e-5, a sixth of an fp16 half-ulp, so P (rounded to fp16)
// is unaffected in all but rare rounding ties.  x is clamped to >= -125 so
// j + the polynomial's exponent stays a normal float (2^-125 rounds to 0 in
// fp16, like the SFU's flushed result).
__device__ __forceinline__ void ex2_poly_pair(uint64_t x, float& lo, float& hi) {
  constexpr float kMagic = 12582912.0f;
  float x0, x1;
  f2_unpack(x, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = f2_add(xc, f2_pack(kMagic, kMagic));
  const uint64_t fr = f2_sub(xc, f2_sub(t, f2_pack(kMagic, kMagic)));
  uint64_t poly = f2_fma(f2_pack(0.05517132207751274f, 0.05517132207751274f), fr,
                         f2_pack(0.24261054396629333f, 0.24261054396629333f));
  poly = f2_fma(poly, fr, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  poly = f2_fma(poly, fr, f2_pack(0.9999281167984009f, 0.9999281167984009f));
  float p0, p1, t0, t1;
  f2_unpack(poly, p0, p1);
  f2_unpack(t, t0, t1);
  lo = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  hi = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Pairs of scores (out of every 8) whose exponentials run on the FMA pipe; the
// rest use the SFU's ex2.approx.  The SFU issues 16 results per clock per SM,
// the bound of a head-dim-64 softmax; moving a share to the FMA pipe balances
// the two.
#ifndef H3B_FA_EMU
#define H3B_FA_EMU 0
#endif
// 1: the two query tiles' softmax warps take turns on the SFU (named-barrier
// ping-pong); 0: both exponentiate whenever their scores are ready.
#ifndef H3B_FA_PINGPONG
#define H3B_FA_PINGPONG 1
#endif
// 1: the row sums come from the tensor core -- V is extended by a block of
// ones (P V at N = 80), so O's column 64 accumulates sum_k P[r,k] in fp32 and
// the exponential loop loses its additions; 0: the softmax warps add P up.
#ifndef H3B_FA_ONES
#define H3B_FA_ONES 1
#endif
// 1: scale and shift pairs of scores with one packed f32x2 FMA.
#ifndef H3B_FA_FMA2
#define H3B_FA_FMA2 1
#endif

constexpr int kFaM = 128;       // queries per tile
constexpr int kFaTiles = 2;     // query tiles per CTA
constexpr int kFaN = 128;       // keys per block
constexpr int kFaD = 64;        // head dim
constexpr int kFaStages = 3;
constexpr int kFaSoftmaxWarps = 4;   // per query tile: one row per thread
constexpr int kFaThreads = 64 + 32 * kFaSoftmaxWarps * kFaTiles;
constexpr uint32_t kFaQBytes = kFaM * kFaD * 2;   // 16 KB per tile
constexpr uint32_t kFaKVBytes = kFaN * kFaD * 2;  // 16 KB each for K and V
constexpr uint32_t kFaPBytes = kFaM * kFaN * 2;   // 32 KB per tile (two 16 KB swizzle columns of 64 keys)
constexpr uint32_t kFaTmemCols = 512;             // per tile: S (128) | O (64, + 16 row-sum columns), at tile * 256
constexpr int kFaDO = H3B_FA_ONES ? kFaD + 16 : kFaD;   // P V output columns
constexpr uint32_t kFaOnesBytes = H3B_FA_ONES ? kFaN * 128 : 0;   // 128 key rows x 64 fp16 ones
constexpr uint32_t kFaSmemBytes =
    kFaTiles * kFaQBytes + 2 * kFaStages * kFaKVBytes + kFaTiles * kFaPBytes + kFaOnesBytes + 1024 + 256;

struct FaParams {
  int q_len, kv_len;
  float scale_log2;
  __half* out;
  int64_t os[3];   // out element strides {batch, head, token}; dim stride 1
};

__global__ void __launch_bounds__(kFaThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv, const FaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                                  // [tile]
  uint8_t* sk = sq + kFaTiles * kFaQBytes;             // [stage]
  uint8_t* sv = sk + kFaStages * kFaKVBytes;           // [stage]
  uint8_t* sp = sv + kFaStages * kFaKVBytes;           // [tile]
  uint8_t* sones = sp + kFaTiles * kFaPBytes;          // fp16 ones, the row-sum columns of V
  uint64_t* bars = reinterpret_cast<uint64_t*>(sones + kFaOnesBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kFaStages;
  uint64_t* s_full = kv_empty + kFaStages;    // [tile]
  uint64_t* s_empty = s_full + kFaTiles;      // [tile]
  uint64_t* p_full = s_empty + kFaTiles;      // [tile]
  uint64_t* o_full = p_full + kFaTiles;       // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + kFaTiles);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt0 = blockIdx.x * kFaTiles, h = blockIdx.y, b = blockIdx.z;
  const int n_blocks = (p.kv_len + kFaN - 1) / kFaN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kFaStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < kFaTiles; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_empty[t], 32 * kFaSoftmaxWarps);
      mbar_init(&p_full[t], 32 * kFaSoftmaxWarps);
      mbar_init(&o_full[t], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mq);
    tma_prefetch_desc(&mk);
    tma_prefetch_desc(&mv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kFaTmemCols);
    tmem_relinquish();
  }
  if (H3B_FA_ONES) {
    for (uint32_t i = threadIdx.x; i < kFaOnesBytes / 16; i += kFaThreads)
      st_shared_v4(smem_u32(sones) + 16 * i, make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u));
    fence_proxy_async_smem();   // the tensor core reads them through the async proxy
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------- TMA ----------------------------------
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(q_full, kFaTiles * kFaQBytes);
      for (int t = 0; t < kFaTiles; ++t) tma_load_4d(sq + t * kFaQBytes, &mq, q_full, 0, (qt0 + t) * kFaM, h, b);
      uint32_t issued = 0;
      for (int j = 0; j < n_blocks; ++j, ++issued) {
        const int s = j % kFaStages;
        if (!mbar_poll(&kv_empty[s], ((j / kFaStages) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kFaKVBytes);
        tma_load_4d(sk + s * kFaKVBytes, &mk, &kv_full[s], 0, j * kFaN, h, b);
        tma_load_4d(sv + s * kFaKVBytes, &mv, &kv_full[s], 0, j * kFaN, h, b);
      }
      // drain: no TMA write may still target this CTA's shared memory at exit
      mbar_wait(q_full, 0, nullptr);
      for (uint32_t s = 0; s < kFaStages && s < issued; ++s) {
        const uint32_t last = issued - 1 - ((issued - 1 - s) % kFaStages);
        mbar_wait(&kv_full[s], (last / kFaStages) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (elect_one_sync()) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kFaM, kFaN);
      constexpr uint32_t idesc_pv = make_idesc_f16(kFaM, kFaDO) | (1u << 16);  // B (V) is MN-major
      bool ok = mbar_poll(q_full, 0, abort_flag);
      // S_j(t) into tile t's S columns; requires K_j resident and S_{j-1}(t) read out.
      auto issue_s = [&](int j, int t) -> bool {
        const int s = j % kFaStages;
        if (!mbar_poll(&kv_full[s], (j / kFaStages) & 1, abort_flag)) return false;
        if (!mbar_poll(&s_empty[t], (j & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t qdesc = make_sw128_desc(smem_u32(sq + t * kFaQBytes));
        const uint64_t kdesc = make_sw128_desc(smem_u32(sk + s * kFaKVBytes));
#pragma unroll
        for (int k = 0; k < kFaD / 16; ++k)  // 16 fp16 = 32 bytes per MMA step
          mma_f16(tmem + t * 256, qdesc + 2 * k, kdesc + 2 * k, idesc_qk, k > 0 ? 1u : 0u);
        tc_commit(&s_full[t]);
        return true;
      };
      for (int t = 0; t < kFaTiles && ok; ++t) ok = issue_s(0, t);
      for (int j = 0; j < n_blocks && ok; ++j) {
        const int s = j % kFaStages;
        // S_{j+1}(t) as soon as the softmax of tile t has copied S_j(t) into its
        // registers, so it overlaps that softmax's exponentials.
        for (int t = 0; t < kFaTiles && ok && j + 1 < n_blocks; ++t) ok = issue_s(j + 1, t);
        for (int t = 0; t < kFaTiles && ok; ++t) {
          // P_j(t) written; O(t) holds the sum over the blocks before j,
          // already rescaled if the reference max moved.
          if (!mbar_poll(&p_full[t], j & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t pbase = smem_u32(sp + t * kFaPBytes);
          const uint32_t vbase = smem_u32(sv + s * kFaKVBytes);
          // V is MN-major with 64 dims = one 128-byte swizzle atom per key row;
          // at N = 80 the second atom column (the ones) sits at the leading
          // byte offset, the same distance from every 16-key step.
          const uint64_t lbo = H3B_FA_ONES ? static_cast<uint64_t>(((smem_u32(sones) - vbase) >> 4) & 0x3FFFu) << 16 : 0;
#pragma unroll
          for (int k = 0; k < kFaN / 16; ++k) {
            const uint64_t pdesc = make_sw128_desc(pbase + (k >> 2) * (kFaPBytes / 2)) + 2 * (k & 3);
            uint64_t vdesc = make_sw128_desc(vbase + k * 16 * 128);
            if (H3B_FA_ONES) vdesc = (vdesc & ~(uint64_t(0x3FFFu) << 16)) | lbo;
            mma_f16(tmem + t * 256 + kFaN, pdesc, vdesc, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&o_full[t]);
        }
        tc_commit(&kv_empty[s]);
      }
    }
  } else {
    // ------------------------------ softmax warps ------------------------------
    const int sw = warp - 2;
    const int tile = sw / kFaSoftmaxWarps;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t t_lane = tmem + tile * 256 + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_s = t_lane;
    const uint32_t t_o = t_lane + kFaN;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    const uint32_t prow = smem_u32(sp + tile * kFaPBytes + row * 128);
    const uint32_t bar_s_full = smem_u32(&s_full[tile]), bar_s_empty = smem_u32(&s_empty[tile]);
    const uint32_t bar_p_full = smem_u32(&p_full[tile]), bar_o_full = smem_u32(&o_full[tile]);
    // Named barriers 1 and 2 (both tiles' 256 softmax threads) pass the SFU turn:
    // tile 0 syncs on 1 and arrives on 2, tile 1 the reverse.  Tile 1 hands
    // tile 0 the first turn and skips its hand-back after the last block, so
    // every barrier completes as often as it is waited on.
    constexpr int kSoftmaxThreads = 32 * kFaSoftmaxWarps * kFaTiles;
    auto exp_turn_begin = [&]() {
      if (H3B_FA_PINGPONG)
        asm volatile("bar.sync %0, %1;" ::"r"(tile == 0 ? 1 : 2), "r"(kSoftmaxThreads) : "memory");
    };
    auto exp_turn_end = [&](int jj) {
      if (H3B_FA_PINGPONG && (tile == 0 || jj + 1 < n_blocks))
        asm volatile("bar.arrive %0, %1;" ::"r"(tile == 0 ? 2 : 1), "r"(kSoftmaxThreads) : "memory");
    };
    if (H3B_FA_PINGPONG && tile == 1) asm volatile("bar.arrive 1, %0;" ::"r"(kSoftmaxThreads) : "memory");
    for (int j = 0; j < n_blocks; ++j) {
      ok = __all_sync(0xffffffffu, ok && mbar_wait_u32(bar_s_full, j & 1, abort_flag));
      const int valid = p.kv_len - j * kFaN;
      // All 128 scores of the row into registers with one TMEM round trip; the
      // S columns are released at once so S_{j+1} can be computed meanwhile.
      uint32_t sv_[128];
      if (ok) {
        tc_fence_after();
        tmem_ld128(t_s, sv_);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive_u32(bar_s_empty);
      } else {
#pragma unroll
        for (int k = 0; k < 128; ++k) sv_[k] = 0xff800000u;   // -inf
      }
      if (valid < kFaN) {
#pragma unroll
        for (int k = 0; k < 128; ++k)
          if (k >= valid) sv_[k] = 0xff800000u;
      }
      // row maximum: four independent chains of 3-input max
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int k = 0; k < 128; k += 2)
        mx[(k >> 1) & 3] = fmax3(mx[(k >> 1) & 3], __uint_as_float(sv_[k]), __uint_as_float(sv_[k + 1]));
      const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      // Lazy reference max: it moves only when a score exceeds it by more than 8
      // (log2 units).  Every block has a valid key, so m is finite from the
      // first block on; exp2(-inf - m) = 0 there.
      const float m_blk = tmax * p.scale_log2;
      const bool move = m_blk > m + 8.0f;
      const float m_new = move ? m_blk : m;
      const float alpha = move ? ex2_approx(m - m_new) : 1.0f;
      // P V of block j-1 has finished: the P buffer is free and O(t) is stable.
      if (j > 0) ok = __all_sync(0xffffffffu, ok && mbar_wait_u32(bar_o_full, (j - 1) & 1, abort_flag));
      // The two tiles take turns on the SFU: tile 0 exponentiates block j after
      // tile 1 finished block j-1, tile 1 after tile 0 finished block j, so one
      // tile's exponentials overlap the other's TMEM reads, maximum and waits.
      exp_turn_begin();
      // P_j = exp2(S * scale - m) over the 128 keys
      const float negm = -m_new;
      float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        __align__(16) __half2 hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = q * 8 + 2 * e;
          float p0, p1;
          if (((q * 4 + e) & 7) < H3B_FA_EMU) {
            ex2_poly_pair(f2_fma(f2_pack(__uint_as_float(sv_[k]), __uint_as_float(sv_[k + 1])),
                                 f2_pack(p.scale_log2, p.scale_log2), f2_pack(negm, negm)),
                          p0, p1);
          } else if (H3B_FA_FMA2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv_[k]), __uint_as_float(sv_[k + 1])),
                             f2_pack(p.scale_log2, p.scale_log2), f2_pack(negm, negm)),
                      x0, x1);
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          } else {
            p0 = ex2_approx(__fmaf_rn(__uint_as_float(sv_[k]), p.scale_log2, negm));
            p1 = ex2_approx(__fmaf_rn(__uint_as_float(sv_[k + 1]), p.scale_log2, negm));
          }
          if (!H3B_FA_ONES) sums[e] += p0 + p1;
          hv[e] = __floats2half2_rn(p0, p1);
        }
        // keys q*8..q*8+7: swizzle column q/8, 16-byte chunk q%8 of this row
        if (ok)
          st_shared_v4(prow + (q >> 3) * (kFaPBytes / 2) + (((q & 7) ^ (row & 7)) << 4),
                       *reinterpret_cast<const uint4*>(hv));
      }
      exp_turn_end(j);
      // O(t) rescale when the reference max moved (before P V of block j reads
      // it).  tcgen05.ld / st are warp-collective, so the whole warp runs it when
      // any of its rows moved (alpha = 1 for the others).
      if (ok && j > 0) {
        tc_fence_after();
        if (__any_sync(0xffffffffu, move)) {
#pragma unroll
          for (int c = 0; c < (H3B_FA_ONES ? 3 : 2); ++c) {   // O and, with the ones, its row sums
            uint32_t r[32];
            tmem_ld32(t_o + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int d = 0; d < 32; ++d) r[d] = __float_as_uint(__fmul_rn(__uint_as_float(r[d]), alpha));
            tmem_st32(t_o + c * 32, r);
          }
          tmem_st_wait();
        }
      }
      if (ok) {
        tc_fence_before();
        fence_proxy_async_smem();
        mbar_arrive_u32(bar_p_full);
      }
      if (!H3B_FA_ONES) l = __fmaf_rn(l, alpha, (sums[0] + sums[1]) + (sums[2] + sums[3]));
      m = m_new;
    }
    if (n_blocks > 0) ok = __all_sync(0xffffffffu, ok && mbar_wait_u32(bar_o_full, (n_blocks - 1) & 1, abort_flag));
    const int qrow = (qt0 + tile) * kFaM + row;
    if (H3B_FA_ONES && ok) {
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(t_o + kFaD, r);
      tmem_ld_wait();
      l = __uint_as_float(r[0]);
    }
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    __half* dst = p.out + b * p.os[0] + h * p.os[1] + static_cast<int64_t>(qrow) * p.os[2];
    if (ok) tc_fence_after();
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      if (ok) {
        tmem_ld32(t_o + c * 32, r);
        tmem_ld_wait();
      }
      if (ok && qrow < p.q_len) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          __align__(16) __half2 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            hv[e] = __floats2half2_rn(__uint_as_float(r[q * 8 + 2 * e]) * inv, __uint_as_float(r[q * 8 + 2 * e + 1]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + q * 8) = *reinterpret_cast<const uint4*>(hv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kFaTmemCols);
}

}  // namespace h3b

namespace {

int make_qkv_map(CUtensorMap* map, const void* base, const int64_t* strides_el, int64_t len, int64_t heads,
                 int64_t batch) {
  uint64_t dims[4] = {64, (uint64_t)len, (uint64_t)heads, (uint64_t)batch};
  uint64_t str[3] = {(uint64_t)strides_el[2] * 2, (uint64_t)strides_el[1] * 2, (uint64_t)strides_el[0] * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  uint32_t es[4] = {1, 1, 1, 1};
  return h3b_host::encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims, str, box, es,
                                CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

extern "C" int h3b_attention_f16(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                 const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                                 int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, float scale,
                                 h3b_stream_t stream) {
  const char* name = "h3b_attention_f16";
  using namespace h3b;
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0)
    return h3b_host::set_error(H3B_EINVAL, "%s: empty problem", name);
  if (batch > 65535 || heads > 65535 || q_len > (int64_t(1) << 30) || kv_len > (int64_t(1) << 30))
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: problem too large", name);
  if ((reinterpret_cast<uintptr_t>(out) & 15u) || out_strides[0] % 8 || out_strides[1] % 8 || out_strides[2] % 8)
    return h3b_host::set_error(H3B_EINVAL, "%s: output rows must be 16-byte aligned", name);
  CUtensorMap mq, mk, mv;
  int rc = make_qkv_map(&mq, q, q_strides, q_len, heads, batch);
  if (rc) return rc;
  rc = make_qkv_map(&mk, k, k_strides, kv_len, heads, batch);
  if (rc) return rc;
  rc = make_qkv_map(&mv, v, v_strides, kv_len, heads, batch);
  if (rc) return rc;
  FaParams p{};
  p.q_len = (int)q_len;
  p.kv_len = (int)kv_len;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__half*>(out);
  for (int i = 0; i < 3; ++i) p.os[i] = out_strides[i];
  constexpr size_t smem = kFaSmemBytes;
  static_assert(smem <= 232448, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  dim3 grid((unsigned)((q_len + kFaTiles * kFaM - 1) / (kFaTiles * kFaM)), (unsigned)heads, (unsigned)batch);
  attention_tc_kernel<<<grid, kFaThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mq, mk, mv, p);
  return h3b_host::check_launch(name);
}
