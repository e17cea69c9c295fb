// Memory-bound encoder producers (HBM roofline kernels).
//
// All activations are NDHWC fp16 ("channels_last_3d").  One thread owns one
// 16-byte vector of 8 consecutive channels, so every global access is a
// coalesced 16-byte (fp16) or 8-byte (int8) transaction.
//
//   gn_partial_kernel   per (b, frame, chunk of positions): per-group chunk mean
//                       and centred M2 (two passes over registers), the
//                       statistic the GroupNorm merge consumes.
//   gn_merge_kernel     Chan merge of the chunk partials -> (mean, rstd) per
//                       (b, frame, group).
//   norm_pack_kernel    GroupNorm affine -> fp16 -> SiLU -> fp16, reflect pad 1
//                       in H/W and two zero frames in front; modes: absmax of the
//                       interior, INT8 with the per-tensor scale, or fp16 output.
//   residual_pack_kernel, quantize kernels, finalize_pixels_kernel,
//   blend_accumulate_kernel (one tile's weighted term added into the blend canvas).

#include "common.cuh"

namespace h3b {

constexpr int kGroups = 32;
constexpr int kVec = 8;            // fp16 channels per thread vector
constexpr int kPackThreads = 256;
constexpr int kStatThreads = 256;
constexpr int kStatVecsPerThread = 64;    // 16-byte vectors each thread streams per chunk
constexpr int kStatElemsPerCta = kStatThreads * kStatVecsPerThread * kVec;

struct NormShape {
  int B, C, D, H, W;        // the stored (source) tensor
  int positions_per_chunk;  // P
  int nchunks;              // ceil(H*W / P)
  // Optional nearest upsampling folded into the producer (fp16 mode only):
  // the normalized tensor is up(x) with spatial factor us (1 or 2) and causal
  // temporal doubling ut (0 or 1: frame 0 once, every later frame twice).
  int us, ut;
  int Du, Hu, Wu;           // logical (upsampled) frame / row / column counts
};

__device__ __forceinline__ void load_h8(const __half* src, float (&v)[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void store_h8(__half* dst, const float (&v)[8]) {
  __align__(16) __half2 h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}

// ---------------------------------------------------------------------------
// GroupNorm statistics, pass 1: chunk partials (+ per-channel min / max).
// grid = (nchunks, B*D), block = 256.  The chunk covers P = 16384 / C positions
// of one (b, frame); thread tid owns channel vector v = tid % (C/8) and the
// positions tid / (C/8) + k * (256 / (C/8)).  Per-channel values are combined
// across the threads that share v with shuffles, then across warps in shared
// memory.
// ---------------------------------------------------------------------------
// Combine a[8] (per-channel values of this thread's vector) over all threads
// holding the same channel vector; result for channel c lands in chan[c].
// kind 0 = sum, 1 = min, 2 = max.
template <int KIND>
__device__ __forceinline__ void channel_reduce(float (&a)[8], int vpp, int C, float* red, float* chan) {
  auto op = [](float x, float y) { return KIND == 0 ? __fadd_rn(x, y) : (KIND == 1 ? fminf(x, y) : fmaxf(x, y)); };
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (vpp < 32) {
    for (int o = 16; o >= vpp; o >>= 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = op(a[j], __shfl_xor_sync(0xffffffffu, a[j], o));
    }
  }
  __syncthreads();  // previous users of red / chan are done
  if (lane < (vpp < 32 ? vpp : 32)) {
#pragma unroll
    for (int j = 0; j < 8; ++j) red[(warp * 32 + lane) * 8 + j] = a[j];
  }
  __syncthreads();
  const int nwarps = kStatThreads / 32;
  for (int c = threadIdx.x; c < C; c += kStatThreads) {
    const int v = c >> 3, j = c & 7;
    float acc;
    if (vpp <= 32) {
      acc = red[v * 8 + j];
      for (int w = 1; w < nwarps; ++w) acc = op(acc, red[(w * 32 + v) * 8 + j]);
    } else {
      const int step = vpp / 32;
      int w = v / 32;
      acc = red[(w * 32 + (v & 31)) * 8 + j];
      for (w += step; w < nwarps; w += step) acc = op(acc, red[(w * 32 + (v & 31)) * 8 + j]);
    }
    chan[c] = acc;
  }
  __syncthreads();
}

// (count, mean, M2) of a set of samples; Chan's pairwise merge.
struct Moments {
  float n, mean, m2;
};

__device__ __forceinline__ Moments merge_moments(Moments a, Moments b) {
  if (b.n == 0.0f) return a;
  if (a.n == 0.0f) return b;
  const float n = a.n + b.n;
  const float d = b.mean - a.mean;
  const float f = __fdiv_rn(b.n, n);
  return Moments{n, __fmaf_rn(d, f, a.mean), a.m2 + b.m2 + d * d * a.n * f};
}

// Streams one chunk of positions of one (b, frame).  GPV = GroupNorm groups
// per 8-channel vector (8 / (C/32) when C/32 < 8, else 1), a compile-time
// constant so every accumulator stays in registers.  Per group of its vector a
// thread keeps a shift (its first sample of the group's first channel), the
// shifted sum and sum of squares; with MINMAX also the per-channel min / max.
// The shifted sums become per-thread (n, mean, M2) per group, merged per group
// in shared memory with Chan's formula; the chunk's (mean, M2) per group goes
// to `partials`.  The shift is taken before the loop so the loop body is
// branch-free and its unrolled loads overlap.
template <int GPV, bool MINMAX>
__global__ void __launch_bounds__(kStatThreads, 3) gn_partial_kernel(const __half* __restrict__ x,
                                                                  const __half* __restrict__ pre_bias,
                                                                  NormShape s, float2* __restrict__ partials,
                                                                  unsigned int* __restrict__ cmin,
                                                                  unsigned int* __restrict__ cmax) {
  constexpr int kPerGroup = kVec / GPV;       // channels of one group inside a vector
  __shared__ Moments slots[kStatThreads][GPV];
  const int tid = threadIdx.x;
  const int chunk = blockIdx.x;
  const int bt = blockIdx.y;
  const int vpp = s.C / kVec;                 // vectors per position
  const int pos_per_iter = kStatThreads / vpp;
  const int v = tid % vpp;
  const int c0 = v * kVec;
  const int HW = s.H * s.W;
  const int p0 = chunk * s.positions_per_chunk;
  const int valid_pos = min(s.positions_per_chunk, HW - p0);
  const int cg = s.C / kGroups;

  // fp16(x + pre_bias) as one fp16 add per pair: identical to rounding the fp32
  // sum to fp16 (fp32 carries more than 2*11 + 2 bits).
  const uint4 pbv = pre_bias != nullptr ? *reinterpret_cast<const uint4*>(pre_bias + c0) : make_uint4(0, 0, 0, 0);
  auto load_biased = [&](const __half* src, float (&v)[8]) {
    uint4 raw = *reinterpret_cast<const uint4*>(src);
    __half2* h = reinterpret_cast<__half2*>(&raw);
    const __half2* pb = reinterpret_cast<const __half2*>(&pbv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(pre_bias != nullptr ? __hadd2(h[j], pb[j]) : h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  };

  const __half* base = x + (static_cast<int64_t>(bt) * HW + p0) * s.C + c0;
  const __half2* pb2 = reinterpret_cast<const __half2*>(&pbv);
  float shift[GPV], s1[GPV], s2[GPV];
  float mn[MINMAX ? 8 : 1], mx[MINMAX ? 8 : 1];
  const int p_first = tid / vpp;
  const int n = p_first < valid_pos ? (valid_pos - p_first + pos_per_iter - 1) / pos_per_iter : 0;
  {
    float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (n > 0) load_biased(base + static_cast<int64_t>(p_first) * s.C, f);
#pragma unroll
    for (int g = 0; g < GPV; ++g) shift[g] = f[g * kPerGroup];
  }
  // Per channel pair (2e, 2e+1): shifted sum and sum of squares as packed
  // fp32 pairs, min / max on the fp16 values themselves (exact).
  float2 sp[4], s1p[4], s2p[4];
  __half2 mn2[4], mx2[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    sp[e] = make_float2(shift[(2 * e) / kPerGroup], shift[(2 * e + 1) / kPerGroup]);
    s1p[e] = make_float2(0.0f, 0.0f);
    s2p[e] = make_float2(0.0f, 0.0f);
    mn2[e] = __floats2half2_rn(INFINITY, INFINITY);
    mx2[e] = __floats2half2_rn(-INFINITY, -INFINITY);
  }
  auto accumulate = [&](const uint4& raw) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __half2 hv = pre_bias != nullptr ? __hadd2(h[e], pb2[e]) : h[e];
      if constexpr (MINMAX) {
        mn2[e] = __hmin2(mn2[e], hv);
        mx2[e] = __hmax2(mx2[e], hv);
      }
      const float2 d = f2x_sub(__half22float2(hv), sp[e]);
      s1p[e] = f2x_add(s1p[e], d);
      s2p[e] = f2x_fma(d, d, s2p[e]);
    }
  };
  // Eight 16-byte loads in flight per thread, then the tail one at a time.
  const int64_t step = static_cast<int64_t>(pos_per_iter) * s.C;
  const __half* src = base + static_cast<int64_t>(p_first) * s.C;
  int left = n;
  for (; left >= 8; left -= 8, src += 8 * step) {
    uint4 raw[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) raw[k] = __ldg(reinterpret_cast<const uint4*>(src + k * step));
#pragma unroll
    for (int k = 0; k < 8; ++k) accumulate(raw[k]);
  }
  for (; left > 0; --left, src += step) accumulate(__ldg(reinterpret_cast<const uint4*>(src)));
#pragma unroll
  for (int g = 0; g < GPV; ++g) {
    s1[g] = 0.0f;
    s2[g] = 0.0f;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    s1[(2 * e) / kPerGroup] += s1p[e].x;
    s2[(2 * e) / kPerGroup] += s2p[e].x;
    s1[(2 * e + 1) / kPerGroup] += s1p[e].y;
    s2[(2 * e + 1) / kPerGroup] += s2p[e].y;
    if constexpr (MINMAX) {
      mn[2 * e] = __low2float(mn2[e]);
      mn[2 * e + 1] = __high2float(mn2[e]);
      mx[2 * e] = __low2float(mx2[e]);
      mx[2 * e + 1] = __high2float(mx2[e]);
    }
  }
  const float fn = static_cast<float>(n * kPerGroup);
#pragma unroll
  for (int g = 0; g < GPV; ++g) {
    Moments m{fn, 0.0f, 0.0f};
    if (n > 0) {
      const float mu = __fdiv_rn(s1[g], fn);
      m.mean = shift[g] + mu;
      m.m2 = fmaxf(s2[g] - s1[g] * mu, 0.0f);
    }
    slots[tid][g] = m;
  }
  __syncthreads();
  if (tid < kGroups) {
    // group tid: channels [tid*cg, (tid+1)*cg) -> vectors v0..v1, slot within the vector
    Moments acc{0.0f, 0.0f, 0.0f};
    const int v0 = (tid * cg) / kVec, v1 = ((tid + 1) * cg - 1) / kVec;
    const int sl = GPV == 1 ? 0 : (tid * cg % kVec) / cg;
    for (int vv = v0; vv <= v1; ++vv)
      for (int t = vv; t < kStatThreads; t += vpp) acc = merge_moments(acc, slots[t][sl]);
    partials[(static_cast<int64_t>(bt) * s.nchunks + chunk) * kGroups + tid] = make_float2(acc.mean, acc.m2);
  }
  if constexpr (MINMAX) {
    __shared__ float red[kStatThreads * kVec];
    __shared__ float chan[2048];
    channel_reduce<1>(mn, vpp, s.C, red, chan);
    for (int c = tid; c < s.C; c += kStatThreads) atomicMin(&cmin[static_cast<int64_t>(bt) * s.C + c], float_to_ordered(chan[c]));
    channel_reduce<2>(mx, vpp, s.C, red, chan);
    for (int c = tid; c < s.C; c += kStatThreads) atomicMax(&cmax[static_cast<int64_t>(bt) * s.C + c], float_to_ordered(chan[c]));
  }
}

__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The producer's per-element value: GroupNorm affine -> fp16 -> SiLU -> fp16.
// exp / divide are the fast SFU forms, the lowering of the reference kernels.
// The affine is folded per channel into one fp32 fma (a = rstd * gamma,
// b = beta - mean * a); SiLU uses the SFU's ex2 and rcp.  norm_pack_kernel
// evaluates exactly this arithmetic, so absmax candidates taken from the
// per-channel extremes match the values it writes.
__device__ __forceinline__ float norm_silu_value(float v, float mean, float rstd, float gamma, float beta) {
  const float a = __fmul_rn(rstd, gamma);
  const float b = __fsub_rn(beta, __fmul_rn(mean, a));
  const float y = round_fp16(__fmaf_rn(v, a, b));
  const float d = __fadd_rn(ex2_ftz(__fmul_rn(y, -1.4426950408889634f)), 1.0f);
  return round_fp16(__fmul_rn(y, rcp_ftz(d)));
}

// GroupNorm statistics, pass 2: one warp per group of one (b, frame).  With
// cmin/cmax it also folds the per-tensor absmax candidates: the normalized
// value is monotone in x per channel and SiLU is increasing for z >= 0 while
// |SiLU(z)| < 0.2786 for z < 0, so the extremes give the exact absmax whenever
// it is >= kAmaxExact; below that the full interior scan decides.
constexpr float kAmaxExact = 0.28f;

__global__ void gn_merge_kernel(const float2* __restrict__ partials, NormShape s, float eps,
                                float2* __restrict__ stats, const unsigned int* __restrict__ cmin,
                                const unsigned int* __restrict__ cmax, const __half* __restrict__ gamma,
                                const __half* __restrict__ beta, float* amax) {
  const int bt = blockIdx.x;
  const int g = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int HW = s.H * s.W;
  const int cg = s.C / kGroups;
  const float total = static_cast<float>(HW) * cg;
  const float2* part = partials + static_cast<int64_t>(bt) * s.nchunks * kGroups + g;
  float wsum = 0.0f;
  for (int i = lane; i < s.nchunks; i += 32) {
    const float cnt = static_cast<float>(min(s.positions_per_chunk, HW - i * s.positions_per_chunk) * cg);
    wsum = __fmaf_rn(part[i * kGroups].x, cnt, wsum);
  }
  const float mean = __fdiv_rn(warp_sum(wsum), total);
  float m2 = 0.0f;
  for (int i = lane; i < s.nchunks; i += 32) {
    const float cnt = static_cast<float>(min(s.positions_per_chunk, HW - i * s.positions_per_chunk) * cg);
    const float2 pm = part[i * kGroups];
    const float delta = pm.x - mean;
    m2 += pm.y + cnt * delta * delta;
  }
  const float var = __fdiv_rn(warp_sum(m2), total);
  const float rstd = rsqrtf(fmaxf(var, 0.0f) + eps);
  if (lane == 0) stats[static_cast<int64_t>(bt) * kGroups + g] = make_float2(mean, rstd);
  if (cmin == nullptr) return;
  float cand = 0.0f;
  for (int c = g * cg + lane; c < (g + 1) * cg; c += 32) {
    const float gm = __half2float(gamma[c]), bb = __half2float(beta[c]);
    const float lo = ordered_to_float(cmin[static_cast<int64_t>(bt) * s.C + c]);
    const float hi = ordered_to_float(cmax[static_cast<int64_t>(bt) * s.C + c]);
    cand = fmaxf(cand, fabsf(norm_silu_value(lo, mean, rstd, gm, bb)));
    cand = fmaxf(cand, fabsf(norm_silu_value(hi, mean, rstd, gm, bb)));
  }
  cand = warp_max(cand);
  if (lane == 0) atomic_max_nonneg(amax, cand);
}

// ---------------------------------------------------------------------------
// Norm -> SiLU -> pad producer.  MODE 0: absmax of the interior (atomic on
// amax_out); MODE 1: INT8 output with scale from amax; MODE 2: fp16 output.
// One CTA per output row (b, frame, h): the row's (w, channel-vector) pairs are
// walked with shifts only (C/8 is a power of two), so the kernel is bound by
// HBM, not by index arithmetic.
// ---------------------------------------------------------------------------
template <int MODE, int GPV>
__global__ void __launch_bounds__(kPackThreads, GPV == 8 ? 3 : 4) norm_pack_kernel(const __half* __restrict__ x,
                                                                    const __half* __restrict__ pre_bias,
                                                                    const __half* __restrict__ gamma,
                                                                    const __half* __restrict__ beta,
                                                                    const float2* __restrict__ stats, NormShape s,
                                                                    float* amax, float* scale_out, void* out) {
  const int vpp = s.C / kVec;
  const int vshift = __ffs(vpp) - 1;
  const int cg = s.C / kGroups;
  // MODE 0 walks the interior rows only: the padded ring duplicates interior
  // values or is zero, so it cannot raise the maximum.
  const int Hr = (MODE == 0) ? s.Hu : s.Hu + 2;
  const int Wr = (MODE == 0) ? s.Wu : s.Wu + 2;
  const int Dr = (MODE == 0) ? s.Du : s.Du + 2;
  int row = blockIdx.x;
  const int hr = row % Hr;
  row /= Hr;
  const int tr = row % Dr;
  const int b = row / Dr;
  const int tu = (MODE == 0) ? tr : tr - 2;                 // logical frame
  int hu = (MODE == 0) ? hr : hr - 1;                        // logical row, reflected
  hu = hu < 0 ? -hu : (hu >= s.Hu ? 2 * s.Hu - 2 - hu : hu);
  const bool frame_ok = tu >= 0;
  const int t = s.ut ? (tu + 1) >> 1 : tu;                   // source frame
  const int h = s.us == 2 ? hu >> 1 : hu;                    // source row
  if (MODE == 0 && *amax >= kAmaxExact) return;  // the extremes already gave the exact absmax
  float scale = 1.0f;
  if (MODE == 1) {
    scale = __fmul_rn(*amax, 1.0f / 127.0f);
    if (!(scale > 0.0f)) scale = 1.0f;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  }
  const float inv_scale = __frcp_rn(scale);
  const int row_vecs = Wr * vpp;
  const __half* xrow = x + ((static_cast<int64_t>(b) * s.D + (frame_ok ? t : 0)) * s.H + h) * s.W * s.C;
  const float2* st = stats + (static_cast<int64_t>(b) * s.D + (frame_ok ? t : 0)) * kGroups;
  const int64_t out_row = static_cast<int64_t>(blockIdx.x) * row_vecs;
  // The block stride (256 vectors) is a multiple of C/8, so every thread keeps
  // one channel vector: its folded affine constants are computed once.
  const int v = threadIdx.x & (vpp - 1);
  const int c0 = v * kVec;
  const uint4 pbv = pre_bias != nullptr ? *reinterpret_cast<const uint4*>(pre_bias + c0) : make_uint4(0, 0, 0, 0);
  // GroupNorm affine folded per channel: ((v - mean) * rstd) * gamma + beta
  // = v * a + b with a = rstd * gamma, b = beta - mean * a (fp32; the fp16
  // rounding that follows absorbs the reassociation).
  float2 aff_a[4], aff_b[4];
  {
    const uint4 gm = *reinterpret_cast<const uint4*>(gamma + c0);
    const uint4 bt = *reinterpret_cast<const uint4*>(beta + c0);
    const __half2* g2 = reinterpret_cast<const __half2*>(&gm);
    const __half2* b2 = reinterpret_cast<const __half2*>(&bt);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 mr0 = st[(c0 + 2 * e) / cg];
      const float2 mr1 = st[(c0 + 2 * e + 1) / cg];
      const float2 gf = __half22float2(g2[e]), bf = __half22float2(b2[e]);
      aff_a[e] = make_float2(__fmul_rn(mr0.y, gf.x), __fmul_rn(mr1.y, gf.y));
      aff_b[e] = make_float2(__fsub_rn(bf.x, __fmul_rn(mr0.x, aff_a[e].x)), __fsub_rn(bf.y, __fmul_rn(mr1.x, aff_a[e].y)));
    }
  }
  auto column = [&](int i) {
    int w = (i >> vshift) - ((MODE == 0) ? 0 : 1);
    w = w < 0 ? -w : (w >= s.Wu ? 2 * s.Wu - 2 - w : w);
    return s.us == 2 ? (w >> 1) : w;
  };
  // GroupNorm affine -> fp16 -> SiLU -> fp16 for 8 channels, two at a time.
  // fp16(x + pre_bias) is one fp16 add (an fp16 sum rounded once equals the
  // fp32 sum rounded to fp16: fp32 carries more than 2*11 + 2 bits), the fp32
  // steps run as packed pairs, every fp16 rounding is one packed conversion.
  // SiLU(y) = y / (1 + 2^(-y log2 e)) with the SFU's ex2 and rcp (the fast
  // exp / divide of the reference kernels' lowering).
  auto values = [&](const uint4& raw, float (&z)[8]) {
    const __half2* xv = reinterpret_cast<const __half2*>(&raw);
    const __half2* p2 = reinterpret_cast<const __half2*>(&pbv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(pre_bias != nullptr ? __hadd2(xv[e], p2[e]) : xv[e]);
      const float2 ya = f2x_fma(f, aff_a[e], aff_b[e]);
      const float2 yr = __half22float2(__floats2half2_rn(ya.x, ya.y));
      const float2 t = f2x_mul(yr, make_float2(-1.4426950408889634f, -1.4426950408889634f));
      const float2 d = f2x_add(make_float2(ex2_ftz(t.x), ex2_ftz(t.y)), make_float2(1.0f, 1.0f));
      const float2 sv = f2x_mul(yr, make_float2(rcp_ftz(d.x), rcp_ftz(d.y)));
      const float2 zz = __half22float2(__floats2half2_rn(sv.x, sv.y));
      z[2 * e] = zz.x;
      z[2 * e + 1] = zz.y;
    }
  };
  float local_max = 0.0f;
  auto load = [&](int i) {
    if (!frame_ok || i >= row_vecs) return make_uint4(0, 0, 0, 0);
    return __ldg(reinterpret_cast<const uint4*>(xrow + static_cast<int64_t>(column(i)) * s.C + c0));
  };
  // Software pipeline: while one vector is computed, the next two of this
  // thread are already in flight.
  uint4 nxt0 = load(threadIdx.x), nxt1 = load(threadIdx.x + kPackThreads);
  for (int i = threadIdx.x; i < row_vecs; i += kPackThreads) {
    const uint4 raw = nxt0;
    nxt0 = nxt1;
    nxt1 = load(i + 2 * kPackThreads);
    float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (frame_ok) values(raw, z);
    if (MODE == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) local_max = fmaxf(local_max, fabsf(z[j]));
    } else if (MODE == 1) {
      uint32_t tb[8];
      quant_bytes8(z, scale, inv_scale, tb);
      reinterpret_cast<uint2*>(out)[out_row + i] =
          make_uint2(pack_low_bytes(tb[0], tb[1], tb[2], tb[3]), pack_low_bytes(tb[4], tb[5], tb[6], tb[7]));
    } else {
      store_h8(reinterpret_cast<__half*>(out) + (out_row + i) * kVec, z);
    }
  }
  if (MODE == 0) {
    __shared__ float wmax[kPackThreads / 32];
    local_max = warp_max(local_max);
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = local_max;
    __syncthreads();
    if (threadIdx.x < 32) {
      float m = threadIdx.x < kPackThreads / 32 ? wmax[threadIdx.x] : 0.0f;
      m = warp_max(m);
      if (threadIdx.x == 0) atomic_max_nonneg(amax, m);
    }
  }
}

// ---------------------------------------------------------------------------
// Per-token INT8 producer: GroupNorm affine -> fp16 -> SiLU -> fp16 -> reflect /
// causal pad, then one scale per padded position (absmax over its C channels
// * fp32(1/127), 0 -> 1) and half-away quantization.  One warp per position:
// lane l owns channels [l*CPL, (l+1)*CPL) with CPL = C/32, which is exactly
// GroupNorm group l, so each lane needs one (mean, rstd) pair; the position's
// absmax is a warp max.
// ---------------------------------------------------------------------------
template <int CPL>
__global__ void __launch_bounds__(256) norm_pack_token_kernel(const __half* __restrict__ x,
                                                              const __half* __restrict__ pre_bias,
                                                              const __half* __restrict__ gamma,
                                                              const __half* __restrict__ beta,
                                                              const float2* __restrict__ stats, NormShape s,
                                                              int8_t* __restrict__ q, float* __restrict__ scales) {
  static_assert(CPL == 4 || CPL == 8 || CPL == 16, "128, 256 or 512 channels");
  constexpr int kPairs = CPL / 2;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int Dp = s.D + 2, Hp = s.H + 2, Wp = s.W + 2;
  const int64_t npos = static_cast<int64_t>(s.B) * Dp * Hp * Wp;
  const int c0 = lane * CPL;
  __half2 g2[kPairs], b2[kPairs], p2[kPairs];
#pragma unroll
  for (int k = 0; k < kPairs; ++k) {
    g2[k] = reinterpret_cast<const __half2*>(gamma + c0)[k];
    b2[k] = reinterpret_cast<const __half2*>(beta + c0)[k];
    p2[k] = pre_bias != nullptr ? reinterpret_cast<const __half2*>(pre_bias + c0)[k] : __floats2half2_rn(0.f, 0.f);
  }
  for (int64_t pos = warp0; pos < npos; pos += nwarps) {
    int64_t r = pos;
    const int wp = static_cast<int>(r % Wp); r /= Wp;
    const int hp = static_cast<int>(r % Hp); r /= Hp;
    const int tp = static_cast<int>(r % Dp);
    const int b = static_cast<int>(r / Dp);
    const int t = tp - 2;
    int h = hp - 1, w = wp - 1;
    h = h < 0 ? -h : (h >= s.H ? 2 * s.H - 2 - h : h);
    w = w < 0 ? -w : (w >= s.W ? 2 * s.W - 2 - w : w);
    float z[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) z[k] = 0.0f;
    if (t >= 0) {
      const __half2* src = reinterpret_cast<const __half2*>(
          x + (((static_cast<int64_t>(b) * s.D + t) * s.H + h) * s.W + w) * s.C + c0);
      __half2 xv[kPairs];
#pragma unroll
      for (int k = 0; k < kPairs; ++k) xv[k] = src[k];
      const float2 mr = stats[(static_cast<int64_t>(b) * s.D + t) * kGroups + lane];
#pragma unroll
      for (int k = 0; k < kPairs; ++k) {
        const float2 f = __half22float2(pre_bias != nullptr ? __hadd2(xv[k], p2[k]) : xv[k]);
        const float2 n = f2x_mul(f2x_sub(f, make_float2(mr.x, mr.x)), make_float2(mr.y, mr.y));
        const float2 ya = f2x_add(f2x_mul(n, __half22float2(g2[k])), __half22float2(b2[k]));
        const float2 yr = __half22float2(__floats2half2_rn(ya.x, ya.y));
        const float s0 = __fdividef(yr.x, __fadd_rn(1.0f, __expf(-yr.x)));
        const float s1 = __fdividef(yr.y, __fadd_rn(1.0f, __expf(-yr.y)));
        const float2 zz = __half22float2(__floats2half2_rn(s0, s1));
        z[2 * k] = zz.x;
        z[2 * k + 1] = zz.y;
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) amax = fmaxf(amax, fabsf(z[k]));
    amax = warp_max(amax);
    float scale = __fmul_rn(amax, 1.0f / 127.0f);
    if (!(scale > 0.0f)) scale = 1.0f;
    const float inv_scale = __frcp_rn(scale);
    uint32_t tb[CPL];
#pragma unroll
    for (int k = 0; k < CPL; k += 2) quant_byte_bits2(z[k], z[k + 1], scale, inv_scale, tb[k], tb[k + 1]);
    int8_t* dst = q + pos * s.C + c0;
    if constexpr (CPL == 4) {
      *reinterpret_cast<uint32_t*>(dst) = pack_low_bytes(tb[0], tb[1], tb[2], tb[3]);
    } else if constexpr (CPL == 8) {
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(pack_low_bytes(tb[0], tb[1], tb[2], tb[3]), pack_low_bytes(tb[4], tb[5], tb[6], tb[7]));
    } else {
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(pack_low_bytes(tb[0], tb[1], tb[2], tb[3]), pack_low_bytes(tb[4], tb[5], tb[6], tb[7]),
                     pack_low_bytes(tb[8], tb[9], tb[10], tb[11]), pack_low_bytes(tb[12], tb[13], tb[14], tb[15]));
    }
    if (lane == 0) scales[pos] = scale;
  }
}

// ---------------------------------------------------------------------------
// Residual + bias pack with right/bottom reflect (+1) and two causal zero
// frames: y = fp16(r + (x + bias)) in fp32.  One CTA per output row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kPackThreads) residual_pack_kernel(const __half* __restrict__ x,
                                                                     const __half* __restrict__ r,
                                                                     const __half* __restrict__ bias, int B, int C,
                                                                     int D, int H, int W, __half* __restrict__ y) {
  const int vpp = C / kVec;
  const int Dp = D + 2, Hp = H + 1, Wp = W + 1;
  int row = blockIdx.x;
  const int hp = row % Hp;
  row /= Hp;
  const int tp = row % Dp;
  const int b = row / Dp;
  const int t = tp - 2;
  const int h = hp == H ? H - 2 : hp;
  const int row_vecs = Wp * vpp;
  const int64_t in_row = ((static_cast<int64_t>(b) * D + (t >= 0 ? t : 0)) * H + h) * W * C;
  const int64_t out_row = static_cast<int64_t>(blockIdx.x) * row_vecs;
  for (int i = threadIdx.x; i < row_vecs; i += kPackThreads) {
    const int v = i % vpp;
    const int wp = i / vpp;
    const int w = wp == W ? W - 2 : wp;
    float out[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (t >= 0) {
      const int64_t off = in_row + static_cast<int64_t>(w) * C + v * kVec;
      float fx[8], fr[8], fb[8];
      load_h8(x + off, fx);
      load_h8(r + off, fr);
      load_h8(bias + v * kVec, fb);
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = __fadd_rn(fr[j], __fadd_rn(fx[j], fb[j]));
    }
    store_h8(y + (out_row + i) * kVec, out);
  }
}

// ---------------------------------------------------------------------------
// Per-tensor quantization of an arbitrary-strided fp16 [B,C,D,H,W] tensor into
// NDHWC int8 (destination-ordered, like the reference's legacy kernel).
// ---------------------------------------------------------------------------
struct Strided5 {
  int64_t n[5];  // B, C, D, H, W
  int64_t s[5];
};

__device__ __forceinline__ int64_t strided_offset_ndhwc(const Strided5& t, int64_t i) {
  const int64_t c = i % t.n[1];
  int64_t r = i / t.n[1];
  const int64_t w = r % t.n[4]; r /= t.n[4];
  const int64_t h = r % t.n[3]; r /= t.n[3];
  const int64_t d = r % t.n[2];
  const int64_t b = r / t.n[2];
  return b * t.s[0] + c * t.s[1] + d * t.s[2] + h * t.s[3] + w * t.s[4];
}

__global__ void tensor_absmax_kernel(const __half* __restrict__ x, Strided5 t, int64_t total, float* amax) {
  float m = 0.0f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(__half2float(x[strided_offset_ndhwc(t, i)])));
  __shared__ float wmax[32];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomic_max_nonneg(amax, v);
  }
}

__global__ void tensor_quant_kernel(const __half* __restrict__ x, Strided5 t, int64_t total, const float* amax,
                                    int8_t* __restrict__ q, float* scale_out) {
  float scale = __fmul_rn(*amax, 1.0f / 127.0f);
  if (!(scale > 0.0f)) scale = 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    q[i] = quant_half_away(__half2float(x[strided_offset_ndhwc(t, i)]), scale);
}

// ---------------------------------------------------------------------------
// Pixel finalization: clamp(x*std + mean, 0, 1) without FMA, NaN preserved.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void finalize_pixels_kernel(const T* __restrict__ x, Strided5 t, const float* __restrict__ std3,
                                       const float* __restrict__ mean3, float* __restrict__ out) {
  // One (b, c, frame, row) per block iteration: its source and destination offsets are formed once,
  // the threads stream the row's columns (unit stride on both sides for the decoder canvases).
  const int64_t rows = t.n[0] * 3 * t.n[2] * t.n[3];
  const int64_t width = t.n[4];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t h = r % t.n[3];
    int64_t q = r / t.n[3];
    const int64_t d = q % t.n[2];
    q /= t.n[2];
    const int c = static_cast<int>(q % 3);
    const int64_t b = q / 3;
    const T* src = x + b * t.s[0] + c * t.s[1] + d * t.s[2] + h * t.s[3];
    float* dst = out + r * width;
    const float sd = std3[c], mn = mean3[c];
    for (int64_t w = threadIdx.x; w < width; w += blockDim.x) {
      float v;
      if constexpr (sizeof(T) == 2) v = __half2float(src[w * t.s[4]]);
      else v = src[w * t.s[4]];
      float value = __fadd_rn(__fmul_rn(v, sd), mn);
      value = value < 0.0f ? 0.0f : (value > 1.0f ? 1.0f : value);
      dst[w] = value;
    }
  }
}

// ---------------------------------------------------------------------------
// Overlap blend: canvas[c, t, y, x] += fp32(tile[c, t, y, x]) * weight[y, x],
// the product and the sum each rounded once (no FMA), as the host-side
// `canvas.add_(tile.float() * weight)` rounds them.  One work item is a
// 128-element piece of one (c, t, y) row, so both tensors are read along their
// unit-stride x axis and the weight row is shared by every (c, t).
// ---------------------------------------------------------------------------
struct Strided4 {
  int64_t n[4];
  int64_t s[4];
};

constexpr int kBlendThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kBlendThreads) blend_accumulate_kernel(const T* __restrict__ tile, Strided4 ts,
                                                                       const float* __restrict__ weight,
                                                                       float* __restrict__ canvas, Strided4 cs,
                                                                       int64_t pieces, int pieces_per_row) {
  for (int64_t p = blockIdx.x; p < pieces; p += gridDim.x) {
    const int64_t row = p / pieces_per_row;
    const int64_t x = (p - row * pieces_per_row) * kBlendThreads + threadIdx.x;
    if (x >= ts.n[3]) continue;
    const int64_t y = row % ts.n[2];
    const int64_t ct = row / ts.n[2];
    const int64_t t = ct % ts.n[1];
    const int64_t c = ct / ts.n[1];
    float v;
    if constexpr (sizeof(T) == 2) v = __half2float(tile[c * ts.s[0] + t * ts.s[1] + y * ts.s[2] + x * ts.s[3]]);
    else v = tile[c * ts.s[0] + t * ts.s[1] + y * ts.s[2] + x * ts.s[3]];
    float* dst = canvas + c * cs.s[0] + t * cs.s[1] + y * cs.s[2] + x * cs.s[3];
    *dst = __fadd_rn(*dst, __fmul_rn(v, __ldg(weight + y * ts.n[3] + x)));
  }
}

}  // namespace h3b

// ===========================================================================
// Host entry points
// ===========================================================================
namespace {

using namespace h3b;

int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(h3b_host::num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

bool norm_shape(int64_t B, int64_t C, int64_t D, int64_t H, int64_t W, NormShape* s) {
  if (B <= 0 || C <= 0 || D <= 0 || H < 2 || W < 2) return false;
  if (C % kGroups != 0 || C % kVec != 0 || (kStatThreads % (C / kVec)) != 0) return false;
  if (B * (D + 2) * (H + 2) * (W + 2) * C >= (int64_t(1) << 40)) return false;
  s->B = (int)B; s->C = (int)C; s->D = (int)D; s->H = (int)H; s->W = (int)W;
  s->positions_per_chunk = kStatElemsPerCta / (int)C;
  s->nchunks = (int)((H * W + s->positions_per_chunk - 1) / s->positions_per_chunk);
  s->us = 1; s->ut = 0;
  s->Du = (int)D; s->Hu = (int)H; s->Wu = (int)W;
  return true;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct NormWorkspace {
  float2* partials;
  float2* stats;
  unsigned int* cmin;
  unsigned int* cmax;
  float* amax;
  size_t minmax_bytes;
  size_t bytes;
};

NormWorkspace norm_workspace_layout(const NormShape& s, void* base) {
  NormWorkspace w{};
  const size_t part = align256(sizeof(float2) * (size_t)s.B * s.D * s.nchunks * kGroups);
  const size_t st = align256(sizeof(float2) * (size_t)s.B * s.D * kGroups);
  const size_t mm = align256(sizeof(unsigned int) * (size_t)s.B * s.D * s.C);
  uint8_t* p = static_cast<uint8_t*>(base);
  w.partials = reinterpret_cast<float2*>(p);
  w.stats = reinterpret_cast<float2*>(p + part);
  w.cmin = reinterpret_cast<unsigned int*>(p + part + st);
  w.cmax = reinterpret_cast<unsigned int*>(p + part + st + mm);
  w.amax = reinterpret_cast<float*>(p + part + st + 2 * mm);
  w.minmax_bytes = mm;
  w.bytes = part + st + 2 * mm + 256;
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// GroupNorm groups inside one 8-channel vector (C / 32 channels per group).
int groups_per_vector(int C) {
  const int cg = C / kGroups;
  return cg >= kVec ? 1 : kVec / cg;
}

// norm_pack_kernel<MODE, GPV> for the runtime group count.
template <int MODE>
void launch_norm_pack(unsigned grid, cudaStream_t st, const __half* x, const __half* pb, const __half* g,
                      const __half* b, const float2* stats, const NormShape& s, float* amax, float* scale, void* out) {
  switch (groups_per_vector(s.C)) {
    case 1: norm_pack_kernel<MODE, 1><<<grid, kPackThreads, 0, st>>>(x, pb, g, b, stats, s, amax, scale, out); break;
    case 2: norm_pack_kernel<MODE, 2><<<grid, kPackThreads, 0, st>>>(x, pb, g, b, stats, s, amax, scale, out); break;
    case 4: norm_pack_kernel<MODE, 4><<<grid, kPackThreads, 0, st>>>(x, pb, g, b, stats, s, amax, scale, out); break;
    default: norm_pack_kernel<MODE, 8><<<grid, kPackThreads, 0, st>>>(x, pb, g, b, stats, s, amax, scale, out); break;
  }
}

// Statistics (+ absmax candidates when want_amax): memsets of the min/max/amax
// words, the chunk-partial kernel and the merge kernel.
int run_norm_stats(const void* x, const void* pre_bias, const void* gamma, const void* beta, float eps,
                   const NormShape& s, const NormWorkspace& w, bool want_amax, cudaStream_t st, const char* name) {
  if (want_amax) {
    if (cudaMemsetAsync(w.cmin, 0xFF, w.minmax_bytes, st) != cudaSuccess ||
        cudaMemsetAsync(w.cmax, 0x00, w.minmax_bytes, st) != cudaSuccess ||
        cudaMemsetAsync(w.amax, 0, sizeof(float), st) != cudaSuccess)
      return h3b_host::set_error(H3B_ECUDA, "%s: memset failed", name);
  }
  dim3 grid(s.nchunks, s.B * s.D);
  const __half* xh = static_cast<const __half*>(x);
  const __half* pb = static_cast<const __half*>(pre_bias);
  unsigned int* cmin = want_amax ? w.cmin : nullptr;
  unsigned int* cmax = want_amax ? w.cmax : nullptr;
  switch (groups_per_vector(s.C) * 2 + (want_amax ? 1 : 0)) {
    case 2: gn_partial_kernel<1, false><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 3: gn_partial_kernel<1, true><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 4: gn_partial_kernel<2, false><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 5: gn_partial_kernel<2, true><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 8: gn_partial_kernel<4, false><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 9: gn_partial_kernel<4, true><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    case 16: gn_partial_kernel<8, false><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
    default: gn_partial_kernel<8, true><<<grid, kStatThreads, 0, st>>>(xh, pb, s, w.partials, cmin, cmax); break;
  }
  int rc = h3b_host::check_launch(name);
  if (rc) return rc;
  gn_merge_kernel<<<s.B * s.D, 32 * kGroups, 0, st>>>(w.partials, s, eps, w.stats, want_amax ? w.cmin : nullptr,
                                                       want_amax ? w.cmax : nullptr, static_cast<const __half*>(gamma),
                                                       static_cast<const __half*>(beta), w.amax);
  return h3b_host::check_launch(name);
}

int check_norm_args(const void* x, const void* pre_bias, const void* gamma, const void* beta, const void* out,
                    void* workspace, size_t workspace_bytes, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                    NormShape* s, NormWorkspace* w, const char* name) {
  if (!x || !gamma || !beta || !out || !workspace) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (!norm_shape(B, C, D, H, W, s))
    return h3b_host::set_error(H3B_EUNSUPPORTED,
                               "%s: unsupported shape B=%lld C=%lld D=%lld H=%lld W=%lld (need H,W>=2, C a power of "
                               "two in [32, 2048])",
                               name, (long long)B, (long long)C, (long long)D, (long long)H, (long long)W);
  for (const void* p : std::initializer_list<const void*>{x, gamma, beta, out})
    if (!aligned16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  if (pre_bias && !aligned16(pre_bias)) return h3b_host::set_error(H3B_EINVAL, "%s: pre_bias must be 16-byte aligned", name);
  *w = norm_workspace_layout(*s, workspace);
  if (workspace_bytes < w->bytes)
    return h3b_host::set_error(H3B_EINVAL, "%s: workspace %zu bytes < required %zu", name, workspace_bytes, w->bytes);
  return H3B_OK;
}

}  // namespace

extern "C" {

size_t h3b_norm_workspace_size(int64_t B, int64_t C, int64_t D, int64_t H, int64_t W) {
  NormShape s;
  if (!norm_shape(B, C, D, H, W, &s)) return 0;
  return norm_workspace_layout(s, nullptr).bytes;
}

int h3b_norm_pad_quant(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W, const void* pre_bias,
                       const void* gamma, const void* beta, float eps, int8_t* q, float* scale, void* workspace,
                       size_t workspace_bytes, h3b_stream_t stream) {
  const char* name = "h3b_norm_pad_quant";
  NormShape s;
  NormWorkspace w;
  int rc = check_norm_args(x, pre_bias, gamma, beta, q, workspace, workspace_bytes, B, C, D, H, W, &s, &w, name);
  if (rc) return rc;
  if (!scale) return h3b_host::set_error(H3B_EINVAL, "%s: NULL scale", name);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = run_norm_stats(x, pre_bias, gamma, beta, eps, s, w, true, st, name);
  if (rc) return rc;
  const __half* xh = static_cast<const __half*>(x);
  const __half* pb = static_cast<const __half*>(pre_bias);
  const __half* gh = static_cast<const __half*>(gamma);
  const __half* bh = static_cast<const __half*>(beta);
  launch_norm_pack<0>((unsigned)(B * s.Du * s.Hu), st, xh, pb, gh, bh, w.stats, s, w.amax, nullptr, nullptr);
  rc = h3b_host::check_launch(name);
  if (rc) return rc;
  launch_norm_pack<1>((unsigned)(B * (s.Du + 2) * (s.Hu + 2)), st, xh, pb, gh, bh, w.stats, s, w.amax, scale, q);
  return h3b_host::check_launch(name);
}

int h3b_norm_pad_quant_token(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                             const void* pre_bias, const void* gamma, const void* beta, float eps, int8_t* q,
                             float* scales, void* workspace, size_t workspace_bytes, h3b_stream_t stream) {
  const char* name = "h3b_norm_pad_quant_token";
  NormShape s;
  NormWorkspace w;
  int rc = check_norm_args(x, pre_bias, gamma, beta, q, workspace, workspace_bytes, B, C, D, H, W, &s, &w, name);
  if (rc) return rc;
  if (!scales) return h3b_host::set_error(H3B_EINVAL, "%s: NULL scales", name);
  if (C != 128 && C != 256 && C != 512)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: per-token producer supports C = 128, 256, 512 (got %lld)", name,
                               (long long)C);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = run_norm_stats(x, pre_bias, gamma, beta, eps, s, w, false, st, name);
  if (rc) return rc;
  const int64_t npos = B * (D + 2) * (H + 2) * (W + 2);
  const int64_t blocks = std::min<int64_t>((npos * 32 + 255) / 256, static_cast<int64_t>(h3b_host::num_sms()) * 16);
  const __half* xh = static_cast<const __half*>(x);
  const __half* pb = static_cast<const __half*>(pre_bias);
  const __half* gh = static_cast<const __half*>(gamma);
  const __half* bh = static_cast<const __half*>(beta);
  if (C == 128)
    norm_pack_token_kernel<4><<<(unsigned)blocks, 256, 0, st>>>(xh, pb, gh, bh, w.stats, s, q, scales);
  else if (C == 256)
    norm_pack_token_kernel<8><<<(unsigned)blocks, 256, 0, st>>>(xh, pb, gh, bh, w.stats, s, q, scales);
  else
    norm_pack_token_kernel<16><<<(unsigned)blocks, 256, 0, st>>>(xh, pb, gh, bh, w.stats, s, q, scales);
  return h3b_host::check_launch(name);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of h3b_norm_pad_quant.  Its scratch (the statistics
// partials, per-frame statistics, per-channel min/max words and the absmax
// word) lives in one file-scope device array instead of a caller workspace.
// The host never passes the array's name to a kernel (in host code that name
// is only a stand-in): every call resolves the array's device address with
// cudaGetSymbolAddress while the calling device is current.  Nothing is
// cached, so the address stays right after a cudaDeviceReset or a primary
// context re-creation reloads the module (the lookup is a table access once
// the module is loaded; the first call on a device loads it).
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNormStaticScratchBytes = size_t(4) << 20;  // 4 MiB, held by every device that loads the library
__device__ __align__(256) unsigned char g_norm_static_scratch[kNormStaticScratchBytes];
}  // namespace

int h3b_norm_pad_quant_noalloc(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                               const void* pre_bias, const void* gamma, const void* beta, float eps, int8_t* q,
                               float* scale, h3b_stream_t stream) {
  const char* name = "h3b_norm_pad_quant_noalloc";
  NormShape s;
  if (!norm_shape(B, C, D, H, W, &s))
    return h3b_host::set_error(H3B_EUNSUPPORTED,
                               "%s: unsupported shape B=%lld C=%lld D=%lld H=%lld W=%lld (need H,W>=2, C a power of "
                               "two in [32, 2048])",
                               name, (long long)B, (long long)C, (long long)D, (long long)H, (long long)W);
  const size_t need = norm_workspace_layout(s, nullptr).bytes;
  if (need > kNormStaticScratchBytes)
    return h3b_host::set_error(H3B_EUNSUPPORTED,
                               "%s: this shape needs %zu bytes of scratch, above the %zu-byte static buffer; use "
                               "h3b_norm_pad_quant with a caller workspace",
                               name, need, kNormStaticScratchBytes);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0)
    return h3b_host::set_error(H3B_ECUDA, "%s: no usable current device (%s)", name, cudaGetErrorString(e));
  void* scratch = nullptr;
  e = cudaGetSymbolAddress(&scratch, g_norm_static_scratch);
  if (e != cudaSuccess || scratch == nullptr)
    return h3b_host::set_error(H3B_ECUDA, "%s: cudaGetSymbolAddress of the static scratch failed: %s", name,
                               cudaGetErrorString(e));
  // h3b_norm_pad_quant clears the min / max / absmax words on the stream before
  // use and fully rewrites the partials and statistics, so stale contents from
  // an earlier call never leak into this one.
  return h3b_norm_pad_quant(x, B, C, D, H, W, pre_bias, gamma, beta, eps, q, scale, scratch,
                            kNormStaticScratchBytes, stream);
}

int h3b_norm_pad_f16(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W, const void* pre_bias,
                     const void* gamma, const void* beta, float eps, void* y, void* workspace, size_t workspace_bytes,
                     h3b_stream_t stream) {
  const char* name = "h3b_norm_pad_f16";
  NormShape s;
  NormWorkspace w;
  int rc = check_norm_args(x, pre_bias, gamma, beta, y, workspace, workspace_bytes, B, C, D, H, W, &s, &w, name);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = run_norm_stats(x, pre_bias, gamma, beta, eps, s, w, false, st, name);
  if (rc) return rc;
  launch_norm_pack<2>((unsigned)(B * (s.Du + 2) * (s.Hu + 2)), st, static_cast<const __half*>(x),
                      static_cast<const __half*>(pre_bias), static_cast<const __half*>(gamma),
                      static_cast<const __half*>(beta), w.stats, s, nullptr, nullptr, y);
  return h3b_host::check_launch(name);
}

int h3b_upsample_norm_pad_f16(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W, int up_spatial,
                              int up_temporal, const void* pre_bias, const void* gamma, const void* beta, float eps,
                              void* y, void* workspace, size_t workspace_bytes, h3b_stream_t stream) {
  const char* name = "h3b_upsample_norm_pad_f16";
  if ((up_spatial != 1 && up_spatial != 2) || (up_temporal != 0 && up_temporal != 1))
    return h3b_host::set_error(H3B_EINVAL, "%s: up_spatial must be 1 or 2 and up_temporal 0 or 1", name);
  NormShape s;
  NormWorkspace w;
  int rc = check_norm_args(x, pre_bias, gamma, beta, y, workspace, workspace_bytes, B, C, D, H, W, &s, &w, name);
  if (rc) return rc;
  s.us = up_spatial;
  s.ut = up_temporal;
  s.Du = up_temporal ? (int)(2 * D - 1) : (int)D;
  s.Hu = (int)(H * up_spatial);
  s.Wu = (int)(W * up_spatial);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = run_norm_stats(x, pre_bias, gamma, beta, eps, s, w, false, st, name);
  if (rc) return rc;
  launch_norm_pack<2>((unsigned)(B * (s.Du + 2) * (s.Hu + 2)), st, static_cast<const __half*>(x),
                      static_cast<const __half*>(pre_bias), static_cast<const __half*>(gamma),
                      static_cast<const __half*>(beta), w.stats, s, nullptr, nullptr, y);
  return h3b_host::check_launch(name);
}

int h3b_residual_pack(const void* x, const void* r, const void* bias, int64_t B, int64_t C, int64_t D, int64_t H,
                      int64_t W, void* y, h3b_stream_t stream) {
  const char* name = "h3b_residual_pack";
  if (!x || !r || !bias || !y) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (B <= 0 || C <= 0 || D <= 0 || H < 2 || W < 2 || C % kVec)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: need H,W >= 2 and C %% 8 == 0", name);
  for (const void* p : std::initializer_list<const void*>{x, r, bias, y})
    if (!aligned16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  residual_pack_kernel<<<(unsigned)(B * (D + 2) * (H + 1)), kPackThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), static_cast<const __half*>(r), static_cast<const __half*>(bias), (int)B, (int)C,
      (int)D, (int)H, (int)W, static_cast<__half*>(y));
  return h3b_host::check_launch(name);
}

size_t h3b_quantize_tensor_workspace_size(void) { return 256; }

int h3b_quantize_tensor_i8(const void* x, const int64_t* dims5, const int64_t* strides5, int8_t* q, float* scale,
                           void* workspace, size_t workspace_bytes, h3b_stream_t stream) {
  const char* name = "h3b_quantize_tensor_i8";
  if (!x || !dims5 || !strides5 || !q || !scale || !workspace)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (workspace_bytes < h3b_quantize_tensor_workspace_size())
    return h3b_host::set_error(H3B_EINVAL, "%s: workspace too small", name);
  Strided5 t{};
  int64_t total = 1;
  for (int i = 0; i < 5; ++i) {
    t.n[i] = dims5[i];
    t.s[i] = strides5[i];
    if (dims5[i] <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: activation must be nonempty", name);
    total *= dims5[i];
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* amax = static_cast<float*>(workspace);
  if (cudaMemsetAsync(amax, 0, sizeof(float), st) != cudaSuccess)
    return h3b_host::set_error(H3B_ECUDA, "%s: memset failed", name);
  tensor_absmax_kernel<<<grid_for(total, 256), 256, 0, st>>>(static_cast<const __half*>(x), t, total, amax);
  int rc = h3b_host::check_launch(name);
  if (rc) return rc;
  tensor_quant_kernel<<<grid_for(total, 256), 256, 0, st>>>(static_cast<const __half*>(x), t, total, amax, q, scale);
  return h3b_host::check_launch(name);
}

int h3b_finalize_pixels(const void* x, int x_is_fp16, const int64_t* dims5, const int64_t* strides5,
                        const float* std3, const float* mean3, float* out, h3b_stream_t stream) {
  const char* name = "h3b_finalize_pixels";
  if (!x || !dims5 || !strides5 || !std3 || !mean3 || !out)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (dims5[1] != 3) return h3b_host::set_error(H3B_EINVAL, "%s: nonempty B,3,T,H,W tensor required", name);
  Strided5 t{};
  for (int i = 0; i < 5; ++i) {
    t.n[i] = dims5[i];
    t.s[i] = strides5[i];
    if (dims5[i] <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: nonempty B,3,T,H,W tensor required", name);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t rows = t.n[0] * 3 * t.n[2] * t.n[3];
  const int threads = t.n[4] >= 256 ? 256 : 128;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, static_cast<int64_t>(h3b_host::num_sms()) * 16));
  if (x_is_fp16)
    finalize_pixels_kernel<__half><<<grid, threads, 0, st>>>(static_cast<const __half*>(x), t, std3, mean3, out);
  else
    finalize_pixels_kernel<float><<<grid, threads, 0, st>>>(static_cast<const float*>(x), t, std3, mean3, out);
  return h3b_host::check_launch(name);
}

int h3b_blend_accumulate(const void* tile, int tile_is_fp16, const int64_t* dims4, const int64_t* tile_strides4,
                         const float* weight, float* canvas, const int64_t* canvas_strides4, h3b_stream_t stream) {
  const char* name = "h3b_blend_accumulate";
  if (!tile || !dims4 || !tile_strides4 || !weight || !canvas || !canvas_strides4)
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  Strided4 ts{}, cs{};
  for (int i = 0; i < 4; ++i) {
    if (dims4[i] <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: nonempty C,T,H,W tile required", name);
    if (tile_strides4[i] < 0 || canvas_strides4[i] < 0)
      return h3b_host::set_error(H3B_EINVAL, "%s: negative strides are not supported", name);
    ts.n[i] = cs.n[i] = dims4[i];
    ts.s[i] = tile_strides4[i];
    cs.s[i] = canvas_strides4[i];
  }
  const int pieces_per_row = static_cast<int>((dims4[3] + kBlendThreads - 1) / kBlendThreads);
  const int64_t pieces = dims4[0] * dims4[1] * dims4[2] * pieces_per_row;
  const int64_t cap = static_cast<int64_t>(h3b_host::num_sms()) * 16;
  const int grid = static_cast<int>(pieces < cap ? pieces : cap);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (tile_is_fp16)
    blend_accumulate_kernel<__half><<<grid, kBlendThreads, 0, st>>>(static_cast<const __half*>(tile), ts, weight,
                                                                     canvas, cs, pieces, pieces_per_row);
  else
    blend_accumulate_kernel<float><<<grid, kBlendThreads, 0, st>>>(static_cast<const float*>(tile), ts, weight,
                                                                    canvas, cs, pieces, pieces_per_row);
  return h3b_host::check_launch(name);
}

}  // extern "C"
