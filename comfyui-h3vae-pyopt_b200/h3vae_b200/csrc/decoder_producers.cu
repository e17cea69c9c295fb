// Memory-bound decoder row producers.  One CTA per row (token): every thread
// owns up to MAXV 16-byte vectors of 8 fp16 columns held in registers, so a
// row is read once, reduced with warp shuffles + one shared-memory step, and
// written once.
#include "common.cuh"

namespace h3b {

constexpr int kRowThreads = 256;

__device__ __forceinline__ void ld8(const __half* src, float (&v)[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(src);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void st8(__half* dst, const float* v) {
  __align__(16) __half2 h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}

template <bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* smem) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) smem[w] = v;
  __syncthreads();
  float r = IS_MAX ? 0.0f : 0.0f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) r = IS_MAX ? fmaxf(r, smem[i]) : __fadd_rn(r, smem[i]);
  return r;
}

// Row quantization of act values held in registers (CK contract).
template <int MAXV>
__device__ __forceinline__ void row_quantize_store(const float (&act)[MAXV][8], int nvec, int8_t* qrow, float* srow,
                                                   float* red) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (threadIdx.x + i * kRowThreads < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(act[i][j]));
    }
  }
  amax = block_reduce<true>(amax, red);
  const float scale = row_scale_ck(amax);
  const float denom = round_fp16(scale);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      __align__(8) int8_t q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = quant_row_ck(act[i][j], denom);
      reinterpret_cast<uint2*>(qrow)[v] = *reinterpret_cast<const uint2*>(q);
    }
  }
  if (threadIdx.x == 0) *srow = scale;
}

template <int MAXV>
__global__ void __launch_bounds__(kRowThreads) row_quant_kernel(const __half* __restrict__ x, int K, int64_t ldx,
                                                                int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  float act[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) ld8(x + row * ldx + v * 8, act[i]);
  }
  row_quantize_store<MAXV>(act, nvec, q + row * K, s + row, red);
}

template <int MAXV>
__global__ void __launch_bounds__(kRowThreads) swiglu_quant_kernel(const __half* __restrict__ x, int K,
                                                                   int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  float act[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float g[8], u[8];
      ld8(x + row * 2 * K + v * 8, g);
      ld8(x + row * 2 * K + K + v * 8, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) act[i][j] = round_fp16(__fmul_rn(__fdiv_rn(g[j], __fadd_rn(1.0f, expf(-g[j]))), u[j]));
    }
  }
  row_quantize_store<MAXV>(act, nvec, q + row * K, s + row, red);
}

// raw = fma(a, g, x); h = fp16(raw); RMS over (round_stats ? h : raw);
// act = fp16(h * inv * w); row quantization.  h may alias x.
template <int MAXV>
__global__ void __launch_bounds__(kRowThreads) residual_rms_quant_kernel(
    const __half* x, const __half* __restrict__ a, const __half* __restrict__ g, const __half* __restrict__ w,
    int K, float eps, int round_stats, __half* h, int8_t* __restrict__ q, float* __restrict__ s,
    __half* __restrict__ norm_out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  float hv[MAXV][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float xv[8], av[8], gv[8];
      ld8(x + row * K + v * 8, xv);
      ld8(a + row * K + v * 8, av);
      ld8(g + v * 8, gv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float raw = __fmaf_rn(av[j], gv[j], xv[j]);
        hv[i][j] = round_fp16(raw);
        const float st = round_stats ? hv[i][j] : raw;
        ss = __fadd_rn(ss, __fmul_rn(st, st));
      }
    }
  }
  // Every thread has read its own x vectors before any h store below, so an
  // in-place h (aliasing x) is safe: each element is owned by one thread.
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec && h != nullptr) st8(h + row * K + v * 8, hv[i]);
  }
  ss = block_reduce<false>(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / static_cast<float>(K)), eps));
  float act[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float wv[8];
      ld8(w + v * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) act[i][j] = round_fp16(__fmul_rn(__fmul_rn(hv[i][j], inv), wv[j]));
      if (norm_out != nullptr) st8(norm_out + row * K + v * 8, act[i]);
    }
  }
  row_quantize_store<MAXV>(act, nvec, q + row * K, s + row, red);
}

// y = fp16(x * rsqrt(mean(x^2) + eps) * gamma); optional row quantization.
template <int MAXV, bool QUANT>
__global__ void __launch_bounds__(kRowThreads) rms_norm_kernel(const __half* __restrict__ x,
                                                               const __half* __restrict__ gamma, int K, float eps,
                                                               __half* __restrict__ y, int8_t* __restrict__ q,
                                                               float* __restrict__ s) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  float xv[MAXV][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      ld8(x + row * K + v * 8, xv[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(xv[i][j], xv[i][j]));
    }
  }
  ss = block_reduce<false>(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps));
  float act[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float gv[8];
      ld8(gamma + v * 8, gv);
#pragma unroll
      for (int j = 0; j < 8; ++j) act[i][j] = round_fp16(__fmul_rn(__fmul_rn(xv[i][j], inv), gv[j]));
      if (!QUANT) st8(y + row * K + v * 8, act[i]);
    }
  }
  if (QUANT) row_quantize_store<MAXV>(act, nvec, q + row * K, s + row, red);
}

// raw = fma(o, gate, h); LayerNorm over the row (two-pass in registers);
// y = fp16(fma((raw - mean) * inv, gamma, beta)).
template <int MAXV>
__global__ void __launch_bounds__(kRowThreads) final_ln_kernel(const __half* __restrict__ h,
                                                               const __half* __restrict__ o,
                                                               const __half* __restrict__ gate,
                                                               const __half* __restrict__ gamma,
                                                               const __half* __restrict__ beta, int K, float eps,
                                                               __half* __restrict__ y) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  float raw[MAXV][8];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float hv[8], ov[8], gv[8];
      ld8(h + row * K + v * 8, hv);
      ld8(o + row * K + v * 8, ov);
      ld8(gate + v * 8, gv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        raw[i][j] = __fmaf_rn(ov[j], gv[j], hv[j]);
        sum = __fadd_rn(sum, raw[i][j]);
      }
    }
  }
  const float mean = __fdiv_rn(block_reduce<false>(sum, red), static_cast<float>(K));
  float m2 = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = __fsub_rn(raw[i][j], mean);
        m2 = __fmaf_rn(d, d, m2);
      }
    }
  }
  const float var = __fdiv_rn(block_reduce<false>(m2, red), static_cast<float>(K));
  const float inv = rsqrtf(__fadd_rn(var, eps));
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float gv[8], bv[8], out[8];
      ld8(gamma + v * 8, gv);
      ld8(beta + v * 8, bv);
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = __fmaf_rn(__fmul_rn(__fsub_rn(raw[i][j], mean), inv), gv[j], bv[j]);
      st8(y + row * K + v * 8, out);
    }
  }
}

// ---------------------------------------------------------------------------
// Row kernels for K a multiple of 1024 (the decoder's hidden / FFN widths):
// WPR = K / 1024 warps per row, 8 / WPR rows per 256-thread CTA; lane l of
// warp w of a row owns the 16-byte vectors v * 32 * WPR + w * 32 + l (v < 4),
// so every load / store instruction of a warp covers 512 contiguous bytes.
// The row stays in registers as packed halves; the reductions are warp
// shuffles (plus one shared-memory step when a row spans several warps).
// ---------------------------------------------------------------------------
constexpr int kFastV = 4;   // vectors per lane

template <int WPR>
__device__ __forceinline__ float row_reduce_max(float v, float* red) {
  v = warp_max(v);
  if constexpr (WPR > 1) {
    const int warp = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const int w0 = warp - warp % WPR;
#pragma unroll
    for (int i = 0; i < WPR; ++i) v = fmaxf(v, red[w0 + i]);
  }
  return v;
}

template <int WPR>
__device__ __forceinline__ float row_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  if constexpr (WPR > 1) {
    const int warp = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const int w0 = warp - warp % WPR;
    v = 0.0f;
#pragma unroll
    for (int i = 0; i < WPR; ++i) v = __fadd_rn(v, red[w0 + i]);
  }
  return v;
}

// CK row quantization of 8 fp16 values (quant_row_ck for each): the quotient
// act / denom is formed with the correctly rounded reciprocal of denom, which
// is within 2 ulp of the IEEE quotient; fp16 rounding of the two can differ
// only within that distance of an fp16 midpoint (low 13 mantissa bits
// 0x1000), so those vectors -- and inf / NaN -- take the exact path.  Clamping
// the fp16 value to [-128, 127] before the round-to-nearest-even equals
// clamping after it.  Returns the 8 bytes (byte j = element j).
__device__ __forceinline__ uint2 quant8_ck(const uint4& raw, float denom, float inv, bool exact_row) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
  constexpr float kMagic = 12582912.0f;
  uint32_t tb[8];
  uint32_t near = exact_row ? 1u : 0u;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = f2x_mul(__half22float2(h[e]), make_float2(inv, inv));
    const uint32_t b0 = __float_as_uint(v.x), b1 = __float_as_uint(v.y);
    near |= (((b0 & 0x1fffu) - 0x0ffdu) < 7u) | (((b1 & 0x1fffu) - 0x0ffdu) < 7u) |
            ((b0 & 0x7f800000u) == 0x7f800000u) | ((b1 & 0x7f800000u) == 0x7f800000u);
    __half2 hv = __floats2half2_rn(v.x, v.y);
    hv = __hmax2(__hmin2(hv, __float2half2_rn(127.0f)), __float2half2_rn(-128.0f));
    const float2 t = f2x_add(__half22float2(hv), make_float2(kMagic, kMagic));
    tb[2 * e] = __float_as_uint(t.x);
    tb[2 * e + 1] = __float_as_uint(t.y);
  }
  if (near) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      tb[2 * e] = static_cast<uint8_t>(quant_row_ck(f.x, denom));
      tb[2 * e + 1] = static_cast<uint8_t>(quant_row_ck(f.y, denom));
    }
  }
  return make_uint2(pack_low_bytes(tb[0], tb[1], tb[2], tb[3]), pack_low_bytes(tb[4], tb[5], tb[6], tb[7]));
}

// Row scale from the row's absmax and the quantized bytes of this lane's
// vectors, written to qrow (vector index vec(v)).
template <int WPR>
__device__ __forceinline__ void row_quant_fast_store(const uint4 (&act)[kFastV], float amax_local, bool valid,
                                                     int64_t row, int wr, int lane, int8_t* __restrict__ q,
                                                     float* __restrict__ s, int K, float* red) {
  const float amax = row_reduce_max<WPR>(amax_local, red);
  const float scale = row_scale_ck(amax);
  const float denom = round_fp16(scale);
  const float inv = __frcp_rn(denom);
  const bool exact_row = !(denom >= 6.103515625e-05f && denom <= 65504.0f);   // fp16 normal range
  if (!valid) return;
  uint2* qrow = reinterpret_cast<uint2*>(q + row * K);
#pragma unroll
  for (int v = 0; v < kFastV; ++v) qrow[(v * WPR + wr) * 32 + lane] = quant8_ck(act[v], denom, inv, exact_row);
  if (wr == 0 && lane == 0) s[row] = scale;
}

__device__ __forceinline__ float absmax_h8(const uint4& raw, float m) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
  const __half2 a = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(m, fmaxf(__low2float(a), __high2float(a)));
}

template <int WPR>
__global__ void __launch_bounds__(256) row_quant_fast_kernel(const __half* __restrict__ x, int64_t M, int K,
                                                             int64_t ldx, int8_t* __restrict__ q,
                                                             float* __restrict__ s) {
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wr = warp % WPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (8 / WPR) + warp / WPR;
  const bool valid = row < M;
  uint4 act[kFastV];
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < kFastV; ++v) {
    act[v] = valid ? __ldg(reinterpret_cast<const uint4*>(x + row * ldx) + (v * WPR + wr) * 32 + lane)
                   : make_uint4(0, 0, 0, 0);
    amax = absmax_h8(act[v], amax);
  }
  row_quant_fast_store<WPR>(act, amax, valid, row, wr, lane, q, s, K, red);
}

// residual_rms_quant_kernel for K a multiple of 1024 (same arithmetic).
template <int WPR>
__global__ void __launch_bounds__(256) residual_rms_quant_fast_kernel(
    const __half* x, const __half* __restrict__ a, const __half* __restrict__ g, const __half* __restrict__ w,
    int64_t M, int K, float eps, int round_stats, __half* h, int8_t* __restrict__ q, float* __restrict__ s,
    __half* __restrict__ norm_out) {
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wr = warp % WPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (8 / WPR) + warp / WPR;
  const bool valid = row < M;
  uint4 hv[kFastV];
  float ss = 0.0f;
#pragma unroll
  for (int v = 0; v < kFastV; ++v) {
    const int vec = (v * WPR + wr) * 32 + lane;
    uint4 xr = make_uint4(0, 0, 0, 0), ar = make_uint4(0, 0, 0, 0);
    if (valid) {
      xr = reinterpret_cast<const uint4*>(x + row * K)[vec];
      ar = __ldg(reinterpret_cast<const uint4*>(a + row * K) + vec);
    }
    const uint4 gr = __ldg(reinterpret_cast<const uint4*>(g) + vec);
    const __half2* xh = reinterpret_cast<const __half2*>(&xr);
    const __half2* ah = reinterpret_cast<const __half2*>(&ar);
    const __half2* gh = reinterpret_cast<const __half2*>(&gr);
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 raw = f2x_fma(__half22float2(ah[e]), __half22float2(gh[e]), __half22float2(xh[e]));
      const __half2 hh = __floats2half2_rn(raw.x, raw.y);
      const float2 st = round_stats ? __half22float2(hh) : raw;
      ss = __fadd_rn(ss, __fmul_rn(st.x, st.x));
      ss = __fadd_rn(ss, __fmul_rn(st.y, st.y));
      ow[e] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    hv[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
  // Each lane read its own x vectors above, so an in-place h (aliasing x) is safe.
  if (valid && h != nullptr) {
#pragma unroll
    for (int v = 0; v < kFastV; ++v) reinterpret_cast<uint4*>(h + row * K)[(v * WPR + wr) * 32 + lane] = hv[v];
  }
  ss = row_reduce_sum<WPR>(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / static_cast<float>(K)), eps));
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < kFastV; ++v) {
    const int vec = (v * WPR + wr) * 32 + lane;
    const uint4 wr4 = __ldg(reinterpret_cast<const uint4*>(w) + vec);
    const __half2* hh = reinterpret_cast<const __half2*>(&hv[v]);
    const __half2* wh = reinterpret_cast<const __half2*>(&wr4);
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = f2x_mul(f2x_mul(__half22float2(hh[e]), make_float2(inv, inv)), __half22float2(wh[e]));
      const __half2 r = __floats2half2_rn(t.x, t.y);
      ow[e] = *reinterpret_cast<const uint32_t*>(&r);
    }
    hv[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);   // now the normalized act
    amax = absmax_h8(hv[v], amax);
    if (valid && norm_out != nullptr) reinterpret_cast<uint4*>(norm_out + row * K)[vec] = hv[v];
  }
  row_quant_fast_store<WPR>(hv, amax, valid, row, wr, lane, q, s, K, red);
}

// Sum of a row's partial sums of squares in a fixed order (the residual GEMM
// epilogue wrote nparts of them), then inv = rsqrt(sum / K + eps).
__device__ __forceinline__ float row_inv_from_parts(const float* __restrict__ parts, int nparts, int K, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < nparts; ++i) ss = __fadd_rn(ss, __ldg(parts + i));
  return rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / static_cast<float>(K)), eps));
}

// act = fp16(h * inv * w) and row quantization, for h written by the residual
// GEMM epilogue together with the row's partial sums of squares (K a multiple
// of 1024: WPR warps per row as in the other fast row kernels).
template <int WPR>
__global__ void __launch_bounds__(256) rms_quant_parts_fast_kernel(const __half* __restrict__ h,
                                                                   const float* __restrict__ parts, int nparts,
                                                                   const __half* __restrict__ w, int64_t M, int K,
                                                                   float eps, int8_t* __restrict__ q,
                                                                   float* __restrict__ s,
                                                                   __half* __restrict__ norm_out) {
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wr = warp % WPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (8 / WPR) + warp / WPR;
  const bool valid = row < M;
  const float inv = valid ? row_inv_from_parts(parts + row * nparts, nparts, K, eps) : 0.0f;
  uint4 act[kFastV];
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < kFastV; ++v) {
    const int vec = (v * WPR + wr) * 32 + lane;
    const uint4 hr = valid ? __ldg(reinterpret_cast<const uint4*>(h + row * K) + vec) : make_uint4(0, 0, 0, 0);
    const uint4 wr4 = __ldg(reinterpret_cast<const uint4*>(w) + vec);
    const __half2* hh = reinterpret_cast<const __half2*>(&hr);
    const __half2* wh = reinterpret_cast<const __half2*>(&wr4);
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = f2x_mul(f2x_mul(__half22float2(hh[e]), make_float2(inv, inv)), __half22float2(wh[e]));
      const __half2 r = __floats2half2_rn(t.x, t.y);
      ow[e] = *reinterpret_cast<const uint32_t*>(&r);
    }
    act[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    amax = absmax_h8(act[v], amax);
    if (valid && norm_out != nullptr) reinterpret_cast<uint4*>(norm_out + row * K)[vec] = act[v];
  }
  row_quant_fast_store<WPR>(act, amax, valid, row, wr, lane, q, s, K, red);
}

// The same for any width: one CTA per row.
template <int MAXV>
__global__ void __launch_bounds__(kRowThreads) rms_quant_parts_kernel(const __half* __restrict__ h,
                                                                      const float* __restrict__ parts, int nparts,
                                                                      const __half* __restrict__ w, int K, float eps,
                                                                      int8_t* __restrict__ q, float* __restrict__ s,
                                                                      __half* __restrict__ norm_out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = K / 8;
  const float inv = row_inv_from_parts(parts + row * nparts, nparts, K, eps);
  float act[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * kRowThreads;
    if (v < nvec) {
      float hv[8], wv[8];
      ld8(h + row * K + v * 8, hv);
      ld8(w + v * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) act[i][j] = round_fp16(__fmul_rn(__fmul_rn(hv[j], inv), wv[j]));
      if (norm_out != nullptr) st8(norm_out + row * K + v * 8, act[i]);
    }
  }
  row_quantize_store<MAXV>(act, nvec, q + row * K, s + row, red);
}

// Standalone QK RMSNorm + rotary: one thread per (token, head).
__global__ void qk_rope_kernel(const __half* __restrict__ qkv, const __half* __restrict__ cos_t,
                               const __half* __restrict__ sin_t, int64_t rows, int heads, int R, float eps,
                               __half* __restrict__ q_out, __half* __restrict__ k_out) {
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= rows * heads) return;
  const int64_t token = idx / heads;
  for (int part = 0; part < 2; ++part) {
    float x[64];
    const __half* src = qkv + idx * 192 + part * 64;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float f[8];
      ld8(src + c * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[c * 8 + j] = f[j];
    }
    qk_norm_rope_store(x, eps, R, cos_t + token * R, sin_t + token * R, (part == 0 ? q_out : k_out) + idx * 64);
  }
}

}  // namespace h3b

namespace {

using namespace h3b;

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int row_check(int64_t M, int64_t K, const char* name, int max_k = 32768) {
  if (M <= 0 || K <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: nonempty rows required", name);
  if (K % 8 != 0 || K > max_k)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: row width %lld must be a multiple of 8 and <= %d", name,
                               (long long)K, max_k);
  if (M > 0x7fffffffLL) return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: too many rows", name);
  return H3B_OK;
}

// Widths served by the warp-per-row kernels: 1024, 2048, 4096 or 8192.
bool fast_row_width(int64_t K) { return K == 1024 || K == 2048 || K == 4096 || K == 8192; }
unsigned fast_row_grid(int64_t M, int wpr) {
  const int64_t rows_per_cta = 8 / wpr;
  return static_cast<unsigned>((M + rows_per_cta - 1) / rows_per_cta);
}

// Dispatch on the number of 8-wide vectors each thread keeps in registers.
template <template <int> class Launch, typename... Args>
int dispatch_maxv(int64_t K, Args... args) {
  const int64_t per = (K / 8 + kRowThreads - 1) / kRowThreads;
  if (per <= 1) return Launch<1>::run(args...);
  if (per <= 2) return Launch<2>::run(args...);
  if (per <= 4) return Launch<4>::run(args...);
  if (per <= 8) return Launch<8>::run(args...);
  return Launch<16>::run(args...);
}

template <int V>
struct LaunchRowQuant {
  static int run(const __half* x, int64_t M, int K, int64_t ldx, int8_t* q, float* s, cudaStream_t st) {
    row_quant_kernel<V><<<(unsigned)M, kRowThreads, 0, st>>>(x, K, ldx, q, s);
    return h3b_host::check_launch("h3b_row_quant");
  }
};

template <int V>
struct LaunchSwiGLUQuant {
  static int run(const __half* x, int64_t M, int K, int8_t* q, float* s, cudaStream_t st) {
    swiglu_quant_kernel<V><<<(unsigned)M, kRowThreads, 0, st>>>(x, K, q, s);
    return h3b_host::check_launch("h3b_swiglu_quant");
  }
};

template <int V>
struct LaunchResidualRms {
  static int run(const __half* x, const __half* a, const __half* g, const __half* w, int64_t M, int K, float eps,
                 int round_stats, __half* h, int8_t* q, float* s, __half* norm_out, cudaStream_t st) {
    residual_rms_quant_kernel<V><<<(unsigned)M, kRowThreads, 0, st>>>(x, a, g, w, K, eps, round_stats, h, q, s,
                                                                      norm_out);
    return h3b_host::check_launch("h3b_residual_rms_quant");
  }
};

template <int V>
struct LaunchRmsParts {
  static int run(const __half* h, const float* parts, int nparts, const __half* w, int64_t M, int K, float eps,
                 int8_t* q, float* s, __half* norm_out, cudaStream_t st) {
    rms_quant_parts_kernel<V><<<(unsigned)M, kRowThreads, 0, st>>>(h, parts, nparts, w, K, eps, q, s, norm_out);
    return h3b_host::check_launch("h3b_rms_quant_parts");
  }
};

template <int V>
struct LaunchRms {
  static int run(const __half* x, const __half* gamma, int64_t M, int K, float eps, __half* y, int8_t* q, float* s,
                 cudaStream_t st) {
    if (q != nullptr)
      rms_norm_kernel<V, true><<<(unsigned)M, kRowThreads, 0, st>>>(x, gamma, K, eps, y, q, s);
    else
      rms_norm_kernel<V, false><<<(unsigned)M, kRowThreads, 0, st>>>(x, gamma, K, eps, y, q, s);
    return h3b_host::check_launch("h3b_rms_norm");
  }
};

template <int V>
struct LaunchFinalLn {
  static int run(const __half* h, const __half* o, const __half* gate, const __half* gamma, const __half* beta,
                 int64_t M, int K, float eps, __half* y, cudaStream_t st) {
    final_ln_kernel<V><<<(unsigned)M, kRowThreads, 0, st>>>(h, o, gate, gamma, beta, K, eps, y);
    return h3b_host::check_launch("h3b_final_residual_layernorm");
  }
};

}  // namespace

extern "C" {

int h3b_row_quant(const void* x, int64_t M, int64_t K, int64_t ldx, int8_t* q, float* s, h3b_stream_t stream) {
  const char* name = "h3b_row_quant";
  if (!x || !q || !s) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  if (ldx < K || ldx % 8 || !al16(x)) return h3b_host::set_error(H3B_EINVAL, "%s: x must be 16-byte aligned rows", name);
  if (fast_row_width(K) && al16(q)) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const __half* xh = static_cast<const __half*>(x);
    switch (K / 1024) {
      case 1: row_quant_fast_kernel<1><<<fast_row_grid(M, 1), 256, 0, st>>>(xh, M, (int)K, ldx, q, s); break;
      case 2: row_quant_fast_kernel<2><<<fast_row_grid(M, 2), 256, 0, st>>>(xh, M, (int)K, ldx, q, s); break;
      case 4: row_quant_fast_kernel<4><<<fast_row_grid(M, 4), 256, 0, st>>>(xh, M, (int)K, ldx, q, s); break;
      default: row_quant_fast_kernel<8><<<fast_row_grid(M, 8), 256, 0, st>>>(xh, M, (int)K, ldx, q, s); break;
    }
    return h3b_host::check_launch(name);
  }
  return dispatch_maxv<LaunchRowQuant>(K, static_cast<const __half*>(x), M, (int)K, ldx, q, s,
                                       reinterpret_cast<cudaStream_t>(stream));
}

int h3b_swiglu_quant(const void* x, int64_t M, int64_t K, int8_t* q, float* s, h3b_stream_t stream) {
  const char* name = "h3b_swiglu_quant";
  if (!x || !q || !s) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name, 16384);
  if (rc) return rc;
  if (!al16(x)) return h3b_host::set_error(H3B_EINVAL, "%s: x must be 16-byte aligned", name);
  return dispatch_maxv<LaunchSwiGLUQuant>(K, static_cast<const __half*>(x), M, (int)K, q, s,
                                          reinterpret_cast<cudaStream_t>(stream));
}

int h3b_residual_rms_quant(const void* x, const void* a, const void* g, const void* w, int64_t M, int64_t K, float eps,
                           int round_stats, void* h, int8_t* q, float* s, void* norm_out, h3b_stream_t stream) {
  const char* name = "h3b_residual_rms_quant";
  if (!x || !a || !g || !w || !q || !s) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  for (const void* p : std::initializer_list<const void*>{x, a, g, w})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  if ((h && !al16(h)) || (norm_out && !al16(norm_out)))
    return h3b_host::set_error(H3B_EINVAL, "%s: outputs must be 16-byte aligned", name);
  if (fast_row_width(K) && al16(q)) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const __half *xh = static_cast<const __half*>(x), *ah = static_cast<const __half*>(a);
    const __half *gh = static_cast<const __half*>(g), *wh = static_cast<const __half*>(w);
    __half *hh = static_cast<__half*>(h), *nh = static_cast<__half*>(norm_out);
    switch (K / 1024) {
      case 1: residual_rms_quant_fast_kernel<1><<<fast_row_grid(M, 1), 256, 0, st>>>(xh, ah, gh, wh, M, (int)K, eps,
                                                                                      round_stats, hh, q, s, nh); break;
      case 2: residual_rms_quant_fast_kernel<2><<<fast_row_grid(M, 2), 256, 0, st>>>(xh, ah, gh, wh, M, (int)K, eps,
                                                                                      round_stats, hh, q, s, nh); break;
      case 4: residual_rms_quant_fast_kernel<4><<<fast_row_grid(M, 4), 256, 0, st>>>(xh, ah, gh, wh, M, (int)K, eps,
                                                                                      round_stats, hh, q, s, nh); break;
      default: residual_rms_quant_fast_kernel<8><<<fast_row_grid(M, 8), 256, 0, st>>>(xh, ah, gh, wh, M, (int)K, eps,
                                                                                       round_stats, hh, q, s, nh); break;
    }
    return h3b_host::check_launch(name);
  }
  return dispatch_maxv<LaunchResidualRms>(K, static_cast<const __half*>(x), static_cast<const __half*>(a),
                                          static_cast<const __half*>(g), static_cast<const __half*>(w), M, (int)K, eps,
                                          round_stats, static_cast<__half*>(h), q, s, static_cast<__half*>(norm_out),
                                          reinterpret_cast<cudaStream_t>(stream));
}

int h3b_rms_quant_parts(const void* h, const float* row_sumsq, int64_t parts, const void* w, int64_t M, int64_t K,
                        float eps, int8_t* q, float* s, void* norm_out, h3b_stream_t stream) {
  const char* name = "h3b_rms_quant_parts";
  if (!h || !row_sumsq || !w || !q || !s) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  if (parts <= 0 || parts > 4096) return h3b_host::set_error(H3B_EINVAL, "%s: parts must be in [1, 4096]", name);
  for (const void* p : std::initializer_list<const void*>{h, w})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  if (norm_out && !al16(norm_out)) return h3b_host::set_error(H3B_EINVAL, "%s: norm_out must be 16-byte aligned", name);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const __half* hh = static_cast<const __half*>(h);
  const __half* wh = static_cast<const __half*>(w);
  __half* nh = static_cast<__half*>(norm_out);
  if (fast_row_width(K) && al16(q)) {
    const int np = (int)parts;
    switch (K / 1024) {
      case 1: rms_quant_parts_fast_kernel<1><<<fast_row_grid(M, 1), 256, 0, st>>>(hh, row_sumsq, np, wh, M, (int)K,
                                                                                    eps, q, s, nh); break;
      case 2: rms_quant_parts_fast_kernel<2><<<fast_row_grid(M, 2), 256, 0, st>>>(hh, row_sumsq, np, wh, M, (int)K,
                                                                                    eps, q, s, nh); break;
      case 4: rms_quant_parts_fast_kernel<4><<<fast_row_grid(M, 4), 256, 0, st>>>(hh, row_sumsq, np, wh, M, (int)K,
                                                                                    eps, q, s, nh); break;
      default: rms_quant_parts_fast_kernel<8><<<fast_row_grid(M, 8), 256, 0, st>>>(hh, row_sumsq, np, wh, M, (int)K,
                                                                                     eps, q, s, nh); break;
    }
    return h3b_host::check_launch(name);
  }
  return dispatch_maxv<LaunchRmsParts>(K, hh, static_cast<const float*>(row_sumsq), (int)parts, wh, M, (int)K, eps, q,
                                       s, nh, st);
}

int h3b_rms_norm_f16(const void* x, const void* gamma, int64_t M, int64_t K, float eps, void* y, h3b_stream_t stream) {
  const char* name = "h3b_rms_norm_f16";
  if (!x || !gamma || !y) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  for (const void* p : std::initializer_list<const void*>{x, gamma, y})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  return dispatch_maxv<LaunchRms>(K, static_cast<const __half*>(x), static_cast<const __half*>(gamma), M, (int)K, eps,
                                  static_cast<__half*>(y), static_cast<int8_t*>(nullptr), static_cast<float*>(nullptr),
                                  reinterpret_cast<cudaStream_t>(stream));
}

int h3b_rms_quant(const void* x, const void* gamma, int64_t M, int64_t K, float eps, int8_t* q, float* s,
                  h3b_stream_t stream) {
  const char* name = "h3b_rms_quant";
  if (!x || !gamma || !q || !s) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  for (const void* p : std::initializer_list<const void*>{x, gamma})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  return dispatch_maxv<LaunchRms>(K, static_cast<const __half*>(x), static_cast<const __half*>(gamma), M, (int)K, eps,
                                  static_cast<__half*>(nullptr), q, s, reinterpret_cast<cudaStream_t>(stream));
}

int h3b_final_residual_layernorm(const void* h, const void* o, const void* gate, const void* gamma, const void* beta,
                                 int64_t M, int64_t K, float eps, void* y, h3b_stream_t stream) {
  const char* name = "h3b_final_residual_layernorm";
  if (!h || !o || !gate || !gamma || !beta || !y) return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  int rc = row_check(M, K, name);
  if (rc) return rc;
  for (const void* p : std::initializer_list<const void*>{h, o, gate, gamma, beta, y})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  return dispatch_maxv<LaunchFinalLn>(K, static_cast<const __half*>(h), static_cast<const __half*>(o),
                                      static_cast<const __half*>(gate), static_cast<const __half*>(gamma),
                                      static_cast<const __half*>(beta), M, (int)K, eps, static_cast<__half*>(y),
                                      reinterpret_cast<cudaStream_t>(stream));
}

int h3b_qk_rope(const void* qkv, const void* cos_t, const void* sin_t, int64_t batch, int64_t tokens, int64_t heads,
                int64_t rot_dims, float eps, void* q_out, void* k_out, h3b_stream_t stream) {
  const char* name = "h3b_qk_rope";
  if (!qkv || !q_out || !k_out || (rot_dims > 0 && (!cos_t || !sin_t)))
    return h3b_host::set_error(H3B_EINVAL, "%s: NULL argument", name);
  if (batch <= 0 || tokens <= 0 || heads <= 0) return h3b_host::set_error(H3B_EINVAL, "%s: empty input", name);
  if (rot_dims != 0 && rot_dims != 16 && rot_dims != 32 && rot_dims != 48 && rot_dims != 64)
    return h3b_host::set_error(H3B_EUNSUPPORTED, "%s: rotary dims must be one of 0, 16, 32, 48, 64", name);
  if (rot_dims > 0 && ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t)) & 15u))
    return h3b_host::set_error(H3B_EINVAL, "%s: cos/sin tables must be 16-byte aligned", name);
  for (const void* p : std::initializer_list<const void*>{qkv, q_out, k_out})
    if (!al16(p)) return h3b_host::set_error(H3B_EINVAL, "%s: tensors must be 16-byte aligned", name);
  const int64_t rows = batch * tokens;
  const int64_t total = rows * heads;
  const int threads = 128;
  qk_rope_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(qkv), static_cast<const __half*>(cos_t), static_cast<const __half*>(sin_t), rows,
      (int)heads, (int)rot_dims, eps, static_cast<__half*>(q_out), static_cast<__half*>(k_out));
  return h3b_host::check_launch(name);
}

}  // extern "C"
