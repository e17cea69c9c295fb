// Non-causal fp16 attention, head dim 64, fp32 online softmax.
//
// One CTA = 4 warps = 64 query rows of one (batch, head); the K/V sequence is
// streamed in 64-key tiles through a cp.async double buffer in XOR-swizzled
// shared memory (16-byte chunk index ^ row % 8, conflict-free ldmatrix).
// S = Q K^T and O += P V use mma.sync m16n8k16 (fp16 in, fp32 accumulate);
// P never leaves registers (the S accumulator layout is reused as the A
// fragment of the PV product).
#include "common.cuh"

namespace h3b {

constexpr int kAttBQ = 64;
constexpr int kAttBK = 64;
constexpr int kAttD = 64;
constexpr int kAttThreads = 128;

struct AttnParams {
  const __half* q;
  const __half* k;
  const __half* v;
  __half* out;
  int64_t qs[3], ks[3], vs[3], os[3];  // {batch, head, token} element strides
  int q_len, kv_len;
  float scale_log2;                    // softmax scale * log2(e)
};

__device__ __forceinline__ uint32_t swz(int row, int col) {
  // element offset of (row, col) in a 64x64 fp16 tile, 16-byte chunks swizzled
  return row * 64 + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load a 64 x 64 tile (rows = tokens) into swizzled shared memory.
__device__ __forceinline__ void load_tile(__half* smem, const __half* src, int64_t row_stride, int row0, int nrows) {
  const uint32_t base = smem_u32(smem);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int chunk = threadIdx.x + i * kAttThreads;  // 512 chunks of 16 B
    const int r = chunk >> 3;
    const int c = (chunk & 7) << 3;
    const bool valid = (row0 + r) < nrows;
    const __half* g = src + static_cast<int64_t>(valid ? row0 + r : 0) * row_stride + c;
    cp_async16(base + swz(r, c) * 2, g, valid);
  }
}

__global__ void __launch_bounds__(kAttThreads) attention_f16_kernel(const AttnParams p) {
  __shared__ __align__(128) __half sq[kAttBQ * kAttD];
  __shared__ __align__(128) __half sk[2][kAttBK * kAttD];
  __shared__ __align__(128) __half sv[2][kAttBK * kAttD];

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * kAttBQ;
  const __half* qg = p.q + b * p.qs[0] + h * p.qs[1];
  const __half* kg = p.k + b * p.ks[0] + h * p.ks[1];
  const __half* vg = p.v + b * p.vs[0] + h * p.vs[1];

  load_tile(sq, qg, p.qs[2], q0, p.q_len);
  load_tile(sk[0], kg, p.ks[2], 0, p.kv_len);
  load_tile(sv[0], vg, p.vs[2], 0, p.kv_len);
  cp_async_commit();

  const int n_tiles = (p.kv_len + kAttBK - 1) / kAttBK;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  uint32_t qf[4][4];

  for (int t = 0; t < n_tiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < n_tiles) {
      load_tile(sk[buf ^ 1], kg, p.ks[2], (t + 1) * kAttBK, p.kv_len);
      load_tile(sv[buf ^ 1], vg, p.vs[2], (t + 1) * kAttBK, p.kv_len);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32(sq) + swz(r, c) * 2, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T for 16 rows x 64 keys per warp.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
    const uint32_t kbase = smem_u32(sk[buf]);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int dim = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + swz(key, dim) * 2, b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kk], b0, b1);
        mma16816(s[2 * np + 1], qf[kk], b2, b3);
      }
    }
    // Mask keys beyond kv_len, online softmax in the log2 domain.
    const int key0 = t * kAttBK;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = key0 + n * 8 + (lane & 3) * 2 + (j & 1);
        float v = s[n][j] * p.scale_log2;
        if (key >= p.kv_len) v = -INFINITY;
        s[n][j] = v;
        mx[j >> 1] = fmaxf(mx[j >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      alpha[r] = (m_run[r] == -INFINITY) ? 0.0f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
      l_run[r] *= alpha[r];
    }
    uint32_t pf[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      float pv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float m = m_run[j >> 1];
        pv[j] = (m == -INFINITY) ? 0.0f : exp2f(s[n][j] - m);
        l_run[j >> 1] += pv[j];
      }
      pf[n >> 1][(n & 1) * 2 + 0] = pack_h2(pv[0], pv[1]);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_h2(pv[2], pv[3]);
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V
    const uint32_t vbase = smem_u32(sv[buf]);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      // A fragment for keys 16kk..16kk+15: n-tiles 2kk (a0,a1) and 2kk+1 (a2,a3).
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int dim = dp * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + swz(key, dim) * 2, b0, b1, b2, b3);
        mma16816(o[2 * dp], a, b0, b1);
        mma16816(o[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  // Finalize: reduce the row sums over the 4 threads of a quad, normalize, store.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
  const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
  const int row0 = q0 + warp * 16 + (lane >> 2);
  __half* og = p.out + b * p.os[0] + h * p.os[1];
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int d = n * 8 + (lane & 3) * 2;
    if (row0 < p.q_len)
      *reinterpret_cast<__half2*>(og + static_cast<int64_t>(row0) * p.os[2] + d) =
          __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
    if (row0 + 8 < p.q_len)
      *reinterpret_cast<__half2*>(og + static_cast<int64_t>(row0 + 8) * p.os[2] + d) =
          __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
}

}  // namespace h3b

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
  AttnParams p{};
  p.q = static_cast<const __half*>(q);
  p.k = static_cast<const __half*>(k);
  p.v = static_cast<const __half*>(v);
  p.out = static_cast<__half*>(out);
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = q_strides[i];
    p.ks[i] = k_strides[i];
    p.vs[i] = v_strides[i];
    p.os[i] = out_strides[i];
  }
  for (const void* ptr : std::initializer_list<const void*>{q, k, v})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return h3b_host::set_error(H3B_EINVAL, "%s: q/k/v must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if (p.qs[i] % 8 || p.ks[i] % 8 || p.vs[i] % 8)
      return h3b_host::set_error(H3B_EINVAL, "%s: q/k/v strides must be multiples of 8 elements", name);
  if ((reinterpret_cast<uintptr_t>(out) & 3u) || p.os[0] % 2 || p.os[1] % 2 || p.os[2] % 2)
    return h3b_host::set_error(H3B_EINVAL, "%s: output must allow 4-byte stores", name);
  p.q_len = (int)q_len;
  p.kv_len = (int)kv_len;
  p.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((unsigned)((q_len + kAttBQ - 1) / kAttBQ), (unsigned)heads, (unsigned)batch);
  attention_f16_kernel<<<grid, kAttThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return h3b_host::check_launch(name);
}
