// Non-causal fp16 attention (head dim 64) on the tcgen05 tensor cores.
//
// One CTA = one (batch, head, 128-query tile); 6 warps:
//   warp 0      TMA: Q once, then K and V tiles of 128 keys through a 3-stage ring
//   warp 1      TMEM owner + MMA issuer:  S_j = Q K_j^T  (M128 N128 K64, fp32 in
//               TMEM, double buffered), then O_j = P_j V_j (M128 N64 K128, P from
//               shared memory, V as the MN-major B operand straight from its TMA tile)
//   warps 2..5  softmax, one query row per thread (TMEM lane): running max, P_j =
//               exp2(S_j * scale*log2e - m_j) rounded to fp16 into 128-byte-swizzled
//               shared memory, running sum, and the O accumulator in registers:
//               o = o * exp2(m_{j-1} - m_j) + O_j.
// While the softmax warps work on S_j the tensor cores compute S_{j+1} and
// O_{j-1}.  Every wait is bounded (see common.cuh).
#include "common.cuh"

namespace h3b {

constexpr int kFaM = 128;       // queries per CTA
constexpr int kFaN = 128;       // keys per tile
constexpr int kFaD = 64;        // head dim
constexpr int kFaStages = 3;
constexpr int kFaThreads = 192;
constexpr uint32_t kFaQBytes = kFaM * kFaD * 2;   // 16 KB
constexpr uint32_t kFaKVBytes = kFaN * kFaD * 2;  // 16 KB each for K and V
constexpr uint32_t kFaPBytes = kFaM * kFaN * 2;   // 32 KB (two 16 KB swizzle columns of 64 keys)
constexpr uint32_t kFaTmemCols = 512;             // S0 | S1 | O0 | O1
constexpr uint32_t kFaS0 = 0, kFaO0 = 256;

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
  uint8_t* sq = smem;
  uint8_t* sk = sq + kFaQBytes;
  uint8_t* sv = sk + kFaStages * kFaKVBytes;
  uint8_t* sp = sv + kFaStages * kFaKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * kFaPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kFaStages;
  uint64_t* s_full = kv_empty + kFaStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_empty = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n_tiles = (p.kv_len + kFaN - 1) / kFaN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kFaStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(q_full, kFaQBytes);
      tma_load_4d(sq, &mq, q_full, 0, qt * kFaM, h, b);
      uint32_t issued = 0;
      for (int j = 0; j < n_tiles; ++j, ++issued) {
        const int s = j % kFaStages;
        if (!mbar_wait(&kv_empty[s], ((j / kFaStages) & 1) ^ 1, abort_flag)) break;
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
    if (elect_one_sync()) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kFaM, kFaN);
      constexpr uint32_t idesc_pv = make_idesc_f16(kFaM, kFaD) | (1u << 16);  // B (V) is MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag);
      const uint64_t qdesc = make_sw128_desc(smem_u32(sq));
      auto issue_s = [&](int j) -> bool {
        const int s = j % kFaStages, sb = j & 1;
        if (!mbar_wait(&kv_full[s], (j / kFaStages) & 1, abort_flag)) return false;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t kdesc = make_sw128_desc(smem_u32(sk + s * kFaKVBytes));
#pragma unroll
        for (int k = 0; k < kFaD / 16; ++k)  // 16 fp16 = 32 bytes per MMA step
          mma_f16(tmem + kFaS0 + sb * kFaN, qdesc + 2 * k, kdesc + 2 * k, idesc_qk, k > 0 ? 1u : 0u);
        tc_commit(&s_full[sb]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        const int s = j % kFaStages, ob = j & 1;
        if (!mbar_wait(&p_full[ob], (j >> 1) & 1, abort_flag)) break;
        if (!mbar_wait(&o_empty[ob], ((j >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t pbase = smem_u32(sp + ob * kFaPBytes);
        const uint32_t vbase = smem_u32(sv + s * kFaKVBytes);
#pragma unroll
        for (int t = 0; t < kFaN / 16; ++t) {
          const uint64_t pdesc = make_sw128_desc(pbase + (t >> 2) * (kFaPBytes / 2)) + 2 * (t & 3);
          const uint64_t vdesc = make_sw128_desc(vbase + t * 16 * 128);
          mma_f16(tmem + kFaO0 + ob * kFaD, pdesc, vdesc, idesc_pv, t > 0 ? 1u : 0u);
        }
        tc_commit(&o_full[ob]);
        tc_commit(&kv_empty[s]);
      }
    }
  } else {
    // ------------------------------ softmax warps ------------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
    float o[kFaD];
#pragma unroll
    for (int d = 0; d < kFaD; ++d) o[d] = 0.0f;
    bool ok = true;
    auto take_o = [&](int jj) -> bool {
      const int ob = jj & 1;
      if (!mbar_wait(&o_full[ob], (jj >> 1) & 1, abort_flag)) return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(tmem + lane_off + kFaO0 + ob * kFaD, r0);
      tmem_ld32(tmem + lane_off + kFaO0 + ob * kFaD + 32, r1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&o_empty[ob]);
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o[d] = __fmaf_rn(o[d], alpha_prev, __uint_as_float(r0[d]));
        o[32 + d] = __fmaf_rn(o[32 + d], alpha_prev, __uint_as_float(r1[d]));
      }
      return true;
    };
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float sv_[kFaN];
#pragma unroll
      for (int c = 0; c < kFaN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + kFaS0 + sb * kFaN + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv_[c * 32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const int valid = p.kv_len - j * kFaN;
      float tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < kFaN; ++i) {
        if (i >= valid) sv_[i] = -INFINITY;
        tmax = fmaxf(tmax, sv_[i]);
      }
      const float m_new = fmaxf(m, tmax * p.scale_log2);
      const float alpha = exp2f(m - m_new);
      float rowsum = 0.0f;
      uint8_t* prow = sp + sb * kFaPBytes + row * 128;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          __align__(16) __half2 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = blk * 64 + c * 8 + 2 * e;
            const float p0 = exp2f(__fmaf_rn(sv_[k], p.scale_log2, -m_new));
            const float p1 = exp2f(__fmaf_rn(sv_[k + 1], p.scale_log2, -m_new));
            rowsum += p0 + p1;
            hv[e] = __floats2half2_rn(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + blk * (kFaPBytes / 2) + ((c ^ (row & 7)) << 4)) =
              *reinterpret_cast<const uint4*>(hv);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[sb]);
      l = __fmaf_rn(l, alpha, rowsum);
      if (j > 0 && !take_o(j - 1)) { ok = false; break; }
      alpha_prev = alpha;
      m = m_new;
    }
    if (ok && n_tiles > 0) ok = take_o(n_tiles - 1);
    const int qrow = qt * kFaM + row;
    if (ok && qrow < p.q_len) {
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      __half* dst = p.out + b * p.os[0] + h * p.os[1] + static_cast<int64_t>(qrow) * p.os[2];
#pragma unroll
      for (int q = 0; q < kFaD / 8; ++q) {
        __align__(16) __half2 hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) hv[e] = __floats2half2_rn(o[q * 8 + 2 * e] * inv, o[q * 8 + 2 * e + 1] * inv);
        *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<const uint4*>(hv);
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
  constexpr size_t smem = kFaQBytes + 2 * kFaStages * kFaKVBytes + 2 * kFaPBytes + 1024 + 256;
  static_assert(smem <= 232448, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  dim3 grid((unsigned)((q_len + kFaM - 1) / kFaM), (unsigned)heads, (unsigned)batch);
  attention_tc_kernel<<<grid, kFaThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mq, mk, mv, p);
  return h3b_host::check_launch(name);
}
