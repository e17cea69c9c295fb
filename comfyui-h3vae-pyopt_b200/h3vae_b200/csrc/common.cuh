// Shared device/host helpers for the sm_100a kernels of the H3 VAE INT8 path.
//
// Everything here is hand-written inline PTX for the Blackwell data-centre
// tensor-core path: mbarriers, per-CTA TMA tiled loads (cp.async.bulk.tensor),
// and the tcgen05 family (TMEM alloc, MMA, commit, ld).
// Every spin-wait is bounded: after kSpinLimit polls it records an error code
// in the caller-visible device error word and reports failure so the kernel
// can unwind instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <initializer_list>

#include "../../../include/h3vae_b200.h"

namespace h3b {

// ---------------------------------------------------------------------------
// Device error word.  Kernels OR a code into it when a bounded wait expires or
// an internal invariant fails; the host reads it with h3b_device_error().
// ---------------------------------------------------------------------------
// Defined here: the library is built as one translation unit.
__device__ unsigned int g_device_error = 0;

enum DeviceErrorBits : unsigned int {
  kErrBarrierTimeout = 1u << 0,
  kErrTmemAlloc = 1u << 1,
  kErrBadGeometry = 1u << 2,
};

// About 2^25 polls of try_wait (each suspends for a few hundred ns at most):
// well above any legitimate wait, well below a watchdog.
constexpr uint32_t kSpinLimit = 1u << 25;

__device__ __forceinline__ void record_error(unsigned int bits) {
  atomicOr(&g_device_error, bits);
}

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// The same waits on a 32-bit shared-memory address (keeps register pressure
// down in kernels that hold many values per thread).
__device__ __forceinline__ bool mbar_try_wait_u32(uint32_t bar, uint32_t parity) {
  uint32_t done = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_u32(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_u32(bar, parity)) return true;
    if ((i & 1023u) == 1023u && abort_flag != nullptr && *abort_flag) return false;
  }
  record_error(kErrBarrierTimeout);
  if (abort_flag != nullptr) *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void mbar_arrive_u32(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded polling wait for the single-thread roles (TMA producer, MMA issuer):
// test_wait never suspends, so the thread sees the phase flip at once instead
// of after try_wait's suspend interval.  Same bound and error reporting as
// mbar_wait.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < 4 * kSpinLimit; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 4095u) == 4095u && abort_flag != nullptr && *abort_flag) return false;
  }
  record_error(kErrBarrierTimeout);
  if (abort_flag != nullptr) *abort_flag = 1;
  return false;
}

// Bounded wait on a phase parity with an explicit poll limit.  Returns false
// (and records the error) if the phase does not complete within `limit` polls
// or if another role already aborted the CTA.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && abort_flag != nullptr && *abort_flag) return false;
  }
  record_error(kErrBarrierTimeout);
  if (abort_flag != nullptr) *abort_flag = 1;
  return false;
}

// The kernels' wait: the same loop with the library-wide bound.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_limit(bar, parity, abort_flag, kSpinLimit);
}

// ---------------------------------------------------------------------------
// TMA (tiled loads into this CTA's shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA issue, commit, loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B^T, fp16 x fp16 -> fp32.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: each thread gets its lane's 32 words.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte swizzle canonical layout: rows of 128 bytes, 8-row atoms of 1024 B
// (stride-byte-offset 1024), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;              // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;      // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;              // descriptor version (Blackwell)
  d |= static_cast<uint64_t>(2u) << 61;              // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: M=128, N=n, signed int8 A/B (K-major), int32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format: S32
         | (1u << 7)          // A format: signed 8-bit
         | (1u << 10)         // B format: signed 8-bit
         | ((n >> 3) << 17)   // N >> 3
         | ((m >> 4) << 24);  // M >> 4
}

// Instruction descriptor: fp16 A/B (K-major), fp32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t m, uint32_t n) {
  return (1u << 4)            // D format: F32
         | (0u << 7)          // A format: F16
         | (0u << 10)         // B format: F16
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers shared by the epilogues and producers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float round_fp16(float v) { return __half2float(__float2half_rn(v)); }

// Half-away-from-zero rounding in the exact fp32 order the encoder quantizer
// uses: floor(s + 0.5) for s >= 0, -floor(-s + 0.5) otherwise, clamp +-127.
__device__ __forceinline__ int8_t quant_half_away(float x, float scale) {
  float s = __fdiv_rn(x, scale);
  float r = (s >= 0.0f) ? floorf(__fadd_rn(s, 0.5f)) : -floorf(__fadd_rn(-s, 0.5f));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// quant_half_away with the quotient formed by the precomputed reciprocal.  The
// reciprocal product differs from the correctly rounded quotient by < 2^-22
// relative (|q| <= 127.5 here), so only quotients within 2^-13 of a rounding
// boundary k + 0.5 are recomputed with the exact division: the result is
// identical to quant_half_away for every input (NaN and inf included).
__device__ __forceinline__ int8_t quant_half_away_fast(float x, float scale, float inv_scale) {
  // s = x / scale through the reciprocal; only within 2^-13 of a .5 tie can
  // that differ in rounding from the true quotient, so those recompute with
  // the IEEE division.  Rounding uses the 1.5 * 2^23 magic constant (fp32 adds
  // on the full-rate pipe) instead of floor / float->int conversions:
  // a + M rounds a = |s| <= 255 to the nearest integer (ties to even), whose
  // value sits in the low mantissa bits of a + M; exact ties then step away
  // from zero.
  constexpr float kMagic = 12582912.0f;
  float s = __fmul_rn(x, inv_scale);
  float a = fminf(fabsf(s), 255.0f);
  float t = __fadd_rn(a, kMagic);
  float d = __fsub_rn(a, __fsub_rn(t, kMagic));   // a - rne(a), in [-0.5, 0.5]
  if (fabsf(d) > 0.5f - 1.0f / 8192.0f) {
    s = __fdiv_rn(x, scale);
    a = fminf(fabsf(s), 255.0f);
    t = __fadd_rn(a, kMagic);
    d = __fsub_rn(a, __fsub_rn(t, kMagic));
  }
  int k = __float_as_int(t) - __float_as_int(kMagic);
  k += (d == 0.5f) ? 1 : 0;
  k = min(k, 127);
  return static_cast<int8_t>(s < 0.0f ? -k : k);
}

// Packed fp32 pair arithmetic (Blackwell f32x2): one instruction per pair, each
// lane rounded exactly like the scalar op.
__device__ __forceinline__ float2 f2x_fma(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("{\n\t.reg .b64 x, y, z;\n\t"
      "mov.b64 x, {%1, %2};\n\tmov.b64 y, {%3, %4};\n\tmov.b64 z, {%5, %6};\n\t"
      "fma.rn.f32x2 %0, x, y, z;\n\t}"
      : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(d)), __uint_as_float(static_cast<uint32_t>(d >> 32)));
}
__device__ __forceinline__ float2 f2x_mul(float2 a, float2 b) {
  uint64_t d;
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%1, %2};\n\tmov.b64 y, {%3, %4};\n\t"
      "mul.rn.f32x2 %0, x, y;\n\t}"
      : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(d)), __uint_as_float(static_cast<uint32_t>(d >> 32)));
}
__device__ __forceinline__ float2 f2x_add(float2 a, float2 b) {
  uint64_t d;
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%1, %2};\n\tmov.b64 y, {%3, %4};\n\t"
      "add.rn.f32x2 %0, x, y;\n\t}"
      : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(d)), __uint_as_float(static_cast<uint32_t>(d >> 32)));
}
__device__ __forceinline__ float2 f2x_sub(float2 a, float2 b) {
  uint64_t d;
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%1, %2};\n\tmov.b64 y, {%3, %4};\n\t"
      "sub.rn.f32x2 %0, x, y;\n\t}"
      : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(d)), __uint_as_float(static_cast<uint32_t>(d >> 32)));
}

// Per-tensor half-away quantization for the producers' hot loop.  Returns a
// float whose low byte is the int8 result: s + 1.5 * 2^23 rounds s to the
// nearest integer (ties to even) and keeps it in the low mantissa bits, so
// the byte needs no float->int conversion, clamp or sign handling; bytes are
// packed with byte permutes.  Only within 2^-13 of a .5 boundary can the
// reciprocal-based quotient or the tie rule differ from the reference's
// half-away rounding of the true quotient, and there the exact path runs.
// |z| <= amax (the scale's own absmax) keeps |s| <= 127 up to rounding, so
// no clamp is needed on the fast path.
__device__ __noinline__ float quant_exact_bits(float z, float scale) {
  constexpr float kMagic = 12582912.0f;
  const float s = __fdiv_rn(z, scale);
  float r = (s >= 0.0f) ? floorf(__fadd_rn(s, 0.5f)) : -floorf(__fadd_rn(-s, 0.5f));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return __fadd_rn(r, kMagic);
}

__device__ __forceinline__ uint32_t quant_byte_bits(float z, float scale, float inv_scale) {
  constexpr float kMagic = 12582912.0f;
  const float s = __fmul_rn(z, inv_scale);
  float t = __fadd_rn(s, kMagic);
  const float d = __fsub_rn(s, __fsub_rn(t, kMagic));   // s - rne(s), in [-0.5, 0.5]
  if (fabsf(d) > 0.5f - 1.0f / 8192.0f) t = quant_exact_bits(z, scale);
  return __float_as_uint(t);
}

// quant_byte_bits for two values with packed fp32 pair arithmetic.
__device__ __forceinline__ void quant_byte_bits2(float z0, float z1, float scale, float inv_scale, uint32_t& t0,
                                                 uint32_t& t1) {
  constexpr float kMagic = 12582912.0f;
  const float2 m2 = make_float2(kMagic, kMagic);
  const float2 sv = f2x_mul(make_float2(z0, z1), make_float2(inv_scale, inv_scale));
  const float2 tv = f2x_add(sv, m2);
  const float2 dv = f2x_sub(sv, f2x_sub(tv, m2));   // s - rne(s)
  constexpr float kNearTie = 0.5f - 1.0f / 8192.0f;
  t0 = fabsf(dv.x) > kNearTie ? __float_as_uint(quant_exact_bits(z0, scale)) : __float_as_uint(tv.x);
  t1 = fabsf(dv.y) > kNearTie ? __float_as_uint(quant_exact_bits(z1, scale)) : __float_as_uint(tv.y);
}

// quant_byte_bits for eight values: one near-tie test for all of them (the
// largest |s - rne(s)|), the exact path for all eight in the rare case.
__device__ __forceinline__ void quant_bytes8(const float (&z)[8], float scale, float inv_scale, uint32_t (&t)[8]) {
  constexpr float kMagic = 12582912.0f;
  const float2 m2 = make_float2(kMagic, kMagic);
  float dmax = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const float2 sv = f2x_mul(make_float2(z[j], z[j + 1]), make_float2(inv_scale, inv_scale));
    const float2 tv = f2x_add(sv, m2);
    const float2 dv = f2x_sub(sv, f2x_sub(tv, m2));   // s - rne(s)
    t[j] = __float_as_uint(tv.x);
    t[j + 1] = __float_as_uint(tv.y);
    dmax = fmaxf(dmax, fmaxf(fabsf(dv.x), fabsf(dv.y)));
  }
  if (dmax > 0.5f - 1.0f / 8192.0f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = quant_byte_bits(z[j], scale, inv_scale);
  }
}

// Low bytes of four words into one word (byte 0 from a).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Order-preserving map of fp32 to uint32 (for atomicMin/atomicMax of signed
// floats): non-negative values set the top bit, negative values are inverted.
__device__ __forceinline__ unsigned int float_to_ordered(float f) {
  const unsigned int u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(unsigned int u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// Row quantization rule of the decoder's INT8 linears: divide in fp32 by the
// fp16-rounded scale, round the quotient to fp16, then to nearest-even,
// NaN -> -128, clamp to [-128, 127].
__device__ __forceinline__ int8_t quant_row_ck(float act, float denom) {
  float v = round_fp16(__fdiv_rn(act, denom));
  v = rintf(v);
  if (v != v) v = -128.0f;
  v = fminf(127.0f, fmaxf(-128.0f, v));
  return static_cast<int8_t>(static_cast<int>(v));
}

__device__ __forceinline__ float row_scale_ck(float amax) {
  return fmaxf(__fmul_rn(amax, 1.0f / 127.0f), 1.0e-30f);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Non-negative floats order like their bit patterns, so an unsigned atomicMax
// on the bits is an exact float max for values >= 0 (NaN excluded).
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// QK RMSNorm (fp32 statistics, no affine) + fp16 round + rotate-half rotary
// embedding on the first R dims of one 64-wide head vector held in registers.
// Products are rounded to fp16 individually before the fp32 sum, and the sum
// is rounded to fp16 on store.  R is a compile-time constant so the vector
// stays in registers; the token's cos / sin values arrive as R / 8 16-byte
// vectors each (loaded early by the caller), dst must be 16-byte aligned.
template <int R>
__device__ __forceinline__ void qk_norm_rope_regs_t(__half2 (&xh)[32], float eps, const uint4 (&rc)[8],
                                                    const uint4 (&rs)[8], uint4 (&out)[8]) {
  static_assert(R % 4 == 0, "rotary width: pairs of halves on both sides of R/2");
  // xh holds the 64 fp16-rounded linear outputs.  The normalized values are
  // fp16 again, and the rotary products fp16(x * cos), fp16(rot * sin) are
  // exactly fp16 multiplies (an 11 x 11-bit product is exact before its one
  // rounding), so the rotation runs on packed halves; the sum of the two
  // products is one fp16 add.
  // sum of squares in four independent chains (short dependency chains)
  float ssa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    const float2 f = __half22float2(xh[d]);
    ssa[d & 3] = __fmaf_rn(f.x, f.x, ssa[d & 3]);
    ssa[d & 3] = __fmaf_rn(f.y, f.y, ssa[d & 3]);
  }
  const float ss = (ssa[0] + ssa[1]) + (ssa[2] + ssa[3]);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / 64.0f), eps));
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    const float2 f = __half22float2(xh[d]);
    xh[d] = __floats2half2_rn(__fmul_rn(f.x, inv), __fmul_rn(f.y, inv));
  }
  // pair i of a row of 8 x uint4 tables, by register selects only (no
  // address is taken, so the tables stay in registers)
  auto tab = [&](const uint4 (&t)[8], int i) {
    const uint4 v = t[i >> 2];
    const int w = i & 3;
    const uint32_t u = w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
    return *reinterpret_cast<const __half2*>(&u);
  };
  auto bits = [](__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); };
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t ow[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = q * 4 + e;        // pair (2i, 2i+1)
      __half2 o = xh[i];
      if (2 * i < R) {
        const __half2 rot = (2 * i < R / 2) ? __hneg2(xh[i + R / 4]) : xh[i - R / 4];
        o = __hadd2(__hmul2(xh[i], tab(rc, i)), __hmul2(rot, tab(rs, i)));
      }
      ow[e] = bits(o);
    }
    out[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// The R cos / sin values of one token as 16-byte vectors (R / 8 of each).
__device__ __forceinline__ void load_rope_row(const __half* cs, const __half* sn, int R, uint4 (&rc)[8],
                                              uint4 (&rs)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    if (q < R / 8) {
      rc[q] = __ldg(reinterpret_cast<const uint4*>(cs) + q);
      rs[q] = __ldg(reinterpret_cast<const uint4*>(sn) + q);
    } else {
      rc[q] = make_uint4(0, 0, 0, 0);
      rs[q] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Runtime-R dispatch with the token's tables already in registers; the
// normalized, rotated 64-wide row comes back as eight 16-byte vectors.
__device__ __forceinline__ void qk_norm_rope_regs(__half2 (&x)[32], float eps, int R, const uint4 (&rc)[8],
                                                  const uint4 (&rs)[8], uint4 (&out)[8]) {
  switch (R) {
    case 48: qk_norm_rope_regs_t<48>(x, eps, rc, rs, out); break;
    case 64: qk_norm_rope_regs_t<64>(x, eps, rc, rs, out); break;
    case 32: qk_norm_rope_regs_t<32>(x, eps, rc, rs, out); break;
    case 16: qk_norm_rope_regs_t<16>(x, eps, rc, rs, out); break;
    default: qk_norm_rope_regs_t<0>(x, eps, rc, rs, out); break;
  }
}

// Runtime-R dispatch over the supported rotary widths {0, 16, 32, 48, 64},
// loading the token's cos / sin rows first.
__device__ __forceinline__ void qk_norm_rope_store(const float (&x)[64], float eps, int R, const __half* cs,
                                                   const __half* sn, __half* dst) {
  uint4 rc[8], rs[8];
  load_rope_row(cs, sn, R, rc, rs);
  __half2 xh[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) xh[d] = __floats2half2_rn(x[2 * d], x[2 * d + 1]);
  uint4 o[8];
  qk_norm_rope_regs(xh, eps, R, rc, rs, o);
#pragma unroll
  for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(dst)[q] = o[q];
}

}  // namespace h3b

// ---------------------------------------------------------------------------
// Host-side helpers (error string, tensor-map encoding through the driver
// entry point so the library does not link libcuda directly).
// ---------------------------------------------------------------------------
namespace h3b_host {

int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* gaddr,
                 const uint64_t* dims, const uint64_t* strides_bytes /* rank-1 entries */,
                 const uint32_t* box, const uint32_t* elem_strides, CUtensorMapSwizzle swizzle);
int num_sms();

}  // namespace h3b_host
