// Host plumbing of the C ABI: thread-local error strings, launch checks,
// tensor-map encoding through the driver entry point, the device error word.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace h3b_host {

static thread_local char g_last_error[1024] = {0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(H3B_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return H3B_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* gaddr,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 const uint32_t* elem_strides, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if ((reinterpret_cast<uintptr_t>(gaddr) & 15u) != 0)
    return set_error(H3B_EINVAL, "TMA base address must be 16-byte aligned");
  for (uint32_t i = 0; i + 1 < rank; ++i) {
    if (strides_bytes[i] % 16 != 0)
      return set_error(H3B_EINVAL, "TMA global stride %u (%llu bytes) is not a multiple of 16", i,
                       (unsigned long long)strides_bytes[i]);
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(gaddr), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box),
                  reinterpret_cast<const cuuint32_t*>(elem_strides), CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(H3B_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return H3B_OK;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

}  // namespace h3b_host

namespace h3b {

// One warp waits on an mbarrier that nothing arrives at, through the same
// bounded wait the kernels use, with a caller-chosen poll limit.  The wait
// runs out, records kErrBarrierTimeout in the device error word and returns.
__global__ void __launch_bounds__(32) wait_timeout_probe_kernel(uint32_t poll_limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncwarp();
  mbar_wait_limit(&bar, 0, &abort_flag, poll_limit);
  __syncwarp();
}

}  // namespace h3b

extern "C" {

int h3b_probe_wait_timeout(uint32_t poll_limit, h3b_stream_t stream) {
  const char* name = "h3b_probe_wait_timeout";
  if (poll_limit == 0 || poll_limit > (1u << 20))
    return h3b_host::set_error(H3B_EINVAL, "%s: poll_limit must be in [1, 2^20], got %u", name, poll_limit);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  h3b::wait_timeout_probe_kernel<<<1, 32, 0, st>>>(poll_limit);
  int rc = h3b_host::check_launch(name);
  if (rc != H3B_OK) return rc;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: %s", name, cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, h3b::g_device_error, sizeof(v));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "%s: read of device error word failed: %s", name,
                                                   cudaGetErrorString(e));
  if (v & h3b::kErrBarrierTimeout)
    return h3b_host::set_error(H3B_EDEVICE, "%s: bounded wait expired after %u polls (device error bits 0x%x)",
                               name, poll_limit, v);
  return H3B_OK;
}

const char* h3b_last_error(void) { return h3b_host::g_last_error; }

int h3b_abi_version(void) { return 100; }

int h3b_device_error(unsigned int* bits, int clear) {
  if (bits == nullptr) return h3b_host::set_error(H3B_EINVAL, "bits is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "device sync failed: %s", cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, h3b::g_device_error, sizeof(v));
  if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "read of device error word failed: %s", cudaGetErrorString(e));
  *bits = v;
  if (clear) {
    unsigned int z = 0;
    e = cudaMemcpyToSymbol(h3b::g_device_error, &z, sizeof(z));
    if (e != cudaSuccess) return h3b_host::set_error(H3B_ECUDA, "reset of device error word failed: %s", cudaGetErrorString(e));
  }
  return H3B_OK;
}

}  // extern "C"
