// Host runtime of libkd_b200: last-error reporting, device properties and TMA descriptor encoding through the
// driver entry point (no link-time dependency on libcuda).
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "kd_internal.h"

namespace kd {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* msg) {
  snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

int record_cuda_error(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KD_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
  return KD_ERR_CUDA;
}

int num_sms(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 1;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 1;
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return set_error(KD_ERR_DRIVER, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[256];
    snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled (2-D) failed with CUresult %d (inner %llu outer %llu ld %llu)",
             (int)r, (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)ld);
    return set_error(KD_ERR_DRIVER, msg);
  }
  return KD_OK;
}

int make_tma_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return set_error(KD_ERR_DRIVER, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1 * (uint64_t)elem_bytes, s2 * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[128];
    snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled (3-D) failed with CUresult %d", (int)r);
    return set_error(KD_ERR_DRIVER, msg);
  }
  return KD_OK;
}

}  // namespace kd

extern "C" int kd_version(void) { return 100; }  // 0.1.0

extern "C" int kd_last_error(char* buf, size_t n) {
  const int len = (int)strlen(kd::g_last_error);
  if (buf && n > 0) snprintf(buf, n, "%s", kd::g_last_error);
  return len;
}

namespace kd {

// Two waiters on an mbarrier that nothing arrives on: warp 0 with `limit_ns`, warp 1 with 64 x that limit. Warp 0's
// wait runs out and records KD_DEVICE_TIMEOUT; warp 1 must then give up on seeing the status, long before its own
// limit, as every other wait of a failed launch does. Each records the nanoseconds it waited in elapsed[warp].
__global__ void wait_selftest_kernel(int* status, uint64_t limit_ns, int64_t* elapsed) {
  __shared__ uint64_t bar;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    const uint64_t start = globaltimer();
    const bool ok = mbar_wait_for(&bar, 0, status, warp == 0 ? limit_ns : 64 * limit_ns);
    elapsed[warp] = ok ? -1 : (int64_t)(globaltimer() - start);
  }
}

}  // namespace kd

extern "C" int kd_wait_selftest(int* status, int64_t limit_ns, int64_t* elapsed, cudaStream_t stream) {
  if (!status || !elapsed || limit_ns <= 0 || limit_ns > 1000000000LL)
    return kd::set_error(KD_ERR_ARGUMENT, "wait_selftest: status, elapsed and a limit in (0, 1 s] required");
  kd::wait_selftest_kernel<<<1, 64, 0, stream>>>(status, (uint64_t)limit_ns, elapsed);
  return kd::record_cuda_error(cudaGetLastError(), "wait_selftest: launch");
}
