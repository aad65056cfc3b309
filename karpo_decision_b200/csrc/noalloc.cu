// kd_qkv_projection_noalloc: the fused QKV projection for callers that cannot allocate device memory.
//
// kd_qkv_projection needs a per-pack scratch buffer, the rotary factors that kd_rope_gather lays out for it
// (rot / 2 x M uint32). A caller that can only hand the library its input and output buffers has nowhere to put that
// buffer: for example a plugin host that owns every device allocation through its own pool and does not let a plugin
// call cudaMalloc, or an embedding runtime that forbids side allocations on its devices. This entry point keeps the
// scratch in a fixed array inside the library instead, and otherwise runs exactly what the caller would run:
// kd_rope_gather into that array, then kd_qkv_projection reading it.
//
// Limits and sharing:
// - the array holds KD_NOALLOC_ROPE_ENTRIES (4 Mi) uint32 entries, 16 MiB, allocated by the CUDA runtime for every
//   device that loads the library and held until the process exits; a call needs (rot / 2) * M entries and is
//   rejected with KD_ERR_ARGUMENT beyond that (e.g. M <= 65,536 tokens at rot = 128);
// - every call on a device uses the same array and leaves its contents behind; the gather overwrites every entry the
//   projection reads, so nothing needs clearing between calls, but two calls whose kernels overlap on the GPU (different
//   streams without ordering between them) race on the array;
// - the first call on each device looks up the array's device address (cudaGetSymbolAddress, with that device
//   current) and caches it; make that first call before any stream capture on the device;
// - every argument is checked before the first launch, so a rejected call launches nothing and leaves the array as
//   it was; positions outside the rotary tables' rows read as the identity rotation, never past the tables.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "kd_internal.h"

#define KD_NOALLOC_ROPE_ENTRIES (4u << 20)

namespace kd {
namespace noalloc {

// The scratch of every kd_qkv_projection_noalloc call on a device (its host-side name is not a device address).
static __device__ __align__(256) uint32_t rope_scratch[KD_NOALLOC_ROPE_ENTRIES];

constexpr int MAX_DEVICES = 64;
static uint32_t* scratch_ptr[MAX_DEVICES] = {nullptr};
static std::mutex scratch_lock;

// The device address of rope_scratch on the current device (looked up once per device).
static int scratch_address(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e, "qkv_projection_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= MAX_DEVICES) return set_error(KD_ERR_ARGUMENT, "qkv_projection_noalloc: device index");
  std::lock_guard<std::mutex> guard(scratch_lock);
  if (scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, rope_scratch);
    if (e != cudaSuccess) return record_cuda_error(e, "qkv_projection_noalloc: cudaGetSymbolAddress");
    scratch_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = scratch_ptr[dev];
  return KD_OK;
}

}  // namespace noalloc
}  // namespace kd

extern "C" int kd_qkv_projection_noalloc(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                                         const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim,
                                         int gated, const void* q_norm_w, const void* k_norm_w, int qk_norm_mode,
                                         int v_norm_mode, float eps, const float* cos_tab, const float* sin_tab,
                                         int64_t positions, int rot, void* q, void* k, void* v, void* gate,
                                         int* status, cudaStream_t stream) {
  // Every check comes before the first launch: a rejected call neither launches the gather nor touches the shared
  // array. Sizes first (no CUDA call), then the gather's own arguments, then the array's address, then every check
  // of the projection (descriptors included) with that address standing in for the caller's buffer.
  if (M < 0 || rot < 0 || rot % 2) return kd::set_error(KD_ERR_ARGUMENT, "qkv_projection_noalloc: bad sizes");
  if (rot > head_dim || rot % 32)
    return kd::set_error(KD_ERR_ARGUMENT,
                         "qkv_projection_noalloc: rotary width must be a multiple of 32 within head_dim");
  const uint64_t entries = (uint64_t)(rot / 2) * (uint64_t)M;
  if (entries > KD_NOALLOC_ROPE_ENTRIES)
    return kd::set_error(KD_ERR_ARGUMENT,
                         "qkv_projection_noalloc: (rot / 2) * M exceeds the static scratch of 4194304 entries");
  const bool gather = M > 0 && rot > 0;
  if (gather && (!seqpos || !cos_tab || !sin_tab || positions <= 0))
    return kd::set_error(KD_ERR_ARGUMENT, "qkv_projection_noalloc: rotary tables, their rows and seqpos required");
  uint32_t* scratch = nullptr;
  int rc = kd::noalloc::scratch_address(&scratch);
  if (rc) return rc;
  rc = kd::qkv_projection_check(A, lda, W, ldw, M, N, K, seqpos, num_heads_q, num_heads_kv, head_dim, gated, q_norm_w,
                                k_norm_w, qk_norm_mode, v_norm_mode, eps, scratch, rot, q, k, v, gate, status);
  if (rc) return rc;
  if (gather) {
    rc = kd_rope_gather(seqpos, M, cos_tab, sin_tab, positions, rot, scratch, stream);
    if (rc) return rc;
  }
  return kd_qkv_projection(A, lda, W, ldw, M, N, K, seqpos, num_heads_q, num_heads_kv, head_dim, gated, q_norm_w,
                           k_norm_w, qk_norm_mode, v_norm_mode, eps, scratch, rot, q, k, v, gate, status, stream);
}
