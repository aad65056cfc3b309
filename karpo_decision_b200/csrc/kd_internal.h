// Host-side helpers shared by the translation units of libkd_b200: error recording, TMA descriptor encoding and
// device properties. Not part of the public C ABI (that is include/kd_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kd_b200.h"

namespace kd {

// Records `msg` as this thread's last error (kd_last_error) and returns `code`.
int set_error(int code, const char* msg);
// KD_OK for cudaSuccess; otherwise records "<what>: <cuda error string>" and returns KD_ERR_CUDA.
int record_cuda_error(cudaError_t e, const char* what);
// Streaming-multiprocessor count of device `dev` (cached).
int num_sms(int dev);

// A 2-D tiled TMA descriptor over a row-major matrix of `outer` rows x `inner` elements (row stride `ld` elements),
// box = box_inner x box_outer elements; out-of-range elements read as zero.
int make_tma_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

// A 3-D tiled TMA descriptor: dims (d0 innermost, d1, d2) with element strides (s1, s2) and box (b0, b1, b2).
int make_tma_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                CUtensorMapSwizzle swizzle);

// Every check kd_qkv_projection makes (sizes, pointers, alignment, the TMA descriptors it would encode) without
// launching anything: KD_OK when that call would be accepted.
int qkv_projection_check(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                         const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim, int gated,
                         const void* q_norm_w, const void* k_norm_w, int qk_norm_mode, int v_norm_mode, float eps,
                         const uint32_t* rope_cs, int rot, void* q, void* k, void* v, void* gate, int* status);

}  // namespace kd
