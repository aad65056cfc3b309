// Memory-bound kernels of the packed forward: embedding gather, RMSNorm variants (with residual sums, layer scalar and
// e4m3 quantization fused), q/k/v norm + RoPE on the fused QKV projection output, rotary tables, the marker head and
// the readout. All use 16-byte vector accesses along contiguous rows; one warp per row (or per token-head).
//
// Numerics follow the reference's fused pointwise ops (families/qwen/fused.py, families/gemma/fused.py,
// serve/fp8.py): float32 math on bf16 inputs with one bf16 rounding per compiled op output.
#include "common.cuh"
#include "kd_internal.h"

namespace kd {
namespace ew {

constexpr int WARPS = 8;  // rows per 256-thread block

KD_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

KD_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

KD_DEVICE void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

KD_DEVICE void store8(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

// Multiplier of the normalized value: none, w, or 1 + w (norm_mode KD_NORM_*).
KD_DEVICE void norm_weights(const __nv_bfloat16* w, int mode, int col, float (&m)[8]) {
  if (mode == KD_NORM_NONE || w == nullptr) {
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = 1.0f;
    return;
  }
  load8(w + col, m);
  if (mode == KD_NORM_ONE_PLUS) {
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = 1.0f + m[i];
  }
}

// 1 / sqrt(mean(x^2) + eps) with IEEE-rounded sqrt and division.
KD_DEVICE float inv_rms(float sumsq, int cols, float eps) { return 1.0f / sqrtf(sumsq / (float)cols + eps); }

// x / s rounded to nearest, as the reference's float division, with r = RN(1 / s) formed once per row: one correction
// step on the product (Markstein's theorem, IBM J. Res. Dev. 34(1), 1990): q0 = RN(x r), e = x - q0 s (exact in one
// fma), q = RN(q0 + e r) is the correctly rounded quotient when r is the correctly rounded reciprocal.
KD_DEVICE float div_by(float x, float s, float r) {
  const float q0 = x * r;
  return fmaf(fmaf(-q0, s, x), r, q0);
}

// Eight values x / s to e4m3, round to nearest even, saturating at +-448 (the reference's clamp to +-448 then cast;
// NaN stays NaN), converted in pairs. A row whose scale is infinite (an infinite input) divides directly.
KD_DEVICE uint2 quantize8(const float (&f)[8], float s, float r) {
  uint32_t p[4];
  const bool finite = isfinite(s);
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-s, -s);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 x = make_float2(f[2 * k], f[2 * k + 1]);
    float2 q;
    if (finite) {  // div_by on a pair
      const float2 q0 = mul2(x, r2);
      q = fma2(fma2(q0, ns2, x), r2, q0);
    } else {
      q = make_float2(x.x / s, x.y / s);
    }
    p[k] = __nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3);
  }
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

// ------------------------------------------------------------------------------------------------ embedding

__global__ void embed_kernel(const int64_t* __restrict__ ids, int64_t T, const __nv_bfloat16* __restrict__ table,
                             int64_t vocab, int hidden, float scale, __nv_bfloat16* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= T) return;
  int64_t id = ids[row];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);  // ids outside the vocabulary clamp (validated on the host)
  const __nv_bfloat16* src = table + id * hidden;
  __nv_bfloat16* dst = out + row * hidden;
  const int lane = threadIdx.x & 31;
  for (int c = lane * 8; c < hidden; c += 256) {
    if (scale == 0.0f) {
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
    } else {
      float f[8];
      load8(src + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] *= scale;  // bf16 x bf16(scale), rounded once
      store8(dst + c, f);
    }
  }
}

// ------------------------------------------------------------------------------------------------ RMSNorm family

// out = norm(x) (optionally gathered rows: src row = rows_idx[row]).
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int64_t* __restrict__ rows_idx,
                               const __nv_bfloat16* __restrict__ w, int mode, float eps, __nv_bfloat16* __restrict__ out,
                               int64_t ldo, int64_t rows, int cols) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t src_row = rows_idx ? rows_idx[row] : row;
  const __nv_bfloat16* xr = x + src_row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  const float inv = inv_rms(warp_sum(ss), cols, eps);
  __nv_bfloat16* orow = out + row * ldo;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8], m[8];
    load8(xr + c, f);
    norm_weights(w, mode, c, m);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (f[i] * inv) * m[i];
    store8(orow + c, f);
  }
}

// Qwen residual: h = bf16(h + x); y = norm(h).
__global__ void add_rmsnorm_kernel(__nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, int mode, float eps,
                                   __nv_bfloat16* __restrict__ y, int64_t rows, int cols) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  __nv_bfloat16* hr = h + row * cols;
  const __nv_bfloat16* xr = x + row * cols;
  float ss = 0.f;
  for (int c = lane * 8; c < cols; c += 256) {
    float a[8], b[8];
    load8(hr + c, a);
    load8(xr + c, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] = bf16_round(a[i] + b[i]);
      ss += a[i] * a[i];
    }
    store8(hr + c, a);
  }
  const float inv = inv_rms(warp_sum(ss), cols, eps);
  __syncwarp();
  __nv_bfloat16* yr = y + row * cols;
  for (int c = lane * 8; c < cols; c += 256) {
    float a[8], m[8];
    load8(hr + c, a);
    norm_weights(w, mode, c, m);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = (a[i] * inv) * m[i];
    store8(yr + c, a);
  }
}

// Gemma residual: out = bf16(h + norm(x)); with a layer scalar: out = bf16((h + bf16(norm(x))) * scalar);
// mode < 0 skips the norm (x is already normed).
__global__ void norm_add_kernel(const __nv_bfloat16* h, const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ w, int mode, float eps,
                                const __nv_bfloat16* __restrict__ scalar, __nv_bfloat16* out, int64_t rows, int cols) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* hr = h + row * cols;
  const __nv_bfloat16* xr = x + row * cols;
  float inv = 1.0f;
  if (mode >= 0) {
    float ss = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8];
      load8(xr + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    inv = inv_rms(warp_sum(ss), cols, eps);
  }
  const float s = scalar ? __bfloat162float(*scalar) : 1.0f;
  __nv_bfloat16* orow = out + row * cols;
  for (int c = lane * 8; c < cols; c += 256) {
    float a[8], b[8], m[8];
    load8(hr + c, a);
    load8(xr + c, b);
    if (mode >= 0) {
      norm_weights(w, mode, c, m);
#pragma unroll
      for (int i = 0; i < 8; ++i) b[i] = (b[i] * inv) * m[i];
    }
    if (scalar) {
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = (a[i] + bf16_round(b[i])) * s;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = a[i] + b[i];
    }
    store8(orow + c, a);
  }
}

// y = bf16(norm(x)) (or x itself when mode < 0), then per-row e4m3: s = max(amax(y), 1e-12) * (1 / 448),
// q = e4m3(clamp(y / s, +-448)) (serve/fp8.py:21-24, :57-69).
__global__ void rmsnorm_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                    const __nv_bfloat16* __restrict__ w, int mode, float eps,
                                    __nv_fp8_e4m3* __restrict__ q, float* __restrict__ scale, int64_t rows, int cols) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + row * ldx;
  float inv = 1.0f;
  if (mode >= 0) {
    float ss = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8];
      load8(xr + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    inv = inv_rms(warp_sum(ss), cols, eps);
  }
  float amax = 0.f;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8], m[8];
    load8(xr + c, f);
    if (mode >= 0) norm_weights(w, mode, c, m);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float yv = mode >= 0 ? bf16_round((f[i] * inv) * m[i]) : f[i];
      amax = fmaxf(amax, fabsf(yv));
    }
  }
  amax = warp_max(amax);
  // torch on CUDA divides a tensor by a scalar as a multiply by the float32 reciprocal (the reference's
  // amax / E4M3_MAX), so the scale is formed the same way; the values divide by the scale exactly.
  const float s = fmaxf(amax, 1e-12f) * (1.0f / 448.0f);
  const float rs = __frcp_rn(s);
  if (lane == 0) scale[row] = s;
  __nv_fp8_e4m3* qr = q + row * (int64_t)cols;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8], m[8];
    load8(xr + c, f);
    if (mode >= 0) {
      norm_weights(w, mode, c, m);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = bf16_round((f[i] * inv) * m[i]);
    }
    *reinterpret_cast<uint2*>(qr + c) = quantize8(f, s, rs);
  }
}

// ---- wide rows: one row per 256-thread block, held in registers between the passes, so it is read from memory once
// (a warp per row re-reads its row for each pass, and rows of several KB from many warps fall out of L1 and L2).
constexpr int ROW_THREADS = 256;
constexpr int ROW_PIECES = 12;   // 8-element pieces per thread: rows up to 12 * 256 * 8 = 24,576 columns
// From this width rmsnorm and rmsnorm_e4m3 take the block path, both of them, so they reduce alike (measured on
// 32,768-row tensors: at 2,560 columns the warp path is as fast or faster, at 3,840 the block path is 17-24% faster).
// norm_add stays a warp per row: inside the forward its x was just written by a GEMM and the second read hits L2.
constexpr int WIDE_COLS = 3072;

KD_DEVICE void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Block-wide sum and max: warp shuffles, then the eight warp results in a fixed tree (every thread gets the same).
KD_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();  // red may still be read by the block's previous reduction
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
}
KD_DEVICE float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])), fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
}

// This thread's pieces of a row: pieces threadIdx.x, threadIdx.x + 256, ... (zero past the row's end).
template <int R>
KD_DEVICE void load_row(const __nv_bfloat16* xr, int cols, uint4 (&v)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (threadIdx.x + r * ROW_THREADS) * 8;
    v[r] = c < cols ? *reinterpret_cast<const uint4*>(xr + c) : make_uint4(0, 0, 0, 0);
  }
}

// 1 / rms of a row held by the block (each thread's pieces summed in order, even and odd elements apart, then
// block_sum): the same value in rmsnorm_row_kernel and rmsnorm_e4m3_row_kernel, so the fused norm + quantization
// equals the two separate ops.
template <int R>
KD_DEVICE float row_inv(const uint4 (&v)[R], int cols, float eps, float* red) {
  float2 ss = make_float2(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if ((threadIdx.x + r * ROW_THREADS) * 8 >= cols) break;
    const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = unpack_bf16x2(w[i]);
      ss = fma2(t, t, ss);
    }
  }
  return inv_rms(block_sum(ss.x + ss.y, red), cols, eps);
}

template <int R>
__global__ void __launch_bounds__(ROW_THREADS) rmsnorm_row_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                  const int64_t* __restrict__ rows_idx,
                                                                  const __nv_bfloat16* __restrict__ w, int mode,
                                                                  float eps, __nv_bfloat16* __restrict__ out,
                                                                  int64_t ldo, int cols) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t src_row = rows_idx ? rows_idx[row] : row;
  uint4 v[R];
  load_row(x + src_row * ldx, cols, v);
  const float inv = row_inv(v, cols, eps, red);
  __nv_bfloat16* orow = out + row * ldo;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (threadIdx.x + r * ROW_THREADS) * 8;
    if (c >= cols) break;
    float f[8], m[8];
    unpack8(v[r], f);
    norm_weights(w, mode, c, m);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (f[i] * inv) * m[i];
    store8(orow + c, f);
  }
}

// rmsnorm_e4m3_kernel for wide rows: the normed bf16 row is kept (packed) in registers for the scale and the cast;
// its maximum magnitude is taken on the packed pairs (exact for a maximum).
template <int R>
__global__ void __launch_bounds__(ROW_THREADS) rmsnorm_e4m3_row_kernel(const __nv_bfloat16* __restrict__ x,
                                                                       int64_t ldx, const __nv_bfloat16* __restrict__ w,
                                                                       int mode, float eps,
                                                                       __nv_fp8_e4m3* __restrict__ q,
                                                                       float* __restrict__ scale, int cols) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  uint4 v[R];
  load_row(x + row * ldx, cols, v);
  if (mode >= 0) {  // y = bf16(norm(x)), kept for the cast below
    const float inv = row_inv(v, cols, eps, red);
    const float2 inv2 = make_float2(inv, inv);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int c = (threadIdx.x + r * ROW_THREADS) * 8;
      if (c >= cols) break;
      float f[8], m[8];
      unpack8(v[r], f);
      norm_weights(w, mode, c, m);
      uint32_t pk[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 y = mul2(mul2(make_float2(f[2 * k], f[2 * k + 1]), inv2), make_float2(m[2 * k], m[2 * k + 1]));
        pk[k] = pack_bf16x2(y.x, y.y);
      }
      v[r] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  __nv_bfloat162 mx2 = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if ((threadIdx.x + r * ROW_THREADS) * 8 >= cols) break;
    const uint32_t wv[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) mx2 = __hmax2(mx2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&wv[k])));
  }
  const float amax = block_max(fmaxf(__low2float(mx2), __high2float(mx2)), red);
  const float s = fmaxf(amax, 1e-12f) * (1.0f / 448.0f);  // as rmsnorm_e4m3_kernel forms it
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[row] = s;
  __nv_fp8_e4m3* qr = q + row * (int64_t)cols;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (threadIdx.x + r * ROW_THREADS) * 8;
    if (c >= cols) break;
    float f[8];
    unpack8(v[r], f);
    *reinterpret_cast<uint2*>(qr + c) = quantize8(f, s, rs);
  }
}

// rmsnorm_e4m3_kernel for rows narrower than WIDE_COLS with the row in registers: one warp per row reads it once (the
// three-pass kernel reads it for the sum of squares, the maximum and the cast), forms the normed bf16 row once,
// takes its maximum on packed pairs and casts from registers. The sum of squares runs in rmsnorm_kernel's order
// (each lane's pieces in turn, then warp_sum), so the fused norm + cast still equals kd_rmsnorm followed by the cast.
template <int R>
__global__ void rmsnorm_e4m3_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                         const __nv_bfloat16* __restrict__ w, int mode, float eps,
                                         __nv_fp8_e4m3* __restrict__ q, float* __restrict__ scale, int64_t rows,
                                         int cols) {
  const int64_t row = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + row * ldx;
  uint4 v[R];  // pieces lane, lane + 32, ... (zero past the row's end)
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (lane + 32 * r) * 8;
    v[r] = c < cols ? *reinterpret_cast<const uint4*>(xr + c) : make_uint4(0, 0, 0, 0);
  }
  if (mode >= 0) {  // y = bf16(norm(x)), kept packed for the maximum and the cast
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if ((lane + 32 * r) * 8 >= cols) break;
      float f[8];
      unpack8(v[r], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    const float inv = inv_rms(warp_sum(ss), cols, eps);
    const float2 inv2 = make_float2(inv, inv);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int c = (lane + 32 * r) * 8;
      if (c >= cols) break;
      float f[8], m[8];
      unpack8(v[r], f);
      norm_weights(w, mode, c, m);
      uint32_t pk[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 y = mul2(mul2(make_float2(f[2 * k], f[2 * k + 1]), inv2), make_float2(m[2 * k], m[2 * k + 1]));
        pk[k] = pack_bf16x2(y.x, y.y);
      }
      v[r] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  __nv_bfloat162 mx2 = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if ((lane + 32 * r) * 8 >= cols) break;
    const uint32_t wv[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) mx2 = __hmax2(mx2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&wv[k])));
  }
  const float amax = warp_max(fmaxf(__low2float(mx2), __high2float(mx2)));
  const float s = fmaxf(amax, 1e-12f) * (1.0f / 448.0f);  // as rmsnorm_e4m3_kernel forms it
  const float rs = __frcp_rn(s);
  if (lane == 0) scale[row] = s;
  __nv_fp8_e4m3* qr = q + row * (int64_t)cols;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int c = (lane + 32 * r) * 8;
    if (c >= cols) break;
    float f[8];
    unpack8(v[r], f);
    *reinterpret_cast<uint2*>(qr + c) = quantize8(f, s, rs);
  }
}

// ------------------------------------------------------------------------------------------------ RoPE

__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int rot, int64_t positions,
                                  float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= positions * rot) return;
  const int64_t p = idx / rot;
  const int i = (int)(idx % rot);
  const float emb = (float)p * inv_freq[i % (rot / 2)];  // freqs = position x inv_freq in float32, cat(f, f)
  cos_out[idx] = bf16_round(cosf(emb));
  sin_out[idx] = bf16_round(sinf(emb));
}

// Per-token tables for M-RoPE (several position axes): row t holds pair i's factors at the position of the axis that
// pair reads, pos[axis(i) * ld_axis + t], with rope_table_kernel's arithmetic (float32 product, then bf16-rounded
// cos / sin). An axis index outside [0, axes) reads axis 0.
__global__ void rope_table_axes_kernel(const float* __restrict__ inv_freq, int rot, const int64_t* __restrict__ pos,
                                       int64_t ld_axis, int64_t T, const int32_t* __restrict__ pair_axis, int axes,
                                       float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * rot) return;
  const int64_t t = idx / rot;
  const int pair = (int)(idx % rot) % (rot / 2);
  int ax = pair_axis[pair];
  if (ax < 0 || ax >= axes) ax = 0;
  const float emb = (float)pos[ax * ld_axis + t] * inv_freq[pair];
  cos_out[idx] = bf16_round(cosf(emb));
  sin_out[idx] = bf16_round(sinf(emb));
}

// dst[i, :] = src[rows[i], :] for bf16 rows of `width` elements (width % 8 == 0): one warp per row, 16-byte copies.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t ld_src,
                                   const int64_t* __restrict__ rows, int64_t n, int width,
                                   __nv_bfloat16* __restrict__ dst, int64_t ld_dst) {
  const int64_t i = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (i >= n) return;
  const int lane = threadIdx.x & 31;
  const uint4* s = reinterpret_cast<const uint4*>(src + rows[i] * ld_src);
  uint4* d = reinterpret_cast<uint4*>(dst + i * ld_dst);
  for (int c = lane; c < width / 8; c += 32) d[c] = s[c];
}

// dst[rows[i], :] = src[i, :] (rows distinct): one warp per row, 16-byte copies.
__global__ void scatter_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t ld_src,
                                    const int64_t* __restrict__ rows, int64_t n, int width,
                                    __nv_bfloat16* __restrict__ dst, int64_t ld_dst) {
  const int64_t i = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (i >= n) return;
  const int lane = threadIdx.x & 31;
  const uint4* s = reinterpret_cast<const uint4*>(src + i * ld_src);
  uint4* d = reinterpret_cast<uint4*>(dst + rows[i] * ld_dst);
  for (int c = lane; c < width / 8; c += 32) d[c] = s[c];
}

// cs[i * T + t] = bf16 cos | bf16 sin << 16 of rotary pair i at seqpos[t] (t fastest: coalesced writes). A position
// outside the table's rows [0, positions) is never read: its entry is the identity rotation (cos 1, sin 0).
__global__ void rope_gather_kernel(const int64_t* __restrict__ seqpos, int64_t T, const float* __restrict__ cos_tab,
                                   const float* __restrict__ sin_tab, int64_t positions, int rot,
                                   uint32_t* __restrict__ cs) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int half = rot / 2;
  if (idx >= T * half) return;
  const int i = (int)(idx / T);
  const int64_t t = idx % T;
  const int64_t pos = seqpos[t];
  if (pos < 0 || pos >= positions) {
    cs[idx] = pack_bf16x2(1.0f, 0.0f);
    return;
  }
  const int64_t off = pos * rot + i;
  cs[idx] = pack_bf16x2(cos_tab[off], sin_tab[off]);
}

// One warp per (token, head). Heads 0..Hq-1 are queries, Hq..Hq+Hkv-1 keys, then Hkv values.
template <int HD>
__global__ void qkv_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld, int64_t T,
                                     const int64_t* __restrict__ seqpos, int hq, int hkv, int gated,
                                     const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                     int qk_mode, int v_mode, float eps, const float* __restrict__ cos_tab,
                                     const float* __restrict__ sin_tab, int rot, __nv_bfloat16* __restrict__ q,
                                     __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v,
                                     __nv_bfloat16* __restrict__ gate) {
  constexpr int PER = HD / 32;  // elements per lane (2, 4, 8 or 16)
  __shared__ float stage[WARPS][HD];
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  const int64_t item = (int64_t)blockIdx.x * WARPS + warp;
  if (item >= T * heads) return;
  const int64_t t = item / heads;
  const int head = (int)(item % heads);
  const int q_cols = hq * HD * (gated ? 2 : 1);
  const __nv_bfloat16* row = qkv + t * ld;
  const bool is_q = head < hq;
  const bool is_k = !is_q && head < hq + hkv;
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  if (is_q) {
    src = row + (int64_t)head * HD * (gated ? 2 : 1);
    dst = q + (t * hq + head) * HD;
  } else if (is_k) {
    src = row + q_cols + (int64_t)(head - hq) * HD;
    dst = k + (t * hkv + (head - hq)) * HD;
  } else {
    src = row + q_cols + (int64_t)hkv * HD + (int64_t)(head - hq - hkv) * HD;
    dst = v + (t * hkv + (head - hq - hkv)) * HD;
  }
  float f[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) f[i] = __bfloat162float(src[lane * PER + i]);

  if (is_q && gated) {  // the query's gate half passes through to the output gate buffer
    const __nv_bfloat16* g = src + HD;
    __nv_bfloat16* gd = gate + (t * hq + head) * HD;
#pragma unroll
    for (int i = 0; i < PER; ++i) gd[lane * PER + i] = g[lane * PER + i];
  }
  if (!is_q && !is_k) {  // values: Gemma's v_norm (no weight) or a plain copy (Qwen)
    if (v_mode >= 0) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) ss += f[i] * f[i];
      const float inv = inv_rms(warp_sum(ss), HD, eps);
#pragma unroll
      for (int i = 0; i < PER; ++i) f[i] *= inv;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[lane * PER + i] = __float2bfloat16_rn(f[i]);
    return;
  }
  // q / k: per-head RMSNorm over HD, then rotate-half RoPE on the first `rot` dims.
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) ss += f[i] * f[i];
  const float inv = inv_rms(warp_sum(ss), HD, eps);
  const __nv_bfloat16* nw = is_q ? qw : kw;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane * PER + i;
    float m = 1.0f;
    if (qk_mode == KD_NORM_WEIGHT) m = __bfloat162float(nw[d]);
    if (qk_mode == KD_NORM_ONE_PLUS) m = 1.0f + __bfloat162float(nw[d]);
    f[i] = (f[i] * inv) * m;
    if (gated) f[i] = bf16_round(f[i]);  // Qwen: the norm is its own op (rounded), RoPE another
    stage[warp][d] = f[i];
  }
  __syncwarp();
  const int64_t pos = seqpos[t];
  const float* ct = cos_tab + (int64_t)pos * rot;
  const float* st = sin_tab + (int64_t)pos * rot;
  const int half = rot / 2;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane * PER + i;
    float o = f[i];
    if (d < rot) {
      const float partner = d < half ? -stage[warp][d + half] : stage[warp][d - half];
      o = f[i] * ct[d] + partner * st[d];
    }
    dst[d] = __float2bfloat16_rn(o);
  }
}

// ------------------------------------------------------------------------------------------------ readout

// logits[m, c] = sum_k float(hidden[m, k]) * W[c, k]; cap * tanh(logits / cap) when cap > 0. One warp per (m, c).
__global__ void readout_kernel(const __nv_bfloat16* __restrict__ hidden, int64_t M, int hs,
                               const float* __restrict__ W, int codes, float cap, float* __restrict__ logits) {
  const int64_t item = (int64_t)blockIdx.x * WARPS + threadIdx.x / 32;
  if (item >= M * codes) return;
  const int lane = threadIdx.x & 31;
  const int64_t m = item / codes;
  const int c = (int)(item % codes);
  const __nv_bfloat16* hr = hidden + m * hs;
  const float* wr = W + (int64_t)c * hs;
  float acc = 0.f;
  for (int k = lane * 8; k < hs; k += 256) {
    float f[8];
    load8(hr + k, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += f[i] * wr[k + i];
  }
  acc = warp_sum(acc);
  if (lane == 0) logits[item] = cap > 0.f ? cap * tanhf(acc / cap) : acc;
}

}  // namespace ew
}  // namespace kd

using namespace kd;
using kd::ew::WARPS;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static unsigned blocks_for(int64_t items) { return (unsigned)((items + WARPS - 1) / WARPS); }

extern "C" int kd_embed(const int64_t* ids, int64_t T, const void* table, int64_t vocab, int hidden, float scale,
                        void* out, cudaStream_t stream) {
  if (T < 0 || vocab <= 0 || hidden <= 0 || hidden % 8) return set_error(KD_ERR_ARGUMENT, "embed: bad sizes");
  if (T == 0) return KD_OK;
  if (!ids || !table || !out || !aligned16(table) || !aligned16(out))
    return set_error(KD_ERR_ARGUMENT, "embed: null or unaligned pointer");
  const float s = scale == 0.0f ? 0.0f : __bfloat162float(__float2bfloat16_rn(scale));
  ew::embed_kernel<<<blocks_for(T), 32 * WARPS, 0, stream>>>(ids, T, static_cast<const __nv_bfloat16*>(table), vocab,
                                                              hidden, s, static_cast<__nv_bfloat16*>(out));
  return record_cuda_error(cudaGetLastError(), "embed: launch");
}

static int check_norm(const void* x, const void* out, int mode, const void* w, int cols, const char* what) {
  if (cols <= 0 || cols % 8) return set_error(KD_ERR_ARGUMENT, "norm: cols must be a positive multiple of 8");
  if (!x || !out || !aligned16(x) || !aligned16(out)) return set_error(KD_ERR_ARGUMENT, what);
  if (mode > KD_NORM_NONE && (!w || !aligned16(w))) return set_error(KD_ERR_ARGUMENT, "norm: weight required");
  if (mode > KD_NORM_ONE_PLUS) return set_error(KD_ERR_ARGUMENT, "norm: unknown norm mode");
  return KD_OK;
}

extern "C" int kd_rmsnorm(const void* x, int64_t ldx, const void* weight, int norm_mode, float eps, void* out,
                          int64_t ldo, int64_t rows, int cols, cudaStream_t stream) {
  if (rows < 0) return set_error(KD_ERR_ARGUMENT, "rmsnorm: rows < 0");
  if (rows == 0) return KD_OK;
  int rc = check_norm(x, out, norm_mode, weight, cols, "rmsnorm: null or unaligned x/out");
  if (rc) return rc;
  if (norm_mode < 0) return set_error(KD_ERR_ARGUMENT, "rmsnorm: norm_mode must be KD_NORM_*");
  if (ldx % 8 || ldo % 8 || ldx < cols || ldo < cols) return set_error(KD_ERR_ARGUMENT, "rmsnorm: bad strides");
  if (cols >= ew::WIDE_COLS && cols <= ew::ROW_PIECES * ew::ROW_THREADS * 8 && rows <= 0x7fffffff) {
    const int pieces = (cols / 8 + ew::ROW_THREADS - 1) / ew::ROW_THREADS;
#define KD_ROW_CASE(R)                                                                                          \
  if (pieces <= R) {                                                                                            \
    ew::rmsnorm_row_kernel<R><<<(unsigned)rows, ew::ROW_THREADS, 0, stream>>>(                                  \
        static_cast<const __nv_bfloat16*>(x), ldx, nullptr, static_cast<const __nv_bfloat16*>(weight), norm_mode, \
        eps, static_cast<__nv_bfloat16*>(out), ldo, cols);                                                      \
    return record_cuda_error(cudaGetLastError(), "rmsnorm: launch");                                            \
  }
    KD_ROW_CASE(2) KD_ROW_CASE(3) KD_ROW_CASE(4) KD_ROW_CASE(6) KD_ROW_CASE(8) KD_ROW_CASE(12)
#undef KD_ROW_CASE
  }
  ew::rmsnorm_kernel<<<blocks_for(rows), 32 * WARPS, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, nullptr, static_cast<const __nv_bfloat16*>(weight), norm_mode, eps,
      static_cast<__nv_bfloat16*>(out), ldo, rows, cols);
  return record_cuda_error(cudaGetLastError(), "rmsnorm: launch");
}

extern "C" int kd_add_rmsnorm(void* h, const void* x, const void* weight, int norm_mode, float eps, void* y,
                              int64_t rows, int cols, cudaStream_t stream) {
  if (rows < 0) return set_error(KD_ERR_ARGUMENT, "add_rmsnorm: rows < 0");
  if (rows == 0) return KD_OK;
  int rc = check_norm(h, y, norm_mode, weight, cols, "add_rmsnorm: null or unaligned h/y");
  if (rc) return rc;
  if (!x || !aligned16(x) || norm_mode < 0) return set_error(KD_ERR_ARGUMENT, "add_rmsnorm: bad x or norm mode");
  ew::add_rmsnorm_kernel<<<blocks_for(rows), 32 * WARPS, 0, stream>>>(
      static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
      norm_mode, eps, static_cast<__nv_bfloat16*>(y), rows, cols);
  return record_cuda_error(cudaGetLastError(), "add_rmsnorm: launch");
}

extern "C" int kd_norm_add(const void* h, const void* x, const void* weight, int norm_mode, float eps,
                           const void* scalar, void* out, int64_t rows, int cols, cudaStream_t stream) {
  if (rows < 0) return set_error(KD_ERR_ARGUMENT, "norm_add: rows < 0");
  if (rows == 0) return KD_OK;
  int rc = check_norm(h, out, norm_mode, weight, cols, "norm_add: null or unaligned h/out");
  if (rc) return rc;
  if (!x || !aligned16(x)) return set_error(KD_ERR_ARGUMENT, "norm_add: null or unaligned x");
  ew::norm_add_kernel<<<blocks_for(rows), 32 * WARPS, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(weight), norm_mode, eps, static_cast<const __nv_bfloat16*>(scalar),
      static_cast<__nv_bfloat16*>(out), rows, cols);
  return record_cuda_error(cudaGetLastError(), "norm_add: launch");
}

extern "C" int kd_rmsnorm_e4m3(const void* x, int64_t ldx, const void* weight, int norm_mode, float eps, void* q,
                               float* scale, int64_t rows, int cols, cudaStream_t stream) {
  if (rows < 0) return set_error(KD_ERR_ARGUMENT, "rmsnorm_e4m3: rows < 0");
  if (rows == 0) return KD_OK;
  int rc = check_norm(x, q, norm_mode, weight, cols, "rmsnorm_e4m3: null or unaligned x/q");
  if (rc) return rc;
  if (!scale || ldx % 8 || ldx < cols) return set_error(KD_ERR_ARGUMENT, "rmsnorm_e4m3: bad scale or ldx");
  if (cols >= ew::WIDE_COLS && cols <= ew::ROW_PIECES * ew::ROW_THREADS * 8 && rows <= 0x7fffffff) {
    const int pieces = (cols / 8 + ew::ROW_THREADS - 1) / ew::ROW_THREADS;
#define KD_ROW_CASE(R)                                                                                       \
  if (pieces <= R) {                                                                                         \
    ew::rmsnorm_e4m3_row_kernel<R><<<(unsigned)rows, ew::ROW_THREADS, 0, stream>>>(                          \
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(weight), norm_mode, eps, \
        static_cast<__nv_fp8_e4m3*>(q), scale, cols);                                                        \
    return record_cuda_error(cudaGetLastError(), "rmsnorm_e4m3: launch");                                    \
  }
    KD_ROW_CASE(2) KD_ROW_CASE(3) KD_ROW_CASE(4) KD_ROW_CASE(6) KD_ROW_CASE(8) KD_ROW_CASE(12)
#undef KD_ROW_CASE
  }
  // Narrower rows: the register-resident warp kernel, except the cast alone beyond 8 pieces a lane, where the
  // three-pass kernel's re-reads hit L1 and measured 3% faster (32,768 x 2,560: 55.7 against 57.2 us; with the norm
  // the register-resident kernel is faster at every width: 94.9 -> 90.0 us there, 78.8 -> 56.4 at 65,536 x 1,024).
  const int lane_pieces = (cols / 8 + 31) / 32;
  if (cols < ew::WIDE_COLS && (norm_mode >= 0 || lane_pieces <= 8)) {
    const int pieces = lane_pieces;
#define KD_WARP_CASE(R)                                                                                       \
  if (pieces <= R) {                                                                                          \
    ew::rmsnorm_e4m3_warp_kernel<R><<<blocks_for(rows), 32 * WARPS, 0, stream>>>(                             \
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(weight), norm_mode, eps, \
        static_cast<__nv_fp8_e4m3*>(q), scale, rows, cols);                                                   \
    return record_cuda_error(cudaGetLastError(), "rmsnorm_e4m3: launch");                                     \
  }
    KD_WARP_CASE(1) KD_WARP_CASE(2) KD_WARP_CASE(3) KD_WARP_CASE(4) KD_WARP_CASE(6) KD_WARP_CASE(8) KD_WARP_CASE(12)
#undef KD_WARP_CASE
  }
  ew::rmsnorm_e4m3_kernel<<<blocks_for(rows), 32 * WARPS, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(weight), norm_mode, eps,
      static_cast<__nv_fp8_e4m3*>(q), scale, rows, cols);
  return record_cuda_error(cudaGetLastError(), "rmsnorm_e4m3: launch");
}

extern "C" int kd_quantize_rows_e4m3(const void* x, int64_t rows, int cols, void* q, float* scale,
                                     cudaStream_t stream) {
  return kd_rmsnorm_e4m3(x, cols, nullptr, -1, 0.0f, q, scale, rows, cols, stream);
}

extern "C" int kd_rope_table(const float* inv_freq, int rot, int64_t positions, float* cos_out, float* sin_out,
                             cudaStream_t stream) {
  if (rot <= 0 || rot % 2 || positions < 0 || !inv_freq || !cos_out || !sin_out)
    return set_error(KD_ERR_ARGUMENT, "rope_table: bad arguments");
  const int64_t n = positions * rot;
  if (n == 0) return KD_OK;
  ew::rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(inv_freq, rot, positions, cos_out, sin_out);
  return record_cuda_error(cudaGetLastError(), "rope_table: launch");
}

extern "C" int kd_rope_table_axes(const float* inv_freq, int rot, const int64_t* pos, int64_t ld_axis, int64_t T,
                                  const int32_t* pair_axis, int axes, float* cos_out, float* sin_out,
                                  cudaStream_t stream) {
  if (rot <= 0 || rot % 2 || T < 0 || axes < 1 || (axes > 1 && ld_axis < T))
    return set_error(KD_ERR_ARGUMENT, "rope_table_axes: bad sizes");
  if (T == 0) return KD_OK;
  if (!inv_freq || !pos || !pair_axis || !cos_out || !sin_out)
    return set_error(KD_ERR_ARGUMENT, "rope_table_axes: null pointer");
  const int64_t n = T * rot;
  ew::rope_table_axes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(inv_freq, rot, pos, ld_axis, T, pair_axis,
                                                                              axes, cos_out, sin_out);
  return record_cuda_error(cudaGetLastError(), "rope_table_axes: launch");
}

extern "C" int kd_qkv_norm_rope(const void* qkv, int64_t ldqkv, int64_t T, const int64_t* seqpos, int num_heads_q,
                                int num_heads_kv, int head_dim, int gated, const void* q_norm_w, const void* k_norm_w,
                                int qk_norm_mode, int v_norm_mode, float eps, const float* cos_tab,
                                const float* sin_tab, int rot, void* q, void* k, void* v, void* gate,
                                cudaStream_t stream) {
  if (T < 0 || num_heads_q <= 0 || num_heads_kv <= 0 || num_heads_q % num_heads_kv)
    return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: bad head counts");
  if (T == 0) return KD_OK;
  if (rot < 0 || rot > head_dim || rot % 2) return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: bad rotary width");
  if (!qkv || !seqpos || !q || !k || !v || (gated && !gate) || (rot > 0 && (!cos_tab || !sin_tab)))
    return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: null pointer");
  if (qk_norm_mode > KD_NORM_NONE && (!q_norm_w || !k_norm_w))
    return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: q/k norm weights required");
  const int64_t width = (int64_t)num_heads_q * head_dim * (gated ? 2 : 1) + 2LL * num_heads_kv * head_dim;
  if (ldqkv < width) return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: ldqkv smaller than the projection width");
  const int64_t items = T * (num_heads_q + 2 * num_heads_kv);
  const auto* in = static_cast<const __nv_bfloat16*>(qkv);
  const auto* qw = static_cast<const __nv_bfloat16*>(q_norm_w);
  const auto* kw = static_cast<const __nv_bfloat16*>(k_norm_w);
  auto* qo = static_cast<__nv_bfloat16*>(q);
  auto* ko = static_cast<__nv_bfloat16*>(k);
  auto* vo = static_cast<__nv_bfloat16*>(v);
  auto* go = static_cast<__nv_bfloat16*>(gate);
#define KD_QKV_CASE(HD)                                                                                          \
  case HD:                                                                                                       \
    ew::qkv_norm_rope_kernel<HD><<<blocks_for(items), 32 * WARPS, 0, stream>>>(                                  \
        in, ldqkv, T, seqpos, num_heads_q, num_heads_kv, gated, qw, kw, qk_norm_mode, v_norm_mode, eps, cos_tab, \
        sin_tab, rot, qo, ko, vo, go);                                                                           \
    break;
  switch (head_dim) {
    KD_QKV_CASE(64)
    KD_QKV_CASE(128)
    KD_QKV_CASE(256)
    KD_QKV_CASE(512)
    default:
      return set_error(KD_ERR_ARGUMENT, "qkv_norm_rope: head_dim must be 64, 128, 256 or 512");
  }
#undef KD_QKV_CASE
  return record_cuda_error(cudaGetLastError(), "qkv_norm_rope: launch");
}

extern "C" int kd_marker_norm(const void* h, int hidden, const int64_t* markers, int64_t M, const void* weight,
                              int norm_mode, float eps, void* out, cudaStream_t stream) {
  if (M < 0) return set_error(KD_ERR_ARGUMENT, "marker_norm: M < 0");
  if (M == 0) return KD_OK;
  int rc = check_norm(h, out, norm_mode, weight, hidden, "marker_norm: null or unaligned h/out");
  if (rc) return rc;
  if (!markers || norm_mode < 0) return set_error(KD_ERR_ARGUMENT, "marker_norm: bad markers or norm mode");
  ew::rmsnorm_kernel<<<blocks_for(M), 32 * WARPS, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(h), hidden, markers, static_cast<const __nv_bfloat16*>(weight), norm_mode,
      eps, static_cast<__nv_bfloat16*>(out), hidden, M, hidden);
  return record_cuda_error(cudaGetLastError(), "marker_norm: launch");
}

extern "C" int kd_readout(const void* hidden, int64_t M, int hidden_size, const float* weight, int codes, float cap,
                          float* logits, cudaStream_t stream) {
  if (M < 0 || codes <= 0 || hidden_size <= 0 || hidden_size % 8)
    return set_error(KD_ERR_ARGUMENT, "readout: bad sizes");
  if (M == 0) return KD_OK;
  if (!hidden || !weight || !logits || !aligned16(hidden)) return set_error(KD_ERR_ARGUMENT, "readout: bad pointers");
  ew::readout_kernel<<<blocks_for(M * codes), 32 * WARPS, 0, stream>>>(static_cast<const __nv_bfloat16*>(hidden), M,
                                                                     hidden_size, weight, codes, cap, logits);
  return record_cuda_error(cudaGetLastError(), "readout: launch");
}

extern "C" int kd_rope_gather(const int64_t* seqpos, int64_t T, const float* cos_tab, const float* sin_tab,
                              int64_t positions, int rot, uint32_t* cs, cudaStream_t stream) {
  if (T < 0 || rot <= 0 || rot % 2 || positions <= 0) return set_error(KD_ERR_ARGUMENT, "rope_gather: bad sizes");
  if (T == 0) return KD_OK;
  if (!seqpos || !cos_tab || !sin_tab || !cs) return set_error(KD_ERR_ARGUMENT, "rope_gather: null pointer");
  const int64_t n = T * (rot / 2);
  ew::rope_gather_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(seqpos, T, cos_tab, sin_tab, positions,
                                                                           rot, cs);
  return record_cuda_error(cudaGetLastError(), "rope_gather: launch");
}

extern "C" int kd_gather_rows(const void* src, int64_t ld_src, const int64_t* rows, int64_t n, int width, void* dst,
                              int64_t ld_dst, cudaStream_t stream) {
  if (n < 0 || width <= 0 || width % 8 || ld_src < width || ld_dst < width || ld_src % 8 || ld_dst % 8)
    return set_error(KD_ERR_ARGUMENT, "gather_rows: bad sizes or strides (width % 8 == 0, 16-byte rows)");
  if (n == 0) return KD_OK;
  if (!src || !rows || !dst || !aligned16(src) || !aligned16(dst))
    return set_error(KD_ERR_ARGUMENT, "gather_rows: null or unaligned pointer");
  ew::gather_rows_kernel<<<blocks_for(n), 32 * WARPS, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), ld_src,
                                                                  rows, n, width, static_cast<__nv_bfloat16*>(dst),
                                                                  ld_dst);
  return record_cuda_error(cudaGetLastError(), "gather_rows: launch");
}

extern "C" int kd_scatter_rows(const void* src, int64_t ld_src, const int64_t* rows, int64_t n, int width, void* dst,
                               int64_t ld_dst, cudaStream_t stream) {
  if (n < 0 || width <= 0 || width % 8 || ld_src < width || ld_dst < width || ld_src % 8 || ld_dst % 8)
    return set_error(KD_ERR_ARGUMENT, "scatter_rows: bad sizes or strides (width % 8 == 0, 16-byte rows)");
  if (n == 0) return KD_OK;
  if (!src || !rows || !dst || !aligned16(src) || !aligned16(dst))
    return set_error(KD_ERR_ARGUMENT, "scatter_rows: null or unaligned pointer");
  ew::scatter_rows_kernel<<<blocks_for(n), 32 * WARPS, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), ld_src,
                                                                   rows, n, width, static_cast<__nv_bfloat16*>(dst),
                                                                   ld_dst);
  return record_cuda_error(cudaGetLastError(), "scatter_rows: launch");
}
