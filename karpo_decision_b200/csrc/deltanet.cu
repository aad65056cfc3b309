// Qwen3.5's Gated DeltaNet token mixer (families/qwen/packed.py:74-106), the kernels between its input projection
// and its output projection:
//   kd_conv_silu         depthwise causal convolution over the [q | k | v] channels, cut at sequence starts, + silu;
//   kd_gated_delta_rule  the gated delta rule per (sequence, value head), its decay and write strength computed from
//                        the projection's a and b columns;
//   kd_gated_norm        Qwen3_5RMSNormGated: RMSNorm of each head's output times silu of the z gate.
//
// The delta rule here is the recurrent form: one CTA per (sequence, value head) holds the head's state S (dk x dv,
// float32) in registers, two threads per value column each owning half of its dk rows, and walks the sequence token
// by token (the next rows fetched while it walks); CTAs take the longest sequences first. Queries and keys are L2-normalized (the reference's use_qk_l2norm_in_kernel), per chunk of tokens staged
// in shared memory by the CTA's warps before the sequential walk.
#include "common.cuh"
#include "kd_internal.h"

namespace kd {
namespace dn {

// ------------------------------------------------------------------------------------------------ convolution

// out[t, c] = bf16(silu(sum_s w[c, K-1-s] x[t-s, c])) over taps s with seqpos[t] >= s, float32 sums in tap order.
// A thread takes 8 channels (16-byte loads) of ROWS_PER_THREAD consecutive rows: its taps are loaded once and the
// K - 1 rows before each row come from registers, so every input row is read from memory about once.
constexpr int ROWS_PER_THREAD = 16;

template <int K>
__global__ void conv_silu_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t T, int C,
                                 const __nv_bfloat16* __restrict__ w, const int64_t* __restrict__ seqpos,
                                 __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int groups = C / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t blocks = (T + ROWS_PER_THREAD - 1) / ROWS_PER_THREAD;
  if (idx >= blocks * groups) return;
  const int c0 = (int)(idx % groups) * 8;  // consecutive threads: consecutive channel groups of the same rows
  const int64_t r0 = (idx / groups) * ROWS_PER_THREAD;
  const int64_t r1 = r0 + ROWS_PER_THREAD < T ? r0 + ROWS_PER_THREAD : T;
  // taps of channels c0..c0+7: 8 x K contiguous bf16
  float taps[8][K];
  {
    const __nv_bfloat16* wp = w + (int64_t)c0 * K;
#pragma unroll
    for (int q = 0; q < K; ++q) {  // 8 * K elements = K 16-byte pieces
      const uint4 raw = *reinterpret_cast<const uint4*>(wp + 8 * q);
      const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(words[e]);
        const int i0 = 8 * q + 2 * e;  // flat index channel * K + tap
        taps[i0 / K][i0 % K] = f.x;
        taps[(i0 + 1) / K][(i0 + 1) % K] = f.y;
      }
    }
  }
  // hist[s]: the row s back from the current one (s = 1 .. K - 1), zero before the pack's first row
  float hist[K][8];
#pragma unroll
  for (int s = 1; s < K; ++s) {
#pragma unroll
    for (int e = 0; e < 8; ++e) hist[s][e] = 0.f;
    if (r0 - s >= 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + (r0 - s) * ldx + c0);
      const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(words[e]);
        hist[s][2 * e] = f.x;
        hist[s][2 * e + 1] = f.y;
      }
    }
  }
  // the next row's values are loaded while the current row is computed (two loads in flight per thread)
  uint4 next = r0 < r1 ? *reinterpret_cast<const uint4*>(x + r0 * ldx + c0) : make_uint4(0, 0, 0, 0);
  int64_t next_pos = r0 < r1 ? seqpos[r0] : 0;
  for (int64_t t = r0; t < r1; ++t) {
    const int64_t pos = next_pos;
    const uint4 raw = next;
    if (t + 1 < r1) {
      next = *reinterpret_cast<const uint4*>(x + (t + 1) * ldx + c0);
      next_pos = seqpos[t + 1];
    }
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    float cur[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(words[e]);
      cur[2 * e] = f.x;
      cur[2 * e + 1] = f.y;
    }
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = cur[e] * taps[e][K - 1];
#pragma unroll
    for (int s = 1; s < K; ++s) {
      if (pos >= s) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(hist[s][e], taps[e][K - 1 - s], acc[e]);
      }
    }
#pragma unroll
    for (int s = K - 1; s > 1; --s)
#pragma unroll
      for (int e = 0; e < 8; ++e) hist[s][e] = hist[s - 1][e];
    if constexpr (K > 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e) hist[1][e] = cur[e];
    }
    uint32_t packed[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) packed[e] = pack_bf16x2(silu(acc[2 * e]), silu(acc[2 * e + 1]));
    *reinterpret_cast<uint4*>(out + t * ldo + c0) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// ------------------------------------------------------------------------------------------------ delta rule

constexpr int CHUNK = 16;  // tokens staged in shared memory per step of the walk
constexpr int ORDER_MAX = 1024;  // packs of up to this many sequences walk their longest sequences first

template <int DK, int DV>
struct Cfg {
  static constexpr int TPC = 2;           // threads per value column, each owning DK / TPC of its rows
  static constexpr int THREADS = TPC * DV;
  static constexpr int ROWS = DK / TPC;   // state rows per thread
  static constexpr int SEG = ROWS + 4;    // a staged q / k row: TPC segments 16 bytes apart (no bank conflicts)
  static constexpr int KSTRIDE = TPC * SEG;
  // shared memory: q and k rows (float32), v rows (float32), then g and beta
  static constexpr int SMEM = (2 * CHUNK * KSTRIDE + CHUNK * DV + 2 * CHUNK) * 4;
};

struct Args {
  const __nv_bfloat16* qkv;  // rows: [q nk*dk | k nk*dk | v nv*dv]
  int64_t ldqkv;
  const __nv_bfloat16* ab;  // rows: [b nv | a nv]
  int64_t ldab;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const int32_t* cu;
  int num_seqs;
  int nk, nv;
  __nv_bfloat16* out;
  int64_t ldo;
};

KD_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The sum over the TPC adjacent lanes that share a value column.
template <int TPC>
KD_DEVICE float column_sum(float v) {
#pragma unroll
  for (int o = 1; o < TPC; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

KD_DEVICE float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

template <int DK, int DV>
__global__ void __launch_bounds__(Cfg<DK, DV>::THREADS) delta_rule_kernel(Args a) {
  using C = Cfg<DK, DV>;
  extern __shared__ float sm[];
  float* q_s = sm;                              // [CHUNK][KSTRIDE]
  float* k_s = q_s + CHUNK * C::KSTRIDE;        // [CHUNK][KSTRIDE]
  float* v_s = k_s + CHUNK * C::KSTRIDE;        // [CHUNK][DV]
  float* g_s = v_s + CHUNK * DV;                // [CHUNK]: decay factor exp(g)
  float* b_s = g_s + CHUNK;                     // [CHUNK]: beta
  // Longest sequences first: CTA b takes value head b % Hv of the (b / Hv)-th longest sequence, so the long walks
  // start in the first wave and the short ones fill in behind them. The order is computed here from the device
  // bounds (every CTA the same way; packs of more than ORDER_MAX sequences keep their order).
  __shared__ int order_s[ORDER_MAX];
  const int rank = blockIdx.x / a.nv;
  const int head = blockIdx.x % a.nv;           // value head
  int seq = rank;
  if (a.num_seqs <= ORDER_MAX) {
    for (int s0 = threadIdx.x; s0 < a.num_seqs; s0 += blockDim.x) {
      const int len = a.cu[s0 + 1] - a.cu[s0];
      int before = 0;
      for (int s1 = 0; s1 < a.num_seqs; ++s1) {
        const int l1 = a.cu[s1 + 1] - a.cu[s1];
        before += (l1 > len) || (l1 == len && s1 < s0);
      }
      order_s[before] = s0;
    }
    __syncthreads();
    seq = order_s[rank];
  }
  const int khead = head / (a.nv / a.nk);       // its key head (repeat_interleave)
  const int64_t t0 = a.cu[seq], t1 = a.cu[seq + 1];
  const int tid = threadIdx.x;
  const int col = tid / C::TPC;                 // value column
  const int part = tid % C::TPC;                // rows [part * ROWS, part * ROWS + ROWS)
  const int warp = tid / 32, lane = tid & 31;
  constexpr int WARPS = C::THREADS / 32;
  const float qscale = rsqrtf((float)DK);
  const float decay_a = -expf(__bfloat162float(a.a_log[head]));
  const float dt_bias = __bfloat162float(a.dt_bias[head]);
  const int64_t kd = (int64_t)a.nk * DK;

  float2 S[C::ROWS / 2];  // this thread's rows of its column of S / gamma, in pairs
#pragma unroll
  for (int i = 0; i < C::ROWS / 2; ++i) S[i] = make_float2(0.f, 0.f);
  float gamma = 1.f, inv_gamma = 1.f;

  // The next chunk's rows are fetched into registers while the current chunk is walked, then normalized into
  // shared memory: one warp per token row (q and k L2-normalized with eps 1e-6, q scaled by dk^-1/2).
  constexpr int PER_WARP = CHUNK / WARPS;
  static_assert(CHUNK % WARPS == 0, "whole rows per warp");
  __nv_bfloat16 rq[PER_WARP][DK / 32], rk[PER_WARP][DK / 32], rv[PER_WARP][DV / 32];
  float ra[PER_WARP], rb[PER_WARP];
  auto fetch = [&](int64_t base, int cnt) {
#pragma unroll
    for (int i = 0; i < PER_WARP; ++i) {
      const int r = warp + i * WARPS;
      if (r >= cnt) break;
      const __nv_bfloat16* row = a.qkv + (base + r) * a.ldqkv;
#pragma unroll
      for (int e = 0; e < DK / 32; ++e) {
        rq[i][e] = row[(int64_t)khead * DK + lane + 32 * e];
        rk[i][e] = row[kd + (int64_t)khead * DK + lane + 32 * e];
      }
#pragma unroll
      for (int e = 0; e < DV / 32; ++e) rv[i][e] = row[2 * kd + (int64_t)head * DV + lane + 32 * e];
      if (lane == 0) {
        const __nv_bfloat16* abr = a.ab + (base + r) * a.ldab;
        rb[i] = __bfloat162float(abr[head]);
        ra[i] = __bfloat162float(abr[a.nv + head]);
      }
    }
  };
  if (t1 > t0) fetch(t0, t1 - t0 < CHUNK ? (int)(t1 - t0) : CHUNK);
  for (int64_t c0 = t0; c0 < t1; c0 += CHUNK) {
    const int n = t1 - c0 < CHUNK ? (int)(t1 - c0) : CHUNK;
    __syncthreads();  // the previous chunk's rows have been read
#pragma unroll
    for (int i = 0; i < PER_WARP; ++i) {
      const int r = warp + i * WARPS;
      if (r >= n) break;
      float qv[DK / 32], kv[DK / 32], sq = 0.f, sk = 0.f;
#pragma unroll
      for (int e = 0; e < DK / 32; ++e) {
        qv[e] = __bfloat162float(rq[i][e]);
        kv[e] = __bfloat162float(rk[i][e]);
        sq += qv[e] * qv[e];
        sk += kv[e] * kv[e];
      }
      const float iq = rsqrtf(warp_sum(sq) + 1e-6f) * qscale;
      const float ik = rsqrtf(warp_sum(sk) + 1e-6f);
#pragma unroll
      for (int e = 0; e < DK / 32; ++e) {
        const int d = lane + 32 * e;
        const int at = (d / C::ROWS) * C::SEG + d % C::ROWS;  // each thread's segment sits 16 bytes further
        q_s[r * C::KSTRIDE + at] = qv[e] * iq;
        k_s[r * C::KSTRIDE + at] = kv[e] * ik;
      }
#pragma unroll
      for (int e = 0; e < DV / 32; ++e) v_s[r * DV + lane + 32 * e] = __bfloat162float(rv[i][e]);
      if (lane == 0) {
        g_s[r] = expf(decay_a * softplus(ra[i] + dt_bias));            // exp(g), g = -exp(A_log) softplus(a + dt)
        b_s[r] = bf16_round(1.0f / (1.0f + expf(-rb[i])));             // beta = sigmoid(b), a bf16 tensor op
      }
    }
    __syncthreads();
    if (c0 + CHUNK < t1) fetch(c0 + CHUNK, t1 - c0 - CHUNK < CHUNK ? (int)(t1 - c0 - CHUNK) : CHUNK);
    // the walk: S = alpha S + k d^T with d = (v - alpha S^T k) beta, then o = S^T q. The decay stays factored out:
    // the registers hold S / gamma with gamma the product of the decays since the last renormalization, folded back
    // into the registers when it falls below 2^-60 (so 1 / gamma stays far from overflow), which saves the per-element
    // multiply by alpha at every token.
    for (int r = 0; r < n; ++r) {
      const float* kr = k_s + r * C::KSTRIDE + part * C::SEG;
      const float* qr = q_s + r * C::KSTRIDE + part * C::SEG;
      const float beta = b_s[r];
      gamma *= g_s[r];
      if (gamma < 0x1p-60f) {  // uniform over the CTA (one decay per head and token)
#pragma unroll
        for (int i = 0; i < C::ROWS / 2; ++i) S[i] = mul2(S[i], make_float2(gamma, gamma));
        gamma = 1.f;
      }
      inv_gamma = 1.0f / gamma;  // off the chain from S^T k to the update
      // paired float instructions: two state rows per fma (S^T k, the rank-1 update and S^T q)
      float2 kreg[C::ROWS / 2];
      float2 acc[2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
      for (int i = 0; i < C::ROWS; i += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kr + i);
        kreg[i / 2] = make_float2(k4.x, k4.y);
        kreg[i / 2 + 1] = make_float2(k4.z, k4.w);
        acc[0] = fma2(S[i / 2], kreg[i / 2], acc[0]);
        acc[1] = fma2(S[i / 2 + 1], kreg[i / 2 + 1], acc[1]);
      }
      const float kvm = column_sum<C::TPC>((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y));
      const float delta = (v_s[r * DV + col] - gamma * kvm) * beta;  // S^T k of the decayed state = gamma (S/gamma)^T k
      const float dscaled = delta * inv_gamma;
      const float2 d2 = make_float2(dscaled, dscaled);
      float2 o[2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
      for (int i = 0; i < C::ROWS; i += 4) {
        const float4 q4 = *reinterpret_cast<const float4*>(qr + i);
        const float2 s0 = fma2(kreg[i / 2], d2, S[i / 2]);
        const float2 s1 = fma2(kreg[i / 2 + 1], d2, S[i / 2 + 1]);
        S[i / 2] = s0;
        S[i / 2 + 1] = s1;
        o[0] = fma2(s0, make_float2(q4.x, q4.y), o[0]);
        o[1] = fma2(s1, make_float2(q4.z, q4.w), o[1]);
      }
      const float ov = column_sum<C::TPC>((o[0].x + o[0].y) + (o[1].x + o[1].y));
      if (part == 0) a.out[(c0 + r) * a.ldo + (int64_t)head * DV + col] = __float2bfloat16_rn(gamma * ov);
    }
  }
}

template <int DK, int DV>
int launch_delta(const Args& a, int num_seqs, cudaStream_t stream) {
  using C = Cfg<DK, DV>;
  auto kernel = delta_rule_kernel<DK, DV>;
  if (C::SMEM > 48 * 1024) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return KD_ERR_ARGUMENT;
    if (!configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
      if (e != cudaSuccess) return record_cuda_error(e, "gated_delta_rule: cudaFuncSetAttribute");
      configured[dev] = true;
    }
  }
  dim3 grid((unsigned)(num_seqs * a.nv));
  kernel<<<grid, C::THREADS, C::SMEM, stream>>>(a);
  return record_cuda_error(cudaGetLastError(), "gated_delta_rule: launch");
}

// ------------------------------------------------------------------------------------------------ gated norm

// One warp per (token, head): out = bf16(bf16(w * bf16(x rsqrt(mean(x^2) + eps))) * silu(float(z))).
template <int DV>
__global__ void gated_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                  const __nv_bfloat16* __restrict__ z, int64_t ldz,
                                  const __nv_bfloat16* __restrict__ w, int64_t T, int heads, float eps,
                                  __nv_bfloat16* __restrict__ out, int64_t ldo) {
  constexpr int PER = DV / 32;
  const int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (item >= T * heads) return;
  const int64_t t = item / heads;
  const int h = (int)(item % heads);
  const __nv_bfloat16* xr = x + t * ldx + (int64_t)h * DV;
  const __nv_bfloat16* zr = z + t * ldz + (int64_t)h * DV;
  float v[PER], ss = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    v[e] = __bfloat162float(xr[lane + 32 * e]);
    ss += v[e] * v[e];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)DV + eps);
  __nv_bfloat16* orow = out + t * ldo + (int64_t)h * DV;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int d = lane + 32 * e;
    const float normed = bf16_round(v[e] * inv);
    const float weighted = bf16_round(__bfloat162float(w[d]) * normed);
    orow[d] = __float2bfloat16_rn(weighted * silu(__bfloat162float(zr[d])));
  }
}

}  // namespace dn
}  // namespace kd

using namespace kd;

extern "C" int kd_conv_silu(const void* x, int64_t ldx, int64_t T, int C, const void* weight, int K,
                            const int64_t* seqpos, void* out, int64_t ldo, cudaStream_t stream) {
  if (T < 0 || C <= 0 || C % 8 || K < 1 || K > 4) return set_error(KD_ERR_ARGUMENT, "conv_silu: bad sizes");
  if (reinterpret_cast<uintptr_t>(weight) & 15) return set_error(KD_ERR_ARGUMENT, "conv_silu: 16-byte aligned taps");
  if (T == 0) return KD_OK;
  if (!x || !weight || !seqpos || !out) return set_error(KD_ERR_ARGUMENT, "conv_silu: null pointer");
  if (ldx < C || ldo < C || ldx % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(KD_ERR_ARGUMENT, "conv_silu: rows must be 16-byte aligned and at least C wide");
  const auto* xi = static_cast<const __nv_bfloat16*>(x);
  const auto* wi = static_cast<const __nv_bfloat16*>(weight);
  auto* oi = static_cast<__nv_bfloat16*>(out);
  const int64_t n = (T + dn::ROWS_PER_THREAD - 1) / dn::ROWS_PER_THREAD * (C / 8);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  switch (K) {
    case 1: dn::conv_silu_kernel<1><<<blocks, 256, 0, stream>>>(xi, ldx, T, C, wi, seqpos, oi, ldo); break;
    case 2: dn::conv_silu_kernel<2><<<blocks, 256, 0, stream>>>(xi, ldx, T, C, wi, seqpos, oi, ldo); break;
    case 3: dn::conv_silu_kernel<3><<<blocks, 256, 0, stream>>>(xi, ldx, T, C, wi, seqpos, oi, ldo); break;
    default: dn::conv_silu_kernel<4><<<blocks, 256, 0, stream>>>(xi, ldx, T, C, wi, seqpos, oi, ldo); break;
  }
  return record_cuda_error(cudaGetLastError(), "conv_silu: launch");
}

extern "C" int kd_gated_delta_rule(const void* qkv, int64_t ldqkv, const void* ab, int64_t ldab, const void* a_log,
                                   const void* dt_bias, const int32_t* cu, int num_seqs, int64_t T, int num_k_heads,
                                   int num_v_heads, int head_k_dim, int head_v_dim, void* out, int64_t ldo,
                                   cudaStream_t stream) {
  if (num_seqs < 0 || T < 0) return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: negative sizes");
  if (num_seqs == 0 || T == 0) return KD_OK;
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: value heads must be a multiple of key heads");
  if (!qkv || !ab || !a_log || !dt_bias || !cu || !out) return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: null");
  const int64_t width = 2LL * num_k_heads * head_k_dim + (int64_t)num_v_heads * head_v_dim;
  if (ldqkv < width || ldab < 2LL * num_v_heads || ldo < (int64_t)num_v_heads * head_v_dim)
    return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: row strides smaller than the rows");
  dn::Args a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldqkv = ldqkv;
  a.ab = static_cast<const __nv_bfloat16*>(ab);
  a.ldab = ldab;
  a.a_log = static_cast<const __nv_bfloat16*>(a_log);
  a.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  a.cu = cu;
  a.num_seqs = num_seqs;
  a.nk = num_k_heads;
  a.nv = num_v_heads;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  if (head_k_dim == 64 && head_v_dim == 64) return dn::launch_delta<64, 64>(a, num_seqs, stream);
  if (head_k_dim == 128 && head_v_dim == 128) return dn::launch_delta<128, 128>(a, num_seqs, stream);
  if (head_k_dim == 128 && head_v_dim == 64) return dn::launch_delta<128, 64>(a, num_seqs, stream);
  if (head_k_dim == 64 && head_v_dim == 128) return dn::launch_delta<64, 128>(a, num_seqs, stream);
  return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: head dims must be 64 or 128");
}

extern "C" int kd_gated_norm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* weight, int64_t T,
                             int heads, int head_dim, float eps, void* out, int64_t ldo, cudaStream_t stream) {
  if (T < 0 || heads <= 0) return set_error(KD_ERR_ARGUMENT, "gated_norm: bad sizes");
  if (T == 0) return KD_OK;
  if (!x || !z || !weight || !out) return set_error(KD_ERR_ARGUMENT, "gated_norm: null pointer");
  const int64_t width = (int64_t)heads * head_dim;
  if (ldx < width || ldz < width || ldo < width) return set_error(KD_ERR_ARGUMENT, "gated_norm: row strides");
  const auto* xi = static_cast<const __nv_bfloat16*>(x);
  const auto* zi = static_cast<const __nv_bfloat16*>(z);
  const auto* wi = static_cast<const __nv_bfloat16*>(weight);
  auto* oi = static_cast<__nv_bfloat16*>(out);
  const int64_t threads = T * heads * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (head_dim == 64)
    dn::gated_norm_kernel<64><<<blocks, 256, 0, stream>>>(xi, ldx, zi, ldz, wi, T, heads, eps, oi, ldo);
  else if (head_dim == 128)
    dn::gated_norm_kernel<128><<<blocks, 256, 0, stream>>>(xi, ldx, zi, ldz, wi, T, heads, eps, oi, ldo);
  else
    return set_error(KD_ERR_ARGUMENT, "gated_norm: head_dim must be 64 or 128");
  return record_cuda_error(cudaGetLastError(), "gated_norm: launch");
}
