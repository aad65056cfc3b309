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

// ------------------------------------------------------------------------------------------------ chunked form
//
// The gated delta rule in its chunked (WY) form on the tensor cores, for 128-dim key and value heads (Qwen3.5's), the
// form flash-linear-attention's chunk_gated_delta_rule evaluates. One CTA walks one (sequence, value head) chain chunk
// by chunk, 128 tokens a chunk (one token per thread and TMEM lane), the state S (dk x dv, float32) in tensor memory.
// Per chunk, with G the running sum of the log decays g from the chunk's start and beta the write strengths (tensor
// memory: two 128-column accumulators, the state, and the float32 columns of the triangular solve):
//   K K^T, Q K^T                       tcgen05, bf16 operands, fp32 in TMEM
//   A = strictly lower (beta_i (K K^T)_ij exp(G_i - G_j)),  P = (Q K^T)_ij exp(G_i - G_j) for j <= i
//   T = (I + A)^-1                     its two 64 x 64 diagonal blocks T_bd by forward substitution on the CUDA
//                                      cores (float32, a column per thread), then T = T_bd - T_bd L T_bd with L the
//                                      lower-left block of A, applied on the tensor cores
//   W = T diag(beta exp(G)) K,  U = T diag(beta) V         tcgen05
//   D = U - W S                        tcgen05 (W S), the difference in float32
//   O = diag(exp(G)) Q S + P D         tcgen05, both products into one accumulator
//   S = exp(G_last) S + (diag(exp(G_last - G)) K)^T D     the rescale in TMEM, then tcgen05 accumulating into S
// Queries and keys are L2-normalized (eps 1e-6) and the queries scaled by dk^-1/2 first, as in the recurrent form.
// Every phase is one MMA issue by thread 0 and a bounded wait on its completion by the whole CTA; on a wait that gives
// up the CTA records KD_DEVICE_TIMEOUT, frees its tensor memory and returns.
namespace ck {

// 2^x on the exponential unit (relative error ~2^-22), for the decay factors exp(G_i - G_j) <= 1.
KD_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int C = 128;                // tokens per chunk = MMA rows = TMEM lanes
constexpr int HD = 128;               // key and value head dim
constexpr int THREADS = 256;          // two threads per token row, each taking half of its columns
constexpr int TILE = C * HD * 2;      // a 128 x 128 bf16 tile: two 64-column halves
constexpr int HALF = C * 128;         // one half: 128 rows of 128 bytes (128-byte swizzle)
constexpr int A_FLOATS = 8320;        // the strictly lower A, each row padded to a multiple of 4 floats
constexpr int A_OFF = 6 * TILE;
constexpr int G_OFF = A_OFF + A_FLOATS * 4;
constexpr int MISC_OFF = G_OFF + C * 4;
constexpr int SMEM = MISC_OFF + 96 + 1024;  // + alignment of the tiles to 1024 bytes
static_assert(SMEM <= 227 * 1024, "shared memory budget");
// tiles: kn then P (K-major A) | qn then q~ (K-major A) | X_w = beta e^G kn (MN-major B) then W (K-major A) |
// X_u = beta v (MN-major B) then S (MN-major B) | k~ = e^(G_last - G) kn (MN-major A) | T (K-major A)
enum { R_KP = 0, R_Q = 1, R_XW = 2, R_XU = 3, R_KT = 4, R_T = 5 };
constexpr uint32_t ACC0 = 0, ACC1 = 128, SST = 256, TCOL = 384, TMEM_COLS = 512;

// First float of row j of the packed A: sum over r < j of r rounded up to a multiple of 4.
KD_DEVICE constexpr int a_row(int j) {
  const int n = j + 2, q = n >> 2, b = n & 3;
  return 4 * (2 * q * (q - 1) + q * (b + 1));
}

// Byte offset of 16-byte unit u (0..15, eight bf16 each) of row r in a 128 x 128 tile stored as a TMA load with
// 128-byte swizzling writes it (64-column halves of 128-byte rows, unit index XOR row % 8).
KD_DEVICE uint32_t unit_at(int r, int u) { return (u >> 3) * HALF + r * 128 + (((u & 7) ^ (r & 7)) << 4); }

KD_DEVICE constexpr uint32_t idesc(uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn << 15) | (b_mn << 16) | ((uint32_t)(HD >> 3) << 17) |
         ((uint32_t)(C >> 4) << 24);
}

// D (+)= A B^T over K = 128 in eight K = 16 steps; A and B each K-major (rows of 128-byte swizzled K) or MN-major
// (one row per K index, 64 M/N elements per 128 bytes, the second half 16 KB on).
KD_DEVICE void mma128(uint32_t d, uint32_t a, bool a_mn, uint32_t b, bool b_mn, bool accumulate, bool neg_a = false) {
  const uint32_t id = idesc(a_mn ? 1u : 0u, b_mn ? 1u : 0u) | (neg_a ? (1u << 13) : 0u);  // bit 13: negate A
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t ad = a_mn ? sw128_mnmajor_desc(a + kk * 2048, HALF) : sw128_kmajor_desc(a + (kk / 4) * HALF + (kk % 4) * 32);
    const uint64_t bd = b_mn ? sw128_mnmajor_desc(b + kk * 2048, HALF) : sw128_kmajor_desc(b + (kk / 4) * HALF + (kk % 4) * 32);
    mma_f16_ss(d, ad, bd, id, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// Half hf of row r of a tile (units 8 hf .. 8 hf + 7, 64 values) from its raw bf16 units times `s`, rounded to bf16.
KD_DEVICE void put_half(uint8_t* tile, int r, int hf, const uint4 (&raw)[8], float s) {
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      o[e] = pack_bf16x2(f.x * s, f.y * s);
    }
    *reinterpret_cast<uint4*>(tile + unit_at(r, 8 * hf + u)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// 32 accumulator columns [32 cc, 32 cc + 32) of this thread's row, as bf16 into units 4 cc .. 4 cc + 3 of row r.
KD_DEVICE void put_cols(uint8_t* tile, int r, int cc, const float* x) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = pack_bf16x2(x[8 * q + 2 * e], x[8 * q + 2 * e + 1]);
    *reinterpret_cast<uint4*>(tile + unit_at(r, 4 * cc + q)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    chunked_delta_kernel(const __grid_constant__ CUtensorMap map_qkv, Args a, int* status) {
  extern __shared__ uint8_t raw_smem[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* tile_kp = sm + R_KP * TILE;
  uint8_t* tile_q = sm + R_Q * TILE;
  uint8_t* tile_xw = sm + R_XW * TILE;
  uint8_t* tile_xu = sm + R_XU * TILE;
  uint8_t* tile_kt = sm + R_KT * TILE;
  uint8_t* tile_t = sm + R_T * TILE;
  float* apk = reinterpret_cast<float*>(sm + A_OFF);
  uint8_t* tile_d = sm + A_OFF;  // D reuses A's space once T is built
  float* g_s = reinterpret_cast<float*>(sm + G_OFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + MISC_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + MISC_OFF + 8);
  int* seq_s = reinterpret_cast<int*>(sm + MISC_OFF + 12);
  float* wtot = reinterpret_cast<float*>(sm + MISC_OFF + 16);  // [8]: per warp, the scan's partial sums
  uint64_t* load_bar = reinterpret_cast<uint64_t*>(sm + MISC_OFF + 48);
  float* red = apk;  // [2][256] before A is built: each thread's half-row sums of squares (k, q)

  // thread (row i, half hf): token row i of the chunk (its TMEM lane, in the warp's lane quarter) and the columns
  // [64 hf, 64 hf + 64) of every row-wise phase; the two halves' warps share the row's TMEM lane quarter
  const int tid = threadIdx.x, i = tid & (C - 1), hf = tid >> 7, warp = tid >> 5, lane = tid & 31;
  // the chain: value head `head` of the `rank`-th longest sequence (ties in pack order), so long chains start first
  const int rank = blockIdx.x / a.nv, head = blockIdx.x % a.nv;
  if (tid == 0) {
    *seq_s = rank;
    mbar_init(bar, 1);
    mbar_init(load_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&map_qkv);
  }
  __syncthreads();
  for (int s0 = tid; s0 < a.num_seqs; s0 += THREADS) {
    const int len = a.cu[s0 + 1] - a.cu[s0];
    int before = 0;
    for (int s1 = 0; s1 < a.num_seqs; ++s1) {
      const int l1 = a.cu[s1 + 1] - a.cu[s1];
      before += (l1 > len) || (l1 == len && s1 < s0);
    }
    if (before == rank) *seq_s = s0;
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const int seq = *seq_s;
  const int64_t t0 = a.cu[seq], t1 = a.cu[seq + 1];
  const int khead = head / (a.nv / a.nk);
  const float qscale = rsqrtf((float)HD);
  const float decay_a = -expf(__bfloat162float(a.a_log[head]));
  const float dt_bias = __bfloat162float(a.dt_bias[head]);
  const int64_t kd = (int64_t)a.nk * HD;
  const uint32_t s_kp = smem_u32(tile_kp), s_q = smem_u32(tile_q), s_xw = smem_u32(tile_xw),
                 s_xu = smem_u32(tile_xu), s_kt = smem_u32(tile_kt), s_t = smem_u32(tile_t),
                 s_d = smem_u32(tile_d);
  uint32_t phase = 0, load_phase = 0;
  bool ok = true;
  // the raw k, q and v rows of the chunk at c0: k into kn's tile, q into qn's, v into X_u's (128-row boxes of 64
  // columns; rows past the pack read as zero, rows of the next sequence are overwritten by the threads past n)
  auto load_chunk = [&](int64_t c0) {
    mbar_arrive_expect_tx(load_bar, 3 * TILE);
    const int y = (int)c0;
    for (int h = 0; h < 2; ++h) {
      tma_load_2d(&map_qkv, load_bar, tile_kp + h * HALF, (int)(kd + (int64_t)khead * HD) + 64 * h, y);
      tma_load_2d(&map_qkv, load_bar, tile_q + h * HALF, khead * HD + 64 * h, y);
      tma_load_2d(&map_qkv, load_bar, tile_xu + h * HALF, (int)(2 * kd + (int64_t)head * HD) + 64 * h, y);
    }
  };
  // one MMA group's completion, agreed by the whole CTA (a wait that gives up ends every thread's walk together)
  auto wait_mma = [&]() -> bool {
    bool mine = mbar_wait(bar, phase, status);
    phase ^= 1u;
    tc_fence_after();
    return __syncthreads_and(mine) != 0;
  };
  {  // S = 0
    uint32_t z[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) z[e] = 0u;
#pragma unroll
    for (int cc = 2 * hf; cc < 2 * hf + 2; ++cc) tmem_st32(lane_base + SST + 32 * cc, z);
    tmem_st_wait();
  }
  if (tid == 0 && t0 < t1) load_chunk(t0);
  // this row's b and a inputs (write strength, decay) of the next chunk, fetched a chunk ahead
  float next_b = 0.f, next_a = 0.f;
  auto fetch_ab = [&](int64_t c0) {
    if (c0 + i < t1) {
      const __nv_bfloat16* abr = a.ab + (c0 + i) * a.ldab;
      next_b = __bfloat162float(abr[head]);
      next_a = __bfloat162float(abr[a.nv + head]);
    }
  };
  fetch_ab(t0);

  for (int64_t c0 = t0; c0 < t1 && ok; c0 += C) {
    const int n = t1 - c0 < C ? (int)(t1 - c0) : C;
    const bool live = i < n;
    // ---------------------------------------------------------------- this row's decay, write strength, q, k, v
    float g = 0.f, beta = 0.f;
    if (live) {
      beta = bf16_round(1.0f / (1.0f + expf(-next_b)));
      g = decay_a * softplus(next_a + dt_bias);
    }
    float gi = g;  // inclusive running sum over the chunk's rows
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, gi, o);
      if (lane >= o) gi += y;
    }
    if (lane == 31) wtot[warp] = gi;
    __syncthreads();
    for (int w2 = 4 * hf; w2 < warp; ++w2) gi += wtot[w2];
    if (hf == 0) g_s[i] = gi;
    __syncthreads();
    const float g_last = g_s[n - 1];
    const float e_g = live ? expf(gi) : 0.f, e_tail = live ? expf(g_last - gi) : 0.f;
    {
      const bool loaded = mbar_wait(load_bar, load_phase, status);
      load_phase ^= 1u;
      if (!(ok = __syncthreads_and(loaded) != 0)) break;
      if (tid == 0 && c0 + C < t1) {  // the next chunk's rows into L2 now: its loads are issued only at this chunk's end
        for (int h = 0; h < 2; ++h) {
          tma_prefetch_l2(&map_qkv, (int)(kd + (int64_t)khead * HD) + 64 * h, (int)(c0 + C));
          tma_prefetch_l2(&map_qkv, khead * HD + 64 * h, (int)(c0 + C));
          tma_prefetch_l2(&map_qkv, (int)(2 * kd + (int64_t)head * HD) + 64 * h, (int)(c0 + C));
        }
      }
      uint4 rk[8], rq[8];
      auto take = [&](uint8_t* tile, uint4 (&r)[8]) -> float {  // this thread's half of the row (zeros past n)
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          r[u] = live ? *reinterpret_cast<const uint4*>(tile + unit_at(i, 8 * hf + u)) : make_uint4(0, 0, 0, 0);
          const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_bf16x2(w[e]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
        return ss;
      };
      red[tid] = take(tile_kp, rk);
      red[THREADS + tid] = take(tile_q, rq);
      __syncthreads();
      // the row's sums: the first half's then the second's, in the same order for both threads of the row
      const float ik = rsqrtf((red[i] + red[C + i]) + 1e-6f);
      const float iq = rsqrtf((red[THREADS + i] + red[THREADS + C + i]) + 1e-6f) * qscale;
      put_half(tile_kp, i, hf, rk, ik);
      put_half(tile_xw, i, hf, rk, ik * beta * e_g);
      put_half(tile_kt, i, hf, rk, ik * e_tail);
      put_half(tile_q, i, hf, rq, iq);
      take(tile_xu, rk);
      put_half(tile_xu, i, hf, rk, beta);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- K K^T -> ACC0, Q K^T -> ACC1
    if (tid == 0) {
      tc_fence_after();
      mma128(tmem + ACC0, s_kp, false, s_kp, false, false);
      mma128(tmem + ACC1, s_q, false, s_kp, false, false);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {  // this row of A (packed, float32) and of P (bf16 over kn's tile); q~ = e^G qn in place
      float* arow = apk + a_row(i);
#pragma unroll 1
      for (int cc = 2 * hf; cc < 2 * hf + 2; ++cc) {
        uint32_t kk[32], qk[32];
        tmem_ld32(lane_base + ACC0 + 32 * cc, kk);
        tmem_ld32(lane_base + ACC1 + 32 * cc, qk);
        tmem_ld_wait_regs(kk, qk);
        float p[32], av[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = 32 * cc + e;
          const float dec = (j <= i && live) ? fast_exp2((gi - g_s[j]) * 1.4426950408889634f) : 0.f;
          av[e] = j < i ? beta * __uint_as_float(kk[e]) * dec : 0.f;
          p[e] = __uint_as_float(qk[e]) * dec;
        }
        put_cols(tile_kp, i, cc, p);
#pragma unroll
        for (int e = 0; e < 32; e += 4)  // the row's entries j < i and its padding to a multiple of 4, 16 bytes at a time
          if (32 * cc + e < i)
            *reinterpret_cast<float4*>(arow + 32 * cc + e) = make_float4(av[e], av[e + 1], av[e + 2], av[e + 3]);
      }
#pragma unroll
      for (int u = 8 * hf; u < 8 * hf + 8; ++u) {
        uint4* at = reinterpret_cast<uint4*>(tile_q + unit_at(i, u));
        const uint4 v = *at;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(w[e]);
          o[e] = pack_bf16x2(f.x * e_g, f.y * e_g);
        }
        *at = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();
    {  // T_bd = blockdiag((I + A_11)^-1, (I + A_22)^-1) over the two 64-row halves, by forward substitution: this
       // thread's column c = i of its half, by blocks of 16 rows (first every earlier block's contribution to the
       // block's rows, 16 independent sums, then the block's own rows in order). The column's float32 values live in
       // this thread's own lane of tensor memory (columns TCOL + row), read 16 at a time, so the loops stay rolled.
      const uint32_t tcol = lane_base + TCOL;
      const int base = i & ~63;  // the half this column belongs to
      if (hf == 0) {  // the column solves run on the first half's threads, a column each
#pragma unroll 1
      for (int b = 0; b < 4; ++b) {
        const int row0 = base + 16 * b;
        float acc[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] = (row0 + r == i) ? 1.f : 0.f;
#pragma unroll 1
        for (int m0 = base; m0 < row0; m0 += 16) {
          uint32_t tv[16];
          tmem_ld16(tcol + m0, tv);
          tmem_ld_wait_regs(tv);
#pragma unroll
          for (int r = 0; r < 16; ++r) {
            const float* arow = apk + a_row(row0 + r) + m0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 av = *reinterpret_cast<const float4*>(arow + 4 * q);
              acc[r] = fmaf(-av.x, __uint_as_float(tv[4 * q]), acc[r]);
              acc[r] = fmaf(-av.y, __uint_as_float(tv[4 * q + 1]), acc[r]);
              acc[r] = fmaf(-av.z, __uint_as_float(tv[4 * q + 2]), acc[r]);
              acc[r] = fmaf(-av.w, __uint_as_float(tv[4 * q + 3]), acc[r]);
            }
          }
        }
        uint32_t tb[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float* arow = apk + a_row(row0 + r) + row0;
          float v = acc[r];
#pragma unroll
          for (int r2 = 0; r2 < r; ++r2) v = fmaf(-arow[r2], __uint_as_float(tb[r2]), v);
          tb[r] = __float_as_uint(v);
        }
        tmem_st16(tcol + row0, tb);
        tmem_st_wait();
      }
      // column c of T_bd (bf16) into the K-major A tile: its half's 64 rows, zeros in the other half's rows
      __nv_bfloat16* col = reinterpret_cast<__nv_bfloat16*>(tile_t);
#pragma unroll 1
      for (int j0 = 0; j0 < C; j0 += 32) {
        uint32_t tv[32];
        const bool mine = (j0 & ~63) == base;
        if (mine) {
          tmem_ld32(tcol + j0, tv);
          tmem_ld_wait_regs(tv);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e)
          col[(unit_at(j0 + e, i >> 3) >> 1) + (i & 7)] = __float2bfloat16_rn(mine ? __uint_as_float(tv[e]) : 0.f);
      }
      }
      // L = A's lower-left 64 x 64 block (rows 64.., columns ..63) as a bf16 K-major tile over A's space, zeros
      // elsewhere: every thread reads its 32 columns of its row first (half hf: columns 32 hf ..), then all write
      float lrow[32];
#pragma unroll
      for (int m = 0; m < 32; ++m) lrow[m] = i >= 64 ? apk[a_row(i) + 32 * hf + m] : 0.f;
      __syncthreads();
      put_cols(tile_d, i, hf, lrow);
      float zero[32];
#pragma unroll
      for (int m = 0; m < 32; ++m) zero[m] = 0.f;
      put_cols(tile_d, i, 2 + hf, zero);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- W = T X_w -> ACC0, U = T X_u -> ACC1
    // with T = T_bd - T_bd L T_bd ((T_bd L)^2 = 0: L has only the lower-left block): Z = T_bd X, Y = L Z, T X = Z - T_bd Y
    if (tid == 0) {
      tc_fence_after();
      mma128(tmem + ACC0, s_t, false, s_xw, true, false);
      mma128(tmem + ACC1, s_t, false, s_xu, true, false);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {  // Z_w, Z_u -> bf16 over X_w, X_u (MN-major B, row = token): four loads in flight, one wait
      uint32_t w0[32], w1[32], u0[32], u1[32];
      tmem_ld32(lane_base + ACC0 + 64 * hf, w0);
      tmem_ld32(lane_base + ACC0 + 64 * hf + 32, w1);
      tmem_ld32(lane_base + ACC1 + 64 * hf, u0);
      tmem_ld32(lane_base + ACC1 + 64 * hf + 32, u1);
      tmem_ld_wait_regs(w0, w1);
      tmem_ld_wait_regs(u0, u1);  // no load left to wait for: ties u0, u1 to the wait above
      put_cols(tile_xw, i, 2 * hf, reinterpret_cast<const float*>(w0));
      put_cols(tile_xw, i, 2 * hf + 1, reinterpret_cast<const float*>(w1));
      put_cols(tile_xu, i, 2 * hf, reinterpret_cast<const float*>(u0));
      put_cols(tile_xu, i, 2 * hf + 1, reinterpret_cast<const float*>(u1));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // Y_w = L Z_w -> TCOL
      tc_fence_after();
      mma128(tmem + TCOL, s_d, false, s_xw, true, false);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {  // Y_w -> bf16 over Z_w (this thread's two 32-column pieces, both loads in flight)
      uint32_t y0[32], y1[32];
      tmem_ld32(lane_base + TCOL + 64 * hf, y0);
      tmem_ld32(lane_base + TCOL + 64 * hf + 32, y1);
      tmem_ld_wait_regs(y0, y1);
      put_cols(tile_xw, i, 2 * hf, reinterpret_cast<const float*>(y0));
      put_cols(tile_xw, i, 2 * hf + 1, reinterpret_cast<const float*>(y1));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // W = Z_w - T_bd Y_w in ACC0; Y_u = L Z_u -> TCOL
      tc_fence_after();
      mma128(tmem + ACC0, s_t, false, s_xw, true, true, true);
      mma128(tmem + TCOL, s_d, false, s_xu, true, false);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {  // Y_u -> bf16 over Z_u; W row -> bf16 (K-major A) over Y_w: four loads in flight, one wait
      uint32_t y0[32], y1[32], w0[32], w1[32];
      tmem_ld32(lane_base + TCOL + 64 * hf, y0);
      tmem_ld32(lane_base + TCOL + 64 * hf + 32, y1);
      tmem_ld32(lane_base + ACC0 + 64 * hf, w0);
      tmem_ld32(lane_base + ACC0 + 64 * hf + 32, w1);
      tmem_ld_wait_regs(y0, y1);
      tmem_ld_wait_regs(w0, w1);  // no load left to wait for: ties w0, w1 to the wait above
      put_cols(tile_xu, i, 2 * hf, reinterpret_cast<const float*>(y0));
      put_cols(tile_xu, i, 2 * hf + 1, reinterpret_cast<const float*>(y1));
      put_cols(tile_xw, i, 2 * hf, reinterpret_cast<const float*>(w0));
      put_cols(tile_xw, i, 2 * hf + 1, reinterpret_cast<const float*>(w1));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // U = Z_u - T_bd Y_u in ACC1
      tc_fence_after();
      mma128(tmem + ACC1, s_t, false, s_xu, true, true, true);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {  // S row (lane = key dim) -> bf16 (MN-major B) over Y_u
      uint32_t s0[32], s1[32];
      tmem_ld32(lane_base + SST + 64 * hf, s0);
      tmem_ld32(lane_base + SST + 64 * hf + 32, s1);
      tmem_ld_wait_regs(s0, s1);
      put_cols(tile_xu, i, 2 * hf, reinterpret_cast<const float*>(s0));
      put_cols(tile_xu, i, 2 * hf + 1, reinterpret_cast<const float*>(s1));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- X = W S -> ACC0
    if (tid == 0) {
      tc_fence_after();
      mma128(tmem + ACC0, s_xw, false, s_xu, true, false);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    {
      const float gamma = expf(g_last);
      {  // D = U - W S -> bf16 (MN-major B, row = token): four loads in flight, one wait
        uint32_t u0[32], u1[32], x0[32], x1[32];
        tmem_ld32(lane_base + ACC1 + 64 * hf, u0);
        tmem_ld32(lane_base + ACC1 + 64 * hf + 32, u1);
        tmem_ld32(lane_base + ACC0 + 64 * hf, x0);
        tmem_ld32(lane_base + ACC0 + 64 * hf + 32, x1);
        tmem_ld_wait_regs(u0, u1);
        tmem_ld_wait_regs(x0, x1);  // no load left to wait for: ties x0, x1 to the wait above
        float d[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = __uint_as_float(u0[e]) - __uint_as_float(x0[e]);
        put_cols(tile_d, i, 2 * hf, d);
#pragma unroll
        for (int e = 0; e < 32; ++e) d[e] = __uint_as_float(u1[e]) - __uint_as_float(x1[e]);
        put_cols(tile_d, i, 2 * hf + 1, d);
      }
      {  // S = gamma S, row by row in place
        uint32_t s0[32], s1[32];
        tmem_ld32(lane_base + SST + 64 * hf, s0);
        tmem_ld32(lane_base + SST + 64 * hf + 32, s1);
        tmem_ld_wait_regs(s0, s1);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          s0[e] = __float_as_uint(__uint_as_float(s0[e]) * gamma);
          s1[e] = __float_as_uint(__uint_as_float(s1[e]) * gamma);
        }
        tmem_st32(lane_base + SST + 64 * hf, s0);
        tmem_st32(lane_base + SST + 64 * hf + 32, s1);
      }
      tmem_st_wait();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- O = q~ S + P D -> ACC0, S += k~^T D
    if (tid == 0) {
      tc_fence_after();
      mma128(tmem + ACC0, s_q, false, s_xu, true, false);
      mma128(tmem + ACC0, s_kp, false, s_d, true, true);
      mma128(tmem + SST, s_kt, true, s_d, true, true);
      mma_commit(bar);
    }
    if (!(ok = wait_mma())) break;
    if (tid == 0 && c0 + C < t1) load_chunk(c0 + C);  // every tile the loads overwrite has been read
    fetch_ab(c0 + C);
    {  // this row's outputs: its two 32-column pieces (both loads in flight), bf16 rows of the head's slice
      uint32_t o0[32], o1[32];
      tmem_ld32(lane_base + ACC0 + 64 * hf, o0);
      tmem_ld32(lane_base + ACC0 + 64 * hf + 32, o1);
      tmem_ld_wait_regs(o0, o1);
      if (live) {
        __nv_bfloat16* orow = a.out + (c0 + i) * a.ldo + (int64_t)head * HD + 64 * hf;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* o = q < 4 ? o0 + 8 * q : o1 + 8 * (q - 4);
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) pk[e] = pack_bf16x2(__uint_as_float(o[2 * e]), __uint_as_float(o[2 * e + 1]));
          *reinterpret_cast<uint4*>(orow + 8 * q) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

int launch(const Args& a, int num_seqs, int64_t T, int* status, cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KD_ERR_ARGUMENT;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(chunked_delta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return record_cuda_error(e, "gated_delta_rule: cudaFuncSetAttribute");
    configured[dev] = true;
  }
  CUtensorMap map;
  const int64_t width = 2LL * a.nk * HD + (int64_t)a.nv * HD;
  int rc = make_tma_2d(&map, a.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)width, (uint64_t)T,
                       (uint64_t)a.ldqkv, 64, C, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  chunked_delta_kernel<<<(unsigned)(num_seqs * a.nv), THREADS, SMEM, stream>>>(map, a, status);
  return record_cuda_error(cudaGetLastError(), "gated_delta_rule: launch");
}

}  // namespace ck

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
                                   int* status, cudaStream_t stream) {
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
  if (head_k_dim == 128 && head_v_dim == 128) {
    if (!status) return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: status word required");
    if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) || ldqkv % 8 || ldo % 8)
      return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: qkv and out rows must be 16-byte aligned");
    if (T > 0x7fffffffLL) return set_error(KD_ERR_ARGUMENT, "gated_delta_rule: more than 2^31 rows");
    return dn::ck::launch(a, num_seqs, T, status, stream);  // the chunked tensor-core form
  }
  if (head_k_dim == 64 && head_v_dim == 64) return dn::launch_delta<64, 64>(a, num_seqs, stream);
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
