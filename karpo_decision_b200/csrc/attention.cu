// Varlen block-diagonal attention forward (GQA, causal / sliding window / bidirectional) on the 5th-generation tensor
// cores: S = Q K^T and O += P V are tcgen05.mma with the scores S, the probabilities P and the output O in tensor
// memory; Q, K and V tiles arrive by TMA (128-byte swizzle).
//
// Replaces torch varlen_attn / flash-attention calls: families/qwen/packed.py:123-124 (causal, scale hd^-0.5, GQA),
// families/gemma/sliding_attention.py:183-191 (window (W-1, 0), scale 1.0) and the global layers' causal attention
// (families/gemma/packed.py:196-220). The visibility rule is the varlen contract with end alignment (the reference's
// tests/test_gemma_blocks.py:28-43): query i of a sequence sees key j iff
//   i + (Lk - Lq) - left <= j <= i + (Lk - Lq) + right        (left/right < 0: unbounded).
// Sequence boundaries are read from device memory when the kernel runs, so a captured graph serves any pack
// composition with the same token count.
//
// One CTA per (128-query tile of one sequence, query head, value slice), two CTAs per SM where memory allows (head
// dim <= 128). Head dim 512 (Gemma 4's global layers) exceeds tensor memory for a whole output row block next to the
// scores, so its output is computed in two 256-wide value slices by separate CTAs, each forming the full scores
// (K and V single-buffered to fit the 128 KB query tile). 6 warps:
//   warp 0      TMA producer: the Q tile once, then K and V tiles through a ring (2 stages; 1 for head dim 512);
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM score buffers, then O += P_j V_j with
//               P_j read from TMEM (A operand, written over S_j) and V_j as an MN-major B operand from shared memory;
//   warps 2..5  softmax, one query row per thread (its TMEM lane): scores -> masked, scaled, exp2 against a running
//               maximum, bf16 probabilities stored back to TMEM. O is rescaled only when the row maximum grows by
//               more than 2^8 (the exponent base stays stale otherwise, which is exact: O and the row sum share it);
//               at the end they normalize O, apply the optional output gate and store bf16 rows.
#include "common.cuh"
#include "kd_internal.h"

namespace kd {
namespace fa {

template <int HD, int DV>
struct Cfg {
  static constexpr int BM = 128;                    // query rows per CTA = TMEM lanes
  static constexpr int BN = 64;                     // keys per tile
  static constexpr int CHUNKS = HD / 64;            // 128-byte swizzle chunks along the head dim (Q, K)
  static constexpr int V_CHUNKS = DV / 64;          // the same along this CTA's value slice (V, O)
  static constexpr int SLICES = HD / DV;            // value slices per head (CTAs along grid z)
  static constexpr int Q_CHUNK = BM * 128;          // bytes of one Q chunk (BM rows x 128 B)
  static constexpr int KV_CHUNK = BN * 128;         // bytes of one K or V chunk
  static constexpr int Q_BYTES = Q_CHUNK * CHUNKS;
  static constexpr int K_BYTES = KV_CHUNK * CHUNKS;
  static constexpr int V_BYTES = KV_CHUNK * V_CHUNKS;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int STAGES = HD <= 256 ? 2 : 1;
  static constexpr int SMEM = Q_BYTES + STAGES * STAGE_BYTES + 1024 + 256;
  // Tensor-memory columns (fp32): O [0, DV), then two score buffers of BN; the bf16 probabilities P_j overwrite the
  // first BN / 2 columns of their own score buffer once the softmax has read it.
  static constexpr int O_COL = 0;
  static constexpr int S_COL = DV;
  static constexpr int TMEM_COLS = DV + 2 * BN <= 256 ? 256 : 512;
  // Two CTAs per SM (their softmax and MMA phases interleave) when shared and tensor memory allow it.
  static constexpr int CTAS_PER_SM = (2 * SMEM <= 227 * 1024 && 2 * TMEM_COLS <= 512) ? 2 : 1;
  static_assert(S_COL + 2 * BN <= TMEM_COLS, "tensor memory budget");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(DV <= 256 && HD % DV == 0, "value slices of at most 256 columns");
};

struct Args {
  const __nv_bfloat16* gate;
  __nv_bfloat16* out;
  int64_t ldo, ldg;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_seqs;
  int hq, hkv;
  float scale_log2;  // softmax scale * log2(e)
  int left, right;
  int* status;
};

constexpr int THREADS = 192;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale O when the row maximum grows by more than 2^8


// 2^x with the hardware exponential (ex2.approx: relative error ~2^-22; the probabilities are rounded to bf16).
KD_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Paired float32 arithmetic (sm_100 f32x2 instructions: one issue slot for two lanes' worth of values).
KD_DEVICE float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}
KD_DEVICE float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
// max(a, b, c) in one instruction.
KD_DEVICE float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int HD, int DV>
__global__ void __launch_bounds__(THREADS, Cfg<HD, DV>::CTAS_PER_SM)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_g, Args a) {
  using C = Cfg<HD, DV>;
  constexpr int BM = C::BM, BN = C::BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;
  uint8_t* s_kv = smem + C::Q_BYTES;  // stage s: K at s * STAGE_BYTES, V right after
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::Q_BYTES + C::STAGES * C::STAGE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                  // [STAGES]
  uint64_t* v_full = k_full + C::STAGES;        // [STAGES]
  uint64_t* k_empty = v_full + C::STAGES;       // [STAGES]: released by the S = Q K^T that read the stage's K
  uint64_t* v_empty = k_empty + C::STAGES;      // [STAGES]: released by the O += P V that read its V
  uint64_t* s_full = v_empty + C::STAGES;       // [2]
  uint64_t* p_full = s_full + 2;                // [2]
  uint64_t* pv_done = p_full + 2;               // [2]
  uint64_t* q_free = pv_done + 2;              // the last S has read Q: its buffer takes the gate tile
  uint64_t* g_full = q_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g_full + 1);

  // ---- this CTA's (sequence, query tile), numbered sequence by sequence from the device bounds
  int tile = blockIdx.x;
  int seq = -1, qs = 0, lq = 0, lk = 0, q0 = 0, k0 = 0;
  for (int s = 0; s < a.num_seqs; ++s) {
    const int qa = a.cu_q[s], qb = a.cu_q[s + 1];
    const int n = (qb - qa + BM - 1) / BM;
    if (tile < n) {
      seq = s;
      q0 = qa;
      lq = qb - qa;
      k0 = a.cu_k[s];
      lk = a.cu_k[s + 1] - k0;
      qs = (n - 1 - tile) * BM;  // the last (most expensive when causal) tiles of a sequence first
      break;
    }
    tile -= n;
  }
  if (seq < 0) return;  // uniform across the CTA: nothing allocated yet
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int vcol = (int)blockIdx.z * DV;  // this CTA's value slice within the head
  const int off = lk - lq;  // end alignment of queries to keys
  const int qe = min(qs + BM, lq);
  int kmin = 0, kmax = lk - 1;
  if (a.left >= 0) kmin = max(0, qs + off - a.left);
  if (a.right >= 0) kmax = min(lk - 1, qe - 1 + off + a.right);
  const int first_tile = kmin / BN;
  const int n_tiles = kmax < kmin ? 0 : kmax / BN - first_tile + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(q_free, 1);
    mbar_init(g_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (n_tiles > 0 && elect_one()) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int c = 0; c < C::CHUNKS; ++c)
        tma_load_2d(&map_q, q_full, s_q + c * C::Q_CHUNK, head * HD + c * 64, q0 + qs);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        const int row = k0 + (first_tile + j) * BN;
        uint8_t* sk = s_kv + st * C::STAGE_BYTES;
        uint8_t* sv = sk + C::K_BYTES;
        if (!mbar_wait(&k_empty[st], ph ^ 1, a.status)) goto done;
        mbar_arrive_expect_tx(&k_full[st], C::K_BYTES);
        for (int c = 0; c < C::CHUNKS; ++c) tma_load_2d(&map_k, &k_full[st], sk + c * C::KV_CHUNK, kvh * HD + c * 64, row);
        if (!mbar_wait(&v_empty[st], ph ^ 1, a.status)) goto done;
        mbar_arrive_expect_tx(&v_full[st], C::V_BYTES);
        for (int c = 0; c < C::V_CHUNKS; ++c)
          tma_load_2d(&map_v, &v_full[st], sv + c * C::KV_CHUNK, kvh * HD + vcol + c * 64, row);
      }
      if (a.gate) {
        // Qwen's output gate tile, into the Q buffer once the last S = Q K^T has read it: the epilogue then reads
        // its row from shared memory instead of scattered global loads.
        if (!mbar_wait(q_free, 0, a.status)) goto done;
        mbar_arrive_expect_tx(g_full, C::V_CHUNKS * C::Q_CHUNK);
        for (int c = 0; c < C::V_CHUNKS; ++c)
          tma_load_2d(&map_g, g_full, s_q + c * C::Q_CHUNK, head * HD + vcol + c * 64, q0 + qs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (n_tiles > 0 && elect_one()) {
      constexpr uint32_t idesc_s = mma_idesc(1, BM, BN);          // bf16, K-major A and B
      constexpr uint32_t idesc_o = mma_idesc(1, BM, DV, 1);       // bf16, A from TMEM, MN-major B (V)
      const uint32_t sq = smem_u32(s_q);
      if (!mbar_wait(q_full, 0, a.status)) goto done;
      auto issue_s = [&](int j) -> bool {
        const int st = j % C::STAGES;
        if (!mbar_wait(&k_full[st], (j / C::STAGES) & 1, a.status)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(s_kv + st * C::STAGE_BYTES);
        const uint32_t d = tmem + C::S_COL + (j & 1) * BN;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int c = kk / 4, w = (kk % 4) * 32;
          mma_f16_ss(d, sw128_kmajor_desc(sq + c * C::Q_CHUNK + w), sw128_kmajor_desc(sk + c * C::KV_CHUNK + w),
                     idesc_s, kk > 0);
        }
        mma_commit(&k_empty[st]);  // the stage's K is free once these MMAs have read it
        mma_commit(&s_full[j & 1]);
        if (j == n_tiles - 1) mma_commit(q_free);  // Q is free once the last S has completed
        return true;
      };
      if (!issue_s(0)) goto done;
      for (int j = 0; j < n_tiles; ++j) {
        // S_{j+1} first, so the softmax of tile j+1 can start while P_j V_j runs. Its score buffer last held
        // P_{j-1}, read by P_{j-1} V_{j-1}: that product must have completed.
        if (j + 1 < n_tiles) {
          if (j >= 1 && !mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status)) goto done;
          if (!issue_s(j + 1)) goto done;
        }
        const int st = j % C::STAGES;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, a.status)) goto done;
        if (!mbar_wait(&v_full[st], (j / C::STAGES) & 1, a.status)) goto done;
        tc_fence_after();
        const uint32_t sv = smem_u32(s_kv + st * C::STAGE_BYTES + C::K_BYTES);
        const uint32_t p = tmem + C::S_COL + (j & 1) * BN;  // P_j over the first BN / 2 columns of S_j
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)  // 16 keys per instruction: 8 columns of bf16 pairs, 2 KB of V rows
          mma_f16_ts(tmem + C::O_COL, p + kk * 8, sw128_mnmajor_desc(sv + kk * 2048, C::KV_CHUNK), idesc_o,
                     (j | kk) != 0);
        mma_commit(&v_empty[st]);
        mma_commit(&pv_done[j & 1]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const int qi = qs + r + off;  // the row's position on the key axis
    float m_used = -INFINITY, l_sum = 0.f;  // running maximum (log2 units, possibly stale) and row sum
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, a.status)) goto done;
      tc_fence_after();
      const uint32_t s_addr = lane_base + C::S_COL + (j & 1) * BN;
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        uint32_t t[32];
        tmem_ld32(s_addr + c, t);
        tmem_ld_wait_regs(t);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[c + e] = __uint_as_float(t[e]);
      }
      const int n0 = (first_tile + j) * BN;
      // Only tiles that cross the causal diagonal, the window's left edge or the sequence end need a mask; the
      // condition is the same for every row of the CTA.
      const bool edge = (n0 + BN > lk) || (a.right >= 0 && n0 + BN - 1 > qs + off + a.right) ||
                        (a.left >= 0 && n0 < qe - 1 + off - a.left);
      if (edge) {
#pragma unroll
        for (int e = 0; e < BN; ++e) {
          const int key = n0 + e;
          bool ok = key < lk;
          if (a.right >= 0) ok = ok && key <= qi + a.right;
          if (a.left >= 0) ok = ok && key >= qi - a.left;
          if (!ok) sv[e] = -INFINITY;
        }
      }
      // row maximum over 8 independent chains (a single chain would serialize BN dependent max operations)
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = sv[e];
#pragma unroll
      for (int e = 8; e < BN; e += 2) mx[(e / 2) & 7] = max3(mx[(e / 2) & 7], sv[e], sv[e + 1]);
      const float mraw = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      const float mt = mraw * a.scale_log2;  // the scale is positive: max commutes with it
      const float m_new = fmaxf(m_used, mt);
      const bool need = m_new > m_used + RESCALE_THRESHOLD || (m_used == -INFINITY && m_new != -INFINITY);
      const float f = !need ? 1.f : (m_used == -INFINITY ? 0.f : fast_exp2(m_used - m_new));
      // tcgen05.ld/st are warp-collective: the warp rescales its O rows together (factor 1 where a row needs none).
      if (j > 0 && __any_sync(0xffffffffu, need && m_used != -INFINITY)) {
        // O holds P_{0..j-1} V: wait for the last product before rescaling it in place.
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status)) goto done;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DV; c += 32) {
          uint32_t t[32];
          tmem_ld32(lane_base + C::O_COL + c, t);
          tmem_ld_wait_regs(t);
#pragma unroll
          for (int e = 0; e < 32; ++e) t[e] = __float_as_uint(__uint_as_float(t[e]) * f);
          tmem_st32(lane_base + C::O_COL + c, t);
        }
        tmem_st_wait();
      }
      if (need) {
        l_sum *= f;
        m_used = m_new;
      }
      const float neg_base = m_used == -INFINITY ? 0.f : -m_used;
      float2 part[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};  // the row sum over independent chains
      const float2 scale2 = make_float2(a.scale_log2, a.scale_log2);
      const float2 base2 = make_float2(neg_base, neg_base);
#pragma unroll
      for (int c = 0; c < BN; c += 64) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float2 x = fma2(make_float2(sv[c + 2 * e], sv[c + 2 * e + 1]), scale2, base2);
          const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          part[e & 3] = add2(part[e & 3], p);
          pk[e] = pack_bf16x2(p.x, p.y);
        }
        tmem_st32(s_addr + c / 2, pk);  // P_j over the score columns this thread has already read
      }
      const float2 ps = add2(add2(part[0], part[1]), add2(part[2], part[3]));
      l_sum += ps.x + ps.y;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    // ---- epilogue: O / l, optional gate, bf16 row
    if (n_tiles > 0) {
      if (!mbar_wait(&pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, a.status)) goto done;
      tc_fence_after();
    }
    // The gate tile sits in the Q buffer (128-byte swizzled rows); without visible keys the output is 0 and needs
    // no gate.
    const bool gated = a.gate != nullptr && n_tiles > 0;
    if (gated && !mbar_wait(g_full, 0, a.status)) goto done;
    const int row = qs + r;
    const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
    __nv_bfloat16* orow = a.out + (int64_t)(q0 + row) * a.ldo + (int64_t)head * HD + vcol;
#pragma unroll 1
    for (int c = 0; c < DV; c += 32) {
      uint32_t t[32];
      if (n_tiles > 0) {
        tmem_ld32(lane_base + C::O_COL + c, t);  // warp-collective: every lane loads, valid rows store
        tmem_ld_wait_regs(t);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) t[e] = 0u;
      }
      if (row < lq) {
        uint32_t gw[16];
        if (gated) {  // this row's 32 gate values: four 16-byte pieces of its swizzled 128-byte row
          const uint8_t* grow = s_q + (c / 64) * C::Q_CHUNK + r * 128;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint4 g4 = *reinterpret_cast<const uint4*>(grow + ((((c % 64) / 8 + k4) ^ (r & 7)) << 4));
            gw[4 * k4] = g4.x;
            gw[4 * k4 + 1] = g4.y;
            gw[4 * k4 + 2] = g4.z;
            gw[4 * k4 + 3] = g4.w;
          }
        }
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float v0 = bf16_round(__uint_as_float(t[2 * e]) * inv);
          float v1 = bf16_round(__uint_as_float(t[2 * e + 1]) * inv);
          if (gated) {  // Qwen's output gate: bf16(o) * sigmoid(gate), rounded once
            const float2 gv = unpack_bf16x2(gw[e]);
            v0 *= sigmoid(gv.x);
            v1 *= sigmoid(gv.y);
          }
          packed[e] = pack_bf16x2(v0, v1);
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<uint4*>(orow + c + 8 * q4) =
              make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int HD, int DV>
int launch(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, int64_t tq, int64_t tk,
           const Args& a, int64_t total_q, cudaStream_t stream) {
  using C = Cfg<HD, DV>;
  CUtensorMap mq, mk, mv;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_tma_2d(&mq, q, dt, 2, (uint64_t)ldq, (uint64_t)tq, (uint64_t)ldq, 64, C::BM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tma_2d(&mk, k, dt, 2, (uint64_t)ldk, (uint64_t)tk, (uint64_t)ldk, 64, C::BN,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tma_2d(&mv, v, dt, 2, (uint64_t)ldv, (uint64_t)tk, (uint64_t)ldv, 64, C::BN,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap mg = mq;  // the gate tile has the Q tile's shape (unused without a gate)
  if (!rc && a.gate)
    rc = make_tma_2d(&mg, a.gate, dt, 2, (uint64_t)a.ldg, (uint64_t)tq, (uint64_t)a.ldg, 64, C::BM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  auto kernel = attention_kernel<HD, DV>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KD_ERR_ARGUMENT;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return record_cuda_error(e, "attention: cudaFuncSetAttribute");
    configured[dev] = true;
  }
  // Upper bound on query tiles over all sequences: sum(ceil(Lq / BM)) <= total_q / BM + num_seqs.
  const int64_t tiles = total_q / C::BM + a.num_seqs;
  if (tiles > 0x7fffffff) return set_error(KD_ERR_ARGUMENT, "attention: too many query tiles");
  dim3 grid((unsigned)tiles, (unsigned)a.hq, (unsigned)C::SLICES);
  kernel<<<grid, THREADS, C::SMEM, stream>>>(mq, mk, mv, mg, a);
  return record_cuda_error(cudaGetLastError(), "attention: launch");
}

}  // namespace fa
}  // namespace kd

using namespace kd;

extern "C" int kd_attention_varlen(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                   void* out, int64_t ldo, const void* gate, int64_t ldg, const int32_t* cu_q,
                                   const int32_t* cu_k, int num_seqs, int max_q, int64_t total_q, int64_t total_k,
                                   int num_heads_q, int num_heads_kv, int head_dim, float scale, int window_left,
                                   int window_right, int* status, cudaStream_t stream) {
  (void)max_q;
  if (num_seqs < 0 || total_q < 0 || total_k < 0) return set_error(KD_ERR_ARGUMENT, "attention: negative sizes");
  if (num_seqs == 0 || total_q == 0) return KD_OK;
  if (num_heads_q <= 0 || num_heads_kv <= 0 || num_heads_q % num_heads_kv)
    return set_error(KD_ERR_ARGUMENT, "attention: query heads must be a multiple of key/value heads");
  if (!q || !k || !v || !out || !cu_q || !cu_k || !status) return set_error(KD_ERR_ARGUMENT, "attention: null pointer");
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(q) || !a16(k) || !a16(v) || !a16(out) || (gate && !a16(gate)) || ldq % 8 || ldk % 8 || ldv % 8 ||
      ldo % 8 || (gate && ldg % 8))
    return set_error(KD_ERR_ARGUMENT, "attention: pointers and row strides must be 16-byte aligned");
  if (ldq < (int64_t)num_heads_q * head_dim || ldo < (int64_t)num_heads_q * head_dim ||
      ldk < (int64_t)num_heads_kv * head_dim || ldv < (int64_t)num_heads_kv * head_dim)
    return set_error(KD_ERR_ARGUMENT, "attention: row strides smaller than heads x head_dim");
  fa::Args a;
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.ldg = ldg;
  a.cu_q = cu_q;
  a.cu_k = cu_k;
  a.num_seqs = num_seqs;
  a.hq = num_heads_q;
  a.hkv = num_heads_kv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.left = window_left;
  a.right = window_right;
  a.status = status;
  const int64_t tk = total_k;
  switch (head_dim) {
    case 64:
      return fa::launch<64, 64>(q, ldq, k, ldk, v, ldv, total_q, tk, a, total_q, stream);
    case 128:
      return fa::launch<128, 128>(q, ldq, k, ldk, v, ldv, total_q, tk, a, total_q, stream);
    case 256:
      return fa::launch<256, 256>(q, ldq, k, ldk, v, ldv, total_q, tk, a, total_q, stream);
    case 512:
      return fa::launch<512, 256>(q, ldq, k, ldk, v, ldv, total_q, tk, a, total_q, stream);
    default:
      return set_error(KD_ERR_ARGUMENT, "attention: head_dim must be 64, 128, 256 or 512");
  }
}
