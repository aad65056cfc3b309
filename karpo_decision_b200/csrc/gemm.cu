// Projection GEMMs of the packed decoder forward on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )
//
// A is the activation (rows = pack tokens, K contiguous), B an nn.Linear weight (out_features x in_features, K
// contiguous), so both operands are K-major. Replaces the cuBLAS / torch._scaled_mm calls behind every projection of
// the reference's layers (families/qwen/packed.py:108-125,144-156; families/gemma/packed.py:183-193,254-265;
// serve/fp8.py:86-101; serve/qwen_fp8.py:38-42).
//
// Design (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: A and B tiles (128-byte rows, 128-byte swizzle) into a 4-stage shared-memory ring;
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128, N=256) into one of two TMEM accumulators
//               (2 x 256 fp32 columns) and commits each stage back to the producer;
//   warps 2..9  epilogue, two warpgroups each taking half of a tile's columns: tcgen05.ld of the accumulator (one
//               TMEM lane = one output row per thread), the fused epilogue, 16-byte stores; the second accumulator
//               lets tile i's epilogue overlap tile i+1's mainloop.
// The k-loop is BK = 64 bf16 (or 128 e4m3) elements: one 128-byte swizzle row per operand row.
#include "common.cuh"
#include "kd_internal.h"

namespace kd {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int ROW_BYTES = 128;  // one swizzle row per operand row per stage
constexpr int A_STAGE_BYTES = BM * ROW_BYTES;  // 16 KB
constexpr int TMEM_COLS = 512;  // two 128 x 256 fp32 accumulators
constexpr int EPI_GROUPS = 2;  // epilogue warpgroups, each taking half of a tile's columns
constexpr int THREADS = 64 + EPI_GROUPS * 128;
// Output staging: per epilogue warp a 32-row x 64-column bf16 box (128-byte swizzled rows) for its TMA stores.
constexpr int OUT_BOX_COLS = 64;
constexpr int OUT_BOX_BYTES = 32 * OUT_BOX_COLS * 2;
constexpr int NORM_BYTES = 2 * 256 * 2;  // the QKV epilogue's q and k norm weights (bf16, head_dim <= 256)
constexpr int NORM_F32_HD = 128;         // up to this head_dim they are stored as float multipliers instead

// The pipeline of one CTA. Single: a 128 x 256 tile per CTA, A (128 rows) and B (256 rows) per stage. Pair (a
// cluster of two CTAs, one cta_group::2 MMA over 256 x 256): each CTA stages its 128 rows of A and its 128 rows of B,
// so a stage is a third smaller and the ring one deeper per byte; the leader issues the MMA over both CTAs' stages.
template <bool PAIR>
struct Pipe {
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_ROWS * ROW_BYTES;
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;  // output rows of one (cluster) tile
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_GROUPS * 4 * OUT_BOX_BYTES + NORM_BYTES +
                              1024 /* alignment slack */ + 256 /* barriers */;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};
// Pack sizes from which the CTA-pair kernel runs (below, the single-CTA one: the pair's second half would idle).
constexpr int PAIR_MIN_ROWS = 256;

// The fused attention-input epilogue (KD_EPI_QKV): the projection's columns are [q heads][k heads][v heads] (Qwen's
// gated queries: [q_h | gate_h] per head); each output row's heads are normalized, rotated and scattered to q, k, v
// and gate, as kd_qkv_norm_rope does from a stored projection.
struct Qkv {
  const int64_t* seqpos;
  const uint32_t* cs;  // per token and rotary pair: bf16 cos | bf16 sin << 16, laid out [rot / 2][M] (coalesced)
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  __nv_bfloat16* gate;
  int hq, hkv, hd, rot, gated, qk_mode, v_mode;
  float eps;
};

struct Args {
  int M, N, K;
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* R;  // residual (EPI_RESIDUAL); may alias C
  int64_t ldr;
  const float* scale_a;  // FP8: one scale per A row
  const float* scale_b;  // FP8: one scale per B row (output column)
  int* status;
  Qkv qkv;
  int tile_group;  // row blocks per group of the tile order (tile_coords)
};

// 16 accumulator columns of one row (raw tcgen05.ld registers) as the projection's bf16 outputs (FP8: scaled first).
template <bool FP8>
KD_DEVICE void to_bf16_16(const Args& a, const uint32_t (&r)[16], int col, float sa, float (&x)[16]) {
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    float v0 = __uint_as_float(r[j]), v1 = __uint_as_float(r[j + 1]);
    if constexpr (FP8) {
      v0 = v0 * sa * a.scale_b[col + j];
      v1 = v1 * sa * a.scale_b[col + j + 1];
    }
    const float2 b = bf16_round2(v0, v1);
    x[j] = b.x;
    x[j + 1] = b.y;
  }
}

// The norm multipliers of 16 consecutive head dims (none, w or 1 + w) from shared memory: for head_dim <= 128 the
// kernel stored them as float (four 16-byte loads), for wider heads as the bf16 weights (two loads, then 1 + w).
KD_DEVICE void norm16(const __nv_bfloat16* w, int mode, int d, int hd, float (&m)[16]) {
  if (mode != KD_NORM_WEIGHT && mode != KD_NORM_ONE_PLUS) {
#pragma unroll
    for (int j = 0; j < 16; ++j) m[j] = 1.0f;
    return;
  }
  if (hd <= NORM_F32_HD) {
    const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + d);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = f[q];
      m[4 * q] = v.x;
      m[4 * q + 1] = v.y;
      m[4 * q + 2] = v.z;
      m[4 * q + 3] = v.w;
    }
    return;
  }
  const uint4 lo = *reinterpret_cast<const uint4*>(w + d);
  const uint4 hi = *reinterpret_cast<const uint4*>(w + d + 8);
  const uint32_t words[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 f = unpack_bf16x2(words[j]);
    m[2 * j] = mode == KD_NORM_ONE_PLUS ? 1.0f + f.x : f.x;
    m[2 * j + 1] = mode == KD_NORM_ONE_PLUS ? 1.0f + f.y : f.y;
  }
}

// This lane's 16 values as bf16 into row `lane` of a 32-row x 16-column staging segment (1 KB, 32-byte rows) in the
// TMA 32-byte swizzle: row i's 16-byte half p at i * 32 + ((p ^ (i / 4 % 2)) << 4), conflict-free for a row per lane.
KD_DEVICE void put16(uint8_t* seg, int lane, const float (&x)[16]) {
  uint32_t p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = pack_bf16x2(x[2 * j], x[2 * j + 1]);
  const int sw = (lane >> 2) & 1;
  *reinterpret_cast<uint4*>(seg + lane * 32 + (sw << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
  *reinterpret_cast<uint4*>(seg + lane * 32 + ((sw ^ 1) << 4)) = make_uint4(p[4], p[5], p[6], p[7]);
}

// Waits until at most 3 of this thread's bulk stores still read shared memory.
// Output tiles in groups of TILE_GROUP row blocks: within a group the tile index runs over the group's row blocks
// first, then over the column blocks. The persistent CTAs work on consecutive tiles at the same time, so at any moment
// they cover a few column blocks of at most TILE_GROUP row blocks: the group's A rows stay in L2 while B's column
// blocks stream past once per group, instead of all of B once per row block (the row-major order, whose B re-reads
// dominate DRAM traffic once B outgrows L2). Measured on B200: gemma-31b's FP8 gate/up projection (32,768 x 43,008 x
// 5,376) 6,166 -> 4,940 us and gemma-12b's bf16 one (32,768 x 30,720 x 3,840) 5,974 -> 4,789 us; shapes whose B
// stays in L2 unchanged. Groups of 8 and 32 row blocks measured no better.
constexpr int TILE_GROUP = 16;
KD_DEVICE void tile_coords(int tile, int m_tiles, int n_tiles, int group_rows, int& mb, int& nb) {
  const int per_group = group_rows * n_tiles;
  const int group = tile / per_group;
  const int first = group * group_rows;
  const int rows = min(m_tiles - first, group_rows);
  const int in = tile - group * per_group;
  mb = first + in % rows;
  nb = in / rows;
}

KD_DEVICE void bulk_wait_read_3() { asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); }

// One row's heads inside the 256 columns [n0, n0 + 256) of the QKV projection: per-head RMSNorm over head_dim, then
// rotate-half RoPE on the first `rot` dims (q, k); Gemma's weightless v norm; gate and plain v copied. Two passes
// over tensor memory: the sum of squares, then the normalized, rotated head in 16-column pieces (a piece below rot / 2
// together with its rotation partner rot / 2 further on). The epilogue warpgroups take alternate head slices (one
// group takes all of a 256-wide head). Each step issues its tensor-memory loads, its rotary factors (the per-pack
// table `cs`, [rot / 2][M]: a warp's lanes read consecutive rows, one coalesced line per pair index) and its norm
// weights (a shared-memory copy: q_norm then k_norm) before waiting on any of them, so their latencies overlap.
// Outputs leave by TMA stores of 16-column pieces of the warp's 32 rows, staged in a ring of four 1 KB segments of
// the warp's box (`nseg` counts the pieces the warp has stored): the tensor copy writes whole 32-byte row pieces,
// where a row per lane would issue 32 scattered 16-byte stores per instruction. Rows past M are clipped by the copy.
template <bool FP8>
KD_DEVICE void qkv_epilogue(const Args& a, int n0, uint32_t t_row, float sa, int group, const __nv_bfloat16* norm_s,
                            uint8_t* box, int row0, int lane, uint32_t& nseg, const CUtensorMap* map_q,
                            const CUtensorMap* map_g, const CUtensorMap* map_k, const CUtensorMap* map_v) {
  const Qkv& g = a.qkv;
  const int hd = g.hd;
  const int q_cols = g.hq * hd * (g.gated ? 2 : 1);
  const int k_end = q_cols + g.hkv * hd;
  const int row = row0 + lane;
  const int crow = row < a.M ? row : a.M - 1;  // rows past M compute (warp-collective loads) but store nothing
  const uint32_t* cs = g.cs + crow;
  const int half = g.rot / 2;
  for (int h0 = (hd < BN ? group * hd : 0); h0 < BN; h0 += (hd < BN ? EPI_GROUPS * hd : BN)) {
    if (hd >= BN && group != 0) break;
    const int c0 = n0 + h0;  // first column of this head slice
    if (c0 >= a.N) break;
    const uint32_t th = t_row + h0;
    int kind;  // 0 q, 1 gate, 2 k, 3 v
    int head;
    if (c0 < q_cols) {
      if (g.gated) {
        head = c0 / (2 * hd);
        kind = (c0 % (2 * hd)) == 0 ? 0 : 1;
      } else {
        head = c0 / hd;
        kind = 0;
      }
    } else if (c0 < k_end) {
      head = (c0 - q_cols) / hd;
      kind = 2;
    } else {
      head = (c0 - k_end) / hd;
      kind = 3;
    }
    const CUtensorMap* map = kind == 0 ? map_q : kind == 1 ? map_g : kind == 2 ? map_k : map_v;
    // 16 columns of the warp's 32 rows to columns [col, col + 16) of their heads
    auto emit = [&](int col, const float (&x)[16]) {
      uint8_t* seg = box + (nseg & 3) * 1024;
      if (lane == 0) bulk_wait_read_3();  // the store that last read this segment is done
      __syncwarp();
      put16(seg, lane, x);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map, seg, head * hd + col, row0);
        bulk_commit();
      }
      ++nseg;
    };
    const bool normed = kind == 0 || kind == 2 || (kind == 3 && g.v_mode >= 0);
    const bool rotated = kind == 0 || kind == 2;
    float inv = 1.0f;
    if (normed) {
      float2 ss0 = make_float2(0.f, 0.f), ss1 = make_float2(0.f, 0.f);
      for (int d = 0; d < hd; d += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld16(th + d, r0);
        tmem_ld16(th + d + 16, r1);
        tmem_ld_wait_regs(r0);
        tmem_ld_wait_regs(r1);
        float x[16], y[16];
        to_bf16_16<FP8>(a, r0, c0 + d, sa, x);
        to_bf16_16<FP8>(a, r1, c0 + d + 16, sa, y);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const float2 x2 = make_float2(x[j], x[j + 1]), y2 = make_float2(y[j], y[j + 1]);
          ss0 = fma2(x2, x2, ss0);
          ss1 = fma2(y2, y2, ss1);
        }
      }
      inv = 1.0f / sqrtf(((ss0.x + ss0.y) + (ss1.x + ss1.y)) / (float)hd + g.eps);
    }
    if (!rotated) {  // gate, v: pieces of 32 columns, normalized for Gemma's v
      for (int d = 0; d < hd; d += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld16(th + d, r0);
        tmem_ld16(th + d + 16, r1);
        tmem_ld_wait_regs(r0);
        tmem_ld_wait_regs(r1);
        float x[16], y[16];
        to_bf16_16<FP8>(a, r0, c0 + d, sa, x);
        to_bf16_16<FP8>(a, r1, c0 + d + 16, sa, y);
        if (normed) {
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float2 xs = mul2(make_float2(x[j], x[j + 1]), inv2), ys = mul2(make_float2(y[j], y[j + 1]), inv2);
            x[j] = xs.x;
            x[j + 1] = xs.y;
            y[j] = ys.x;
            y[j + 1] = ys.y;
          }
        }
        emit(d, x);
        emit(d + 16, y);
      }
      continue;
    }
    // this head's norm multipliers: float for head_dim <= 128, else the bf16 weights
    const __nv_bfloat16* w = hd <= NORM_F32_HD
                                 ? reinterpret_cast<const __nv_bfloat16*>(reinterpret_cast<const float*>(norm_s) +
                                                                          (kind == 0 ? 0 : hd))
                                 : norm_s + (kind == 0 ? 0 : hd);
    // rotation pairs: the piece at d < rot / 2 with its partner at d + rot / 2
    for (int d = 0; d < half; d += 16) {
      uint32_t rx[16], ry[16], f[16];
      tmem_ld16(th + d, rx);
      tmem_ld16(th + d + half, ry);
#pragma unroll
      for (int j = 0; j < 16; ++j) f[j] = cs[(int64_t)(d + j) * a.M];
      float mx[16], my[16];
      norm16(w, g.qk_mode, d, hd, mx);
      norm16(w, g.qk_mode, d + half, hd, my);
      tmem_ld_wait_regs(rx);
      tmem_ld_wait_regs(ry);
      float x[16], y[16];
      to_bf16_16<FP8>(a, rx, c0 + d, sa, x);
      to_bf16_16<FP8>(a, ry, c0 + d + half, sa, y);
      float ox[16], oy[16];
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int j = 0; j < 16; j += 2) {  // two rotation pairs at a time, on paired float instructions
        float2 xn = mul2(mul2(make_float2(x[j], x[j + 1]), inv2), make_float2(mx[j], mx[j + 1]));
        float2 yn = mul2(mul2(make_float2(y[j], y[j + 1]), inv2), make_float2(my[j], my[j + 1]));
        if (g.gated) {  // Qwen: the norm is its own op (rounded), RoPE another
          xn = bf16_round2(xn.x, xn.y);
          yn = bf16_round2(yn.x, yn.y);
        }
        // cos and sin of pairs d + j, d + j + 1 (the same for their partners rot / 2 further on)
        const float2 c0s = unpack_bf16x2(f[j]), c1s = unpack_bf16x2(f[j + 1]);
        const float2 cc = make_float2(c0s.x, c1s.x), sn = make_float2(c0s.y, c1s.y);
        const float2 o1 = fma2(xn, cc, mul2(yn, make_float2(-sn.x, -sn.y)));  // x cos - y sin
        const float2 o2 = fma2(yn, cc, mul2(xn, sn));                         // y cos + x sin
        ox[j] = o1.x;
        ox[j + 1] = o1.y;
        oy[j] = o2.x;
        oy[j + 1] = o2.y;
      }
      emit(d, ox);
      emit(d + half, oy);
    }
    // the unrotated rest, pieces of 16 columns
    for (int d = g.rot; d < hd; d += 16) {
      uint32_t r[16];
      tmem_ld16(th + d, r);
      float m[16];
      norm16(w, g.qk_mode, d, hd, m);
      tmem_ld_wait_regs(r);
      float x[16];
      to_bf16_16<FP8>(a, r, c0 + d, sa, x);
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        float2 xn = mul2(mul2(make_float2(x[j], x[j + 1]), inv2), make_float2(m[j], m[j + 1]));
        if (g.gated) xn = bf16_round2(xn.x, xn.y);
        x[j] = xn.x;
        x[j + 1] = xn.y;
      }
      emit(d, x);
    }
  }
}

template <int EPI, bool FP8, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_r,
                const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v, Args args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using P = Pipe<PAIR>;
  constexpr int STAGES = P::STAGES;
  constexpr int STAGE_BYTES = P::STAGE_BYTES;
  uint8_t* out_stage = smem + STAGES * STAGE_BYTES;  // epilogue warp e's box at e * OUT_BOX_BYTES
  __nv_bfloat16* norm_s = reinterpret_cast<__nv_bfloat16*>(out_stage + EPI_GROUPS * 4 * OUT_BOX_BYTES);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(out_stage + EPI_GROUPS * 4 * OUT_BOX_BYTES + NORM_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* res_bar = acc_empty + 2;  // [epilogue warps]: the residual box of that warp has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bar + EPI_GROUPS * 4);
  if constexpr (EPI == KD_EPI_QKV) {  // q / k norm weights into shared memory: the epilogue reads them per head piece
    const int hd = args.qkv.hd;
    const bool weighted = args.qkv.qk_mode == KD_NORM_WEIGHT || args.qkv.qk_mode == KD_NORM_ONE_PLUS;
    if (hd <= NORM_F32_HD) {  // float multipliers (w or 1 + w, as the reference forms them in float)
      for (int i = threadIdx.x; weighted && i < 2 * hd; i += THREADS) {
        const float w = __bfloat162float(i < hd ? args.qkv.q_norm[i] : args.qkv.k_norm[i - hd]);
        reinterpret_cast<float*>(norm_s)[i] = args.qkv.qk_mode == KD_NORM_ONE_PLUS ? 1.0f + w : w;
      }
    } else {
      for (int i = threadIdx.x; weighted && i < 2 * hd / 8; i += THREADS) {
        const __nv_bfloat16* src = i < hd / 8 ? args.qkv.q_norm + 8 * i : args.qkv.k_norm + 8 * (i - hd / 8);
        reinterpret_cast<uint4*>(norm_s)[i] = *reinterpret_cast<const uint4*>(src);
      }
    }
  }

  const int warp = threadIdx.x / 32;
  const uint32_t rank = PAIR ? cluster_rank() : 0;  // this CTA's half of a pair tile: rows rank * 128 ..
  const bool leader = rank == 0;
  const int first_tile = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  const int m_tiles = (args.M + P::TILE_M - 1) / P::TILE_M;
  const int n_tiles = (args.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int elems_per_row = FP8 ? ROW_BYTES : ROW_BYTES / 2;  // BK in elements
  const int k_blocks = (args.K + elems_per_row - 1) / elems_per_row;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      // single: every epilogue thread arrives; pair: one arrival per epilogue warp of both CTAs, on the leader's
      mbar_init(&acc_empty[b], PAIR ? 2 * EPI_GROUPS * 4 : EPI_GROUPS * 128);
    }
    for (int e = 0; e < EPI_GROUPS * 4; ++e) mbar_init(&res_bar[e], 1);
    fence_barrier_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers initialized before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        int mb, nb;
        tile_coords(tile, m_tiles, n_tiles, args.tile_group, mb, nb);
        const int m0 = mb * P::TILE_M;
        const int n0 = nb * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.status)) goto done;
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_STAGE_BYTES;
          if constexpr (PAIR) {
            // both CTAs' halves land on the leader's full barrier, which expects the bytes of both
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * STAGE_BYTES);
            tma_load_2d_pair(&map_a, &full_bar[stage], sa, kb * elems_per_row, m0 + (int)rank * BM);
            tma_load_2d_pair(&map_b, &full_bar[stage], sb, kb * elems_per_row, n0 + (int)rank * P::B_ROWS);
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
            tma_load_2d(&map_a, &full_bar[stage], sa, kb * elems_per_row, m0);
            tma_load_2d(&map_b, &full_bar[stage], sb, kb * elems_per_row, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = mma_idesc(FP8 ? 0u : 1u, P::TILE_M, BN);
    if (leader && elect_one()) {  // pair: the leader issues the MMA for both CTAs
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.status)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, args.status)) goto done;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < ROW_BYTES / 32; ++k) {  // 32 bytes of K per instruction (16 bf16 or 32 e4m3)
            const uint64_t da = sw128_kmajor_desc(sa + 32 * k);
            const uint64_t db = sw128_kmajor_desc(sb + 32 * k);
            if constexpr (PAIR) {
              if constexpr (FP8)
                mma_f8_ss_pair(d_tmem, da, db, idesc, (kb | k) != 0);
              else
                mma_f16_ss_pair(d_tmem, da, db, idesc, (kb | k) != 0);
            } else {
              if constexpr (FP8)
                mma_f8_ss(d_tmem, da, db, idesc, (kb | k) != 0);
              else
                mma_f16_ss(d_tmem, da, db, idesc, (kb | k) != 0);
            }
          }
          // the stage is free once these MMAs have read it (pair: in both CTAs)
          if constexpr (PAIR)
            mma_commit_pair(&empty_bar[stage]);
          else
            mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        // the accumulator is complete once every MMA above has finished (pair: both CTAs' halves)
        if constexpr (PAIR)
          mma_commit_pair(&acc_full[acc]);
        else
          mma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int group = (warp - 2) / 4;  // this warp's epilogue warpgroup: its half of each tile's columns
    const int lane = threadIdx.x & 31;
    uint8_t* box = out_stage + (warp - 2) * OUT_BOX_BYTES;  // this warp's output staging box
    uint64_t* my_res = &res_bar[warp - 2];
    uint32_t res_phase = 0;
    uint32_t qkv_seg = 0;  // QKV: the 16-column pieces this warp has stored (its staging ring position)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      int mb, nb;
      tile_coords(tile, m_tiles, n_tiles, args.tile_group, mb, nb);
      const int m0 = mb * P::TILE_M + (int)rank * BM;  // this CTA's 128 rows of the tile
      const int n0 = nb * BN;
      if (!mbar_wait(&acc_full[acc], acc_phase, args.status)) goto done;
      tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      float sa = 1.0f;
      if constexpr (FP8) sa = (row < args.M) ? args.scale_a[row] : 0.0f;
      if constexpr (EPI == KD_EPI_QKV) {
        // QKV: map_c is q, map_r the gate
        qkv_epilogue<FP8>(args, n0, t_row, sa, group, norm_s, box, m0 + quarter * 32, lane, qkv_seg, &map_c, &map_r,
                          &map_k, &map_v);
      } else {
        // Output through this warp's staging box and TMA stores: 64-column chunks of the warp's 32 rows, written
        // into 128-byte swizzled smem rows (conflict-free: 8 consecutive rows cover all bank groups), then one bulk
        // tensor store per chunk. The residual (R may alias C) arrives the same way, by a TMA load into the box.
        constexpr bool gated = EPI == KD_EPI_SWIGLU || EPI == KD_EPI_GEGLU;
        const int n_out = gated ? args.N / 2 : args.N;
        const int out0 = (gated ? n0 / 2 : n0) + group * (gated ? BN / 4 : BN / 2);  // this group's first column
        const int chunks = gated ? 1 : 2;
        const int ybox = m0 + quarter * 32;
        for (int k = 0; k < chunks; ++k) {
          const int oc = out0 + k * OUT_BOX_COLS;
          if (oc >= n_out) break;
          if (lane == 0) bulk_wait_read();  // the previous chunk's store has read the box
          __syncwarp();
          if constexpr (EPI == KD_EPI_RESIDUAL) {
            if (lane == 0) {
              mbar_arrive_expect_tx(my_res, OUT_BOX_BYTES);
              tma_load_2d(&map_r, my_res, box, oc, ybox);
            }
            if (!mbar_wait(my_res, res_phase, args.status)) goto done;
            res_phase ^= 1;
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // two 32-column halves of the chunk
            float v[32];
            if constexpr (gated) {
              // tile columns [0,128) are gate rows, [128,256) the matching up rows (weights interleaved at load):
              // act(gate) * up, each operand rounded to bf16 first as the reference's Linear outputs are
#pragma unroll
              for (int s16 = 0; s16 < 2; ++s16) {  // 16 columns at a time keeps gate and up in registers
                const int cg = group * (BN / 4) + h * 32 + s16 * 16;
                uint32_t g[16], u[16];
                tmem_ld16(t_row + cg, g);
                tmem_ld16(t_row + BN / 2 + cg, u);
                tmem_ld_wait_regs(g);
                tmem_ld_wait_regs(u);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  float gf = __uint_as_float(g[j]);
                  float uf = __uint_as_float(u[j]);
                  if constexpr (FP8) {
                    gf *= sa * args.scale_b[n0 + cg + j];
                    uf *= sa * args.scale_b[n0 + BN / 2 + cg + j];
                  }
                  gf = bf16_round(gf);
                  uf = bf16_round(uf);
                  v[s16 * 16 + j] = (EPI == KD_EPI_SWIGLU ? silu(gf) : gelu_tanh(gf)) * uf;
                }
              }
            } else {
              const int c = group * (BN / 2) + k * OUT_BOX_COLS + h * 32;
              uint32_t r[32];
              tmem_ld32(t_row + c, r);
              tmem_ld_wait_regs(r);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float x = __uint_as_float(r[j]);
                if constexpr (FP8) {
                  const int col = n0 + c + j;
                  x = x * sa * (col < args.N ? args.scale_b[col] : 0.0f);
                }
                v[j] = x;
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // four 16-byte pieces: chunk index h * 4 + q of the 128-byte row
              uint8_t* piece = box + lane * 128 + (((h * 4 + q) ^ (lane & 7)) << 4);
              uint32_t w[4];
              if constexpr (EPI == KD_EPI_RESIDUAL) {
                const uint4 rv = *reinterpret_cast<const uint4*>(piece);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const float2 r2 = unpack_bf16x2(rw[t]);
                  // h + bf16(x): the residual add of two bf16 tensors, rounded once
                  w[t] = pack_bf16x2(r2.x + bf16_round(v[8 * q + 2 * t]), r2.y + bf16_round(v[8 * q + 2 * t + 1]));
                }
              } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) w[t] = pack_bf16x2(v[8 * q + 2 * t], v[8 * q + 2 * t + 1]);
              }
              *reinterpret_cast<uint4*>(piece) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_c, box, oc, ybox);
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      if constexpr (PAIR) {  // one arrival per warp, on the leader's barrier
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&acc_empty[acc]);
      } else {
        mbar_arrive(&acc_empty[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
done:
  bulk_wait();  // the epilogue's TMA stores have completed (no-op for threads that issued none) before the CTA exits
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // neither CTA leaves while the other may still signal its barriers or use the pair's TMEM
  else
    __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int EPI, bool FP8, bool PAIR>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr,
           const CUtensorMap& mk, const CUtensorMap& mv, const Args& args, cudaStream_t stream) {
  using P = Pipe<PAIR>;
  auto kernel = gemm_kernel<EPI, FP8, PAIR>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KD_ERR_ARGUMENT;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P::SMEM);
    if (e != cudaSuccess) return record_cuda_error(e, "gemm: cudaFuncSetAttribute");
    configured[dev] = true;
  }
  const int m_tiles = (args.M + P::TILE_M - 1) / P::TILE_M;
  const int n_tiles = (args.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  if constexpr (!PAIR) {
    const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
    kernel<<<grid, THREADS, P::SMEM, stream>>>(ma, mb, mc, mr, mk, mv, args);
  } else {
    const int pairs = num_sms(dev) / 2;
    const int grid = 2 * (tiles < pairs ? tiles : pairs);
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3((unsigned)grid);
    config.blockDim = dim3(THREADS);
    config.dynamicSmemBytes = P::SMEM;
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&config, kernel, ma, mb, mc, mr, mk, mv, args);
    if (e != cudaSuccess) return record_cuda_error(e, "gemm: cluster launch");
  }
  return record_cuda_error(cudaGetLastError(), "gemm: launch");
}

}  // namespace gemm
}  // namespace kd

using namespace kd;

static int gemm_common(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
                       int64_t ldr, const float* scale_a, const float* scale_b, int M, int N, int K, int epilogue,
                       int fp8, int* status, cudaStream_t stream, const gemm::Qkv* qkv = nullptr,
                       bool launch = true) {
  if (M < 0 || N <= 0 || K <= 0) return set_error(KD_ERR_ARGUMENT, "gemm: M >= 0, N > 0 and K > 0 required");
  if (M == 0) return KD_OK;
  if (!A || !B || !C || !status) return set_error(KD_ERR_ARGUMENT, "gemm: null pointer");
  const int esize = fp8 ? 1 : 2;
  if ((lda * esize) % 16 || (ldb * esize) % 16 || (reinterpret_cast<uintptr_t>(A) % 16) ||
      (reinterpret_cast<uintptr_t>(B) % 16))
    return set_error(KD_ERR_ARGUMENT, "gemm: A and B need 16-byte aligned bases and row strides");
  if (lda < K || ldb < K) return set_error(KD_ERR_ARGUMENT, "gemm: lda and ldb must be >= K");
  if (N % 32) return set_error(KD_ERR_ARGUMENT, "gemm: N must be a multiple of 32");
  const bool gated = epilogue == KD_EPI_SWIGLU || epilogue == KD_EPI_GEGLU;
  if (gated && N % gemm::BN) return set_error(KD_ERR_ARGUMENT, "gemm: gated epilogues need N % 256 == 0");
  const int n_out = gated ? N / 2 : N;
  if (ldc < n_out || (ldc % 8) || (reinterpret_cast<uintptr_t>(C) % 16))
    return set_error(KD_ERR_ARGUMENT, "gemm: C needs a 16-byte aligned base and ldc % 8 == 0, ldc >= output width");
  if (epilogue == KD_EPI_RESIDUAL && (!R || ldr < N || (ldr % 8) || (reinterpret_cast<uintptr_t>(R) % 16)))
    return set_error(KD_ERR_ARGUMENT, "gemm: residual epilogue needs R with ldr >= N, ldr % 8 == 0, 16-byte base");
  if (fp8 && (!scale_a || !scale_b)) return set_error(KD_ERR_ARGUMENT, "gemm: fp8 needs scale_a and scale_b");

  CUtensorMap ma, mb;
  const CUtensorMapDataType dt = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t box_k = gemm::ROW_BYTES / esize;
  int rc = make_tma_2d(&ma, A, dt, esize, K, M, lda, box_k, gemm::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const bool pair = M >= gemm::PAIR_MIN_ROWS;  // pair: each CTA of a pair stages half of a tile's B rows
  rc = make_tma_2d(&mb, B, dt, esize, K, N, ldb, box_k, pair ? gemm::BN / 2 : gemm::BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  gemm::Args args;
  args.M = M;
  args.N = N;
  args.K = K;
  args.C = static_cast<__nv_bfloat16*>(C);
  args.ldc = ldc;
  args.R = static_cast<const __nv_bfloat16*>(R);
  args.ldr = ldr;
  args.scale_a = scale_a;
  args.scale_b = scale_b;
  args.status = status;
  args.qkv = qkv ? *qkv : gemm::Qkv{};
  args.tile_group = gemm::TILE_GROUP;

  // output (and residual) boxes for the TMA-store epilogue: 64 columns x 32 rows, 128-byte swizzle; the QKV epilogue
  // stores 16 columns x 32 rows of q (mc), the gate (mr), k (mk) and v (mv), 32-byte swizzle
  CUtensorMap mc = ma, mr = ma, mk = ma, mv = ma;
  if (epilogue == KD_EPI_QKV) {
    const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_32B;
    const uint64_t qw = (uint64_t)qkv->hq * qkv->hd, kw = (uint64_t)qkv->hkv * qkv->hd;
    rc = make_tma_2d(&mc, qkv->q, bf, 2, qw, M, qw, 16, 32, sw);
    if (!rc && qkv->gated) rc = make_tma_2d(&mr, qkv->gate, bf, 2, qw, M, qw, 16, 32, sw);
    if (!rc) rc = make_tma_2d(&mk, qkv->k, bf, 2, kw, M, kw, 16, 32, sw);
    if (!rc) rc = make_tma_2d(&mv, qkv->v, bf, 2, kw, M, kw, 16, 32, sw);
    if (rc) return rc;
  } else {
    rc = make_tma_2d(&mc, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n_out, M, ldc, gemm::OUT_BOX_COLS, 32,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc && epilogue == KD_EPI_RESIDUAL)
      rc = make_tma_2d(&mr, R, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, ldr, gemm::OUT_BOX_COLS, 32,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (!launch) return KD_OK;  // a check-only call: every argument and descriptor accepted, nothing launched
#define KD_GEMM_CASE(E)                                                                                \
  case E:                                                                                              \
    if (pair)                                                                                          \
      return fp8 ? gemm::launch<E, true, true>(ma, mb, mc, mr, mk, mv, args, stream)                           \
                 : gemm::launch<E, false, true>(ma, mb, mc, mr, mk, mv, args, stream);                         \
    return fp8 ? gemm::launch<E, true, false>(ma, mb, mc, mr, mk, mv, args, stream)                            \
               : gemm::launch<E, false, false>(ma, mb, mc, mr, mk, mv, args, stream);
  switch (epilogue) {
    KD_GEMM_CASE(KD_EPI_STORE)
    KD_GEMM_CASE(KD_EPI_RESIDUAL)
    KD_GEMM_CASE(KD_EPI_SWIGLU)
    KD_GEMM_CASE(KD_EPI_GEGLU)
    KD_GEMM_CASE(KD_EPI_QKV)
    default:
      return set_error(KD_ERR_ARGUMENT, "gemm: unknown epilogue");
  }
#undef KD_GEMM_CASE
}

static int qkv_common(const void* A, int64_t lda, const float* scale_a, const void* W, int64_t ldw,
                      const float* scale_w, int M, int N, int K, const int64_t* seqpos, int num_heads_q,
                      int num_heads_kv, int head_dim, int gated, const void* q_norm_w, const void* k_norm_w,
                      int qk_norm_mode, int v_norm_mode, float eps, const uint32_t* rope_cs, int rot, void* q,
                      void* k, void* v, void* gate, int fp8, int* status, cudaStream_t stream,
                      bool launch = true) {
  if (num_heads_q <= 0 || num_heads_kv <= 0 || num_heads_q % num_heads_kv)
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: bad head counts");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: head_dim must be 64, 128 or 256");
  const int64_t width = (int64_t)num_heads_q * head_dim * (gated ? 2 : 1) + 2LL * num_heads_kv * head_dim;
  if (N != width || N % gemm::BN)
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: N must equal the q/k/v width and be a multiple of 256");
  if (rot < 0 || rot > head_dim || rot % 32)
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: rotary width must be a multiple of 32 within head_dim");
  if (M > 0 && (!seqpos || !q || !k || !v || (gated && !gate) || (rot > 0 && !rope_cs) ||
                (qk_norm_mode > KD_NORM_NONE && (!q_norm_w || !k_norm_w))))
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: null pointer");
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(q) || !a16(k) || !a16(v) || (gate && !a16(gate)))
    return set_error(KD_ERR_ARGUMENT, "qkv_projection: outputs must be 16-byte aligned");
  gemm::Qkv g;
  g.seqpos = seqpos;
  g.cs = rope_cs;
  g.q_norm = static_cast<const __nv_bfloat16*>(q_norm_w);
  g.k_norm = static_cast<const __nv_bfloat16*>(k_norm_w);
  g.q = static_cast<__nv_bfloat16*>(q);
  g.k = static_cast<__nv_bfloat16*>(k);
  g.v = static_cast<__nv_bfloat16*>(v);
  g.gate = static_cast<__nv_bfloat16*>(gate);
  g.hq = num_heads_q;
  g.hkv = num_heads_kv;
  g.hd = head_dim;
  g.rot = rot;
  g.gated = gated;
  g.qk_mode = qk_norm_mode;
  g.v_mode = v_norm_mode;
  g.eps = eps;
  // C is unused by this epilogue; q stands in for the pointer checks.
  return gemm_common(A, lda, W, ldw, q, N, nullptr, 0, scale_a, scale_w, M, N, K, KD_EPI_QKV, fp8, status, stream,
                     &g, launch);
}

namespace kd {
int qkv_projection_check(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                         const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim, int gated,
                         const void* q_norm_w, const void* k_norm_w, int qk_norm_mode, int v_norm_mode, float eps,
                         const uint32_t* rope_cs, int rot, void* q, void* k, void* v, void* gate, int* status) {
  return qkv_common(A, lda, nullptr, W, ldw, nullptr, M, N, K, seqpos, num_heads_q, num_heads_kv, head_dim, gated,
                    q_norm_w, k_norm_w, qk_norm_mode, v_norm_mode, eps, rope_cs, rot, q, k, v, gate, 0, status,
                    nullptr, false);
}
}  // namespace kd

extern "C" int kd_qkv_projection(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                                 const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim, int gated,
                                 const void* q_norm_w, const void* k_norm_w, int qk_norm_mode, int v_norm_mode,
                                 float eps, const uint32_t* rope_cs, int rot, void* q, void* k, void* v,
                                 void* gate, int* status, cudaStream_t stream) {
  return qkv_common(A, lda, nullptr, W, ldw, nullptr, M, N, K, seqpos, num_heads_q, num_heads_kv, head_dim, gated,
                    q_norm_w, k_norm_w, qk_norm_mode, v_norm_mode, eps, rope_cs, rot, q, k, v, gate, 0,
                    status, stream);
}

extern "C" int kd_qkv_projection_fp8(const void* A, int64_t lda, const float* scale_a, const void* W, int64_t ldw,
                                     const float* scale_w, int M, int N, int K, const int64_t* seqpos,
                                     int num_heads_q, int num_heads_kv, int head_dim, int gated, const void* q_norm_w,
                                     const void* k_norm_w, int qk_norm_mode, int v_norm_mode, float eps,
                                     const uint32_t* rope_cs, int rot, void* q, void* k, void* v, void* gate,
                                     int* status, cudaStream_t stream) {
  return qkv_common(A, lda, scale_a, W, ldw, scale_w, M, N, K, seqpos, num_heads_q, num_heads_kv, head_dim, gated,
                    q_norm_w, k_norm_w, qk_norm_mode, v_norm_mode, eps, rope_cs, rot, q, k, v, gate, 1,
                    status, stream);
}

extern "C" int kd_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                            const void* R, int64_t ldr, int M, int N, int K, int epilogue, int* status,
                            cudaStream_t stream) {
  if (epilogue == KD_EPI_QKV) return set_error(KD_ERR_ARGUMENT, "gemm: the QKV epilogue is kd_qkv_projection");
  return gemm_common(A, lda, B, ldb, C, ldc, R, ldr, nullptr, nullptr, M, N, K, epilogue, 0, status, stream);
}

extern "C" int kd_gemm_fp8(const void* A, int64_t lda, const float* scale_a, const void* B, int64_t ldb,
                           const float* scale_b, void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N, int K,
                           int epilogue, int* status, cudaStream_t stream) {
  if (epilogue == KD_EPI_QKV) return set_error(KD_ERR_ARGUMENT, "gemm: the QKV epilogue is kd_qkv_projection_fp8");
  return gemm_common(A, lda, B, ldb, C, ldc, R, ldr, scale_a, scale_b, M, N, K, epilogue, 1, status, stream);
}
