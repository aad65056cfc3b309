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
// Persistent CTAs, as many as fit on the device (two per SM for head dim <= 128), take work items: a 128-query tile of
// one sequence for one query head (and value slice). Each CTA's first item is its index; the rest come from a
// device counter that the last CTA to finish returns to zero. Items are ordered sequence by sequence, each
// sequence's tiles from the last (the most expensive when causal) to the first, query heads innermost, so the heads
// of one key/value group run at about the same time and share the key/value reads in L2; a sequence whose keys and
// values outgrow L2 runs key/value head by key/value head (next_item). Head dim 512 (Gemma 4's
// global layers) exceeds tensor memory for a whole output row block next to the scores, so its output is computed in
// two 256-wide value slices (separate items), each forming the full scores (K and V single-buffered to fit the
// 128 KB query tile). 6 warps:
//   warp 0      work fetch + TMA producer: publishes each item to the other roles through a two-slot ring, then its
//               Q tile and its K and V tiles through a ring (2 stages; 1 for head dim 512) counted across items;
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into one of 2-4 TMEM score buffers (as many as the allocation
//               holds beside O), then O += P_j V_j with
//               P_j read from TMEM (A operand, written over S_j) and V_j as an MN-major B operand from shared memory;
//               an item's first S can run while the previous item's epilogue reads O;
//   warps 2..5  softmax, one query row per thread (its TMEM lane): scores -> masked, scaled, exp2 against a running
//               maximum, bf16 probabilities stored back to TMEM. O is rescaled only when the row maximum grows by
//               more than 2^8 (the exponent base stays stale otherwise, which is exact: O and the row sum share it);
//               at the end of an item they normalize O, apply the optional output gate (its tile brought into L2 by
//               the producer) and store bf16 rows.
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
  static constexpr int BASE_SMEM = Q_BYTES + STAGES * STAGE_BYTES + 1024 + 512;  // + alignment, items, barriers
  // The epilogue's staging areas: 32 rows x 32 columns of bf16 (2 KB) per softmax warp, for coalesced gate loads and
  // output stores; left out where shared memory has no room (head dim 512 stores row by row).
  static constexpr bool STAGED = BASE_SMEM + 4 * 2048 <= 227 * 1024;
  static constexpr int EPI_BYTES = STAGED ? 4 * 2048 : 0;
  static constexpr int SMEM = BASE_SMEM + EPI_BYTES;
  // Tensor-memory columns (fp32): O [0, DV), then two score buffers of BN; the bf16 probabilities P_j overwrite the
  // first BN / 2 columns of their own score buffer once the softmax has read it.
  static constexpr int O_COL = 0;
  static constexpr int S_COL = DV;
  static constexpr int TMEM_COLS = DV + 2 * BN <= 256 ? 256 : 512;
  // Score buffers: as many as the allocation holds beyond O (at most 4). Score tile G goes to buffer G % NS, whose
  // probabilities P_{G-NS} were read by P_{G-NS} V_{G-NS}; more buffers leave that product more time to complete.
  static constexpr int NS = (TMEM_COLS - DV) / BN < 4 ? (TMEM_COLS - DV) / BN : 4;
  // Two CTAs per SM (their softmax and MMA phases interleave) when shared and tensor memory allow it.
  static constexpr int CTAS_PER_SM = (2 * SMEM <= 227 * 1024 && 2 * TMEM_COLS <= 512) ? 2 : 1;
  static_assert(NS >= 2 && S_COL + NS * BN <= TMEM_COLS, "tensor memory budget");
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
  int* sched;  // [2]: the work counter beyond the first item of each CTA, and the number of CTAs finished
};

// One unit of work: a 128-query tile of one sequence for one query head and value slice.
struct Item {
  int q0, lq, k0, lk;       // the sequence's first query and key rows, its query and key lengths
  int qs;                   // the tile's first query within the sequence
  int head, slice;
  int first_tile, n_tiles;  // visible key tiles; n_tiles < 0: no more work
  int pad[3];
};

constexpr int THREADS = 192;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale O when the row maximum grows by more than 2^8


// 2^x with the hardware exponential (ex2.approx: relative error ~2^-22; the probabilities are rounded to bf16).
KD_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Keys and values of a sequence (all its key/value heads) beyond which its items run key/value head by key/value head:
// half of the 126 MB L2.
constexpr int64_t KV_MAJOR_BYTES = 64ll << 20;

// The next work item: item `idx` in the order sequences (pack order) > query tiles of the sequence, from its last
// (the most expensive when causal) to its first > query heads > value slices, so that the heads of one key/value
// group run at about the same time and share the key/value reads in L2, and the launch ends on short items. A
// sequence whose keys and values exceed KV_MAJOR_BYTES with no left window bound runs key/value head by key/value
// head instead (tiles from the last, the group's query heads innermost): the CTAs running at one time then stream one
// or two heads' keys and values, which stay in L2 however long the sequence (all heads of a 131,072-token sequence at
// once re-read them from DRAM: 520 GB per launch at a 51% L2 hit rate, 950 TFLOP/s; head by head 1,110). (cs, cbase) is
// the caller's cursor: a sequence and the number of query tiles before it. A CTA's item indices only grow, so the
// cursor only moves forward.
template <int HD, int DV>
KD_DEVICE void next_item(const Args& a, int idx, int& cs, int& cbase, Item& w) {
  using C = Cfg<HD, DV>;
  constexpr int BM = C::BM, BN = C::BN;
  const int rest = idx / C::SLICES;
  w.slice = idx - rest * C::SLICES;
  const int coarse = rest / a.hq;  // a sequence of n query tiles holds n * hq consecutive values of `rest`
  w.n_tiles = -1;
  while (cs < a.num_seqs) {
    const int qa = a.cu_q[cs], qb = a.cu_q[cs + 1];
    const int n = (qb - qa + BM - 1) / BM;
    if (coarse < cbase + n) {
      const int local = rest - cbase * a.hq;  // the item within its sequence
      const int lk = a.cu_k[cs + 1] - a.cu_k[cs];
      int tile;                                // 0: the sequence's last query tile
      if (a.left < 0 && (int64_t)lk * a.hkv * HD * 4 > KV_MAJOR_BYTES) {
        const int group = a.hq / a.hkv;
        const int kvh = local / (n * group);
        const int within = local - kvh * (n * group);
        tile = within / group;
        w.head = kvh * group + (within - tile * group);
      } else {
        tile = local / a.hq;
        w.head = local - tile * a.hq;
      }
      w.q0 = qa;
      w.lq = qb - qa;
      w.k0 = a.cu_k[cs];
      w.lk = a.cu_k[cs + 1] - w.k0;
      w.qs = (n - 1 - tile) * BM;
      const int off = w.lk - w.lq;  // end alignment of queries to keys
      const int qe = min(w.qs + BM, w.lq);
      int kmin = 0, kmax = w.lk - 1;
      if (a.left >= 0) kmin = max(0, w.qs + off - a.left);
      if (a.right >= 0) kmax = min(w.lk - 1, qe - 1 + off + a.right);
      w.first_tile = kmin / BN;
      w.n_tiles = kmax < kmin ? 0 : kmax / BN - w.first_tile + 1;
      return;
    }
    cbase += n;
    ++cs;
  }
}

// 16 bytes of the gate tensor (read-only for the kernel's lifetime).
KD_DEVICE uint4 load_gate16(const __nv_bfloat16* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Two gated outputs: bf16 pairs o and g -> bf16(o * sigmoid(g)) (the product rounded once). sigmoid(x) =
// 1 / (1 + 2^(-x log2 e)): the exponential on the MUFU, the reciprocal by Newton steps on the FMA pipe (the epilogue
// would otherwise issue two MUFU operations per output): a first guess with the exponent reflected (bits
// 254 * 2^23 - bits(y), within 12.5% of 1 / y for y in [1, 2^126]) and three steps r <- r + r (1 - y r), relative
// error 0.125 -> 1.6e-2 -> 2.4e-4 -> 6e-8.
KD_DEVICE uint32_t gate_pair(uint32_t o, uint32_t g) {
  const float2 ov = unpack_bf16x2(o), gv = unpack_bf16x2(g);
  const float2 xs = fma2(gv, make_float2(-1.4426950408889634f, -1.4426950408889634f), make_float2(0.f, 0.f));
  const float2 e = make_float2(fast_exp2(fminf(xs.x, 126.f)), fast_exp2(fminf(xs.y, 126.f)));
  const float2 y = add2(e, make_float2(1.f, 1.f));  // in [1, 2^126]
  float2 r = make_float2(__int_as_float(0x7F000000 - __float_as_int(y.x)),
                         __int_as_float(0x7F000000 - __float_as_int(y.y)));
  const float2 ny = make_float2(-y.x, -y.y);
#pragma unroll
  for (int i = 0; i < 3; ++i) r = fma2(r, fma2(ny, r, make_float2(1.f, 1.f)), r);
  return pack_bf16x2(ov.x * r.x, ov.y * r.y);
}

// The epilogue of a 128-row tile, one warp's 32 rows: O / l, the optional output gate, bf16 rows. Through the warp's
// 2 KB staging area (32 rows x 64 bytes: row i at 64 i, its 16-byte piece p at slot (p + i / 2) % 4, conflict-free
// both for a row per lane and for 8 rows of 4 lanes): each lane writes its row's normalized bf16 values, then reads
// back 4 pieces of 8 rows, multiplies them by the gate pieces it loaded (coalesced, two 32-column chunks ahead) and
// stores 64 contiguous bytes per row. The gate rows (brought into L2 by the producer) are read before the wait on
// `done` (the item's last O += P V); without visible keys (n == 0) the output is 0 and needs no gate.
template <int DV>
KD_DEVICE bool staged_epilogue(const Args& a, const Item& w, int n, int64_t col0, uint8_t* ws, int quarter, int lane,
                               uint32_t o_addr, uint64_t* done, uint32_t parity, float l_sum) {
  const bool gated = a.gate != nullptr && n > 0;
  const int tr_row = lane >> 2, tr_piece = lane & 3;  // the transposed access: rows tr_row + 8 m, one piece
  const int wrow0 = w.qs + quarter * 32;              // the warp's first row within the sequence
  auto at = [&](int i, int p) -> uint4* {
    return reinterpret_cast<uint4*>(ws + i * 64 + (((p + (i >> 1)) & 3) << 4));
  };
  constexpr int NCH = DV / 32;
  uint4 g4[2][4];
  auto load_gates = [&](int cc) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int row = wrow0 + tr_row + 8 * m;
      g4[cc & 1][m] = row < w.lq ? load_gate16(a.gate + (int64_t)(w.q0 + row) * a.ldg + col0 + cc * 32 + tr_piece * 8)
                                 : make_uint4(0, 0, 0, 0);
    }
  };
  if (gated) {
    load_gates(0);
    if (NCH > 1) load_gates(1);
  }
  if (n > 0) {
    if (!mbar_wait(done, parity, a.status)) return false;
    tc_fence_after();
  }
  const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll
  for (int cc = 0; cc < NCH; ++cc) {
    {  // this row's 32 columns: bf16(o / l)
      uint32_t t[32];
      if (n > 0) {
        tmem_ld32(o_addr + cc * 32, t);  // warp-collective
        tmem_ld_wait_regs(t);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) t[e] = 0u;
      }
#pragma unroll
      for (int pc = 0; pc < 4; ++pc) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pk[e] = pack_bf16x2(__uint_as_float(t[8 * pc + 2 * e]) * inv, __uint_as_float(t[8 * pc + 2 * e + 1]) * inv);
        *at(lane, pc) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    __syncwarp();
#pragma unroll
    for (int m = 0; m < 4; ++m) {  // 8 rows x 4 pieces out
      const int row = wrow0 + tr_row + 8 * m;
      uint4 x = *at(tr_row + 8 * m, tr_piece);
      if (gated) {  // Qwen's output gate: bf16(o) * sigmoid(gate), rounded once
        const uint4 gq = g4[cc & 1][m];
        x.x = gate_pair(x.x, gq.x);
        x.y = gate_pair(x.y, gq.y);
        x.z = gate_pair(x.z, gq.z);
        x.w = gate_pair(x.w, gq.w);
      }
      if (row < w.lq)
        *reinterpret_cast<uint4*>(a.out + (int64_t)(w.q0 + row) * a.ldo + col0 + cc * 32 + tr_piece * 8) = x;
    }
    if (gated && cc + 2 < NCH) load_gates(cc + 2);
    __syncwarp();
  }
  return true;
}

template <int HD, int DV>
__global__ void __launch_bounds__(THREADS, Cfg<HD, DV>::CTAS_PER_SM)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_g, Args a) {
  using C = Cfg<HD, DV>;
  constexpr int BM = C::BM, BN = C::BN, ST = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem;
  uint8_t* s_kv = smem + C::Q_BYTES;  // stage s: K at s * STAGE_BYTES, V right after
  uint8_t* s_epi = smem + C::Q_BYTES + ST * C::STAGE_BYTES;  // [4 warps][2 KB] when staged
  Item* items = reinterpret_cast<Item*>(s_epi + C::EPI_BYTES);  // [2]: the work item ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(items + 2);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;         // released by an item's last S = Q K^T
  uint64_t* k_full = bars + 2;          // [ST]
  uint64_t* v_full = k_full + ST;       // [ST]
  uint64_t* k_empty = v_full + ST;      // [ST]: released by the S = Q K^T that read the stage's K
  uint64_t* v_empty = k_empty + ST;     // [ST]: released by the O += P V that read its V
  constexpr int NS = C::NS;
  uint64_t* s_full = v_empty + ST;      // [NS]
  uint64_t* p_full = s_full + NS;       // [NS]
  uint64_t* pv_done = p_full + NS;      // [NS]
  uint64_t* item_full = pv_done + NS;   // [2]
  uint64_t* item_empty = item_full + 2; // [2]: read by the MMA thread and the four softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&item_full[b], 1);
      mbar_init(&item_empty[b], 5);
    }
    for (int b = 0; b < NS; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&pv_done[b], 1);
    }
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
  const int group = a.hq / a.hkv;

  // Every role walks the same item sequence; K/V ring slots, score buffers and the Q buffer are counted across items.
  if (warp == 0) {
    // ------------------------------------------------------------ work fetch + TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      if (a.gate) tma_prefetch_desc(&map_g);
      int cs = 0, cbase = 0;
      uint32_t slot = 0, nq = 0;
      for (uint32_t it = 0;; ++it) {
        Item w;
        const int idx = it == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(a.sched, 1);
        next_item<HD, DV>(a, idx, cs, cbase, w);
        if (!mbar_wait(&item_empty[it & 1], ((it >> 1) & 1) ^ 1, a.status)) goto done;
        items[it & 1] = w;
        mbar_arrive(&item_full[it & 1]);
        if (w.n_tiles < 0) break;
        const int kvh = w.head / group;
        const int vcol = w.slice * DV;
        if (w.n_tiles > 0) {
          if (!mbar_wait(q_empty, (nq & 1) ^ 1, a.status)) goto done;
          ++nq;
          mbar_arrive_expect_tx(q_full, C::Q_BYTES);
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_2d(&map_q, q_full, s_q + c * C::Q_CHUNK, w.head * HD + c * 64, w.q0 + w.qs);
        }
        // Keys run one tile ahead of values: a tile's keys wait only for the S = Q K^T that last read their stage,
        // not behind the previous tile's values (which wait for an O += P V).
        for (int j = 0; j <= w.n_tiles; ++j) {
          if (j < w.n_tiles) {
            const uint32_t sl = slot + j;
            const int st = sl % ST;
            uint8_t* sk = s_kv + st * C::STAGE_BYTES;
            if (!mbar_wait(&k_empty[st], ((sl / ST) & 1) ^ 1, a.status)) goto done;
            mbar_arrive_expect_tx(&k_full[st], C::K_BYTES);
            for (int c = 0; c < C::CHUNKS; ++c)
              tma_load_2d(&map_k, &k_full[st], sk + c * C::KV_CHUNK, kvh * HD + c * 64,
                          w.k0 + (w.first_tile + j) * BN);
          }
          if (j >= 1) {
            const uint32_t sl = slot + j - 1;
            const int st = sl % ST;
            uint8_t* sv = s_kv + st * C::STAGE_BYTES + C::K_BYTES;
            if (!mbar_wait(&v_empty[st], ((sl / ST) & 1) ^ 1, a.status)) goto done;
            mbar_arrive_expect_tx(&v_full[st], C::V_BYTES);
            for (int c = 0; c < C::V_CHUNKS; ++c)
              tma_load_2d(&map_v, &v_full[st], sv + c * C::KV_CHUNK, kvh * HD + vcol + c * 64,
                          w.k0 + (w.first_tile + j - 1) * BN);
          }
        }
        slot += w.n_tiles > 0 ? w.n_tiles : 0;
        // Qwen's output gate for this tile, into L2 while the last key tiles run: the epilogue reads it from there.
        if (a.gate && w.n_tiles > 0)
          for (int c = 0; c < C::V_CHUNKS; ++c) tma_prefetch_l2(&map_g, w.head * HD + vcol + c * 64, w.q0 + w.qs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_s = mma_idesc(1, BM, BN);          // bf16, K-major A and B
      constexpr uint32_t idesc_o = mma_idesc(1, BM, DV, 1);       // bf16, A from TMEM, MN-major B (V)
      const uint32_t sq = smem_u32(s_q);
      uint32_t slot = 0, g = 0, nq = 0;
      for (uint32_t it = 0;; ++it) {
        if (!mbar_wait(&item_full[it & 1], (it >> 1) & 1, a.status)) goto done;
        const int n = items[it & 1].n_tiles;
        mbar_arrive(&item_empty[it & 1]);
        if (n < 0) break;
        if (n == 0) continue;
        if (!mbar_wait(q_full, nq & 1, a.status)) goto done;
        ++nq;
        // S_G = Q K^T of the item's tile j (G = g + j counts tiles across items) into score buffer G % NS, whose
        // probabilities P_{G-NS} were read by P_{G-NS} V_{G-NS}: that product must have completed.
        auto issue_s = [&](int j) -> bool {
          const uint32_t G = g + j, sl = slot + j;
          const int st = sl % ST;
          if (G >= NS && !mbar_wait(&pv_done[G % NS], ((G - NS) / NS) & 1, a.status)) return false;
          if (!mbar_wait(&k_full[st], (sl / ST) & 1, a.status)) return false;
          tc_fence_after();
          const uint32_t sk = smem_u32(s_kv + st * C::STAGE_BYTES);
          const uint32_t d = tmem + C::S_COL + (G % NS) * BN;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const int c = kk / 4, w = (kk % 4) * 32;
            mma_f16_ss(d, sw128_kmajor_desc(sq + c * C::Q_CHUNK + w), sw128_kmajor_desc(sk + c * C::KV_CHUNK + w),
                       idesc_s, kk > 0);
          }
          mma_commit(&k_empty[st]);  // the stage's K is free once these MMAs have read it
          mma_commit(&s_full[G % NS]);
          if (j == n - 1) mma_commit(q_empty);  // Q is free once the item's last S has completed
          return true;
        };
        if (!issue_s(0)) goto done;
        for (int j = 0; j < n; ++j) {
          // S_{j+1} first, so the softmax of tile j+1 can start while P_j V_j runs.
          if (j + 1 < n && !issue_s(j + 1)) goto done;
          const uint32_t G = g + j, sl = slot + j;
          const int st = sl % ST;
          if (!mbar_wait(&p_full[G % NS], (G / NS) & 1, a.status)) goto done;
          if (!mbar_wait(&v_full[st], (sl / ST) & 1, a.status)) goto done;
          tc_fence_after();
          const uint32_t sv = smem_u32(s_kv + st * C::STAGE_BYTES + C::K_BYTES);
          const uint32_t p = tmem + C::S_COL + (G % NS) * BN;  // P_G over the first BN / 2 columns of S_G
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)  // 16 keys per instruction: 8 columns of bf16 pairs, 2 KB of V rows
            mma_f16_ts(tmem + C::O_COL, p + kk * 8, sw128_mnmajor_desc(sv + kk * 2048, C::KV_CHUNK), idesc_o,
                       (j | kk) != 0);
          mma_commit(&v_empty[st]);
          mma_commit(&pv_done[G % NS]);
        }
        slot += n;
        g += n;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t g = 0;
    for (uint32_t it = 0;; ++it) {
      if (!mbar_wait(&item_full[it & 1], (it >> 1) & 1, a.status)) goto done;
      const Item w = items[it & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[it & 1]);
      if (w.n_tiles < 0) break;
      const int n = w.n_tiles;
      const int off = w.lk - w.lq;
      const int qe = min(w.qs + BM, w.lq);
      const int qi = w.qs + r + off;  // the row's position on the key axis
      // the row's visible keys [key_lo, key_hi] (the mask of an edge tile is two compares and a select per key)
      const int key_lo = a.left >= 0 ? qi - a.left : INT_MIN / 2;
      const int key_hi = min(w.lk - 1, a.right >= 0 ? qi + a.right : INT_MAX / 2);
      float m_used = -INFINITY, l_sum = 0.f;  // running maximum (log2 units, possibly stale) and row sum
      for (int j = 0; j < n; ++j) {
        const uint32_t G = g + j;
        if (!mbar_wait(&s_full[G % NS], (G / NS) & 1, a.status)) goto done;
        tc_fence_after();
        const uint32_t s_addr = lane_base + C::S_COL + (G % NS) * BN;
        float sv[BN];
#pragma unroll
        for (int c = 0; c < BN; c += 64) {  // two loads in flight, one wait
          uint32_t t0[32], t1[32];
          tmem_ld32(s_addr + c, t0);
          tmem_ld32(s_addr + c + 32, t1);
          tmem_ld_wait_regs(t0, t1);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[c + e] = __uint_as_float(t0[e]);
            sv[c + 32 + e] = __uint_as_float(t1[e]);
          }
        }
        const int n0 = (w.first_tile + j) * BN;
        // Only tiles that cross the causal diagonal, the window's left edge or the sequence end need a mask; the
        // condition is the same for every row of the tile.
        const bool edge = (n0 + BN > w.lk) || (a.right >= 0 && n0 + BN - 1 > w.qs + off + a.right) ||
                          (a.left >= 0 && n0 < qe - 1 + off - a.left);
        if (edge) {
          const int lo = key_lo - n0, hi = key_hi - n0;
#pragma unroll
          for (int e = 0; e < BN; ++e) sv[e] = (e >= lo && e <= hi) ? sv[e] : -INFINITY;
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
          if (!mbar_wait(&pv_done[(G - 1) % NS], ((G - 1) / NS) & 1, a.status)) goto done;
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
          tmem_st32(s_addr + c / 2, pk);  // P_G over the score columns this thread has already read
        }
        const float2 ps = add2(add2(part[0], part[1]), add2(part[2], part[3]));
        l_sum += ps.x + ps.y;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[G % NS]);
      }
      // ---- epilogue: O / l, optional gate, bf16 rows. The gate rows (in L2 by now) are read while the last product
      // completes; without visible keys the output is 0 and needs no gate.
      const bool gated = a.gate != nullptr && n > 0;
      const int64_t col0 = (int64_t)w.head * HD + w.slice * DV;
      constexpr int GC = DV < 128 ? DV : 128;  // gate columns held in registers at a time
      if constexpr (C::STAGED) {
        const uint32_t gl = n > 0 ? g + n - 1 : 0;  // the item's last tile
        if (!staged_epilogue<DV>(a, w, n, col0, s_epi + quarter * 2048, quarter, lane, lane_base + C::O_COL,
                                 &pv_done[gl % NS], (gl / NS) & 1, l_sum))
          goto done;
      } else {
        const int row = w.qs + r;
        const bool live = row < w.lq;
        const __nv_bfloat16* grow = gated && live ? a.gate + (int64_t)(w.q0 + row) * a.ldg + col0 : nullptr;
        uint4 g4[GC / 8];
#pragma unroll
        for (int e = 0; e < GC / 8; ++e) g4[e] = grow ? load_gate16(grow + 8 * e) : make_uint4(0, 0, 0, 0);
        if (n > 0) {
          const uint32_t G = g + n - 1;
          if (!mbar_wait(&pv_done[G % NS], (G / NS) & 1, a.status)) goto done;
          tc_fence_after();
        }
        const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
        __nv_bfloat16* orow = a.out + (int64_t)(w.q0 + row) * a.ldo + col0;
#pragma unroll
        for (int h = 0; h < DV; h += GC) {
          if (h > 0) {
#pragma unroll
            for (int e = 0; e < GC / 8; ++e) g4[e] = grow ? load_gate16(grow + h + 8 * e) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int c = 0; c < GC; c += 32) {
            uint32_t t[32];
            if (n > 0) {
              tmem_ld32(lane_base + C::O_COL + h + c, t);  // warp-collective: every lane loads, valid rows store
              tmem_ld_wait_regs(t);
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) t[e] = 0u;
            }
            if (live) {
              uint32_t packed[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                float v0 = bf16_round(__uint_as_float(t[2 * e]) * inv);
                float v1 = bf16_round(__uint_as_float(t[2 * e + 1]) * inv);
                if (grow) {
                  const uint4 q4 = g4[(c + 2 * e) / 8];
                  const int k = ((c + 2 * e) % 8) / 2;
                  const float2 gv = unpack_bf16x2(k == 0 ? q4.x : k == 1 ? q4.y : k == 2 ? q4.z : q4.w);
                  v0 *= sigmoid(gv.x);
                  v1 *= sigmoid(gv.y);
                }
                packed[e] = pack_bf16x2(v0, v1);
              }
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
                *reinterpret_cast<uint4*>(orow + h + c + 8 * q4) =
                    make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
            }
          }
        }
      }
      g += n > 0 ? n : 0;
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
  if (threadIdx.x == 0) {
    // The last CTA to finish returns the work counter to zero for the next launch: every CTA stopped fetching work
    // before counting itself here.
    __threadfence();
    if (atomicAdd(a.sched + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(a.sched, 0);
      atomicExch(a.sched + 1, 0);
    }
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
  // Work items: sum over sequences of ceil(Lq / BM) query tiles <= total_q / BM + num_seqs, times heads and slices.
  // Persistent CTAs (as many as fit on the device at once) take them in order, the first one each by its index and
  // the rest from the shared counter.
  const int64_t items = (total_q / C::BM + a.num_seqs) * a.hq * C::SLICES;
  if (items > 0x7fffffff - 4096) return set_error(KD_ERR_ARGUMENT, "attention: too many work items");
  const int64_t resident = (int64_t)num_sms(dev) * C::CTAS_PER_SM;
  const int grid = (int)(items < resident ? items : resident);
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
                                   int window_right, int* status, int* sched, cudaStream_t stream) {
  (void)max_q;
  if (num_seqs < 0 || total_q < 0 || total_k < 0) return set_error(KD_ERR_ARGUMENT, "attention: negative sizes");
  if (num_seqs == 0 || total_q == 0) return KD_OK;
  if (num_heads_q <= 0 || num_heads_kv <= 0 || num_heads_q % num_heads_kv)
    return set_error(KD_ERR_ARGUMENT, "attention: query heads must be a multiple of key/value heads");
  if (!q || !k || !v || !out || !cu_q || !cu_k || !status || !sched) return set_error(KD_ERR_ARGUMENT, "attention: null pointer");
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
  a.sched = sched;
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
