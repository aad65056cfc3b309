// Varlen block-diagonal attention forward (GQA, causal / sliding window / bidirectional), flash-attention style:
// one CTA per (query tile of one sequence, query head), K/V tiles streamed through a double-buffered shared-memory
// ring with cp.async, S = Q K^T and O += P V on the tensor cores (warp-level bf16 MMA, fp32 accumulation), online
// softmax in registers, optional fused output gate.
//
// Replaces torch varlen_attn / flash-attention calls: families/qwen/packed.py:123-124 (causal, scale hd^-0.5, GQA),
// families/gemma/sliding_attention.py:183-191 (window (W-1, 0), scale 1.0) and the global layers' causal attention
// (families/gemma/packed.py:196-220). The visibility rule is the varlen contract with end alignment (the reference's
// tests/test_gemma_blocks.py:28-43): query i of a sequence sees key j iff
//   i + (Lk - Lq) - left <= j <= i + (Lk - Lq) + right.
// Sequence boundaries (cu_q, cu_k) are read from device memory when the kernel runs, so a captured graph serves any
// pack composition of the same token count.
#include "common.cuh"
#include "kd_internal.h"

namespace kd {
namespace attn {

constexpr int BN = 64;  // keys per tile

struct Args {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* out;
  const __nv_bfloat16* gate;
  int64_t ldq, ldk, ldv, ldo, ldg;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_seqs;
  int hq, hkv;
  float scale_log2;  // softmax scale * log2(e)
  int left, right;
};

KD_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
KD_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KD_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

KD_DEVICE void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
KD_DEVICE void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

KD_DEVICE void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a [rows][HD] bf16 tile, chunks XOR-swizzled by row % 8 so that
// the 8 rows an ldmatrix reads hit 8 different bank groups.
template <int HD>
KD_DEVICE uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * HD * 2 + ((chunk ^ (row & 7)) << 4));
}

// Loads rows [r0, r0 + ROWS) of a [T, ld] bf16 matrix (head columns at `col`) into a swizzled tile; rows >= limit
// are zero-filled.
template <int HD, int ROWS, int THREADS>
KD_DEVICE void load_tile(uint32_t smem, const __nv_bfloat16* base, int64_t ld, int r0, int limit) {
  constexpr int CHUNKS = HD / 8;
  for (int i = threadIdx.x; i < ROWS * CHUNKS; i += THREADS) {
    const int row = i / CHUNKS;
    const int chunk = i % CHUNKS;
    const bool valid = r0 + row < limit;
    const __nv_bfloat16* src = base + (int64_t)(valid ? r0 + row : 0) * ld + chunk * 8;
    cp_async16(smem + swz<HD>(row, chunk), src, valid);
  }
}

template <int HD, int BM>
__global__ void __launch_bounds__(BM * 2, 1) attention_kernel(Args a) {
  constexpr int WARPS = BM / 16;
  constexpr int THREADS = WARPS * 32;
  constexpr int DT = HD / 8;  // 8-wide output tiles along the head dim
  constexpr int NT = BN / 8;  // 8-wide score tiles along the keys
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_q = smem_u32(smem);
  const uint32_t s_kv = s_q + BM * HD * 2;  // [stage][K | V], each BN x HD
  constexpr uint32_t KV_TILE = BN * HD * 2;

  // ---- find this CTA's (sequence, query tile): tiles are numbered sequence by sequence from the device bounds.
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
      qs = (n - 1 - tile) * BM;  // the last (most expensive when causal) tiles first
      break;
    }
    tile -= n;
  }
  if (seq < 0) return;
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int off = lk - lq;  // end alignment
  const int qe = min(qs + BM, lq);

  // Key range any query of this tile may see.
  int kmin = 0, kmax = lk - 1;
  if (a.left >= 0) kmin = max(0, qs + off - a.left);
  if (a.right >= 0) kmax = min(lk - 1, qe - 1 + off + a.right);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const __nv_bfloat16* qbase = a.q + (int64_t)q0 * a.ldq + (int64_t)head * HD;
  const __nv_bfloat16* kbase = a.k + (int64_t)k0 * a.ldk + (int64_t)kvh * HD;
  const __nv_bfloat16* vbase = a.v + (int64_t)k0 * a.ldv + (int64_t)kvh * HD;

  float o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  const int first_tile = kmax < kmin ? 1 : kmin / BN;
  const int last_tile = kmax < kmin ? 0 : kmax / BN;

  load_tile<HD, BM, THREADS>(s_q, qbase, a.ldq, qs, lq);
  if (first_tile <= last_tile) {
    load_tile<HD, BN, THREADS>(s_kv, kbase, a.ldk, first_tile * BN, lk);
    load_tile<HD, BN, THREADS>(s_kv + KV_TILE, vbase, a.ldv, first_tile * BN, lk);
  }
  cp_async_commit();

  const int row_a = qs + warp * 16 + g;  // this thread's two query rows (within the sequence)
  const int row_b = row_a + 8;

  for (int kt = first_tile; kt <= last_tile; ++kt) {
    const int stage = (kt - first_tile) & 1;
    if (kt < last_tile) {  // prefetch the next K/V tile into the other stage
      const uint32_t nxt = s_kv + (stage ^ 1) * 2 * KV_TILE;
      load_tile<HD, BN, THREADS>(nxt, kbase, a.ldk, (kt + 1) * BN, lk);
      load_tile<HD, BN, THREADS>(nxt + KV_TILE, vbase, a.ldv, (kt + 1) * BN, lk);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint32_t sk = s_kv + stage * 2 * KV_TILE;
    const uint32_t sv = sk + KV_TILE;

    // ---- S = Q K^T for this warp's 16 rows x BN keys
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldmatrix_x4(s_q + swz<HD>(r, c), a0, a1, a2, a3);
      }
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = j * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(sk + swz<HD>(r, c), b0, b1, b2, b3);
        mma_bf16(s[j], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[j + 1], a0, a1, a2, a3, b2, b3);
      }
    }

    // ---- mask (only tiles that cross a boundary), online softmax
    const int n0 = kt * BN;
    const bool edge = (n0 + BN - 1 > qs + off + (a.right >= 0 ? a.right : lk)) ||
                      (a.left >= 0 && n0 < qe - 1 + off - a.left) || (n0 + BN > lk);
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * a.scale_log2;
        if (edge) {
          const int key = n0 + j * 8 + 2 * t + (e & 1);
          const int qi = (e < 2 ? row_a : row_b) + off;
          bool ok = key < lk;
          if (a.right >= 0) ok = ok && key <= qi + a.right;
          if (a.left >= 0) ok = ok && key >= qi - a.left;
          if (!ok) x = -INFINITY;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], base[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      base[r] = mx[r] == -INFINITY ? 0.f : mx[r];  // a fully masked row so far keeps zeros
      corr[r] = exp2f(m_run[r] - base[r]);
      m_run[r] = mx[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t p[NT][2];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float p0 = exp2f(s[j][0] - base[0]);
      const float p1 = exp2f(s[j][1] - base[0]);
      const float p2 = exp2f(s[j][2] - base[1]);
      const float p3 = exp2f(s[j][3] - base[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      p[j][0] = pack_bf16x2(p0, p1);
      p[j][1] = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int i = 0; i < DT; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }

    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint32_t a0 = p[2 * kk][0], a1 = p[2 * kk][1], a2 = p[2 * kk + 1][0], a3 = p[2 * kk + 1][1];
#pragma unroll
      for (int i = 0; i < DT; i += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = i + (lane >> 4);
        ldmatrix_x4_trans(sv + swz<HD>(r, c), b0, b1, b2, b3);
        mma_bf16(o[i], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[i + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // this stage is overwritten by the prefetch two iterations on
  }
  cp_async_wait<0>();

  // ---- normalize, gate, store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  const float inv[2] = {l_run[0] > 0.f ? 1.f / l_run[0] : 0.f, l_run[1] > 0.f ? 1.f / l_run[1] : 0.f};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r == 0 ? row_a : row_b;
    if (row >= lq) continue;
    __nv_bfloat16* orow = a.out + (int64_t)(q0 + row) * a.ldo + (int64_t)head * HD;
    const __nv_bfloat16* grow = a.gate ? a.gate + (int64_t)(q0 + row) * a.ldg + (int64_t)head * HD : nullptr;
#pragma unroll
    for (int i = 0; i < DT; ++i) {
      const int d = i * 8 + 2 * t;
      float v0 = bf16_round(o[i][2 * r] * inv[r]);
      float v1 = bf16_round(o[i][2 * r + 1] * inv[r]);
      if (grow) {  // Qwen's output gate: bf16(o) * sigmoid(gate), rounded once
        const float2 gv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(grow + d));
        v0 *= sigmoid(gv.x);
        v1 *= sigmoid(gv.y);
      }
      *reinterpret_cast<uint32_t*>(orow + d) = pack_bf16x2(v0, v1);
    }
  }
}

template <int HD, int BM>
int launch(const Args& a, int64_t total_q, int num_seqs, cudaStream_t stream) {
  constexpr int SMEM = BM * HD * 2 + 2 * 2 * BN * HD * 2;
  auto kernel = attention_kernel<HD, BM>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KD_ERR_ARGUMENT;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return record_cuda_error(e, "attention: cudaFuncSetAttribute");
    configured[dev] = true;
  }
  // Upper bound on query tiles over all sequences: sum(ceil(Lq / BM)) <= total_q / BM + num_seqs.
  const int64_t tiles = total_q / BM + num_seqs;
  if (tiles > 0x7fffffff) return set_error(KD_ERR_ARGUMENT, "attention: too many query tiles");
  dim3 grid((unsigned)tiles, (unsigned)a.hq);
  kernel<<<grid, BM * 2, SMEM, stream>>>(a);
  return record_cuda_error(cudaGetLastError(), "attention: launch");
}

}  // namespace attn
}  // namespace kd

using namespace kd;

extern "C" int kd_attention_varlen(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                   void* out, int64_t ldo, const void* gate, int64_t ldg, const int32_t* cu_q,
                                   const int32_t* cu_k, int num_seqs, int max_q, int64_t total_q, int num_heads_q,
                                   int num_heads_kv, int head_dim, float scale, int window_left, int window_right,
                                   int* status, cudaStream_t stream) {
  (void)max_q;
  (void)status;
  if (num_seqs < 0 || total_q < 0) return set_error(KD_ERR_ARGUMENT, "attention: negative sizes");
  if (num_seqs == 0 || total_q == 0) return KD_OK;
  if (num_heads_q <= 0 || num_heads_kv <= 0 || num_heads_q % num_heads_kv)
    return set_error(KD_ERR_ARGUMENT, "attention: query heads must be a multiple of key/value heads");
  if (!q || !k || !v || !out || !cu_q || !cu_k) return set_error(KD_ERR_ARGUMENT, "attention: null pointer");
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(q) || !a16(k) || !a16(v) || !a16(out) || (gate && !a16(gate)) || ldq % 8 || ldk % 8 || ldv % 8 ||
      ldo % 8 || (gate && ldg % 8))
    return set_error(KD_ERR_ARGUMENT, "attention: pointers and row strides must be 16-byte aligned");
  if (ldq < (int64_t)num_heads_q * head_dim || ldo < (int64_t)num_heads_q * head_dim ||
      ldk < (int64_t)num_heads_kv * head_dim || ldv < (int64_t)num_heads_kv * head_dim)
    return set_error(KD_ERR_ARGUMENT, "attention: row strides smaller than heads x head_dim");
  attn::Args a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
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
  switch (head_dim) {
    case 64:
      return attn::launch<64, 128>(a, total_q, num_seqs, stream);
    case 128:
      return attn::launch<128, 128>(a, total_q, num_seqs, stream);
    case 256:
      return attn::launch<256, 64>(a, total_q, num_seqs, stream);
    default:
      return set_error(KD_ERR_ARGUMENT, "attention: head_dim must be 64, 128 or 256");
  }
}
