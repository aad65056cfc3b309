/* libkd_b200 — the C ABI of the B200-native (sm_100a) packed prefill forward of karpo-decision.
 *
 * Every entry point takes device pointers, element strides, sizes and a cudaStream_t, launches on that stream and
 * returns an int status: KD_OK (0), or a negative code with a message kept for kd_last_error(). Arguments are checked
 * before anything is launched; a rejected call launches nothing. The library allocates no device memory at run time:
 * every buffer, scratch included, belongs to the caller, so the calls can be captured in CUDA graphs. The one
 * exception is kd_qkv_projection_noalloc, whose rotary scratch is a static 16 MiB device array owned by the library
 * and shared by all its calls on a device (created when the library loads; its first call on a device looks up the
 * array's address and must come before any stream capture on that device).
 *
 * Pipelined kernels (GEMM, attention) also take `status`, a device int the caller zeroes once: a kernel whose
 * internal wait gives up (KD_WAIT_LIMIT_NS, 4 s) writes KD_DEVICE_TIMEOUT there and returns instead of hanging.
 *
 * Tensors are row-major. "bf16" is __nv_bfloat16, "e4m3" is __nv_fp8_e4m3 (one byte).
 *
 * Reference interfaces replaced (paths inside the karpo-decision source tree, src/karpo_decision/):
 *   the packed forward         families/qwen/packed.py:149-187, families/gemma/packed.py:228-323
 *   the pointwise ops          families/qwen/fused.py:17-48, families/gemma/fused.py:21-50
 *   the FP8 projections        serve/fp8.py:21-117, serve/qwen_fp8.py:20-56
 *   the readout head           model/readout.py:30-33
 */
#ifndef KD_B200_H
#define KD_B200_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------------------------- status codes */
#define KD_OK 0
#define KD_ERR_ARGUMENT (-1) /* an argument failed validation; nothing was launched */
#define KD_ERR_CUDA (-2)     /* a CUDA runtime call or launch failed */
#define KD_ERR_DRIVER (-3)   /* the driver entry point for TMA descriptors is unavailable or refused the tensor */
#define KD_DEVICE_TIMEOUT 1  /* written to a kernel's device status word when one of its waits gave up */

/* ---------------------------------------------------------------------------------------------- GEMM epilogues */
#define KD_EPI_STORE 0    /* C = bf16(acc) */
#define KD_EPI_RESIDUAL 1 /* C = bf16(R + bf16(acc)); R may alias C (h += x) */
#define KD_EPI_SWIGLU 2   /* B rows interleaved per 256: [128 gate | 128 up]; C[:, j] = silu(gate_j) * up_j */
#define KD_EPI_GEGLU 3    /* as SWIGLU with gelu_tanh (gelu_pytorch_tanh) */
#define KD_EPI_QKV 4      /* internal: the epilogue of kd_qkv_projection (not accepted by kd_gemm_*) */

/* ---------------------------------------------------------------------------------------------- norm weights */
#define KD_NORM_NONE 0    /* x * rsqrt(mean(x^2) + eps)                 (Gemma4RMSNorm without scale: v_norm) */
#define KD_NORM_WEIGHT 1  /* x * rsqrt(mean(x^2) + eps) * w             (Gemma4RMSNorm) */
#define KD_NORM_ONE_PLUS 2 /* x * rsqrt(mean(x^2) + eps) * (1 + w)      (Qwen3_5RMSNorm) */

/* Library version: major * 10000 + minor * 100 + patch. */
int kd_version(void);

/* Copies this thread's last error message (NUL-terminated, truncated to n bytes) into buf; returns its length. */
int kd_last_error(char* buf, size_t n);

/* A check of the bounded waits every pipelined kernel relies on: one launch with two waiters on a shared-memory
 * barrier that nothing arrives on. The first gives up after `limit_ns` (at most 1 s) and writes KD_DEVICE_TIMEOUT to
 * *status (a device int the caller zeroed); the second, allowed 64 x as long, gives up as soon as it sees that status.
 * elapsed[0], elapsed[1] (device int64) receive the nanoseconds each waited. The launch returns; the context stays
 * usable. No counterpart in the reference (its kernels come from libraries): the failure-detection test of this
 * library's own device waits. */
int kd_wait_selftest(int* status, int64_t limit_ns, int64_t* elapsed, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------- projections
 * C[M, N] = epilogue(A[M, K] . B[N, K]^T): tcgen05 MMA with fp32 accumulation in tensor memory.
 * Replaces nn.Linear (cuBLAS) in every projection: families/qwen/packed.py:113-125,147 (q/k/v/o, gate/up/down),
 * families/gemma/packed.py:185-193,254 and fused.py:96-98.
 * A, B: 16-byte aligned, lda/ldb (elements) with row pitch a multiple of 16 bytes; N % 32 == 0 (gated: % 256). */
int kd_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
                 int64_t ldr, int M, int N, int K, int epilogue, int* status, cudaStream_t stream);

/* FP8 e4m3 x e4m3 with fp32 accumulation: C = epilogue(acc * scale_a[row] * scale_b[col]) in bf16.
 * Replaces torch._scaled_mm with rowwise scales: serve/fp8.py:98-101 (Fp8Linear.forward), serve/qwen_fp8.py:38-42. */
int kd_gemm_fp8(const void* A, int64_t lda, const float* scale_a, const void* B, int64_t ldb, const float* scale_b,
                void* C, int64_t ldc, const void* R, int64_t ldr, int M, int N, int K, int epilogue, int* status,
                cudaStream_t stream);

/* The attention inputs straight from the QKV projection: the GEMM qkv = A W^T (W = [W_q; W_k; W_v], N = its
 * width, a multiple of 256) whose epilogue applies what kd_qkv_norm_rope does (per-head RMSNorm over head_dim, RoPE on
 * the first `rot` dims (rot % 32 == 0), Gemma's v norm) and writes q[M, Hq, hd], k/v[M, Hkv, hd] and, for gated
 * queries, gate[M, Hq * hd]; the projection itself is never stored. rope_cs is the pack's rotary table from
 * kd_rope_gather ([rot / 2][M]).
 * Replaces families/qwen/packed.py:108-121 (_qkv, q/k norm, fused.rope) and families/gemma/packed.py:183-193. */
int kd_qkv_projection(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                      const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim, int gated,
                      const void* q_norm_w, const void* k_norm_w, int qk_norm_mode, int v_norm_mode, float eps,
                      const uint32_t* rope_cs, int rot, void* q, void* k, void* v, void* gate, int* status,
                      cudaStream_t stream);

/* The same with e4m3 A and W and per-row scales (the FP8 path: serve/fp8.py:92-101, serve/qwen_fp8.py:38-42). */
int kd_qkv_projection_fp8(const void* A, int64_t lda, const float* scale_a, const void* W, int64_t ldw,
                          const float* scale_w, int M, int N, int K, const int64_t* seqpos, int num_heads_q,
                          int num_heads_kv, int head_dim, int gated, const void* q_norm_w, const void* k_norm_w,
                          int qk_norm_mode, int v_norm_mode, float eps, const uint32_t* rope_cs, int rot, void* q,
                          void* k, void* v, void* gate, int* status, cudaStream_t stream);

/* kd_qkv_projection for callers that cannot allocate device memory (a plugin host that owns every allocation and
 * passes only inputs and outputs, a runtime that forbids side allocations): the per-pack rotary scratch lives in a
 * static device array of the library (4 Mi uint32 entries, 16 MiB per device that loads the library, held until exit)
 * instead of a caller buffer. Takes the rotary tables of kd_rope_table and their row count `positions`; calls needing
 * more than 4 Mi entries ((rot / 2) * M) are rejected. Every argument is checked before the first launch, so a
 * rejected call launches nothing and leaves the array untouched. All calls on a device share the array (overlapping
 * calls race); the first call on a device looks up the array's address and should come before any stream capture.
 * Allocates nothing.
 * No counterpart in the reference: an addition of this library for allocation-free callers. */
int kd_qkv_projection_noalloc(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                              const int64_t* seqpos, int num_heads_q, int num_heads_kv, int head_dim, int gated,
                              const void* q_norm_w, const void* k_norm_w, int qk_norm_mode, int v_norm_mode, float eps,
                              const float* cos_tab, const float* sin_tab, int64_t positions, int rot, void* q,
                              void* k, void* v, void* gate, int* status, cudaStream_t stream);

/* A pack's rotary factors for kd_qkv_projection: cs[i * T + t] = bf16 cos[seqpos[t], i] | bf16 sin[seqpos[t], i] << 16
 * for the rot / 2 distinct pairs i (tables from kd_rope_table, `positions` rows). A position outside [0, positions) is
 * never read: its entry is the identity rotation (cos 1, sin 0). One gather per pack and rotary kind. */
int kd_rope_gather(const int64_t* seqpos, int64_t T, const float* cos_tab, const float* sin_tab, int64_t positions,
                   int rot, uint32_t* cs, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------- pointwise
 * out[t, :] = table[ids[t], :] (times bf16(scale) when scale != 0: Gemma's scaled embedding, sqrt(hidden)).
 * Replaces embed_tokens: families/qwen/packed.py:158-159, families/gemma/packed.py:283-285. */
int kd_embed(const int64_t* ids, int64_t T, const void* table, int64_t vocab, int hidden, float scale, void* out,
             cudaStream_t stream);

/* out = norm(x) row by row (fp32 math, one bf16 rounding); norm_mode KD_NORM_*; weight bf16 [cols] or NULL.
 * Replaces fused.rms_norm: families/qwen/fused.py:17-19, families/gemma/fused.py:21-26. */
int kd_rmsnorm(const void* x, int64_t ldx, const void* weight, int norm_mode, float eps, void* out, int64_t ldo,
               int64_t rows, int cols, cudaStream_t stream);

/* Qwen residual: h = bf16(h + x); y = norm(h). Replaces fused.add_rms_norm / residual_norm
 * (families/qwen/fused.py:22-25, :92-94). */
int kd_add_rmsnorm(void* h, const void* x, const void* weight, int norm_mode, float eps, void* y, int64_t rows,
                   int cols, cudaStream_t stream);

/* Gemma residual: out = bf16(h + norm(x)) (times bf16 layer scalar when scalar != NULL, i.e. add_scale).
 * Replaces fused.add_norm / residual_norm (families/gemma/fused.py:29-30, :91-93) and, with x already normed and
 * norm_mode < 0, fused.add_scale (:33-34). out may alias h. */
int kd_norm_add(const void* h, const void* x, const void* weight, int norm_mode, float eps, const void* scalar,
                void* out, int64_t rows, int cols, cudaStream_t stream);

/* RMSNorm fused with per-row e4m3 quantization of its bf16-rounded output: q = e4m3(clamp(y / s)),
 * s = max(amax(y), 1e-12) / 448. Replaces serve/fp8.py:57-69 (norm_e4m3) and, with norm_mode < 0 (no norm),
 * the activation quantization of serve/fp8.py:21-33 / serve/qwen_fp8.py:20-23. */
int kd_rmsnorm_e4m3(const void* x, int64_t ldx, const void* weight, int norm_mode, float eps, void* q, float* scale,
                    int64_t rows, int cols, cudaStream_t stream);

/* Per-row e4m3 quantization of a weight (load time): serve/fp8.py:21-24, serve/qwen_fp8.py:20-23. */
int kd_quantize_rows_e4m3(const void* x, int64_t rows, int cols, void* q, float* scale, cudaStream_t stream);

/* RoPE tables: cos/sin[p, i] = bf16(cos/sin(p * inv_freq[i % (rot/2)])) stored as float, p < positions, i < rot.
 * Replaces the backbone's rotary_emb (Transformers Qwen3_5TextRotaryEmbedding / Gemma4TextRotaryEmbedding), called
 * at families/qwen/packed.py:186 and families/gemma/packed.py:287-289. */
int kd_rope_table(const float* inv_freq, int rot, int64_t positions, float* cos_out, float* sin_out,
                  cudaStream_t stream);

/* M-RoPE tables, one row per token (Qwen3.5 joint layouts with images): cos/sin[t, i] = bf16(cos/sin(pos[a, t] *
 * inv_freq[i % (rot/2)])) stored as float, t < T, i < rot, where a = pair_axis[i % (rot/2)] picks the position axis
 * (time, height, width: `axes` rows of `pos`, `ld_axis` apart) a frequency pair reads; an axis outside [0, axes) reads
 * axis 0. The same arithmetic as kd_rope_table, so a token whose axes all hold p gets row p of that table. Rows feed
 * kd_rope_gather / kd_qkv_norm_rope with positions 0..T-1. Replaces Transformers' Qwen3_5TextRotaryEmbedding with
 * its interleaved M-RoPE sections (apply_interleaved_mrope), called with the pack's M-RoPE positions at
 * families/qwen/packed.py:186 (Pack.rope, model/packed.py:64-70). */
int kd_rope_table_axes(const float* inv_freq, int rot, const int64_t* pos, int64_t ld_axis, int64_t T,
                       const int32_t* pair_axis, int axes, float* cos_out, float* sin_out, cudaStream_t stream);

/* The attention inputs from the fused QKV projection output qkv[T, ldqkv]: per head RMSNorm over head_dim and RoPE
 * (rotate-half on the first `rot` dims, table rows at seqpos[t]); writes q[T, Hq, hd], k[T, Hkv, hd], v[T, Hkv, hd]
 * and, for Qwen's gated queries, gate[T, Hq * hd].
 * Column layout of qkv: gated (Qwen3.5 q_proj) [Hq x (q_hd | gate_hd)] then [Hkv x k_hd] then [Hkv x v_hd];
 * ungated (Gemma 4) [Hq x q_hd][Hkv x k_hd][Hkv x v_hd].
 * q/k norm modes KD_NORM_*; v_norm_mode < 0 leaves v unnormalised (Qwen), KD_NORM_NONE is Gemma's v_norm.
 * head_dim 64, 128, 256 or 512 (Gemma 4 global layers; attention_k_eq_v: the v columns repeat the k projection).
 * Replaces families/qwen/packed.py:108-121 (_qkv + fused.rope) and families/gemma/packed.py:183-193 (_q, _kv). */
int kd_qkv_norm_rope(const void* qkv, int64_t ldqkv, int64_t T, const int64_t* seqpos, int num_heads_q,
                     int num_heads_kv, int head_dim, int gated, const void* q_norm_w, const void* k_norm_w,
                     int qk_norm_mode, int v_norm_mode, float eps, const float* cos_tab, const float* sin_tab, int rot,
                     void* q, void* k, void* v, void* gate, cudaStream_t stream);

/* Varlen block-diagonal attention, GQA: per sequence s, query i (0-based) sees key j when
 *   i + (Lk - Lq) - left <= j <= i + (Lk - Lq) + right      (left/right < 0: unbounded; right 0: causal)
 * i.e. the contract of torch varlen_attn / flash attention with end alignment (families/qwen/packed.py:123-124,
 * families/gemma/sliding_attention.py:183-191, the reference test contract tests/test_gemma_blocks.py:28-43).
 * q (Tq, Hq, hd), k/v (Tk, Hkv, hd) with row strides in elements; cu_q/cu_k int32 [num_seqs + 1] on the device
 * (read when the kernel runs); q holds total_q rows and k/v total_k rows. max_q bounds every Lq. When gate != NULL,
 * out = bf16(bf16(o) * sigmoid(gate))
 * (Qwen's output gate, families/qwen/fused.py:38-39). head_dim 64, 128, 256 or 512 (Gemma 4's global layers,
 * families/gemma/global_attention.py: two 256-wide value slices per head, each CTA forming the full scores).
 * sched: two ints of device scratch for the persistent CTAs' work counter, zero before the first launch and left
 * zero by every launch; launches that may run at the same time need separate pairs. */
int kd_attention_varlen(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* out,
                        int64_t ldo, const void* gate, int64_t ldg, const int32_t* cu_q, const int32_t* cu_k,
                        int num_seqs, int max_q, int64_t total_q, int64_t total_k, int num_heads_q,
                        int num_heads_kv, int head_dim, float scale, int window_left, int window_right, int* status,
                        int* sched, cudaStream_t stream);

/* dst[i, :] = src[rows[i], :] for n bf16 rows of `width` elements (width % 8 == 0): the key and value rows of a
 * branched block layout's virtual sequences (the shared block, or its last window - 1 rows, then the branch).
 * Replaces _gather / index_select in families/gemma/packed.py:222-226. */
int kd_gather_rows(const void* src, int64_t ld_src, const int64_t* rows, int64_t n, int width, void* dst,
                   int64_t ld_dst, cudaStream_t stream);

/* dst[rows[i], :] = src[i, :] for n bf16 rows of `width` elements (rows distinct, width % 8 == 0): image features
 * written at their soft-token rows, and the image rows' attention written back over a sliding layer's output.
 * Replaces index_copy in families/gemma/packed.py:318-320 and families/gemma/vision.py:210. */
int kd_scatter_rows(const void* src, int64_t ld_src, const int64_t* rows, int64_t n, int width, void* dst,
                    int64_t ld_dst, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------- Gated DeltaNet
 * Qwen3.5's linear-attention token mixer (families/qwen/packed.py:74-106) between its input projection
 * [q | k | v | z | b | a] and its output projection. */

/* Depthwise causal convolution + silu over the [q | k | v] channels: out[t, c] = bf16(silu(sum_s w[c, K-1-s]
 * x[t-s, c])), float32 sums, over taps s with seqpos[t] >= s (no tap before the token's sequence start). x and out
 * bf16 (T, C) with 16-byte aligned rows, C % 8 == 0; weight bf16 (C, K), K <= 4 (conv1d weight squeezed).
 * Replaces flash-linear-attention's causal_conv1d with cu_seqlens (families/qwen/packed.py:82-87) and packed_conv
 * (:45-53). */
int kd_conv_silu(const void* x, int64_t ldx, int64_t T, int C, const void* weight, int K, const int64_t* seqpos,
                 void* out, int64_t ldo, cudaStream_t stream);

/* The gated delta rule per sequence (cu int32 [num_seqs + 1] on the device) and value head h, its key head
 * h / (Hv / Hk): q, k L2-normalized (eps 1e-6), q scaled by dk^-1/2, state S (dk x dv) from zero at each sequence
 * start, per token S = exp(g) S, d = beta (v - S^T k), S += k d^T, o = S^T q; with g = -exp(A_log)
 * softplus(a + dt_bias) in float32 and beta = sigmoid(b) rounded to bf16 (families/qwen/fused.py:42-44).
 * qkv rows [q Hk*dk | k Hk*dk | v Hv*dv] bf16 (the convolution's output); ab rows [b Hv | a Hv] bf16; a_log,
 * dt_bias bf16 [Hv]; out bf16 (T, Hv*dv). dk, dv in {64, 128}. dk = dv = 128 (Qwen3.5) runs the chunked form on the
 * tensor cores (128-token chunks: K K^T, the unit-lower-triangular inverse, W and U, then the state step per chunk with
 * S in tensor memory; bf16 operands, fp32 accumulation, as flash-linear-attention's chunked kernels compute it);
 * `status` is its device status word (KD_DEVICE_TIMEOUT when a wait gave up). The other head dims run the recurrent
 * form on the CUDA cores.
 * Replaces flash-linear-attention's chunk_gated_delta_rule (use_qk_l2norm_in_kernel, cu_seqlens) as
 * families/qwen/packed.py:88-103 calls it. */
int kd_gated_delta_rule(const void* qkv, int64_t ldqkv, const void* ab, int64_t ldab, const void* a_log,
                        const void* dt_bias, const int32_t* cu, int num_seqs, int64_t T, int num_k_heads,
                        int num_v_heads, int head_k_dim, int head_v_dim, void* out, int64_t ldo, int* status,
                        cudaStream_t stream);

/* Qwen3_5RMSNormGated per (token, head) of head_dim values: out = bf16(bf16(w * bf16(x rsqrt(mean(x^2) + eps))) *
 * silu(z)) (families/qwen/fused.py:28-31). head_dim 64 or 128. */
int kd_gated_norm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* weight, int64_t T, int heads,
                  int head_dim, float eps, void* out, int64_t ldo, cudaStream_t stream);

/* The head: out[m, :] = norm(h[markers[m], :]) (final norm at the readout markers).
 * Replaces families/qwen/packed.py:173-176 and families/gemma/packed.py:297-303. */
int kd_marker_norm(const void* h, int hidden, const int64_t* markers, int64_t M, const void* weight, int norm_mode,
                   float eps, void* out, cudaStream_t stream);

/* The readout: logits[m, c] = sum_k float(hidden[m, k]) * W[c, k] in fp32, then cap * tanh(logits / cap) when
 * cap > 0. Replaces Readout.forward (model/readout.py:30-33). */
int kd_readout(const void* hidden, int64_t M, int hidden_size, const float* weight, int codes, float cap,
               float* logits, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KD_B200_H */
