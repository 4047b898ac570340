/*
 * fastmka_b200.h — C ABI of the B200 (sm_100a) FastMKA attention forward.
 *
 * Every entry point takes device pointers, sizes and element strides, an
 * explicit cudaStream_t, and returns an int status (FMKA_OK == 0). On failure
 * fmka_get_last_error() returns the message of the calling thread's last error.
 * The caller owns every buffer; scratch memory ("workspace") is passed in by the
 * caller with its size, and each *_workspace_size() function reports how much a
 * call needs. No entry point but fmka_peer_alloc allocates device memory; kernels report bounded-
 * wait timeouts through a status word that lives in the library's own device
 * data. Calls on distinct streams with distinct buffers may run concurrently.
 *
 * bf16 tensors are passed as `void*` holding __nv_bfloat16 values. Layout names:
 *   [B, T, D]        token rows, element strides (sb, st), channels contiguous
 *   [B, H, T, 128]   head-split K/V/Q, element strides (sb, sh, st), dims contiguous
 *
 * The entry points replace these reference interfaces (FastLM/MKA):
 *   fmka_qr_proj            q = wq(x) and the router's first layer
 *                           (mka/layers/fastmka.py:79,91; mka/hf/attention.py:95,104)
 *   fmka_route_ema_blend    causal_prefix_ema, repeat_retrieval_to_length, the gate
 *                           softmax and the route blend
 *                           (mka/layers/session_memory.py:6-39;
 *                            mka/layers/fastmka.py:82-96; mka/hf/attention.py:97-107)
 *   fmka_route_ema_blend_state  the same with the EMA state carried across calls
 *                           (extends session_memory.py:6-22, which restarts at zero)
 *   fmka_route_ema_blend_kv the same on y = x [Wk ; Wv]^T (and y3 = L3 [Wk ; Wv]^T
 *                           for three levels), writing K/V (the blend and
 *                           k/v_proj of fastmka.py:94-99 and hf/attention.py:105-119
 *                           in the commuted order)
 *   fmka_kv_proj            k/v projection of the fused memory (+ RoPE on k)
 *                           (mka/layers/fastmka.py:98-99; mka/hf/attention.py:110-119)
 *   fmka_attn_fwd_prefill   causal attention: fastmka_attn (mka/cuda/ops.py:73,
 *                           mka/cuda/fastmka_attn.cpp:11-17, fastmka_attn.cu:133-172)
 *                           and the SDPA calls at fastmka.py:134,157 /
 *                           hf/attention.py:142
 *   fmka_attn_decode_splitkv  the single-token decode attention
 *                           (fastmka.py:166-174; hf/attention.py:188-193)
 *   fmka_gemm_bf16          the output projection wo / o_proj
 *                           (fastmka.py:175-176; hf/attention.py:194-195)
 *   fmka_get_last_error     the TORCH_CHECK / cudaGetLastError error reporting of
 *                           fastmka_attn.cu:134-150,169-170
 *   fmka_gemm_bf16_swiglu   outside the attention path: the gate/up projections and
 *                           SiLU product of the Llama MLP around the patched
 *                           self_attn (transformers LlamaMLP), one GEMM
 *   fmka_rmsnorm_bf16,      outside the attention path: the RMSNorm and the MLP's
 *   fmka_silu_mul_bf16      SiLU product of the decoder layers around the patched
 *                           self_attn (transformers LlamaRMSNorm / LlamaMLP), one
 *                           pass each
 *   fmka_l3_*, fmka_gemm_bf16_f32out
 *                           the L3 chunk recall producing R, which the reference
 *                           describes (memory_hierarchy.py:1-10,30-34) but does
 *                           not implement
 *   fmka_attn_fwd_prefill_scatter, fmka_gemm_bf16_kblocked_scatter, fmka_peer_*
 *                           the head-sharded layer over several GPUs of a box:
 *                           attention rows and o_proj rows stored straight into
 *                           the other ranks' buffers, which replaces an all-gather
 *                           in front of o_proj (the reference keeps distributed
 *                           code in scripts/train_hf_patch.py:97-129)
 */
#ifndef FASTMKA_B200_H_
#define FASTMKA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FMKA_API __attribute__((visibility("default")))
#else
#define FMKA_API
#endif

typedef struct CUstream_st* fmka_stream_t; /* same handle as cudaStream_t */

enum {
  FMKA_OK = 0,
  FMKA_ERR_INVALID_ARGUMENT = 1,
  FMKA_ERR_UNSUPPORTED = 2,
  FMKA_ERR_CUDA = 3,
  FMKA_ERR_WORKSPACE = 4,
  FMKA_ERR_DEVICE = 5
};

/* Device status bits set by kernels (see fmka_device_status). */
enum {
  FMKA_STATUS_WAIT_TIMEOUT = 1,     /* a pipeline wait in a kernel ran out of time */
  FMKA_STATUS_LOOKBACK_TIMEOUT = 2, /* the EMA scan's look-back ran out of time */
  FMKA_STATUS_BAD_LAUNCH = 4,
  FMKA_STATUS_PEER_TIMEOUT = 8      /* a cross-GPU barrier (fmka_peer_barrier) ran out of time */
};

/* Library version string. */
FMKA_API const char* fmka_version(void);

/* Last error of the calling thread: returns its status code and copies the
 * NUL-terminated message into buf (truncated to buflen). */
FMKA_API int fmka_get_last_error(char* buf, int buflen);

/* Reads the current device's kernel status word into *status (after
 * synchronising `stream`) and clears it when `clear` is nonzero. A nonzero
 * word means some kernel gave up on a bounded wait; its outputs are invalid. */
FMKA_API int fmka_device_status(uint32_t* status, int clear, fmka_stream_t stream);

/* Number of SMs of the current device. */
FMKA_API int fmka_num_sms(void);

/* ---------------------------------------------------------------- GEMMs ---
 * fmka_gemm_bf16: C[M, N] = A[M, K] * W[N, K]^T (+ bias[N]), bf16 in/out,
 * fp32 accumulation (tcgen05). K, lda, ldw, ldc multiples of 8. */
FMKA_API int fmka_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, const float* bias, void* c, int64_t ldc,
                   int M, int N, int K, fmka_stream_t stream);

/* fmka_gemm_bf16_f32out: C[M, N] = A[M, K] * W[N, K]^T with bf16 operands and an
 * fp32 output (row stride ldc, a multiple of 8; C 16-byte aligned). Scores of
 * the L3 chunk recall (no counterpart in the reference). */
FMKA_API int fmka_gemm_bf16_f32out(const void* a, int64_t lda, const void* w, int64_t ldw, float* c, int64_t ldc,
                                   int M, int N, int K, fmka_stream_t stream);

/* fmka_gemm_bf16_kblocked: the same GEMM with A stored as K / a_kblk blocks of
 * [M, a_kblk] (row stride lda, blocks a_blk_stride elements apart): A[m, k] =
 * block[k / a_kblk][m][k % a_kblk]. This reads an all-gathered attention output
 * ([ranks, B*T, heads_per_rank*128]) as the o_proj input without a permute copy.
 * a_kblk % 64 == 0 and K % a_kblk == 0. Replaces the o_proj call of the
 * head-sharded layer (mka/hf/attention.py:194-195). */
FMKA_API int fmka_gemm_bf16_kblocked(const void* a, int a_kblk, int64_t a_blk_stride, int64_t lda, const void* w,
                                     int64_t ldw, const float* bias, void* c, int64_t ldc, int M, int N, int K,
                                     fmka_stream_t stream);

/* fmka_qr_proj: one GEMM over x[M = B*T, D] with the stacked weight
 * w_qr = [Wq ; W1 * Wq]  ([Nq + R, D]) and fp32 bias_qr ([Nq + R] or NULL).
 *   columns [0, Nq)      -> q in head-split layout [B, Hq, T, 128] at strides
 *                           (q_sb, q_sh, q_st), token slots from t_offset, with
 *                           rotate-half RoPE when cos/sin are given
 *                           (fp32 [.., T, 128] at strides (rope_sb, rope_st))
 *   columns [Nq, Nq + R) -> router hidden h = act(. + bias), accumulated as
 *                           logits[m, l] += sum_r w2[l, r] * h[r]
 *                           (logits fp32 [M, L]; the caller zeroes it first)
 * act: 0 = SiLU, 1 = GELU (erf). Nq = Hq * 128, Nq % 128 == 0. */
FMKA_API int fmka_qr_proj(const void* x, int64_t ldx, const void* w_qr, int64_t ldw, const float* bias_qr, int B, int T,
                 int D, int Hq, int R, void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, int t_offset,
                 const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st, const float* w2,
                 int L, int act, float* logits, fmka_stream_t stream);

/* fmka_kv_proj: one GEMM over h[M = B*T, D] with w_kv = [Wk ; Wv]
 * ([2 * Hkv * 128, D]) and fp32 bias_kv ([2 * Hkv * 128] or NULL). k and v are
 * written in head-split layout at token slots [t_offset, t_offset + T), RoPE on
 * k when cos/sin are given. */
FMKA_API int fmka_kv_proj(const void* h, int64_t ldh, const void* w_kv, int64_t ldw, const float* bias_kv, int B, int T,
                 int D, int Hkv, void* k, void* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, int t_offset,
                 const float* rope_cos, const float* rope_sin, int64_t rope_sb, int64_t rope_st,
                 fmka_stream_t stream);

/* ------------------------------------------------- stage 1: route + EMA ---
 * lam = softmax(logits + b2) (or `gate` given directly), L2 = causal prefix EMA
 * of x with decay beta (zero initial state), H = lam0*x + lam1*L2 (+ lam2*L3).
 * L3 row for token t is min(t, T3 - 1) (the reference's repeat / truncate /
 * pad-with-last-row rule); l3_st may be 0 to broadcast one row. Exactly one of
 * logits / gate is non-NULL. lam (fp32 [B, T, L]) may be NULL. */
FMKA_API size_t fmka_route_ema_blend_workspace_size(int B, int T, int D);
FMKA_API int fmka_route_ema_blend(const void* x, int64_t x_sb, int64_t x_st, const float* logits, const float* b2,
                         const float* gate, int L, const void* l3, int64_t l3_sb, int64_t l3_st, int T3, float beta,
                         int B, int T, int D, void* h, int64_t h_sb, int64_t h_st, float* lam, void* workspace,
                         size_t workspace_bytes, fmka_stream_t stream);

/* fmka_route_ema_blend_noalloc: the same computation as fmka_route_ema_blend,
 * for callers that cannot allocate device memory at call time (a runtime that
 * reserved the whole GPU for its own pools, a real-time path that must not
 * trigger cudaMalloc's synchronisation, a C program with no allocator). No
 * counterpart in the reference. It allocates nothing: its scratch is a static
 * device array of fmka_route_ema_blend_noalloc_scratch_bytes() (4 MiB) held by
 * every GPU that loads the library, so shapes whose
 * fmka_route_ema_blend_workspace_size() exceeds that are rejected with
 * FMKA_ERR_UNSUPPORTED. The first call on a device looks up the array's device
 * address (make it before any stream capture) and keeps it for the life of the
 * process: after a cudaDeviceReset of that device, unload and reload the library
 * before calling this again. All calls share the array: calls that overlap on
 * the GPU race. */
FMKA_API int fmka_route_ema_blend_noalloc(const void* x, int64_t x_sb, int64_t x_st, const float* logits,
                                          const float* b2, const float* gate, int L, const void* l3, int64_t l3_sb,
                                          int64_t l3_st, int T3, float beta, int B, int T, int D, void* h,
                                          int64_t h_sb, int64_t h_st, float* lam, fmka_stream_t stream);
FMKA_API size_t fmka_route_ema_blend_noalloc_scratch_bytes(void);

/* fmka_route_ema_blend_state: fmka_route_ema_blend with the EMA carried across
 * calls. It extends causal_prefix_ema (mka/layers/session_memory.py:6-22),
 * whose state starts at zero on every call (:17-21), with an initial state:
 * L2[t] = beta * L2[t-1] + (1 - beta) * x[t] with L2[-1] = ema_init (fp32
 * [B, D], contiguous; NULL = zero, which is fmka_route_ema_blend). ema_final
 * (fp32 [B, D], may be NULL) receives L2[T-1], the state to pass to the next
 * call; it must not alias ema_init. Both 16-byte aligned. */
FMKA_API int fmka_route_ema_blend_state(const void* x, int64_t x_sb, int64_t x_st, const float* logits,
                                        const float* b2, const float* gate, int L, const void* l3, int64_t l3_sb,
                                        int64_t l3_st, int T3, float beta, int B, int T, int D, void* h,
                                        int64_t h_sb, int64_t h_st, float* lam, const float* ema_init,
                                        float* ema_final, void* workspace, size_t workspace_bytes,
                                        fmka_stream_t stream);

/* fmka_route_ema_blend_kv: stage 1 on the projected memory.
 * Input y = x [Wk ; Wv]^T (bf16 [B, T, 2*Hkv*128], rows y_st apart, batches
 * y_sb; from fmka_gemm_bf16 without bias). Output the reference's k_proj /
 * v_proj of the fused memory (mka/hf/attention.py:97-119,
 * mka/layers/fastmka.py:82-99) head-split into k_out / v_out
 * ([B, Hkv, Tcap, 128], strides kv_sb, kv_sh, kv_st, written at token slot
 * t + t_offset): with lam = softmax(logits + b2),
 *   K = lam0 * yk + lam1 * EMA(yk) + bk, then rotate-half RoPE (cos/sin fp32
 *   [*, T, 128], may be NULL), and V likewise without RoPE,
 * which equals projecting lam0 * x + lam1 * EMA(x) because the EMA (along
 * tokens) commutes with the projection (along channels) and the gate sums to
 * one. The scan runs over 2*Hkv*128 channels instead of d_model. A third
 * level is given as y3 = l3 [Wk ; Wv]^T ([B, T3, 2*Hkv*128] at strides
 * (y3_sb, y3_st), row t uses min(t, T3 - 1), y3_st may be 0) and adds
 * lam2 * y3 (logits and b2 then have 3 levels); y3 = NULL for two levels.
 * lam (fp32 [B, T, L]), ema_init / ema_final (fp32 [B, 2*Hkv*128], the state of
 * EMA(y), as for fmka_route_ema_blend_state) may be NULL. The library picks the
 * scan: token by token for T <= 32, a streaming scan whose CTAs recompute their
 * incoming state from a warm-up window when |beta| leaves a short memory, else
 * a chunk-parallel scan with a decoupled look-back; only the last uses the
 * workspace, which is required all the same. */
FMKA_API size_t fmka_route_ema_blend_kv_workspace_size(int B, int T, int Hkv);
FMKA_API int fmka_route_ema_blend_kv(const void* y, int64_t y_sb, int64_t y_st, const float* logits,
                                     const float* b2, const void* y3, int64_t y3_sb, int64_t y3_st, int T3,
                                     float beta, int B, int T, int Hkv, const float* bias,
                                     void* k_out, void* v_out, int64_t kv_sb, int64_t kv_sh, int64_t kv_st,
                                     int t_offset, const float* rope_cos, const float* rope_sin, int64_t rope_sb,
                                     int64_t rope_st, float* lam, const float* ema_init, float* ema_final,
                                     void* workspace, size_t workspace_bytes, fmka_stream_t stream);

/* Route blend with all three memories given (no scan):
 * H = gate0*l1 + gate1*l2 (+ gate2*l3), gate fp32 [B*T, L]. This is the blend
 * inside the reference's fused route kernel (mka/cuda/fused_route_mka.cu:60-67,
 * reached through fused_route_mka_attn, mka/cuda/ops.py:47-70). */
FMKA_API int fmka_route_blend(const void* l1, int64_t l1_sb, int64_t l1_st, const void* l2, int64_t l2_sb, int64_t l2_st,
                     const void* l3, int64_t l3_sb, int64_t l3_st, int T3, const float* gate, int L, int B, int T,
                     int D, void* h, int64_t h_sb, int64_t h_st, fmka_stream_t stream);

/* ------------------------------------------------------------ attention ---
 * Prefill: o[b, t, hq, :] = softmax(scale * q k^T + causal mask) v, with GQA
 * (kv head = hq / (Hq / Hkv)) and bottom-right causal alignment (query t sees
 * keys <= t + Tk - Tq). lse[b, hq, t] (natural log of the scaled scores) may be
 * NULL. head_dim must be 128. */
FMKA_API int fmka_attn_fwd_prefill(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k, const void* v,
                          int64_t kv_sb, int64_t kv_sh, int64_t kv_st, void* o, int64_t o_sb, int64_t o_st,
                          int64_t o_sh, float* lse, int64_t lse_sb, int64_t lse_sh, int B, int Hq, int Hkv, int Tq,
                          int Tk, int head_dim, int causal, float scale, fmka_stream_t stream);

/* Decode: one query token per sequence against Tk cached keys.
 * q[b, hq, :] at (q_sb, q_sh); o[b, hq, :] at (o_sb, o_sh); lse[b, hq] may be
 * NULL. num_splits <= 0 picks a split count for the device; the workspace size
 * depends on it. At most 16 query heads per kv head. */
FMKA_API int fmka_attn_decode_num_splits(int B, int Hkv, int Tk);
FMKA_API size_t fmka_attn_decode_workspace_size(int B, int Hq, int Hkv, int Tk, int num_splits);
FMKA_API int fmka_attn_decode_splitkv(const void* q, int64_t q_sb, int64_t q_sh, const void* k, const void* v, int64_t kv_sb,
                             int64_t kv_sh, int64_t kv_st, void* o, int64_t o_sb, int64_t o_sh, float* lse,
                             int64_t lse_sb, int B, int Hq, int Hkv, int Tk, int head_dim, float scale,
                             int num_splits, void* workspace, size_t workspace_bytes, fmka_stream_t stream);

/* SwiGLU feed-forward input projection (the gate_proj / up_proj / act_fn of a
 * Llama MLP, fused): c[m, i] = silu(a w_g[i]^T + b_g[i]) * (a w_u[i]^T + b_u[i])
 * for i < I, bf16 out with fp32 accumulation. w_gu [2I, K] holds the two
 * weights interleaved in blocks of 128 rows: rows 256j .. 256j+127 are gate
 * rows 128j .. 128j+127 and rows 256j+128 .. 256j+255 the matching up rows
 * (bias_gu [2I] fp32 in the same order, or NULL). I must be a multiple of 128. */
FMKA_API int fmka_gemm_bf16_swiglu(const void* a, int64_t lda, const void* w_gu, int64_t ldw, const float* bias_gu,
                          void* c, int64_t ldc, int M, int I, int K, fmka_stream_t stream);

/* RMSNorm of the decoder layers around the patched self_attn (no counterpart
 * in the reference's own code: it is transformers' LlamaRMSNorm, which the
 * patched models run): y[r, :] = bf16(w * bf16(x[r, :] * rsqrt(mean(x[r, :]^2)
 * + eps))) for r < rows, with the mean in fp32 and the same two roundings as the
 * module. x, y bf16 with row strides ldx, ldy (elements); w bf16 [D]; D a
 * multiple of 8, at most 8192. */
FMKA_API int fmka_rmsnorm_bf16(const void* x, int64_t ldx, const void* w, float eps, void* y, int64_t ldy, int rows,
                               int D, fmka_stream_t stream);

/* SiLU product of the MLP around the patched self_attn (no counterpart in the
 * reference's own code: transformers' LlamaMLP computes act_fn(gate) * up):
 * out[i] = bf16(bf16(silu(g[i])) * u[i]) for n contiguous bf16 elements (n a
 * multiple of 8); out may be g. */
FMKA_API int fmka_silu_mul_bf16(const void* g, const void* u, void* out, int64_t n, fmka_stream_t stream);

/* ------------------------------------------------------ L3 chunk recall ---
 * The retrieval that produces the L3 memory R from a bank of historical chunks.
 * The reference describes it (mka/config/memory_hierarchy.py:1-10,30-34:
 * "DRAM (vectorized hash, chunk recall)", l3_recall_top_r "top-R chunks per
 * query") and implements none; this algorithm is the library's own:
 *   q = fmka_l3_block_mean_bf16(x)             block summaries, bf16 [B*nq, D],
 *                                              nq = ceil(T / block_len)
 *   s = fmka_gemm_bf16_f32out(q, keys)         fp32 scores [B*nq, n_chunks]
 *   (idx, w) = fmka_l3_topr_f32(s, R, scale)   the R best chunks of each row
 *                                              (ties: lower index first) and
 *                                              softmax(scale * score) over them
 *   R = fmka_l3_recall_gather_bf16(idx, w, values)
 *                                              R[b, t] = sum_r w values[idx] for
 *                                              every token t of block t / block_len
 * x, values, out: bf16 with contiguous channels, strides in elements, multiples
 * of 8; D a multiple of 8; R in 1..32 and at most n_chunks. */
FMKA_API int fmka_l3_block_mean_bf16(const void* x, int64_t x_sb, int64_t x_st, int B, int T, int D, int block_len,
                                     void* q, int64_t ldq, fmka_stream_t stream);
FMKA_API int fmka_l3_topr_f32(const float* scores, int64_t lds, int M, int N, int R, float scale, int32_t* idx,
                              float* w, fmka_stream_t stream);
FMKA_API int fmka_l3_recall_gather_bf16(const int32_t* idx, const float* w, int R, const void* values, int64_t ldv,
                                        int n_chunks, int D, int B, int T, int block_len, void* out, int64_t o_sb,
                                        int64_t o_st, fmka_stream_t stream);

/* ------------------------------------------------ several GPUs of a box ---
 * The ranks of a sequence group (one process per GPU) share buffers through
 * peer mappings: fmka_peer_alloc makes a zero-filled device allocation (the one
 * entry point that allocates: a mapping covers a whole allocation), whose
 * FMKA_PEER_HANDLE_BYTES-byte handle from fmka_peer_export another process of
 * the box opens with fmka_peer_import (close it with fmka_peer_close before the
 * owner calls fmka_peer_free). No multicast object is created.
 *
 * fmka_peer_barrier: flags[j] is rank j's array of n uint32 slots as mapped in
 * the calling process (its own array for j == rank). In stream order, the
 * caller stores `epoch` into slot `rank` of every array and waits until every
 * slot of its own array holds `epoch` or later; epochs must grow by one per
 * barrier, starting from 1 on zero-filled arrays. A wait that runs out of time
 * (2 s) sets FMKA_STATUS_PEER_TIMEOUT and returns. */
#define FMKA_PEER_HANDLE_BYTES 64
FMKA_API int fmka_peer_alloc(size_t bytes, void** ptr);
FMKA_API int fmka_peer_free(void* ptr);
FMKA_API int fmka_peer_export(const void* ptr, void* handle);
FMKA_API int fmka_peer_import(const void* handle, void** ptr);
FMKA_API int fmka_peer_close(void* ptr);
FMKA_API int fmka_peer_barrier(uint32_t* const* flags, int rank, int n, uint32_t epoch, fmka_stream_t stream);

/* fmka_attn_fwd_prefill with the output rows split over n_dst (<= 8) buffers:
 * query rows [j * rows_per_dst, (j + 1) * rows_per_dst) of every sequence go to
 * o_dst[j] (row t - j * rows_per_dst there, strides o_sb / o_st / o_sh), local
 * or peer-mapped. No LSE. n_dst * rows_per_dst must cover Tq. */
FMKA_API int fmka_attn_fwd_prefill_scatter(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                                  const void* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_st, void* const* o_dst,
                                  int n_dst, int rows_per_dst, int64_t o_sb, int64_t o_st, int64_t o_sh, int B,
                                  int Hq, int Hkv, int Tq, int Tk, int head_dim, int causal, float scale,
                                  fmka_stream_t stream);

/* fmka_gemm_bf16_kblocked whose output row m is written to row c_row0 + m of
 * each of the n_dst (<= 8) buffers c_dst[0 .. n_dst-1] (row stride ldc), local
 * or peer-mapped: o_proj on this rank's rows, delivered to every rank of the
 * group. N and ldc must be multiples of 8, the buffers 16-byte aligned. */
FMKA_API int fmka_gemm_bf16_kblocked_scatter(const void* a, int a_kblk, int64_t a_blk_stride, int64_t lda,
                                    const void* w, int64_t ldw, const float* bias, void* const* c_dst, int n_dst,
                                    int64_t c_row0, int64_t ldc, int M, int N, int K, fmka_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTMKA_B200_H_ */
