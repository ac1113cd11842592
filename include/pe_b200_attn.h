/*
 * pe_b200_attn.h -- C ABI of the B200 (sm_100a) packed variable-length attention backend.
 *
 * Plain pointers and sizes only. Every tensor lives in device memory of the current CUDA
 * device and is owned by the caller; the library never allocates, frees or synchronises.
 * Calls are enqueued on the stream given; no host reads of cu_seqlens values happen, so a
 * call can be captured in a CUDA graph.
 *
 * Status codes: 0 ok; < 0 a rejected argument (nothing enqueued); see pe_b200_status_string.
 */
#ifndef PE_B200_ATTN_H
#define PE_B200_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PE_B200_ABI_VERSION 4

enum {
  PE_B200_OK = 0,
  PE_B200_ERR_NULL = -1,          /* a required pointer is NULL */
  PE_B200_ERR_SHAPE = -2,         /* heads / kv_heads / head_dim / token counts invalid */
  PE_B200_ERR_STRIDE = -3,        /* a stride or base address breaks the 16-byte TMA rule */
  PE_B200_ERR_WINDOW = -4,        /* window_left / window_right < -1 */
  PE_B200_ERR_WORKSPACE = -5,     /* workspace missing or smaller than pe_b200_attn_workspace_size */
  PE_B200_ERR_DEVICE = -6,        /* current device is not sm_100 */
  PE_B200_ERR_CUDA = -7,          /* a CUDA runtime/driver call failed (launch, tensor map) */
  PE_B200_ERR_UNSUPPORTED = -8,   /* head_dim or layout outside what the kernels implement */
  PE_B200_ERR_SCRATCH_LIMIT = -9, /* call too large for pe_b200_attn_fwd_noalloc's fixed scratch */
};

/* Device-side error bits, readable from the first 8 bytes of the workspace after a call. */
enum {
  PE_B200_DEVERR_WAIT_TIMEOUT = 1,
  PE_B200_DEVERR_SCHEDULE_OVERFLOW = 2,
  PE_B200_DEVERR_BAD_SEGMENTS = 4,
};

/*
 * One packed attention call.
 *
 * q   [total_q, heads,    head_dim] bf16, element strides (q_stride_token, q_stride_head), D contiguous
 * k,v [total_k, kv_heads, head_dim] bf16, likewise
 * out [total_q, heads,    head_dim] bf16, likewise
 * lse [heads, total_q] fp32 natural-log softmax denominator (optional, NULL to skip)
 * cu_seqlens_q / cu_seqlens_k: int32 [n_seq + 1] device arrays, non-decreasing from 0.
 *   For self attention pass the same pointer twice. When a query segment is shorter than
 *   its key segment, the queries are the LAST rows of that key segment (end-aligned causal
 *   mask), as in the reference's prefixed form.
 * window_left / window_right: -1 unbounded, else the band (i - j) <= left, (j - i) <= right.
 * causal: right context forced to 0.
 * workspace: device memory of at least pe_b200_attn_workspace_size(...) bytes, 256-byte
 *   aligned. It holds the tile schedule and the device error word; its contents are
 *   rebuilt by every call, so one workspace serves calls on one stream in sequence.
 * gate [total_q, heads, head_dim] bf16 (optional, NULL to skip), element strides
 *   (g_stride_token, g_stride_head), D contiguous: out = bf16(o * bf16(sigmoid(gate))) with o
 *   the bf16 attention output, the roundings of the reference's separate gate kernel
 *   (packed_encoders/_kernels/hybrid.py:196-205, applied after attention at
 *   packed_encoders/arch/qwen3_5/engine.py:570). The library applies it with its own gate pass
 *   on `stream` right after the attention kernel (or, with the environment variable
 *   PE_B200_GATE=fused, inside the attention epilogue); both give the same bits.
 * rope_cos, rope_sin [total_q, head_dim] bf16 (optional, both or neither; row stride
 *   rope_stride_token elements, D contiguous): q and k arrive un-rotated (e.g. views of the fused
 *   qkv projection); the call rotates them into the workspace (which then also holds
 *   T*H*D + T*KV*D bf16, see pe_b200_attn_workspace_size) with the reference's per-token tables
 *   and rotate-half rule (packed_encoders/_kernels/rope.py:5-6, 140-200: y_lo = x_lo*cos -
 *   x_hi*sin, y_hi = x_hi*cos + x_lo*sin in fp32, rounded to bf16) and attends over the rotated
 *   copies, in place of the reference's apply_rope_bshd pass (packed_encoders/forward.py:199-205).
 *   head_dim 64 and self-attention only (cu_seqlens_k == cu_seqlens_q, total_k == total_q);
 *   other calls with tables return PE_B200_ERR_UNSUPPORTED.
 *
 * Replaces (packed-encoders 0.3.0):
 *   packed_short_attention()      packed_encoders/_kernels/triton_packed_attention.py:175-236
 *   flash_attn_varlen_func calls  packed_encoders/ops.py:432-461, :521-532
 *   AttentionChoice.packed/.prefixed kernels
 *                                 packed_encoders/runtime/attention.py:66-96, 104-126
 *   pe_local_attention (CPU)      packed_encoders/cpu/local_attention_x86.c:192-235
 */
typedef struct PeB200AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* lse;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int32_t n_seq;
  int32_t total_q;
  int32_t total_k;
  int32_t max_seqlen_q; /* host-known upper bound on any query segment length */
  int32_t max_seqlen_k; /* host-known upper bound on any key segment length */
  int32_t heads;
  int32_t kv_heads;
  int32_t head_dim;
  int64_t q_stride_token, q_stride_head;
  int64_t k_stride_token, k_stride_head;
  int64_t v_stride_token, v_stride_head;
  int64_t o_stride_token, o_stride_head;
  float scale;
  int32_t window_left;
  int32_t window_right;
  int32_t causal;
  void* workspace;
  size_t workspace_bytes;
  const void* gate;
  int64_t g_stride_token, g_stride_head;
  const void* rope_cos; /* ABI 3: optional rotary tables, see above */
  const void* rope_sin;
  int64_t rope_stride_token;
} PeB200AttnParams;

/* ABI version of the loaded library (PE_B200_ABI_VERSION). */
int pe_b200_abi_version(void);

/* Human-readable text for a status code. */
const char* pe_b200_status_string(int status);

/*
 * The CUDA error behind the last PE_B200_ERR_CUDA returned on the calling host thread (which
 * call failed and cudaGetErrorString of its error); "" if none. No counterpart in the
 * reference (its kernels are launched by Triton / FlashAttention, which raise their own errors).
 */
const char* pe_b200_last_error_detail(void);

/* 1 if `device` is an sm_100 part this library runs on, else 0. */
int pe_b200_device_supported(int device);

/*
 * Bytes of workspace a call with these shapes needs (n_seq, total_q, max_seqlen_q,
 * max_seqlen_k, head_dim are read; pointers are not). Returns a status code.
 * Replaces the scratch sizing of CPUAttention._native_args, cpu/attention.py:418-430.
 */
int pe_b200_attn_workspace_size(const PeB200AttnParams* p, size_t* bytes);

/*
 * Enqueue packed attention on `stream` (a cudaStream_t; NULL = legacy default stream):
 * the device tile-schedule builder, then the persistent tcgen05 attention kernel.
 */
int pe_b200_attn_fwd(const PeB200AttnParams* p, void* stream);

/*
 * Enqueue only the device tile-schedule builder into `p->workspace` (the first half of
 * pe_b200_attn_fwd). Exposed for tests and for callers that reuse one schedule.
 * Replaces the host-side sequence/tile bookkeeping of triton_packed_attention.py:212-215.
 */
int pe_b200_build_schedule(const PeB200AttnParams* p, void* stream);

/* Enqueue the attention kernel on an already built schedule in `p->workspace`. */
int pe_b200_attn_run(const PeB200AttnParams* p, void* stream);

/*
 * Same as pe_b200_attn_fwd, for callers that cannot give this library any device memory:
 * a plugin whose host framework passes only a stream and the tensors, a binding from a
 * language runtime without its own CUDA allocation calls, or a server that reserves all
 * device memory at start-up and allows no allocation per request. p->workspace and
 * p->workspace_bytes are ignored; the tile schedule and error word live in a fixed 1 MiB
 * array inside the library's device memory (held on every GPU that loads the library until
 * the process exits). Limit: pe_b200_attn_workspace_size(p) <= 1 MiB, else
 * PE_B200_ERR_SCRATCH_LIMIT and nothing is enqueued; without rotary tables that is
 * n_seq + total_q / 128 + 2 <= 65,520, and a rotary call also needs room for its rotated q and
 * k, so only small rotary calls fit. The first call on a device (and the first after its
 * context was re-created, e.g. by cudaDeviceReset) looks up the array's address with that
 * device current; make it before any stream capture. All calls share the array, so calls that
 * overlap on the GPU race: serialise them. Device-side errors of the last call are read with
 * pe_b200_noalloc_error_word. Nothing here allocates. This entry point has no counterpart in
 * the reference.
 */
int pe_b200_attn_fwd_noalloc(const PeB200AttnParams* p, void* stream);

/*
 * The device error word (PE_B200_DEVERR_* bits) of the last pe_b200_attn_fwd_noalloc call on
 * the current device, copied into *out with one copy on `stream` (ordered after the calls
 * enqueued there) and a wait for it; 0 when that call saw no bounded-wait timeout, schedule
 * overflow or malformed cu_seqlens. Allocates nothing. No counterpart in the reference (it is
 * the no-allocation path's view of the workspace error word of pe_b200_attn_fwd).
 */
int pe_b200_noalloc_error_word(int* out, void* stream);

/*
 * Backward of packed self-attention (ABI 4): dq, dk, dv of out = attention(q, k, v) given dout,
 * the forward's out and its natural-log lse [heads, total] (pe_b200_attn_fwd with lse != NULL).
 * head_dim 64, heads == kv_heads, one cu_seqlens for queries and keys, the forward's window /
 * causal / scale. bf16 tensors [total, heads, 64] with element strides (token, head), D
 * contiguous, 16-byte aligned. The workspace (pe_b200_attn_bwd_workspace_size bytes, 256-byte
 * aligned) holds the tile schedule, an fp32 dq accumulator [total, heads, 64] and two fp32
 * [heads, total] row vectors. Enqueues the schedule builder, a row pass (rowsum(dout * out)), the
 * tcgen05 backward kernel and the dq conversion on `stream`. No counterpart in the reference:
 * its training path keeps SDPA's own backward (packed_encoders/pack.py:231-235).
 */
typedef struct PeB200AttnBwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* out;
  const void* dout;
  const float* lse;
  void* dq;
  void* dk;
  void* dv;
  const int32_t* cu_seqlens;
  int32_t n_seq;
  int32_t total;
  int32_t max_seqlen;
  int32_t heads;
  int32_t head_dim;
  int64_t q_stride_token, q_stride_head;
  int64_t k_stride_token, k_stride_head;
  int64_t v_stride_token, v_stride_head;
  int64_t o_stride_token, o_stride_head;
  int64_t do_stride_token, do_stride_head;
  int64_t dq_stride_token, dq_stride_head;
  int64_t dk_stride_token, dk_stride_head;
  int64_t dv_stride_token, dv_stride_head;
  float scale;
  int32_t window_left;
  int32_t window_right;
  int32_t causal;
  void* workspace;
  size_t workspace_bytes;
} PeB200AttnBwdParams;

int pe_b200_attn_bwd_workspace_size(const PeB200AttnBwdParams* p, size_t* bytes);
int pe_b200_attn_bwd(const PeB200AttnBwdParams* p, void* stream);

/*
 * Rotary embedding of q and k into contiguous copies, the reference's BSHD RoPE pass
 * (packed_encoders/_kernels/rope.py:302-345, apply_rope_bshd; rotate-half in fp32 rounded to
 * bf16, rope.py:5-6): q [total, heads, 64] and k [total, kv_heads, 64] bf16 with any 16-byte
 * token / head strides (D contiguous; e.g. views of the fused qkv projection); cos / sin bf16
 * tables with 64-element rows, row stride table_stride_token; token t uses row t % table_rows
 * (table_rows = total for per-token gathered tables, S for one [S, 64] table over a [B, S]
 * batch). Writes q_out [total, heads, 64] and k_out [total, kv_heads, 64] contiguous, enqueued
 * on `stream`. head_dim must be 64 (PE_B200_ERR_UNSUPPORTED otherwise).
 */
int pe_b200_rope_qk(const void* q, const void* k, int64_t q_stride_token, int64_t q_stride_head,
                    int64_t k_stride_token, int64_t k_stride_head, const void* cos_table, const void* sin_table,
                    int64_t table_stride_token, int32_t table_rows, int32_t total, int32_t heads, int32_t kv_heads,
                    int32_t head_dim, void* q_out, void* k_out, void* stream);

/*
 * Debug / layout probes (one CTA, no schedule): QK^T of one 128-row query tile against one
 * key tile into fp32 s_out [128, block_n]; and P.V with fp32 p_in [128, block_n] rounded to
 * bf16 through TMEM into fp32 o_out [128, head_dim]. Rows/keys past the given counts are
 * read as zero. Used by tests to pin the tcgen05 operand layouts.
 */
int pe_b200_debug_qk(const void* q, const void* k, int64_t q_stride_token, int64_t k_stride_token, int rows_q,
                     int rows_k, int head_dim, float* s_out, void* stream);
int pe_b200_debug_pv(const float* p_in, const void* v, int64_t v_stride_token, int rows_k, int head_dim,
                     float* o_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PE_B200_ATTN_H */
