/*
 * starkv.h — C ABI of the B200 (sm_100a) compressed-KV decode-attention path.
 *
 * These entry points replace, for the decode step, the kernels and cache
 * update that STAR-KV's attention modules call:
 *
 *   reference interface (PriyanshBhatnagar/STAR-KV)            replaced by
 *   ------------------------------------------------------------------------
 *   quant_utils.quantize_r_split_int8_int4_packed               starkv_quantize_prefill,
 *     (LlamaLoRaAttention_headwise_quant.py:107-117)              starkv_append
 *   Cache.update (LlamaLoRaAttention_headwise.py:99,           starkv_append
 *     LlamaLoRaAttention_headwise_quant.py:119-127, model.py:419)
 *   abx_rope_batched.abx (abx_rope_batched.py:135-186)          starkv_k_logits
 *   bx_quant.bx (bx_quant.py:117-166)                           starkv_v_latent
 *   the decode branch of LlamaCustomAttention.forward from      starkv_decode_attention
 *     the latent append to the V up-projection
 *     (LlamaLoRaAttention_headwise.py:98-133,
 *      LlamaLoRaAttention_headwise_quant.py:119-186,
 *      model.py:450-487)
 *
 * Conventions: every pointer is a device pointer unless stated; all launches
 * go on the given stream; nothing allocates device memory (scratch comes from
 * the caller's workspace); every function returns a starkv_status.
 */
#ifndef STARKV_H
#define STARKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STARKV_ABI_VERSION 2
#define STARKV_MAX_KV_HEADS 64
#define STARKV_MAX_V_BLOCKS 32
#define STARKV_HEAD_DIM 128
#define STARKV_MAX_K_RANK 128

typedef struct CUstream_st* starkv_stream_t; /* == cudaStream_t */

typedef enum starkv_status {
  STARKV_OK = 0,
  STARKV_ERR_INVALID = 1,       /* bad shape, null pointer, inconsistent layout */
  STARKV_ERR_UNSUPPORTED = 2,   /* rank / head count / dtype outside what the kernels support */
  STARKV_ERR_LAUNCH = 3,        /* CUDA launch error (cudaGetLastError) */
  STARKV_ERR_WORKSPACE = 4,     /* workspace too small */
  STARKV_ERR_DEVICE = 5         /* device is not sm_100 */
} starkv_status;

typedef enum starkv_dtype {
  STARKV_F32 = 0,
  STARKV_F16 = 1,
  STARKV_BF16 = 2
} starkv_dtype;

/*
 * Layout of one layer's latent cache.
 *
 * K (per KV head h, rank r_h = k_rank[h], multiple of 16, <= 128), in units
 *   of the cache element (int8 code when quantised, latent dtype otherwise;
 *   e bytes, n = 16 / e elements per 16-byte chunk):
 *   row-major (k_tiled = 0): element (b, slot, c) lives at
 *     k_offset[h] + b * k_batch_stride[h] + slot * r_h + c;
 *     the reference's (B, Hkv, L, r) tensor is k_offset[h] = h*L*r,
 *     k_batch_stride = Hkv*L*r;
 *   tiled (k_tiled = 1, capacity a multiple of 128): tiles of 128 slots, each
 *     the r_h / n column chunks of its 128 rows, a chunk 128 x 16 bytes:
 *     k_offset[h] + b * k_batch_stride[h] + (slot / 128) * 128 * r_h
 *       + (c / n) * 128 * n + (slot % 128) * n + c % n.
 *     A 16-byte piece of 128 consecutive rows is one contiguous 2 KiB run: the
 *     K kernel reads its staged tiles without shared-memory bank conflicts.
 * K scales (quantised): fp16, (B, sum r_h): scale(b, h, c) at b*k_rank_total + k_col[h] + c.
 * V (blocks j of v_num_kv[j] consecutive KV heads starting at v_first_kv[j],
 *   rank r_j = v_rank[j], multiple of 32): the latents of all blocks of one
 *   token are one row, as in the reference's (B, L, R):
 *   quantised codes: uint8 (B, capacity, R/2), channel v_col[j]+c of (b, slot)
 *     in byte (b*capacity + slot)*R/2 + (v_col[j]+c)/2, even channel in the low nibble;
 *   quantised params: fp16 pairs (scale, zero) (B, capacity, R/32, 2);
 *   unquantised: latent dtype (B, capacity, R).
 */
typedef struct starkv_layout {
  int32_t abi_version;     /* STARKV_ABI_VERSION */
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;        /* 128 */
  int32_t num_v_blocks;
  int32_t capacity;        /* token slots per sequence */
  int32_t quantized;       /* 1: int8 K / int4 V codes; 0: latents stored in latent_dtype */
  int32_t latent_dtype;    /* starkv_dtype of latents fed to the quantiser / stored unquantised */
  int32_t k_rank_total;    /* sum k_rank */
  int32_t v_rank_total;    /* sum v_rank = R */
  int32_t k_tiled;         /* 1: K tiles of 128 slots stored as 16-byte column chunks (see above) */
  int32_t k_rank[STARKV_MAX_KV_HEADS];
  int32_t k_col[STARKV_MAX_KV_HEADS];          /* prefix sums of k_rank */
  int64_t k_offset[STARKV_MAX_KV_HEADS];
  int64_t k_batch_stride[STARKV_MAX_KV_HEADS];
  int32_t v_rank[STARKV_MAX_V_BLOCKS];
  int32_t v_col[STARKV_MAX_V_BLOCKS];          /* prefix sums of v_rank */
  int32_t v_first_kv[STARKV_MAX_V_BLOCKS];
  int32_t v_num_kv[STARKV_MAX_V_BLOCKS];
} starkv_layout;

/* sizeof(starkv_layout) as compiled into the library (ABI check for bindings). */
size_t starkv_layout_size(void);

/* Checks a layout; STARKV_OK if every kernel accepts it. Host only, no CUDA calls. */
int starkv_validate_layout(const starkv_layout* lay);

/*
 * Prefill: write tokens [0, num_tokens) of every sequence into the cache.
 *   k_lat: (B, num_tokens, k_rank_total) latent_dtype — the K latent projection
 *          ``hidden @ k_proj.VS.weight^T`` (LlamaLoRaAttention_headwise.py:88-92);
 *   v_lat: (B, num_tokens, v_rank_total) latent_dtype (:96).
 * Quantised layouts compute the per-channel K scales over these tokens and
 * write k_scales (fp16, (B, k_rank_total)); V is quantised per token.
 */
int starkv_quantize_prefill(const starkv_layout* lay, const void* k_lat, const void* v_lat,
                            int32_t num_tokens, void* k_cache, void* k_scales,
                            void* v_cache, void* v_params, starkv_stream_t stream);

/*
 * Append num_tokens new tokens per sequence at slots [start_slot, start_slot+num_tokens)
 * (the in-place replacement of Cache.update's torch.cat).  Quantised layouts use
 * the existing K scales (read-only here).
 */
int starkv_append(const starkv_layout* lay, const void* k_lat, const void* v_lat,
                  int32_t num_tokens, int32_t start_slot, void* k_cache, const void* k_scales,
                  void* v_cache, void* v_params, starkv_stream_t stream);

/*
 * Fused latent projection + quantise-append of one decode token per sequence:
 * k_lat = hidden @ vs_k^T, v_lat = hidden @ vs_v^T (fp32 dot products rounded to
 * the latent dtype), then the same quantiser / append as starkv_append at `slot`.
 * Replaces the k_proj.VS / v_proj.VS projections and the cache update of
 * LlamaLoRaAttention_headwise.py:86-99 (LlamaLoRaAttention_headwise_quant.py:94-127).
 * hidden: (batch, hidden_size); vs_k: (k_rank_total, hidden_size) (the heads'
 * rows concatenated); vs_v: (v_rank_total, hidden_size); all in the latent dtype,
 * 16-byte aligned rows.  k_lat_out / v_lat_out (nullable): (batch, k_rank_total) /
 * (batch, v_rank_total) receive the rounded latents.
 */
int starkv_project_append(const starkv_layout* lay, const void* hidden, int32_t hidden_size,
                          const void* vs_k, const void* vs_v, int32_t slot, void* k_cache,
                          const void* k_scales, void* v_cache, void* v_params, void* k_lat_out,
                          void* v_lat_out, starkv_stream_t stream);

typedef struct starkv_decode_args {
  const void* q;            /* (B, Hq, 128) rotated query, q_dtype, contiguous */
  int32_t q_dtype;
  int32_t w_dtype;          /* dtype of k_u and v_u */
  const void* k_u;          /* K up-projections: head h is (128, r_h) row-major at element 128*k_col[h]
                               (the reference's k_proj.U[h], model.py:318-324) */
  const void* v_u;          /* (Hkv*128, v_rank_total) row-major: v_proj.U.weight (model.py:348-356),
                               only the block-diagonal part is read */
  const float* inv_freq;    /* (64,) fp32 RoPE inverse frequencies (HF LlamaRotaryEmbedding.inv_freq) */
  const float* mask;        /* optional (B, num_tokens) additive fp32 mask, or NULL */
  float scaling;            /* softmax scale, head_dim^-0.5 in the reference */
  int32_t num_tokens;       /* attended slots [0, num_tokens); slot l has RoPE position l */
  const void* k_cache;
  const void* k_scales;
  const void* v_cache;
  const void* v_params;
  void* out;                /* (B, Hq, 128) out_dtype */
  int32_t out_dtype;
  int32_t num_splits;       /* sequence splits per (sequence, head group); 0 = automatic */
  void* workspace;          /* scratch, 256-byte aligned */
  size_t workspace_bytes;
  void* const* events;      /* optional: 4 cudaEvent_t recorded on the stream before the K kernel, after
                               it, after the V kernel and after the merge (per-kernel timing); or NULL */
} starkv_decode_args;

/* Workspace bytes starkv_decode_attention needs for this layout / token count / split count. */
int starkv_decode_workspace_size(const starkv_layout* lay, int32_t num_tokens, int32_t num_splits,
                                 size_t* bytes);

/* Number of sequence splits the automatic choice (num_splits = 0) uses. */
int32_t starkv_auto_splits(const starkv_layout* lay, int32_t num_tokens);

/*
 * One decode step of attention over slots [0, num_tokens): K reconstruction
 * from the latents on the tensor cores + RoPE + q.k, softmax over the whole
 * sequence (split-K with a merge), P.X_v in latent space, then the V
 * up-projection once per head.  Output: per-head attention (B, Hq, 128), the
 * tensor the reference feeds to o_proj (before its reshape).
 */
int starkv_decode_attention(const starkv_layout* lay, const starkv_decode_args* args,
                            starkv_stream_t stream);

/*
 * Logits only (abx_rope_batched.abx): logits[b, qh, l] = q[b, qh] . RoPE_l(X_k[b, kv(qh), l] @ U^T)
 * for l < num_tokens, unscaled, fp32, (B, Hq, num_tokens) contiguous.  The
 * args' workspace (starkv_decode_workspace_size bytes) holds the per-head W
 * images; mask / v_* / out are ignored.
 */
int starkv_k_logits(const starkv_layout* lay, const starkv_decode_args* args, float* logits,
                    starkv_stream_t stream);

/*
 * P.X_v in latent space (bx_quant.bx): probs (B, Hq, num_tokens) fp32 ->
 * out (B, Hq, v_rank_total) fp32 where the columns of the head's V block hold
 * sum_l p[l] * dequant(X_v[l]) and the other columns are 0.
 */
int starkv_v_latent(const starkv_layout* lay, const float* probs, int32_t num_tokens,
                    const void* v_cache, const void* v_params, float* out, starkv_stream_t stream);

/*
 * starkv_decode_attention for callers that cannot allocate device memory when
 * they run a decode step (plugins that receive only input/output buffers, code
 * running under another framework's memory pool or a locked-down allocator).
 * No counterpart in the reference.  The scratch of the step lives in a fixed
 * static device array of starkv_static_scratch_bytes() bytes (32 MiB) that
 * every GPU loading the library reserves until the process exits; args->
 * workspace and workspace_bytes are ignored.  Steps whose scratch would exceed
 * it (starkv_decode_workspace_size) are rejected with STARKV_ERR_WORKSPACE.
 * The first call on a device looks up the array's device address with that
 * device current, so make it before any stream capture.  All calls share the
 * one array: calls that can overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller.  Allocates nothing.
 */
int starkv_decode_attention_static(const starkv_layout* lay, const starkv_decode_args* args,
                                   starkv_stream_t stream);

/* Size in bytes of the static scratch used by starkv_decode_attention_static. */
size_t starkv_static_scratch_bytes(void);

/* starkv_read_device_error for the static scratch of starkv_decode_attention_static
 * (whose callers never see its address): reads and clears the device error word
 * that a timed-out device wait leaves there (synchronises the stream).  No
 * counterpart in the reference. */
int starkv_static_read_device_error(int* out_code, starkv_stream_t stream);

/*
 * The reference's split quantiser (quant_utils.quantize_r_split_int8_int4_packed,
 * called at LlamaLoRaAttention_headwise_quant.py:107-117, absent from the reference
 * tree): x (rows, r) of dtype -> per row, ranks [0, split_r) as int8 up_q
 * (rows, split_r) with fp16 scale s_up (rows) = absmax / 127, ranks [split_r, r)
 * as signed int4 lo_q (rows, ceil((r - split_r) / 2)) packed as nibble q + 8
 * (even rank low) with fp16 scale s_lo (rows) = absmax / 7.  Symmetric,
 * round-half-even, IEEE fp32; a zero row gets scale 1.
 */
int starkv_quantize_split(const void* x, int32_t dtype, int64_t rows, int32_t r, int32_t split_r, void* up_q,
                          void* s_up, void* lo_q, void* s_lo, starkv_stream_t stream);

/*
 * Test hooks for the device-side failure path (no counterpart in the
 * reference): wait_limit_ns (> 0; 0 restores the default 2 s) bounds every
 * mbarrier wait of the K kernel; skip_copy_unit >= 0 makes the K kernel's
 * first CTA (split 0, head group 0, sequence 0) never issue that unit's staging
 * copy, so that its consumers' waits
 * run out, record an error code in the workspace's first word and return.
 * (0, -1) restores normal operation.  Not for production use.
 */
int starkv_set_test_hooks(int64_t wait_limit_ns, int32_t skip_copy_unit);

/* Reads and clears the device error word at the start of a decode workspace
 * (synchronises the stream); *out_code = 0 means no device-side error. */
int starkv_read_device_error(void* workspace, int* out_code, starkv_stream_t stream);

/*
 * Causal prompt (prefill) attention over K / V rebuilt from the latents: the
 * SDPA call of the reference's prompt path (model.py:429-449,
 * LlamaLoRaAttention_headwise.py:100-116: F.scaled_dot_product_attention with
 * is_causal over RoPE(X_k U_k^T) and X_v U_v^T, GQA by repeat_kv).  q (B, Hq, T,
 * 128) rotated queries, k (B, Hkv, T, 128) rotated keys, v (B, Hkv, T, 128), all
 * of `dtype` (fp16 / bf16) with arbitrary element strides (batch, head, token;
 * multiples of 8, 16-byte aligned bases, the 128 channels contiguous), so the
 * projections' (B, T, H, 128) tensors are read in place.  Query t attends to
 * keys [0, t]; query head h uses KV head h / (Hq / Hkv).  out (B, Hq, T, 128) of
 * out_dtype with its own strides.  error_word (nullable): device int that a
 * timed-out device wait sets (see starkv_read_device_error).  Allocates nothing.
 */
typedef struct starkv_prefill_args {
  const void* q;
  const void* k;
  const void* v;
  int64_t q_strides[3];     /* elements: batch, head, token */
  int64_t k_strides[3];
  int64_t v_strides[3];
  int32_t dtype;            /* STARKV_F16 or STARKV_BF16 */
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t num_tokens;
  float scaling;            /* softmax scale, head_dim^-0.5 in the reference */
  void* out;
  int32_t out_dtype;
  int64_t out_strides[3];
  int* error_word;
} starkv_prefill_args;

int starkv_prefill_attention(const starkv_prefill_args* args, starkv_stream_t stream);

/* Last CUDA error string seen by the library on this thread (for diagnostics). */
const char* starkv_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* STARKV_H */
