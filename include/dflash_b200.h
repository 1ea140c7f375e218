/*
 * dflash_b200.h -- C ABI of the B200-native DFlash draft-model forward.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer
 * (caller-owned) unless stated otherwise; `stream` is a cudaStream_t passed as
 * void*.  Every call returns a status code; dflash_last_error() gives the
 * message of the last failure on the calling thread.  Status mapping for a
 * Python shim: DFLASH_ERR_INVALID -> ValueError, anything else -> RuntimeError
 * (the reference raises PyValueError on weight-length mismatches and
 * PyRuntimeError("ANE kernel '<name>' ... failed") on execution errors,
 * ane/src/wrapper.rs:397-405 and :204-209).
 *
 * Threading: calls on different handles are independent; dflash_forward on
 * one handle serialises internally (its workspace is shared), like the
 * reference's kernels that must not be re-entered on the same buffers.
 * None of these calls needs the Python GIL (ctypes releases it), matching the
 * reference's py.allow_threads around every native call (wrapper.rs:58-221).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   dflash_create    ANEDraftModel.__init__ + load_weights_q8
 *                    (mirror_sd/ane_model.py:47-110, :312-344) and the native
 *                    compile_dflash_kernels_q8 / Q8LayerWeights
 *                    (ane/src/wrapper.rs:363-428, :437-502)
 *   dflash_forward   DFlashDraftModel.__call__ (mirror_sd/dflash.py:384-403)
 *                    and its ANE twin forward / run_kernels /
 *                    read_draft_tokens (ane_model.py:384-416, :564-604),
 *                    followed by lm_head + greedy sample on the last block-1
 *                    rows (mirror_sd/generate.py:604-606)
 *   dflash_accept    the longest-prefix acceptance loop (generate.py:722-728)
 *   dflash_quantize_q8  ANEDraftModel._quantize_weight_q8 (ane_model.py:265-279)
 *   dflash_destroy   drop of the native kernels / buffers (wrapper.rs)
 *   dflash_cache_*   DFlashKVCache and DFlashDraftModel.make_cache
 *                    (mirror_sd/dflash.py:139-212, :405-406): the append with
 *                    sink + window eviction happens inside dflash_forward
 *                    (update_and_fetch, dflash.py:168-193); trim / offset /
 *                    keys are the cache object's own methods
 */
#ifndef DFLASH_B200_H
#define DFLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFLASH_OK 0
#define DFLASH_ERR_INVALID 1 /* bad argument or shape */
#define DFLASH_ERR_CUDA 2    /* CUDA runtime / launch error */
#define DFLASH_ERR_OOM 3     /* device allocation failed */
#define DFLASH_ERR_DEVICE 4  /* a bounded device-side wait expired */

/* Model dimensions (DFlashConfig, mirror_sd/dflash.py:34-50) plus the
 * capacities the workspace is sized for. head_dim must be 128. */
typedef struct DFlashDims {
  int32_t hidden_size;
  int32_t num_hidden_layers;
  int32_t intermediate_size;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  int32_t vocab_size;
  int32_t num_target_features; /* len(target_layer_ids), 5 in every config */
  float rms_norm_eps;
  float rope_theta;
  int32_t max_batch;
  int32_t max_block;
  int32_t max_ctx;      /* context rows of one sequence in one step */
  int32_t max_ctx_rows; /* context rows of one step, all sequences together
                           (0: max_batch * max_ctx).  A stateless step of b
                           sequences also needs b * (max C_s + block) <=
                           max_ctx_rows + max_batch * max_block. */
} DFlashDims;

/* One decoder layer in the reference's W8A16 format: row-major int8
 * [out, in] weights with per-output-channel fp16 scales (the bytes
 * _quantize_weight_q8 returns), fp32 norm weights.  Copied and repacked by
 * dflash_create; the caller may free them afterwards. */
typedef struct DFlashLayerWeights {
  const int8_t* wq; const uint16_t* sq; /* [NQ*128, H] */
  const int8_t* wk; const uint16_t* sk; /* [NKV*128, H] */
  const int8_t* wv; const uint16_t* sv; /* [NKV*128, H] */
  const int8_t* wo; const uint16_t* so; /* [H, NQ*128] */
  const int8_t* wg; const uint16_t* sg; /* [I, H] */
  const int8_t* wu; const uint16_t* su; /* [I, H] */
  const int8_t* wd; const uint16_t* sd; /* [H, I] */
  const float* input_layernorm;          /* [H] */
  const float* post_attention_layernorm; /* [H] */
  const float* q_norm;                   /* [128] */
  const float* k_norm;                   /* [128] */
} DFlashLayerWeights;

typedef struct DFlashWeightsView {
  const uint16_t* fc;          /* bf16 [H, F*H]; copied */
  const float* hidden_norm;    /* [H]; copied */
  const float* norm;           /* [H]; copied */
  const uint16_t* lm_head;     /* bf16 [V, H]: the target's (tied) embedding; copied
                                  into 128-row swizzled tiles (the caller may free it) */
  const DFlashLayerWeights* layers; /* HOST array of num_hidden_layers entries */
} DFlashWeightsView;

/* One draft step.  Sequence s brings C_s new context rows (ctx_lens[s], or
 * ctx_len for every sequence when ctx_lens is NULL) and `block` noise rows.
 * Without a cache (cache=None in dflash.py) the step attends to exactly those
 * C_s + block rows, at RoPE positions off_s + row (rope_offsets[s], or
 * rope_offset), and keeps nothing.  With a cache (dflash_cache_create) the new
 * rows are appended to sequence s of the cache at positions offset_s + row,
 * sink + window eviction is applied, and the step attends to everything the
 * cache then holds (dflash.py:287-317); afterwards the caller trims the block
 * rows with dflash_cache_trim, as generate.py:608-609 does. */
typedef struct DFlashForwardArgs {
  int32_t batch;
  int32_t block;          /* block_size, 2..max_block, batch*block <= 64 */
  int32_t ctx_len;        /* context rows per sequence, 0..max_ctx (when ctx_lens is NULL) */
  int32_t rope_offset;    /* without a cache: position of row 0 (when rope_offsets is NULL) */
  int32_t num_layers;     /* 1..num_hidden_layers (DFlashDraftModel.num_draft_layers) */
  const uint16_t* noise;          /* bf16 [batch, block, H] */
  const uint16_t* target_hidden;  /* bf16 context rows of all sequences packed in order:
                                     [sum_s C_s, F*H] ([batch, ctx_len, F*H] when uniform) */
  void* out_hidden;               /* [batch, block, H] final-normed hidden states, or NULL:
                                     bf16, or fp32 when out_hidden_fp32 != 0 */
  int32_t out_hidden_fp32;
  int32_t* out_tokens;            /* [batch, block-1] greedy draft ids, or NULL */
  const int32_t* target_tokens;   /* [batch, block] verifier posterior, or NULL */
  int32_t* acc_len;               /* [batch], written when target_tokens != NULL */
  int32_t* correction;            /* [batch], target_tokens[b][acc_len[b]] */
  /* Optional phase timing: when n_phase_events >= DFLASH_PHASES, event k
   * (a cudaEvent_t) is recorded on `stream` at phase boundary k:
   * 0 start, 1 after RoPE table + residual init, 2 after the fc GEMM,
   * 3 after hidden_norm (fused into the two GEMMs: recorded with 2),
   * 4 after the context K/V GEMM, 5 after the decoder
   * layers, 6 after the final norm, 7 after lm_head + argmax (+ accept). */
  void* const* phase_events;
  int32_t n_phase_events;
  const int32_t* ctx_lens;        /* HOST array [batch] of C_s, or NULL */
  const int32_t* rope_offsets;    /* HOST array [batch], or NULL; not used with a cache */
  void* cache;                    /* from dflash_cache_create, or NULL (cache=None) */
  /* Soft anchor (generate.py:1422-1436): when anchor_logits is not NULL, row 0
   * of every sequence's block is not read from `noise` but embedded as the
   * softmax-weighted sum of the top-k rows of lm_head under that sequence's
   * logits (the previous verify step at the correction position,
   * generate.py:1639).  NULL keeps the hard anchor (the first step). */
  const void* anchor_logits;      /* device [batch, anchor_logits_ld], fp32 or bf16 */
  int64_t anchor_logits_ld;       /* elements between rows; 0 = vocab_size */
  int32_t anchor_logits_bf16;
  int32_t anchor_top_k;           /* 1..16; 0 = 8, the reference's k */
  /* extract_context_feature fused into the fc GEMM (dflash.py:122-130): when
   * target_layers is not NULL, target_hidden is not read; the fc GEMM loads
   * its A operand from the F selected target layers where they lie.
   * target_layers is a HOST array of num_target_features device pointers,
   * layer f holding bf16 [sum_s C_s, H] context rows (packed like
   * target_hidden) target_layers_ld elements apart (0 = H; 16-byte aligned
   * base and row pitch). */
  const uint16_t* const* target_layers;
  int64_t target_layers_ld;
  /* With a cache: HOST array [batch] of distinct cache sequence indices
   * (< the cache's max_batch): sequence s of this step is cache sequence
   * cache_seqs[s], so one cache serves any subset of its sequences per step
   * (prefill a few, decode all).  NULL: sequences 0..batch-1. */
  const int32_t* cache_seqs;
} DFlashForwardArgs;

#define DFLASH_PHASES 8

/* ---- fp32-accumulate mode ------------------------------------------------
 * A handle made by dflash_create_f32 runs the whole draft step in fp32 on the
 * CUDA cores: fp32 weights (no quantisation), fp32 activations and fp32
 * accumulation everywhere -- the arithmetic of mirror_sd/dflash.py on fp32
 * weights (DFlashDraftModel.__call__, dflash.py:384-403) -- so its greedy draft
 * ids and accepted lengths follow an fp32 evaluation of the reference.
 * dflash_forward on such a handle reads `noise` as fp32 [batch, block, H] and
 * `target_hidden` as fp32 [sum_s C_s, F*H] (same pointers, fp32 data), writes
 * `out_hidden` as fp32 (out_hidden_fp32 is ignored), and takes the stateless
 * arguments only: `cache`, `anchor_logits` and `target_layers` must be NULL.
 * All weights are device pointers, row-major [out, in], copied by the call. */
typedef struct DFlashLayerWeightsF32 {
  const float* wq; /* [NQ*128, H] */
  const float* wk; /* [NKV*128, H] */
  const float* wv; /* [NKV*128, H] */
  const float* wo; /* [H, NQ*128] */
  const float* wg; /* [I, H] */
  const float* wu; /* [I, H] */
  const float* wd; /* [H, I] */
  const float* input_layernorm;          /* [H] */
  const float* post_attention_layernorm; /* [H] */
  const float* q_norm;                   /* [128] */
  const float* k_norm;                   /* [128] */
} DFlashLayerWeightsF32;

typedef struct DFlashWeightsViewF32 {
  const float* fc;           /* [H, F*H] */
  const float* hidden_norm;  /* [H] */
  const float* norm;         /* [H] */
  const float* lm_head;      /* [V, H]: the target's (tied) embedding */
  const DFlashLayerWeightsF32* layers; /* HOST array of num_hidden_layers entries */
} DFlashWeightsViewF32;

/* DFlashDraftModel over fp32 weights (dflash.py:365-382 with an fp32
 * checkpoint; the reference's MLX CPU path computes in the weights' dtype). */
int dflash_create_f32(const DFlashDims* dims, const DFlashWeightsViewF32* weights, int device,
                      void** handle);

int dflash_create(const DFlashDims* dims, const DFlashWeightsView* weights, int device,
                  void** handle);
int dflash_forward(void* handle, const DFlashForwardArgs* args, void* stream);
int dflash_accept(const int32_t* draft, const int32_t* target, int batch, int block,
                  int32_t* acc_len, int32_t* correction, void* stream);
int dflash_quantize_q8(const float* w, int oc, int ic, int8_t* q, uint16_t* scale_fp16,
                       void* stream);
/* Reads and clears the handle's device error word (DFLASH_ERR_DEVICE when a
 * kernel gave up on a bounded wait).  Synchronises the given stream. */
int dflash_device_status(void* handle, void* stream);
/* Failure-reporting self test (no reference counterpart): enqueues one
 * bounded mbarrier wait that nothing completes, `polls` tries long.  It gives
 * up, records the timeout in the handle's error word like any expired wait of
 * the library, and returns; the next dflash_device_status reports
 * DFLASH_ERR_DEVICE and clears it, and the context stays usable. */
int dflash_probe_bounded_wait(void* handle, uint32_t polls, void* stream);
int dflash_destroy(void* handle);
/* Number of kernel launches the last dflash_forward on this handle issued. */
int dflash_last_launch_count(void* handle);
int dflash_last_error(char* buf, size_t len);
int dflash_version(void);

/* ---- draft KV cache (dflash.py:139-212) ---------------------------------
 * K/V rows of every layer and sequence stay on the device in
 * [layer][sequence][kv head][slot][128] f16 rings.  Eviction of the middle rows
 * moves a ring start, trim shortens the list: no row is ever copied.  Eviction
 * is on when sink_size > 0 and window_size > 0 (dflash.py:180-181); the cache
 * then holds sink_size + window_size + max_ctx + max_block slots per sequence.
 * Without eviction it holds max_len slots and a step that would overflow them
 * is rejected.  Offsets and lengths are host-side state: the cache ops below
 * enqueue no device work (dflash_cache_read excepted). */
int dflash_cache_create(void* handle, int num_layers, int max_batch, int sink_size, int window_size,
                        int max_len, void** cache);
/* DFlashKVCache.trim(n) (dflash.py:195-207) on one layer, or on every layer
 * when layer < 0, for every sequence: length -> max(length - n, 0),
 * offset -> offset - n.  n <= 0 does nothing. */
int dflash_cache_trim(void* cache, int layer, int n);
/* trim(counts[i]) of cache sequence seqs[i] only, i < count (HOST arrays;
 * layer -1 = every layer): per-sequence rollback in a batched decode. */
int dflash_cache_trim_seqs(void* cache, int layer, const int32_t* seqs, const int32_t* counts, int count);
/* Empty every sequence (offset 0).  Device contents are not touched. */
int dflash_cache_reset(void* cache);
/* Empty cache sequences seqs[0..count) (offset 0, no rows), e.g. to give a
 * slot to a new request; the other sequences keep their rows. */
int dflash_cache_reset_seqs(void* cache, const int32_t* seqs, int count);
/* DFlashKVCache.offset and keys.shape[2] of one layer and sequence. */
int dflash_cache_state(void* cache, int layer, int seq, int32_t* offset, int32_t* length);
/* DFlashKVCache.keys / .values of one layer and sequence, in logical order, as
 * f16 [NKV, length, 128] into caller buffers (either may be NULL). */
int dflash_cache_read(void* cache, int layer, int seq, uint16_t* keys, uint16_t* values,
                      void* stream);
int dflash_cache_destroy(void* cache);

/* ---- kernel-level entry points (one hot-path kernel each) ---------------- */

/* y[M, N] (f16) = x[M, K] (f16) . (q[N, K] * s[N])^T on the W8A16 skinny
 * kernel (the q/k/v/o/gate/up/down projections of the block rows; the
 * reference's conv1x1_proj_q8, ane/src/dflash.rs:146-149).  M <= 64. */
int dflash_w8_linear(const int8_t* q, const uint16_t* s_fp16, int N, int K, const uint16_t* x_f16,
                     int M, uint16_t* y_f16, void* stream);

/* D[M, N] (fp32) = A[M, K] . B[N, K]^T on the tcgen05 GEMM; ab_bf16 selects
 * bf16 (1) or f16 (0) operands (the fc projection, dflash.py:373-378, and the
 * context K/V projection, dflash.py:293-294). */
int dflash_tc_gemm(const uint16_t* A, const uint16_t* B, int M, int N, int K, int ab_bf16,
                   float* D, void* stream);

/* Fused per-head QK RMSNorm + neox RoPE + non-causal GQA attention
 * (dflash.py:291-317; ANE gqa_tile + attn_out, ane/src/dflash.rs:226-278).
 * q [batch, NQ, block, 128], k/v [batch, NKV, kv_len, 128] f16;
 * out [batch, block, NQ*128] f16.  When normrope != 0, q row j is normalised
 * and rotated at position q_pos0 + j and k row i at k_pos0 + i; otherwise q/k
 * are used as given.  workspace: dflash_attention_workspace_size() bytes. */
size_t dflash_attention_workspace_size(int batch, int nq, int nkv, int block, int kv_len);
int dflash_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int batch, int nq,
                     int nkv, int block, int kv_len, int normrope, const float* q_norm,
                     const float* k_norm, float rope_theta, int q_pos0, int k_pos0, float eps,
                     uint16_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* The same attention without any device allocation and without a caller
 * workspace.  It has no counterpart in the reference.  It is for callers that
 * cannot call cudaMalloc: a host runtime that has reserved the device's memory
 * up front for its own pool and forbids side allocations, or a binding that
 * has no way to pass a workspace buffer.
 *
 * Scratch: the split-KV partials and the RoPE table live in one static device
 * array of DFLASH_ATTN_STATIC_SCRATCH_BYTES.  Every GPU that loads this library
 * holds that array until the process exits.  A shape whose
 * dflash_attention_workspace_size() exceeds the array is rejected with
 * DFLASH_ERR_INVALID.
 *
 * Device address: every call looks the array's address up on the caller's
 * current device (cudaGetSymbolAddress; cheap once the library's device code
 * is loaded there).  The first call on a device loads that code, so make the
 * first call outside any stream capture.
 *
 * Sharing: all calls on a device share the one array, and it keeps whatever
 * the last call left in it.  Every byte a call reads is written earlier in
 * that call, so nothing needs clearing.  Two calls whose kernels overlap on
 * the GPU (different streams, no ordering between them) race on the array.
 * Serialise them on one stream, or use dflash_attention with separate
 * workspaces. */
#define DFLASH_ATTN_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int dflash_attention_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, int batch,
                             int nq, int nkv, int block, int kv_len, int normrope,
                             const float* q_norm, const float* k_norm, float rope_theta,
                             int q_pos0, int k_pos0, float eps, uint16_t* out, void* stream);


/* Soft anchor on its own (generate.py:1422-1436): for each of `batch` rows
 * of logits ([batch, ld], fp32 or bf16 when logits_bf16), the k largest
 * entries (larger first, lower index first on ties), their fp32 softmax, and
 * out[row] = bf16(sum_q w_q * E[id_q]) with E [V, H] bf16 row-major
 * (H % 8 == 0, 16-byte aligned).  workspace: dflash_soft_anchor_workspace_size()
 * bytes. */
size_t dflash_soft_anchor_workspace_size(int batch);
int dflash_soft_anchor(const void* logits, int logits_bf16, int batch, int V, int64_t ld, int k,
                       const uint16_t* E, int H, uint16_t* out, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Tied lm_head + greedy argmax (+ acceptance when target != NULL) on
 * final-normed hidden rows: hn [batch, block, H] bf16, E [V, H] bf16; writes
 * tokens [batch, block-1] for rows 1..block-1 (generate.py:604-606, :722-728).
 * workspace: dflash_lm_head_workspace_size() bytes; it also holds the copy of
 * E repacked into the kernel's vocabulary tiles, so the call allocates
 * nothing. */
size_t dflash_lm_head_workspace_size(int batch, int block, int V, int H);
int dflash_lm_head_argmax(const uint16_t* hn, const uint16_t* E, int batch, int block, int H,
                          int V, int32_t* tokens, const int32_t* target, int32_t* acc_len,
                          int32_t* correction, void* workspace, size_t workspace_bytes,
                          void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DFLASH_B200_H */
