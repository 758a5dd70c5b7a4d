/*
 * ps_attn.h -- C ABI of the B200 paged split-KV ("PS") attention library.
 *
 * libps_attn.so replaces the two GPU calls that vLLM's FlashAttention backend
 * makes per decoder layer (vllm/v1/attention/backends/flash_attn.py):
 *
 *   do_kv_cache_update -> reshape_and_cache_flash      (flash_attn.py:874-883)
 *   forward            -> flash_attn_varlen_func(...)   (flash_attn.py:796-817)
 *
 * Conventions shared by every entry point:
 *   - plain device pointers, element strides (not bytes) and sizes; no
 *     framework types cross this boundary;
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default);
 *     nothing synchronises the host, nothing allocates device memory;
 *   - the return value is a ps_status; on failure ps_last_error() returns a
 *     message for the calling thread;
 *   - device-side range checks never trap: they set bits in a caller-owned
 *     int32 status word (PS_DEV_*) and skip the offending access.
 */
#ifndef PS_ATTN_H_
#define PS_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PS_ATTN_ABI_VERSION 3

/* host-side return codes */
typedef enum {
  PS_OK = 0,
  PS_ERR_INVALID_ARGUMENT = 1, /* shape, stride, alignment or pointer error */
  PS_ERR_UNSUPPORTED = 2,      /* valid request this build does not handle */
  PS_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  PS_ERR_CUDA = 4              /* a CUDA runtime/driver call failed */
} ps_status;

/* bits of the device status word */
#define PS_DEV_SLOT_OUT_OF_RANGE 0x1  /* kv_append: slot >= num_blocks*block_size */
#define PS_DEV_BLOCK_OUT_OF_RANGE 0x2 /* attention: block_table entry outside the pool */
#define PS_DEV_WAIT_TIMEOUT 0x4       /* a bounded device wait gave up */
#define PS_DEV_BAD_METADATA 0x8       /* seq_lens / query_start_loc inconsistent */

/* element types */
typedef enum { PS_DTYPE_FP16 = 0, PS_DTYPE_BF16 = 1, PS_DTYPE_FP32 = 2 } ps_dtype;

/* KV-cache element type (ps_paged_problem.kv_cache_dtype). */
#define PS_KV_AUTO 0      /* the problem's dtype */
#define PS_KV_FP8_E4M3 1  /* e4m3fn codes (uint8), per-tensor scales k_scale / v_scale */

int ps_abi_version(void);
const char* ps_last_error(void);

/*
 * KV append.  Replaces torch.ops._C_cache_ops.reshape_and_cache_flash
 * (vllm/_custom_ops.py:2591-2610; semantics of its readable twin
 * vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:44-87, NHD layout):
 *
 *   for t < num_tokens with s = slot_mapping[t] >= 0:
 *     key_cache  [s / block_size, s % block_size, h, :] = key  [t, h, :]
 *     value_cache[s / block_size, s % block_size, h, :] = value[t, h, :]
 *
 * An exact byte copy for any element size (2 or 4 bytes).  key/value may hold
 * more than num_tokens rows (vLLM pads them); slot_mapping's length rules.
 * The last dimension of every tensor is contiguous.  status (nullable) gets
 * PS_DEV_SLOT_OUT_OF_RANGE for slots beyond the pool; those rows are skipped.
 */
int ps_kv_append(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                 const void* value, int64_t value_stride_token, int64_t value_stride_head,
                 void* key_cache, void* value_cache, int64_t cache_stride_block,
                 int64_t cache_stride_slot, int64_t cache_stride_head, int64_t num_blocks,
                 const int64_t* slot_mapping, int64_t num_tokens, int num_kv_heads,
                 int head_size, int block_size, int elem_bytes, int32_t* status, void* stream);

/*
 * A batch of paged attention problems: the argument set of
 * flash_attn_varlen_func's paged branch (vllm/vllm_flash_attn/
 * flash_attn_interface.py:176-394) as the FlashAttention backend calls it.
 * Sequence b owns query rows [query_start_loc[b], query_start_loc[b+1]) and
 * the first seq_lens[b] tokens of its pages; page p of sequence b is cache
 * block block_table[b * block_table_stride + p].  Attention is causal with
 * bottom-right alignment (query row i of a q_len-row sequence sees keys
 * j <= seq_len - q_len + i), which for decode (q_len = 1) is all seq_len keys.
 */
typedef struct {
  /* query [num_tokens, num_q_heads, head_size] */
  const void* q;
  int64_t q_stride_token, q_stride_head;
  /* paged cache: key_cache/value_cache [num_blocks, block_size, num_kv_heads,
     head_size] (the two halves of vLLM's [2, num_blocks, ...] tensor) */
  const void* key_cache;
  const void* value_cache;
  int64_t cache_stride_block, cache_stride_slot, cache_stride_head;
  int64_t num_blocks;
  /* metadata (device) */
  const int32_t* block_table;     /* [num_seqs, max_blocks_per_seq] */
  int64_t block_table_stride;
  int32_t max_blocks_per_seq;
  const int32_t* seq_lens;        /* [num_seqs], includes the new tokens */
  const int32_t* query_start_loc; /* [num_seqs + 1]; NULL = one query row per sequence */
  int32_t num_seqs;
  /* output [num_tokens, num_q_heads, head_size], same dtype as q */
  void* out;
  int64_t out_stride_token, out_stride_head;
  /* natural-log LSE, fp32, nullable: lse[h * lse_stride_head + t * lse_stride_token] */
  float* lse;
  int64_t lse_stride_head, lse_stride_token;
  /* shape */
  int32_t num_q_heads, num_kv_heads, head_size, block_size;
  int32_t dtype; /* ps_dtype of q, cache and out */
  float softmax_scale;
  /* rows of q / out (the extent chunked prefill's Q tile loads are bounded by) */
  int64_t num_tokens;
  /* device status word (PS_DEV_* bits), nullable; ps_paged_decode uses the
     one in its workspace instead */
  int32_t* status;
  /* Optional KV append fused into ps_paged_decode (NULL new_key = off; the
     other entry points ignore these fields).  For each sequence b with a
     query row t, the new key/value rows [t, :, :] are written to the cache at
     slot_mapping[t] (slot < 0: skipped) -- the contract of ps_kv_append --
     and attention sees them as the sequence's last token.  The slot must be
     that of position seq_lens[b] - 1 (it always is for vLLM decode); a
     mismatch sets PS_DEV_BAD_METADATA. */
  const void* new_key;
  int64_t new_key_stride_token, new_key_stride_head;
  const void* new_value;
  int64_t new_value_stride_token, new_value_stride_head;
  const int64_t* slot_mapping;
  /* KV-cache element type, PS_KV_AUTO (0) or PS_KV_FP8_E4M3.  An fp8 cache
     holds e4m3(x / scale) codes (ps_kv_append_fp8, or the fused append) --
     vLLM's kv_cache_dtype "fp8" with layer._k_scale / _v_scale; its strides
     are in bytes.  ps_paged_decode takes it; chunked prefill attends over
     the pages ps_kv_dequant_gather copies out (the other entry points return
     PS_ERR_UNSUPPORTED).  k_scale / v_scale (device fp32 scalars, NULL =
     1.0): attention reads K * k_scale and V * v_scale, for any cache dtype
     (ps_paged_decode, the cascade decode, chunked prefill; DCP takes none). */
  int32_t kv_cache_dtype;
  const float* k_scale;
  const float* v_scale;
} ps_paged_problem;

/*
 * KV append into an fp8 (e4m3) cache: cache[slot] = e4m3(x / k_scale) for
 * the key, e4m3(x / v_scale) for the value (the quotient rounded to fp32,
 * then to the nearest e4m3, ties to even, saturating at +-448), slot < 0
 * skipped -- reshape_and_cache_flash with kv_cache_dtype "fp8"
 * (triton_reshape_and_cache_flash.py:93-110).  key/value: fp16 or bf16
 * (dtype), rows 16-byte aligned; caches: uint8 [num_blocks, block_size,
 * num_kv_heads, head_size] with byte strides that are multiples of 8;
 * head_size a multiple of 8; k_scale / v_scale: device fp32 scalars (NULL =
 * 1.0).
 */
int ps_kv_append_fp8(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                     const void* value, int64_t value_stride_token, int64_t value_stride_head,
                     void* key_cache, void* value_cache, int64_t cache_stride_block,
                     int64_t cache_stride_slot, int64_t cache_stride_head, int64_t num_blocks,
                     const int64_t* slot_mapping, int64_t num_tokens, int32_t num_kv_heads,
                     int32_t head_size, int32_t block_size, int32_t dtype, const float* k_scale,
                     const float* v_scale, int32_t* status, void* stream);

/*
 * The pages of an fp8 cache that a batch of sequences reads, dequantized
 * into a 16-bit scratch cache, for the entry points that take 16-bit pages
 * (chunked prefill over an fp8 cache): page p < ceil(seq_lens[b] /
 * block_size) of sequence b -- cache block block_table[b * stride + p] --
 * becomes scratch block b * max_pages + p of out_key / out_value
 * ([num_seqs * max_pages, block_size, num_kv_heads, 128], problem->dtype),
 * each element code * scale rounded to that dtype.  Other scratch blocks are
 * left untouched; attend over the scratch with the block table
 * [b][p] = b * max_pages + p.  Uses the problem's fp8 cache (contiguous
 * blocks), block table, seq_lens, num_seqs, shape, dtype, k_scale / v_scale
 * and status (nullable).
 */
int ps_kv_dequant_gather(const ps_paged_problem* problem, int32_t max_pages, void* out_key,
                         void* out_value, void* stream);

/*
 * Bytes of workspace ps_paged_decode needs for up to num_seqs sequences on
 * the current device.  The size does not depend on sequence lengths, so one
 * buffer sized for max_num_seqs serves every step and every CUDA-graph
 * replay.  The buffer must be zeroed once before first use (the kernel keeps
 * its counters at zero between calls); its first int32 is the status word.
 * After PS_DEV_WAIT_TIMEOUT the buffer must be zeroed again.
 */
int64_t ps_paged_decode_workspace_size(int32_t num_seqs, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_size);

/*
 * Paged decode: one query row per sequence (q_len 1; a sequence with q_len 0
 * is skipped).  Replaces flash_attn_varlen_func(..., block_table=...,
 * seqused_k=seq_lens, fa_version=4) for max_seqlen_q == 1
 * (flash_attn.py:796-817 -> vllm/vllm_flash_attn/cute/interface.py:289-1063)
 * and the split combine FA4 launches after it (cute/interface.py:1052-1060,
 * cute/flash_fwd_combine.py:21-698), which here is fused: the last split of a
 * (sequence, kv head) to finish merges all splits.  With problem->new_key set
 * it also performs the KV append of the decode tokens (the caches are then
 * written), replacing the separate ps_kv_append launch.
 */
int ps_paged_decode(const ps_paged_problem* problem, void* workspace, int64_t workspace_bytes,
                    void* stream);

/*
 * Paged decode with library-owned scratch memory.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory, such
 * as a backend running inside an inference engine that reserved the GPU's
 * memory up front (vLLM sizes its KV cache to most of HBM at start-up) and
 * hands none of it to plugins.  Same semantics and outputs as
 * ps_paged_decode, but no workspace argument: the split counters and partials
 * live in a 16 MiB array inside the library, of which every GPU that loads it
 * holds one copy until the process exits.  A problem is rejected with
 * PS_ERR_WORKSPACE when its decode scratch (ps_paged_decode_workspace_size:
 * a split record per warp, 8 warps per SM with either cache dtype, plus one
 * per (sequence, kv head)) exceeds 16 MiB -- with 8 KV heads, GQA group <= 8
 * and 148 SMs, at most 352 sequences per call.  Allocates nothing (no cudaMalloc / cudaFree).  The
 * first call on a device looks up the array's device address for that device;
 * make that first call before any stream capture.  All calls share the one
 * array: calls that can overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller.  problem->status (nullable)
 * receives this call's PS_DEV_* bits.
 */
int ps_paged_decode_static_scratch(const ps_paged_problem* problem, void* stream);

/*
 * Shared-prefix ("cascade") decode.  vLLM's FlashAttention backend runs
 * cascade attention only when every request of the batch shares one prefix
 * (flash_attn.py:1088-1130 use_cascade_attention, :1132-1223
 * cascade_attention + merge_attn_states); GRPO rollouts instead share one
 * prompt per group of samples.  These three calls generalise it to per-group
 * prefixes; they have no single counterpart in the reference.
 *
 * ps_cascade_plan_build finds groups of adjacent decode sequences whose
 * leading block-table entries are identical (what prefix caching produces
 * for samples of one prompt) and writes them to `plan`, a device buffer of
 * ps_cascade_plan_bytes(num_seqs) bytes, zeroed once before its first use.
 * Only pages that are complete in every member count as shared; a group
 * needs >= 2 members and >= min_shared_pages shared 16-token pages.  The
 * plan is a function of block_table, seq_lens and query_start_loc: build it
 * once per step and reuse it for every layer.  Plan layout (int32 words, B =
 * num_seqs, Gm = max(1, B / 2)): [0] number of groups, [1] internal,
 * [32, 32 + B) group of each sequence (-1: none), then first sequence, member
 * count and shared pages of each group (Gm words each), then the pages each
 * sequence shares with its predecessor (B words).
 *
 * ps_paged_decode_cascade computes exactly what ps_paged_decode computes
 * (same outputs, LSE and fused append) for the problem the plan was built
 * from: each group's shared pages are read once per 16 query columns
 * (members x GQA heads) instead of once per member, and the prefix result is
 * merged into each member's split combine.  num_seqs <= 2048 and GQA group <=
 * 8.  A plan inconsistent with the problem sets PS_DEV_BAD_METADATA and the
 * call runs as a plain decode.  The workspace (zeroed once) may be shared
 * with ps_paged_decode if it has the larger of the two sizes.
 */
int64_t ps_cascade_plan_bytes(int32_t num_seqs);
int ps_cascade_plan_build(const ps_paged_problem* problem, int32_t min_shared_pages, void* plan,
                          int64_t plan_bytes, void* stream);
int64_t ps_paged_decode_cascade_workspace_size(int32_t num_seqs, int32_t num_q_heads,
                                               int32_t num_kv_heads, int32_t head_size);
int ps_paged_decode_cascade(const ps_paged_problem* problem, const void* plan, int64_t plan_bytes,
                            void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Fused rotary embedding + KV append.  Replaces the custom op
 * fused_rope_and_unified_kv_cache_update
 * (vllm/compilation/passes/fusion/rope_kvcache_fusion.py:40-73), i.e.
 * AttentionImpl.do_rope_and_kv_cache_update (vllm/v1/attention/backend.py:
 * 815-841), which vLLM's fusion pass substitutes for rotary_embedding followed
 * by the KV update:
 *
 *   query[t, h, :], key[t, h, :] <- RoPE(., positions[t])       (in place)
 *   key_cache / value_cache at slot_mapping[t] <- rotated key, value
 *                                   (ps_kv_append's contract; slot < 0 skipped)
 *
 * RoPE as vLLM's torch-native rotary embedding
 * (rotary_embedding/base.py:140-181): cos_sin_cache rows are [cos | sin] of
 * rotary_dim / 2 entries each, cast to the model dtype; neox style pairs
 * element i with i + rotary_dim / 2, GPT-J style 2i with 2i + 1; every
 * product and sum is rounded to the model dtype (bit-identical to the
 * reference); dims past rotary_dim pass through.  Positions outside
 * [0, max_position) set PS_DEV_BAD_METADATA and leave that token untouched.
 * Strides in elements; the last dimension of every tensor is contiguous.
 */
typedef struct {
  void* query;        /* [num_tokens, num_q_heads, head_size] */
  int64_t query_stride_token, query_stride_head;
  void* key;          /* [num_tokens, num_kv_heads, head_size] */
  int64_t key_stride_token, key_stride_head;
  const void* value;  /* [num_tokens, num_kv_heads, head_size] */
  int64_t value_stride_token, value_stride_head;
  void* key_cache;
  void* value_cache;  /* [num_blocks, block_size, num_kv_heads, head_size] */
  int64_t cache_stride_block, cache_stride_slot, cache_stride_head;
  int64_t num_blocks;
  int32_t block_size;
  const int64_t* slot_mapping; /* [num_tokens] */
  const int64_t* positions;    /* [num_tokens] */
  const void* cos_sin_cache;   /* [max_position, rotary_dim] */
  int64_t cos_sin_stride;      /* elements between rows */
  int64_t max_position;
  int32_t cos_sin_dtype;       /* PS_DTYPE_FP32 or the model dtype */
  int32_t rotary_dim;          /* even, <= head_size */
  int32_t is_neox;
  int64_t num_tokens;
  int32_t num_q_heads, num_kv_heads, head_size;
  int32_t dtype;               /* PS_DTYPE_BF16 or PS_DTYPE_FP16 */
  int32_t* status;             /* nullable, PS_DEV_* bits */
} ps_rope_append_problem;

int ps_rope_kv_append(const ps_rope_append_problem* problem, void* stream);

/*
 * Chunked prefill: any q_len >= 1 per sequence, causal bottom-right, over the
 * same paged cache.  Replaces flash_attn_varlen_func for max_seqlen_q > 1
 * (flash_attn.py:796-817 -> cute/flash_fwd_sm100.py).  Tensor-core path:
 * tcgen05 MMA with TMEM accumulators.  No workspace; problem->num_tokens
 * must be the row count of q/out and problem->status (nullable) receives
 * PS_DEV_* bits.
 */
int ps_chunked_prefill(const ps_paged_problem* problem, void* stream);

/*
 * ps_chunked_prefill with dynamic work distribution: the (sequence, kv head,
 * pair of 128-row Q tiles) units are claimed by the CTAs through two int32
 * counters at bytes 16..23 of `workspace` (>= 256 bytes, 256-byte aligned,
 * zeroed once; a ps_paged_decode workspace serves, its counters are
 * elsewhere) instead of the fixed round-robin of ps_chunked_prefill, so
 * CTAs that finish early take the remaining units.  Same outputs.  Prefill
 * calls that can overlap on the GPU must not share a workspace.  No
 * counterpart in the reference (an implementation choice inside the
 * flash_attn_varlen_func replacement).
 */
int ps_chunked_prefill_ws(const ps_paged_problem* problem, void* workspace,
                          int64_t workspace_bytes, void* stream);

/*
 * Decode context parallelism (DCP).  The `world` ranks of a DCP group (one
 * GPU each, up to PS_DCP_MAX_WORLD, NVLink peers) hold interleaved slices of
 * every sequence's KV tokens: position p is stored by rank (p / I) % world
 * (I = interleave) at local index (p / (world*I)) * I + p % I of that rank's
 * paged cache, under a block table that is the same on every rank -- vLLM's
 * placement (vllm/v1/worker/block_table.py:357-376, cp_kv_cache_interleave_size).
 * Each rank holds hq_local query heads; the group attends with the
 * world * hq_local heads in rank order.
 *
 * Ranks exchange data through a "slab" of device memory each allocates
 * (ps_dcp_slab_alloc, zeroed) and the others map (ps_dcp_ipc_handle /
 * ps_dcp_ipc_open, CUDA IPC).  One slab serves every layer and every call.
 * Replaces: vLLM's query all_gather and context attention with LSE
 * (flash_attn.py:906-940), cp_lse_ag_out_rs (vllm/v1/attention/ops/common.py:195-225
 * with correct_attn_out :99-170), the new tokens' attention and
 * merge_attn_states (flash_attn.py:950-983), and reshape_and_cache_flash of
 * the new tokens -- without NCCL: peer loads plus two flag barriers per call
 * whose waits are bounded (1 s; then PS_DEV_WAIT_TIMEOUT, after which the
 * workspace must be zeroed and the slabs recreated).
 */
#define PS_DCP_MAX_WORLD 8
#define PS_DCP_IPC_HANDLE_BYTES 64

/* Slab bytes for calls of up to max_tokens decode tokens (<= 4096). */
int64_t ps_dcp_slab_bytes(int32_t max_tokens, int32_t hq_local, int32_t world);
/* cudaMalloc + zero a slab on the current device (synchronous). */
int ps_dcp_slab_alloc(int64_t bytes, void** slab);
int ps_dcp_slab_free(void* slab);
/* 64-byte CUDA IPC handle of a slab from ps_dcp_slab_alloc, for the peers. */
int ps_dcp_ipc_handle(const void* slab, void* handle);
/* Map a peer's slab into this process (another process's handle). */
int ps_dcp_ipc_open(const void* handle, void** peer_slab);
int ps_dcp_ipc_close(void* peer_slab);

typedef struct {
  /* This rank's call, decode only (one query row per sequence):
     q / out [num_seqs, hq_local, 128] (num_q_heads = hq_local), lse
     (nullable) [hq_local, num_seqs]; key_cache / value_cache / num_blocks:
     this rank's cache; block_table: the group's; seq_lens: GLOBAL lengths,
     the new token included; query_start_loc must be NULL; num_tokens =
     num_seqs; new_key / new_value [num_seqs, num_kv_heads, 128]: the new
     tokens' rows (every rank has them); slot_mapping: this rank's slots,
     < 0 where another rank stores the token. */
  ps_paged_problem local;
  int32_t world, rank, interleave; /* interleave divides block_size */
  int32_t max_tokens;              /* the slabs were sized for it */
  void* slabs[PS_DCP_MAX_WORLD];   /* every rank's slab, addressed from this GPU */
  int32_t flags;                   /* PS_DCP_* */
} ps_dcp_problem;

/* ps_dcp_problem.flags: PS_DCP_CONTEXT_ONLY -- the step stops after the
   cross-rank correction: out / lse receive the attention over the context
   alone (the new tokens' own attention and the append are left to the
   caller; new_key / new_value / slot_mapping are not read).  The first half
   of a DCP step over multi-token chunks: one row per chunk token, each row a
   one-row "sequence" whose seq_lens entry is its context length + 1. */
#define PS_DCP_CONTEXT_ONLY 1

/*
 * One DCP decode step on this rank (every rank of the group makes the same
 * calls in the same order, each on its own GPU): out[t, h] = attention of
 * the group's query head rank*hq_local + h over the sequence's whole context
 * (all ranks' slices plus the new token), the new token appended where
 * slot_mapping >= 0.  The workspace is a ps_paged_decode workspace for
 * (num_seqs, world * hq_local, num_kv_heads); its status word receives the
 * PS_DEV_* bits.  Four launches on `stream`, no host synchronisation, CUDA
 * graph safe.
 */
int ps_dcp_decode(const ps_dcp_problem* problem, void* workspace, int64_t workspace_bytes,
                  void* stream);

/*
 * The same step split at its barriers, for one process that drives every
 * rank of a group on one GPU in turn (a rank's barrier wait must not run
 * before the other ranks have signalled, since kernels on one GPU are not
 * guaranteed to run concurrently): phase 0 stages the query rows, 1
 * signals barrier 0, 2 gathers the queries and attends over the local
 * context, 3 signals barrier 1, 4 combines and appends.  Run phase k for
 * every rank before phase k+1 for any.
 */
int ps_dcp_decode_phase(const ps_dcp_problem* problem, int32_t phase, void* workspace,
                        int64_t workspace_bytes, void* stream);

/*
 * merge_attn_states (vllm/v1/attention/ops/merge_attn_states.py:9, Triton
 * kernel triton_merge_attn_states.py:58-140): two partial attentions of the
 * same query rows over disjoint key sets, outputs [num_tokens, num_heads, 128]
 * (fp16/bf16, element strides) and natural-log LSEs [num_heads, num_tokens]
 * (fp32, contiguous; +inf counts as -inf), into out (may alias an input) and
 * out_lse (nullable).
 */
int ps_merge_attn_states(const void* prefix_out, int64_t prefix_stride_token,
                         int64_t prefix_stride_head, const float* prefix_lse,
                         const void* suffix_out, int64_t suffix_stride_token,
                         int64_t suffix_stride_head, const float* suffix_lse, void* out,
                         int64_t out_stride_token, int64_t out_stride_head, float* out_lse,
                         int64_t num_tokens, int32_t num_heads, int32_t head_size, int32_t dtype,
                         void* stream);

/*
 * Head all-gather of a KV-head-sharded decode over peer memory: the
 * all_gather_into_tensor + permute that follows tensor-parallel attention
 * (each rank owns KV heads [r*Hkv/world, ...) and their query heads), done by
 * NVLink loads instead of NCCL.  Each rank's decode writes its rows
 * [num_tokens, hq_local, 128] (2-byte elements, contiguous) into its own slab
 * at byte offset PS_HEAD_GATHER_ROWS_OFFSET (ps_paged_decode with that `out`);
 * ps_head_gather then writes every rank's rows into out[t, r*hq_local + j, :].
 * Slabs: ps_dcp_slab_alloc of ps_head_gather_slab_bytes, mapped in the peers
 * with ps_dcp_ipc_handle / ps_dcp_ipc_open, one per rank, reused by every
 * call.  Two flag barriers per call (rows ready; rows pulled, so that no
 * rank's next decode overwrites rows a peer still reads), bounded as in
 * ps_dcp_decode: PS_DEV_WAIT_TIMEOUT in *status (required, device int32).
 */
#define PS_HEAD_GATHER_ROWS_OFFSET 256
int64_t ps_head_gather_slab_bytes(int32_t max_tokens, int32_t hq_local);

typedef struct {
  int32_t world, rank;
  int32_t num_tokens, hq_local;
  int32_t max_tokens;             /* the slabs were sized for it */
  int32_t dtype;                  /* PS_DTYPE_BF16 or PS_DTYPE_FP16 */
  void* slabs[PS_DCP_MAX_WORLD];  /* every rank's slab, addressed from this GPU */
  void* out;                      /* [num_tokens, world * hq_local, 128] */
  int64_t out_stride_token, out_stride_head;
  int32_t* status;
} ps_head_gather_problem;

int ps_head_gather(const ps_head_gather_problem* problem, void* stream);
/* Split at the barriers, for one process playing every rank on one GPU:
   phase 0 signals "rows ready", 1 pulls and signals "rows pulled", 2 waits
   for every rank's "rows pulled".  Run phase k for every rank before phase
   k+1 for any. */
int ps_head_gather_phase(const ps_head_gather_problem* problem, int32_t phase, void* stream);

/*
 * KV-head-sharded decode with the head all-gather fused in: one launch per
 * rank does ps_paged_decode (with the fused append when the problem asks for
 * it) and ps_head_gather's exchange, so the NVLink transfers overlap the
 * decode instead of following it.  The reference has no single counterpart:
 * it is tensor-parallel attention (vLLM splits heads over ranks,
 * vllm/model_executor/models/qwen3.py:78-107) followed by
 * all_gather_into_tensor of the head outputs, in one kernel.
 *
 * problem: this rank's decode (its query heads, num_q_heads == gather->hq_local,
 * and its KV heads' caches); problem->out and its strides are ignored -- the
 * rows go to gather->out at heads [rank * hq_local, (rank + 1) * hq_local),
 * and every finished row is also stored over NVLink into each peer's slab,
 * [max_tokens, world * hq_local, 128] at byte offset 256.  At the end every
 * rank copies the peers' rows from its own slab into gather->out, so when
 * the launch completes gather->out holds [num_tokens, world * hq_local, 128]
 * on every rank.  Slabs: ps_dcp_slab_alloc of
 * ps_decode_head_gather_slab_bytes(max_tokens, world * hq_local), mapped in
 * the peers with ps_dcp_ipc_handle / ps_dcp_ipc_open, one per rank, reused
 * by every call (not shared with ps_head_gather's slabs).  Every rank makes
 * the same calls in the same order; a rank's query rows must be < num_tokens
 * (else PS_DEV_BAD_METADATA and the row is not sent).  Two flag rounds per
 * call (rows written; rows copied, so that no rank's next call overwrites
 * rows a peer has not copied), bounded as in ps_dcp_decode:
 * PS_DEV_WAIT_TIMEOUT in *gather->status.  Plain decode only (no cascade
 * plan); 16-bit or fp8 caches.
 */
int64_t ps_decode_head_gather_slab_bytes(int32_t max_tokens, int32_t num_q_heads);
int ps_paged_decode_head_gather(const ps_paged_problem* problem, void* workspace, int64_t workspace_bytes,
                                const ps_head_gather_problem* gather, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PS_ATTN_H_ */
