// Internal launch interfaces between the C-ABI layer (ps_attn_api.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ps {

struct AppendArgs {
  const char* key;
  const char* value;
  char* key_cache;
  char* value_cache;
  const int64_t* slot_mapping;
  int64_t key_st, key_sh, val_st, val_sh;  // bytes
  int64_t c_sblock, c_sslot, c_shead;      // bytes
  int64_t num_slots;                       // num_blocks * block_size
  int64_t num_tokens;
  int32_t num_heads;
  int32_t block_size;
  int32_t vecs_per_head;  // head_size * elem_bytes / VEC
  int32_t* status;
};

// Paged decode launch parameters (device-visible copy of ps_paged_problem plus
// derived values).  Strides are in elements.
struct DecodeParams {
  const void* q;
  int64_t q_st, q_sh;
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t max_blocks_per_seq;
  const int32_t* seq_lens;
  const int32_t* qsl;
  int32_t num_seqs;
  void* out;
  int64_t o_st, o_sh;
  float* lse;
  int64_t lse_sh, lse_st;
  int32_t num_q_heads, num_kv_heads, group;  // group = q heads per kv head
  int32_t block_size;                        // tokens per cache block (multiple of 16)
  int64_t num_blocks;
  float scale_log2;                          // softmax_scale * log2(e)
  // workspace
  int32_t* status;
  int32_t* counters;     // [num_seqs * num_kv_heads]
  float* part;           // [slots] records: [kg][128] output rows then [kg] LSEs
  int64_t num_part_slots;
  // fused KV append (new_key == nullptr: off); element strides
  const void* new_key;
  const void* new_value;
  int64_t nk_st, nk_sh, nv_st, nv_sh;
  const int64_t* slot_mapping;
  void* key_cache;
  void* value_cache;
  int64_t c_sblock, c_sslot, c_shead;
  // shared-prefix (cascade) plan (cas_num_groups == nullptr: off)
  const int32_t* cas_num_groups;   // [1]
  const int32_t* cas_seq_group;    // [num_seqs] group of each sequence, -1 none
  const int32_t* cas_group_first;  // [cas_max_groups]
  const int32_t* cas_group_size;   // [cas_max_groups]
  const int32_t* cas_group_pages;  // [cas_max_groups] shared 16-token pages
  int32_t cas_max_groups;
  int32_t* pre_counters;           // [num_seqs * num_kv_heads] prefix-segment split counters
  // per-tensor cache scales (device; nullptr = 1): attention reads K * k_scale,
  // V * v_scale (an fp8 cache's dequantization)
  const float* k_scale;
  const float* v_scale;
  // fused head all-gather of a KV-head-sharded group (gather_world == 0: off).
  // `out` is then this rank's first head of the group's [T, Hq, 128] output;
  // every finished row is also stored into each peer's slab rows region
  // (gather_rows[r]: peer r's region offset to this rank's first head,
  // nullptr for this rank; token t at + t * gather_row_st bytes, local head j
  // at + j * 256).  The kernel's tail waits for every peer's rows and copies
  // them from this rank's slab into gather_out.
  int32_t gather_world, gather_rank, gather_hq_local, gather_tokens;
  char* gather_slab[8];   // every rank's slab (barrier header at byte 0)
  char* gather_rows[8];
  int64_t gather_row_st;  // bytes per token row of a slab's rows region
  char* gather_out;       // [T, world * hq_local, 128] (this rank's `out` is inside it)
  int64_t gather_o_st, gather_o_sh;  // bytes
  int32_t* gather_status;
};

// Static sizing of the decode kernel, shared by the workspace-size query.
// The defaults are the tuned values; the macros exist for tuning sweeps.
#ifndef PS_DECODE_WARPS
#define PS_DECODE_WARPS 8
#endif
#ifndef PS_DECODE_STAGES
#define PS_DECODE_STAGES 2
#endif
#ifndef PS_DECODE_CTAS_PER_SM
#define PS_DECODE_CTAS_PER_SM 1
#endif
#ifndef PS_DECODE_FP8_WARPS
#define PS_DECODE_FP8_WARPS 8
#endif
#ifndef PS_DECODE_FP8_STAGES
#define PS_DECODE_FP8_STAGES 2
#endif
constexpr int kDecodeWarps = PS_DECODE_WARPS;           // warps per CTA
// fp8 caches: a unit is two pages (the same 8 KB per stage as a 16-bit page),
// so the same warps and stages as the 16-bit kernel
constexpr int kDecodeFp8Warps = PS_DECODE_FP8_WARPS;
constexpr int kDecodeFp8Stages = PS_DECODE_FP8_STAGES;
constexpr int kDecodeMaxWarps = kDecodeWarps > kDecodeFp8Warps ? kDecodeWarps : kDecodeFp8Warps;
constexpr int kDecodeStages = PS_DECODE_STAGES;         // pages in flight per warp
constexpr int kDecodeCtasPerSm = PS_DECODE_CTAS_PER_SM; // persistent CTAs per SM
constexpr int kDecodeMaxSeqs = 4096;                    // sequences per launch (prefix table in smem)
constexpr int kCascadeMaxSeqs = 2048;                   // per cascade launch (plan tables in smem)

}  // namespace ps

namespace ps {
// Chunked-prefill launch parameters.  Strides in elements.
struct PrefillParams {
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t max_blocks_per_seq;
  const int32_t* seq_lens;
  const int32_t* qsl;
  int32_t num_seqs;
  void* out;
  int64_t o_st, o_sh;
  float* lse;
  int64_t lse_sh, lse_st;
  int32_t num_q_heads, num_kv_heads, group;
  int32_t tokens_per_tile;  // floor(128 / group): tokens of one M tile
  int32_t block_size;
  int64_t num_blocks;
  float scale_log2;
  // per-tensor cache scales (device; nullptr = 1): attention reads K * k_scale, V * v_scale
  const float* k_scale;
  const float* v_scale;
  int32_t* status;
  // dynamic unit scheduling: [0] units claimed past the grid, [1] CTAs done
  // (both zero between launches); nullptr: static round-robin
  int32_t* sched;
};
constexpr int kPrefillMaxSeqs = 4096;
}  // namespace ps

// Sets the calling thread's ps_last_error() message; returns `code`.
int ps_set_last_error(int code, const char* msg);

int ps_launch_kv_append(const ps::AppendArgs& a, int vec, int sm_count, cudaStream_t stream);

// Returns a cudaError_t value.
// fp8_cache: K/V caches of e4m3 codes (plain decode only)
int ps_launch_paged_decode(const ps::DecodeParams& p, const CUtensorMap& kmap,
                           const CUtensorMap& vmap, int dtype_bf16, int sm_count,
                           cudaStream_t stream, int fp8_cache = 0);
int ps_launch_kv_append_fp8(const ps::AppendArgs& a, const float* k_scale, const float* v_scale,
                            int dtype_bf16, int sm_count, cudaStream_t stream);

// Split-record slots a decode launch may use: its warps plus one per unit.
int64_t ps_decode_partial_slots(int num_seqs, int num_kv_heads, int sm_count, int cascade, int fp8 = 0);
// Workspace bytes of the decode kernel a problem of this kind launches
// (ps_paged_decode_workspace_size returns the largest over the kinds).
int64_t ps_decode_workspace_bytes(int num_seqs, int num_q_heads, int num_kv_heads, int sm_count,
                                  int cascade, int fp8);

// Shared-prefix plan (cascade_plan.cu).  Plan buffer layout in int32 words,
// Gm = max(1, num_seqs / 2):
//   [0] num_groups  [1] CTA arrival counter  [2, 32) reserved
//   [32, 32 + B) seq_group  then group_first[Gm], group_size[Gm],
//   group_pages[Gm], shared_pages[B] (pages each sequence shares with its
//   predecessor)
namespace ps {
struct PlanArgs {
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t max_blocks_per_seq;
  const int32_t* seq_lens;
  const int32_t* qsl;
  int32_t num_seqs;
  int32_t block_size;
  int32_t min_shared_pages;
  int32_t enabled;  // 0: write an empty plan
  int32_t* plan;
};
}  // namespace ps
namespace ps {
// Fused rotary embedding + KV append.  Strides in bytes.
struct RopeArgs {
  char* q;
  int64_t q_st, q_sh;
  char* k;
  int64_t k_st, k_sh;
  const char* v;
  int64_t v_st, v_sh;
  char* key_cache;
  char* value_cache;
  int64_t c_sblock, c_sslot, c_shead;
  int64_t num_slots;  // num_blocks * block_size
  int32_t block_size;
  const int64_t* slot_mapping;
  const int64_t* positions;
  const char* cos_sin;  // [max_position, rotary_dim]: cos then sin halves
  int64_t cs_stride_bytes;
  int64_t max_position;
  int32_t cs_fp32;  // cache in fp32 (else the model dtype)
  int32_t rotary_dim, neox;
  int64_t num_tokens;
  int32_t num_q_heads, num_kv_heads, head_size;
  int32_t bf16;
  int32_t* status;
};

// Decode context parallelism: one rank's view of its group and of one call.
// Byte strides unless noted.
constexpr int kDcpMaxWorld = 8;
static_assert(kDcpMaxWorld == 8, "DecodeParams' gather arrays hold kDcpMaxWorld ranks");
struct DcpArgs {
  int32_t world, rank, interleave;
  char* slab[kDcpMaxWorld];  // every rank's slab as addressed from this GPU
  int64_t off_q, off_part, off_lse, off_qall, off_lens;
  int32_t signal_first;      // gather/combine publish their phase at their start
  int32_t context_only;      // combine: corrected context attention only (no self term, no append)
  // this rank's query rows [T, hq_local, 128] and output
  const char* q;
  int64_t q_st, q_sh;
  char* out;
  int64_t o_st, o_sh;
  float* lse;                // nullable, element strides
  int64_t lse_sh, lse_st;
  // the new tokens' key/value rows [T, num_kv_heads, 128]
  const char* new_key;
  int64_t nk_st, nk_sh;
  const char* new_value;
  int64_t nv_st, nv_sh;
  const int64_t* slot_mapping;  // local slots, < 0: stored by another rank
  char* key_cache;
  char* value_cache;
  int64_t c_sblock, c_sslot, c_shead;
  int64_t num_slots;
  int32_t block_size;
  const int32_t* seq_lens;   // global lengths, the new token included
  int32_t num_tokens;        // = sequences (one query row each)
  int32_t hq_local, hq_all, num_kv_heads, group;
  float softmax_scale;
  int32_t bf16;
  int32_t* status;
};

// Dequantizing page gather (fp8 cache -> 16-bit scratch).  Byte strides.
struct DequantArgs {
  const char* key_cache;
  const char* value_cache;
  int64_t c_sblock;
  int64_t block_bytes;      // block_size * num_kv_heads * head_size
  int64_t num_blocks;
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t max_blocks_per_seq;
  const int32_t* seq_lens;
  int32_t num_seqs, max_pages, block_size;
  const float* k_scale;
  const float* v_scale;
  char* out_key;            // [num_seqs * max_pages, block_size, num_kv_heads, head_size]
  char* out_value;
  int32_t* status;
};

// Head all-gather over peer memory (KV-head-sharded decode).  Byte strides.
constexpr int64_t kHeadGatherRowsOffset = 256;  // this rank's rows in its slab
// The fused decode + head gather: the group's rows [T, Hq, 128] in every
// rank's slab at this offset; slab header word 34 counts the second round of
// CTA arrivals (word 33 the first).
constexpr int64_t kDecodeGatherRowsOffset = 256;
constexpr int kDecodeGatherDone2Word = 34;
struct HeadGatherArgs {
  int32_t world, rank;
  char* slab[kDcpMaxWorld];
  int32_t num_tokens, hq_local;
  char* out;              // [T, world * hq_local, 128]
  int64_t o_st, o_sh;
  int32_t* status;
  int32_t mode;           // set by the launcher
};
}  // namespace ps
int ps_launch_dcp(const ps::DcpArgs& a, int which, int sm_count, cudaStream_t stream);
int ps_launch_head_gather(const ps::HeadGatherArgs& a, int which, int sm_count, cudaStream_t stream);
int ps_launch_kv_dequant_gather(const ps::DequantArgs& a, int dtype_bf16, int sm_count,
                                cudaStream_t stream);
namespace ps {
struct MergeArgs {
  const char* p_out;
  int64_t p_st, p_sh;  // bytes
  const float* p_lse;
  const char* s_out;
  int64_t s_st, s_sh;
  const float* s_lse;
  char* out;
  int64_t o_st, o_sh;
  float* out_lse;
  int64_t num_tokens;
  int32_t num_heads;
};
}  // namespace ps
int ps_launch_merge_attn_states(const ps::MergeArgs& a, int dtype_bf16, int sm_count,
                                cudaStream_t stream);

// vec: the 16-byte path (rows, strides and cos/sin rows 16-byte aligned,
// head_size % 8 == 0, rotary_dim % 16 == 0)
int ps_launch_rope_kv_append(const ps::RopeArgs& a, int sm_count, int vec, cudaStream_t stream);

int64_t ps_cascade_plan_words(int num_seqs);
int ps_launch_cascade_plan(const ps::PlanArgs& a, cudaStream_t stream);

int ps_launch_chunked_prefill(const ps::PrefillParams& p, const CUtensorMap& qmap,
                              const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype_bf16,
                              int grid, cudaStream_t stream);
