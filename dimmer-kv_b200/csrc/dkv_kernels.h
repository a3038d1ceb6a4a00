// dkv_kernels.h — parameter blocks and launchers of the DimmerKV sm_100a kernels (internal).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace dkv {

// Return codes shared with the C ABI (include/dimmer_kv.h).
enum : int {
  kDkvOk = 0,
  kDkvErrArgs = 1,     // a pointer, size or shape argument is invalid
  kDkvErrConfig = 2,   // a shape this build has no kernel for (head_dim, GQA group, ...)
  kDkvErrCuda = 3,     // a CUDA runtime call or launch failed
  kDkvErrTensorMap = 4 // cuTensorMapEncodeTiled rejected the basis layout
};

struct TileDesc;
struct GroupDesc;

// Fused key rebuild + RoPE + query-key products (key_scores.cu).
struct KeyScoreParams {
  const uint8_t* code;            // key plane blocks
  uint64_t code_size;
  const TileDesc* tiles;
  const GroupDesc* groups;
  const int32_t* tok_pos;         // absolute RoPE position per key token; < 0 hides the token
  const int32_t* items;           // work items: tile * (n_cols / NB) + column block
  int n_items;
  uint32_t n_union_groups;        // groups covered by the basis tensor map
  const __nv_bfloat16* query;     // [n_seq][n_q_heads][q_len][head_dim]
  const __nv_bfloat16* mean;      // [.][n_layers][n_cols], conversation stride mean_seq_stride (0 = shared)
  int64_t mean_seq_stride;
  const __nv_bfloat16* cos_t;     // [max_pos][head_dim / 2]
  const __nv_bfloat16* sin_t;
  int max_pos;
  const int64_t* seq_score_off;   // [n_seq] first score of each conversation
  const int32_t* seq_m;           // [n_seq] score-order length (row stride of the scores)
  float* scores;                  // [sum over seq][n_q_heads][q_len][M_s]
  int layer, n_cols, n_q_heads, q_per_kv, q_len, head_dim;
  float scaling;
  int max_planes;                 // largest plane count of any key block (> 8: raw blocks present)
  int* status;
  const int32_t* cta_begin;       // optional static schedule (see ValueWeightParams)
  const int32_t* item_order;
  int f16;                        // 16-bit operands (query, mean, cos / sin, basis, codes' raw values) are fp16, not bf16
  const int32_t* pairs;           // CTA-pair kernel: [n_pairs][4] = tile 0, tile 1 (-1: none), merged groups,
                                  // first pair_groups entry; items = pair * (n_cols / 512) + column block
  const int32_t* pair_groups;     // [entries][4] = union group, descriptor of tile 0, of tile 1 (-1: none), 0
  int n_tiles;                    // key tiles (rows of the decoded key buffer / 128, for the dense kernel)
};
int run_key_scores(const CUtensorMap& bmap, const KeyScoreParams& p, int nb, int grid, cudaStream_t stream);
int run_key_scores_pair(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream);
// The CTA-pair key kernel over key coefficients decoded once per step (key_scores_dense.cu).
int run_key_scores_dense(const CUtensorMap& bmap, const CUtensorMap& amap, const KeyScoreParams& p, int grid,
                         cudaStream_t stream);

// Softmax statistics over compressed + exact tokens (softmax.cu).
struct SoftmaxParams {
  const float* scores;
  const int64_t* seq_score_off;
  const int32_t* seq_m;
  const __nv_bfloat16* query;     // [n_seq][n_q_heads][q_len][head_dim]
  const __nv_bfloat16* exact_k;   // [n_seq][n_kv_heads][n_exact][head_dim]
  const float* mask;              // [n_seq][q_len][n_exact] additive, or null
  int n_seq, n_q_heads, q_per_kv, q_len, head_dim, n_exact;
  float scaling;
  float* row_stats;               // [n_seq][n_q_heads][q_len][4]: max, 1/sum, compressed mass, 0
  float* p_exact;                 // [n_seq][n_q_heads][q_len][n_exact], fp32 (unrounded)
  int mode;                       // kSoftmaxFull, kSoftmaxLocal or kSoftmaxGlobal
  float* scratch;                 // optional: per-(row, slice) partials when few rows are long
  int64_t scratch_floats;
  int n_sms;                      // SMs of the device (sizes the slices)
  const int* status;              // the call's status word (read at entry: non-zero means no work)
  int f16;                        // query and exact keys are fp16 (else bf16); probabilities round to that dtype
};
constexpr int kSoftmaxFull = 0;
constexpr int kSoftmaxLocal = 1;   // row_stats <- (max, sum of exponentials) of this shard
constexpr int kSoftmaxGlobal = 2;  // row_stats[0..1] hold the merged (max, 1 / sum); fills mass, p_exact
int run_softmax_stats(const SoftmaxParams& p, cudaStream_t stream);

// Probability-weighted value coefficients (value_weights.cu).
struct ValueWeightParams {
  const uint8_t* code;
  uint64_t code_size;
  const TileDesc* tiles;
  const GroupDesc* groups;
  const int32_t* tok_sidx;        // value token -> index in its conversation's score order
  const int32_t* items;           // [n_items][4]: seq, tile_begin, tile_end, first union group
  const int32_t* item_ranges;     // [n_items][tile_chunk][2]: descriptor range of each tile inside the item's groups
  int tile_chunk;
  int n_items;
  int item_groups;                // union groups covered by one item (2 x pairs)
  int max_planes;                 // largest plane count of any value block (> 8: raw blocks present)
  const float* scores;
  const int64_t* seq_score_off;
  const int32_t* seq_m;
  const float* row_stats;
  int n_q_heads, q_len;
  int row_begin, n_rows, n_rows_pad;  // rows = q_head * q_len + qi; N of the MMA = n_rows_pad
  float* partial;                 // [n_items][n_rows_pad][item_groups * 64]
  int* status;
  const int32_t* cta_begin;       // optional static schedule: CTA b takes item_order[cta_begin[b] .. cta_begin[b+1])
  const int32_t* item_order;
  uint8_t* p_img;                 // optional [n_tiles][2][n_rows_pad][128 B]: P^T images (vprobs_kernel)
  int n_tiles;                    // value tiles (with p_img)
  int f16;                        // probabilities and coefficients in fp16 (else bf16)
};
int run_value_weights(const ValueWeightParams& p, int grid, cudaStream_t stream);
// P^T images of every value tile (vprobs_kernel), used by both value kernels.
int run_vprobs(const ValueWeightParams& p, cudaStream_t stream);
// The value stage over coefficients decoded once per step (value_dense.cu): vmap is a 2-D tensor map of
// the tile-padded bf16 buffer [n_tiles * 128][width], box 64 components x 128 rows, 128B swizzle.
int run_value_dense(const CUtensorMap& vmap, const ValueWeightParams& p, int grid, cudaStream_t stream);
int dense_value_stages(int n_rows_pad);

// Value basis, mean and exact tokens -> attention output (finalize.cu).
struct FinalizeParams {
  const float* partial;
  const int32_t* items;           // value items [n_items][4]
  const int32_t* seq_items;       // [n_seq][2] item range of each conversation
  int item_groups, n_rows_pad, row_begin, n_rows;
  const __nv_bfloat16* basis_v;   // [n_layers][r_v][n_cols]
  int r_v;                        // union components of the value basis
  const __nv_bfloat16* mean_v;    // [.][n_layers][n_cols]
  int64_t mean_seq_stride;
  const float* row_stats;
  const float* p_exact;
  const __nv_bfloat16* exact_v;   // [n_seq][n_kv_heads][n_exact][head_dim]
  int n_seq, n_q_heads, q_per_kv, q_len, head_dim, n_exact, layer, n_cols;
  void* out;                      // [n_seq][q_len][n_q_heads][head_dim]
  int out_f32;                    // fp32 output instead of bf16
  float* vpart;                   // finalize_vpart_floats(r_v, n_seq, n_rows_pad, head_dim) floats of scratch
  int* status;
  int f16;                        // 16-bit operands and output in fp16 (else bf16)
};
int64_t finalize_vpart_floats(int r_v, int n_seq, int rows_pad, int head_dim);
int run_finalize(const FinalizeParams& p, cudaStream_t stream);

// Encode side of the progressive codec: quantize8 + per-rung errors (encode.cu).
struct EncodeParams {
  const float* coeff;
  int64_t coeff_stride;
  int tokens, features;
  const uint8_t* rung_planes;   // [n_rungs][features / 64]
  int n_rungs;
  uint8_t* codes;               // [tokens][features]
  uint16_t* low;                // [tokens][features / 64] f16 bits
  uint16_t* span;
  float* rung_error;            // [tokens][n_rungs]
  float* energy;                // [tokens] or nullptr
  int* status;
};
int run_encode(const EncodeParams& p, cudaStream_t stream);

// Tier management: demotion by dropping planes (demote.cu).
struct DemoteParams {
  const uint8_t* old_code;
  uint64_t old_code_size;
  const GroupDesc* old_groups;
  int64_t n_old_groups;
  uint8_t* new_code;              // zero-filled by the caller (block padding stays zero)
  uint64_t new_code_size;
  const GroupDesc* new_groups;    // [n_new]: the new blocks' layout
  const int32_t* old_index;       // [n_new]: the old block each new block comes from
  const int32_t* n_tokens;        // [n_new]: tokens of the block's tile
  int64_t n_new;
  int* status;
};
int run_demote(const DemoteParams& p, cudaStream_t stream);

// Per-token rung allocator (allocate.cu).
struct AllocParams {
  const float* errors;            // [slots][levels], keys' slots first (middle of them), then values'
  const int64_t* level_bytes;     // [2][levels]: bytes of each level, key stream then value stream
  int64_t slots, middle;
  int levels;
  int64_t remaining;              // budget minus every slot's coarsest level
  int64_t* counts;                // [slots]: upgrades taken
  void* workspace;                // alloc_workspace_bytes(slots, levels) bytes, 256-byte aligned
  int64_t workspace_bytes;
  int* status;
};
int64_t alloc_workspace_bytes(int64_t slots, int levels);
int run_allocate(const AllocParams& p, cudaStream_t stream);

// Restore of the kvtc byte format (storage.cu).
struct StorageSegment {
  uint64_t codes_offset, low_offset, scale_offset;  // byte offsets into the stored bytes
  int32_t count, n_groups, width;                    // tokens, groups of this bit width, bits per code
  int32_t rows_offset, groups_offset, pad;           // into rows[] / groups[]
};
struct StorageParams {
  const uint8_t* data;
  uint64_t data_size;
  const StorageSegment* segments;
  int n_segments;
  int64_t max_units;              // largest count * n_groups * 4 (16-component units) of any segment
  const int32_t* rows;            // token row of each segment's tokens
  const int32_t* groups;          // group index of each segment's groups
  int64_t n_rows_idx, n_groups_idx;  // entries of rows[] and groups[]
  float* out;                     // [out_rows][out_cols], zero where no segment writes
  int64_t out_rows, out_cols;
  int* status;
};
int run_storage_unpack(const StorageParams& p, cudaStream_t stream);

// Standalone ragged bit-plane unpack (unpack.cu).
struct UnpackParams {
  const uint8_t* code;
  uint64_t code_size;
  const TileDesc* tiles;
  const GroupDesc* groups;
  int n_tiles;
  void* out;                      // [tokens][out_cols] fp32 or bf16, stream order (or tile-padded)
  int64_t out_cols;
  int out_bf16;
  int max_planes;                 // 0: unknown (slots sized for raw blocks)
  int* status;
  int out_tile_rows;              // 0: rows in stream order; 128: tile t's tokens at rows t * 128 ..
  int f16;                        // 16-bit output (and raw blocks) in fp16 instead of bf16
};
int run_unpack(const UnpackParams& p, cudaStream_t stream);

// Question-time scoring, selection and refinement (question.cu).
struct ImportanceParams {
  const float* scores;
  const int64_t* seq_score_off;
  const int32_t* seq_m;
  const int32_t* seq_k_base;      // first importance slot of each conversation
  const float* row_stats;
  const float* p_exact;
  int n_seq, n_q_heads, q_len, n_exact;
  float* imp_compressed;          // [sum of seq_m], one slot per score (score order), accumulated
  float* imp_exact;               // [n_seq][n_exact], accumulated
};
int run_importance(const ImportanceParams& p, int max_m, cudaStream_t stream);

struct TopkParams {
  const float* importance;        // [sum of seq_m] slots, score order
  const int32_t* positions;       // position of every slot, < 0 = not selectable
  const int32_t* seq_k_base;
  const int32_t* seq_m;
  const int32_t* counts;          // [n_seq] tokens to select
  const int32_t* out_offset;      // [n_seq]
  int n_seq;
  int32_t* out;                   // selected positions, ascending per conversation
  int* status;
};
int run_topk(const TopkParams& p, int max_k, cudaStream_t stream);

struct RefineParams {
  const uint8_t* hot_code;
  const TileDesc* hot_tiles;
  const GroupDesc* hot_groups;
  const int32_t* hot_tile;        // [n_selected] hot tile of each selected token
  const int32_t* hot_row;         // [n_selected] its row in that tile
  const uint64_t* cold_words;     // [n_selected][n_groups][8] plane words of the full codes
  const uint32_t* cold_headers;   // [n_selected][n_groups] f16 low | f16 mult << 16
  int n_selected, n_groups;
  const GroupDesc* out_groups;    // [ceil(n_selected / 128)][n_groups] refined block descriptors
  uint8_t* out_code;
  int* status;
};
int run_refine(const RefineParams& p, cudaStream_t stream);

}  // namespace dkv
