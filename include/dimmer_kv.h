/* dimmer_kv.h — C ABI of the DimmerKV B200 library (libdimmerkv.so).
 *
 * Attention directly over a compressed KV cache (bit-plane / ladder PCA codes), for the
 * path of SrikanthBalaaji/Dimmer-KV named by scripts/compressed_attention.py and
 * scripts/progressive.py. Every entry point takes plain device pointers, sizes and a
 * cudaStream_t (passed as void*), enqueues work on that stream and returns a status
 * code (DKV_OK or one of the DKV_ERR_* values). Kernels report device-side failures
 * (a descriptor out of bounds, a wait that timed out) in the int pointed to by
 * `status`; the caller reads it after synchronising.
 *
 * The reference is Python and has no FFI of its own: each entry point below names the
 * reference function whose work it replaces. The Python host package (dimmerkv) binds
 * these symbols with ctypes (dimmerkv/_lib.py).
 *
 * Kernels read `status` as they start and do no work while it is non-zero, so after a
 * failure every later call that shares the word is inert until the caller clears it.
 * Every wait inside a kernel is bounded (about two seconds); a wait that runs out records
 * its code in `status` and the kernel leaves without touching the rest of its work.
 */
#ifndef DIMMER_KV_H_
#define DIMMER_KV_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DKV_OK 0
#define DKV_ERR_ARGS 1       /* invalid pointer, size or shape argument */
#define DKV_ERR_CONFIG 2     /* no kernel for this head_dim / GQA group / width */
#define DKV_ERR_CUDA 3       /* CUDA runtime call or launch failed */
#define DKV_ERR_TENSORMAP 4  /* cuTensorMapEncodeTiled rejected the basis layout */
#define DKV_ERR_SCRATCH 5    /* the call needs more scratch than dkv_attend_layer_static's fixed array */

/* Packed plane-stream descriptors. A stream is cut into tiles of up to 128 tokens; per (tile, union group)
 * one 16-byte-aligned block holds the f16 (low, scale) headers of the tokens with at least one plane, then
 * for every plane j one 64-bit word per token holding it (tokens sorted by plane count, so the holders of
 * plane j start at first[j]). dimmerkv/planes.py writes this layout. */
typedef struct dkv_tile {
  int32_t seq, token_base, n_tokens, n_groups, group_base, score_base, reserved0, reserved1;
} dkv_tile;

typedef struct dkv_group {
  uint32_t group, code_offset, code_bytes;
  uint8_t kind, max_planes, pad0, pad1;
  uint8_t first[16];
} dkv_group;

/* Arguments of one attention layer over a batch of compressed conversations. */
typedef struct dkv_attend_args {
  /* key stream (tokens in score order) */
  const uint8_t* k_code;
  uint64_t k_code_size;
  const dkv_tile* k_tiles;
  const dkv_group* k_groups;
  const int32_t* k_pos;          /* RoPE position per key token; < 0 hides the token */
  const int32_t* k_items;        /* work items: tile * (n_cols / k_block_cols) + column block */
  int32_t n_k_items;
  int32_t k_block_cols;          /* key columns per work item: 128, 256 or 512 */
  const void* k_basis;           /* bf16 [n_layers * n_cols][k_width]: per layer, per key column, its components */
  int32_t k_width;               /* union components of the key basis, multiple of 64 */
  const void* k_mean;            /* bf16 [.][n_layers][n_cols] */
  int64_t k_mean_seq_stride;     /* elements between conversations' means; 0 = one shared mean */
  /* value stream (tokens in value-rung order) */
  const uint8_t* v_code;
  uint64_t v_code_size;
  const dkv_tile* v_tiles;
  const dkv_group* v_groups;
  const int32_t* v_sidx;         /* value token -> index in its conversation's score order */
  const int32_t* v_items;        /* [n_v_items][4]: seq, first tile, end tile, first union group */
  int32_t n_v_items;
  int32_t v_item_groups;         /* union groups per value item; (v_item_groups / 2) * rows_pad <= 512 */
  const int32_t* v_seq_items;    /* [n_seq][2]: value item range of each conversation */
  const void* v_basis;           /* bf16 [n_layers][v_width][n_cols] */
  int32_t v_width;
  const void* v_mean;            /* bf16 [.][n_layers][n_cols] */
  int64_t v_mean_seq_stride;
  /* RoPE tables of the model (cos, sin per position, first half of head_dim), bf16 */
  const void* cos_t;
  const void* sin_t;
  int32_t max_pos;
  /* batch */
  int32_t n_seq;
  const int64_t* seq_score_off;  /* [n_seq] offset of each conversation's scores */
  const int32_t* seq_m;          /* [n_seq] key tokens in score order */
  /* model geometry */
  int32_t n_layers, layer, n_kv_heads, n_q_heads, head_dim, q_len;
  float scaling;
  /* per-call tensors (bf16) */
  const void* query;             /* [n_seq][n_q_heads][q_len][head_dim], RoPE applied */
  const void* exact_k;           /* [n_seq][n_kv_heads][n_exact][head_dim] sinks, recent, new tokens */
  const void* exact_v;
  int32_t n_exact;
  const float* mask;             /* [n_seq][q_len][n_exact] additive, or NULL */
  /* workspace (device, caller-allocated) */
  float* scores;                 /* sum_s n_q_heads * q_len * seq_m[s] */
  float* row_stats;              /* n_seq * n_q_heads * q_len * 4 */
  float* p_exact;                /* n_seq * n_q_heads * q_len * n_exact */
  float* partial;                /* n_v_items * rows_pad * v_item_groups * 64 */
  int32_t rows_pad;              /* value MMA width: multiple of 16, <= 128 */
  int32_t grid_k, grid_v;        /* CTAs of the key / value kernels (0 = one per SM) */
  /* output */
  void* out;                     /* [n_seq][q_len][n_q_heads][head_dim], bf16 or fp32 */
  int32_t out_f32;               /* 1: fp32 output (parity checks), 0: bf16 (the cache dtype) */
  int* status;                   /* device int32 */
  int32_t k_max_planes;          /* largest plane count of any key block (16 = raw blocks present) */
  int32_t v_max_planes;          /* the same for the value stream */
  const int32_t* v_item_ranges;  /* [n_v_items][v_tile_chunk][2]: per tile, the descriptor range inside the item's groups */
  int32_t v_tile_chunk;          /* value tiles per item (at most) */
  /* value-basis stage scratch: dkv_vpart_floats(v_width, n_seq, rows_pad, head_dim) floats */
  float* vpart;
  /* Optional static schedules (NULL: items are dealt round-robin over the grid). CTA b of the key
   * (value) kernel processes items k_item_order[k_cta_begin[b] .. k_cta_begin[b+1]) (item order NULL:
   * items k_cta_begin[b] .. k_cta_begin[b+1]); grid_k (grid_v) must then equal the number of lists. */
  const int32_t* k_cta_begin;    /* [grid_k + 1] */
  const int32_t* k_item_order;   /* [n_k_items] */
  const int32_t* v_cta_begin;    /* [grid_v + 1] */
  const int32_t* v_item_order;   /* [n_v_items] */
  /* Key kernel on CTA pairs (two SMs of a TPC per item, half the basis traffic per SM): [n_pairs][4] =
   * key tile of the even CTA, key tile of the odd CTA (-1: none), number of distinct groups of the two
   * tiles, first entry in k_pair_groups. k_items = pair * (n_cols / 512) + column block,
   * k_block_cols = 512, and a schedule (if any) with one list per pair of CTAs (grid_k = number of
   * lists). NULL: one CTA per item. */
  const int32_t* k_pairs;
  /* [entries][4]: per pair, the sorted union of its tiles' groups as (union group, k_groups index of
   * the even CTA's block or -1, of the odd CTA's block or -1, 0). */
  const int32_t* k_pair_groups;
  /* dkv_softmax_stats mode: 0 one softmax over this call's tokens; for one conversation split over GPUs
   * (split-K), 1 writes row_stats[0..1] = this shard's (max, sum of exponentials), and 2 takes
   * row_stats[0..1] = the merged (max, 1 / sum) and fills the compressed mass and p_exact.
   * dkv_attend_layer requires 0. */
  int32_t softmax_mode;
  /* Optional scratch for the value stage: [n_v_tiles][rows_pad * 256] bytes, 16-byte aligned. Given,
   * each value tile's bf16 probabilities are built once per call (and row chunk) and fetched by the
   * weighting kernel for every group range of the tile; NULL builds them inside the weighting kernel. */
  uint8_t* p_img;
  int32_t n_v_tiles;
  /* Optional: the value coefficients decoded once per decode step by dkv_unpack (bf16, out_tile_rows = 128:
   * [n_v_tiles * 128][v_width], tile t's tokens at rows t * 128 .., the other rows zero), 16-byte aligned.
   * Given with p_img, the value stage streams them with TMA instead of decoding the planes again in every
   * layer (the coefficients are the same for every layer); NULL decodes the planes in the value kernel. */
  const void* v_dense;
  /* The cache dtype of every 16-bit operand (query, exact keys / values, bases, means, RoPE tables, v_dense,
   * the raw 16-bit planes of the streams) and of a 16-bit output: 0 bf16, 1 fp16 (the reference's default
   * CompressedContext dtype). Probabilities are rounded to it where the reference rounds them. fp16 needs the
   * CTA-pair key kernel (k_pairs). */
  int32_t fp16;
  /* Optional: the key coefficients decoded once per decode step by dkv_unpack of the key stream (16-bit in
   * the cache dtype, out_tile_rows = 128: [n_k_tiles * 128][k_width], key tile t's tokens at rows t * 128 ..,
   * zeros for groups a tile does not hold), 16-byte aligned. Given with k_pairs, the key stage streams them
   * with TMA instead of decoding the planes again in every layer (the coefficients are the same for every
   * layer); NULL decodes the planes in the key kernel. */
  const void* k_dense;
  int32_t n_k_tiles;
} dkv_attend_args;

/* Floats of dkv_attend_args.vpart for a value basis of v_width components. */
int64_t dkv_vpart_floats(int32_t v_width, int32_t n_seq, int32_t rows_pad, int32_t head_dim);

/* One attention layer, all four stages below in order.
 * Replaces CompressedContext.attend (scripts/compressed_attention.py:113-137), batched over
 * conversations: compressed_attention.py:118-137 for every conversation of the batch. */
int dkv_attend_layer(const dkv_attend_args* args, void* stream);

/* Stage 1: key rebuild (tcgen05) + RoPE + q.k -> fp32 scores.
 * Replaces CompressedContext._keys (compressed_attention.py:105-111) and the compressed
 * score einsum of attend (compressed_attention.py:118-120). */
int dkv_key_scores(const dkv_attend_args* args, void* stream);

/* Stage 2: exact-token scores and the softmax statistics over compressed + exact tokens.
 * Replaces compressed_attention.py:122-128. */
int dkv_softmax_stats(const dkv_attend_args* args, void* stream);

/* Stage 3: probabilities (bf16, as the reference rounds them) times value coefficients (tcgen05).
 * Replaces the per-block einsum of compressed_attention.py:132-133. */
int dkv_value_weights(const dkv_attend_args* args, void* stream);

/* Stages 3 and 4 for every chunk of rows_pad rows (the part of dkv_attend_layer after the softmax
 * statistics; split-K callers run it after merging the shards' statistics). */
int dkv_attend_tail(const dkv_attend_args* args, void* stream);

/* Stage 4: value basis per head + mean + exact-token values -> output.
 * Replaces compressed_attention.py:130-131, 134-137. */
int dkv_finalize(const dkv_attend_args* args, void* stream);

/* dkv_attend_layer for callers that cannot allocate device memory. No counterpart in the reference.
 * Callers inside another framework's memory manager (which owns every device allocation and forbids
 * cudaMalloc / cudaFree) or in latency-critical loops pass the same arguments as to
 * dkv_attend_layer except the scratch pointers (scores, row_stats, p_exact, partial, vpart, p_img), which are
 * ignored; the scratch comes from a fixed 32 MiB array declared by the library in device memory.
 * n_scores = sum over conversations of n_q_heads * q_len * seq_m[s] (the score offsets seq_score_off the
 * caller passes must lie inside it): the library cannot read seq_m without a device-to-host copy, and an
 * n_scores below that sum lets the key kernel write past the scores region into the other scratch
 * regions and, near the limit, past the array. The Python binding computes it from its own host copy
 * (CompressedBatch.attend_layer_static). Returns DKV_ERR_SCRATCH, having launched nothing, when the
 * scratch would not fit. The first call on a device (and the first after a device reset) looks up the
 * array's address and must come before any stream capture. Calls share the array: calls that overlap on
 * the GPU race. Allocates nothing. */
int dkv_attend_layer_static(const dkv_attend_args* args, int64_t n_scores, void* stream);

/* Ragged bit-plane unpack of a packed stream to dense coefficients (stream order).
 * Replaces progressive.dequantize (scripts/progressive.py:47-55) and the ladder decode of
 * kvtc.quantize_groups (scripts/kvtc.py:78). Every element of the out rows is written: a token's
 * groups at its own plane count, zeros for union groups its tile holds no block of. `out` must be
 * 16-byte aligned. */
typedef struct dkv_unpack_args {
  const uint8_t* code;
  uint64_t code_size;
  const dkv_tile* tiles;
  int32_t n_tiles;
  const dkv_group* groups;
  void* out;                     /* [tokens][out_cols] */
  int64_t out_cols;
  int32_t out_bf16;              /* 1: bf16 (the reference's .to(dtype)), 0: fp32 */
  int* status;
  int32_t max_planes;            /* largest plane count of any block (16: raw bf16 blocks); 0: unknown */
  int32_t out_tile_rows;         /* 0: token rows in stream order; 128: tile t's tokens at rows t * 128 ..
                                  * (rows past a tile's tokens are not written) */
  int32_t f16;                   /* 1: a 16-bit output is fp16 (not bf16), and raw blocks hold fp16 patterns */
} dkv_unpack_args;
int dkv_unpack(const dkv_unpack_args* args, void* stream);

/* Question-time importance: adds, for every context token, the attention probability it receives from
 * every query head and question row of one layer (call once per layer after the softmax statistics).
 * Replaces the scoring branch of dimmer_attention (scripts/dimmer.py:62-75) summed by
 * question_importance (scripts/progressive.py:239-254). */
typedef struct dkv_importance_args {
  const float* scores;           /* the layer's score buffer (dkv_attend_args.scores) */
  const int64_t* seq_score_off;
  const int32_t* seq_m;
  const int32_t* seq_k_base;     /* [n_seq] first importance slot of each conversation */
  const float* row_stats;
  const float* p_exact;
  int32_t n_seq, n_q_heads, q_len, n_exact, max_m;
  float* imp_compressed;         /* [sum of seq_m] accumulated, one slot per score (score order) */
  float* imp_exact;              /* [n_seq][n_exact] accumulated */
} dkv_importance_args;
int dkv_importance(const dkv_importance_args* args, void* stream);

/* Top-k token selection per conversation, ties by lowest position; positions out in ascending order.
 * Replaces importance[start:end].topk(count) (scripts/methods.py:246-247). */
typedef struct dkv_topk_args {
  const float* importance;       /* [sum of seq_m] slots, score order */
  const int32_t* positions;      /* position of every slot, < 0 = not selectable */
  const int32_t* seq_k_base;
  const int32_t* seq_m;
  const int32_t* counts;         /* [n_seq] */
  const int32_t* out_offset;     /* [n_seq] */
  int32_t n_seq, max_k;
  int32_t* out;
  int* status;
} dkv_topk_args;
int dkv_topk(const dkv_topk_args* args, void* stream);

/* Merge of refined tokens: the hot planes of every selected token (from its packed hot block) and its
 * cold planes (staged from pinned host memory) written as new 8-plane blocks.
 * Replaces the full-precision re-decode of ProgressiveCache.refine (scripts/progressive.py:224-236). */
typedef struct dkv_refine_args {
  const uint8_t* hot_code;
  const dkv_tile* hot_tiles;
  const dkv_group* hot_groups;
  const int32_t* hot_tile;       /* [n_selected] */
  const int32_t* hot_row;        /* [n_selected] */
  const uint64_t* cold_words;    /* [n_selected][n_groups][8] */
  const uint32_t* cold_headers;  /* [n_selected][n_groups] */
  int32_t n_selected, n_groups;
  const dkv_group* out_groups;   /* [ceil(n_selected / 128)][n_groups] */
  uint8_t* out_code;
  int* status;
} dkv_refine_args;
int dkv_refine_merge(const dkv_refine_args* args, void* stream);

/* Encode side of the progressive codec, on the GPU: quantize8 of every (token, group of 64) and the
 * squared error of each token at each rung of the progressive order. Replaces quantize8
 * (scripts/progressive.py:37-44) and the error table of ProgressiveCodec.encode
 * (scripts/progressive.py:152-163): the reference's [tokens, groups, 9] table of errors at 0..8 planes,
 * gathered at the rungs' plane counts and summed over groups, is produced without the table.
 * codes / low / span are bit-exact with quantize8 on the same float32 coefficients; rung_error and
 * energy are float32 sums (fixed order) of the same squared differences. The caller divides rung_error
 * by the mean energy and runs the (host) allocator, as the reference does. */
typedef struct dkv_encode_args {
  const float* coeff;            /* [tokens][coeff_stride] float32, 16-byte aligned rows */
  int64_t coeff_stride;          /* elements between rows, multiple of 4 */
  int32_t tokens;
  int32_t features;              /* multiple of 64; groups = features / 64 */
  const uint8_t* rung_planes;    /* [n_rungs][groups]: planes (0..8) of each group at each rung */
  int32_t n_rungs;               /* 1..32 */
  uint8_t* codes;                /* [tokens][features]: the 8-bit codes (4-byte aligned) */
  uint16_t* low;                 /* [tokens][groups]: f16 bits of the group minimum */
  uint16_t* span;                /* [tokens][groups]: f16 bits of max(max - low, 1e-8) */
  float* rung_error;             /* [tokens][n_rungs]: sum over groups of the squared error at the rung */
  float* energy;                 /* [tokens]: sum of squared coefficients (NULL: not written) */
  int* status;
} dkv_encode_args;
int dkv_encode_groups(const dkv_encode_args* args, void* stream);

/* Restore side of the kvtc byte format (scripts/kvtc_storage.py:42-135): the bit-packed ladder codes of
 * every (rung, bit width) segment of a stream, decoded to float32 coefficients code * scale + low (a
 * multiply, then an add, as the reference's float32 torch ops; kvtc_storage.py:103-114) in the rows of
 * the segment's tokens and the 64 columns of each of its groups. Replaces that loop of decode_bytes; the
 * host reads the format's layout (the rung of every token is stored in the clear) and fills one
 * dkv_storage_segment per (rung, width). Rows and groups no segment covers are left as they are (the
 * reference starts from zeros). `data` may hold its arrays at any byte offset; `out` 16-byte aligned. */
typedef struct dkv_storage_segment {
  uint64_t codes_offset;         /* packed codes: 8 / width per byte, the first in the low bits */
  uint64_t low_offset;           /* f16 [count][n_groups] */
  uint64_t scale_offset;         /* f16 [count][n_groups] */
  int32_t count;                 /* tokens of the rung */
  int32_t n_groups;              /* groups stored at this width */
  int32_t width;                 /* 2, 4 or 8 */
  int32_t rows_offset;           /* first of the segment's count token rows in `rows` */
  int32_t groups_offset;         /* first of its n_groups group indices in `groups` */
  int32_t pad;
} dkv_storage_segment;

typedef struct dkv_storage_args {
  const uint8_t* data;           /* the stored bytes (device) */
  uint64_t data_size;
  const dkv_storage_segment* segments;
  int32_t n_segments;
  int64_t max_units;             /* largest count * n_groups * 4 (units of 16 components) over the segments */
  const int32_t* rows;
  const int32_t* groups;
  int64_t n_rows_idx;            /* entries of `rows` */
  int64_t n_groups_idx;          /* entries of `groups` */
  float* out;                    /* [out_rows][out_cols] */
  int64_t out_rows, out_cols;
  int* status;
} dkv_storage_args;
int dkv_storage_unpack(const dkv_storage_args* args, void* stream);

/* Tier management: demote the hot tier by dropping the least significant planes of whole tiles (the
 * "real cold tier" of the progressive codec: the dropped planes remain in the cold tier, which holds every
 * plane; scripts/progressive.py:11-19, 47-55 define the plane order). Each new block is copied from its
 * old block: the headers of the tokens keeping a plane, then per plane j the words of its new holders
 * (first'[j] = first[j + d] for tiles losing d planes). The caller lays the new blocks out (new_groups:
 * offsets, sizes, first tables; see dimmerkv.context.CompressedBatch.demote) and zero-fills new_code.
 * Progressive blocks only (raw and ladder blocks are rejected in the status word). Both code buffers and
 * both descriptor arrays must be 16-byte aligned, old_index and n_tokens 4-byte aligned (DKV_ERR_ARGS
 * otherwise). */
typedef struct dkv_demote_args {
  const uint8_t* old_code;
  uint64_t old_code_size;
  const dkv_group* old_groups;
  int64_t n_old_groups;
  uint8_t* new_code;
  uint64_t new_code_size;
  const dkv_group* new_groups;   /* [n_new] */
  const int32_t* old_index;      /* [n_new]: source block of each new block */
  const int32_t* n_tokens;       /* [n_new]: tokens of the block's tile */
  int64_t n_new;
  int* status;
} dkv_demote_args;
int dkv_demote(const dkv_demote_args* args, void* stream);

/* The per-token rung allocator of DimmerKV, on the GPU. Replaces kvtc.allocate_rungs (scripts/kvtc.py:
 * 277-298): upgrades valued by error drop per extra byte (made non-increasing along each slot's levels),
 * taken greedily in descending value (ties by flat index) while they fit the budget; counts[slot] = the
 * upgrades taken. Bit-exact with the sort-based reference (integer byte sums; a radix select on the
 * values' order instead of a sort). The caller checks that the coarsest levels fit (the reference's
 * ValueError) and passes what is left of the budget. */
typedef struct dkv_alloc_args {
  const float* errors;           /* [slots][levels] float32, the key stream's middle slots first */
  const int64_t* level_bytes;    /* [2][levels]: each level's bytes, key stream then value stream */
  int64_t slots;
  int64_t middle;                /* key slots */
  int32_t levels;                /* 2..64 */
  int64_t remaining;             /* budget - sum over slots of the coarsest level's bytes, >= 0 */
  int64_t* counts;               /* [slots] out */
  void* workspace;               /* dkv_alloc_workspace_bytes(slots, levels) bytes, 256-byte aligned */
  int64_t workspace_bytes;
  int* status;
} dkv_alloc_args;
int64_t dkv_alloc_workspace_bytes(int64_t slots, int32_t levels);
int dkv_allocate_rungs(const dkv_alloc_args* args, void* stream);

/* Library version (major * 10000 + minor * 100 + patch). */
int dkv_version(void);

/* Text of a DKV_* status code. */
const char* dkv_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* DIMMER_KV_H_ */
