// capi.cu — extern "C" entry points of libdimmerkv.so (declared in include/dimmer_kv.h).
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dimmer_kv.h"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace {

using dkv::GroupDesc;
using dkv::TileDesc;

static_assert(sizeof(dkv_tile) == sizeof(TileDesc), "tile layout");
static_assert(sizeof(dkv_group) == sizeof(GroupDesc), "group layout");

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D tensor maps of 16-bit row-major matrices (bases, decoded coefficients), cached by (address, rows,
// width, box rows, dtype).
std::mutex g_map_mutex;
std::map<std::tuple<uintptr_t, uint64_t, uint64_t, uint32_t, int>, CUtensorMap> g_maps;

int basis_map(const void* basis, uint64_t rows, uint64_t width, uint32_t box_rows, CUtensorMap* out, int f16 = 0) {
  if (basis == nullptr || rows == 0 || width == 0 || width % 64 != 0) return DKV_ERR_ARGS;
  if (reinterpret_cast<uintptr_t>(basis) % 16 != 0) return DKV_ERR_ARGS;
  const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(basis), rows, width, box_rows, f16 ? 1 : 0);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return DKV_OK;
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return DKV_ERR_TENSORMAP;
  CUtensorMap map;
  cuuint64_t gdim[2] = {width, rows};
  cuuint64_t gstride[1] = {width * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(&map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(basis), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return DKV_ERR_TENSORMAP;
  if (g_maps.size() > 256) g_maps.clear();
  g_maps[key] = map;
  *out = map;
  return DKV_OK;
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

int check_common(const dkv_attend_args* a) {
  if (a == nullptr) return DKV_ERR_ARGS;
  if (a->n_seq < 0 || a->q_len < 1 || a->n_kv_heads < 1 || a->n_q_heads < 1 || a->n_q_heads % a->n_kv_heads != 0)
    return DKV_ERR_ARGS;
  if (a->layer < 0 || a->layer >= a->n_layers) return DKV_ERR_ARGS;
  if (a->head_dim != 64 && a->head_dim != 128) return DKV_ERR_CONFIG;
  return DKV_OK;
}

}  // namespace

extern "C" {

int dkv_version(void) { return 100; }

const char* dkv_status_string(int status) {
  switch (status) {
    case DKV_OK: return "ok";
    case DKV_ERR_ARGS: return "invalid argument";
    case DKV_ERR_CONFIG: return "unsupported configuration";
    case DKV_ERR_CUDA: return "CUDA error";
    case DKV_ERR_TENSORMAP: return "tensor map encoding failed";
    case DKV_ERR_SCRATCH: return "scratch larger than the static array of dkv_attend_layer_static";
    default: return "unknown status";
  }
}

int dkv_key_scores(const dkv_attend_args* a, void* stream) {
  int rc = check_common(a);
  if (rc != DKV_OK) return rc;
  if (a->n_k_items == 0) return DKV_OK;
  const int n_cols = a->n_kv_heads * a->head_dim;
  const int nb = a->k_block_cols;
  const bool pairs = a->k_pairs != nullptr;
  if ((nb != 128 && nb != 256 && nb != 512) || n_cols % nb != 0 || nb % a->head_dim != 0) return DKV_ERR_CONFIG;
  if (pairs && nb != 512) return DKV_ERR_CONFIG;  // CTA pairs: 512 columns per item, 128-row basis boxes
  if (a->fp16 && !pairs) return DKV_ERR_CONFIG;  // fp16 operands: the CTA-pair kernel only
  CUtensorMap map;
  rc = basis_map(a->k_basis, static_cast<uint64_t>(a->n_layers) * n_cols, static_cast<uint64_t>(a->k_width),
                 pairs ? 128u : (nb > 256 ? 256u : static_cast<uint32_t>(nb)), &map, a->fp16);
  if (rc != DKV_OK) return rc;
  dkv::KeyScoreParams p{};
  p.code = a->k_code;
  p.code_size = a->k_code_size;
  p.tiles = reinterpret_cast<const TileDesc*>(a->k_tiles);
  p.groups = reinterpret_cast<const GroupDesc*>(a->k_groups);
  p.tok_pos = a->k_pos;
  p.items = a->k_items;
  p.n_items = a->n_k_items;
  p.n_union_groups = static_cast<uint32_t>(a->k_width / 64);
  p.query = static_cast<const __nv_bfloat16*>(a->query);
  p.mean = static_cast<const __nv_bfloat16*>(a->k_mean);
  p.mean_seq_stride = a->k_mean_seq_stride;
  p.cos_t = static_cast<const __nv_bfloat16*>(a->cos_t);
  p.sin_t = static_cast<const __nv_bfloat16*>(a->sin_t);
  p.max_pos = a->max_pos;
  p.seq_score_off = a->seq_score_off;
  p.seq_m = a->seq_m;
  p.scores = a->scores;
  p.layer = a->layer;
  p.n_cols = n_cols;
  p.n_q_heads = a->n_q_heads;
  p.q_per_kv = a->n_q_heads / a->n_kv_heads;
  p.q_len = a->q_len;
  p.head_dim = a->head_dim;
  p.scaling = a->scaling;
  p.max_planes = a->k_max_planes;
  p.status = a->status;
  p.cta_begin = a->k_cta_begin;
  p.item_order = a->k_item_order;
  p.f16 = a->fp16 ? 1 : 0;
  if ((a->k_item_order != nullptr && a->k_cta_begin == nullptr) || (a->k_cta_begin != nullptr && a->grid_k <= 0))
    return DKV_ERR_ARGS;
  p.pairs = a->k_pairs;
  p.pair_groups = a->k_pair_groups;
  if (pairs && a->k_pair_groups == nullptr) return DKV_ERR_ARGS;
  if (pairs) {
    // Two CTAs per cluster; grid_k counts the schedule's lists (one per cluster).
    const int clusters = a->grid_k > 0 ? a->grid_k : sm_count() / 2;
    if (a->k_dense != nullptr) {
      // Key coefficients decoded once per step: both operands by TMA (64 x 128 boxes of the decoded buffer).
      if (a->n_k_tiles <= 0 || (reinterpret_cast<uintptr_t>(a->k_dense) & 15u) != 0) return DKV_ERR_ARGS;
      CUtensorMap amap;
      rc = basis_map(a->k_dense, static_cast<uint64_t>(a->n_k_tiles) * 128, static_cast<uint64_t>(a->k_width), 128u,
                     &amap, a->fp16);
      if (rc != DKV_OK) return rc;
      p.n_tiles = a->n_k_tiles;
      return dkv::run_key_scores_dense(map, amap, p, 2 * clusters, static_cast<cudaStream_t>(stream));
    }
    return dkv::run_key_scores_pair(map, p, 2 * clusters, static_cast<cudaStream_t>(stream));
  }
  const int grid = a->grid_k > 0 ? a->grid_k : (a->n_k_items < sm_count() ? a->n_k_items : sm_count());
  return dkv::run_key_scores(map, p, nb, grid, static_cast<cudaStream_t>(stream));
}

int dkv_softmax_stats(const dkv_attend_args* a, void* stream) {
  int rc = check_common(a);
  if (rc != DKV_OK) return rc;
  dkv::SoftmaxParams p{};
  p.scores = a->scores;
  p.seq_score_off = a->seq_score_off;
  p.seq_m = a->seq_m;
  p.query = static_cast<const __nv_bfloat16*>(a->query);
  p.exact_k = static_cast<const __nv_bfloat16*>(a->exact_k);
  p.mask = a->mask;
  p.n_seq = a->n_seq;
  p.n_q_heads = a->n_q_heads;
  p.q_per_kv = a->n_q_heads / a->n_kv_heads;
  p.q_len = a->q_len;
  p.head_dim = a->head_dim;
  p.n_exact = a->n_exact;
  p.scaling = a->scaling;
  p.row_stats = a->row_stats;
  p.p_exact = a->p_exact;
  if (a->softmax_mode < 0 || a->softmax_mode > 2) return DKV_ERR_ARGS;
  p.mode = a->softmax_mode;
  // The value stage's partial-sum buffer is free until the value weights run: it holds the softmax's
  // per-slice partials when few long rows are split over several CTAs.
  p.scratch = a->partial;
  p.scratch_floats = a->partial != nullptr ? static_cast<int64_t>(a->n_v_items) * a->rows_pad * a->v_item_groups * 64 : 0;
  p.n_sms = sm_count();
  p.status = a->status;
  p.f16 = a->fp16 ? 1 : 0;
  return dkv::run_softmax_stats(p, static_cast<cudaStream_t>(stream));
}

static int value_weights_rows(const dkv_attend_args* a, int row_begin, int n_rows, void* stream) {
  dkv::ValueWeightParams p{};
  p.code = a->v_code;
  p.code_size = a->v_code_size;
  p.tiles = reinterpret_cast<const TileDesc*>(a->v_tiles);
  p.groups = reinterpret_cast<const GroupDesc*>(a->v_groups);
  p.tok_sidx = a->v_sidx;
  p.items = a->v_items;
  p.item_ranges = a->v_item_ranges;
  p.tile_chunk = a->v_tile_chunk;
  p.max_planes = a->v_max_planes;
  p.n_items = a->n_v_items;
  p.item_groups = a->v_item_groups;
  p.scores = a->scores;
  p.seq_score_off = a->seq_score_off;
  p.seq_m = a->seq_m;
  p.row_stats = a->row_stats;
  p.n_q_heads = a->n_q_heads;
  p.q_len = a->q_len;
  p.row_begin = row_begin;
  p.n_rows = n_rows;
  p.n_rows_pad = a->rows_pad;
  p.partial = a->partial;
  p.status = a->status;
  p.cta_begin = a->v_cta_begin;
  p.item_order = a->v_item_order;
  p.p_img = a->p_img;
  p.n_tiles = a->n_v_tiles;
  p.f16 = a->fp16 ? 1 : 0;
  if ((a->v_item_order != nullptr && a->v_cta_begin == nullptr) || (a->v_cta_begin != nullptr && a->grid_v <= 0))
    return DKV_ERR_ARGS;
  const int grid = a->grid_v > 0 ? a->grid_v : (a->n_v_items < sm_count() ? a->n_v_items : sm_count());
  if (a->v_dense != nullptr && a->p_img != nullptr) {
    // Coefficients decoded once per step: TMA boxes of 64 components x 128 token rows.
    CUtensorMap map;
    const int rc = basis_map(a->v_dense, static_cast<uint64_t>(a->n_v_tiles) * 128, static_cast<uint64_t>(a->v_width),
                             128u, &map, a->fp16);
    if (rc != DKV_OK) return rc;
    return dkv::run_value_dense(map, p, grid, static_cast<cudaStream_t>(stream));
  }
  return dkv::run_value_weights(p, grid, static_cast<cudaStream_t>(stream));
}

static int finalize_rows(const dkv_attend_args* a, int row_begin, int n_rows, void* stream) {
  dkv::FinalizeParams p{};
  p.partial = a->partial;
  p.items = a->v_items;
  p.seq_items = a->v_seq_items;
  p.item_groups = a->v_item_groups;
  p.n_rows_pad = a->rows_pad;
  p.row_begin = row_begin;
  p.n_rows = n_rows;
  p.basis_v = static_cast<const __nv_bfloat16*>(a->v_basis);
  p.r_v = a->v_width;
  p.mean_v = static_cast<const __nv_bfloat16*>(a->v_mean);
  p.mean_seq_stride = a->v_mean_seq_stride;
  p.row_stats = a->row_stats;
  p.p_exact = a->p_exact;
  p.exact_v = static_cast<const __nv_bfloat16*>(a->exact_v);
  p.n_seq = a->n_seq;
  p.n_q_heads = a->n_q_heads;
  p.q_per_kv = a->n_q_heads / a->n_kv_heads;
  p.q_len = a->q_len;
  p.head_dim = a->head_dim;
  p.n_exact = a->n_exact;
  p.layer = a->layer;
  p.n_cols = a->n_kv_heads * a->head_dim;
  p.out = a->out;
  p.out_f32 = a->out_f32;
  p.vpart = a->vpart;
  p.status = a->status;
  p.f16 = a->fp16 ? 1 : 0;
  if (a->vpart == nullptr) return DKV_ERR_ARGS;
  return dkv::run_finalize(p, static_cast<cudaStream_t>(stream));
}

int dkv_value_weights(const dkv_attend_args* a, void* stream) {
  int rc = check_common(a);
  if (rc != DKV_OK) return rc;
  const int rows = a->n_q_heads * a->q_len;
  if (a->rows_pad < 16 || a->rows_pad > 128 || a->rows_pad % 16) return DKV_ERR_CONFIG;
  for (int r0 = 0; r0 < rows; r0 += a->rows_pad) {
    const int n = rows - r0 < a->rows_pad ? rows - r0 : a->rows_pad;
    rc = value_weights_rows(a, r0, n, stream);
    if (rc != DKV_OK) return rc;
  }
  return DKV_OK;
}

int dkv_finalize(const dkv_attend_args* a, void* stream) {
  int rc = check_common(a);
  if (rc != DKV_OK) return rc;
  const int rows = a->n_q_heads * a->q_len;
  if (rows > a->rows_pad) return DKV_ERR_CONFIG;  // multi-chunk rows go through dkv_attend_layer
  return finalize_rows(a, 0, rows, stream);
}

int64_t dkv_vpart_floats(int32_t v_width, int32_t n_seq, int32_t rows_pad, int32_t head_dim) {
  if (v_width < 0 || n_seq < 0 || rows_pad < 0 || head_dim < 0) return -1;
  return dkv::finalize_vpart_floats(v_width, n_seq, rows_pad, head_dim);
}

int dkv_attend_tail(const dkv_attend_args* a, void* stream) {
  int rc = check_common(a);
  if (rc != DKV_OK) return rc;
  const int rows = a->n_q_heads * a->q_len;
  if (a->rows_pad < 16 || a->rows_pad > 128 || a->rows_pad % 16) return DKV_ERR_CONFIG;
  for (int r0 = 0; r0 < rows; r0 += a->rows_pad) {
    const int n = rows - r0 < a->rows_pad ? rows - r0 : a->rows_pad;
    rc = value_weights_rows(a, r0, n, stream);
    if (rc != DKV_OK) return rc;
    rc = finalize_rows(a, r0, n, stream);
    if (rc != DKV_OK) return rc;
  }
  return DKV_OK;
}

int dkv_attend_layer(const dkv_attend_args* a, void* stream) {
  if (a != nullptr && a->softmax_mode != 0) return DKV_ERR_ARGS;  // split-K runs the stages one by one
  int rc = dkv_key_scores(a, stream);
  if (rc != DKV_OK) return rc;
  rc = dkv_softmax_stats(a, stream);
  if (rc != DKV_OK) return rc;
  const int rows = a->n_q_heads * a->q_len;
  if (a->rows_pad < 16 || a->rows_pad > 128 || a->rows_pad % 16) return DKV_ERR_CONFIG;
  for (int r0 = 0; r0 < rows; r0 += a->rows_pad) {
    const int n = rows - r0 < a->rows_pad ? rows - r0 : a->rows_pad;
    rc = value_weights_rows(a, r0, n, stream);
    if (rc != DKV_OK) return rc;
    rc = finalize_rows(a, r0, n, stream);
    if (rc != DKV_OK) return rc;
  }
  return DKV_OK;
}

int dkv_importance(const dkv_importance_args* a, void* stream) {
  if (a == nullptr || a->scores == nullptr || a->imp_compressed == nullptr) return DKV_ERR_ARGS;
  dkv::ImportanceParams p{};
  p.scores = a->scores;
  p.seq_score_off = a->seq_score_off;
  p.seq_m = a->seq_m;
  p.seq_k_base = a->seq_k_base;
  p.row_stats = a->row_stats;
  p.p_exact = a->p_exact;
  p.n_seq = a->n_seq;
  p.n_q_heads = a->n_q_heads;
  p.q_len = a->q_len;
  p.n_exact = a->n_exact;
  p.imp_compressed = a->imp_compressed;
  p.imp_exact = a->imp_exact;
  return dkv::run_importance(p, a->max_m, static_cast<cudaStream_t>(stream));
}

int dkv_topk(const dkv_topk_args* a, void* stream) {
  if (a == nullptr || a->importance == nullptr || a->positions == nullptr || a->out == nullptr) return DKV_ERR_ARGS;
  dkv::TopkParams p{};
  p.importance = a->importance;
  p.positions = a->positions;
  p.seq_k_base = a->seq_k_base;
  p.seq_m = a->seq_m;
  p.counts = a->counts;
  p.out_offset = a->out_offset;
  p.n_seq = a->n_seq;
  p.out = a->out;
  p.status = a->status;
  return dkv::run_topk(p, a->max_k, static_cast<cudaStream_t>(stream));
}

int dkv_refine_merge(const dkv_refine_args* a, void* stream) {
  if (a == nullptr || a->hot_code == nullptr || a->out_code == nullptr) return DKV_ERR_ARGS;
  dkv::RefineParams p{};
  p.hot_code = a->hot_code;
  p.hot_tiles = reinterpret_cast<const TileDesc*>(a->hot_tiles);
  p.hot_groups = reinterpret_cast<const GroupDesc*>(a->hot_groups);
  p.hot_tile = a->hot_tile;
  p.hot_row = a->hot_row;
  p.cold_words = a->cold_words;
  p.cold_headers = a->cold_headers;
  p.n_selected = a->n_selected;
  p.n_groups = a->n_groups;
  p.out_groups = reinterpret_cast<const GroupDesc*>(a->out_groups);
  p.out_code = a->out_code;
  p.status = a->status;
  return dkv::run_refine(p, static_cast<cudaStream_t>(stream));
}

int dkv_unpack(const dkv_unpack_args* a, void* stream) {
  if (a == nullptr || a->code == nullptr || a->tiles == nullptr || a->groups == nullptr || a->out == nullptr)
    return DKV_ERR_ARGS;
  dkv::UnpackParams p{};
  p.code = a->code;
  p.code_size = a->code_size;
  p.tiles = reinterpret_cast<const TileDesc*>(a->tiles);
  p.groups = reinterpret_cast<const GroupDesc*>(a->groups);
  p.n_tiles = a->n_tiles;
  p.out = a->out;
  p.out_cols = a->out_cols;
  p.out_bf16 = a->out_bf16;
  p.max_planes = a->max_planes;
  p.status = a->status;
  p.out_tile_rows = a->out_tile_rows;
  p.f16 = a->f16 ? 1 : 0;
  return dkv::run_unpack(p, static_cast<cudaStream_t>(stream));
}

int dkv_encode_groups(const dkv_encode_args* a, void* stream) {
  if (a == nullptr || a->coeff == nullptr || a->rung_planes == nullptr || a->codes == nullptr ||
      a->low == nullptr || a->span == nullptr || a->rung_error == nullptr || a->status == nullptr)
    return DKV_ERR_ARGS;
  dkv::EncodeParams p{};
  p.coeff = a->coeff;
  p.coeff_stride = a->coeff_stride;
  p.tokens = a->tokens;
  p.features = a->features;
  p.rung_planes = a->rung_planes;
  p.n_rungs = a->n_rungs;
  p.codes = a->codes;
  p.low = a->low;
  p.span = a->span;
  p.rung_error = a->rung_error;
  p.energy = a->energy;
  p.status = a->status;
  return dkv::run_encode(p, static_cast<cudaStream_t>(stream));
}

int dkv_storage_unpack(const dkv_storage_args* a, void* stream) {
  if (a == nullptr || a->data == nullptr || a->segments == nullptr || a->rows == nullptr || a->groups == nullptr ||
      a->out == nullptr || a->status == nullptr || a->out_rows < 0 || a->out_cols < 0)
    return DKV_ERR_ARGS;
  static_assert(sizeof(dkv_storage_segment) == sizeof(dkv::StorageSegment), "segment layout");
  dkv::StorageParams p{};
  p.data = a->data;
  p.data_size = a->data_size;
  p.segments = reinterpret_cast<const dkv::StorageSegment*>(a->segments);
  p.n_segments = a->n_segments;
  p.max_units = a->max_units;
  p.rows = a->rows;
  p.groups = a->groups;
  p.n_rows_idx = a->n_rows_idx;
  p.n_groups_idx = a->n_groups_idx;
  p.out = a->out;
  p.out_rows = a->out_rows;
  p.out_cols = a->out_cols;
  p.status = a->status;
  return dkv::run_storage_unpack(p, static_cast<cudaStream_t>(stream));
}

int dkv_demote(const dkv_demote_args* a, void* stream) {
  if (a == nullptr || a->old_code == nullptr || a->old_groups == nullptr || a->new_code == nullptr ||
      a->new_groups == nullptr || a->old_index == nullptr || a->n_tokens == nullptr || a->status == nullptr)
    return DKV_ERR_ARGS;
  dkv::DemoteParams p{};
  p.old_code = a->old_code;
  p.old_code_size = a->old_code_size;
  p.old_groups = reinterpret_cast<const GroupDesc*>(a->old_groups);
  p.n_old_groups = a->n_old_groups;
  p.new_code = a->new_code;
  p.new_code_size = a->new_code_size;
  p.new_groups = reinterpret_cast<const GroupDesc*>(a->new_groups);
  p.old_index = a->old_index;
  p.n_tokens = a->n_tokens;
  p.n_new = a->n_new;
  p.status = a->status;
  return dkv::run_demote(p, static_cast<cudaStream_t>(stream));
}

int64_t dkv_alloc_workspace_bytes(int64_t slots, int32_t levels) { return dkv::alloc_workspace_bytes(slots, levels); }

int dkv_allocate_rungs(const dkv_alloc_args* a, void* stream) {
  if (a == nullptr || a->errors == nullptr || a->level_bytes == nullptr || a->counts == nullptr ||
      a->status == nullptr)
    return DKV_ERR_ARGS;
  dkv::AllocParams p{};
  p.errors = a->errors;
  p.level_bytes = a->level_bytes;
  p.slots = a->slots;
  p.middle = a->middle;
  p.levels = a->levels;
  p.remaining = a->remaining;
  p.counts = a->counts;
  p.workspace = a->workspace;
  p.workspace_bytes = a->workspace_bytes;
  p.status = a->status;
  return dkv::run_allocate(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
