// static_scratch.cu — dkv_attend_layer_static: one attention layer without any device allocation.
//
// dkv_attend_layer needs four scratch buffers between its kernels (scores, row statistics, exact-token
// probabilities, value partial sums) and expects the caller to allocate them. Some callers cannot:
// a plugin running inside another framework's memory manager (an inference-server backend, a custom
// runtime) that owns every device allocation and forbids direct cudaMalloc / cudaFree, or a
// latency-critical loop that may not pay for an allocation (cudaMalloc and cudaFree can synchronise
// the device). For them this entry point carves the scratch out of one fixed array in device memory
// that the library itself declares; the caller still passes the inputs, the output and the status word.
//
// Limits and behaviour:
//   - the array holds kStaticScratchBytes (32 MiB). Every GPU that loads the library keeps it until the
//     process exits. A call whose scratch does not fit returns DKV_ERR_SCRATCH and launches nothing.
//     One conversation of 16K tokens of a Llama-3.2-3B-shaped model needs about 6 MiB per decode step.
//   - the first call on a device looks the array's device address up (cudaGetSymbolAddress, with that
//     device current) and caches it with the device's current CUDA context; make that first call before
//     any stream capture. After a cudaDeviceReset (or any new primary context) the module is loaded again,
//     possibly at another address: the next call sees the new context and looks the address up again.
//   - all calls share the array and it keeps the last call's contents. Every scratch byte the kernels
//     read is written earlier in the same call, so nothing needs clearing between calls, but two calls
//     that overlap on the GPU (different streams, or different host threads) race on it.
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dimmer_kv.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mutex;
void* g_static_addr[kMaxDevices] = {};
CUcontext g_static_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The calling thread's current driver context (the runtime's primary context of the current device).
CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Sizes saturate at kSizeCap, one byte more than the array: an overflowing product or sum reads as a
// request that does not fit instead of wrapping to a small size.
constexpr size_t kSizeCap = kStaticScratchBytes + 1;
size_t sat_mul(size_t a, size_t b) { return (a != 0 && b > kSizeCap / a) ? kSizeCap : (a * b < kSizeCap ? a * b : kSizeCap); }
size_t sat_add(size_t a, size_t b) { return a + b < kSizeCap ? a + b : kSizeCap; }
size_t align256(size_t x) { return x >= kSizeCap ? kSizeCap : ((x + 255) & ~size_t(255)); }

// Device address of the array on the current device, looked up once per device and context.
int static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DKV_ERR_CUDA;
  void* ptr = nullptr;
  // cudaGetSymbolAddress also makes the device's primary context current if none was yet.
  std::lock_guard<std::mutex> lock(g_static_mutex);
  CUcontext ctx = current_context();
  if (g_static_addr[dev] == nullptr || ctx == nullptr || ctx != g_static_ctx[dev]) {
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr) return DKV_ERR_CUDA;
    g_static_addr[dev] = ptr;
    g_static_ctx[dev] = current_context();
  }
  *out = g_static_addr[dev];
  return DKV_OK;
}

}  // namespace

extern "C" int dkv_attend_layer_static(const dkv_attend_args* args, int64_t n_scores, void* stream) {
  if (args == nullptr || n_scores < 0 || args->n_seq < 0 || args->n_q_heads < 1 || args->q_len < 1 ||
      args->n_exact < 0 || args->n_v_items < 0 || args->rows_pad < 0 || args->v_item_groups < 0)
    return DKV_ERR_ARGS;
  const size_t rows = sat_mul(sat_mul(static_cast<size_t>(args->n_seq), static_cast<size_t>(args->n_q_heads)),
                              static_cast<size_t>(args->q_len));
  const size_t scores_bytes = align256(sat_mul(static_cast<size_t>(n_scores), sizeof(float)));
  const size_t stats_bytes = align256(sat_mul(rows, 4 * sizeof(float)));
  const size_t exact_bytes = align256(sat_mul(sat_mul(rows, static_cast<size_t>(args->n_exact)), sizeof(float)));
  const size_t partial_bytes = align256(sat_mul(sat_mul(sat_mul(static_cast<size_t>(args->n_v_items),
                                                                static_cast<size_t>(args->rows_pad)),
                                                        static_cast<size_t>(args->v_item_groups)),
                                                64 * sizeof(float)));
  // dkv_vpart_floats is n_seq * rows_pad * (a per-(conversation, row) factor of v_width and head_dim): take the
  // factor and multiply the rest here with saturation.
  const int64_t vpart_row = dkv_vpart_floats(args->v_width, 1, 1, args->head_dim);
  if (vpart_row < 0) return DKV_ERR_ARGS;
  const size_t vpart_floats = sat_mul(sat_mul(static_cast<size_t>(vpart_row), static_cast<size_t>(args->n_seq)),
                                      static_cast<size_t>(args->rows_pad));
  const size_t vpart_bytes = align256(sat_mul(vpart_floats, sizeof(float)));
  const size_t total =
      sat_add(sat_add(sat_add(sat_add(scores_bytes, stats_bytes), exact_bytes), partial_bytes), vpart_bytes);
  if (total > kStaticScratchBytes) return DKV_ERR_SCRATCH;
  void* base = nullptr;
  const int rc = static_scratch_address(&base);
  if (rc != DKV_OK) return rc;
  unsigned char* p = static_cast<unsigned char*>(base);
  dkv_attend_args a = *args;
  a.scores = reinterpret_cast<float*>(p);
  a.row_stats = reinterpret_cast<float*>(p + scores_bytes);
  a.p_exact = reinterpret_cast<float*>(p + scores_bytes + stats_bytes);
  a.partial = reinterpret_cast<float*>(p + scores_bytes + stats_bytes + exact_bytes);
  a.vpart = reinterpret_cast<float*>(p + scores_bytes + stats_bytes + exact_bytes + partial_bytes);
  a.p_img = nullptr;  // the value kernel builds its probability tiles itself
  return dkv_attend_layer(&a, stream);
}
