// la_paged_decode_noalloc: the paged decode entry point for callers that
// cannot allocate device memory. It runs exactly la_paged_decode, with the
// split-KV partials kept in a fixed array that belongs to this library
// instead of in a caller-provided workspace.
//
// Why: some callers of this library cannot call cudaMalloc at the point where
// they run decode attention — a host framework that owns every device
// allocation (a plugin may not allocate behind its back), a runtime whose
// device memory is a fixed arena handed out at start-up, or a latency-bound
// loop where an allocation would synchronise the device. They pass the inputs
// and outputs only.
//
// Set-up: the first call on each device resolves the array's device address
// (loading the module in that device's context); make that first call before
// any stream capture.
//
// Cost and limits: the array is LA_NOALLOC_SCRATCH_BYTES (4 MiB) of device
// memory on every GPU that loads the library, held until the process exits.
// It holds 2 * #SMs partial rows per query head, which is up to 27 query
// heads on a 148-SM B200 (Qwen3-0.6B has 16); a call that needs more is
// rejected with LA_ERR_WORKSPACE before anything is launched. Every call uses
// the same array: two calls whose kernels overlap on the GPU (different
// streams, different threads) race on it.
// Nothing in it has to start at zero, because every partial the combine pass
// reads was written earlier in the same call.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "la_internal.h"

namespace la {
namespace noalloc {

static __device__ __align__(256) unsigned char g_scratch[LA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static std::mutex g_mutex;
// Per device: the device address of g_scratch and the context it was
// resolved in. The address belongs to the module loaded in that context; a
// device reset, or a caller that makes another context current, loads the
// module again at a new address, so a changed context resolves it again.
static void* g_scratch_addr[kMaxDevices];
static CUcontext g_scratch_ctx[kMaxDevices];

static PFN_cuCtxGetCurrent_v4000 ctx_get_current_fn() {
  static std::once_flag once;
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

// The device address of g_scratch in the current context. In host code the
// name g_scratch is a host-side stand-in, not a device address; the runtime
// resolves the real address (loading the module there on first use).
static int scratch_address(int device, void** out) {
  auto get_ctx = ctx_get_current_fn();
  if (!get_ctx) return LA_ERR_CUDA;
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return LA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (ctx == nullptr || g_scratch_addr[device] == nullptr || g_scratch_ctx[device] != ctx) {
    // With no context current yet, this first runtime call makes the
    // device's primary context current; the context is read again after it.
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return LA_ERR_CUDA;
    g_scratch_addr[device] = addr;
    g_scratch_ctx[device] = ctx;
  }
  *out = g_scratch_addr[device];
  return LA_OK;
}

}  // namespace noalloc
}  // namespace la

extern "C" int la_paged_decode_noalloc(const void* q, int64_t q_batch_stride, int64_t q_head_stride,
                                       const void* k_cache, const void* v_cache, int64_t kv_block_stride,
                                       int64_t kv_token_stride, int64_t kv_head_stride, int64_t num_blocks,
                                       int block_size, const int32_t* block_table, int64_t bt_seq_stride,
                                       int max_blocks_per_seq, const int32_t* cache_seqlens, int batch,
                                       int num_q_heads, int num_kv_heads, int head_dim, float softmax_scale,
                                       void* out, int64_t out_batch_stride, int64_t out_head_stride,
                                       float* softmax_lse, int* dev_error, cudaStream_t stream) {
  const int device = la::current_device();
  if (device < 0 || device >= la::noalloc::kMaxDevices) return LA_ERR_CUDA;
  size_t need = 0;
  int st = la_paged_decode_workspace_size(device, num_q_heads, num_kv_heads, head_dim, &need);
  if (st != LA_OK) return st;
  if (need > LA_NOALLOC_SCRATCH_BYTES) return LA_ERR_WORKSPACE;  // beyond the fixed array
  void* scratch = nullptr;
  st = la::noalloc::scratch_address(device, &scratch);
  if (st != LA_OK) return st;
  return la_paged_decode(q, q_batch_stride, q_head_stride, k_cache, v_cache, kv_block_stride, kv_token_stride,
                         kv_head_stride, num_blocks, block_size, block_table, bt_seq_stride, max_blocks_per_seq,
                         cache_seqlens, batch, num_q_heads, num_kv_heads, head_dim, softmax_scale, out,
                         out_batch_stride, out_head_stride, softmax_lse, scratch, LA_NOALLOC_SCRATCH_BYTES,
                         dev_error, stream);
}
