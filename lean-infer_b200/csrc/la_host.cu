// Library-wide host code: status strings, device queries, tensor-map encoding
// and la_init().
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "la_internal.h"

namespace la {

static thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return LA_OK;
  g_last_cuda_error = static_cast<int>(e);
  return LA_ERR_CUDA;
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

static constexpr int kMaxDevices = 64;
static std::atomic<int> g_sms[kMaxDevices];

int num_sms(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  int v = g_sms[device].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  g_sms[device].store(n, std::memory_order_relaxed);
  return n;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_tensor_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  auto fn = get_encode_fn();
  if (!fn) return LA_ERR_TENSOR_MAP;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gstride[i] = strides_bytes[i];
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                  gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LA_OK : LA_ERR_TENSOR_MAP;
}

}  // namespace la

extern "C" {

int la_version(void) { return LA_VERSION; }

const char* la_status_string(int status) {
  switch (status) {
    case LA_OK: return "ok";
    case LA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LA_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case LA_ERR_ALIGNMENT: return "pointer or stride misaligned";
    case LA_ERR_WORKSPACE: return "workspace missing or too small";
    case LA_ERR_CUDA: return "CUDA error";
    case LA_ERR_TENSOR_MAP: return "tensor map encoding failed";
    default: return "unknown status";
  }
}

int la_last_cuda_error(void) { return la::g_last_cuda_error; }

int la_init(int device) {
  if (device < 0) return LA_ERR_INVALID_ARGUMENT;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return la::cuda_status(e);
  int st = LA_OK;
  if (la::num_sms(device) <= 0) st = LA_ERR_CUDA;
  if (st == LA_OK) st = la::decode_init(device);
  if (st == LA_OK) st = la::pre_attn_init(device);
  if (st == LA_OK) st = la::prefill_init(device);
  if (st == LA_OK) st = la::oproj_init(device);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return st;
}

}  // extern "C"
