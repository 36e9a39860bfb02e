// Host-side helpers shared by the entry points of liblean_attn.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <utility>

#include "lean_attn.h"

namespace la {

// Records `e` as this thread's last CUDA error and maps it to a status code.
int cuda_status(cudaError_t e);

// Number of SMs of `device` (cached per device).
int num_sms(int device);

// Current device of the calling thread, or -1.
int current_device();

// Encode a bf16 tiled tensor map (rank 2..5). dims / strides_bytes are in the
// cuTensorMapEncodeTiled order (dimension 0 innermost, strides for 1..rank-1).
int encode_tensor_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch with the programmatic-stream-serialization attribute (PDL) so the
// kernel's prologue can overlap the tail of the previous kernel in the stream.
// Kernels launched this way call griddepcontrol.wait before touching data
// the previous kernel may write.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Per-kernel init hooks called by la_init().
int decode_init(int device);
int pre_attn_init(int device);
int prefill_init(int device);
int oproj_init(int device);

}  // namespace la
