// Peer memory for the KV-head-sharded decode all-gather over NVLink.
//
// Each rank allocates one buffer (signal words + gather slots) with
// la_p2p_alloc, exports its CUDA IPC handle, and maps every peer's buffer
// with la_p2p_open. la_paged_decode_allgather then stores this rank's heads
// into every rank's gather slot; la_p2p_barrier, next on the same stream,
// publishes this rank's next epoch into every rank's signal words and waits
// (bounded) until every peer's epoch has caught up with it. Signal words of a
// rank: [q] = the last epoch rank q published, [world] = its own epoch.
#include <cuda_runtime.h>

#include <cstring>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace p2p {

constexpr int kMaxPeers = 8;

struct Signals {
  unsigned int* words[kMaxPeers];  // every rank's signal words, rank order
};

// One warp. Lane 0 bumps this rank's epoch and stores it, with release
// semantics at system scope, into word [rank] of every rank (the stores of
// earlier kernels on this stream are ordered before it: they fenced at system
// scope). Lane q then waits until rank q's epoch in this rank's word [q] has
// reached the same value: from then on rank q's stores of the same call are
// visible here.
// With wait == 0 (la_p2p_publish) the kernel only publishes: a later kernel
// waits for each peer's epoch itself (la_o_proj_gathered).
__global__ void __launch_bounds__(32) barrier_kernel(Signals s, int world, int rank, int wait, int* err) {
  const int q = threadIdx.x;
  unsigned int* own = s.words[rank];
  unsigned int epoch = 0;
  grid_dependency_wait();  // launched with programmatic serialization: the previous kernel must be done
  if (q == 0) {
    epoch = own[world] + 1u;
    own[world] = epoch;
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(s.words[r] + rank), "r"(epoch) : "memory");
  }
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  if (!wait || q >= world || q == rank) return;
  const unsigned int* sig = own;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(sig + q) : "memory");
    if (static_cast<int>(v - epoch) >= 0) return;
    if (globaltimer_ns() - t0 > LA_WAIT_LIMIT_NS) {
      if (err) atomicCAS(err, 0, LA_DEVERR_WAIT_TIMEOUT);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace p2p
}  // namespace la

extern "C" int la_p2p_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return LA_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return la::cuda_status(e);
  e = cudaMemset(p, 0, bytes);  // signal words start at epoch 0
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return la::cuda_status(e);
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return LA_OK;
}

extern "C" int la_p2p_open(const void* ipc_handle, void** peer_ptr) {
  if (!ipc_handle || !peer_ptr) return LA_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return la::cuda_status(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int la_p2p_close(void* peer_ptr) { return la::cuda_status(cudaIpcCloseMemHandle(peer_ptr)); }

extern "C" int la_p2p_free(void* ptr) { return la::cuda_status(cudaFree(ptr)); }

namespace la {
namespace p2p {
static int launch_barrier(unsigned int* const* signals, int world, int rank, int wait, int* dev_error,
                          cudaStream_t stream) {
  if (!signals || world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return LA_ERR_INVALID_ARGUMENT;
  Signals s{};
  for (int r = 0; r < world; ++r) {
    if (!signals[r] || !aligned(signals[r], 4)) return LA_ERR_INVALID_ARGUMENT;
    s.words[r] = signals[r];
  }
  return cuda_status(launch_pdl(barrier_kernel, dim3(1), dim3(32), 0, stream, s, world, rank, wait, dev_error));
}
}  // namespace p2p
}  // namespace la

extern "C" int la_p2p_barrier(unsigned int* const* signals, int world, int rank, int* dev_error,
                              cudaStream_t stream) {
  return la::p2p::launch_barrier(signals, world, rank, 1, dev_error, stream);
}

extern "C" int la_p2p_publish(unsigned int* const* signals, int world, int rank, int* dev_error,
                              cudaStream_t stream) {
  return la::p2p::launch_barrier(signals, world, rank, 0, dev_error, stream);
}
