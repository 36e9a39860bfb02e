// o_proj fused with the KV-head-sharded all-gather (tcgen05 GEMM, sm_100a).
//
// In the KV-head-sharded partition every rank's decode pass stores its query
// heads' attention outputs straight into every rank's gather slot over NVLink
// (la_paged_decode_allgather) and then publishes a new epoch into every
// rank's signal words (la_p2p_publish: no wait). This kernel then computes
//   y[B, N] = O[B, K] . W[N, K]^T     (leaninfer/qwen3/model.py:68-69)
// from this rank's gather slot O, where column block [q * K/P, (q + 1) * K/P)
// of O holds rank q's heads: before its first load from rank q's block the
// producer waits (bounded) until rank q's signal word has reached this
// rank's epoch, i.e. until rank q's stores of this call are visible. The
// peers' slices are consumed as they land, in a fixed column order (so every
// rank's y is bit-identical), and the GEMM's waits replace the barrier.
//
// Tiling: CTA tile 128 rows of B x BN columns of N (BN = 64, or 32 when the
// 64-wide grid would leave most SMs idle), K in 64-wide blocks staged by TMA
// (128-byte swizzle) through a kStages ring; one thread issues
// tcgen05.mma (M128 x BN x K16, bf16 in, fp32 accumulators in TMEM); four
// epilogue warps read the accumulators back (tcgen05.ld), round to bf16 and
// store.
//
// Slot reuse: call n+1's stores go to slot (n+1) % 2, which this rank's GEMM
// of call n-1 read. They come after this rank's GEMM of call n in stream
// order, and that GEMM waited for every peer's epoch n, which each peer
// publishes only after its own GEMM of call n-1 has finished: two slots are
// enough, as with the barrier.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace oproj {

constexpr int kBM = 128;             // rows of O (tokens) per CTA tile
constexpr int kBK = 64;              // K per stage (one 128-byte swizzle row)
constexpr int kStages = 6;
constexpr int kATile = kBM * kBK * 2;  // 16 KB
constexpr int kMaxPeers = 8;
constexpr int kThreads = 192;        // warp 0 TMA producer, 1 MMA + TMEM, 2-5 epilogue

struct Params {
  __nv_bfloat16* out;
  long long out_stride;
  int m, n, k;
  int k_per_rank;                    // K columns owned by each rank (K / world)
  const unsigned int* signals;       // this rank's signal words: [q] = rank q's epoch, [world] = own epoch
  int world;
  int rank;
  int bn;
  int* err;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    o_proj_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                  const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kWTile = BN * kBK * 2;
  constexpr int kStage = kATile + kWTile;  // multiple of 1024: swizzle atoms stay aligned
  static_assert(kStage % 1024 == 0, "stage tiles must keep 1024-byte alignment");
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  constexpr uint32_t kCols = BN < 32 ? 32 : BN;
  constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, BN, false, false);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * BN;
  const int kb_count = p.k / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The gather slot and the epoch word are written by earlier kernels.
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const unsigned int epoch = *reinterpret_cast<const volatile unsigned int*>(p.signals + p.world);
      int ready = -1;  // highest rank whose block is known visible (blocks are consumed in rank order)
      bool failed = false;
      for (int kb = 0; kb < kb_count; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = static_cast<uint32_t>((kb / kStages) & 1);
        mbar_wait(&empty[s], ph ^ 1u, p.err, LA_DEVERR_WAIT_TIMEOUT);
        const int q = (kb * kBK) / p.k_per_rank;
        if (!failed && q > ready) {
          // Rank q's stores of this call are visible once its epoch has
          // reached ours (its release at system scope pairs with this
          // acquire); then order the TMA (async proxy) reads after it.
          if (q != p.rank) {
            const uint64_t t0 = globaltimer_ns();
            while (true) {
              unsigned int v;
              asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.signals + q) : "memory");
              if (static_cast<int>(v - epoch) >= 0) break;
              if (globaltimer_ns() - t0 > LA_WAIT_LIMIT_NS) {
                if (p.err) atomicCAS(p.err, 0, LA_DEVERR_WAIT_TIMEOUT);
                failed = true;
                break;
              }
              __nanosleep(32);
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
          ready = q;
        }
        uint8_t* st = smem + s * kStage;
        if (failed) {
          // A peer never arrived: the error word says so. Complete the
          // stage without data so every role still finishes (y is invalid).
          mbar_arrive(&full[s]);
          continue;
        }
        mbar_arrive_expect_tx(&full[s], kStage);
        tma_load_2d(st, &tm_a, &full[s], kb * kBK, m0);
        tma_load_2d(st + kATile, &tm_w, &full[s], kb * kBK, n0);
      }
      // The copies issued last must land before the CTA's shared memory is
      // released (already true unless the MMA role gave up early; bounded).
      for (int kb = (kb_count > kStages ? kb_count - kStages : 0); kb < kb_count; ++kb)
        mbar_wait(&full[kb % kStages], static_cast<uint32_t>((kb / kStages) & 1), nullptr, 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    bool dead = false;  // a wait ran out: stop waiting, let every role finish
    for (int kb = 0; kb < kb_count; ++kb) {
      const int s = kb % kStages;
      const uint32_t ph = static_cast<uint32_t>((kb / kStages) & 1);
      const bool ok = !dead && __all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.err, LA_DEVERR_WAIT_TIMEOUT));
      dead = !ok;
      tc_fence_after();
      if (lane == 0) {
        if (ok) {
          const uint8_t* st = smem + s * kStage;
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            const uint64_t ad = smem_desc_sw128(smem_u32(st) + ks * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(smem_u32(st + kATile) + ks * 32, 16, 1024);
            umma_f16_ss(tmem, ad, bd, kIdesc, (kb > 0 || ks > 0) ? 1u : 0u);
          }
        }
        umma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(acc_full);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32 * (warp % 4) ..
    const int row = m0 + quarter * 32 + lane;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, p.err, LA_DEVERR_WAIT_TIMEOUT));
    tc_fence_after();
    if (ok) {
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        tc_wait_ld();
        if (row < p.m) {
          __nv_bfloat16* dst = p.out + static_cast<long long>(row) * p.out_stride + n0 + c * 32;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 u;
            u.x = pack_bf16x2(v[q4 * 8 + 0], v[q4 * 8 + 1]);
            u.y = pack_bf16x2(v[q4 * 8 + 2], v[q4 * 8 + 3]);
            u.z = pack_bf16x2(v[q4 * 8 + 4], v[q4 * 8 + 5]);
            u.w = pack_bf16x2(v[q4 * 8 + 6], v[q4 * 8 + 7]);
            if (n0 + c * 32 + q4 * 8 < p.n) *reinterpret_cast<uint4*>(dst + q4 * 8) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + static_cast<size_t>(kStages) * (kATile + BN * kBK * 2) + 256;
}

}  // namespace oproj

int oproj_init(int device) {
  (void)device;
  cudaError_t e = cudaFuncSetAttribute(oproj::o_proj_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(oproj::smem_bytes<64>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(oproj::o_proj_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(oproj::smem_bytes<32>()));
  return cuda_status(e);
}

}  // namespace la

extern "C" int la_o_proj_gathered(const void* gathered, int64_t gathered_row_stride, const void* weight,
                                  int64_t weight_row_stride, void* out, int64_t out_row_stride, int m, int n, int k,
                                  const unsigned int* signals, int world, int rank, int* dev_error,
                                  cudaStream_t stream) {
  using namespace la;
  using namespace la::oproj;
  if (!gathered || !weight || !out || !signals) return LA_ERR_INVALID_ARGUMENT;
  if (m < 0 || n <= 0 || k <= 0 || world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return LA_ERR_INVALID_ARGUMENT;
  if (m == 0) return LA_OK;
  if (k % (kBK * world) != 0 || n % 32 != 0) return LA_ERR_UNSUPPORTED;
  if (!aligned(gathered, 16) || !aligned(weight, 16) || !aligned(out, 16) || !aligned(signals, 4))
    return LA_ERR_ALIGNMENT;
  if (gathered_row_stride < k || weight_row_stride < k || out_row_stride < n || gathered_row_stride % 8 ||
      weight_row_stride % 8 || out_row_stride % 8)
    return LA_ERR_ALIGNMENT;
  const int device = current_device();
  const int sms = device >= 0 ? num_sms(device) : 0;
  if (sms <= 0) return LA_ERR_CUDA;
  CUtensorMap ta, tw;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(gathered_row_stride) * 2};
    const uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(kBM)};
    const int st = encode_tensor_map_bf16(&ta, gathered, 2, dims, strides, box, true);
    if (st != LA_OK) return st;
  }
  const int m_tiles = (m + kBM - 1) / kBM;
  // 64-wide column tiles when they give the grid at least half the SMs,
  // else 32-wide ones (twice the CTAs for small batches)
  const int bn = (n % 64 == 0 && m_tiles * (n / 64) >= sms / 2) ? 64 : 32;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(weight_row_stride) * 2};
    const uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(bn)};
    const int st = encode_tensor_map_bf16(&tw, weight, 2, dims, strides, box, true);
    if (st != LA_OK) return st;
  }
  Params p;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_row_stride;
  p.m = m;
  p.n = n;
  p.k = k;
  p.k_per_rank = k / world;
  p.signals = signals;
  p.world = world;
  p.rank = rank;
  p.bn = bn;
  p.err = dev_error;
  const dim3 grid(static_cast<unsigned>(n / bn), static_cast<unsigned>(m_tiles));
  cudaError_t e = bn == 64 ? launch_pdl(o_proj_kernel<64>, grid, dim3(kThreads), smem_bytes<64>(), stream, ta, tw, p)
                           : launch_pdl(o_proj_kernel<32>, grid, dim3(kThreads), smem_bytes<32>(), stream, ta, tw, p);
  return cuda_status(e);
}
