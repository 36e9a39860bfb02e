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
// Tiling: CTA tile 128 rows of B x BN columns of N (BN = 128, 64 or 32), K
// in 64-wide blocks staged by TMA (128-byte swizzle) through a kStages ring;
// one thread issues tcgen05.mma (M128 x BN x K16, bf16 in, fp32
// accumulators in TMEM). Split-K over a thread-block cluster of S CTAs (S =
// 1, 2 or 4, chosen so the grid fills the SMs): CTA z of a cluster takes the
// z-th 1/S of K (and so waits only for the ranks owning it), its epilogue
// warps move the fp32 partial tile from TMEM to its shared memory, and after
// a cluster barrier each CTA sums 1/S of the tile's rows over the S partials
// through distributed shared memory, in cluster-rank order, and stores bf16.
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

__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int BN, int S>
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
  const int z = S > 1 ? static_cast<int>(blockIdx.z) : 0;  // cluster rank: the cluster spans z
  const int kb_count = p.k / kBK / S;                       // this CTA's K blocks
  const int kb0 = z * kb_count;

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
        const int q = ((kb0 + kb) * kBK) / p.k_per_rank;
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
        tma_load_2d(st, &tm_a, &full[s], (kb0 + kb) * kBK, m0);
        tma_load_2d(st + kATile, &tm_w, &full[s], (kb0 + kb) * kBK, n0);
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
    const int trow = quarter * 32 + lane;  // row of the tile
    const int row = m0 + trow;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, p.err, LA_DEVERR_WAIT_TIMEOUT));
    tc_fence_after();
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    if constexpr (S == 1) {
      if (ok) {
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
              *reinterpret_cast<uint4*>(dst + q4 * 8) = u;
            }
          }
        }
      }
    } else {
      // fp32 partial tile [128][BN] into this CTA's shared memory (the ring
      // is idle: every load landed and every MMA completed before acc_full)
      float* red = reinterpret_cast<float*>(smem);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<float4*>(red + trow * BN + c * 32 + q4 * 4) =
              make_float4(ok ? v[q4 * 4] : 0.f, ok ? v[q4 * 4 + 1] : 0.f, ok ? v[q4 * 4 + 2] : 0.f,
                          ok ? v[q4 * 4 + 3] : 0.f);
      }
    }
  }
  if constexpr (S > 1) {
    // every CTA of the cluster has its partial in shared memory
    cluster_sync();
    if (warp >= 2) {
      // rows [z * 128 / S, (z + 1) * 128 / S) of the tile, summed over the S
      // partials in cluster-rank order; 4 columns per thread per step
      const int t = threadIdx.x - 64;
      constexpr int kRowsPer = kBM / S;
      constexpr int kChunks = kRowsPer * BN / 4;
      const uint32_t base = smem_u32(smem);
      for (int c = t; c < kChunks; c += 128) {
        const int trow = z * kRowsPer + c / (BN / 4);
        const int col = (c % (BN / 4)) * 4;
        const uint32_t off = static_cast<uint32_t>((trow * BN + col) * 4);
        float4 acc = ld_cluster_f4(cluster_map(base + off, 0));
#pragma unroll
        for (int r = 1; r < S; ++r) {
          const float4 v = ld_cluster_f4(cluster_map(base + off, static_cast<uint32_t>(r)));
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        const int row = m0 + trow;
        if (row < p.m) {
          uint2 u;
          u.x = pack_bf16x2(acc.x, acc.y);
          u.y = pack_bf16x2(acc.z, acc.w);
          *reinterpret_cast<uint2*>(p.out + static_cast<long long>(row) * p.out_stride + n0 + col) = u;
        }
      }
    }
    // no CTA leaves while a peer may still read its shared memory
    cluster_sync();
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
static_assert(kStages * (kATile + 32 * kBK * 2) >= kBM * 128 * 4, "the ring holds the fp32 partial tile");

template <int BN, int S>
static cudaError_t set_attr() {
  return cudaFuncSetAttribute(o_proj_kernel<BN, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem_bytes<BN>()));
}

template <int BN, int S>
static cudaError_t launch(dim3 grid, cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                          const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<BN>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = S;
  cfg.attrs = attr;
  cfg.numAttrs = S > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, o_proj_kernel<BN, S>, ta, tw, p);
}

}  // namespace oproj

int oproj_init(int device) {
  (void)device;
  using namespace oproj;
  cudaError_t e = set_attr<128, 1>();
  if (e == cudaSuccess) e = set_attr<128, 2>();
  if (e == cudaSuccess) e = set_attr<128, 4>();
  if (e == cudaSuccess) e = set_attr<64, 1>();
  if (e == cudaSuccess) e = set_attr<64, 2>();
  if (e == cudaSuccess) e = set_attr<64, 4>();
  if (e == cudaSuccess) e = set_attr<32, 1>();
  if (e == cudaSuccess) e = set_attr<32, 2>();
  if (e == cudaSuccess) e = set_attr<32, 4>();
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
  // Tile width and split: the most CTAs not above the SM count, then the
  // widest tile, then the smallest split.
  int bn = 32, split = 1;
  {
    long long best = -1;
    for (int cb : {128, 64, 32}) {
      if (n % cb) continue;
      for (int cs : {1, 2, 4}) {
        if ((k / kBK) % cs) continue;
        const long long ctas = static_cast<long long>(m_tiles) * (n / cb) * cs;
        const long long score = ctas <= sms ? ctas : -1;
        if (score > best) {
          best = score;
          bn = cb;
          split = cs;
        }
      }
    }
    if (best < 0) {  // even the smallest grid exceeds the SMs: no split, widest tile
      split = 1;
      bn = n % 128 == 0 ? 128 : (n % 64 == 0 ? 64 : 32);
    }
  }
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
  const dim3 grid(static_cast<unsigned>(n / bn), static_cast<unsigned>(m_tiles), static_cast<unsigned>(split));
  cudaError_t e;
#define LA_OPROJ_LAUNCH(BN_, S_) \
  if (bn == BN_ && split == S_) e = launch<BN_, S_>(grid, stream, ta, tw, p);
  LA_OPROJ_LAUNCH(128, 1) else LA_OPROJ_LAUNCH(128, 2) else LA_OPROJ_LAUNCH(128, 4)
  else LA_OPROJ_LAUNCH(64, 1) else LA_OPROJ_LAUNCH(64, 2) else LA_OPROJ_LAUNCH(64, 4)
  else LA_OPROJ_LAUNCH(32, 1) else LA_OPROJ_LAUNCH(32, 2) else LA_OPROJ_LAUNCH(32, 4)
  else return LA_ERR_UNSUPPORTED;
#undef LA_OPROJ_LAUNCH
  return cuda_status(e);
}
