// (b) Paged GQA decode attention for sm_100a: a persistent, warp-specialised
// split-KV kernel plus a combine kernel.
//
// Semantics (leaninfer/qwen3/model.py:60-67 -> flash_attn_with_kvcache with a
// block table, one query token, causal bottom-right alignment, which at
// q_len = 1 means "all keys 0..cache_seqlens[b]-1"):
//   out[b, h] = softmax(scale * q[b, h] . K[b, :, h / G]^T) . V[b, :, h / G]
// where K[b, t] = k_cache[block_table[b, t / BS], t % BS].
//
// Work decomposition. The key range of every sequence is cut into units of
// TC = 16 * (8 / Hkv) tokens; a unit is one pipeline stage: 128 (token, kv
// head) rows of K and of V, 32 KB each. The units of all sequences, laid end
// to end, are split into gridDim.x equal contiguous ranges, one per CTA
// (grid = #SMs, one CTA per SM), so every SM streams the same number of bytes
// whatever the length mix. The partition is recomputed on the device from
// cache_seqlens, so the launch shape never depends on device data and the
// call can be captured in a CUDA graph. A CTA range covers whole sequences
// (written straight to `out`) and at most two partial sequences at its ends
// (written as fp32 (O, lse) partials to the workspace and merged by the
// combine kernel).
//
// CTA: warps 8 and 9 are the producers (partition walk, block-table lookups,
// TMA issue), taking even and odd units in turn; warps 0-7 consume. Consumer warp w handles kv head w % Hkv and the
// 16-token sub-chunk w / Hkv of each stage: S^T = K Q^T and O^T += V^T P^T on
// mma.m16n8k16 (bf16 in, fp32 accumulate) with K/V fragments read by ldmatrix
// from 128-byte-swizzled TMA tiles, online softmax in fp32 with warp-shuffle
// max reductions, P transposed into the B operand with movmatrix.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace decode {

constexpr int kD = 128;
constexpr int kSub = 16;                 // tokens per consumer warp per stage (MMA M)
constexpr int kCWarps = 8;               // consumer warps
constexpr int kMaxProducers = 2;  // producer warps (units alternate between them); the launch picks 1 or 2
constexpr int kThreads = (kCWarps + kMaxProducers) * 32;
constexpr int kTileBytes = kSub * 128;   // 16 rows x 64 dims bf16 (one swizzle-128B tile)
constexpr int kWarpBytes = 2 * kTileBytes;
constexpr int kKVHalf = kCWarps * kTileBytes;   // one 64-dim half of all warps' tiles: 16 KB
constexpr int kKVBytes = 2 * kKVHalf;           // 32 KB per tensor per stage
// Stage layout per tensor: [half][warp w][16 rows][128 B]; warp w = j*Hkv + h
// holds kv head h of sub-chunk j, so the Hkv heads of a sub-chunk are one
// contiguous run that a single TMA box [64 dims, 16 tokens, Hkv heads] fills.
constexpr int kMaxStages = 4;

constexpr int kMaxPeers = 8;  // ranks of a KV-head-sharded group
constexpr int kFlagFirst = 1;  // first stage of this CTA's segment of the sequence
constexpr int kFlagLast = 2;   // last stage of the segment
constexpr int kFlagWhole = 4;  // the segment is the whole sequence

struct StageDesc {
  int b;
  int tok0;
  int ctx;
  int flags;
  int slot;  // partial slot base (2*cta + 0/1) for segments that are not whole
  int pad[3];
};

struct Params {
  const int* seqlens;
  const int* block_table;
  long long bt_stride;
  int max_blocks;
  int batch;
  int hq, hkv, group, nsub;  // nsub = 8 / hkv consumer warps per kv head
  int block_size;
  int bs_shift;              // log2(block_size) when it is a power of two, else -1
  int tc_shift;              // log2(tc)
  long long num_blocks;
  int tc;                    // tokens per stage
  float scale_log2;
  __nv_bfloat16* out;
  long long out_b_stride, out_h_stride;
  // The decode pass writes `out` only. The combine pass stores every output
  // row to outs[0..nouts): `out` alone, or, for the KV-head-sharded
  // all-gather, every rank's gather buffer (peer pointers over NVLink; rows
  // the decode pass finished are forwarded from `out` with coalesced 8-byte
  // stores). With peer_stores set, each combine CTA then fences once at
  // system scope, so the epoch a later barrier publishes orders after its
  // stores.
  __nv_bfloat16* outs[kMaxPeers];
  int nouts;
  int peer_stores;
  float* lse_out;
  float* part_o;    // [slots][hq][D]
  float* part_lse;  // [slots][hq] (log2 domain, scaled)
  int* err;
  int q_bytes;      // Q bytes landed per stage (both halves)
  int q_half_bytes; // stride between the two Q halves (1024-byte aligned)
  int stage_bytes;
  int big_box;      // 1: K/V maps are [D, BS, Hkv, NB] with box (64, 16, Hkv, 1)
  // 1: one or two kv heads over blocks of a multiple of tc tokens: the K/V
  // maps are 5-D [D, 16 tokens, Hkv, BS / 16, NB] with box
  // (64, 16, Hkv, nsub, 1), whose rows land in the stage's order [sub-chunk
  // j][kv head][16 tokens]: a whole unit per half per tensor in one box.
  int unit_box;
};

// Number of stage units of a sequence, with the same clamping everywhere.
__device__ __forceinline__ int seq_ctx(const Params& p, int b) {
  int c = p.seqlens[b];
  if (c < 0) c = 0;
  const long long cap = static_cast<long long>(p.max_blocks) * p.block_size;
  if (c > cap) {
    if (p.err) atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
    c = static_cast<int>(cap);
  }
  return c;
}
__device__ __forceinline__ int units_of(int ctx, int tc) { return (ctx + tc - 1) / tc; }
// Division by the block size and the unit size on the producer's per-unit
// path: shifts (a division by a run-time value is a dependent chain of about
// twenty instructions, and the producer paced the pipeline at one kv head).
__device__ __forceinline__ int div_bs(const Params& p, int x) {
  return p.bs_shift >= 0 ? (x >> p.bs_shift) : (x / p.block_size);
}
__device__ __forceinline__ int units_p(const Params& p, int ctx) { return (ctx + p.tc - 1) >> p.tc_shift; }

__device__ __forceinline__ float warp_max_g(float v) {
  // max over the 8 lanes that share lane % 4
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}
__device__ __forceinline__ float warp_sum_g(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// Total units over all sequences, computed by one warp.
__device__ long long total_units(const Params& p, int lane) {
  long long tot = 0;
  for (int base = 0; base < p.batch; base += 32) {
    const int b = base + lane;
    int n = (b < p.batch) ? units_of(seq_ctx(p, b), p.tc) : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    tot += n;
  }
  return tot;
}

// The split for up to 32 x kChunks sequences from their lengths held in
// registers, lane l holding the kChunks consecutive sequences l * kChunks + i:
// total units T, this CTA's range [u0, u1), the sequence b0 it starts in and
// that sequence's first unit pb0. Each lane sums its own sequences, one warp
// scan orders the lanes, and the lane whose sequences hold unit u0 walks its
// registers (a scan per 32 sequences, one after another, took 18k clocks at
// 1024 sequences before the first copy could be issued).
__device__ __forceinline__ long long cta_start(long long c, long long T, long long G);
template <int kChunks>
__device__ __forceinline__ void split_from_regs(const Params& p, int lane, const int (&un)[kChunks], long long& T,
                                                long long& u0, long long& u1, int& b0, long long& pb0) {
  long long own = 0;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) own += un[i];
  long long incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const long long excl = incl - own;
  T = __shfl_sync(0xffffffffu, incl, 31);
  const long long G = gridDim.x;
  u0 = cta_start(blockIdx.x, T, G);
  u1 = cta_start(blockIdx.x + 1, T, G);
  b0 = p.batch;
  pb0 = T;
  if (u1 <= u0) return;
  const unsigned hit = __ballot_sync(0xffffffffu, excl <= u0 && u0 < incl);
  const int src = __ffs(hit) - 1;  // u0 < T, so exactly one lane holds it
  int bl = 0;
  long long pbl = 0;
  if (lane == src) {
    long long acc = excl;
    bool found = false;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      if (!found && u0 < acc + un[i]) {
        found = true;
        bl = lane * kChunks + i;
        pbl = acc;
      }
      acc += un[i];
    }
  }
  b0 = __shfl_sync(0xffffffffu, bl, src);
  pb0 = __shfl_sync(0xffffffffu, pbl, src);
}

// The lengths of sequences lane * kChunks + i (0 past the batch), read
// through L2 only; 16-byte loads where the run is aligned and inside the
// batch.
template <int kChunks>
__device__ __forceinline__ void load_lens(const Params& p, int lane, int (&raw)[kChunks]) {
  static_assert(kChunks % 4 == 0, "lengths are loaded four at a time");
  const int b0 = lane * kChunks;
  const bool vec = (reinterpret_cast<uintptr_t>(p.seqlens) & 15) == 0;
#pragma unroll
  for (int v = 0; v < kChunks / 4; ++v) {
    const int b = b0 + 4 * v;
    if (vec && b + 3 < p.batch) {
      const int4 x = __ldcg(reinterpret_cast<const int4*>(p.seqlens + b));
      raw[4 * v] = x.x;
      raw[4 * v + 1] = x.y;
      raw[4 * v + 2] = x.z;
      raw[4 * v + 3] = x.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) raw[4 * v + e] = (b + e < p.batch) ? __ldcg(p.seqlens + b + e) : 0;
    }
  }
}

// First unit of CTA c: floor(c * T / G).
__device__ __forceinline__ long long cta_start(long long c, long long T, long long G) { return c * T / G; }
// CTA whose range contains unit x: floor(((x + 1) * G - 1) / T).
__device__ __forceinline__ long long cta_of(long long x, long long T, long long G) { return ((x + 1) * G - 1) / T; }

// kChunks: the split is held in registers for up to 32 x kChunks sequences
// (8 for the engine's batches, 32 for the many short rows of the KV-head-
// sharded partition).
template <int kStages, int kChunks>
__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_k1,
                        const __grid_constant__ CUtensorMap tm_v1, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ctrl = smem + kStages * p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
  uint64_t* empty = full + kMaxStages;
  StageDesc* descs = reinterpret_cast<StageDesc*>(ctrl + 128);
  uint8_t* zero_row = ctrl + 256;
  long long* sched = reinterpret_cast<long long*>(ctrl + 384);
  uint64_t* mg_full = reinterpret_cast<uint64_t*>(ctrl + 448);   // all consumer warps wrote their state
  uint64_t* mg_empty = reinterpret_cast<uint64_t*>(ctrl + 456);  // the j = 0 warps read it
  float* merge = reinterpret_cast<float*>(ctrl + 1024);          // [8 warps][TQ][8][36] fp32 (nsub > 1)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    mbar_init(mg_full, kCWarps);
    mbar_init(mg_empty, p.hkv);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) reinterpret_cast<uint32_t*>(zero_row)[threadIdx.x] = 0u;
  if (warp == kCWarps && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  // The split is computed speculatively before the dependency wait from the
  // lengths as they are now (read through L2 only, so no stale line stays in
  // L1), then the lengths are read again after the wait: if any changed (the
  // previous kernel wrote them) the split is recomputed from the final ones.
  const bool spec = p.batch <= 32 * kChunks;
  int raw[kChunks];
  long long sT = 0, su0 = 0, su1 = 0, spb0 = 0;
  int sb0 = 0;
  if (warp >= kCWarps && spec) {
    int un[kChunks];
    const long long cap = static_cast<long long>(p.max_blocks) * p.block_size;
    load_lens(p, lane, raw);
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const long long c = raw[i] < 0 ? 0 : (raw[i] > cap ? cap : raw[i]);
      un[i] = units_of(static_cast<int>(c), p.tc);
    }
    split_from_regs(p, lane, un, sT, su0, su1, sb0, spb0);
  }
  // Everything below may read data written by the previous kernel in the stream.
  grid_dependency_wait();

  // Producer lookups go through two windows held across its 32 lanes, so
  // that a unit's copies wait on no global load in the common case: lane i
  // holds the (clamped) length of sequence sb + i, and the raw block id of
  // block wl + i of sequence bb. Entering a sequence also loads the first 32
  // block ids of the next one, which are read at the next sequence change
  // (with one kv head a sequence is ~6 units, and two dependent global round
  // trips per unit made the producer the slowest part of the pipeline). The
  // windows of the first sequence are loaded with the speculative split,
  // together with the re-read that checks it.
  int sb = 0, swin = 0, bb = -1, wl = 0, bwin = -1;
  auto load_swin = [&](int base) {
    sb = base;
    swin = (sb + lane < p.batch) ? seq_ctx(p, sb + lane) : 0;
  };
  auto load_bwin = [&](int seq, int first) {
    bb = seq;
    wl = first;
    bwin = (seq < p.batch && wl + lane < p.max_blocks)
               ? p.block_table[static_cast<long long>(seq) * p.bt_stride + wl + lane]
               : -1;
  };
  if (warp >= kCWarps) {
    if (spec && su1 > su0) {
      load_swin(sb0);
      load_bwin(sb0, static_cast<int>((su0 - spb0) * p.tc / p.block_size));
    }
    bool same = spec;
    if (spec) {
      int now[kChunks];
      load_lens(p, lane, now);
#pragma unroll
      for (int i = 0; i < kChunks; ++i)
        if (now[i] != raw[i]) same = false;
      same = __all_sync(0xffffffffu, same);
    }
    // Partition: this CTA's unit range and the sequence it starts in.
    const long long T = same ? sT : total_units(p, lane);
    const long long G = gridDim.x;
    const long long u0 = same ? su0 : cta_start(blockIdx.x, T, G);
    const long long u1 = same ? su1 : cta_start(blockIdx.x + 1, T, G);
    long long acc = 0;
    int b0 = same ? sb0 : p.batch;
    long long pb0 = same ? spb0 : T;
    if (!same && u1 > u0) {
      for (int base = 0; base < p.batch; base += 32) {
        const int b = base + lane;
        const int n = (b < p.batch) ? units_of(seq_ctx(p, b), p.tc) : 0;
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const long long end = acc + incl;  // cumulative end of sequence b
        const unsigned hit = __ballot_sync(0xffffffffu, b < p.batch && end > u0);
        if (hit) {
          const int src = __ffs(hit) - 1;
          const int incl_src = __shfl_sync(0xffffffffu, incl, src);
          const int n_src = __shfl_sync(0xffffffffu, n, src);
          b0 = base + src;
          pb0 = acc + incl_src - n_src;
          break;
        }
        acc += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (u1 > u0 && b0 < p.batch) {
        load_swin(b0);
        load_bwin(b0, static_cast<int>((u0 - pb0) * p.tc / p.block_size));
      }
    }
    if (warp == kCWarps && lane == 0) {
      sched[0] = u0;
      sched[1] = (u1 > u0) ? u1 : u0;
      sched[2] = b0;
      sched[3] = pb0;
    }
  }
  __syncthreads();
  // The next kernel (the combine pass) may start its launch now; it waits for
  // this grid's completion before reading the partials.
  grid_launch_dependents();

  const long long u0 = sched[0];
  const long long n_units = sched[1] - sched[0];
  const int hkv = p.hkv;

  if (warp >= kCWarps) {
    // ------------------------------------------------------------ producers
    // Producer pid issues units k = pid, pid + nprod, ...; every producer
    // walks every unit to follow the sequences. One warp's per-unit path
    // (stage wait, descriptor, four TMA boxes whose issue alone takes ~650
    // clocks) paced the pipeline when sequences are short; two alternate.
    const int pid = warp - kCWarps;
    const int nprod = static_cast<int>(blockDim.x >> 5) - kCWarps;
    const int nu = static_cast<int>(n_units);
    int b = static_cast<int>(sched[2]);
    int uis = static_cast<int>(u0 - sched[3]);  // unit of the current sequence at k
    int seq_k0 = -uis;                          // k of the current sequence's unit 0
    int ctx = (nu > 0) ? __shfl_sync(0xffffffffu, swin, 0) : 0;
    int nb = units_p(p, ctx);
    int nbb = -1, nbwin = -1;  // the next sequence's first block ids
    // This lane's warp slot (lanes 0..7): sub-chunk jl, kv head hl.
    const int jl = (lane < kCWarps) ? lane / hkv : 0;
    const int hl = (lane < kCWarps) ? lane - jl * hkv : 0;
    int k = 0;
    for (; k < nu; ++k, ++uis) {
      while (uis >= nb && b + 1 < p.batch) {
        ++b;
        uis = 0;
        seq_k0 = k;
        if (b - sb >= 32) load_swin(b);
        ctx = __shfl_sync(0xffffffffu, swin, b - sb);
        nb = units_p(p, ctx);
      }
      if (uis >= nb) break;  // seqlens changed under the kernel: stop issuing
      if (k % nprod != pid) continue;
      const int tok0 = uis * p.tc;
      {
        // Blocks of this unit's sub-chunks that hold keys: [lbf, lbl].
        const int lbf = div_bs(p, tok0);
        const int lbl = div_bs(p, min(tok0 + p.tc, ctx) - 1);
        if (bb != b || lbf < wl || lbl >= wl + 32) {
          if (b == nbb && lbf == 0 && lbl < 32) {
            bb = b;
            wl = 0;
            bwin = nbwin;
          } else {
            load_bwin(b, lbf);
          }
        }
        if (nbb <= b) {  // read at the next sequence change, not before
          nbb = b + 1;
          nbwin = (nbb < p.batch && lane < p.max_blocks)
                      ? p.block_table[static_cast<long long>(nbb) * p.bt_stride + lane]
                      : -1;
        }
      }
      const int s = k % kStages;
      const uint32_t ph = static_cast<uint32_t>((k / kStages) & 1);
      if (!mbar_wait(&empty[s], ph ^ 1u, p.err, LA_DEVERR_WAIT_TIMEOUT)) break;
      uint8_t* st = smem + s * p.stage_bytes;

      // Sub-chunk of warp-slot `lane` (lanes 0..7).
      bool active = false;
      int phys = -1, off = 0, head = 0, lb = 0;
      if (lane < kCWarps) {
        head = hl;
        const int t = tok0 + kSub * jl;
        if (t < ctx) {
          active = true;
          lb = div_bs(p, t);
          off = t - lb * p.block_size;
        }
      }
      // every lane takes part in the shuffle; inactive ones read lane 0
      const int id = __shfl_sync(0xffffffffu, bwin, active ? lb - wl : 0);
      if (active) {
        if (lb < p.max_blocks) {
          phys = id;
          // Out-of-pool ids are reported; TMA zero-fills the box for them.
          if ((phys < 0 || phys >= p.num_blocks) && p.err) atomicCAS(p.err, 0, LA_DEVERR_BLOCK_ID);
        } else if (p.err) {
          atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
        }
      }
      const unsigned act = __ballot_sync(0xffffffffu, active);
      if (lane == 0) {
        StageDesc d;
        d.b = b;
        d.tok0 = tok0;
        d.ctx = ctx;
        int flags = 0;
        if (k == 0 || uis == 0) flags |= kFlagFirst;
        if (k == nu - 1 || uis == nb - 1) flags |= kFlagLast;
        if (seq_k0 >= 0 && seq_k0 + nb <= nu) flags |= kFlagWhole;
        d.flags = flags;
        d.slot = 2 * static_cast<int>(blockIdx.x) + (seq_k0 <= 0 ? 0 : 1);
        descs[s] = d;
        // Q is read only on a sequence's first unit (kFlagFirst): load it there.
        const bool first = (flags & kFlagFirst) != 0;
        const bool whole_unit = tok0 + p.tc <= ctx;
        const uint32_t boxes =
            (p.unit_box && whole_unit) ? static_cast<uint32_t>(kCWarps) : static_cast<uint32_t>(__popc(act));
        const uint32_t bytes = boxes * (2 * kWarpBytes) + (first ? p.q_bytes : 0u);
        mbar_arrive_expect_tx(&full[s], bytes);
        if (first) {
          uint8_t* qs = st + 2 * kKVBytes;
          tma_load_3d(qs, &tm_q, &full[s], 0, 0, b);
          tma_load_3d(qs + p.q_half_bytes, &tm_q, &full[s], 64, 0, b);
        }
      }
      __syncwarp();
      if (phys < 0) phys = -1;  // outside the pool: TMA fills zeros
      // The four boxes of a sub-chunk (K and V, two 64-dim halves each) are
      // issued by four lanes in one instruction rather than one lane in four.
      const int piece = lane & 3;
      const int tens = piece >> 1, half = piece & 1;
      if (p.unit_box && tok0 + p.tc <= ctx) {
        // Lane 0's sub-chunk 0 starts the unit, inside one block.
        const int ph0 = __shfl_sync(0xffffffffu, phys, 0);
        const int grp = __shfl_sync(0xffffffffu, off, 0) / kSub;
        if (lane < 4)
          tma_load_5d(st + tens * kKVBytes + half * kKVHalf, tens ? &tm_v : &tm_k, &full[s], half * 64, 0, 0, grp,
                      ph0);
      } else if (p.unit_box) {
        // A sequence's last unit, not full: only the sub-chunks that hold
        // keys, one box [64 dims, 16 tokens, Hkv heads] per half per tensor
        // each (the whole-unit box would read up to 7/8 of a unit of rows
        // past ctx: 8.5 % more bytes at one kv head over U[512, 1024]).
        // Rows past ctx inside the last active sub-chunk are loaded and
        // masked by its consumers; sub-chunks past ctx are neither loaded
        // nor read.
        if (active && head == 0) {
          const int grp = off / kSub;
          uint8_t* kd = st + lane * kTileBytes;
          uint8_t* vd = st + kKVBytes + lane * kTileBytes;
          tma_load_5d(kd, &tm_k1, &full[s], 0, 0, 0, grp, phys);
          tma_load_5d(kd + kKVHalf, &tm_k1, &full[s], 64, 0, 0, grp, phys);
          tma_load_5d(vd, &tm_v1, &full[s], 0, 0, 0, grp, phys);
          tma_load_5d(vd + kKVHalf, &tm_v1, &full[s], 64, 0, 0, grp, phys);
        }
      } else if (p.big_box) {
        // Sub-chunk j (all kv heads in one box per half, the lane of its head
        // 0 holding id and offset) is issued by lanes 4j .. 4j + 3.
        const int jj = lane >> 2;
        const int src = (jj < p.nsub ? jj : 0) * hkv;
        const int sph = __shfl_sync(0xffffffffu, phys, src);
        const int sof = __shfl_sync(0xffffffffu, off, src);
        const bool sact = __shfl_sync(0xffffffffu, active ? 1 : 0, src) != 0;
        if (jj < p.nsub && sact)
          tma_load_4d(st + tens * kKVBytes + half * kKVHalf + src * kTileBytes, tens ? &tm_v : &tm_k, &full[s],
                      half * 64, sof, 0, sph);
      } else if (active) {
        uint8_t* kd = st + lane * kTileBytes;
        uint8_t* vd = st + kKVBytes + lane * kTileBytes;
        tma_load_4d(kd, &tm_k, &full[s], 0, head, off, phys);
        tma_load_4d(kd + kKVHalf, &tm_k, &full[s], 64, head, off, phys);
        tma_load_4d(vd, &tm_v, &full[s], 0, head, off, phys);
        tma_load_4d(vd + kKVHalf, &tm_v, &full[s], 64, head, off, phys);
      }
    }
    // On an early exit, let the copies this warp issued land before the CTA
    // releases its shared memory (bounded).
    if (k < nu) {
      for (int kk = (k > kStages ? k - kStages : 0); kk < k; ++kk)
        if (kk % nprod == pid) mbar_wait(&full[kk % kStages], static_cast<uint32_t>((kk / kStages) & 1), nullptr, 0);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int w = warp;
  const int j = w / hkv;
  const int h = w - j * hkv;
  const int G = p.group;
  const int g = lane >> 2;
  const int tq = lane & 3;
  const float sl2 = p.scale_log2;
  const float NEG_INF = -__int_as_float(0x7f800000);

  float o[8][4];
  float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;
  uint32_t qf[8][2];
  int seg_ends = 0;  // segment ends seen (phase of the merge barriers)

  const int nu = static_cast<int>(n_units);
  for (int k = 0; k < nu; ++k) {
    const int s = k % kStages;
    const uint32_t ph = static_cast<uint32_t>((k / kStages) & 1);
    if (!mbar_wait(&full[s], ph, p.err, LA_DEVERR_WAIT_TIMEOUT)) return;
    const StageDesc d = descs[s];
    uint8_t* st = smem + s * p.stage_bytes;

    if (d.flags & kFlagFirst) {
      m0 = m1 = NEG_INF;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      // Q^T B-fragments for the 8 k-steps (128 dims); rows n >= G read zeros.
      const uint8_t* qs = st + 2 * kKVBytes;
      const int n = lane & 7;
      const int mq = lane >> 3;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int chunk_all = 4 * kk + mq;  // 16-byte chunk index over 128 dims
        const int half = chunk_all >> 3;
        const int chunk = chunk_all & 7;
        uint32_t addr;
        if (n < G) {
          const int row = h * G + n;
          addr = smem_u32(qs + half * p.q_half_bytes) + swz128(row, chunk);
        } else {
          addr = smem_u32(zero_row);
        }
        uint32_t r[4];
        ldmatrix_x4(r, addr);
        qf[2 * kk][0] = r[0];
        qf[2 * kk][1] = r[1];
        qf[2 * kk + 1][0] = r[2];
        qf[2 * kk + 1][1] = r[3];
      }
    }

    const int t0 = d.tok0 + kSub * j;
    int valid = d.ctx - t0;
    valid = valid < 0 ? 0 : (valid > kSub ? kSub : valid);
    if (valid > 0) {
      const uint8_t* ks = st + w * kTileBytes;  // + half * kKVHalf
      uint8_t* vs = st + kKVBytes + w * kTileBytes;
      // S^T = K Q^T (16 tokens x 8 query columns)
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int mq = lane >> 3;
        const int r = (lane & 7) + ((mq & 1) << 3);
        const uint32_t kbase = smem_u32(ks);
#pragma unroll
        for (int kstep = 0; kstep < 8; ++kstep) {
          const int half = kstep >> 2;
          const int chunk = ((kstep & 3) << 1) + (mq >> 1);
          uint32_t a[4];
          ldmatrix_x4(a, kbase + half * kKVHalf + swz128(r, chunk));
          mma_bf16_16816(sacc, a, qf[kstep][0], qf[kstep][1]);
        }
      }
      // Mask, online softmax (columns 2tq, 2tq+1; tokens g, g+8).
      const bool v0 = g < valid, v1 = (g + 8) < valid;
      const float x0 = v0 ? sacc[0] * sl2 : NEG_INF;
      const float x1 = v0 ? sacc[1] * sl2 : NEG_INF;
      const float x2 = v1 ? sacc[2] * sl2 : NEG_INF;
      const float x3 = v1 ? sacc[3] * sl2 : NEG_INF;
      const float mn0 = fmaxf(m0, warp_max_g(fmaxf(x0, x2)));
      const float mn1 = fmaxf(m1, warp_max_g(fmaxf(x1, x3)));
      const float a0 = ex2(m0 - mn0), a1 = ex2(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      const float p0 = ex2(x0 - mn0), p1 = ex2(x1 - mn1), p2 = ex2(x2 - mn0), p3 = ex2(x3 - mn1);
      l0 = l0 * a0 + (p0 + p2);
      l1 = l1 * a1 + (p1 + p3);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= a0;
        o[mt][1] *= a1;
        o[mt][2] *= a0;
        o[mt][3] *= a1;
      }
      const uint32_t pb0 = movmatrix_trans(pack_bf16x2(p0, p1));
      const uint32_t pb1 = movmatrix_trans(pack_bf16x2(p2, p3));
      if (valid < kSub) {
        // Rows past the sequence end may hold anything (even NaN): zero them so
        // that P = 0 cannot meet a non-finite V in the MMA.
        for (int i = lane; i < (kSub - valid) * 16; i += 32) {
          const int row = valid + (i >> 4);
          const int half = (i >> 3) & 1;
          const int chunk = i & 7;
          *reinterpret_cast<uint4*>(vs + half * kKVHalf + row * 128 + chunk * 16) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      // O^T += V^T P^T
      {
        const int mq = lane >> 3;
        const int r = (lane & 7) + ((mq >> 1) << 3);  // token row
        const uint32_t vbase = smem_u32(vs);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int dd = mt * 16 + ((mq & 1) << 3);
          const int half = dd >> 6;
          const int chunk = (dd & 63) >> 3;
          uint32_t a[4];
          ldmatrix_x4_trans(a, vbase + half * kKVHalf + swz128(r, chunk));
          mma_bf16_16816(o[mt], a, pb0, pb1);
        }
      }
      if (valid < kSub) fence_proxy_async_smem();  // generic writes before the next TMA into this stage
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (d.flags & kFlagLast) {
      float L0 = warp_sum_g(l0), L1 = warp_sum_g(l1);
      const int c0 = 2 * tq, c1 = 2 * tq + 1;
      bool writer = true;
      if (p.nsub > 1) {
        // Several warps hold partial states of the same kv head (one per
        // sub-chunk j). They park them in shared memory and one of them
        // merges them, so every segment leaves one state per head, as with
        // nsub == 1. The merging warp rotates with the segment end (j =
        // seg_ends % nsub), so the merges of a CTA's many short sequences
        // (the KV-head-sharded rank crosses ~7 per CTA) are shared by the
        // warps instead of all landing on j = 0, whose lag held back every
        // stage's release. The merger folds the states in sub-chunk order
        // 0, 1, ..., nsub-1 whoever it is, so the result does not depend on
        // which warp merges.
        const int TQ = (G + 1) >> 1;  // lanes (per g) that hold real columns
        const uint32_t par = static_cast<uint32_t>(seg_ends & 1);
        const int jm = seg_ends & (p.nsub - 1);  // nsub is a power of two
        if (!mbar_wait(mg_empty, par ^ 1u, p.err, LA_DEVERR_WAIT_TIMEOUT)) return;
        if (tq < TQ) {
          float* slot = merge + ((w * TQ + tq) * 8 + g) * 36;
          slot[0] = m0;
          slot[1] = m1;
          slot[2] = L0;
          slot[3] = L1;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt)
#pragma unroll
            for (int r = 0; r < 4; ++r) slot[4 + mt * 4 + r] = o[mt][r];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(mg_full);
        writer = (j == jm);
        if (writer) {
          if (!mbar_wait(mg_full, par, p.err, LA_DEVERR_WAIT_TIMEOUT)) return;
          if (tq < TQ) {
            if (jm != 0) {  // start from sub-chunk 0's state (this warp's own is in its slot)
              const float* sl = merge + ((h * TQ + tq) * 8 + g) * 36;
              m0 = sl[0];
              m1 = sl[1];
              L0 = sl[2];
              L1 = sl[3];
#pragma unroll
              for (int mt = 0; mt < 8; ++mt)
#pragma unroll
                for (int r = 0; r < 4; ++r) o[mt][r] = sl[4 + mt * 4 + r];
            }
            for (int jj = 1; jj < p.nsub; ++jj) {
              const float* sl = merge + (((jj * hkv + h) * TQ + tq) * 8 + g) * 36;
              const float om0 = sl[0], om1 = sl[1], oL0 = sl[2], oL1 = sl[3];
              const float n0 = fmaxf(m0, om0), n1 = fmaxf(m1, om1);
              // a side with no keys (m = -inf) contributes nothing
              const float a0 = (m0 == NEG_INF) ? 0.f : ex2(m0 - n0), b0 = (om0 == NEG_INF) ? 0.f : ex2(om0 - n0);
              const float a1 = (m1 == NEG_INF) ? 0.f : ex2(m1 - n1), b1 = (om1 == NEG_INF) ? 0.f : ex2(om1 - n1);
#pragma unroll
              for (int mt = 0; mt < 8; ++mt) {
                o[mt][0] = o[mt][0] * a0 + sl[4 + mt * 4 + 0] * b0;
                o[mt][1] = o[mt][1] * a1 + sl[4 + mt * 4 + 1] * b1;
                o[mt][2] = o[mt][2] * a0 + sl[4 + mt * 4 + 2] * b0;
                o[mt][3] = o[mt][3] * a1 + sl[4 + mt * 4 + 3] * b1;
              }
              L0 = L0 * a0 + oL0 * b0;
              L1 = L1 * a1 + oL1 * b1;
              m0 = n0;
              m1 = n1;
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(mg_empty);
        }
        ++seg_ends;
      }
      if (writer && (d.flags & kFlagWhole)) {
        const float i0 = L0 > 0.f ? 1.f / L0 : 0.f;
        const float i1 = L1 > 0.f ? 1.f / L1 : 0.f;
        {
          __nv_bfloat16* ob = p.out + static_cast<long long>(d.b) * p.out_b_stride;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            const int d0 = mt * 16 + g;
            if (c0 < G) {
              __nv_bfloat16* oh = ob + static_cast<long long>(h * G + c0) * p.out_h_stride;
              oh[d0] = __float2bfloat16_rn(o[mt][0] * i0);
              oh[d0 + 8] = __float2bfloat16_rn(o[mt][2] * i0);
            }
            if (c1 < G) {
              __nv_bfloat16* oh = ob + static_cast<long long>(h * G + c1) * p.out_h_stride;
              oh[d0] = __float2bfloat16_rn(o[mt][1] * i1);
              oh[d0 + 8] = __float2bfloat16_rn(o[mt][3] * i1);
            }
          }
        }
        if (p.lse_out && g == 0) {
          const float ln2 = 0.6931471805599453f;
          if (c0 < G) p.lse_out[static_cast<long long>(d.b) * p.hq + h * G + c0] = L0 > 0.f ? (m0 + __log2f(L0)) * ln2 : NEG_INF;
          if (c1 < G) p.lse_out[static_cast<long long>(d.b) * p.hq + h * G + c1] = L1 > 0.f ? (m1 + __log2f(L1)) * ln2 : NEG_INF;
        }
      } else if (writer) {
        float* po = p.part_o + static_cast<long long>(d.slot) * p.hq * kD;
        const float i0 = L0 > 0.f ? 1.f / L0 : 0.f;
        const float i1 = L1 > 0.f ? 1.f / L1 : 0.f;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + g;
          if (c0 < G) {
            float* oh = po + (h * G + c0) * kD;
            oh[d0] = o[mt][0] * i0;
            oh[d0 + 8] = o[mt][2] * i0;
          }
          if (c1 < G) {
            float* oh = po + (h * G + c1) * kD;
            oh[d0] = o[mt][1] * i1;
            oh[d0 + 8] = o[mt][3] * i1;
          }
        }
        if (g == 0) {
          float* pl = p.part_lse + static_cast<long long>(d.slot) * p.hq;
          if (c0 < G) pl[h * G + c0] = L0 > 0.f ? m0 + __log2f(L0) : NEG_INF;
          if (c1 < G) pl[h * G + c1] = L1 > 0.f ? m1 + __log2f(L1) : NEG_INF;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ combine
// Grid (batch, Hq / warps per CTA), one warp per (sequence, query head) (a
// CTA is one warp, or up to kCombinePeerWarps with peer stores); lane l owns
// dims 4l..4l+3. Sequences whose key range lies inside one CTA's range were
// written directly by the decode kernel and are skipped. Rows over a few
// CTAs (at most kCombineFew) merge their slots one after another. The others
// merge their partials: up to 32 slots per round, one per lane (each lane finds
// its CTA's slot with its own two divisions and loads that slot's lse, so a
// round costs one division latency whatever the slot count); the round's
// max and weight sum are warp reductions, then the O rows are read 8 at a
// time with independent loads.
constexpr int kCombineBatch = 8;
constexpr int kCombineFew = 4;  // rows over at most this many CTAs take the sequential merge

__device__ __forceinline__ float warp_max_all(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_all(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// With peer stores (the KV-head-sharded all-gather) a CTA holds kCombinePeerWarps
// warps, one query head each, so that it ends with one system-scope fence for
// all of them: one fence per one-warp CTA, 2048 of them at 256 rows x 8 heads,
// cost 6.4 us per layer on one GPU. Otherwise a CTA is one warp.
constexpr int kCombinePeerWarps = 4;

// kMany: the instance for small batches, whose rows are split over many
// CTAs (one round of up to 32 slots): the round's first kManyBatch O rows
// are loaded together with its lse values, so a row over up to 16 CTAs is
// merged after one load round trip (the general path loads the lse, then the
// O rows of the slots that hold keys 8 at a time: four dependent round trips
// for a row over 18 CTAs). Slots are read whether or not they hold keys;
// those without are skipped by a warp-uniform test, never weighted by zero,
// so whatever they hold does not reach the sum.
constexpr int kManyBatch = 16;

template <bool kMany>
__global__ void __launch_bounds__(32 * kCombinePeerWarps, 1) paged_decode_combine_kernel(const Params p, int grid) {
  const int b = blockIdx.x;
  const int hh = blockIdx.y * static_cast<int>(blockDim.x >> 5) + static_cast<int>(threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const float NEG_INF = -__int_as_float(0x7f800000);

  // T (all units) and P_b (units before sequence b). They depend only on
  // cache_seqlens, which were final before the decode grid started (it does
  // not write them), so they are computed while that grid still runs; every
  // CTA waits for it before touching outputs or partials. Each lane sums its
  // own sequences (lane + 32 i, coalesced, 16 independent loads at a time)
  // and two warp sums finish: a round trip per 512 sequences. (A warp sum
  // after every 32 sequences, one round trip each, took ~15 us at 1024
  // sequences, and the combine CTAs that launch only as decode CTAs leave
  // run it after the decode grid.)
  long long T = 0, Pb = 0;
  {
    constexpr int kLoads = 16;
    int own = 0, before = 0;
    for (int base = 0; base < p.batch; base += 32 * kLoads) {
      int n[kLoads];
#pragma unroll
      for (int k = 0; k < kLoads; ++k) {
        const int bb = base + 32 * k + lane;
        n[k] = (bb < p.batch) ? units_of(seq_ctx(p, bb), p.tc) : 0;
      }
#pragma unroll
      for (int k = 0; k < kLoads; ++k) {
        own += n[k];
        if (base + 32 * k + lane < b) before += n[k];
      }
    }
    long long o = own, bf = before;
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) {
      o += __shfl_xor_sync(0xffffffffu, o, x);
      bf += __shfl_xor_sync(0xffffffffu, bf, x);
    }
    T = o;
    Pb = bf;
  }
  const int nb = units_of(seq_ctx(p, b), p.tc);
  const long long Gl = grid;
  const long long oofs = static_cast<long long>(b) * p.out_b_stride + static_cast<long long>(hh) * p.out_h_stride +
                         lane * 4;
  float* lse = p.lse_out ? p.lse_out + static_cast<long long>(b) * p.hq + hh : nullptr;
  // The row's CTAs cf..cl and the partial slots they wrote, also from the
  // lengths alone (64-bit divisions), so after the wait only the loads and
  // the merge remain: for rows over a few CTAs every slot, for the others
  // this lane's slot of the first round of 32 (-1: no slot, or an empty
  // range, T < G, that wrote nothing).
  const long long cf = nb > 0 ? cta_of(Pb, T, Gl) : 0;
  const long long cl = nb > 0 ? cta_of(Pb + nb - 1, T, Gl) : -1;
  auto slot_of = [&](long long c) -> int {
    const long long s0 = cta_start(c, T, Gl);
    return s0 != cta_start(c + 1, T, Gl) ? 2 * static_cast<int>(c) + (s0 >= Pb ? 0 : 1) : -1;
  };
  int few[kCombineFew];
#pragma unroll
  for (int u = 0; u < kCombineFew; ++u)
    few[u] = (cf < cl && cl - cf < kCombineFew && cf + u <= cl) ? slot_of(cf + u) : -1;
  const int first_round = (cl - cf >= kCombineFew && cf + lane <= cl) ? slot_of(cf + lane) : -1;
  grid_dependency_wait();

  if (nb == 0) {
    for (int r = 0; r < p.nouts; ++r) *reinterpret_cast<uint2*>(p.outs[r] + oofs) = make_uint2(0u, 0u);
    if (lse && lane == 0) *lse = NEG_INF;
  } else {
    if (cf == cl) {  // written by the decode pass; forward it to the peers
      if (p.peer_stores) {
        const uint2 v = *reinterpret_cast<const uint2*>(p.out + oofs);
        for (int r = 0; r < p.nouts; ++r)
          if (p.outs[r] != p.out) *reinterpret_cast<uint2*>(p.outs[r] + oofs) = v;
      }
    } else if (cl - cf < kCombineFew) {
      // A few slots (rows split across two to four CTAs, the usual case at
      // large batches): merge them one after another, all loads issued first.
      float m = NEG_INF, l = 0.f;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      float ls[kCombineFew];
      float4 ov[kCombineFew];
#pragma unroll
      for (int u = 0; u < kCombineFew; ++u) {
        ls[u] = NEG_INF;
        if (few[u] >= 0) {
          const long long slot = few[u];
          ls[u] = p.part_lse[slot * p.hq + hh];
          ov[u] = *reinterpret_cast<const float4*>(p.part_o + (slot * p.hq + hh) * kD + lane * 4);
        }
      }
#pragma unroll
      for (int u = 0; u < kCombineFew; ++u) {
        if (ls[u] != NEG_INF) {
          const float mn = fmaxf(m, ls[u]);
          const float a = ex2(m - mn), w = ex2(ls[u] - mn);
          acc[0] = acc[0] * a + w * ov[u].x;
          acc[1] = acc[1] * a + w * ov[u].y;
          acc[2] = acc[2] * a + w * ov[u].z;
          acc[3] = acc[3] * a + w * ov[u].w;
          l = l * a + w;
          m = mn;
        }
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint2 v;
      v.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      v.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      for (int r = 0; r < p.nouts; ++r) *reinterpret_cast<uint2*>(p.outs[r] + oofs) = v;
      if (lse && lane == 0) *lse = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : NEG_INF;
    } else if constexpr (kMany) {
      float m = NEG_INF, l = 0.f;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (long long c0 = cf; c0 <= cl; c0 += 32) {
        const long long c = c0 + lane;
        const int slot = c0 == cf ? first_round : (c <= cl ? slot_of(c) : -1);
        const int nr = static_cast<int>(cl - c0 + 1 < 32 ? cl - c0 + 1 : 32);  // lanes of this round
        const float ls = slot >= 0 ? p.part_lse[static_cast<long long>(slot) * p.hq + hh] : NEG_INF;
        int su[kManyBatch];
        float4 ov[kManyBatch];
#pragma unroll
        for (int k = 0; k < kManyBatch; ++k) su[k] = __shfl_sync(0xffffffffu, slot, k);
#pragma unroll
        for (int k = 0; k < kManyBatch; ++k)
          ov[k] = (k < nr && su[k] >= 0) ? *reinterpret_cast<const float4*>(
                                               p.part_o + (static_cast<long long>(su[k]) * p.hq + hh) * kD + lane * 4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        const float mr = warp_max_all(ls);
        if (mr == NEG_INF) continue;  // warp-uniform: no keys in this round
        const float mn = fmaxf(m, mr);
        const float a = ex2(m - mn);  // 0 while m is -inf
        const bool use = slot >= 0 && ls != NEG_INF;
        const float wl = use ? ex2(ls - mn) : 0.f;
        l = l * a + warp_sum_all(wl);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] *= a;
        m = mn;
        const unsigned usem = __ballot_sync(0xffffffffu, use);
#pragma unroll
        for (int k = 0; k < kManyBatch; ++k) {
          const float w = __shfl_sync(0xffffffffu, wl, k);
          if ((usem >> k) & 1u) {
            acc[0] += w * ov[k].x;
            acc[1] += w * ov[k].y;
            acc[2] += w * ov[k].z;
            acc[3] += w * ov[k].w;
          }
        }
        for (int j0 = kManyBatch; j0 < nr; j0 += kManyBatch) {
#pragma unroll
          for (int k = 0; k < kManyBatch; ++k) su[k] = __shfl_sync(0xffffffffu, slot, (j0 + k) & 31);
#pragma unroll
          for (int k = 0; k < kManyBatch; ++k)
            ov[k] = (j0 + k < nr && ((usem >> ((j0 + k) & 31)) & 1u))
                        ? *reinterpret_cast<const float4*>(p.part_o + (static_cast<long long>(su[k]) * p.hq + hh) * kD +
                                                           lane * 4)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < kManyBatch; ++k) {
            const float w = __shfl_sync(0xffffffffu, wl, (j0 + k) & 31);
            if (j0 + k < nr && ((usem >> ((j0 + k) & 31)) & 1u)) {
              acc[0] += w * ov[k].x;
              acc[1] += w * ov[k].y;
              acc[2] += w * ov[k].z;
              acc[3] += w * ov[k].w;
            }
          }
        }
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint2 v;
      v.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      v.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      for (int r = 0; r < p.nouts; ++r) *reinterpret_cast<uint2*>(p.outs[r] + oofs) = v;
      if (lse && lane == 0) *lse = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : NEG_INF;
    } else {
      float m = NEG_INF, l = 0.f;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (long long c0 = cf; c0 <= cl; c0 += 32) {
        const long long c = c0 + lane;
        const int slot = c0 == cf ? first_round : (c <= cl ? slot_of(c) : -1);
        const float ls = slot >= 0 ? p.part_lse[static_cast<long long>(slot) * p.hq + hh] : NEG_INF;
        const float mr = warp_max_all(ls);
        if (mr == NEG_INF) continue;  // warp-uniform: no keys in this round
        const float mn = fmaxf(m, mr);
        const float a = ex2(m - mn);  // 0 while m is -inf
        const bool use = slot >= 0 && ls != NEG_INF;
        const float wl = use ? ex2(ls - mn) : 0.f;
        l = l * a + warp_sum_all(wl);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] *= a;
        m = mn;
        unsigned todo = __ballot_sync(0xffffffffu, use);
        while (todo) {
          int su[kCombineBatch];
          float wu[kCombineBatch];
#pragma unroll
          for (int k = 0; k < kCombineBatch; ++k) {
            const int u = todo ? __ffs(todo) - 1 : 0;
            const bool have = todo != 0;
            todo &= todo - 1u;
            const int sv = __shfl_sync(0xffffffffu, slot, u);
            const float wv = __shfl_sync(0xffffffffu, wl, u);
            su[k] = have ? sv : -1;
            wu[k] = have ? wv : 0.f;
          }
          float4 ov[kCombineBatch];
#pragma unroll
          for (int k = 0; k < kCombineBatch; ++k)
            ov[k] = su[k] >= 0 ? *reinterpret_cast<const float4*>(
                                     p.part_o + (static_cast<long long>(su[k]) * p.hq + hh) * kD + lane * 4)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < kCombineBatch; ++k) {
            if (su[k] >= 0) {
              acc[0] += wu[k] * ov[k].x;
              acc[1] += wu[k] * ov[k].y;
              acc[2] += wu[k] * ov[k].z;
              acc[3] += wu[k] * ov[k].w;
            }
          }
        }
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint2 v;
      v.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      v.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      for (int r = 0; r < p.nouts; ++r) *reinterpret_cast<uint2*>(p.outs[r] + oofs) = v;
      if (lse && lane == 0) *lse = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : NEG_INF;
    }
  }
  if (p.peer_stores) {
    // One system-scope fence per CTA: __syncthreads orders every thread's
    // peer stores before thread 0's fence, which is cumulative over them, so
    // the epoch the barrier kernel publishes next on this stream (a release
    // at system scope, after this grid completes) orders after all of them.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
  }
}

// ------------------------------------------------------------------ host
static int stages_for(int q_area_bytes, int merge_bytes, int* stage_bytes, size_t* smem) {
  const int sb = 2 * kKVBytes + q_area_bytes;
  *stage_bytes = sb;
  const size_t ctrl = 1024 + merge_bytes;
  const size_t limit = 227 * 1024;
  for (int st = 3; st >= 2; --st) {
    const size_t need = 1024 /*align slack*/ + static_cast<size_t>(st) * sb + ctrl;
    if (need <= limit) {
      *smem = need;
      return st;
    }
  }
  return 0;
}

static int grid_for(int device) { return num_sms(device); }

}  // namespace decode

int decode_init(int device) {
  (void)device;
  const int lim = 227 * 1024;
  cudaError_t e = cudaFuncSetAttribute(decode::paged_decode_kernel<3, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode::paged_decode_kernel<2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode::paged_decode_kernel<3, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode::paged_decode_kernel<2, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  if (e == cudaSuccess) {
    cudaFuncAttributes a;
    e = cudaFuncGetAttributes(&a, decode::paged_decode_combine_kernel<false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, decode::paged_decode_combine_kernel<true>);
  }
  return cuda_status(e);
}

}  // namespace la

extern "C" int la_paged_decode_workspace_size(int device, int num_q_heads, int num_kv_heads, int head_dim,
                                              size_t* bytes) {
  if (!bytes || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim != 128 || num_kv_heads > 8 ||
      8 % num_kv_heads != 0)
    return LA_ERR_INVALID_ARGUMENT;
  const int grid = la::decode::grid_for(device);
  if (grid <= 0) return LA_ERR_CUDA;
  const size_t slots = static_cast<size_t>(2) * grid;
  const size_t o_bytes = slots * num_q_heads * head_dim * sizeof(float);
  const size_t l_bytes = slots * num_q_heads * sizeof(float);
  *bytes = ((o_bytes + 255) & ~size_t(255)) + ((l_bytes + 255) & ~size_t(255));
  return LA_OK;
}

namespace la {
namespace decode {

// Peer outputs of the KV-head-sharded all-gather (nullptr: local output only).
struct PeerOut {
  void* const* outs;  // [npeers] gather buffers, rank order (own included)
  int npeers;
};

static int paged_decode_impl(const void* q, int64_t q_batch_stride, int64_t q_head_stride, const void* k_cache,
                             const void* v_cache, int64_t kv_block_stride, int64_t kv_token_stride,
                             int64_t kv_head_stride, int64_t num_blocks, int block_size,
                             const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
                             const int32_t* cache_seqlens, int batch, int num_q_heads, int num_kv_heads,
                             int head_dim, float softmax_scale, void* out, int64_t out_batch_stride,
                             int64_t out_head_stride, float* softmax_lse, void* workspace, size_t workspace_bytes,
                             int* dev_error, cudaStream_t stream, const PeerOut* peers) {
  if (!q || !k_cache || !v_cache || !block_table || !cache_seqlens || !out) return LA_ERR_INVALID_ARGUMENT;
  if (batch < 0 || num_blocks <= 0 || block_size <= 0 || max_blocks_per_seq <= 0) return LA_ERR_INVALID_ARGUMENT;
  if (batch == 0) return LA_OK;
  if (head_dim != kD) return LA_ERR_UNSUPPORTED;
  if (num_kv_heads <= 0 || num_kv_heads > 8 || 8 % num_kv_heads != 0) return LA_ERR_UNSUPPORTED;
  if (num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return LA_ERR_INVALID_ARGUMENT;
  const int group = num_q_heads / num_kv_heads;
  if (group > 8 || num_q_heads > 256) return LA_ERR_UNSUPPORTED;
  if (block_size % kSub != 0) return LA_ERR_UNSUPPORTED;
  if (!(softmax_scale > 0.f)) return LA_ERR_INVALID_ARGUMENT;
  // TMA: 16-byte aligned bases and byte strides.
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16)) return LA_ERR_ALIGNMENT;
  if ((q_batch_stride * 2) % 16 || (q_head_stride * 2) % 16 || (kv_block_stride * 2) % 16 ||
      (kv_token_stride * 2) % 16 || (kv_head_stride * 2) % 16)
    return LA_ERR_ALIGNMENT;
  if (q_batch_stride <= 0 || q_head_stride <= 0 || kv_block_stride <= 0 || kv_token_stride <= 0 ||
      kv_head_stride <= 0 || out_batch_stride <= 0 || out_head_stride <= 0)
    return LA_ERR_INVALID_ARGUMENT;
  // the combine pass stores 4 bf16 per lane
  if (!aligned(out, 8) || out_batch_stride % 4 || out_head_stride % 4) return LA_ERR_ALIGNMENT;

  const int device = current_device();
  if (device < 0) return LA_ERR_CUDA;
  const int grid = grid_for(device);
  if (grid <= 0) return LA_ERR_CUDA;
  size_t need = 0;
  int st = la_paged_decode_workspace_size(device, num_q_heads, num_kv_heads, head_dim, &need);
  if (st != LA_OK) return st;
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return LA_ERR_WORKSPACE;

  CUtensorMap tq, tk, tv, tk1, tv1;
  {
    const uint64_t dims[3] = {128, static_cast<uint64_t>(num_q_heads), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(q_head_stride) * 2, static_cast<uint64_t>(q_batch_stride) * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(num_q_heads), 1};
    if ((st = encode_tensor_map_bf16(&tq, q, 3, dims, strides, box, true)) != LA_OK) return st;
  }
  int big_box = 0;
  const int nsub = 8 / num_kv_heads;
  if (nsub >= 4 && block_size % (kSub * nsub) == 0) {
    // A whole unit (tc = 16 * nsub tokens of every kv head) per box: the
    // 16-token groups of a block as their own axis, after the heads, so the
    // box's rows come in the stage's order [group][head][token]. With one
    // kv head this replaces 32 boxes of 2 KB per stage by 4 of 16 KB (the
    // 8-GPU KV-head-sharded rank: 109 -> 89 us per layer at B = 1024), with
    // two 16 boxes of 4 KB (even); with four it measured slower than a box
    // per sub-chunk.
    const uint64_t dims[5] = {128, static_cast<uint64_t>(kSub), static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(block_size / kSub), static_cast<uint64_t>(num_blocks)};
    const uint64_t strides[4] = {static_cast<uint64_t>(kv_token_stride) * 2, static_cast<uint64_t>(kv_head_stride) * 2,
                                 static_cast<uint64_t>(kv_token_stride) * 2 * kSub,
                                 static_cast<uint64_t>(kv_block_stride) * 2};
    const uint32_t box[5] = {64, static_cast<uint32_t>(kSub), static_cast<uint32_t>(num_kv_heads),
                             static_cast<uint32_t>(nsub), 1};
    // The same layout with one 16-token group per box, for a sequence's
    // last unit when it is not full.
    const uint32_t box1[5] = {64, static_cast<uint32_t>(kSub), static_cast<uint32_t>(num_kv_heads), 1, 1};
    if (encode_tensor_map_bf16(&tk, k_cache, 5, dims, strides, box, true) == LA_OK &&
        encode_tensor_map_bf16(&tv, v_cache, 5, dims, strides, box, true) == LA_OK &&
        encode_tensor_map_bf16(&tk1, k_cache, 5, dims, strides, box1, true) == LA_OK &&
        encode_tensor_map_bf16(&tv1, v_cache, 5, dims, strides, box1, true) == LA_OK)
      big_box = 2;
  }
  if (!big_box) {
    // Token axis before the head axis, so one box covers all kv heads of 16
    // tokens (strides need not grow with the dimension index).
    const uint64_t dims[4] = {128, static_cast<uint64_t>(block_size), static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(kv_token_stride) * 2, static_cast<uint64_t>(kv_head_stride) * 2,
                                 static_cast<uint64_t>(kv_block_stride) * 2};
    const uint32_t box[4] = {64, static_cast<uint32_t>(kSub), static_cast<uint32_t>(num_kv_heads), 1};
    if (encode_tensor_map_bf16(&tk, k_cache, 4, dims, strides, box, true) == LA_OK &&
        encode_tensor_map_bf16(&tv, v_cache, 4, dims, strides, box, true) == LA_OK)
      big_box = 1;
  }
  if (!big_box) {
    const uint64_t dims[4] = {128, static_cast<uint64_t>(num_kv_heads), static_cast<uint64_t>(block_size),
                              static_cast<uint64_t>(num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(kv_head_stride) * 2, static_cast<uint64_t>(kv_token_stride) * 2,
                                 static_cast<uint64_t>(kv_block_stride) * 2};
    const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kSub), 1};
    if ((st = encode_tensor_map_bf16(&tk, k_cache, 4, dims, strides, box, true)) != LA_OK) return st;
    if ((st = encode_tensor_map_bf16(&tv, v_cache, 4, dims, strides, box, true)) != LA_OK) return st;
  }
  if (big_box != 2) {  // the one-group maps are read only with whole-unit boxes
    tk1 = tk;
    tv1 = tv;
  }

  Params p;
  p.seqlens = cache_seqlens;
  p.block_table = block_table;
  p.bt_stride = bt_seq_stride;
  p.max_blocks = max_blocks_per_seq;
  p.batch = batch;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = group;
  p.nsub = 8 / num_kv_heads;
  p.block_size = block_size;
  p.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(block_size)) : -1;
  p.num_blocks = num_blocks;
  p.tc = kSub * p.nsub;
  p.tc_shift = __builtin_ctz(static_cast<unsigned>(p.tc));
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_b_stride = out_batch_stride;
  p.out_h_stride = out_head_stride;
  p.nouts = 1;
  p.outs[0] = p.out;
  p.peer_stores = 0;
  if (peers) {
    if (peers->npeers < 1 || peers->npeers > kMaxPeers || !peers->outs) return LA_ERR_INVALID_ARGUMENT;
    p.nouts = peers->npeers;
    for (int r = 0; r < peers->npeers; ++r) {
      if (!peers->outs[r] || !aligned(peers->outs[r], 8)) return LA_ERR_INVALID_ARGUMENT;
      p.outs[r] = static_cast<__nv_bfloat16*>(peers->outs[r]);
    }
    p.peer_stores = 1;
  }
  p.lse_out = softmax_lse;
  const size_t slots = static_cast<size_t>(2) * grid;
  const size_t o_bytes = (slots * num_q_heads * kD * sizeof(float) + 255) & ~size_t(255);
  p.part_o = static_cast<float*>(workspace);
  p.part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + o_bytes);
  p.err = dev_error;
  // Each Q half tile starts on a 1024-byte boundary (the 128-byte swizzle atom).
  p.big_box = big_box == 1;
  p.unit_box = big_box == 2;
  p.q_half_bytes = (num_q_heads * 128 + 1023) & ~1023;
  p.q_bytes = 2 * num_q_heads * 128;
  size_t smem = 0;
  const int merge_bytes = (p.nsub > 1) ? kCWarps * ((group + 1) / 2) * 8 * 36 * 4 : 0;
  const int stages = stages_for(2 * p.q_half_bytes, merge_bytes, &p.stage_bytes, &smem);
  if (stages == 0) return LA_ERR_UNSUPPORTED;

  // A second producer warp pays off once units are many per CTA (at 1024
  // one-kv-head rows it took the pipeline off the producer's path); with a
  // few short sequences (B = 8) the extra warp measured slower.
  const int threads = (kCWarps + (batch >= 16 ? 2 : 1)) * 32;
  cudaError_t e;
  if (stages == 3)
    e = batch <= 256 ? launch_pdl(paged_decode_kernel<3, 8>, dim3(grid), dim3(threads), smem, stream, tq, tk, tv, tk1, tv1, p)
                     : launch_pdl(paged_decode_kernel<3, 32>, dim3(grid), dim3(threads), smem, stream, tq, tk, tv, tk1, tv1, p);
  else
    e = batch <= 256 ? launch_pdl(paged_decode_kernel<2, 8>, dim3(grid), dim3(threads), smem, stream, tq, tk, tv, tk1, tv1, p)
                     : launch_pdl(paged_decode_kernel<2, 32>, dim3(grid), dim3(threads), smem, stream, tq, tk, tv, tk1, tv1, p);
  if (e != cudaSuccess) return cuda_status(e);
  // peer stores: kCombinePeerWarps heads per CTA (fewer when they do not divide the heads)
  int wpc = 1;
  if (peers)
    for (int c = kCombinePeerWarps; c > 1; c >>= 1)
      if (num_q_heads % c == 0) {
        wpc = c;
        break;
      }
  // Rows over more than kCombineFew CTAs on average (batch * kCombineFew <
  // grid) take the many-slot instance.
  const dim3 cgrid(batch, num_q_heads / wpc), cblock(32 * wpc);
  e = static_cast<long long>(batch) * kCombineFew < grid
          ? launch_pdl(paged_decode_combine_kernel<true>, cgrid, cblock, 0, stream, p, grid)
          : launch_pdl(paged_decode_combine_kernel<false>, cgrid, cblock, 0, stream, p, grid);
  return cuda_status(e);
}

}  // namespace decode
}  // namespace la

extern "C" int la_paged_decode(const void* q, int64_t q_batch_stride, int64_t q_head_stride, const void* k_cache,
                               const void* v_cache, int64_t kv_block_stride, int64_t kv_token_stride,
                               int64_t kv_head_stride, int64_t num_blocks, int block_size,
                               const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
                               const int32_t* cache_seqlens, int batch, int num_q_heads, int num_kv_heads,
                               int head_dim, float softmax_scale, void* out, int64_t out_batch_stride,
                               int64_t out_head_stride, float* softmax_lse, void* workspace,
                               size_t workspace_bytes, int* dev_error, cudaStream_t stream) {
  return la::decode::paged_decode_impl(q, q_batch_stride, q_head_stride, k_cache, v_cache, kv_block_stride,
                                       kv_token_stride, kv_head_stride, num_blocks, block_size, block_table,
                                       bt_seq_stride, max_blocks_per_seq, cache_seqlens, batch, num_q_heads,
                                       num_kv_heads, head_dim, softmax_scale, out, out_batch_stride, out_head_stride,
                                       softmax_lse, workspace, workspace_bytes, dev_error, stream, nullptr);
}

extern "C" int la_paged_decode_allgather(
    const void* q, int64_t q_batch_stride, int64_t q_head_stride, const void* k_cache, const void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride, int64_t num_blocks, int block_size,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq, const int32_t* cache_seqlens,
    int batch, int num_q_heads, int num_kv_heads, int head_dim, float softmax_scale, void* const* gather_bufs,
    int64_t out_batch_stride, int64_t out_head_stride, int rank, int world, void* workspace,
    size_t workspace_bytes, int* dev_error, cudaStream_t stream) {
  if (!gather_bufs || world < 1 || world > la::decode::kMaxPeers || rank < 0 || rank >= world)
    return LA_ERR_INVALID_ARGUMENT;
  // This rank's query heads sit at [rank * Hq_local, (rank + 1) * Hq_local) of
  // every gather buffer.
  void* outs[la::decode::kMaxPeers];
  const int64_t head0 = static_cast<int64_t>(rank) * num_q_heads * out_head_stride;
  for (int r = 0; r < world; ++r) {
    if (!gather_bufs[r]) return LA_ERR_INVALID_ARGUMENT;
    outs[r] = static_cast<__nv_bfloat16*>(gather_bufs[r]) + head0;
  }
  la::decode::PeerOut peers{outs, world};
  return la::decode::paged_decode_impl(q, q_batch_stride, q_head_stride, k_cache, v_cache, kv_block_stride,
                                       kv_token_stride, kv_head_stride, num_blocks, block_size, block_table,
                                       bt_seq_stride, max_blocks_per_seq, cache_seqlens, batch, num_q_heads,
                                       num_kv_heads, head_dim, softmax_scale, outs[rank], out_batch_stride,
                                       out_head_stride, nullptr, workspace, workspace_bytes, dev_error, stream,
                                       &peers);
}
