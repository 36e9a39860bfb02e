// (c) Causal varlen prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA), sm_100a.
//
// Semantics: for every packed sequence s (queries cu_seqlens[s] ..
// cu_seqlens[s+1]-1) and query head h, softmax(scale * Q K^T) V over the keys of
// the same sequence and kv head h / G, causal — the reference's
// F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True) at
// leaninfer/qwen3/model.py:56-57, applied to many prompts at once (flash-attn
// varlen contract). With paged keys (la_prefill_paged) the keys come from the
// block-table pool and causal masking is bottom-right aligned (chunked
// prefill).
//
// One persistent CTA per SM. A work item is a pair of query tiles of the same
// (sequence, kv head): each tile is 128 rows = the tq = 128/G consecutive
// tokens of the G query heads that share the kv head (GQA packing), and the
// two tiles are consecutive in the sequence. Both tiles read the same K/V
// tiles of 128 keys, staged once by TMA in a 4-stage ring. TMEM (512 columns):
//   S0 [0,128)   S1 [128,256)   O0 [256,384)   O1 [384,512)
// Per KV tile j and tile i:
//   S_i  = Q_i K_j^T    tcgen05.mma M128 N128 K16 x8, fp32 into S_i
//   P_i  = exp2(S_i*scale*log2e - m)  by softmax warpgroup i (one thread per
//          row), written back as bf16 over the first 64 columns of S_i
//   O_i += P_i V_j      tcgen05.mma M128 N128 K16 x8, A = P_i from TMEM, B = V
//                       read MN-major from its TMA tile
// The MMA warp interleaves the two tiles (PV_0(j), S_0(j+1), PV_1(j),
// S_1(j+1)) so the tensor core computes one tile's products while the other
// tile's softmax runs. S_i(j+1) overwrites P_i(j); it is issued right behind
// PV_i(j), which the tensor core executes first, and when softmax i sees
// S_i(j+1), O_i is complete and can be rescaled in place. The row max is
// raised (and O, l rescaled) only when a tile's max exceeds the running one
// by more than 8 (log2 units), so most tiles skip the rescale.
//
// Warps (16): 0-3 softmax of tile 0, 4-7 softmax of tile 1 (for items of one
// query tile, both warpgroups work on tile 0: see kSplit), 8-11 epilogue
// (normalise O_i, store it through shared memory with coalesced rows, lse),
// 12 MMA issuer + TMEM owner, 13 TMA producer, 14-15 idle. Warp w reads TMEM
// lanes 32*(w%4)..+31. Registers are moved between warpgroups with
// setmaxnreg: the softmax warpgroups hold a 128-column S row per thread.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace prefill {

constexpr int kD = 128;
constexpr int kRows = 128;             // query rows per Q tile
constexpr int kKeys = 128;             // keys per KV tile
constexpr int kQHalf = kRows * 128;    // one 64-dim half of a Q tile: 128 rows x 128 B = 16 KB
constexpr int kQTile = 2 * kQHalf;     // 32 KB
constexpr int kKVHalf = kKeys * 128;   // one 64-dim half of a K or V tile: 16 KB
constexpr int kKVTile = 2 * kKVHalf;   // 32 KB
constexpr int kStages = 4;             // K/V ring (K(j) and V(j) take one stage each)
static_assert(kStages >= 4, "the split instance requests its first two K/V tiles into stages 0..3 at once");
constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;        // O_i at kColO + 128 i; S_i at 128 i
constexpr uint32_t kIdescQK = idesc_bf16_f32(128, kKeys, false, false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, false, true);
// Per-thread registers after the split (the launch gives 512 x 128).
constexpr int kRegSoftmax = 160, kRegEpilogue = 88, kRegOther = 104;
static_assert(256 * kRegSoftmax + 128 * kRegEpilogue + 128 * kRegOther <= kThreads * 128,
              "the register split must fit in the registers the CTA is launched with");
// setmaxnreg.inc may only raise and .dec only lower a warp's count (128 at
// launch); the other direction is an illegal instruction.
static_assert(kRegSoftmax >= 128 && kRegEpilogue <= 128 && kRegOther <= 128,
              "softmax warpgroups use setmaxnreg.inc, the others setmaxnreg.dec");
static_assert(kRegSoftmax % 8 == 0 && kRegEpilogue % 8 == 0 && kRegOther % 8 == 0 && kRegEpilogue >= 24 &&
                  kRegSoftmax <= 256,
              "setmaxnreg counts are multiples of 8 in [24, 256]");
// The split instance's softmax holds half an S row per thread: it gives 8
// registers per thread to the epilogue and the MMA/TMA warps (no spills).
constexpr int kRegSoftmaxSplit = 152, kRegEpilogueSplit = 104, kRegOtherSplit = 104;
static_assert(256 * kRegSoftmaxSplit + 128 * kRegEpilogueSplit + 128 * kRegOtherSplit <= kThreads * 128,
              "the register split must fit in the registers the CTA is launched with");
static_assert(kRegSoftmaxSplit >= 128 && kRegEpilogueSplit <= 128 && kRegOtherSplit <= 128,
              "softmax warpgroups use setmaxnreg.inc, the others setmaxnreg.dec");
static_assert(kRegSoftmaxSplit % 8 == 0 && kRegEpilogueSplit % 8 == 0 && kRegOtherSplit % 8 == 0,
              "setmaxnreg counts are multiples of 8");
// Shared memory: Q0 Q1 | K/V ring | O staging (4 KB per epilogue warp) |
// row statistics (l, m of both tiles) | barriers | softmax walk state | the
// split softmax's row maxima; base aligned to 1024 B (the 128-byte swizzle
// atom) at run time.
constexpr int kOffKV = 2 * kQTile;                         // 64 KB
constexpr int kOffStage = kOffKV + kStages * kKVTile;      // 192 KB
constexpr int kStageBytes = 32 * 128;                      // 32 rows x 64 dims bf16
constexpr int kOffStats = kOffStage + 4 * kStageBytes;     // 208 KB
constexpr int kOffBar = kOffStats + 2 * 2 * kRows * 4;     // + 2 KB
// After the barriers: per softmax warp its Walker + Item (128 B); the split
// instance has 256 B more of barriers and, after the walk state, its row
// maxima [step % 2][half][row].
template <bool kSplit>
__host__ __device__ constexpr int off_state() { return kOffBar + (kSplit ? 512 : 256); }
template <bool kSplit>
__host__ __device__ constexpr int off_xmax() { return off_state<kSplit>() + 8 * 128; }
// The split instance's item walk table: the total item count, then the
// query-tile levels of each sequence (uint16) for up to kMaxSeqs sequences.
// That instance runs only when the items do not fill the SMs (fewer than
// #SMs sequence x kv-head tiles), so 256 sequences cover it; more fall back
// to cu_seqlens. Kept small: shared memory taken here is L1 cache lost.
constexpr int kOffWalk = off_xmax<true>() + 2 * 2 * kRows * 4;
constexpr int kMaxSeqs = 256;
constexpr size_t kSmemBytes = kOffWalk + 16 + 2 * kMaxSeqs + 1024;  // + the run-time 1024-byte alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
// The split instance also keeps its first item (Walker at +0, Item at +32,
// found flag at +80) and a copy of cu_seqlens [kMaxSeqs + 1], read before its
// dependency wait and checked after it.
constexpr int kOffFirst = (kOffWalk + 16 + 2 * kMaxSeqs + 15) & ~15;
constexpr int kOffCu = kOffFirst + 96;
constexpr size_t kSmemBytesSplit = kOffCu + 4 * (kMaxSeqs + 1) + 1024;
static_assert(kSmemBytesSplit <= 227 * 1024, "shared memory per CTA (split instance)");

struct Params {
  const int* cu;  // query starts [num_seqs + 1], or null: sequence s has q_len queries from token s * q_len
  int q_len;
  int num_seqs;
  int n_qp;  // items (query-tile pairs, or single tiles) of the longest sequence
  int pair;  // query tiles per item: 2, or 1 when pairs would leave SMs idle
  int tq;    // tokens per query tile (128 / group)
  int tq_shift;  // log2(tq)
  int hq, hkv, group;
  int hkv_shift;  // log2(hkv) when hkv is a power of two, else -1
  int causal;
  float scale_log2;
  __nv_bfloat16* out;
  long long out_ts, out_hs;
  float* lse;  // [hq, total] natural log, or null
  long long total;
  int* err;
  // Keys. Contiguous (paged == 0): the sequence's own tokens, at the same
  // packed rows as its queries. Paged: k_lens[s] keys of sequence s in the
  // pool [num_blocks, bs, hkv, D] through block-table row s; causal masking
  // is then bottom-right aligned (query i sees key j iff
  // j <= i + k_lens[s] - q_count).
  int paged;
  const int* k_lens;
  const int* bt;
  long long bt_stride;
  int max_blocks;
  int bs;         // block size
  int box_keys;   // keys per TMA box: min(bs, kKeys)
  int num_blocks;
};

// K-major operand of 128-byte SW128 rows whose 128-wide reduction dimension is
// split into two 64-wide halves `half_bytes` apart: k-step ks covers elements
// 16ks..16ks+15.
__device__ __forceinline__ uint64_t desc_kmajor(const uint8_t* tile, int half_bytes, int ks) {
  return smem_desc_sw128(smem_u32(tile) + (ks >> 2) * half_bytes + (ks & 3) * 32, 16, 1024);
}
// MN-major V tile (rows = keys, 128 B = 64 dims per half): k-step ks covers
// keys 16ks..16ks+15 = two 8-row groups (SBO 1024 B); the second 64-dim half
// is LBO = kKVHalf away.
__device__ __forceinline__ uint64_t desc_v(const uint8_t* tile, int ks) {
  return smem_desc_sw128(smem_u32(tile) + ks * 2048, kKVHalf, 1024);
}

template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Work items are (sequence, kv head, query-tile pair) in descending cost:
// pair level qp from the top down (a pair's KV length grows with qp), at each
// level only the sequences long enough to have that pair, then the kv heads.
// The valid items are ranked in that order and dealt to the G persistent CTAs
// as a snake over 2G columns (CTA c takes ranks c, 2G-1-c, 2G+c, 4G-1-c, ...),
// which evens out the summed cost per CTA. Every warp walks its CTA's item
// list itself (the walk is warp-collective), so no item descriptors are
// exchanged between roles.
struct Item {
  int s, h, q0, seq0, L;
  int K, off;       // keys of the sequence; causal offset K - L (0 for contiguous keys)
  int has1;         // the pair's second tile holds queries
  int n0, n1, n;    // KV tiles of tile 0, tile 1 (0 if absent), and their max
};

struct Walker {
  int taken;       // items this CTA has taken so far
  int level;       // current pair level
  long long base;  // rank of the first item of `level`
  int count;       // items at `level`
};

// kRo: read cu_seqlens through the read-only data cache (they are constant
// for the kernel's lifetime), where the few lines that every role of the
// pair instance walks at each item boundary stay resident; the split
// instance walks its shared-memory table and keeps plain loads.
template <bool kRo = false>
__device__ __forceinline__ int q_start(const Params& p, int s) {
  if (!p.cu) return s * p.q_len;
  return kRo ? __ldg(p.cu + s) : p.cu[s];
}
template <bool kRo = false>
__device__ __forceinline__ int q_count(const Params& p, int s) {
  if (!p.cu) return p.q_len;
  return kRo ? __ldg(p.cu + s + 1) - __ldg(p.cu + s) : p.cu[s + 1] - p.cu[s];
}

// The walk table, built once per CTA after the dependency wait: lv[s] = the
// number of levels of sequence s (its query tiles, or tile pairs, capped at
// n_qp), held in shared memory, so that level counts and the search for an
// item's sequence read shared memory rather than cu_seqlens in global memory
// (a dependent global round trip per level, which every role paid at each
// item boundary and, walking down every remaining level, at the end of the
// kernel); total = all items, so a walker past it stops at once. With more
// than kMaxSeqs sequences lv is null and the levels come from cu_seqlens.
// Laid out at kOffWalk of the CTA's shared memory: [0] total (int64), [8]
// lv cached (int32), [16] lv[kMaxSeqs] (uint16). Read through the shared
// memory base at each use, so nothing of it stays live in registers.
struct WalkTable {
  const uint8_t* smem;
  __device__ __forceinline__ long long total() const { return *reinterpret_cast<const long long*>(smem + kOffWalk); }
  __device__ __forceinline__ bool cached() const { return *reinterpret_cast<const int*>(smem + kOffWalk + 8) != 0; }
  __device__ __forceinline__ int lv(int s) const {
    return reinterpret_cast<const uint16_t*>(smem + kOffWalk + 16)[s];
  }
  // The split instance's copy of cu_seqlens (valid when cached()).
  __device__ __forceinline__ int cu(int s) const { return reinterpret_cast<const int*>(smem + kOffCu)[s]; }
};

__device__ __forceinline__ int levels_of(const Params& p, int s) {
  const int per = p.pair * p.tq;
  return min((q_count(p, s) + per - 1) / per, p.n_qp);
}

// kTable: levels from the shared-memory table (the split instance, whose
// CTAs hold one item each, most at high levels, so the walk down to the end
// dominated its tail); otherwise from cu_seqlens (the pair instance, whose
// hot loops measured slower with the table's code in the kernel).
template <bool kRo>
__device__ __forceinline__ bool seq_has_pair(const Params& p, int s, int q0) {
  return s < p.num_seqs && q_count<kRo>(p, s) > q0;
}

// Whether sequence s has an item at `level` (its query tiles, or pairs, reach it).
template <bool kTable>
__device__ __forceinline__ bool seq_at_level(const Params& p, const WalkTable& t, int s, int level) {
  if constexpr (kTable) {
    if (t.cached()) return s < p.num_seqs && static_cast<int>(t.lv(s)) > level;
  }
  return seq_has_pair<!kTable>(p, s, level * p.pair * p.tq);
}

// Items at one level (warp-collective).
template <bool kTable>
__device__ __forceinline__ int level_count(const Params& p, const WalkTable& t, int level) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int b = 0; b < p.num_seqs; b += 32)
    n += __popc(__ballot_sync(0xffffffffu, seq_at_level<kTable>(p, t, b + lane, level)));
  return n * p.hkv;
}

template <bool kTable>
__device__ __forceinline__ void walker_init(const Params& p, const WalkTable& t, Walker& w) {
  w.taken = 0;
  w.level = p.n_qp - 1;
  w.base = 0;
  w.count = level_count<kTable>(p, t, w.level);
}

// KV tiles a query tile starting at token q0 needs (at least one, so every
// item runs the same pipeline; rows that see no key come out as zeros).
__device__ __forceinline__ int kv_tiles(const Params& p, const Item& it, int q0) {
  const int kv_end = p.causal ? min(q0 + p.tq + it.off, it.K) : it.K;
  return max((kv_end + kKeys - 1) / kKeys, 1);
}

// Next item of this CTA (warp-collective; identical result in every lane).
template <bool kTable>
__device__ __forceinline__ bool walker_next(const Params& p, const WalkTable& t, Walker& w, Item& it) {
  const int lane = threadIdx.x & 31;
  const long long g2 = 2LL * gridDim.x;
  const long long r = static_cast<long long>(w.taken >> 1) * g2 +
                      ((w.taken & 1) ? (g2 - 1 - blockIdx.x) : static_cast<long long>(blockIdx.x));
  if constexpr (kTable) {
    if (r >= t.total()) return false;
  }
  while (r >= w.base + w.count) {
    if (w.level == 0) return false;
    w.base += w.count;
    --w.level;
    w.count = level_count<kTable>(p, t, w.level);
  }
  const int idx = static_cast<int>(r - w.base);
  // the ord-th sequence (index order) that has this level's pair
  const int ord = p.hkv_shift >= 0 ? (idx >> p.hkv_shift) : idx / p.hkv;
  const int q0 = w.level * p.pair * p.tq;
  int seen = 0, s = 0;
  for (int b = 0; b < p.num_seqs; b += 32) {
    const unsigned m = __ballot_sync(0xffffffffu, seq_at_level<kTable>(p, t, b + lane, w.level));
    const int c = __popc(m);
    if (ord < seen + c) {
      s = b + static_cast<int>(__fns(m, 0, ord - seen + 1));  // its (ord - seen + 1)-th set bit
      break;
    }
    seen += c;
  }
  it.s = s;
  it.h = idx - ord * p.hkv;
  if constexpr (kTable) {
    if (t.cached()) {
      it.seq0 = t.cu(s);
      it.L = t.cu(s + 1) - it.seq0;
    } else {
      it.seq0 = q_start<false>(p, s);
      it.L = q_count<false>(p, s);
    }
  } else {
    it.seq0 = q_start<true>(p, s);
    it.L = q_count<true>(p, s);
  }
  it.K = p.paged ? max(kTable ? p.k_lens[s] : __ldg(p.k_lens + s), 0) : it.L;
  it.off = it.K - it.L;
  it.q0 = q0;
  it.has1 = p.pair == 2 && it.L > q0 + p.tq;
  it.n0 = kv_tiles(p, it, q0);
  it.n1 = it.has1 ? kv_tiles(p, it, q0 + p.tq) : 0;
  it.n = max(it.n0, it.n1);
  ++w.taken;
  return true;
}

// A role's walker: the split instance's roles take their first item (and
// the walker state after it) from shared memory, where it was built before
// the dependency wait; later items, and every item of the pair instance, are
// walked by the role itself.
template <bool kSplit>
__device__ __forceinline__ void walker_start(const Params& p, const WalkTable& t, Walker& w) {
  if constexpr (kSplit)
    w.taken = 0;
  else
    walker_init<kSplit>(p, t, w);
}
template <bool kSplit>
__device__ __forceinline__ bool walker_step(const Params& p, const WalkTable& t, Walker& w, Item& it) {
  if constexpr (kSplit) {
    if (w.taken == 0) {
      // checked against cu_seqlens after the dependency wait (v_bar, at the
      // barrier area's word 41)
      uint64_t* v_bar = reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(t.smem) + kOffBar) + 41;
      if (!__all_sync(0xffffffffu, mbar_wait(v_bar, 0, p.err, LA_DEVERR_WAIT_TIMEOUT))) return false;
      w = *reinterpret_cast<const Walker*>(t.smem + kOffFirst);
      it = *reinterpret_cast<const Item*>(t.smem + kOffFirst + 32);
      return *reinterpret_cast<const int*>(t.smem + kOffFirst + 80) != 0;
    }
  }
  return walker_next<kSplit>(p, t, w, it);
}

// kSplit (items of single query tiles): both softmax warpgroups work on tile
// 0, warpgroup h on keys 64h..64h+63 of each 128-key tile, exchanging their
// row maxima through shared memory, so one tile's softmax takes half as long;
// and S is double buffered in the TMEM columns a second tile would use, so
// S(j+1) is computed while the softmax works on S(j) and the softmax runs
// from one KV tile to the next without waiting for the tensor core.
template <bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;            // Q0, Q1
  uint8_t* sKV = smem + kOffKV;  // ring
  float* stats = reinterpret_cast<float*>(smem + kOffStats);  // [tile][l | m][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;        // both Q tiles of an item landed
  uint64_t* q_empty = bars + 1;       // an item's last S issued and done
  uint64_t* kv_full = bars + 2;       // [kStages]
  uint64_t* kv_empty = bars + 6;      // [kStages]
  uint64_t* s_full = bars + 10;       // [2] S_i written
  uint64_t* s_free = bars + 12;       // [2] PV_i done: O_i complete
  uint64_t* p_full = bars + 14;       // [2] P_i written (128 arrivals)
  uint64_t* o_empty = bars + 16;      // [2] the epilogue has read O_i (128 arrivals)
  uint64_t* st_full = bars + 18;      // [2] row statistics of tile i written (128)
  uint64_t* st_empty = bars + 20;     // [2] ... read by the epilogue (128)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  // kSplit: the two softmax warpgroups may be one step apart (S is double
  // buffered), so their exchange and their P-ready arrivals alternate
  // between two barriers by step parity, [2 * (step % 2) + h] and
  // [2 * h + step % 2] (128 arrivals each).
  uint64_t* x_full = bars + 32;       // [4] warpgroup h's row maxima of a step written
  uint64_t* ph_full = bars + 36;      // [4] warpgroup h's half of P(step) written
  // kSplit: an item's last PV done. The softmax no longer waits for each PV
  // before the next S, so s_free may lag the epilogue by more than one phase
  // and its parity cannot name the item's last PV.
  uint64_t* o_full = bars + 40;
  // kSplit: the first item (built before the dependency wait) checked
  // against cu_seqlens read after it; every role waits here before using it.
  uint64_t* v_bar = bars + 41;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  const float NEG_INF = -__int_as_float(0x7f800000);

  // Barriers and TMEM: they read nothing that a previous kernel writes.
  auto setup = [&]() {
    if (threadIdx.x == 0) {
      mbar_init(q_full, 1);
      mbar_init(q_empty, 1);
      for (int i = 0; i < kStages; ++i) {
        mbar_init(&kv_full[i], 1);
        mbar_init(&kv_empty[i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&s_full[i], 1);
        mbar_init(&s_free[i], 1);
        mbar_init(&p_full[i], 128);
        mbar_init(&o_empty[i], 128);
        mbar_init(&st_full[i], kSplit && i == 0 ? 256 : 128);
        if (kSplit) {
          if (i == 0) {
            mbar_init(o_full, 1);
            mbar_init(v_bar, 1);
          }
          mbar_init(&x_full[i], 128);
          mbar_init(&x_full[i + 2], 128);
          mbar_init(&ph_full[i], 128);
          mbar_init(&ph_full[i + 2], 128);
        }
        mbar_init(&st_empty[i], 128);
      }
      fence_barrier_init();
    }
    if (warp == 12) {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  const WalkTable wt{smem};
  if constexpr (kSplit) {
    // The split instance (a grid of fewer CTAs than SMs) sets up before the
    // dependency wait, so with programmatic dependent launch that overlaps
    // the previous kernel's tail; once the previous kernel's memory is
    // visible it lets the next kernel launch: its CTAs take the idle SMs and
    // those this grid's CTAs leave, and wait for this grid's completion
    // before touching memory. (The pair instance, a full grid, measured
    // slower both ways.)
    setup();
    // The walk table and the CTA's first item are built before the
    // dependency wait, from cu_seqlens read through L2 only (so no stale line
    // stays in L1), while the previous kernel still runs: measured inside a
    // CUDA graph of one-prompt calls, building them after the wait (a cold
    // first pass through this code on every SM) took 3.3-4.5 us before the
    // first Q tile landed. After the wait cu_seqlens are read again; if any
    // value changed (the previous kernel wrote them), everything is rebuilt.
    // Paged keys (k_lens, maybe written by the previous kernel) and more
    // than kMaxSeqs sequences build after the wait.
    uint16_t* lv = reinterpret_cast<uint16_t*>(smem + kOffWalk + 16);
    long long* total = reinterpret_cast<long long*>(smem + kOffWalk);
    int* cuc = reinterpret_cast<int*>(smem + kOffCu);
    const bool cached = p.num_seqs <= kMaxSeqs && p.n_qp <= 65535;
    auto build = [&]() {
      if (threadIdx.x == 0) *reinterpret_cast<int*>(smem + kOffWalk + 8) = cached ? 1 : 0;
      if (cached) {
        for (int x = threadIdx.x; x <= p.num_seqs; x += kThreads) cuc[x] = p.cu ? __ldcg(p.cu + x) : x * p.q_len;
        __syncthreads();
        const int per = p.pair * p.tq;
        for (int x = threadIdx.x; x < p.num_seqs; x += kThreads)
          lv[x] = static_cast<uint16_t>(min((cuc[x + 1] - cuc[x] + per - 1) / per, p.n_qp));
      }
      __syncthreads();
      if (warp == 0) {
        long long tot = 0;
        for (int b = 0; b < p.num_seqs; b += 32) {
          int n = (b + lane < p.num_seqs) ? (cached ? static_cast<int>(lv[b + lane]) : levels_of(p, b + lane)) : 0;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
          tot += n;
        }
        if (lane == 0) *total = tot * p.hkv;
        __syncwarp();
        // the CTA's first item, for every role
        Walker w;
        walker_init<true>(p, wt, w);
        Item it;
        const bool have = walker_next<true>(p, wt, w, it);
        if (lane == 0) {
          *reinterpret_cast<Walker*>(smem + kOffFirst) = w;
          *reinterpret_cast<Item*>(smem + kOffFirst + 32) = it;
          *reinterpret_cast<int*>(smem + kOffFirst + 80) = have ? 1 : 0;
        }
      }
      __syncthreads();
    };
    const bool early = cached && !p.paged;
    if (early) {
      if (warp == 13 && lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
      }
      build();
    }
    // whether this CTA has no item, decided from the table every thread saw
    // (warp 14 may rewrite it after the wait)
    bool nowork = early && static_cast<long long>(blockIdx.x) >= wt.total();
    grid_dependency_wait();
    int* pre = reinterpret_cast<int*>(smem + kOffFirst + 84);  // Q and the first K/V tiles already issued
    if (early) {
      // The first item's Q and its first two K/V tiles (the whole 4-stage
      // ring) are requested right away. Warp 14 (idle otherwise) reads
      // cu_seqlens again while the roles start, and releases them through
      // v_bar: each role waits there before its first item. If a value
      // changed, warp 14 alone drains the early copies, initialises their
      // barriers again and rebuilds the table and the first item.
      const Item& f = *reinterpret_cast<const Item*>(smem + kOffFirst + 32);
      const bool have = *reinterpret_cast<const int*>(smem + kOffFirst + 80) != 0;
      if (warp == 13 && lane == 0) {
        *pre = have ? 1 : 0;
        if (have) {
          mbar_arrive_expect_tx(q_full, kQTile);
          for (int g = 0; g < p.group; ++g)
            for (int half = 0; half < 2; ++half)
              tma_load_3d(sQ + half * kQHalf + g * p.tq * 128, &tm_q, q_full, half * 64, f.h * p.group + g,
                          f.seq0 + f.q0);
          for (int x = 0; x < 2 * min(f.n, 2); ++x) {  // K(0), V(0), K(1), V(1): ring stage x
            mbar_arrive_expect_tx(&kv_full[x], kKVTile);
            for (int half = 0; half < 2; ++half)
              tma_load_3d(sKV + x * kKVTile + half * kKVHalf, (x & 1) ? &tm_v : &tm_k, &kv_full[x], half * 64, f.h,
                          f.seq0 + (x >> 1) * kKeys);
          }
        }
      }
      if (warp == 14) {
        bool changed = false;
        if (p.cu)
          for (int x = lane; x <= p.num_seqs; x += 32) changed |= __ldcg(p.cu + x) != cuc[x];
        if (__any_sync(0xffffffffu, changed)) {
          if (lane == 0 && have) {  // the copies warp 13 requested (it set *pre before them)
            const int nkv = 2 * min(f.n, 2);
            mbar_wait(q_full, 0, nullptr, 0);
            mbar_init(q_full, 1);
            for (int x = 0; x < nkv; ++x) {
              mbar_wait(&kv_full[x], 0, nullptr, 0);
              mbar_init(&kv_full[x], 1);
            }
            fence_barrier_init();
            *pre = 0;
          }
          __syncwarp();
          for (int x = lane; x <= p.num_seqs; x += 32) cuc[x] = p.cu ? __ldcg(p.cu + x) : x * p.q_len;
          __syncwarp();
          const int per = p.pair * p.tq;
          for (int x = lane; x < p.num_seqs; x += 32)
            lv[x] = static_cast<uint16_t>(min((cuc[x + 1] - cuc[x] + per - 1) / per, p.n_qp));
          __syncwarp();
          long long tot = 0;
          for (int b = 0; b < p.num_seqs; b += 32) {
            int n = (b + lane < p.num_seqs) ? static_cast<int>(lv[b + lane]) : 0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
            tot += n;
          }
          if (lane == 0) *total = tot * p.hkv;
          __syncwarp();
          Walker w;
          walker_init<true>(p, wt, w);
          Item it;
          const bool h2 = walker_next<true>(p, wt, w, it);
          if (lane == 0) {
            *reinterpret_cast<Walker*>(smem + kOffFirst) = w;
            *reinterpret_cast<Item*>(smem + kOffFirst + 32) = it;
            *reinterpret_cast<int*>(smem + kOffFirst + 80) = h2 ? 1 : 0;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(v_bar);  // release semantics: the writes above are visible to its waiters
      }
    } else {
      if (threadIdx.x == 0) *pre = 0;
      build();
      if (threadIdx.x == 0) mbar_arrive(v_bar);
      nowork = static_cast<long long>(blockIdx.x) >= wt.total();
    }
    grid_launch_dependents();
    // a CTA without work (its first item's rank is blockIdx.x) frees its
    // TMEM and leaves, once the item count is checked; a CTA that turns out
    // to have none after the check runs its roles, which find no item
    if (nowork) {
      mbar_wait(v_bar, 0, p.err, LA_DEVERR_WAIT_TIMEOUT);
      if (static_cast<long long>(blockIdx.x) >= wt.total()) {
        if (warp == 12) tmem_dealloc(*tmem_slot, kTmemCols);
        return;
      }
    }
  } else {
    grid_dependency_wait();
    // a CTA without work (no first item) leaves before touching barriers or TMEM
    Walker w;
    walker_init<false>(p, wt, w);
    Item it;
    if (!walker_next<false>(p, wt, w, it)) return;
    setup();
  }
  const uint32_t tmem = *tmem_slot;

  auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err, LA_DEVERR_WAIT_TIMEOUT));
  };

  if (wg < 2 && kSplit) {
    regs_inc<kSplit ? kRegSoftmaxSplit : kRegSoftmax>();
    // ------------------------------------------------- softmax of tile 0, keys 64h..64h+63
    const int h = wg;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    float* xmax = reinterpret_cast<float*>(smem + off_xmax<kSplit>());  // [step % 2][half][row]
    Walker& w = *reinterpret_cast<Walker*>(smem + off_state<kSplit>() + warp * 128);
    Item& it = *reinterpret_cast<Item*>(smem + off_state<kSplit>() + warp * 128 + 32);
    walker_start<kSplit>(p, wt, w);
    uint32_t t = 0;    // S_0 tiles seen
    uint32_t nst = 0;  // items whose statistics were written
    bool ok = true;
    while (ok && walker_step<kSplit>(p, wt, w, it)) {
      const int ni = it.n0;
      const int tok = it.q0 + (row & (p.tq - 1));
      const int lim = p.causal ? min(max(tok + 1 + it.off, 0), it.K) : it.K;
      float m = NEG_INF, l = 0.f;
      for (int j = 0; j < ni; ++j, ++t) {
        const uint32_t colS = (t & 1) * 128;  // S double buffer
        if (!(ok = wait_all(&s_full[t & 1], (t >> 1) & 1))) break;
        tc_fence_after();
        float sv[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_ld32(taddr + colS + h * 64 + c * 32, sv[c]);
        tc_wait_ld();
        const int nvis = lim - j * kKeys - h * 64;  // visible columns of this half
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = NEG_INF;
        const bool whole = __all_sync(0xffffffffu, nvis >= 64);
        if (whole) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2) mx[(e >> 1) & 7] = fmax3(mx[(e >> 1) & 7], sv[c][e], sv[c][e + 1]);
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float x0 = (c * 32 + e < nvis) ? sv[c][e] : NEG_INF;
              const float x1 = (c * 32 + e + 1 < nvis) ? sv[c][e + 1] : NEG_INF;
              sv[c][e] = x0;
              sv[c][e + 1] = x1;
              mx[(e >> 1) & 7] = fmax3(mx[(e >> 1) & 7], x0, x1);
            }
        }
        const float mh = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7]));
        // Exchange the halves' maxima. Both halves' S loads have completed
        // once the other warpgroup's arrival is seen, so warpgroup 1 may then
        // write its P over S columns 32-63 (keys 32-63 of warpgroup 0).
        const uint32_t sb = t & 1;
        xmax[(sb * 2 + h) * kRows + row] = mh;
        mbar_arrive(&x_full[sb * 2 + h]);
        if (!(ok = wait_all(&x_full[sb * 2 + (h ^ 1)], (t >> 1) & 1))) break;
        const float mt = fmaxf(mh, xmax[(sb * 2 + (h ^ 1)) * kRows + row]) * sl2;
        const float m_new = (mt > m + 8.f) ? mt : m;
        const float m_ref = (m_new == NEG_INF) ? 0.f : m_new;
        const float alpha = ex2(m - m_ref);
        const float neg_m = -m_ref;
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(neg_m, neg_m);
        uint64_t acc2[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc2[a] = 0ull;
        float pk[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const uint64_t y2 = f2_fma(f2_pack(sv[x >> 4][(x & 15) * 2], sv[x >> 4][(x & 15) * 2 + 1]), sl2x2, negm2);
          float e0, e1;
          f2_unpack(y2, e0, e1);
          e0 = ex2(e0);
          e1 = ex2(e1);
          acc2[x & 3] = f2_add(acc2[x & 3], f2_pack(e0, e1));
          pk[x] = __uint_as_float(pack_bf16x2(e0, e1));
        }
        tmem_st32(taddr + colS + h * 32, pk);  // P of keys 64h..64h+63: columns 32h..32h+31
        float ps[8];
#pragma unroll
        for (int a = 0; a < 4; ++a) f2_unpack(acc2[a], ps[2 * a], ps[2 * a + 1]);
        l = l * alpha + (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
        if (j >= 1 && __any_sync(0xffffffffu, m_new != m)) {  // this half's 64 columns of O
          // S(j) may have been issued before PV(j-1): wait for it (the
          // (t-1)-th PV) before touching O. The parity names that PV: the
          // tensor core completes this thread's MMAs in order, so PV(t-2)
          // is done once S(t) is, and PV(t) waits for this warpgroup's P(t).
          if (!(ok = wait_all(&s_free[0], (t - 1) & 1))) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(taddr + kColO + h * 64 + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(taddr + kColO + h * 64 + c * 32, o);
          }
        }
        m = m_new;
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&ph_full[h * 2 + sb]);
      }
      if (!ok) break;
      // Row statistics: the two halves' partial sums (same max) in the l
      // rows of tiles 0 and 1, the max in tile 0's; the epilogue adds them.
      if (!(ok = wait_all(&st_empty[0], (nst & 1) ^ 1u))) break;
      stats[(h * 2 + 0) * kRows + row] = l;
      if (h == 0) stats[kRows + row] = m;
      mbar_arrive(&st_full[0]);
      ++nst;
    }
  } else if (wg < 2) {
    regs_inc<kSplit ? kRegSoftmaxSplit : kRegSoftmax>();
    // ------------------------------------------------------------ softmax of tile i = wg
    const int i = wg;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t colS = i * 128, colO = kColO + i * 128;
    const float sl2 = p.scale_log2;
    // The walk state lives in shared memory: it is only needed between
    // tiles, and keeping it out of registers leaves them to the
    // exponential loop.
    Walker& w = *reinterpret_cast<Walker*>(smem + off_state<kSplit>() + warp * 128);
    Item& it = *reinterpret_cast<Item*>(smem + off_state<kSplit>() + warp * 128 + 32);
    walker_init<kSplit>(p, wt, w);
    uint32_t t = 0;      // S_i tiles seen
    uint32_t nst = 0;    // items whose statistics were written
    bool ok = true;
    while (ok && walker_next<kSplit>(p, wt, w, it)) {
      const int ni = i ? it.n1 : it.n0;
      if (ni == 0) continue;
      const int tok = it.q0 + i * p.tq + (row & (p.tq - 1));        // token index within the sequence
      const int lim = p.causal ? min(max(tok + 1 + it.off, 0), it.K) : it.K;  // keys [0, lim) are visible
      float m = NEG_INF, l = 0.f;
      for (int j = 0; j < ni; ++j, ++t) {
        // tcgen05.ld is warp-collective: keep the decision to continue warp-uniform
        if (!(ok = wait_all(&s_full[i], t & 1))) break;
        tc_fence_after();
        float sv[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(taddr + colS + c * 32, sv[c]);
        tc_wait_ld();

        // Row max of the raw scores with 8 independent partial maxima.
        const int nvis = lim - j * kKeys;  // visible columns of this tile
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = NEG_INF;
        const bool whole = __all_sync(0xffffffffu, nvis >= kKeys);  // whole tile visible: no mask
        if (whole) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2) mx[(e >> 1) & 7] = fmax3(mx[(e >> 1) & 7], sv[c][e], sv[c][e + 1]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float x0 = (c * 32 + e < nvis) ? sv[c][e] : NEG_INF;
              const float x1 = (c * 32 + e + 1 < nvis) ? sv[c][e + 1] : NEG_INF;
              sv[c][e] = x0;
              sv[c][e + 1] = x1;
              mx[(e >> 1) & 7] = fmax3(mx[(e >> 1) & 7], x0, x1);
            }
        }
        const float mt = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) * sl2;
        const float m_new = (mt > m + 8.f) ? mt : m;
        // A row that has seen no key yet keeps m = -inf: use 0 as its
        // reference so P and alpha come out 0 instead of NaN.
        const float m_ref = (m_new == NEG_INF) ? 0.f : m_new;
        const float alpha = ex2(m - m_ref);  // 0 on the first tile, 1 when m is kept
        const float neg_m = -m_ref;
        // P = exp2(S*scale*log2e - m) -> bf16 pairs over the first 64 columns
        // of S_i, one 64-key half at a time (S values become packed P as
        // they are used, which keeps the live registers near one S row).
        // Scale and shift (and later sum) in packed pairs; 2^x on the MUFU
        // unit. (Moving part of the exponentials to an FMA-pipe polynomial
        // was measured slower: the softmax is issue-bound, not MUFU-bound.)
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(neg_m, neg_m);
        uint64_t acc2[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc2[a] = 0ull;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          float pk[32];
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const uint64_t y2 =
                f2_fma(f2_pack(sv[2 * c2 + (x >> 4)][(x & 15) * 2], sv[2 * c2 + (x >> 4)][(x & 15) * 2 + 1]), sl2x2, negm2);
            float e0, e1;
            f2_unpack(y2, e0, e1);
            e0 = ex2(e0);  // masked: -inf -> 0
            e1 = ex2(e1);
            acc2[x & 3] = f2_add(acc2[x & 3], f2_pack(e0, e1));
            pk[x] = __uint_as_float(pack_bf16x2(e0, e1));
          }
          tmem_st32(taddr + colS + c2 * 32, pk);
        }
        float ps[8];
#pragma unroll
        for (int a = 0; a < 4; ++a) f2_unpack(acc2[a], ps[2 * a], ps[2 * a + 1]);
        const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        l = l * alpha + rs;
        // O_i holds PV of tiles < j (S_i(j) was issued after PV_i(j-1), and
        // the commit that signalled S_i(j) covers every earlier MMA of the
        // issuing thread) and PV_i(j) waits for P_i(j): rescale it in place
        // when a row of this warp raised its max. (A first tile's PV
        // overwrites O.)
        if (j >= 1 && __any_sync(0xffffffffu, m_new != m)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(taddr + colO + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(taddr + colO + c * 32, o);
          }
        }
        m = m_new;
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[i]);
      }
      if (!ok) break;
      // Row statistics for the epilogue.
      if (!(ok = wait_all(&st_empty[i], (nst & 1) ^ 1u))) break;
      stats[(i * 2 + 0) * kRows + row] = l;
      stats[(i * 2 + 1) * kRows + row] = m;
      mbar_arrive(&st_full[i]);
      ++nst;
    }
  } else if (wg == 2) {
    regs_dec<kSplit ? kRegEpilogueSplit : kRegEpilogue>();
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    uint8_t* stage = smem + kOffStage + quarter * kStageBytes;
    Walker w;
    walker_start<kSplit>(p, wt, w);
    Item it;
    uint32_t cp[2] = {0, 0};       // PV_i so far (through this item)
    uint32_t items_i[2] = {0, 0};  // items in which tile i ran
    bool ok = true;
    while (ok && walker_step<kSplit>(p, wt, w, it)) {
      for (int i = 0; i < 2 && ok; ++i) {
        const int ni = i ? it.n1 : it.n0;
        if (ni == 0) continue;
        cp[i] += ni;
        if (!(ok = wait_all(&st_full[i], items_i[i] & 1))) break;
        const float l = kSplit ? stats[row] + stats[2 * kRows + row] : stats[(i * 2 + 0) * kRows + row];
        const float m = stats[(i * 2 + 1) * kRows + row];
        mbar_arrive(&st_empty[i]);
        // the item's last PV_i
        if (!(ok = kSplit ? wait_all(o_full, items_i[i] & 1) : wait_all(&s_free[i], (cp[i] - 1) & 1))) break;
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int qt0 = it.q0 + i * p.tq;
        {
          const int g = row >> p.tq_shift;
          const int tok = qt0 + (row & (p.tq - 1));
          if (p.lse && tok < it.L)
            p.lse[static_cast<long long>(it.h * p.group + g) * p.total + it.seq0 + tok] =
                l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : NEG_INF;
        }
        // O_i rows -> global through this warp's staging buffer, one 64-dim
        // half at a time: each thread writes its row (8 chunks of 16 B,
        // XOR-swizzled by row), then each store instruction writes 4 rows x
        // 128 contiguous bytes. Rows past the sequence's end are not stored.
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tmem_ld32(taddr + kColO + i * 128 + h2 * 64 + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint4 u;
              u.x = pack_bf16x2(o[q4 * 8 + 0] * inv, o[q4 * 8 + 1] * inv);
              u.y = pack_bf16x2(o[q4 * 8 + 2] * inv, o[q4 * 8 + 3] * inv);
              u.z = pack_bf16x2(o[q4 * 8 + 4] * inv, o[q4 * 8 + 5] * inv);
              u.w = pack_bf16x2(o[q4 * 8 + 6] * inv, o[q4 * 8 + 7] * inv);
              const int ch = c * 4 + q4;
              *reinterpret_cast<uint4*>(stage + lane * 128 + ((ch ^ (lane & 7)) << 4)) = u;
            }
          }
          if (h2 == 1) {  // all of O_i is in registers or staged: the next item may overwrite it
            tc_fence_before();
            mbar_arrive(&o_empty[i]);
          }
          __syncwarp();
#pragma unroll 1
          for (int x = 0; x < 8; ++x) {
            const int r = x * 4 + (lane >> 3), ch = lane & 7;
            const int rrow = quarter * 32 + r;
            const int rg = rrow >> p.tq_shift;
            const int rtok = qt0 + (rrow & (p.tq - 1));
            const uint4 u = *reinterpret_cast<const uint4*>(stage + r * 128 + ((ch ^ (r & 7)) << 4));
            if (rtok < it.L)
              *reinterpret_cast<uint4*>(p.out + static_cast<long long>(it.seq0 + rtok) * p.out_ts +
                                        static_cast<long long>(it.h * p.group + rg) * p.out_hs + h2 * 64 + ch * 8) = u;
          }
          __syncwarp();
        }
        ++items_i[i];
      }
    }
  } else {
    regs_dec<kSplit ? kRegOtherSplit : kRegOther>();
    if (warp == 13) {
      // ---------------------------------------------------------- TMA producer (lane 0 issues)
      // Per item: Q0 (+ Q1), then K(j), V(j) for j = 0..n-1 into the ring, in
      // the order the MMA warp consumes them.
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
      }
      // One 128-key K or V tile (both 64-dim halves) of item `it`, tile j.
      // Paged: one box per run of box_keys keys, through the block table;
      // keys at or past the sequence's end, and ids outside the table or the
      // pool (also reported), load from block `num_blocks`, outside the
      // tensor map, which the copy engine fills with zeros. Either way the
      // full tile's bytes land.
      auto load_kv = [&](uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, const Item& it, int j) {
        if (!p.paged) {
          for (int half = 0; half < 2; ++half)
            tma_load_3d(dst + half * kKVHalf, tm, bar, half * 64, it.h, it.seq0 + j * kKeys);
          return;
        }
        for (int b = 0; b < kKeys; b += p.box_keys) {
          const int key = j * kKeys + b;
          const int lb = key / p.bs;
          int blk = p.num_blocks;
          if (key < it.K) {
            if (lb >= p.max_blocks) {
              if (p.err) atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
            } else {
              const int id = __ldg(p.bt + static_cast<long long>(it.s) * p.bt_stride + lb);
              if (id >= 0 && id < p.num_blocks)
                blk = id;
              else if (p.err)
                atomicCAS(p.err, 0, LA_DEVERR_BLOCK_ID);
            }
          }
          for (int half = 0; half < 2; ++half)
            tma_load_4d(dst + half * kKVHalf + b * 128, tm, bar, half * 64, key - lb * p.bs, it.h, blk);
        }
      };
      Walker w;
      walker_start<kSplit>(p, wt, w);
      Item it;
      int kq = 0;
      long long nld = 0;  // K/V tiles loaded
      bool ok = true;
      while (ok && walker_step<kSplit>(p, wt, w, it)) {
        if (lane == 0 && it.q0 + p.pair * p.tq >= p.n_qp * p.pair * p.tq && it.L > p.n_qp * p.pair * p.tq && p.err)
          atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);  // longer than max_seqlen: the tail is not computed
        // the split instance may have requested its first item's Q, K(0)
        // and V(0) before the roles started
        const bool pre0 = kSplit && kq == 0 && *reinterpret_cast<const int*>(smem + kOffFirst + 84) != 0;
        if (!pre0 && !(ok = wait_all(q_empty, (kq & 1) ^ 1u))) break;
        if (lane == 0 && !pre0) {
          mbar_arrive_expect_tx(q_full, (it.has1 ? 2 : 1) * kQTile);
          for (int t = 0; t < 1 + it.has1; ++t)
            for (int g = 0; g < p.group; ++g)
              for (int half = 0; half < 2; ++half)
                tma_load_3d(sQ + t * kQTile + half * kQHalf + g * p.tq * 128, &tm_q, q_full, half * 64,
                            it.h * p.group + g, it.seq0 + it.q0 + t * p.tq);
        }
        ++kq;
        for (int j = 0; j < it.n && ok; ++j) {
          for (int kv = 0; kv < 2; ++kv, ++nld) {
            if (pre0 && j < 2) continue;  // issued before the roles started
            const int st = static_cast<int>(nld % kStages);
            const uint32_t use = static_cast<uint32_t>(nld / kStages);
            if (!(ok = wait_all(&kv_empty[st], (use & 1) ^ 1u))) break;
            if (lane == 0) {
              mbar_arrive_expect_tx(&kv_full[st], kKVTile);
              load_kv(sKV + st * kKVTile, kv ? &tm_v : &tm_k, &kv_full[st], it, j);
            }
          }
        }
      }
      if (!ok && lane == 0) {  // early exit: let the copies already issued land (bounded)
        for (long long u = (nld > kStages ? nld - kStages : 0); u < nld; ++u)
          mbar_wait(&kv_full[u % kStages], static_cast<uint32_t>(u / kStages) & 1, nullptr, 0);
        if (kq > 0) mbar_wait(q_full, (kq - 1) & 1, nullptr, 0);
      }
      __syncwarp();
    } else if (warp == 12 && kSplit) {
      // ------------------------------------ MMA issuer, single-tile items (lane 0 issues)
      // S is double-buffered in TMEM (S(j) in columns 128 (j % 2) + [0, 128),
      // P(j) over the first 64 of them): S(j+2) is issued right behind PV(j),
      // which reads P(j) from the same columns (the tensor core executes this
      // thread's MMAs in order), while the softmax works on S(j+1).
      Walker w;
      walker_start<kSplit>(p, wt, w);
      Item it;
      int kq = 0;
      long long nld = 0;  // K/V ring position of the item's K(0)
      uint32_t sc = 0;    // S tiles issued
      uint32_t cp = 0;    // PVs issued
      uint32_t items = 0;
      bool ok = true;
      auto slot_of = [&](long long idx) -> int { return static_cast<int>(idx % kStages); };
      auto wait_full = [&](long long idx) -> bool {
        return wait_all(&kv_full[slot_of(idx)], static_cast<uint32_t>(idx / kStages) & 1);
      };
      // The next S from the K tile at ring position kpos; the item's last S
      // frees Q.
      auto issue_s = [&](long long kpos, bool last_s) -> bool {
        if (!wait_full(kpos)) return false;
        const uint32_t b = sc & 1;
        if (lane == 0) {
          const uint64_t ad = desc_kmajor(sQ, kQHalf, 0);
          const uint64_t bd = desc_kmajor(sKV + slot_of(kpos) * kKVTile, kKVHalf, 0);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16_ss(tmem + b * 128, ad + (((ks >> 2) * kQHalf + (ks & 3) * 32) >> 4),
                        bd + (((ks >> 2) * kKVHalf + (ks & 3) * 32) >> 4), kIdescQK, ks > 0 ? 1u : 0u);
          umma_commit(&s_full[b]);
          umma_commit(&kv_empty[slot_of(kpos)]);
          if (last_s) umma_commit(q_empty);
        }
        __syncwarp();
        ++sc;
        return true;
      };
      while (ok && walker_step<kSplit>(p, wt, w, it)) {
        if (!(ok = wait_all(q_full, kq & 1))) break;
        ++kq;
        const int n = it.n0;
        const long long base = nld;  // K(j) at base + 2j, V(j) at base + 2j + 1
        nld += 2LL * n;
        const uint32_t b0 = sc & 1;  // S buffer of this item's S(0)
        if (!(ok = issue_s(base, n == 1))) break;
        if (n >= 2 && !(ok = issue_s(base + 2, n == 2))) break;
        for (int j = 0; j < n && ok; ++j) {
          const long long vi = base + 2 * j + 1;
          if (!(ok = wait_full(vi))) break;
          uint8_t* vt = sKV + slot_of(vi) * kKVTile;
          const int vrows = it.K - j * kKeys;  // valid V rows of this tile
          if (p.paged && vrows < kKeys) {
            // Pool slots past the sequence's last key hold whatever was there
            // (possibly NaN); P is 0 for them but 0 * NaN is not, so zero them.
            const int r0 = max(vrows, 0);
            const int n16 = (kKeys - r0) * 8;  // 16-byte chunks per half
            for (int x = lane; x < 2 * n16; x += 32) {
              const int half = x / n16, c = x - half * n16;
              *reinterpret_cast<uint4*>(vt + half * kKVHalf + r0 * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async_smem();
            __syncwarp();
          }
          if (!(ok = wait_all(&ph_full[cp & 1], (cp >> 1) & 1))) break;   // both halves of P(j)
          if (!(ok = wait_all(&ph_full[2 + (cp & 1)], (cp >> 1) & 1))) break;
          if (j == 0) {  // O is overwritten: the epilogue must have read the previous item's
            if (items > 0 && !(ok = wait_all(&o_empty[0], (items - 1) & 1))) break;
            ++items;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t pt = tmem + ((b0 + j) & 1) * 128;  // P(j): 16 keys per 8 columns
            const uint64_t vd = desc_v(vt, 0);                 // k-step ks: + 2048 B / 16
#pragma unroll
            for (int ks = 0; ks < kKeys / 16; ++ks)
              umma_f16_ts(tmem + kColO, pt + ks * 8, vd + ks * 128, kIdescPV, (j > 0 || ks > 0) ? 1u : 0u);
            umma_commit(&s_free[0]);
            umma_commit(&kv_empty[slot_of(vi)]);
            if (j + 1 == n) umma_commit(o_full);
          }
          __syncwarp();
          ++cp;
          if (j + 2 < n && !(ok = issue_s(base + 2 * (j + 2), j + 3 == n))) break;
        }
      }
      __syncwarp();
    } else if (warp == 12) {
      // ---------------------------------------------------------- MMA issuer (lane 0 issues)
      Walker w;
      walker_init<kSplit>(p, wt, w);
      Item it;
      int kq = 0;
      long long nld = 0;               // K/V ring position of the item's K(0)
      uint32_t cp[2] = {0, 0};         // PV_i issued
      uint32_t items_i[2] = {0, 0};    // items in which tile i ran
      bool ok = true;
      // S_i(j+1) is written over P_i(j), which PV_i(j) reads: both are issued
      // by this thread, PV_i(j) first, and the tensor core executes one
      // thread's MMAs in issue order, so S_i(j+1) is issued right behind
      // PV_i(j) without waiting for it to complete (waiting left the tensor
      // core idle for the commit -> mbarrier -> issue round trip).
      auto issue_s = [&](int i, const uint8_t* kt) -> bool {
        if (lane == 0) {
          // k-step ks: descriptor start address + (64-dim half, 32-byte step) / 16
          const uint64_t ad = desc_kmajor(sQ + i * kQTile, kQHalf, 0), bd = desc_kmajor(kt, kKVHalf, 0);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16_ss(tmem + i * 128, ad + (((ks >> 2) * kQHalf + (ks & 3) * 32) >> 4),
                        bd + (((ks >> 2) * kKVHalf + (ks & 3) * 32) >> 4), kIdescQK, ks > 0 ? 1u : 0u);
          umma_commit(&s_full[i]);
        }
        __syncwarp();
        return true;
      };
      auto issue_pv = [&](int i, int j, const uint8_t* vt) -> bool {
        if (!wait_all(&p_full[i], cp[i] & 1)) return false;
        if (j == 0) {  // O_i is overwritten: the epilogue must have read the previous item's
          if (items_i[i] > 0 && !wait_all(&o_empty[i], (items_i[i] - 1) & 1)) return false;
          ++items_i[i];
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t pt = tmem + i * 128;  // P_i: 16 keys per 8 columns
          const uint64_t vd = desc_v(vt, 0);   // k-step ks: + 2048 B / 16
#pragma unroll
          for (int ks = 0; ks < kKeys / 16; ++ks)
            umma_f16_ts(tmem + kColO + i * 128, pt + ks * 8, vd + ks * 128, kIdescPV, (j > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&s_free[i]);
        }
        __syncwarp();
        ++cp[i];
        return true;
      };
      auto slot_of = [&](long long idx) -> int { return static_cast<int>(idx % kStages); };
      auto wait_full = [&](long long idx) -> bool {
        return wait_all(&kv_full[slot_of(idx)], static_cast<uint32_t>(idx / kStages) & 1);
      };
      while (ok && walker_next<kSplit>(p, wt, w, it)) {
        if (!(ok = wait_all(q_full, kq & 1))) break;
        const long long base = nld;  // K(j) at base + 2j, V(j) at base + 2j + 1
        nld += 2LL * it.n;
        // S_0(0), S_1(0)
        if (!(ok = wait_full(base))) break;
        {
          const uint8_t* kt = sKV + slot_of(base) * kKVTile;
          if (!(ok = issue_s(0, kt))) break;
          if (it.n1 > 0 && !(ok = issue_s(1, kt))) break;
          if (lane == 0) {
            umma_commit(&kv_empty[slot_of(base)]);
            if (it.n == 1) umma_commit(q_empty);
          }
          __syncwarp();
        }
        for (int j = 0; j < it.n && ok; ++j) {
          const long long vi = base + 2 * j + 1, ki = vi + 1;  // V(j), K(j+1)
          const bool a0 = j < it.n0, a1 = j < it.n1;
          const bool nx0 = j + 1 < it.n0, nx1 = j + 1 < it.n1;
          if (!(ok = wait_full(vi))) break;
          uint8_t* vt = sKV + slot_of(vi) * kKVTile;
          const int vrows = it.K - j * kKeys;  // valid V rows of this tile
          if (p.paged && vrows < kKeys) {
            // Pool slots past the sequence's last key hold whatever was there
            // (possibly NaN); P is 0 for them but 0 * NaN is not, so zero them.
            const int r0 = max(vrows, 0);
            const int n16 = (kKeys - r0) * 8;  // 16-byte chunks per half
            for (int x = lane; x < 2 * n16; x += 32) {
              const int half = x / n16, c = x - half * n16;
              *reinterpret_cast<uint4*>(vt + half * kKVHalf + r0 * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async_smem();
            __syncwarp();
          }
          if ((nx0 || nx1) && !(ok = wait_full(ki))) break;
          const uint8_t* kt = sKV + slot_of(ki) * kKVTile;
          if (a0 && !(ok = issue_pv(0, j, vt))) break;
          if (nx0 && !(ok = issue_s(0, kt))) break;
          if (a1 && !(ok = issue_pv(1, j, vt))) break;
          if (lane == 0) umma_commit(&kv_empty[slot_of(vi)]);  // V(j) read once both PVs are done
          __syncwarp();
          if (nx1 && !(ok = issue_s(1, kt))) break;
          if (j + 1 < it.n) {
            if (lane == 0) {
              umma_commit(&kv_empty[slot_of(ki)]);
              if (j + 2 == it.n) umma_commit(q_empty);  // this item's last S
            }
            __syncwarp();
          }
        }
        ++kq;
      }
      __syncwarp();
    }
    // warps 14, 15: no role
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 12) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill

int prefill_init(int device) {
  (void)device;
  cudaError_t e = cudaFuncSetAttribute(prefill::prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(prefill::kSmemBytes));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill::prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(prefill::kSmemBytesSplit));
  return cuda_status(e);
}

}  // namespace la

namespace la {
namespace prefill {

// Common tail of the two entry points: the persistent grid over the items.
// n_qt: query tiles of the longest sequence. Items are pairs of query tiles
// (the two tiles share every K/V tile); when even the upper bound on the
// pair count cannot fill the SMs (one short prompt), items are single tiles:
// twice as many items, each half as long.
static int launch(const CUtensorMap& tq_map, const CUtensorMap& tk_map, const CUtensorMap& tv_map, Params p,
                  int n_qt, cudaStream_t stream) {
  const int device = current_device();
  const int sms = device >= 0 ? num_sms(device) : 0;
  if (sms <= 0) return LA_ERR_CUDA;
  p.pair = 2;
  p.n_qp = (n_qt + 1) / 2;
  if (static_cast<long long>(p.n_qp) * p.num_seqs * p.hkv < sms) {
    p.pair = 1;
    p.n_qp = n_qt;
  }
  const long long items = static_cast<long long>(p.n_qp) * p.num_seqs * p.hkv;
  if (items > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  const long long ctas = sms;  // one persistent CTA per SM (all of its TMEM and most of its shared memory)
  const dim3 grid(static_cast<unsigned>(items < ctas ? items : ctas));
  return cuda_status(p.pair == 1 ? launch_pdl(prefill_kernel<true>, grid, dim3(kThreads), kSmemBytesSplit, stream, tq_map,
                                               tk_map, tv_map, p)
                                 : launch_pdl(prefill_kernel<false>, grid, dim3(kThreads), kSmemBytes, stream, tq_map,
                                              tk_map, tv_map, p));
}

// Q map [total, Hq, D] with a (64 dims, 1 head, tq tokens) box, and the
// checks shared by both entry points.
static int common_setup(const void* q, int64_t q_token_stride, int64_t q_head_stride, int64_t total_tokens,
                        int num_q_heads, int num_kv_heads, int head_dim, float softmax_scale, void* out,
                        int64_t out_token_stride, int64_t out_head_stride, CUtensorMap* tq_map, Params* p) {
  if (head_dim != kD) return LA_ERR_UNSUPPORTED;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return LA_ERR_INVALID_ARGUMENT;
  const int group = num_q_heads / num_kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8) return LA_ERR_UNSUPPORTED;
  if (!(softmax_scale > 0.f)) return LA_ERR_INVALID_ARGUMENT;
  if (total_tokens > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(out, 16)) return LA_ERR_ALIGNMENT;
  const long long st[] = {q_token_stride, q_head_stride, out_token_stride, out_head_stride};
  for (long long x : st)
    if (x <= 0 || x % 8) return LA_ERR_ALIGNMENT;
  const int tq = kRows / group;
  const uint64_t dims[3] = {128, static_cast<uint64_t>(num_q_heads), static_cast<uint64_t>(total_tokens)};
  const uint64_t strides[2] = {static_cast<uint64_t>(q_head_stride) * 2, static_cast<uint64_t>(q_token_stride) * 2};
  const uint32_t box[3] = {64, 1, static_cast<uint32_t>(tq)};
  const int stt = encode_tensor_map_bf16(tq_map, q, 3, dims, strides, box, true);
  if (stt != LA_OK) return stt;
  *p = Params{};
  p->tq = tq;
  p->tq_shift = __builtin_ctz(static_cast<unsigned>(tq));
  p->hq = num_q_heads;
  p->hkv = num_kv_heads;
  p->hkv_shift = (num_kv_heads & (num_kv_heads - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(num_kv_heads)) : -1;
  p->group = group;
  p->scale_log2 = softmax_scale * 1.4426950408889634f;
  p->out = static_cast<__nv_bfloat16*>(out);
  p->out_ts = out_token_stride;
  p->out_hs = out_head_stride;
  p->total = total_tokens;
  return LA_OK;
}

}  // namespace prefill
}  // namespace la

extern "C" int la_prefill_varlen(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
                                 int64_t k_token_stride, int64_t k_head_stride, const void* v, int64_t v_token_stride,
                                 int64_t v_head_stride, const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                                 int64_t total_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                                 float softmax_scale, int causal, void* out, int64_t out_token_stride,
                                 int64_t out_head_stride, float* softmax_lse, int* dev_error, cudaStream_t stream) {
  using namespace la;
  using namespace la::prefill;
  if (!q || !k || !v || !cu_seqlens || !out) return LA_ERR_INVALID_ARGUMENT;
  if (num_seqs < 0 || max_seqlen < 0 || total_tokens < 0) return LA_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || max_seqlen == 0 || total_tokens == 0) return LA_OK;
  if (!aligned(k, 16) || !aligned(v, 16)) return LA_ERR_ALIGNMENT;
  const long long kst[] = {k_token_stride, k_head_stride, v_token_stride, v_head_stride};
  for (long long x : kst)
    if (x <= 0 || x % 8) return LA_ERR_ALIGNMENT;
  CUtensorMap tq_map, tk_map, tv_map;
  Params p;
  int stt = common_setup(q, q_token_stride, q_head_stride, total_tokens, num_q_heads, num_kv_heads, head_dim,
                         softmax_scale, out, out_token_stride, out_head_stride, &tq_map, &p);
  if (stt != LA_OK) return stt;
  {
    const uint64_t dims[3] = {128, static_cast<uint64_t>(num_kv_heads), static_cast<uint64_t>(total_tokens)};
    const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kKeys)};
    const uint64_t ks[2] = {static_cast<uint64_t>(k_head_stride) * 2, static_cast<uint64_t>(k_token_stride) * 2};
    const uint64_t vs[2] = {static_cast<uint64_t>(v_head_stride) * 2, static_cast<uint64_t>(v_token_stride) * 2};
    if ((stt = encode_tensor_map_bf16(&tk_map, k, 3, dims, ks, box, true)) != LA_OK) return stt;
    if ((stt = encode_tensor_map_bf16(&tv_map, v, 3, dims, vs, box, true)) != LA_OK) return stt;
  }
  p.cu = cu_seqlens;
  p.num_seqs = num_seqs;
  const int n_qt = (max_seqlen + p.tq - 1) / p.tq;
  p.causal = causal ? 1 : 0;
  p.lse = softmax_lse;
  p.err = dev_error;
  return launch(tq_map, tk_map, tv_map, p, n_qt, stream);
}

extern "C" int la_prefill_paged(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k_cache,
                                const void* v_cache, int64_t kv_block_stride, int64_t kv_token_stride,
                                int64_t kv_head_stride, int64_t num_blocks, int block_size,
                                const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
                                const int32_t* cache_seqlens, const int32_t* cu_seqlens_q, int q_len, int num_seqs,
                                int max_seqlen_q, int64_t total_q, int num_q_heads, int num_kv_heads, int head_dim,
                                float softmax_scale, int causal, void* out, int64_t out_token_stride,
                                int64_t out_head_stride, float* softmax_lse, int* dev_error, cudaStream_t stream) {
  using namespace la;
  using namespace la::prefill;
  if (!q || !k_cache || !v_cache || !block_table || !cache_seqlens || !out) return LA_ERR_INVALID_ARGUMENT;
  if (num_seqs < 0 || total_q < 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || bt_seq_stride < 0)
    return LA_ERR_INVALID_ARGUMENT;
  if (cu_seqlens_q) {
    if (max_seqlen_q < 0) return LA_ERR_INVALID_ARGUMENT;
  } else {
    if (q_len < 0 || total_q != static_cast<int64_t>(q_len) * num_seqs) return LA_ERR_INVALID_ARGUMENT;
    max_seqlen_q = q_len;
  }
  if (num_seqs == 0 || max_seqlen_q == 0 || total_q == 0) return LA_OK;
  if (num_blocks > 0x7ffffffeLL) return LA_ERR_UNSUPPORTED;
  // 128-key tiles must not straddle blocks, or be whole blocks of 16 / 32 / 64.
  if (block_size <= 0 || block_size % 16 || (block_size % kKeys && kKeys % block_size)) return LA_ERR_UNSUPPORTED;
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16)) return LA_ERR_ALIGNMENT;
  const long long kst[] = {kv_block_stride, kv_token_stride, kv_head_stride};
  for (long long x : kst)
    if (x <= 0 || x % 8) return LA_ERR_ALIGNMENT;
  CUtensorMap tq_map, tk_map, tv_map;
  Params p;
  int stt = common_setup(q, q_token_stride, q_head_stride, total_q, num_q_heads, num_kv_heads, head_dim,
                         softmax_scale, out, out_token_stride, out_head_stride, &tq_map, &p);
  if (stt != LA_OK) return stt;
  const int box_keys = block_size < kKeys ? block_size : kKeys;
  {
    // Pool [NB, BS, Hkv, D] as a 4-D map (D, BS, Hkv, NB): one box is
    // (64 dims, box_keys tokens, 1 head, 1 block).
    const uint64_t dims[4] = {128, static_cast<uint64_t>(block_size), static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(kv_token_stride) * 2, static_cast<uint64_t>(kv_head_stride) * 2,
                                 static_cast<uint64_t>(kv_block_stride) * 2};
    const uint32_t box[4] = {64, static_cast<uint32_t>(box_keys), 1, 1};
    if ((stt = encode_tensor_map_bf16(&tk_map, k_cache, 4, dims, strides, box, true)) != LA_OK) return stt;
    if ((stt = encode_tensor_map_bf16(&tv_map, v_cache, 4, dims, strides, box, true)) != LA_OK) return stt;
  }
  p.cu = cu_seqlens_q;
  p.q_len = q_len;
  p.num_seqs = num_seqs;
  const int n_qt = (max_seqlen_q + p.tq - 1) / p.tq;
  p.causal = causal ? 1 : 0;
  p.lse = softmax_lse;
  p.err = dev_error;
  p.paged = 1;
  p.k_lens = cache_seqlens;
  p.bt = block_table;
  p.bt_stride = bt_seq_stride;
  p.max_blocks = max_blocks_per_seq;
  p.bs = block_size;
  p.box_keys = box_keys;
  p.num_blocks = static_cast<int>(num_blocks);
  return launch(tq_map, tk_map, tv_map, p, n_qt, stream);
}
