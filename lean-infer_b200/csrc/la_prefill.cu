// (c) Causal varlen prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA), sm_100a.
//
// Semantics: for every packed sequence s (tokens cu_seqlens[s] ..
// cu_seqlens[s+1]-1) and query head h, softmax(scale * Q K^T) V over the keys of
// the same sequence and kv head h / G, causal (key j visible to query i iff
// j <= i) — the reference's F.scaled_dot_product_attention(q, k, v,
// is_causal=True, enable_gqa=True) at leaninfer/qwen3/model.py:56-57, applied
// to many prompts at once (flash-attn varlen contract).
//
// CTA tile: 128 query rows = the tq = 128/G consecutive tokens of the G query
// heads that share one kv head (GQA packing: every K/V tile feeds all G
// heads), against KV tiles of 64 keys. Per KV tile j:
//   S_j  = Q K_j^T        tcgen05.mma M128 N64 K16 x8, fp32 in TMEM (2 buffers)
//   P_j  = exp2(S_j*scale*log2e - m)  by 4 softmax warps, one thread per row,
//          written back as bf16 over the first half of S_j's TMEM columns
//   O   += P_j V_j        tcgen05.mma M128 N128 K16 x4, A = P from TMEM, B = V
//                         read MN-major from its TMA tile, fp32 in TMEM
// S_j's buffer is released by the completion of PV_j, so P is double-buffered
// with S and softmax of tile j waits for PV_{j-1} only to rescale O.
// The row max is only raised (and O, l rescaled) when a tile's max exceeds the
// running one by more than 8 (log2 units), so P stays <= 256 and most tiles
// skip the O rescale. S_{j+1} is issued while softmax works on S_j.
//
// Persistent CTAs walk a heaviest-first list of (sequence, kv head, query
// tile) items. A CTA needs 112 KB of shared memory, 256 TMEM columns and
// <= 170 registers per thread, so two CTAs share each SM: while one CTA's
// softmax warps work, the other's MMAs run, and each scheduler has two
// softmax warps to switch between.
//
// Warps: 0 = TMA producer, 1 = MMA issuer + TMEM owner, 2..5 = softmax and
// epilogue (warp w reads TMEM lanes 32*(w%4)..+31, i.e. rows of that quarter).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace prefill {

constexpr int kD = 128;
constexpr int kRows = 128;            // query rows per CTA
constexpr int kKeys = 64;             // keys per KV tile
constexpr int kQHalf = kRows * 128;   // one 64-dim half of the Q tile: 128 rows x 128 B = 16 KB
constexpr int kQTile = 2 * kQHalf;    // 32 KB
constexpr int kKVHalf = kKeys * 128;  // one 64-dim half of a K or V tile: 8 KB
constexpr int kKVTile = 2 * kKVHalf;  // 16 KB
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;  // S0/P0 [0,64) S1/P1 [64,128) O [128,256)
constexpr uint32_t kColO = 128;
constexpr uint32_t kIdescQK = idesc_bf16_f32(128, kKeys, false, false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, false, true);
// Q | K x2 | V x2 | O staging (4 KB per softmax warp) | barriers. Two CTAs
// must fit in an SM's 228 KB, so no alignment slack is requested: the kernel
// checks that the dynamic shared memory base is 1024-byte aligned (the
// 128-byte swizzle atom) and reports LA_DEVERR_SMEM_ALIGN otherwise.
constexpr int kStageOffset = kQTile + 4 * kKVTile;     // 96 KB
constexpr int kStageBytes = 32 * 128;                  // 32 rows x 64 dims bf16 per warp
constexpr int kBarOffset = kStageOffset + 4 * kStageBytes;  // 112 KB
constexpr size_t kSmemBytes = kBarOffset + 256;

struct Params {
  const int* cu;  // query starts [num_seqs + 1], or null: sequence s has q_len queries from token s * q_len
  int q_len;
  int num_seqs;
  int n_qt;  // query tiles of the longest sequence
  int tq;    // tokens per query tile (128 / group)
  int hq, hkv, group;
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

// Work items are (sequence, kv head, query tile) in descending cost: query-
// tile level qt from the top down (a tile's KV length grows with qt), at each
// level only the sequences long enough to have that tile, then the kv heads.
// The valid items are ranked in that order and dealt to the G persistent CTAs
// as a snake over 2G columns (CTA c takes ranks c, 2G-1-c, 2G+c, 4G-1-c, ...),
// which evens out the summed cost per CTA. Every warp walks its CTA's item
// list itself (the walk is warp-collective), so no item descriptors are
// exchanged between roles.
struct Item {
  int s, h, q0, seq0, L, n_kv;
  int K, off;  // keys of the sequence; causal offset K - L (0 for contiguous keys)
};

struct Walker {
  int taken;       // items this CTA has taken so far
  int level;       // current query-tile level
  long long base;  // rank of the first item of `level`
  int count;       // items at `level`
};

__device__ __forceinline__ int q_start(const Params& p, int s) { return p.cu ? p.cu[s] : s * p.q_len; }
__device__ __forceinline__ int q_count(const Params& p, int s) { return p.cu ? p.cu[s + 1] - p.cu[s] : p.q_len; }

__device__ __forceinline__ bool seq_has_tile(const Params& p, int s, int q0) {
  return s < p.num_seqs && q_count(p, s) > q0;
}

// Items at one level (warp-collective).
__device__ int level_count(const Params& p, int level) {
  const int lane = threadIdx.x & 31;
  const int q0 = level * p.tq;
  int n = 0;
  for (int b = 0; b < p.num_seqs; b += 32) n += __popc(__ballot_sync(0xffffffffu, seq_has_tile(p, b + lane, q0)));
  return n * p.hkv;
}

__device__ void walker_init(const Params& p, Walker& w) {
  w.taken = 0;
  w.level = p.n_qt - 1;
  w.base = 0;
  w.count = level_count(p, w.level);
}

// Next item of this CTA (warp-collective; identical result in every lane).
__device__ bool walker_next(const Params& p, Walker& w, Item& it) {
  const int lane = threadIdx.x & 31;
  const long long g2 = 2LL * gridDim.x;
  const long long r = static_cast<long long>(w.taken >> 1) * g2 +
                      ((w.taken & 1) ? (g2 - 1 - blockIdx.x) : static_cast<long long>(blockIdx.x));
  while (r >= w.base + w.count) {
    if (w.level == 0) return false;
    w.base += w.count;
    --w.level;
    w.count = level_count(p, w.level);
  }
  const int idx = static_cast<int>(r - w.base);
  const int ord = idx / p.hkv;  // the ord-th sequence (index order) that has this level's tile
  const int q0 = w.level * p.tq;
  int seen = 0, s = 0;
  for (int b = 0; b < p.num_seqs; b += 32) {
    const unsigned m = __ballot_sync(0xffffffffu, seq_has_tile(p, b + lane, q0));
    const int c = __popc(m);
    if (ord < seen + c) {
      unsigned mm = m;
      for (int k = seen; k < ord; ++k) mm &= mm - 1;  // drop the lower set bits
      s = b + __ffs(mm) - 1;
      break;
    }
    seen += c;
  }
  it.s = s;
  it.h = idx - ord * p.hkv;
  it.seq0 = q_start(p, s);
  it.L = q_count(p, s);
  it.K = p.paged ? max(p.k_lens[s], 0) : it.L;
  it.off = it.K - it.L;
  it.q0 = q0;
  const int kv_end = p.causal ? min(q0 + p.tq + it.off, it.K) : it.K;
  // At least one tile, so every item runs the same pipeline (rows that see
  // no key come out as zeros).
  it.n_kv = max((kv_end + kKeys - 1) / kKeys, 1);
  ++w.taken;
  return true;
}

__global__ void __launch_bounds__(kThreads, 2)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQTile;                // 2 stages
  uint8_t* sV = smem + kQTile + 2 * kKVTile;  // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOffset);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [2]  K ring: freed once QK^T has read it
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]  V ring: freed once PV has read it
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [2]  S_j in TMEM buffer j%2
  uint64_t* s_empty = bars + 12;  // [2]  buffer j%2 free: PV_j (which read P_j from it) done
  uint64_t* p_full = bars + 14;   // [2]  P_j written over S_j
  uint64_t* o_done = bars + 16;   // [2]  PV_j done (barrier j%2: a parity wait is never 2 phases behind)
  uint64_t* o_empty = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const float NEG_INF = -__int_as_float(0x7f800000);

  grid_dependency_wait();
  {  // a CTA without work leaves before touching barriers or TMEM
    Walker w;
    walker_init(p, w);
    Item it;
    if (!walker_next(p, w, it)) return;
  }
  if (smem_u32(smem) & 1023u) {  // the swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, LA_DEVERR_SMEM_ALIGN);
    return;
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(o_empty, 128);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (lane 0 issues)
    // Two streams over the CTA's KV tiles in global order: K runs one tile
    // ahead of V (issue order K(t+1), V(t)), so a K load waits only for the
    // QK^T two tiles back, never for a PV. Q of a new item is loaded just
    // before that item's first K.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    Walker wk, wv;
    walker_init(p, wk);
    walker_init(p, wv);
    Item ik, iv;
    bool k_more = walker_next(p, wk, ik), v_more = walker_next(p, wv, iv);
    int jk = 0, jv = 0;  // tile index within the K / V stream's current item
    int tk = 0, tv = 0;  // global tile counters of the two streams
    int items_q = 0;     // items whose Q has been loaded
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err, LA_DEVERR_WAIT_TIMEOUT));
    };
    // One 64-key K or V tile (both 64-dim halves) of item `it`, tile j. Paged:
    // one box per run of box_keys keys, through the block table; keys at or
    // past the sequence's end, and ids outside the table or the pool (also
    // reported), load from block `num_blocks`, outside the tensor map, which
    // the copy engine fills with zeros. Either way the full tile's bytes land.
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
    // Issue K tile tk (loading the item's Q first when it is the item's first tile).
    auto issue_k = [&]() -> bool {
      if (jk == 0) {
        if (lane == 0 && ik.q0 == (p.n_qt - 1) * p.tq && ik.L > p.n_qt * p.tq && p.err)
          atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
        // Q of item k replaces item k-1's once its last QK^T has completed.
        if (!wait_all(q_empty, (items_q & 1) ^ 1u)) return false;
        if (lane == 0) {
          mbar_arrive_expect_tx(q_full, kQTile);
          for (int g = 0; g < p.group; ++g)
            for (int half = 0; half < 2; ++half)
              tma_load_3d(sQ + half * kQHalf + g * p.tq * 128, &tm_q, q_full, half * 64, ik.h * p.group + g,
                          ik.seq0 + ik.q0);
        }
        ++items_q;
      }
      const int st = tk & 1;
      if (!wait_all(&k_empty[st], ((tk >> 1) & 1) ^ 1u)) return false;
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[st], kKVTile);
        load_kv(sK + st * kKVTile, &tm_k, &k_full[st], ik, jk);
      }
      ++tk;
      if (++jk == ik.n_kv) {
        jk = 0;
        k_more = walker_next(p, wk, ik);
      }
      return true;
    };
    auto issue_v = [&]() -> bool {
      const int st = tv & 1;
      if (!wait_all(&v_empty[st], ((tv >> 1) & 1) ^ 1u)) return false;
      if (lane == 0) {
        mbar_arrive_expect_tx(&v_full[st], kKVTile);
        load_kv(sV + st * kKVTile, &tm_v, &v_full[st], iv, jv);
      }
      ++tv;
      if (++jv == iv.n_kv) {
        jv = 0;
        v_more = walker_next(p, wv, iv);
      }
      return true;
    };
    if (k_more) ok = issue_k();  // K(0)
    while (ok && v_more) {
      if (k_more && !(ok = issue_k())) break;  // K(t+1)
      ok = issue_v();                           // V(t)
    }
    if (!ok && lane == 0) {  // early exit: let the copies already issued land (bounded)
      for (int u = (tk > 2 ? tk - 2 : 0); u < tk; ++u) mbar_wait(&k_full[u & 1], (u >> 1) & 1, nullptr, 0);
      for (int u = (tv > 2 ? tv - 2 : 0); u < tv; ++u) mbar_wait(&v_full[u & 1], (u >> 1) & 1, nullptr, 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (lane 0 issues)
    Walker w;
    walker_init(p, w);
    Item it;
    int k = 0, t = 0;
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err, LA_DEVERR_WAIT_TIMEOUT));
    };
    auto pv = [&](int u, int ju, int kk) -> bool {  // O += P V for global tile u (item-local ju)
      if (!wait_all(&p_full[u & 1], (u >> 1) & 1) || !wait_all(&v_full[u & 1], (u >> 1) & 1)) return false;
      if (ju == 0 && kk >= 1 && !wait_all(o_empty, (kk - 1) & 1)) return false;
      const int vrows = it.K - ju * kKeys;  // valid V rows of this tile
      if (p.paged && vrows < kKeys) {
        // Pool slots past the sequence's last key hold whatever was there
        // (possibly NaN); P is 0 for them but 0 * NaN is not, so zero them.
        uint8_t* vt = sV + (u & 1) * kKVTile;
        const int r0 = max(vrows, 0);
        const int n16 = (kKeys - r0) * 8;  // 16-byte chunks per half
        for (int i = lane; i < 2 * n16; i += 32) {
          const int half = i / n16, c = i - half * n16;
          *reinterpret_cast<uint4*>(vt + half * kKVHalf + r0 * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint8_t* vt = sV + (u & 1) * kKVTile;
        const uint32_t pt = tmem + (u & 1) * kKeys;  // P_u: 16 keys per 8 columns
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          umma_f16_ts(tmem + kColO, pt + ks * 8, desc_v(vt, ks), kIdescPV, (ju > 0 || ks > 0) ? 1u : 0u);
        umma_commit(&o_done[u & 1]);
        umma_commit(&v_empty[u & 1]);
        umma_commit(&s_empty[u & 1]);  // S/P buffer u%2 may take S_{u+2}
      }
      __syncwarp();
      return true;
    };
    while (ok && walker_next(p, w, it)) {
      if (!wait_all(q_full, k & 1)) break;
      const int t0 = t;
      for (int j = 0; j < it.n_kv; ++j, ++t) {
        const int st = t & 1;
        ok = wait_all(&k_full[st], (t >> 1) & 1) && wait_all(&s_empty[st], ((t >> 1) & 1) ^ 1u);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint8_t* kt = sK + st * kKVTile;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16_ss(tmem + st * kKeys, desc_kmajor(sQ, kQHalf, ks), desc_kmajor(kt, kKVHalf, ks), kIdescQK,
                        ks > 0 ? 1u : 0u);
          umma_commit(&s_full[st]);
          umma_commit(&k_empty[st]);  // K tile read
          if (j == it.n_kv - 1) umma_commit(q_empty);  // this item's Q is no longer read
        }
        __syncwarp();
        if (j >= 1 && !(ok = pv(t - 1, j - 1, k))) break;
      }
      if (!ok || !(ok = pv(t0 + it.n_kv - 1, it.n_kv - 1, k))) break;
      ++k;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int g = row / p.tq;
    const float sl2 = p.scale_log2;
    Walker w;
    walker_init(p, w);
    Item it;
    int k = 0, t = 0;
    bool ok = true;
    while (ok && walker_next(p, w, it)) {
      const int tok = it.q0 + (row - g * p.tq);  // token index within the sequence
      const int lim = p.causal ? min(max(tok + 1 + it.off, 0), it.K) : it.K;  // keys [0, lim) are visible
      float m = NEG_INF, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++t) {
        const int sb = t & 1;
        // tcgen05.ld is warp-collective: keep the decision to continue warp-uniform
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (t >> 1) & 1, p.err, LA_DEVERR_WAIT_TIMEOUT))) {
          ok = false;
          break;
        }
        tc_fence_after();
        constexpr int kC = kKeys / 32;  // 32-column TMEM loads per row
        float sv[kC][32];
#pragma unroll
        for (int c = 0; c < kC; ++c) tmem_ld32(taddr + sb * kKeys + c * 32, sv[c]);
        tc_wait_ld();

        // Row max of the raw scores with 8 independent partial maxima (short
        // dependency chains: one warp per scheduler cannot hide a 128-long one).
        const int nvis = lim - j * kKeys;  // visible columns of this tile
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = NEG_INF;
        if (__all_sync(0xffffffffu, nvis >= kKeys)) {  // whole tile visible: no mask
#pragma unroll
          for (int c = 0; c < kC; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], sv[c][e]);
        } else {
#pragma unroll
          for (int c = 0; c < kC; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float x = (c * 32 + e < nvis) ? sv[c][e] : NEG_INF;
              sv[c][e] = x;
              mx[e & 7] = fmaxf(mx[e & 7], x);
            }
        }
        const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
        const float m_new = (mt > m + 8.f) ? mt : m;
        // A row that has seen no key yet keeps m = -inf: use 0 as its
        // reference so P and alpha come out 0 instead of NaN.
        const float m_ref = (m_new == NEG_INF) ? 0.f : m_new;
        const float alpha = ex2(m - m_ref);  // 0 on the first tile, 1 when m is kept
        const float neg_m = -m_ref;
        float ps[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) ps[a] = 0.f;
#pragma unroll
        for (int c = 0; c < kC; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float pe = ex2(fmaf(sv[c][e], sl2, neg_m));  // masked: -inf -> 0
            sv[c][e] = pe;
            ps[e & 7] += pe;
          }
        const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        l = l * alpha + rs;
        // O is rescaled only when a row of this warp raised its max; then
        // PV of the previous tile must be complete first. (An item's first
        // tile needs neither: its PV overwrites O.)
        if (j >= 1 && __any_sync(0xffffffffu, m_new != m)) {
          const int u = t - 1;
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[u & 1], (u >> 1) & 1, p.err, LA_DEVERR_WAIT_TIMEOUT))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(taddr + kColO + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(taddr + kColO + c * 32, o);
          }
        }
        m = m_new;
        // P row -> TMEM over the first 32 columns of S's buffer, bf16 pairs.
        {
          float pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = __uint_as_float(pack_bf16x2(sv[i >> 4][(i & 15) * 2], sv[i >> 4][(i & 15) * 2 + 1]));
          tmem_st32(taddr + sb * kKeys, pk);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!__all_sync(0xffffffffu, mbar_wait(&o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, p.err,
                                             LA_DEVERR_WAIT_TIMEOUT)))
        break;
      tc_fence_after();
      float o[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(taddr + kColO + c * 32, o[c]);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(o_empty);  // O may now be overwritten by the next item's first PV
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int qh = it.h * p.group + g;
      if (p.lse && tok < it.L)
        p.lse[static_cast<long long>(qh) * p.total + it.seq0 + tok] =
            l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : NEG_INF;
      // O rows -> global through this warp's staging buffer, one 64-dim half
      // at a time: each thread writes its row (8 chunks of 16 B, XOR-swizzled
      // by row), then each store instruction writes 4 rows x 128 contiguous
      // bytes. Rows past the sequence's end are not stored.
      uint8_t* stage = smem + kStageOffset + quarter * kStageBytes;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int c = 2 * h2 + (ch >> 2), e0 = (ch & 3) * 8;
          uint4 u;
          u.x = pack_bf16x2(o[c][e0 + 0] * inv, o[c][e0 + 1] * inv);
          u.y = pack_bf16x2(o[c][e0 + 2] * inv, o[c][e0 + 3] * inv);
          u.z = pack_bf16x2(o[c][e0 + 4] * inv, o[c][e0 + 5] * inv);
          u.w = pack_bf16x2(o[c][e0 + 6] * inv, o[c][e0 + 7] * inv);
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((ch ^ (lane & 7)) << 4)) = u;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = i * 4 + (lane >> 3), ch = lane & 7;
          const int rrow = quarter * 32 + r;
          const int rg = rrow / p.tq;
          const int rtok = it.q0 + rrow - rg * p.tq;
          const uint4 u = *reinterpret_cast<const uint4*>(stage + r * 128 + ((ch ^ (r & 7)) << 4));
          if (rtok < it.L)
            *reinterpret_cast<uint4*>(p.out + static_cast<long long>(it.seq0 + rtok) * p.out_ts +
                                      static_cast<long long>(it.h * p.group + rg) * p.out_hs + h2 * 64 + ch * 8) = u;
        }
        __syncwarp();
      }
      ++k;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill

int prefill_init(int device) {
  (void)device;
  cudaError_t e = cudaFuncSetAttribute(prefill::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(prefill::kSmemBytes));
  // all of the unified L1/shared storage as shared memory, so two CTAs fit
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill::prefill_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  return cuda_status(e);
}

}  // namespace la

namespace la {
namespace prefill {

// Common tail of the two entry points: the persistent grid over the items.
static int launch(const CUtensorMap& tq_map, const CUtensorMap& tk_map, const CUtensorMap& tv_map, const Params& p,
                  cudaStream_t stream) {
  const long long items = static_cast<long long>(p.n_qt) * p.num_seqs * p.hkv;
  if (items > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  const int device = current_device();
  const int sms = device >= 0 ? num_sms(device) : 0;
  if (sms <= 0) return LA_ERR_CUDA;
  // Two CTAs per SM by design (registers, shared memory and TMEM are sized
  // for it); if fewer fit, the extra CTAs simply run as a second wave.
  const long long ctas = static_cast<long long>(sms) * 2;
  const dim3 grid(static_cast<unsigned>(items < ctas ? items : ctas));  // persistent
  return cuda_status(launch_pdl(prefill_kernel, grid, dim3(kThreads), kSmemBytes, stream, tq_map, tk_map, tv_map, p));
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
  p->hq = num_q_heads;
  p->hkv = num_kv_heads;
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
  p.n_qt = (max_seqlen + p.tq - 1) / p.tq;
  p.causal = causal ? 1 : 0;
  p.lse = softmax_lse;
  p.err = dev_error;
  return launch(tq_map, tk_map, tv_map, p, stream);
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
  // 64-key tiles must not straddle blocks, or be whole blocks of 16 / 32.
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
  p.n_qt = (max_seqlen_q + p.tq - 1) / p.tq;
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
  return launch(tq_map, tk_map, tv_map, p, stream);
}
