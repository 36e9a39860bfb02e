// (a) Fused pre-attention kernel: per-head QK RMSNorm + NeoX RoPE + paged KV
// scatter, one warp per (token, head row).
//
// Reference op sequence (one layer), all replaced by one launch:
//   q = q_norm(q.view(b, n, Hq, D))              leaninfer/qwen3/model.py:50
//   k = k_norm(k.view(b, n, Hkv, D))             model.py:51
//   q, k = apply_rope(q|k, cos, sin)             model.py:53-54, layers.py:18-23
//   cache.write(layer, block_tables, pos, k, v)  model.py:55, cache_manager.py:63-76
//
// Rounding follows the reference exactly: RMSNorm in fp32 — sum of squares,
// mean, +eps, 1/sqrt, x*r, *w — rounded once to bf16; then x*cos and
// rotate_half(x)*sin each rounded to bf16 and their fp32 sum rounded to bf16.
// The only freedom is the order of the 128-term fp32 sum of squares: here each
// lane adds its 4 squares left to right, then a 5-step xor butterfly
// (offsets 16, 8, 4, 2, 1). The oracle restates that order, so the kernel is
// bit-exact against it; against torch's own reduction order the normalised
// values can differ by one bf16 ulp in a few elements per million.
//
// cos/sin come from [max_pos, D/2] bf16 tables built once with the reference's
// formula (layers.py:7-15); cos[p, d] for d >= D/2 equals cos[p, d - D/2]
// because build_rope concatenates the angles with themselves.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace pre {

constexpr int kD = 128;
constexpr int kWarps = 8;

struct Params {
  const __nv_bfloat16* q;
  long long q_ts, q_hs;
  const __nv_bfloat16* k;
  long long k_ts, k_hs;
  const __nv_bfloat16* v;
  long long v_ts, v_hs;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  float eps;
  const __nv_bfloat16* rcos;
  const __nv_bfloat16* rsin;
  long long max_pos;
  const long long* pos;
  const int* cu;
  int num_seqs, q_len;
  long long num_tokens;
  const int* bt;
  long long bt_stride;
  int max_blocks;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  long long kv_bs, kv_ts, kv_hs;
  long long nb;
  int bs;
  __nv_bfloat16* qo;
  long long qo_ts, qo_hs;
  __nv_bfloat16* ko;  // optional contiguous copy of the rotated k
  long long ko_ts, ko_hs;
  int hq, hkv;
  bool norm_rope;  // false: plain scatter of k/v (no q)
  int* err;
};

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  x[0] = __uint_as_float(u.x << 16);
  x[1] = __uint_as_float(u.x & 0xffff0000u);
  x[2] = __uint_as_float(u.y << 16);
  x[3] = __uint_as_float(u.y & 0xffff0000u);
}

__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&x)[4]) {
  uint2 u;
  u.x = pack_bf16x2(x[0], x[1]);
  u.y = pack_bf16x2(x[2], x[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// RMSNorm of one 128-wide row held 4 per lane, then RoPE; x is replaced by the
// bf16-rounded result (as fp32 values).
__device__ __forceinline__ void norm_rope_row(float (&x)[4], const float (&w)[4], const float (&c)[4],
                                              const float (&s)[4], float eps, int lane) {
  float ss = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])), __fmul_rn(x[2], x[2])),
                       __fmul_rn(x[3], x[3]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float mean = __fmul_rn(ss, 1.0f / 128.0f);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = bf16_round(__fmul_rn(__fmul_rn(x[i], r), w[i]));
  // rotate_half: lanes 0-15 hold dims 0..63 and need -x[d + 64] (lane + 16);
  // lanes 16-31 hold dims 64..127 and need x[d - 64] (lane - 16).
  float part[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float rh = lo ? -part[i] : part[i];
    const float a = bf16_round(__fmul_rn(y[i], c[i]));
    const float b = bf16_round(__fmul_rn(rh, s[i]));
    x[i] = bf16_round(__fadd_rn(a, b));
  }
}

// One warp per (token, row): rows 0..Hq-1 are q heads, then Hkv k heads, then
// Hkv v heads (no q rows and no norm for the plain write). Every warp does one
// load -> (norm, rope) -> store chain, so the launch is one memory round trip
// deep whatever the head count.
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_write_kernel(const Params p) {
  grid_dependency_wait();
  // Let the attention kernel that follows start its prologue.
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int rows = p.hq + 2 * p.hkv;
  const long long wg = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const long long tok = wg / rows;
  const int r = static_cast<int>(wg - tok * rows);
  if (tok >= p.num_tokens) return;

  int s;
  long long t;
  if (p.cu == nullptr) {
    s = static_cast<int>(tok / p.q_len);
    t = tok - static_cast<long long>(s) * p.q_len;
  } else {
    int lo = 0, hi = p.num_seqs;  // find s with cu[s] <= tok < cu[s + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.cu[mid] <= tok) lo = mid;
      else hi = mid;
    }
    s = lo;
    t = tok - p.cu[s];
  }
  const long long col = p.pos[s] + t;
  const int d0 = lane * 4;
  if (p.pos[s] < 0) {  // idle sequence: no cache write, zero outputs, no error
    const float z[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < p.hq) {
      store4(p.qo + tok * p.qo_ts + r * p.qo_hs + d0, z);
    } else if (r < p.hq + p.hkv && p.ko) {
      store4(p.ko + tok * p.ko_ts + (r - p.hq) * p.ko_hs + d0, z);
    }
    return;
  }

  if (r < p.hq) {  // q row: norm + rope -> q_out
    float c[4], sn[4], w[4], x[4];
    long long rp = col;
    if (rp < 0 || rp >= p.max_pos) {
      if (p.err) atomicCAS(p.err, 0, LA_DEVERR_ROPE_POS);
      rp = 0;
    }
    load4(p.q + tok * p.q_ts + r * p.q_hs + d0, x);
    load4(p.rcos + rp * (kD / 2) + (d0 & 63), c);
    load4(p.rsin + rp * (kD / 2) + (d0 & 63), sn);
    load4(p.qw + d0, w);
    norm_rope_row(x, w, c, sn, p.eps, lane);
    store4(p.qo + tok * p.qo_ts + r * p.qo_hs + d0, x);
    return;
  }

  // k or v row: destination row in the paged cache.
  const bool is_k = r < p.hq + p.hkv;
  const int h = is_k ? r - p.hq : r - p.hq - p.hkv;
  long long dst = -1;
  if (col >= 0) {
    const long long lb = col / p.bs;
    if (lb < p.max_blocks) {
      const int phys = p.bt[static_cast<long long>(s) * p.bt_stride + lb];
      if (phys >= 0 && phys < p.nb) dst = phys * p.kv_bs + (col - lb * p.bs) * p.kv_ts;
      else if (p.err) atomicCAS(p.err, 0, LA_DEVERR_BLOCK_ID);
    } else if (p.err) {
      atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
    }
  } else if (p.err) {
    atomicCAS(p.err, 0, LA_DEVERR_SEQLEN);
  }

  if (is_k && p.norm_rope) {
    float c[4], sn[4], w[4], x[4];
    long long rp = col;
    if (rp < 0 || rp >= p.max_pos) {
      if (p.err) atomicCAS(p.err, 0, LA_DEVERR_ROPE_POS);
      rp = 0;
    }
    load4(p.k + tok * p.k_ts + h * p.k_hs + d0, x);
    load4(p.rcos + rp * (kD / 2) + (d0 & 63), c);
    load4(p.rsin + rp * (kD / 2) + (d0 & 63), sn);
    load4(p.kw + d0, w);
    norm_rope_row(x, w, c, sn, p.eps, lane);
    if (dst >= 0) store4(p.kc + dst + h * p.kv_hs + d0, x);
    if (p.ko) store4(p.ko + tok * p.ko_ts + h * p.ko_hs + d0, x);
  } else if (dst >= 0) {  // plain copy: v rows, and k rows of the plain write
    const __nv_bfloat16* src = is_k ? p.k + tok * p.k_ts + h * p.k_hs : p.v + tok * p.v_ts + h * p.v_hs;
    __nv_bfloat16* dc = (is_k ? p.kc : p.vc) + dst + h * p.kv_hs;
    *reinterpret_cast<uint2*>(dc + d0) = *reinterpret_cast<const uint2*>(src + d0);
  }
}

static int check_common(const Params& p) {
  if (p.num_tokens < 0 || p.num_seqs < 0) return LA_ERR_INVALID_ARGUMENT;
  if (!p.k || !p.v || !p.pos || !p.bt || !p.kc || !p.vc) return LA_ERR_INVALID_ARGUMENT;
  if (p.cu == nullptr) {
    if (p.q_len <= 0 || p.num_tokens != static_cast<long long>(p.num_seqs) * p.q_len) return LA_ERR_INVALID_ARGUMENT;
  } else if (p.num_seqs <= 0) {
    return LA_ERR_INVALID_ARGUMENT;
  }
  if (p.bs <= 0 || p.nb <= 0 || p.max_blocks <= 0 || p.hkv <= 0) return LA_ERR_INVALID_ARGUMENT;
  // 8-byte vector accesses of 4 bf16 per lane.
  const long long st[] = {p.k_ts, p.k_hs, p.v_ts, p.v_hs, p.kv_bs, p.kv_ts, p.kv_hs};
  for (long long x : st)
    if (x % 4) return LA_ERR_ALIGNMENT;
  if (!aligned(p.k, 8) || !aligned(p.v, 8) || !aligned(p.kc, 8) || !aligned(p.vc, 8)) return LA_ERR_ALIGNMENT;
  return LA_OK;
}

static int launch(const Params& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return LA_OK;
  const long long warps = p.num_tokens * (p.hq + 2 * p.hkv);
  const long long blocks = (warps + kWarps - 1) / kWarps;
  if (blocks > 0x7fffffffLL) return LA_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_pdl(qk_norm_rope_write_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kWarps * 32), 0,
                                stream, p));
}

}  // namespace pre

int pre_attn_init(int device) {
  (void)device;
  cudaFuncAttributes a;
  return cuda_status(cudaFuncGetAttributes(&a, pre::qk_norm_rope_write_kernel));
}

}  // namespace la

extern "C" int la_qk_norm_rope_paged_write(
    const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k, int64_t k_token_stride,
    int64_t k_head_stride, const void* v, int64_t v_token_stride, int64_t v_head_stride, const void* q_norm_weight,
    const void* k_norm_weight, float eps, const void* rope_cos, const void* rope_sin, int64_t rope_max_pos,
    const int64_t* seq_start_pos, const int32_t* cu_seqlens, int num_seqs, int q_len, int64_t num_tokens,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq, void* k_cache, void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride, int64_t num_blocks, int block_size,
    void* q_out, int64_t qo_token_stride, int64_t qo_head_stride, void* k_out, int64_t ko_token_stride,
    int64_t ko_head_stride, int num_q_heads, int num_kv_heads, int head_dim, int* dev_error, cudaStream_t stream) {
  using namespace la;
  if (head_dim != pre::kD) return LA_ERR_UNSUPPORTED;
  pre::Params p = {};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_ts = q_token_stride;
  p.q_hs = q_head_stride;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_ts = k_token_stride;
  p.k_hs = k_head_stride;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_ts = v_token_stride;
  p.v_hs = v_head_stride;
  p.qw = static_cast<const __nv_bfloat16*>(q_norm_weight);
  p.kw = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.eps = eps;
  p.rcos = static_cast<const __nv_bfloat16*>(rope_cos);
  p.rsin = static_cast<const __nv_bfloat16*>(rope_sin);
  p.max_pos = rope_max_pos;
  p.pos = reinterpret_cast<const long long*>(seq_start_pos);
  p.cu = cu_seqlens;
  p.num_seqs = num_seqs;
  p.q_len = q_len;
  p.num_tokens = num_tokens;
  p.bt = block_table;
  p.bt_stride = bt_seq_stride;
  p.max_blocks = max_blocks_per_seq;
  p.kc = static_cast<__nv_bfloat16*>(k_cache);
  p.vc = static_cast<__nv_bfloat16*>(v_cache);
  p.kv_bs = kv_block_stride;
  p.kv_ts = kv_token_stride;
  p.kv_hs = kv_head_stride;
  p.nb = num_blocks;
  p.bs = block_size;
  p.qo = static_cast<__nv_bfloat16*>(q_out);
  p.qo_ts = qo_token_stride;
  p.qo_hs = qo_head_stride;
  p.ko = static_cast<__nv_bfloat16*>(k_out);
  p.ko_ts = ko_token_stride;
  p.ko_hs = ko_head_stride;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.norm_rope = true;
  p.err = dev_error;
  int st = pre::check_common(p);
  if (st != LA_OK) return st;
  if (!q || !q_out || !q_norm_weight || !k_norm_weight || !rope_cos || !rope_sin || rope_max_pos <= 0 ||
      num_q_heads <= 0)
    return LA_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f)) return LA_ERR_INVALID_ARGUMENT;
  const long long st2[] = {q_token_stride, q_head_stride, qo_token_stride, qo_head_stride,
                           k_out ? ko_token_stride : 0, k_out ? ko_head_stride : 0};
  for (long long x : st2)
    if (x % 4) return LA_ERR_ALIGNMENT;
  if (k_out && !aligned(k_out, 8)) return LA_ERR_ALIGNMENT;
  if (!aligned(q, 8) || !aligned(q_out, 8) || !aligned(q_norm_weight, 8) || !aligned(k_norm_weight, 8) ||
      !aligned(rope_cos, 8) || !aligned(rope_sin, 8))
    return LA_ERR_ALIGNMENT;
  return pre::launch(p, stream);
}

extern "C" int la_paged_kv_write(const void* k, int64_t k_token_stride, int64_t k_head_stride, const void* v,
                                 int64_t v_token_stride, int64_t v_head_stride, const int64_t* seq_start_pos,
                                 const int32_t* cu_seqlens, int num_seqs, int q_len, int64_t num_tokens,
                                 const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
                                 void* k_cache, void* v_cache, int64_t kv_block_stride, int64_t kv_token_stride,
                                 int64_t kv_head_stride, int64_t num_blocks, int block_size, int num_kv_heads,
                                 int head_dim, int* dev_error, cudaStream_t stream) {
  using namespace la;
  if (head_dim != pre::kD) return LA_ERR_UNSUPPORTED;
  pre::Params p = {};
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_ts = k_token_stride;
  p.k_hs = k_head_stride;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_ts = v_token_stride;
  p.v_hs = v_head_stride;
  p.pos = reinterpret_cast<const long long*>(seq_start_pos);
  p.cu = cu_seqlens;
  p.num_seqs = num_seqs;
  p.q_len = q_len;
  p.num_tokens = num_tokens;
  p.bt = block_table;
  p.bt_stride = bt_seq_stride;
  p.max_blocks = max_blocks_per_seq;
  p.kc = static_cast<__nv_bfloat16*>(k_cache);
  p.vc = static_cast<__nv_bfloat16*>(v_cache);
  p.kv_bs = kv_block_stride;
  p.kv_ts = kv_token_stride;
  p.kv_hs = kv_head_stride;
  p.nb = num_blocks;
  p.bs = block_size;
  p.hq = 0;
  p.hkv = num_kv_heads;
  p.norm_rope = false;
  p.err = dev_error;
  int st = pre::check_common(p);
  if (st != LA_OK) return st;
  return pre::launch(p, stream);
}
