// Decode-step glue around the attention path, fused so each is one launch:
//   la_add_rms_norm: h' = h + a (bf16), x = RMSNorm(h') * w — the residual add
//     that closes a sub-layer and the RMSNorm that opens the next one
//     (Qwen3DecoderLayer, leaninfer/qwen3/model.py:80-83; nn.RMSNorm at
//     model.py:75-76, 92).
//   la_silu_mul: SiLU(gate) * up on the fused gate_up projection
//     (Qwen3MLP, model.py:32-33).
// Both read their inputs once and round their outputs to bf16 once, from fp32.
//   la_argmax_rows: the greedy next token, logits[:, -1].argmax(-1)
//     (leaninfer/engine/llm_engine.py:86, 111, 135), with torch.argmax's
//     rules: the first index of the maximum, and NaN above every number.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "la_internal.h"
#include "la_ptx.cuh"

namespace la {
namespace elementwise {

constexpr int kThreads = 128;

struct NormParams {
  const __nv_bfloat16* h;    // residual stream in [rows, n]
  const __nv_bfloat16* a;    // addend [rows, n] or null
  __nv_bfloat16* h_out;      // h + a [rows, n] or null (may alias h)
  __nv_bfloat16* x_out;      // RMSNorm(h + a) * w
  const __nv_bfloat16* w;    // [n]
  long long h_rs, a_rs, ho_rs, xo_rs;  // row strides (elements)
  int n;
  float eps;
};

// One CTA per row; each thread handles 8 consecutive elements per pass.
__global__ void __launch_bounds__(kThreads) add_rms_norm_kernel(const NormParams p) {
  grid_dependency_wait();
  grid_launch_dependents();
  const long long row = blockIdx.x;
  const __nv_bfloat16* h = p.h + row * p.h_rs;
  const __nv_bfloat16* a = p.a ? p.a + row * p.a_rs : nullptr;
  constexpr int kMaxPer = 4;  // up to 4 x 8 x 128 = 4096 elements per row in registers
  float v[kMaxPer][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int c = (it * kThreads + threadIdx.x) * 8;
    if (c < p.n) {
      const uint4 hu = *reinterpret_cast<const uint4*>(h + c);
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&hu);
      uint4 au = make_uint4(0u, 0u, 0u, 0u);
      if (a) au = *reinterpret_cast<const uint4*>(a + c);
      const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&au);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // the residual stream stays bf16: round the sum once, then use it
        const float s = a ? __bfloat162float(__float2bfloat16_rn(__bfloat162float(hb[e]) + __bfloat162float(ab[e])))
                          : __bfloat162float(hb[e]);
        v[it][e] = s;
        ss = fmaf(s, s, ss);
      }
      if (a && p.h_out) {
        uint4 o;
        o.x = pack_bf16x2(v[it][0], v[it][1]);
        o.y = pack_bf16x2(v[it][2], v[it][3]);
        o.z = pack_bf16x2(v[it][4], v[it][5]);
        o.w = pack_bf16x2(v[it][6], v[it][7]);
        *reinterpret_cast<uint4*>(p.h_out + row * p.ho_rs + c) = o;
      }
    }
  }
  __shared__ float red[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(p.n) + p.eps);
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int c = (it * kThreads + threadIdx.x) * 8;
    if (c < p.n) {
      const uint4 wu = *reinterpret_cast<const uint4*>(p.w + c);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = v[it][e] * r * __bfloat162float(wb[e]);
      uint4 o;
      o.x = pack_bf16x2(y[0], y[1]);
      o.y = pack_bf16x2(y[2], y[3]);
      o.z = pack_bf16x2(y[4], y[5]);
      o.w = pack_bf16x2(y[6], y[7]);
      *reinterpret_cast<uint4*>(p.x_out + row * p.xo_rs + c) = o;
    }
  }
}

struct SiluParams {
  const __nv_bfloat16* gu;  // [rows, 2 * n]: gate | up
  __nv_bfloat16* out;       // [rows, n]
  long long gu_rs, out_rs;
  int n;
  long long total8;         // rows * n / 8
};

__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  grid_dependency_wait();
  grid_launch_dependents();
  const long long i8 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i8 >= p.total8) return;
  const int per_row = p.n / 8;
  const long long row = i8 / per_row;
  const int c = static_cast<int>(i8 - row * per_row) * 8;
  const uint4 gu = *reinterpret_cast<const uint4*>(p.gu + row * p.gu_rs + c);
  const uint4 uu = *reinterpret_cast<const uint4*>(p.gu + row * p.gu_rs + p.n + c);
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gu);
  const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uu);
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x = __bfloat162float(g[e]);
    y[e] = x / (1.f + __expf(-x)) * __bfloat162float(u[e]);
  }
  uint4 o;
  o.x = pack_bf16x2(y[0], y[1]);
  o.y = pack_bf16x2(y[2], y[3]);
  o.z = pack_bf16x2(y[4], y[5]);
  o.w = pack_bf16x2(y[6], y[7]);
  *reinterpret_cast<uint4*>(p.out + row * p.out_rs + c) = o;
}

// ---------------------------------------------------------------- argmax
// Order key of a bf16 value: larger key = larger value, equal values (+0 and
// -0 included) get equal keys, every NaN gets the largest key.
__device__ __forceinline__ uint32_t argmax_key(uint32_t b) {
  b &= 0xffffu;
  if ((b & 0x7fffu) > 0x7f80u) return 0x10000u;
  if (b == 0x8000u) b = 0u;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxUnroll = 8;  // 16-byte loads in flight per thread

struct ArgmaxParams {
  const __nv_bfloat16* x;
  long long rs;  // row stride (elements)
  int cols;
  int vec;       // every row starts 16-byte aligned: 8-element chunks
  long long* out;
};

// One CTA per row. Thread t reads chunks t, t + 512, ... of 8 values with
// 16-byte loads and keeps the first chunk holding its largest key (a chunk's
// max from three packed bf16x2 max operations, NaN-propagating); afterwards it
// finds the first index of that key inside the chunk, and the block keeps the
// largest key with the smallest index.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const ArgmaxParams p) {
  grid_dependency_wait();
  grid_launch_dependents();
  const __nv_bfloat16* row = p.x + static_cast<long long>(blockIdx.x) * p.rs;
  const int t = threadIdx.x;
  uint32_t best = 0;  // below every key
  int best_idx = 0x7fffffff;
  const int nchunk = p.vec ? p.cols / 8 : 0;
  int best_chunk = -1;
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  for (int c0 = t; c0 < nchunk; c0 += kArgmaxThreads * kArgmaxUnroll) {
    uint4 u[kArgmaxUnroll];
#pragma unroll
    for (int k = 0; k < kArgmaxUnroll; ++k) {
      const int c = c0 + k * kArgmaxThreads;
      if (c < nchunk) u[k] = __ldcs(rv + c);  // read once: do not keep in L1/L2
    }
#pragma unroll
    for (int k = 0; k < kArgmaxUnroll; ++k) {
      const int c = c0 + k * kArgmaxThreads;
      if (c < nchunk) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[k]);
        const __nv_bfloat162 m2 = __hmax2_nan(__hmax2_nan(h[0], h[1]), __hmax2_nan(h[2], h[3]));
        const uint32_t mb = *reinterpret_cast<const uint32_t*>(&m2);
        const uint32_t key = max(argmax_key(mb), argmax_key(mb >> 16));
        if (key > best) {
          best = key;
          best_chunk = c;
        }
      }
    }
  }
  if (best_chunk >= 0) {  // first element of the chunk with the chunk's best key
    const uint4 u = rv[best_chunk];
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
    for (int k = 7; k >= 0; --k)
      if (argmax_key(e[k]) == best) best_idx = best_chunk * 8 + k;
  }
  // Elements outside the chunks (the tail, or every element when rows are not
  // 16-byte aligned): indices above every chunk, visited in increasing order.
  const uint16_t* rb = reinterpret_cast<const uint16_t*>(row);
  for (int i = nchunk * 8 + t; i < p.cols; i += kArgmaxThreads) {
    const uint32_t key = argmax_key(rb[i]);
    if (key > best) {
      best = key;
      best_idx = i;
    }
  }
  // Largest key, then smallest index.
  unsigned long long v = (static_cast<unsigned long long>(best) << 32) | static_cast<uint32_t>(~best_idx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __shared__ unsigned long long part[kArgmaxThreads / 32];
  if ((t & 31) == 0) part[t >> 5] = v;
  __syncthreads();
  if (t < 32) {
    v = t < kArgmaxThreads / 32 ? part[t] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w > v ? w : v;
    }
    if (t == 0) p.out[blockIdx.x] = static_cast<long long>(~static_cast<uint32_t>(v));
  }
}

}  // namespace elementwise
}  // namespace la

extern "C" int la_add_rms_norm(const void* h, int64_t h_row_stride, const void* a, int64_t a_row_stride, void* h_out,
                               int64_t h_out_row_stride, void* x_out, int64_t x_out_row_stride, const void* weight,
                               int64_t rows, int n, float eps, cudaStream_t stream) {
  using namespace la;
  using namespace la::elementwise;
  if (!h || !x_out || !weight || rows < 0 || n <= 0) return LA_ERR_INVALID_ARGUMENT;
  if (n % 8 || n > 4 * 8 * kThreads) return LA_ERR_UNSUPPORTED;
  if (rows == 0) return LA_OK;
  if (rows > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  const void* ptrs[] = {h, a, h_out, x_out, weight};
  for (const void* q : ptrs)
    if (q && !aligned(q, 16)) return LA_ERR_ALIGNMENT;
  const long long st[] = {h_row_stride, a ? a_row_stride : h_row_stride, h_out ? h_out_row_stride : h_row_stride,
                          x_out_row_stride};
  for (long long x : st)
    if (x < n || x % 8) return LA_ERR_ALIGNMENT;
  NormParams p;
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.h_out = static_cast<__nv_bfloat16*>(h_out);
  p.x_out = static_cast<__nv_bfloat16*>(x_out);
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.h_rs = h_row_stride;
  p.a_rs = a_row_stride;
  p.ho_rs = h_out_row_stride;
  p.xo_rs = x_out_row_stride;
  p.n = n;
  p.eps = eps;
  return cuda_status(launch_pdl(add_rms_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kThreads), 0, stream, p));
}

extern "C" int la_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride,
                           int64_t rows, int n, cudaStream_t stream) {
  using namespace la;
  using namespace la::elementwise;
  if (!gate_up || !out || rows < 0 || n <= 0) return LA_ERR_INVALID_ARGUMENT;
  if (n % 8) return LA_ERR_UNSUPPORTED;
  if (rows == 0) return LA_OK;
  if (!aligned(gate_up, 16) || !aligned(out, 16)) return LA_ERR_ALIGNMENT;
  if (gate_up_row_stride < 2LL * n || gate_up_row_stride % 8 || out_row_stride < n || out_row_stride % 8)
    return LA_ERR_ALIGNMENT;
  SiluParams p;
  p.gu = static_cast<const __nv_bfloat16*>(gate_up);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.gu_rs = gate_up_row_stride;
  p.out_rs = out_row_stride;
  p.n = n;
  p.total8 = rows * (n / 8);
  const long long blocks = (p.total8 + 255) / 256;
  if (blocks > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  return cuda_status(launch_pdl(silu_mul_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, p));
}

extern "C" int la_argmax_rows(const void* x, int64_t row_stride, int64_t rows, int64_t cols, int64_t* out,
                              cudaStream_t stream) {
  using namespace la;
  using namespace la::elementwise;
  if (!x || !out || rows < 0 || cols <= 0 || cols > 0x7fffffffLL - 8 || row_stride < cols)
    return LA_ERR_INVALID_ARGUMENT;
  if (rows > 0x7fffffffLL) return LA_ERR_UNSUPPORTED;
  if (rows == 0) return LA_OK;
  if (!aligned(x, 2) || !aligned(out, 8)) return LA_ERR_ALIGNMENT;
  ArgmaxParams p;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.rs = row_stride;
  p.cols = static_cast<int>(cols);
  p.vec = aligned(x, 16) && row_stride % 8 == 0;
  p.out = reinterpret_cast<long long*>(out);
  return cuda_status(
      launch_pdl(argmax_rows_kernel, dim3(static_cast<unsigned>(rows)), dim3(kArgmaxThreads), 0, stream, p));
}
