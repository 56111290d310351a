// Row LayerNorm with an optional fused residual add.
//
//   ln     : h = LN(x)                      (reference ln_fwd,     src/fused_kernels.py:164-193)
//   add_ln : s = x + y (fp32, stored); h = LN(s)   (reference add_ln_fwd, src/fused_kernels.py:196-238)
//   ln with s : h = LN(x) and s = x (a copy of the input in x's dtype, written
//            while the row is in registers)
//
// Statistics are fp32 and two-pass in registers (mean, then the centred
// variance), rstd = rsqrtf(var + eps), then the affine and the cast -- the
// same order as the reference kernels (src/fused_kernels.py:79-161).
//
// One warp owns one row for d <= 1024: each lane holds NV groups of four
// consecutive columns, loaded with 128-bit (fp32) or 64-bit (fp16) vector
// loads when the row pointers allow it. Wider rows (<= 8192) use one
// 256-thread CTA per row with a shared-memory reduction. HBM-bound by design:
// bytes/row = d * (sizeof x + sizeof y + sizeof s + sizeof h).
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "tk_ptx.cuh"

namespace tk {
namespace ln {

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  static __device__ __forceinline__ void load(const float* p, bool vec, int n_valid, float (&v)[4]) {
    if (vec && n_valid == 4) {
      float4 t = __ldg(reinterpret_cast<const float4*>(p));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = i < n_valid ? __ldg(p + i) : 0.f;
    }
  }
  static __device__ __forceinline__ void store(float* p, bool vec, int n_valid, const float (&v)[4]) {
    if (vec && n_valid == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i < n_valid) p[i] = v[i];
    }
  }
};
template <>
struct Vec4<__half> {
  static __device__ __forceinline__ void load(const __half* p, bool vec, int n_valid, float (&v)[4]) {
    if (vec && n_valid == 4) {
      uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
      float2 a = __half22float2(*reinterpret_cast<__half2*>(&t.x));
      float2 b = __half22float2(*reinterpret_cast<__half2*>(&t.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = i < n_valid ? __half2float(p[i]) : 0.f;
    }
  }
  static __device__ __forceinline__ void store(__half* p, bool vec, int n_valid, const float (&v)[4]) {
    if (vec && n_valid == 4) {
      __half2 a = __floats2half2_rn(v[0], v[1]);
      __half2 b = __floats2half2_rn(v[2], v[3]);
      uint2 t;
      t.x = *reinterpret_cast<uint32_t*>(&a);
      t.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(p) = t;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i < n_valid) p[i] = __float2half_rn(v[i]);
    }
  }
};

struct Args {
  const void* x;
  const void* y;      // residual branch, may be null
  void* s;            // x + y (a copy of x when y is null), may be null
  const float* gamma;
  const float* beta;
  void* h;
  int64_t rows, d, ld_x, ld_y, ld_s, ld_h;
  float eps;
  bool vec;           // all row starts are vector aligned and d % 4 == 0
  const int* row_len; // optional prefix lengths: rows at position >= row_len[row / seq_len]
  int64_t seq_len;    //   get s = 0 and h = 0 (the harness's padded-token zeroing)
};

__device__ __forceinline__ bool row_is_padding(const Args& a, int64_t row) {
  return a.row_len != nullptr && (row % a.seq_len) >= a.row_len[row / a.seq_len];
}

// NV = groups of 4 columns per lane; d <= NV * 128.
template <int NV, typename TX, typename TY, typename TS, typename TH>
__global__ void __launch_bounds__(256, 3) ln_warp_rows(Args a) {
  grid_dep_wait();  // the previous kernel's outputs are complete and visible
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int d = static_cast<int>(a.d);
  const float inv_d = 1.f / static_cast<float>(d);

  for (int64_t row = warp; row < a.rows; row += nwarps) {
    const TX* xr = static_cast<const TX*>(a.x) + row * a.ld_x;
    const bool pad = row_is_padding(a, row);
    float v[NV][4];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      const int n = max(0, min(4, d - c));
      Vec4<TX>::load(xr + c, a.vec, n, v[i]);
      if (a.y != nullptr) {
        float w[4];
        Vec4<TY>::load(static_cast<const TY*>(a.y) + row * a.ld_y + c, a.vec, n, w);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[i][k] = pad ? 0.f : v[i][k] + w[k];
      }
      // s = x + y, or a copy of x when there is no y
      if (a.s != nullptr && n > 0) Vec4<TS>::store(static_cast<TS*>(a.s) + row * a.ld_s + c, a.vec, n, v[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) sum += v[i][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float t = (c + k < d) ? v[i][k] - mean : 0.f;
        sq += t * t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq * inv_d + a.eps);
    TH* hr = static_cast<TH*>(a.h) + row * a.ld_h;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      const int n = max(0, min(4, d - c));
      if (n <= 0) continue;
      // gamma/beta are re-read per row (L1-resident) to keep registers low
      float g[4], b[4], o[4];
      Vec4<float>::load(a.gamma + c, a.vec, n, g);
      Vec4<float>::load(a.beta + c, a.vec, n, b);
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = pad ? 0.f : (v[i][k] - mean) * rstd * g[k] + b[k];
      Vec4<TH>::store(hr + c, a.vec, n, o);
    }
  }
}

// The forward's LayerNorm (no residual branch, vector-aligned rows, d <= NV *
// 128): the same row math as ln_warp_rows, on a persistent grid where each
// warp loads its next row while it reduces, normalises and stores the
// current one, so a row's loads are always in flight behind the previous
// row's arithmetic and stores (one row at a time leaves the loads idle for
// the whole reduction).
template <int NV, typename TX, typename TS, typename TH>
__global__ void __launch_bounds__(256, 2) ln_warp_rows_prefetch(Args a) {
  grid_dep_wait();  // the previous kernel's outputs are complete and visible
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int d = static_cast<int>(a.d);
  const float inv_d = 1.f / static_cast<float>(d);
  int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  float cur[NV][4], nxt[NV][4];
  auto load_row = [&](int64_t r, float (&v)[NV][4]) {
    const TX* xr = static_cast<const TX*>(a.x) + r * a.ld_x;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      Vec4<TX>::load(xr + c, true, max(0, min(4, d - c)), v[i]);
    }
  };
  if (row < a.rows) load_row(row, cur);
  for (; row < a.rows; row += nwarps) {
    const int64_t next = row + nwarps;
    if (next < a.rows) load_row(next, nxt);  // in flight during this row's work
    const bool pad = row_is_padding(a, row);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      const int n = max(0, min(4, d - c));
      if (a.s != nullptr && n > 0) Vec4<TS>::store(static_cast<TS*>(a.s) + row * a.ld_s + c, true, n, cur[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) sum += cur[i][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float t = (c + k < d) ? cur[i][k] - mean : 0.f;
        sq += t * t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq * inv_d + a.eps);
    TH* hr = static_cast<TH*>(a.h) + row * a.ld_h;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      const int n = max(0, min(4, d - c));
      if (n <= 0) continue;
      float g[4], b[4], o[4];
      Vec4<float>::load(a.gamma + c, true, n, g);
      Vec4<float>::load(a.beta + c, true, n, b);
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = pad ? 0.f : (cur[i][k] - mean) * rstd * g[k] + b[k];
      Vec4<TH>::store(hr + c, true, n, o);
    }
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) cur[i][k] = nxt[i][k];
  }
}

// One 256-thread CTA per row, d <= 8192 (8 groups of 4 per thread).
template <typename TX, typename TY, typename TS, typename TH>
__global__ void __launch_bounds__(256) ln_cta_rows(Args a) {
  grid_dep_wait();
  constexpr int NV = 8;
  __shared__ float red[8];
  const int d = static_cast<int>(a.d);
  const float inv_d = 1.f / static_cast<float>(d);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const TX* xr = static_cast<const TX*>(a.x) + row * a.ld_x;
    const bool pad = row_is_padding(a, row);
    float v[NV][4];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 256 + tid) * 4;
      const int n = max(0, min(4, d - c));
      Vec4<TX>::load(xr + c, a.vec, n, v[i]);
      if (a.y != nullptr) {
        float w[4];
        Vec4<TY>::load(static_cast<const TY*>(a.y) + row * a.ld_y + c, a.vec, n, w);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[i][k] = pad ? 0.f : v[i][k] + w[k];
      }
      // s = x + y, or a copy of x when there is no y
      if (a.s != nullptr && n > 0) Vec4<TS>::store(static_cast<TS*>(a.s) + row * a.ld_s + c, a.vec, n, v[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) sum += v[i][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[wid] = sum;
    __syncthreads();
    sum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sum += red[w];
    __syncthreads();
    const float mean = sum * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 256 + tid) * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float t = (c + k < d) ? v[i][k] - mean : 0.f;
        sq += t * t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) red[wid] = sq;
    __syncthreads();
    sq = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sq += red[w];
    __syncthreads();
    const float rstd = rsqrtf(sq * inv_d + a.eps);
    TH* hr = static_cast<TH*>(a.h) + row * a.ld_h;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 256 + tid) * 4;
      const int n = max(0, min(4, d - c));
      if (n <= 0) continue;
      float g[4], b[4], o[4];
      Vec4<float>::load(a.gamma + c, a.vec, n, g);
      Vec4<float>::load(a.beta + c, a.vec, n, b);
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = pad ? 0.f : (v[i][k] - mean) * rstd * g[k] + b[k];
      Vec4<TH>::store(hr + c, a.vec, n, o);
    }
  }
}

}  // namespace ln
}  // namespace tk
