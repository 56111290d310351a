// Whole-stack forward of one sequence per CTA, for the small shapes the
// layer-by-layer kernels run launch-bound (d_model 128, ffn 128, S <= 128;
// the reference harness's case 1 and the appendix shapes around it,
// configs/shapes.json cases 1-6, 10, 12).
//
// Same math and op order as the layer-by-layer path (and the harness,
// src/torch_transformer_benchmark.py:85-172): per layer
//   h = LN1(x);  q,k,v = h Wqkv^T + b;  attention (fp32 scores scaled after
//   q.k, causal / key-padding masks, fp32 softmax, P V);  x += ctx Wo^T + bo;
//   h = LN2(x);  x += W2 gelu_erf(W1 h + b1) + b2;  padded rows zeroed;
// then the final LayerNorm written as fp32. fp16 GEMM / attention operands,
// fp32 accumulation, fp32 residual stream and LayerNorm statistics.
//
// One CTA holds one sequence (its rows 0..127; rows past S are inert
// padding) through all layers, so a forward is one launch. Warps: 0 TMA
// (weight tiles, streamed through two 32 KB slots), 1 TMEM owner + MMA
// issuer, 2..5 row warps (thread = row: LayerNorm statistics, softmax rows
// and epilogues are thread-local). TMEM (512 columns): the residual stream
// X in [0, 128) for the whole forward; [128, 512) holds, in turn, the QKV
// accumulators (3 x 128), the attention scores of two heads at a time
// (128 each, P written over the first 64) with O in [384, 512), and the
// 128-column accumulators of the O-projection and the two FFN GEMMs.
// Shared memory: the A operand (h, ctx or u: 128 x 128 fp16, two 128-byte
// swizzle atoms), two weight slots, and q / k / v as per-head tiles.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "tk_attn.cuh"
#include "tk_gemm.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace small {

constexpr int kRows = 128;      // rows per CTA (one sequence, S <= 128)
constexpr int kD = 128;         // d_model (= ffn)
constexpr int kThreads = 192;   // TMA, MMA, 4 row warps
constexpr int kTmemCols = 512;
constexpr int kColX = 0, kColAcc = 128, kColO = 384;
constexpr int kTileBytes = kRows * kD * 2;       // 32 KB: a 128 x 128 fp16 operand
constexpr int kAtomBytes = kRows * 64 * 2;       // 16 KB: 128 rows x one 64-column swizzle atom
constexpr int kWRowsPerLayer = 768;              // packed weight rows: Wqkv 384, Wo 128, W1 128, W2 128
constexpr int kVecPerLayer = 1280;               // packed fp32: bqkv 384, bo, b1, b2, ln1 g/b, ln2 g/b
constexpr int kTilesPerLayer = 6;                // weight tiles: Q, K, V, O, FFN-in, FFN-out
// Stacks of up to kVecSmemLayers layers keep every layer's biases and
// LayerNorm affines (and the final affine) in shared memory, copied once by
// the row warps, so the per-chunk parameter reads of the row passes are
// shared-memory broadcasts instead of L1 / L2 round trips.
constexpr int kVecSmemLayers = 5;
constexpr int kVecSmemBytes = (kVecSmemLayers * kVecPerLayer + 2 * kD) * 4;

struct Params {
  const float* x;          // [B, S, 128] fp32
  float* out;              // [B, S, 128] fp32
  const float* vec;        // [L, 1280] fp32 (biases, LayerNorm affines)
  const float* final_g;    // [128]
  const float* final_b;
  const int* row_len;      // optional [B] prefix lengths
  int B, S, H, L, causal;
  float eps;
  float scale_log2;        // hd**-0.5 * log2(e)
  uint64_t wait_limit_ns;
};

template <int HD>
struct Cfg {
  static_assert(HD == 32 || HD == 64, "head_dim");
  static constexpr int H = kD / HD;
  static constexpr int ROW_BYTES = HD * 2;
  static constexpr SmemLayout LAYOUT = HD == 64 ? kLayoutSW128 : kLayoutSW64;
  static constexpr int HEAD_TILE = kRows * ROW_BYTES;   // one head of q, k or v
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = kTileBytes;               // two weight slots
  static constexpr int OFF_Q = 3 * kTileBytes;
  static constexpr int OFF_K = 4 * kTileBytes;
  static constexpr int OFF_V = 5 * kTileBytes;
  static constexpr int OFF_VEC = 6 * kTileBytes;          // parameter vectors (short stacks)
  static constexpr int SMEM_BYTES = 6 * kTileBytes + kVecSmemBytes + 1024;
};

enum : unsigned { kSiteA = 1, kSiteW = 2, kSiteAcc = 3, kSiteQkv = 4, kSiteS = 5, kSiteP = 6, kSitePv = 7,
                  kSiteAttn = 8, kSiteEmpty = 9 };

// 16-byte unit u of row r of a swizzled tile with `units` 16-byte units per
// row (8 for the 128-byte swizzle, 4 for 64-byte).
__device__ __forceinline__ uint32_t swz_unit(int r, int u, int units) {
  return units == 8 ? (u ^ (r & 7)) : (u ^ ((r >> 1) & 3));
}

// Four consecutive fp32 parameters (bias, LayerNorm affine); every thread of
// the CTA reads the same addresses, in shared memory (short stacks) or in
// global memory (generic load: the pointer may be either).
__device__ __forceinline__ float4 ldg4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// 32 fp32 values of this thread's TMEM lane from column t.
__device__ __forceinline__ void tmem_chunk(uint32_t t, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(t, r);
  tmem_ld_wait(r);
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
}

__device__ __forceinline__ void tmem_store_chunk(uint32_t t, const float (&v)[32]) {
  uint32_t lo[16], hi[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    lo[k] = __float_as_uint(v[k]);
    hi[k] = __float_as_uint(v[16 + k]);
  }
  tmem_st16(t, lo);
  tmem_st16(t + 16, hi);
}

// body(v, q) for the 32-column TMEM chunks q = 0..n-1 at addr(q), with the
// load of chunk q+1 in flight while chunk q is processed. tcgen05.wait::ld
// waits for all of a thread's loads, so the loop alternates two register
// buffers. n must be warp-uniform.
template <typename Addr, typename Body>
__device__ __forceinline__ void tmem_pipeline(int n, Addr addr, Body body) {
  if (n <= 0) return;
  uint32_t a[32], b[32];
  tmem_ld32(addr(0), a);
  tmem_ld_wait(a);
#pragma unroll 1
  for (int q = 0; q < n; q += 2) {
    if (q + 1 < n) tmem_ld32(addr(q + 1), b);
    body(a, q);
    if (q + 1 < n) {
      tmem_ld_wait(b);
      if (q + 2 < n) tmem_ld32(addr(q + 2), a);
      body(b, q + 1);
      if (q + 2 < n) tmem_ld_wait(a);
    }
  }
}

// Mean and 1/sqrt(var + eps) of the 128 values in TMEM at t (two-pass fp32
// statistics, 32 columns at a time: the loops stay rolled, so the kernel's
// code stays small enough for the instruction cache).
__device__ __forceinline__ void row_stats(uint32_t t, float eps, float& mean, float& rstd) {
  // four partial sums per pass: short dependency chains
  auto col = [t](int q) { return t + q * 32; };
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
  tmem_pipeline(4, col, [&](uint32_t(&v)[32], int) {
#pragma unroll
    for (int k = 0; k < 32; ++k) s4[k & 3] += __uint_as_float(v[k]);
  });
  mean = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.f / kD);
  float v4[4] = {0.f, 0.f, 0.f, 0.f};
  tmem_pipeline(4, col, [&](uint32_t(&v)[32], int) {
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float d = __uint_as_float(v[k]) - mean;
      v4[k & 3] = fmaf(d, d, v4[k & 3]);
    }
  });
  rstd = rsqrtf(((v4[0] + v4[1]) + (v4[2] + v4[3])) * (1.f / kD) + eps);
}

// LayerNorm of the 128 values in TMEM at t into row r of the A operand tile
// (fp16, 128-byte swizzle, two atoms).
__device__ __forceinline__ void ln_tmem_to_a(uint32_t t, const float* g, const float* b, float eps, uint8_t* sA,
                                             int r) {
  float mean, rstd;
  row_stats(t, eps, mean, rstd);
  tmem_pipeline(4, [t](int q) { return t + q * 32; }, [&](uint32_t(&raw)[32], int q) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(raw[k]);
#pragma unroll
    for (int u4 = 0; u4 < 4; ++u4) {
      const int c8 = q * 32 + u4 * 8;
      const float4 g0 = ldg4(g + c8), g1 = ldg4(g + c8 + 4), b0 = ldg4(b + c8), b1 = ldg4(b + c8 + 4);
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int cl = u4 * 8 + 2 * k;
        w[k] = pack_half2((v[cl] - mean) * rstd * gg[2 * k] + bb[2 * k],
                          (v[cl + 1] - mean) * rstd * gg[2 * k + 1] + bb[2 * k + 1]);
      }
      const int u = q * 4 + u4;
      uint8_t* atom = sA + (u >> 3) * kAtomBytes;
      *reinterpret_cast<uint4*>(atom + r * 128 + swz_unit(r, u & 7, 8) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  });
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    stack_small_kernel(const __grid_constant__ CUtensorMap map_w, Params p) {
  using C = Cfg<HD>;
  constexpr int H = C::H;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t w_full[2], w_empty[2];
  __shared__ __align__(8) uint64_t a_ready, acc_full, qkv_ready, attn_done, pv_bar, drain_bar;
  // Per score buffer (head parity): scores ready / P stored. One barrier per
  // buffer, so a warp that finishes head h early and moves on to head h+1
  // arrives on the other barrier and cannot complete head h's phase.
  __shared__ __align__(8) uint64_t s_full[2], p_full[2];
  __shared__ float inv_l_sh[4][kRows];  // per head, per row: 1 / softmax row sum
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sW = smem + C::OFF_W;
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int seq = static_cast<int>(blockIdx.x);
  const unsigned kid = 0xC0u + HD / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
    }
    mbar_init(&a_ready, 4);
    mbar_init(&acc_full, 1);
    mbar_init(&qkv_ready, 4);
    mbar_init(&attn_done, 1);
    mbar_init(&pv_bar, 1);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  grid_dep_wait();  // the previous kernel's outputs are complete and visible

  if (warp == 0) {
    // ---------------- TMA: weight tiles, 6 per layer, two slots ----------------
    if (lane == 0) {
      prefetch_tensormap(&map_w);
      constexpr int kRowOff[kTilesPerLayer] = {0, 128, 256, 384, 512, 640};
      int n = 0;
      bool ok = true;
      for (int l = 0; l < p.L && ok; ++l) {
        for (int t = 0; t < kTilesPerLayer; ++t, ++n) {
          const int s = n & 1;
          if (!mbar_wait(&w_empty[s], ((n >> 1) & 1) ^ 1u, &abort_flag, p.wait_limit_ns)) {
            report_error(kDevWaitTimeout, kid * 256 + kSiteEmpty);
            abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* dst = sW + s * kTileBytes;
          mbar_arrive_expect_tx(&w_full[s], kTileBytes);
          const int row = l * kWRowsPerLayer + kRowOff[t];
          tma_load_2d(dst, &map_w, &w_full[s], 0, row);
          tma_load_2d(dst + kAtomBytes, &map_w, &w_full[s], 64, row);
        }
      }
      if (!ok) {
        for (int t = max(0, n - 2); t < n; ++t) mbar_wait(&w_full[t & 1], (t >> 1) & 1, nullptr, kDrainLimitNs);
      }
      grid_dep_launch();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_g = idesc_f16_f32(kRows, 128, false, false);  // GEMM n-tile / scores
      constexpr uint32_t idesc_o = idesc_f16_f32(kRows, HD, false, true);    // P V (V MN-major)
      int nw = 0, na = 0, npv = 0, np0 = 0, np1 = 0;
      bool ok = true;
      auto fail = [&](unsigned site) {
        report_error(kDevWaitTimeout, kid * 256 + site);
        ok = false;
      };
      auto wait_a = [&]() {
        if (ok && !mbar_wait(&a_ready, na & 1, &abort_flag, p.wait_limit_ns)) fail(kSiteA);
        ++na;
        tc_fence_after();
      };
      // acc (128 columns at d_col) = A (sA) x next weight tile^T
      auto gemm_tile = [&](uint32_t d_col) {
        if (!ok) return;
        const int s = nw & 1;
        if (!mbar_wait(&w_full[s], (nw >> 1) & 1, &abort_flag, p.wait_limit_ns)) {
          fail(kSiteW);
          return;
        }
        ++nw;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA);
        const uint32_t b_addr = smem_u32(sW + s * kTileBytes);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kAtomBytes + (ks & 3) * 32;
          mma_f16_ss(tmem_base + d_col, smem_desc(a_addr + off, 16, 1024, kLayoutSW128),
                     smem_desc(b_addr + off, 16, 1024, kLayoutSW128), idesc_g, ks > 0 ? 1u : 0u);
        }
        mma_commit(&w_empty[s]);
      };
      // scores of head h into score buffer h & 1
      auto issue_s = [&](int h) {
        const uint32_t q_addr = smem_u32(sQ + h * C::HEAD_TILE);
        const uint32_t k_addr = smem_u32(sK + h * C::HEAD_TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_f16_ss(tmem_base + kColAcc + (h & 1) * 128, smem_desc(q_addr + kk * 32, 16, 8 * C::ROW_BYTES, C::LAYOUT),
                     smem_desc(k_addr + kk * 32, 16, 8 * C::ROW_BYTES, C::LAYOUT), idesc_g, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[h & 1]);
      };
      for (int l = 0; l < p.L && ok; ++l) {
        // q | k | v = h Wqkv^T
        wait_a();
        for (int t = 0; t < 3; ++t) gemm_tile(kColAcc + t * 128);
        if (!ok) break;
        mma_commit(&acc_full);
        // attention, two heads' scores in flight
        if (!mbar_wait(&qkv_ready, l & 1, &abort_flag, p.wait_limit_ns)) {
          fail(kSiteQkv);
          break;
        }
        tc_fence_after();
        issue_s(0);
        if (H > 1) issue_s(1);
        for (int h = 0; h < H && ok; ++h) {
          const uint32_t p_phase = (h & 1) == 0 ? (np0++ & 1) : (np1++ & 1);
          if (!mbar_wait(&p_full[h & 1], p_phase, &abort_flag, p.wait_limit_ns)) {
            fail(kSiteP);
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + h * C::HEAD_TILE);
          const uint32_t p_col = kColAcc + (h & 1) * 128;  // P over the first 64 score columns
#pragma unroll
          for (int ks = 0; ks < kRows / 16; ++ks) {
            const uint64_t dv = smem_desc(v_addr + ks * 16 * C::ROW_BYTES, C::HEAD_TILE, 8 * C::ROW_BYTES, C::LAYOUT);
            mma_f16_ts(tmem_base + kColO + h * HD, tmem_base + p_col + ks * 8, dv, idesc_o, ks > 0 ? 1u : 0u);
          }
          if (h + 2 < H) {
            // head h+2 reuses this score buffer: P of head h must have been read
            mma_commit(&pv_bar);
            if (!mbar_wait(&pv_bar, npv & 1, &abort_flag, p.wait_limit_ns)) {
              fail(kSitePv);
              break;
            }
            ++npv;
            tc_fence_after();
            issue_s(h + 2);
          }
        }
        if (!ok) break;
        mma_commit(&attn_done);
        // x += ctx Wo^T + bo (epilogue), then the FFN
        wait_a();
        gemm_tile(kColAcc);
        if (!ok) break;
        mma_commit(&acc_full);
        wait_a();
        gemm_tile(kColAcc);
        if (!ok) break;
        mma_commit(&acc_full);
        wait_a();
        gemm_tile(kColAcc);
        if (!ok) break;
        mma_commit(&acc_full);
      }
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, ok ? p.wait_limit_ns : kDrainLimitNs);
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ---------------- row warps: thread = row r of the sequence ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + static_cast<int>(lane);
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    int len = p.S;
    if (p.row_len != nullptr) len = max(0, min(p.S, p.row_len[seq]));
    const bool row_valid = r < p.S;
    const bool row_pad = r >= len;  // padded (or past S): output rows zeroed
    int nacc = 0, nsf0 = 0, nsf1 = 0;
    bool ok = true;
    auto fail = [&](unsigned site) {
      report_error(kDevWaitTimeout, kid * 256 + site);
      abort_flag = 1;
      ok = false;
    };
    auto signal = [&](uint64_t* bar) {
      fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
    };
    auto wait_acc = [&]() -> bool {
      if (!mbar_wait_warp(&acc_full, nacc & 1, &abort_flag, p.wait_limit_ns)) {
        fail(kSiteAcc);
        return false;
      }
      ++nacc;
      tc_fence_after();
      return true;
    };
    // Parameter vectors: copied into shared memory by the 128 row threads
    // (then a barrier of those 4 warps only, reached by all of them before
    // any wait that could end early), or read from global memory.
    const float* vbase = p.vec;
    const float* fgp = p.final_g;
    const float* fbp = p.final_b;
    if (p.L <= kVecSmemLayers) {
      float* sv = reinterpret_cast<float*>(smem + C::OFF_VEC);
      const int n4 = p.L * kVecPerLayer / 4;
      for (int i = r; i < n4; i += kRows) reinterpret_cast<float4*>(sv)[i] = reinterpret_cast<const float4*>(p.vec)[i];
      float* sg = sv + kVecSmemLayers * kVecPerLayer;
      if (r < kD / 4) {
        reinterpret_cast<float4*>(sg)[r] = reinterpret_cast<const float4*>(p.final_g)[r];
        reinterpret_cast<float4*>(sg + kD)[r] = reinterpret_cast<const float4*>(p.final_b)[r];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kRows) : "memory");
      vbase = sv;
      fgp = sg;
      fbp = sg + kD;
    }
    // The residual stream lives in TMEM (columns [0, 128) of this thread's
    // lane); every pass over a row goes 32 columns at a time.
    const uint32_t t_x = t_lane + kColX;
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float v[32];
      const float4* src = reinterpret_cast<const float4*>(p.x + (static_cast<int64_t>(seq) * p.S + r) * kD + q * 32);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 f = row_valid ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        v[4 * c] = f.x;
        v[4 * c + 1] = f.y;
        v[4 * c + 2] = f.z;
        v[4 * c + 3] = f.w;
      }
      tmem_store_chunk(t_x + q * 32, v);
    }
    tmem_st_wait();
    ln_tmem_to_a(t_x, vbase + 768, vbase + 896, p.eps, sA, r);
    signal(&a_ready);
    // x += bias + acc, unless `keep` (the row keeps x); `zero` clears the row.
    auto residual = [&](const float* bias, bool keep, bool zero) {
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        // x and the accumulator chunk with one wait
        uint32_t xr[32], ar[32];
        tmem_ld32(t_x + q * 32, xr);
        tmem_ld32(t_lane + kColAcc + q * 32, ar);
        tmem_ld_wait(xr);
        tmem_ld_wait(ar);
        float v[32];
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
          const float4 bq = ldg4(bias + q * 32 + 4 * k4);
          const float bb[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int k = 4 * k4 + j;
            const float xk = __uint_as_float(xr[k]);
            const float y = keep ? xk : xk + (__uint_as_float(ar[k]) + bb[j]);
            v[k] = zero ? 0.f : y;
          }
        }
        tmem_store_chunk(t_x + q * 32, v);
      }
      tmem_st_wait();
    };
    for (int l = 0; l < p.L && ok; ++l) {
      const float* vec = vbase + static_cast<int64_t>(l) * kVecPerLayer;
      // ---- q | k | v: + bias, fp16, into the per-head tiles ----
      if (!wait_acc()) break;
      // the 12 chunks of the q | k | v accumulators are contiguous in TMEM
      tmem_pipeline(12, [&](int i) { return t_lane + kColAcc + i * 32; }, [&](uint32_t(&raw)[32], int i) {
        const int t = i >> 2, q = i & 3;
        uint8_t* dst = t == 0 ? sQ : t == 1 ? sK : sV;
        // 32 columns = part of one head: head (q*32)/HD, columns from (q*32)%HD
        const int hh = (q * 32) / HD;
        const int c0 = (q * 32) % HD;
        uint8_t* tile = dst + hh * C::HEAD_TILE + r * C::ROW_BYTES;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int g8 = i * 32 + u * 8;
          const float4 bq0 = ldg4(vec + g8), bq1 = ldg4(vec + g8 + 4);
          const float bb[8] = {bq0.x, bq0.y, bq0.z, bq0.w, bq1.x, bq1.y, bq1.z, bq1.w};
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int c = u * 8 + 2 * k;
            w[k] = pack_half2(__uint_as_float(raw[c]) + bb[2 * k], __uint_as_float(raw[c + 1]) + bb[2 * k + 1]);
          }
          const int unit = c0 / 8 + u;
          *reinterpret_cast<uint4*>(tile + swz_unit(r, unit, C::ROW_BYTES / 16) * 16) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      });
      signal(&qkv_ready);
      // ---- attention: one query row per thread; the key row (S <= 128) in one tile ----
      int lim = len;  // keys < lim are valid
      if (p.causal) lim = min(lim, r + 1);
      const float sl = p.scale_log2;
      // 32-key chunks with any valid key for some row of this warp (rows
      // 32*quad .. 32*quad+31): the rest are skipped and their P written as 0.
      int q_end = (len + 31) / 32;
      if (p.causal) q_end = min(q_end, quad + 1);
#pragma unroll 1
      for (int h = 0; h < H && ok; ++h) {
        const int b = h & 1;
        const uint32_t phase = b == 0 ? (nsf0++ & 1) : (nsf1++ & 1);
        if (!mbar_wait_warp(&s_full[b], phase, &abort_flag, p.wait_limit_ns)) {
          fail(kSiteS);
          break;
        }
        tc_fence_after();
        const uint32_t t_s = t_lane + kColAcc + b * 128;
        // The row's scores (up to 128 keys, q_end 32-key chunks, warp-uniform)
        // come out of TMEM with one round of loads and one wait; then the
        // row max over the valid keys, and P = 2^(s*c - m*c) packed fp16 over
        // the scores already read.
        uint32_t sv[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < q_end) tmem_ld32(t_s + q * 32, sv[q]);
        // one wait; each call names its chunk's registers, so no use of them
        // can be scheduled above it
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < q_end) tmem_ld_wait(sv[q]);
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < q_end) {
#pragma unroll
            for (int k = 0; k < 32; ++k)
              mx4[k & 3] = fmaxf(mx4[k & 3], q * 32 + k < lim ? __uint_as_float(sv[q][k]) : -INFINITY);
          }
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        const float neg_mc = (mx == -INFINITY) ? 0.f : -mx * sl;
        float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q >= q_end) continue;
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const int c = q * 32 + k;
            const float e0 = (c < lim) ? ex2_approx(fmaf(__uint_as_float(sv[q][k]), sl, neg_mc)) : 0.f;
            const float e1 = (c + 1 < lim) ? ex2_approx(fmaf(__uint_as_float(sv[q][k + 1]), sl, neg_mc)) : 0.f;
            ls4[(k >> 1) & 3] += e0 + e1;
            w[k / 2] = pack_half2(e0, e1);
          }
          tmem_st16(t_s + q * 16, w);  // P over scores this thread has already read
        }
#pragma unroll 1
        for (int q = q_end; q < 4; ++q) {
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) w[k] = 0u;
          tmem_st16(t_s + q * 16, w);
        }
        const float lsum = (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
        inv_l_sh[h][r] = lsum > 0.f ? 1.f / lsum : 0.f;
        tmem_st_wait();
        signal(&p_full[b]);
      }
      if (!ok) break;
      if (!mbar_wait_warp(&attn_done, l & 1, &abort_flag, p.wait_limit_ns)) {
        fail(kSiteAttn);
        break;
      }
      tc_fence_after();
      // ---- ctx = O / l (fp16) into the A tile; padded query rows give 0 ----
#pragma unroll 1
      for (int h = 0; h < H; ++h) {
        const float il = row_pad ? 0.f : inv_l_sh[h][r];
        // the head's HD columns of O with one round of loads and one wait
        uint32_t oh[HD / 16][16];
#pragma unroll
        for (int q = 0; q < HD / 16; ++q) tmem_ld16(t_lane + kColO + h * HD + q * 16, oh[q]);
#pragma unroll
        for (int q = 0; q < HD / 16; ++q) tmem_ld_wait(oh[q]);
#pragma unroll
        for (int q = 0; q < HD / 16; ++q) {
          const uint32_t* o = oh[q];
          const int c = h * HD + q * 16;  // ctx column
          uint32_t w[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            w[k] = pack_half2(__uint_as_float(o[2 * k]) * il, __uint_as_float(o[2 * k + 1]) * il);
          uint8_t* atom = sA + (c >> 6) * kAtomBytes + r * 128;
          const int u = (c & 63) >> 3;
          *reinterpret_cast<uint4*>(atom + swz_unit(r, u, 8) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(atom + swz_unit(r, u + 1, 8) * 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      signal(&a_ready);
      // ---- x += ctx Wo^T + bo (0 for padded rows); h = LN2(x) ----
      if (!wait_acc()) break;
      residual(vec + 384, row_pad, false);
      ln_tmem_to_a(t_x, vec + 1024, vec + 1152, p.eps, sA, r);
      signal(&a_ready);
      // ---- u = gelu(h W1^T + b1) ----
      if (!wait_acc()) break;
      tmem_pipeline(4, [&](int q) { return t_lane + kColAcc + q * 32; }, [&](uint32_t(&raw)[32], int q) {
        float a[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) a[k] = __uint_as_float(raw[k]);
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int c8 = q * 32 + u4 * 8;
          const float4 c0 = ldg4(vec + 512 + c8), c1 = ldg4(vec + 516 + c8);
          const float bb[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int cl = u4 * 8 + 2 * k;
            const float2 gl = gemm::gelu_erf2(make_float2(a[cl] + bb[2 * k], a[cl + 1] + bb[2 * k + 1]));
            w[k] = pack_half2(gl.x, gl.y);
          }
          const int u = q * 4 + u4;
          uint8_t* atom = sA + (u >> 3) * kAtomBytes;
          *reinterpret_cast<uint4*>(atom + r * 128 + swz_unit(r, u & 7, 8) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      });
      signal(&a_ready);
      // ---- x += u W2^T + b2, padded rows zeroed; next LN1 or the final LN ----
      if (!wait_acc()) break;
      residual(vec + 640, false, row_pad);
      if (l + 1 < p.L) {
        const float* nvec = vec + kVecPerLayer;
        ln_tmem_to_a(t_x, nvec + 768, nvec + 896, p.eps, sA, r);
        signal(&a_ready);
      } else {
        // final LayerNorm, fp32 output; padded rows are zero. The TMEM loads
        // are warp-collective (.sync.aligned), so every lane runs them and
        // only the stores are limited to the sequence's rows.
        float mean, rstd;
        row_stats(t_x, p.eps, mean, rstd);
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          float v[32];
          tmem_chunk(t_x + q * 32, v);
          float4* dst = reinterpret_cast<float4*>(p.out + (static_cast<int64_t>(seq) * p.S + r) * kD + q * 32);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4 o;
            const int gc = q * 32 + 4 * c;
            const float4 fg = ldg4(fgp + gc), fb = ldg4(fbp + gc);
            o.x = (v[4 * c] - mean) * rstd * fg.x + fb.x;
            o.y = (v[4 * c + 1] - mean) * rstd * fg.y + fb.y;
            o.z = (v[4 * c + 2] - mean) * rstd * fg.z + fb.z;
            o.w = (v[4 * c + 3] - mean) * rstd * fg.w + fb.w;
            if (row_pad) o = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row_valid) dst[c] = o;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace small
}  // namespace tk
