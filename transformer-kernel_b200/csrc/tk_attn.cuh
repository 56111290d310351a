// Blackwell flash-attention forward over the fused QKV buffer.
//
// Replaces the reference's attention (F.scaled_dot_product_attention,
// src/optimized.py:615-624, and the Triton FA2 kernel src/kernels.py:136-247)
// with the baseline's op order (src/torch_transformer_benchmark.py:85-122):
// fp32 scores q.k, scaled by hd**-0.5 after the product, -inf above the
// diagonal (causal) and for keys >= kv_len[b], fp32 softmax, P.V, heads
// merged into the [B, S, H*hd] output (the layout src/kernels.py:272-276
// writes), so no transpose pass precedes the O-projection.
//
// Inputs: q, k, v fp16, logically [B, H, S, hd] with any strides whose last
// dimension is contiguous -- in the model they are views into the QKV GEMM's
// [B, S, 3*d] output, so no head-split copy is made. One 4-D tensor map per
// operand lets TMA fetch the tile of one (b, h) directly, zero-filling rows
// past S. The map lists dimensions in increasing stride order, as the
// tensor-map encoder requires: {hd, H, S, B} for views into the fused
// projection (head stride hd < row stride 3d), {hd, S, H, B} for [B,H,S,hd]
// contiguous tensors.
//
// Per CTA: one (b, h, 128-query tile). Warp 0 issues TMA, warp 1 owns TMEM
// and issues tcgen05.mma, warps 2..5 (one TMEM lane quadrant each, one query
// row per thread) run the softmax. TMEM (256 columns): S = Q K^T in columns
// [0,128) fp32; P = softmax numerators as packed fp16 pairs written back over
// S columns [0,64); O in columns [128, 128+HD) fp32.
//   S_j   : tcgen05.mma SS, M=128 N=128 K=16 x (HD/16)         (A=Q, B=K, both K-major)
//   O    += P_j V_j : tcgen05.mma TS, M=128 N=HD K=16 x 8      (A=P from TMEM, B=V MN-major)
// tcgen05.mma issued by one thread execute in order, so S_{j+1} (which
// overwrites P_j) is issued only after PV_j, and the completion of S_{j+1}
// also tells the softmax warps that PV_j has finished with O.
//
// Online softmax keeps the running max m in raw-score units and rescales
// O and l only when the max grows by more than 2^8 in the exponent (lazy
// rescaling); P values stay <= 2^8, well inside fp16 range.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "tk_ptx.cuh"

namespace tk {
namespace attn {

constexpr int kBM = 128;  // queries per CTA
constexpr int kBN = 128;  // keys per KV tile
constexpr int kThreads = 192;
constexpr int kStages = 2;
constexpr int kTmemCols = 256;
constexpr int kColO = 128;
constexpr float kLazyRescaleLog2 = 8.f;

struct Params {
  __half* out;          // [B, S, ld_out] fp16, head h at columns [h*HD, h*HD+HD)
  int64_t ld_out;
  int B, S, H;
  float scale_log2;     // hd**-0.5 * log2(e)
  int causal;
  const int* kv_len;    // optional [B]: keys >= kv_len[b] are masked
  int heads_inner;      // tensor-map dim order {hd, H, S, B} (1) or {hd, S, H, B} (0)
  uint64_t wait_limit_ns;
};

// TMA coordinates of the tile of (b, h) starting at sequence row `row`.
__device__ __forceinline__ void load_tile(void* dst, const CUtensorMap* map, uint64_t* bar, const Params& p, int row,
                                          int h, int b) {
  if (p.heads_inner)
    tma_load_4d(dst, map, bar, 0, h, row, b);
  else
    tma_load_4d(dst, map, bar, 0, row, h, b);
}

template <int HD>
struct Cfg {
  static_assert(HD == 32 || HD == 64, "head_dim");
  static constexpr int ROW_BYTES = HD * 2;                     // swizzle span
  static constexpr SmemLayout LAYOUT = HD == 64 ? kLayoutSW128 : kLayoutSW64;
  static constexpr int TILE_BYTES = kBM * ROW_BYTES;           // Q, K or V tile
  static constexpr int SBO = 8 * ROW_BYTES;                    // 8-row core-matrix group
  static constexpr int SMEM_BYTES = TILE_BYTES * (1 + 2 * kStages) + 1024;
};

enum : unsigned { kSiteQ = 1, kSiteKV = 2, kSiteS = 3, kSiteP = 4, kSiteO = 5, kSiteEmpty = 6, kSiteDrain = 7 };

template <int HD>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, Params p) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t kv_full[kStages];
  __shared__ __align__(8) uint64_t kv_empty[kStages];
  __shared__ __align__(8) uint64_t s_full;
  __shared__ __align__(8) uint64_t p_full;
  __shared__ __align__(8) uint64_t o_full;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::TILE_BYTES;                           // kStages tiles
  uint8_t* sV = smem + C::TILE_BYTES * (1 + kStages);           // kStages tiles

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int q_tiles = (p.S + kBM - 1) / kBM;
  const int bh_count = p.B * p.H;
  // Heaviest (last, for causal) query tiles are launched first.
  const int qt = q_tiles - 1 - static_cast<int>(blockIdx.x / bh_count);
  const int bh = static_cast<int>(blockIdx.x % bh_count);
  const int b = bh / p.H, h = bh % p.H;
  int kv_bound = p.S;
  if (p.kv_len != nullptr) kv_bound = max(0, min(p.S, p.kv_len[b]));
  int n_kv = (kv_bound + kBN - 1) / kBN;
  if (p.causal) n_kv = min(n_kv, qt + 1);
  const unsigned kid = 0x80u + HD;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
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

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_kv > 0) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      mbar_arrive_expect_tx(&q_full, C::TILE_BYTES);
      load_tile(sQ, &map_q, &q_full, p, qt * kBM, h, b);
      bool ok = true;
      int j = 0;
      for (; j < n_kv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1u, &abort_flag, p.wait_limit_ns)) {
          report_error(kDevWaitTimeout, kid * 256 + kSiteEmpty);
          abort_flag = 1;
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * C::TILE_BYTES);
        load_tile(sK + s * C::TILE_BYTES, &map_k, &kv_full[s], p, j * kBN, h, b);
        load_tile(sV + s * C::TILE_BYTES, &map_v, &kv_full[s], p, j * kBN, h, b);
      }
      if (!ok) {
        mbar_wait(&q_full, 0, nullptr, kDrainLimitNs);
        for (int t = max(0, j - kStages); t < j; ++t)
          mbar_wait(&kv_full[t % kStages], (t / kStages) & 1, nullptr, kDrainLimitNs);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kBM, kBN, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(kBM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(&q_full, 0, &abort_flag, p.wait_limit_ns);
      if (!ok) report_error(kDevWaitTimeout, kid * 256 + kSiteQ);
      // iteration j: O += P_{j-1} V_{j-1} (j > 0), then S_j = Q K_j^T (j < n_kv)
      for (int j = 0; j <= n_kv && ok; ++j) {
        if (j > 0) {
          if (!mbar_wait(&p_full, (j - 1) & 1, &abort_flag, p.wait_limit_ns)) {
            report_error(kDevWaitTimeout, kid * 256 + kSiteP);
            ok = false;
            break;
          }
          tc_fence_after();
          const int sp = (j - 1) % kStages;
          const uint32_t v_addr = smem_u32(sV + sp * C::TILE_BYTES);
#pragma unroll
          for (int ks = 0; ks < kBN / 16; ++ks) {
            const uint64_t dv = smem_desc(v_addr + ks * 16 * C::ROW_BYTES, C::TILE_BYTES, C::SBO, C::LAYOUT);
            mma_f16_ts(tmem_base + kColO, tmem_base + ks * 8, dv, idesc_o, (j > 1 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&kv_empty[sp]);
          if (j == n_kv) mma_commit(&o_full);
        }
        if (j < n_kv) {
          const int s = j % kStages;
          if (!mbar_wait(&kv_full[s], (j / kStages) & 1, &abort_flag, p.wait_limit_ns)) {
            report_error(kDevWaitTimeout, kid * 256 + kSiteKV);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + s * C::TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t dq = smem_desc(q_addr + kk * 32, 16, C::SBO, C::LAYOUT);
            const uint64_t dk = smem_desc(k_addr + kk * 32, 16, C::SBO, C::LAYOUT);
            mma_f16_ss(tmem_base, dq, dk, idesc_s, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full);
        }
      }
      if (!ok) {
        abort_flag = 1;
        mma_commit(&o_full);  // completes once every MMA issued so far is done
        mbar_wait(&o_full, 0, nullptr, kDrainLimitNs);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax (one query row per thread) ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + static_cast<int>(lane);
    const int q_idx = qt * kBM + r;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    float m = -INFINITY;  // running max, raw score units
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait(&s_full, j & 1, &abort_flag, p.wait_limit_ns)) {
        report_error(kDevWaitTimeout, kid * 256 + kSiteS);
        abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kBN;
      // keys k0 + c are valid iff c < lim (causal diagonal and the kv bound)
      int lim = kv_bound - k0;
      if (p.causal) lim = min(lim, q_idx - k0 + 1);
      lim = max(0, min(kBN, lim));

      // The whole 128-column score row in registers: one TMEM round trip.
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_lane + c * 32, sv[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_wait(sv[c]);  // first waits, the rest only pin registers
      // Masking is only needed on the causal diagonal tile and the tile
      // holding the kv bound; `full` is warp-uniform elsewhere.
      const bool full = lim >= kBN;
      // row max with four independent chains
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int t = 0; t < 32; ++t) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(sv[c][t]));
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (c * 32 + t < lim) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(sv[c][t]));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      float m_use = m;
      float alpha = 1.f;
      if (mx > m) {
        if (m == -INFINITY || (mx - m) * p.scale_log2 > kLazyRescaleLog2) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - mx) * p.scale_log2);
          m_use = mx;
        }
      }
      const float neg_mc = (m_use == -INFINITY) ? 0.f : -m_use * p.scale_log2;
      // P = 2^(s*c - m*c), packed fp16 pairs over S columns [0, 64); the
      // columns written for chunk c were all read into registers above.
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float p0 = ex2_approx(fmaf(__uint_as_float(sv[c][t]), p.scale_log2, neg_mc));
          float p1 = ex2_approx(fmaf(__uint_as_float(sv[c][t + 1]), p.scale_log2, neg_mc));
          if (!full) {
            p0 = (c * 32 + t < lim) ? p0 : 0.f;
            p1 = (c * 32 + t + 1 < lim) ? p1 : 0.f;
          }
          rs4[(t >> 1) & 3] += p0 + p1;
          pk[t / 2] = pack_half2(p0, p1);
        }
        tmem_st16(t_lane + c * 16, pk);
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      // O rescale: S_j's completion implies PV_{j-1} (issued before it) is done.
      const bool need = (j > 0) && (alpha != 1.f);
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          uint32_t o[16];
          tmem_ld16(t_lane + kColO + c, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st16(t_lane + kColO + c, o);
        }
      }
      l = l * alpha + rs;
      m = m_use;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    // epilogue: O / l -> fp16 [b, q, h*HD + c]
    if (ok && n_kv > 0) {
      if (!mbar_wait(&o_full, 0, &abort_flag, p.wait_limit_ns)) {
        report_error(kDevWaitTimeout, kid * 256 + kSiteO);
        abort_flag = 1;
        ok = false;
      }
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      __half* dst = p.out + (static_cast<int64_t>(b) * p.S + q_idx) * p.ld_out + h * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        uint32_t o[16];
        if (n_kv > 0) {
          tmem_ld16(t_lane + kColO + c, o);
          tmem_ld_wait(o);
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = 0u;
        }
        if (q_idx < p.S) {
          uint4 w0, w1;
          w0.x = pack_half2(__uint_as_float(o[0]) * inv_l, __uint_as_float(o[1]) * inv_l);
          w0.y = pack_half2(__uint_as_float(o[2]) * inv_l, __uint_as_float(o[3]) * inv_l);
          w0.z = pack_half2(__uint_as_float(o[4]) * inv_l, __uint_as_float(o[5]) * inv_l);
          w0.w = pack_half2(__uint_as_float(o[6]) * inv_l, __uint_as_float(o[7]) * inv_l);
          w1.x = pack_half2(__uint_as_float(o[8]) * inv_l, __uint_as_float(o[9]) * inv_l);
          w1.y = pack_half2(__uint_as_float(o[10]) * inv_l, __uint_as_float(o[11]) * inv_l);
          w1.z = pack_half2(__uint_as_float(o[12]) * inv_l, __uint_as_float(o[13]) * inv_l);
          w1.w = pack_half2(__uint_as_float(o[14]) * inv_l, __uint_as_float(o[15]) * inv_l);
          reinterpret_cast<uint4*>(dst + c)[0] = w0;
          reinterpret_cast<uint4*>(dst + c)[1] = w1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace attn
}  // namespace tk
