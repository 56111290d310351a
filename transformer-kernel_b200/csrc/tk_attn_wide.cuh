// Flash-attention forward for head_dim 128 and 256.
//
// Same contract and op order as attn_fwd_kernel (tk_attn.cuh) -- fp32
// scores scaled after q.k, -inf above the diagonal and past kv_len, fp32
// online softmax, P.V, output [B, S, H*hd] -- for the head dims of the
// reference's appendix shapes that the two-group kernel cannot hold: its
// TMEM budget (two groups x (S 128 + P 64 + O hd columns)) only fits
// hd <= 64 (src/kernels.py:70-77 tiles hd up to 256; configs/shapes.json
// cases 8 and 9 use hd 256 and 128).
//
// One CTA per (b, h, 128-query tile), heaviest query tiles first; warps:
// 0 TMA, 1 TMEM owner + MMA issuer, 2..5 softmax (one query row per
// thread, the same code as the two-group kernel). TMEM: S 128 fp32
// columns, P 64 columns of packed fp16 pairs, O hd fp32 columns (<= 448).
// Q stays in shared memory as hd/64 chunks of 64 columns (one 128-byte
// swizzle row each); K and V tiles stream through a ring of 8 such chunk
// slots in the order K_j chunks, V_j chunks, K_{j+1} chunks, ...:
//   S(j)  = sum_c Q_c K_{j,c}^T   (SS MMA, M=128 N=128 K=16, 4 per chunk)
//   O    += P(j) V_{j,c} into O columns [64c, 64c+64)   (TS MMA, N=64)
// A K chunk is released when S(j) completes, a V chunk when its PV does,
// so S(j+1) overlaps the softmax of tile j.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "tk_attn.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace attn {
namespace wide {

constexpr int kChunk = 64;                      // head-dim columns per TMA chunk
constexpr int kChunkBytes = kBM * kChunk * 2;   // 16 KB: 128 rows x 128 bytes
constexpr int kSlots = 8;                       // K/V chunk ring
constexpr int kThreads = 192;                   // TMA, MMA, 4 softmax warps
constexpr int kTmemCols = 512;
constexpr int kColS = 0, kColP = 128, kColO = 192;

template <int HD>
struct Cfg {
  static_assert(HD == 128 || HD == 256, "head_dim");
  static constexpr int NC = HD / kChunk;
  static constexpr int SMEM_BYTES = (NC + kSlots) * kChunkBytes + 1024;
};

enum : unsigned { kSiteQ = 1, kSiteSlot = 2, kSiteS = 3, kSiteP = 4, kSiteO = 5, kSiteEmpty = 6, kSitePv = 9,
                  kSiteSFree = 10 };

struct Item {
  int b, h, tq, kv_bound, n;  // n = KV tiles attended
};

__device__ __forceinline__ Item make_item(const Params& p, int idx, int q_tiles) {
  const int bh_count = p.B * p.H;
  Item it;
  it.tq = q_tiles - 1 - idx / bh_count;  // heaviest (last) query tiles first
  const int bh = idx % bh_count;
  it.b = bh / p.H;
  it.h = bh % p.H;
  it.kv_bound = p.S;
  if (p.kv_len != nullptr) it.kv_bound = max(0, min(p.S, p.kv_len[it.b]));
  const int n_all = (it.kv_bound + kBN - 1) / kBN;
  it.n = p.causal ? min(n_all, it.tq + 1) : n_all;
  return it;
}

// TMA load of head-dim chunk starting at column x of the tile of (b, h) at
// sequence row `row`.
__device__ __forceinline__ void load_chunk(void* dst, const CUtensorMap* map, uint64_t* bar, const Params& p,
                                           int row, int h, int b, int x) {
  if (p.heads_inner)
    tma_load_4d(dst, map, bar, x, h, row, b);
  else
    tma_load_4d(dst, map, bar, x, row, h, b);
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_wide_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, Params p) {
  using C = Cfg<HD>;
  constexpr int NC = C::NC;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, s_full, p_full, pv_done, s_free, o_full, drain_bar;
  __shared__ __align__(8) uint64_t slot_full[kSlots];
  __shared__ __align__(8) uint64_t slot_empty[kSlots];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                     // NC chunks
  uint8_t* sR = smem + NC * kChunkBytes;  // kSlots chunk slots

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int q_tiles = (p.S + kBM - 1) / kBM;
  const Item it = make_item(p, static_cast<int>(blockIdx.x), q_tiles);
  const unsigned kid = 0xA0u + HD / 64;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 4);
    mbar_init(&pv_done, 1);
    mbar_init(&s_free, 4);
    mbar_init(&o_full, 1);
    mbar_init(&drain_bar, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], 1);
    }
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
    // ---------------- TMA producer ----------------
    if (lane == 0 && it.n > 0) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      mbar_arrive_expect_tx(&q_full, NC * kChunkBytes);
      for (int c = 0; c < NC; ++c)
        load_chunk(sQ + c * kChunkBytes, &map_q, &q_full, p, it.tq * kBM, it.h, it.b, c * kChunk);
      int n = 0;  // chunks loaded: tile j holds chunks [2*NC*j, 2*NC*(j+1)): K first, then V
      bool ok = true;
      for (int j = 0; j < it.n && ok; ++j) {
        for (int part = 0; part < 2 && ok; ++part) {
          for (int c = 0; c < NC; ++c, ++n) {
            const int s = n % kSlots;
            if (!mbar_wait(&slot_empty[s], ((n / kSlots) & 1) ^ 1u, &abort_flag, p.wait_limit_ns)) {
              report_error(kDevWaitTimeout, kid * 256 + kSiteEmpty);
              abort_flag = 1;
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&slot_full[s], kChunkBytes);
            load_chunk(sR + s * kChunkBytes, part == 0 ? &map_k : &map_v, &slot_full[s], p, j * kBN, it.h, it.b,
                       c * kChunk);
          }
        }
      }
      if (!ok) {
        // let copies already in flight land before the CTA can exit
        for (int t = max(0, n - kSlots); t < n; ++t)
          mbar_wait(&slot_full[t % kSlots], (t / kSlots) & 1, nullptr, kDrainLimitNs);
        mbar_wait(&q_full, 0, nullptr, kDrainLimitNs);
      }
    }
    if (lane == 0) grid_dep_launch();  // every load of this CTA is issued
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && it.n > 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kBM, kBN, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(kBM, kChunk, false, true);
      bool ok = true;
      auto fail = [&](unsigned site) {
        report_error(kDevWaitTimeout, kid * 256 + site);
        ok = false;
      };
      if (!mbar_wait(&q_full, 0, &abort_flag, p.wait_limit_ns)) fail(kSiteQ);
      auto wait_slot = [&](int n) -> uint32_t {
        const int s = n % kSlots;
        if (!mbar_wait(&slot_full[s], (n / kSlots) & 1, &abort_flag, p.wait_limit_ns)) fail(kSiteSlot);
        tc_fence_after();
        return static_cast<uint32_t>(s);
      };
      // S(j) = sum_c Q_c K_{j,c}^T into S's TMEM columns; the softmax must
      // have pulled S(j-1) into registers first (s_free).
      auto issue_s = [&](int j) {
        if (!ok) return;
        if (j > 0 && !mbar_wait(&s_free, (j - 1) & 1, &abort_flag, p.wait_limit_ns)) {
          fail(kSiteSFree);
          return;
        }
        for (int c = 0; c < NC && ok; ++c) {
          const uint32_t s = wait_slot(2 * NC * j + c);
          if (!ok) return;
          const uint32_t q_addr = smem_u32(sQ + c * kChunkBytes);
          const uint32_t k_addr = smem_u32(sR + s * kChunkBytes);
#pragma unroll
          for (int kk = 0; kk < kChunk / 16; ++kk) {
            const uint64_t dq = smem_desc(q_addr + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t dk = smem_desc(k_addr + kk * 32, 16, 1024, kLayoutSW128);
            mma_f16_ss(tmem_base + kColS, dq, dk, idesc_s, (c | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&slot_empty[s]);  // K chunk released when these MMAs complete
        }
        if (ok) mma_commit(&s_full);
      };
      // O[:, 64c:64c+64] += P(j) V_{j,c} once the softmax stored P(j) (p_full).
      auto issue_pv = [&](int j) {
        if (!ok) return;
        if (!mbar_wait(&p_full, j & 1, &abort_flag, p.wait_limit_ns)) {
          fail(kSiteP);
          return;
        }
        tc_fence_after();
        for (int c = 0; c < NC && ok; ++c) {
          const uint32_t s = wait_slot(2 * NC * j + NC + c);
          if (!ok) return;
          const uint32_t v_addr = smem_u32(sR + s * kChunkBytes);
#pragma unroll
          for (int ks = 0; ks < kBN / 16; ++ks) {
            const uint64_t dv = smem_desc(v_addr + ks * 16 * 128, kChunkBytes, 1024, kLayoutSW128);
            mma_f16_ts(tmem_base + kColO + c * kChunk, tmem_base + kColP + ks * 8, dv, idesc_o,
                       (j > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&slot_empty[s]);
        }
        if (!ok) return;
        mma_commit(&pv_done);  // P and O free for the softmax of tile j+1
        if (j + 1 == it.n) mma_commit(&o_full);
      };
      issue_s(0);
      for (int j = 0; j < it.n && ok; ++j) {
        if (j + 1 < it.n) issue_s(j + 1);
        issue_pv(j);
      }
      // everything issued is complete before TMEM can be released
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr, ok ? p.wait_limit_ns : kDrainLimitNs);
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ---------------- softmax, one query row per thread ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + static_cast<int>(lane);
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_s = t_lane + kColS;
    const uint32_t t_p = t_lane + kColP;
    const uint32_t t_o = t_lane + kColO;
    const float sl = p.scale_log2;
    const int q_idx = it.tq * kBM + r;
    float m = -INFINITY;  // running max, raw score units
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < it.n; ++j) {
      if (!mbar_wait_warp(&s_full, j & 1, &abort_flag, p.wait_limit_ns)) {
        report_error(kDevWaitTimeout, kid * 256 + kSiteS);
        abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kBN;
      // keys k0 + c are valid iff c < lim (causal diagonal and the kv bound)
      int lim = it.kv_bound - k0;
      if (p.causal) lim = min(lim, q_idx - k0 + 1);
      lim = max(0, min(kBN, lim));
      const bool full = lim >= kBN;
      // the score row 64 columns at a time (as in attn_fwd_kernel)
      uint32_t sv[2][32];
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      auto row_max = [&](const int col0) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (full || col0 + c * 32 + t < lim) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(sv[c][t]));
      };
      tmem_ld32(t_s, sv[0]);
      tmem_ld32(t_s + 32, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      row_max(0);
      tmem_ld32(t_s + 64, sv[0]);
      tmem_ld32(t_s + 96, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      row_max(64);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      float m_use = m;
      float alpha = 1.f;
      if (mx > m) {
        if (m == -INFINITY || (mx - m) * sl > kLazyRescaleLog2) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - mx) * sl);
          m_use = mx;
        }
      }
      const float neg_mc = (m_use == -INFINITY) ? 0.f : -m_use * sl;
      float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      auto exp_half = [&](const int col0) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            float x0, x1;
            fma2(x0, x1, __uint_as_float(sv[c][t]), __uint_as_float(sv[c][t + 1]), sl, neg_mc);
            sv[c][t] = __float_as_uint(x0);
            sv[c][t + 1] = __float_as_uint(x1);
          }
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) exp2_cols(sv[c][t], sv[c][t + 1], t);
        if (!full) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (col0 + c * 32 + t >= lim) sv[c][t] = 0u;
        }
        uint32_t pk[2][16];
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            const float p0 = __uint_as_float(sv[c][t]), p1 = __uint_as_float(sv[c][t + 1]);
            const int a = ((t >> 1) & 3) * 2;
            add2(rs[a], rs[a + 1], p0, p1);
            pk[c][t / 2] = pack_half2(p0, p1);
          }
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_st16(t_p + col0 / 2 + c * 16, pk[c]);
      };
      // PV(j-1) reads P and writes O: complete before P is overwritten or O rescaled.
      if (j > 0) {
        if (!mbar_wait_warp(&pv_done, (j - 1) & 1, &abort_flag, p.wait_limit_ns)) {
          report_error(kDevWaitTimeout, kid * 256 + kSitePv);
          abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
      }
      exp_half(64);
      tmem_ld32(t_s, sv[0]);
      tmem_ld32(t_s + 32, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      // S is fully in registers: the MMA warp may compute the next tile's scores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free);
      exp_half(0);
      const float row_sum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      const bool need = (j > 0) && (alpha != 1.f);
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          uint32_t o[16];
          tmem_ld16(t_o + c, o);
          tmem_ld_wait(o);
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st16(t_o + c, o);
        }
      }
      l = l * alpha + row_sum;
      m = m_use;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    // epilogue: O / l -> fp16 [b, q, h*HD + c]
    if (ok && it.n > 0) {
      if (!mbar_wait_warp(&o_full, 0, &abort_flag, p.wait_limit_ns)) {
        report_error(kDevWaitTimeout, kid * 256 + kSiteO);
        abort_flag = 1;
        ok = false;
      }
      tc_fence_after();
    }
    if (ok && it.tq < q_tiles) {
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      __half* dst = p.out + (static_cast<int64_t>(it.b) * p.S + q_idx) * p.ld_out + it.h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 16) {
        uint32_t o[16];
        if (it.n > 0) {
          tmem_ld16(t_o + c, o);
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

}  // namespace wide
}  // namespace attn
}  // namespace tk
