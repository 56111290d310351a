// Blackwell flash-attention forward.
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
// Persistent: one CTA per SM loops over work items (b, h, pair of 128-query
// tiles), heaviest first; TMEM stays allocated, Q is double-buffered, the
// K/V ring and all barrier phases run on across items, and the next item's
// first S = QK^T overlaps the current item's epilogue. Three warpgroups:
// warp 0 TMA, warp 1 TMEM owner + MMA issuer (warps 2 and 3 have no role),
// warps 4..7 softmax group 0 (query tile 2p), warps 8..11 softmax group 1
// (tile 2p+1). setmaxnreg moves registers from the first warpgroup to the
// softmax groups (224 per thread), so each softmax thread holds its query
// row's whole 128-column score tile (its warp's TMEM lane quadrant). Both groups
// share every K/V tile. TMEM (512 columns): S_g = Q_g K^T in columns
// [128g, 128g+128) fp32, P_g = softmax numerators as packed fp16 pairs in
// [256+64g, 320+64g), O_g in [384+64g, 384+64g+HD).
//   S_g(j) : tcgen05.mma SS, M=128 N=128 K=16 x (HD/16)     (A=Q_g, B=K_j, both K-major)
//   O_g   += P_g(j) V_j : tcgen05.mma TS, M=128 N=HD K=16 x 8 (A=P_g in TMEM, B=V_j MN-major)
// Group g signals s_free as soon as it has pulled S_g(j) into registers; the
// MMA warp then computes S_g(j+1) during tile j's exponentials, and issues
// PV_g(j) once P_g(j) is written (p_full). Group g waits for PV_g(j)
// (pv_done) only right before it overwrites P_g or rescales O_g.
// With two groups, one group's softmax runs while the tensor core works for
// the other.
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

constexpr int kBM = 128;  // queries per tile (two tiles per CTA)
constexpr int kBN = 128;  // keys per KV tile
constexpr int kThreads = 384;
// Register split (setmaxnreg): the kernel is built for kLaunchRegs registers
// per thread (the 384-thread cap of 65,536 / 384, rounded down to 8); warpgroup
// 0 (TMA, MMA, two idle warps) drops to kProducerRegs and the two softmax
// warpgroups take what it frees. The split uses exactly the launch allocation
// (an inc above it would wait forever), and each sub-partition holds one
// warpgroup-0 warp and two softmax warps: 56 * 32 + 2 * 224 * 32 = 16,128 of
// its 16,384 registers. The host refuses to launch if the built register
// count is not kLaunchRegs.
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 56;
constexpr int kSoftmaxRegs = 224;
static_assert(4 * 32 * kProducerRegs + 8 * 32 * kSoftmaxRegs == kThreads * kLaunchRegs, "register split");
static_assert(kProducerRegs * 32 + 2 * kSoftmaxRegs * 32 <= 16384, "sub-partition register file");
constexpr int kStages = 4;
constexpr int kTmemCols = 512;
constexpr int kColP = 256;  // P_g at kColP + 64 g (packed fp16 pairs)
constexpr int kColO = 384;  // O_g at kColO + 64 g (fp32, HD <= 64 columns)
constexpr float kLazyRescaleLog2 = 8.f;
// Of every 8 consecutive score columns, this many take 2^x on the FMA pipe
// (exp2_fma_pair, two columns per f32x2 instruction) instead of the SFU: the
// SFU (16 results/clk/SM) is the softmax's bottleneck at head_dim 64, and the
// FMA pipe has room. Even, so that column pairs stay on one pipe.
constexpr int kExpFmaPer8 = 2;
static_assert(kExpFmaPer8 % 2 == 0, "FMA-pipe exponentials go in column pairs");

// 2^x on the FMA/ALU pipes for a pair of values x <= 8 (scores minus the
// running max), two columns per f32x2 instruction. Cody-Waite style range
// reduction x = n + f with n = rint(x), |f| <= 1/2 (adding 1.5 * 2^23 rounds
// x to an integer in the low mantissa bits), then 2^f by a degree-3
// polynomial fitted here for minimum maximum relative error on [-1/2, 1/2]
// (7.5e-5, below the 2^-11 fp16 rounding that P gets), and 2^n added into
// the exponent field. x is clamped at -126 so the exponent cannot wrap;
// 2^-126 becomes 0 in the fp16 P.
__device__ __forceinline__ float2 exp2_fma_pair(float2 x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr float kC0 = 0.99992811f, kC1 = 0.69326099f, kC2 = 0.24261054f, kC3 = 0.05517132f;
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = fadd2(x, splat2(kRound));                            // n + 1.5 * 2^23
  const float2 f = ffma2(fadd2(t, splat2(-kRound)), splat2(-1.f), x);  // x - n
  const float2 q = ffma2(ffma2(ffma2(splat2(kC3), f, splat2(kC2)), f, splat2(kC1)), f, splat2(kC0));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// 2^x of score columns t and t + 1 (t even) in place: the pair goes to the
// FMA pipe when its columns are among the last kExpFmaPer8 of their group of
// eight, else each value to the SFU.
__device__ __forceinline__ void exp2_cols(uint32_t& a, uint32_t& b, int t) {
  const float2 x = make_float2(__uint_as_float(a), __uint_as_float(b));
  float2 y;
  if ((t & 7) >= 8 - kExpFmaPer8) {
    y = exp2_fma_pair(x);
  } else {
    y.x = ex2_approx(x.x);
    y.y = ex2_approx(x.y);
  }
  a = __float_as_uint(y.x);
  b = __float_as_uint(y.y);
}

struct Params {
  __half* out;          // [B, S, ld_out] fp16, head h at columns [h*HD, h*HD+HD)
  int64_t ld_out;
  int B, S, H;
  float scale_log2;     // hd**-0.5 * log2(e)
  int causal;
  const int* kv_len;    // optional [B]: keys >= kv_len[b] are masked
  int heads_inner;      // tensor-map dim order {hd, H, S, B} (1) or {hd, S, H, B} (0)
  int hd;               // head_dim of the data: HD, or 8 for the HD = 16 kernel (zero-padded by TMA)
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
  static_assert(HD == 16 || HD == 32 || HD == 64, "head_dim");
  static constexpr int ROW_BYTES = HD * 2;                     // swizzle span
  static constexpr SmemLayout LAYOUT = HD == 64 ? kLayoutSW128 : HD == 32 ? kLayoutSW64 : kLayoutSW32;
  static constexpr int TILE_BYTES = kBM * ROW_BYTES;           // Q, K or V tile
  static constexpr int SBO = 8 * ROW_BYTES;                    // 8-row core-matrix group
  static constexpr int SMEM_BYTES = TILE_BYTES * (4 + 2 * kStages) + 1024;  // 2 Q sets of 2 tiles
};

enum : unsigned { kSiteQ = 1, kSiteKV = 2, kSiteS = 3, kSiteP = 4, kSiteO = 5, kSiteEmpty = 6, kSiteOFree = 7,
                  kSiteQEmpty = 8, kSitePv = 9, kSiteSFree = 10 };

// One work item = (b, h, pair of query tiles); heaviest (last, for causal)
// pairs first so the static round-robin over CTAs stays balanced.
struct Item {
  int b, h, tq0, tq1, kv_bound;
  int last[2];  // KV tiles attended by group 0 / group 1 (0 = group idle)
  int n_kv;
  bool has1;
};

__device__ __forceinline__ Item make_item(const Params& p, int idx, int q_tiles, int q_pairs) {
  Item it;
  const int bh_count = p.B * p.H;
  const int qp = q_pairs - 1 - idx / bh_count;
  const int bh = idx % bh_count;
  it.b = bh / p.H;
  it.h = bh % p.H;
  it.tq0 = 2 * qp;
  it.tq1 = 2 * qp + 1;
  it.has1 = it.tq1 < q_tiles;
  it.kv_bound = p.S;
  if (p.kv_len != nullptr) it.kv_bound = max(0, min(p.S, p.kv_len[it.b]));
  const int n_all = (it.kv_bound + kBN - 1) / kBN;
  it.last[0] = p.causal ? min(n_all, it.tq0 + 1) : n_all;
  it.last[1] = it.has1 ? (p.causal ? min(n_all, it.tq1 + 1) : n_all) : 0;
  it.n_kv = max(it.last[0], it.last[1]);
  return it;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, Params p) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full[2];      // per Q buffer set
  __shared__ __align__(8) uint64_t q_empty[2];
  __shared__ __align__(8) uint64_t kv_full[kStages];
  __shared__ __align__(8) uint64_t kv_empty[kStages];
  __shared__ __align__(8) uint64_t s_full[2];      // per softmax group
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t o_full[2];
  __shared__ __align__(8) uint64_t o_free[2];
  __shared__ __align__(8) uint64_t pv_done[2];
  __shared__ __align__(8) uint64_t s_free[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // 2 sets x 2 tiles
  uint8_t* sK = smem + 4 * C::TILE_BYTES;               // kStages tiles
  uint8_t* sV = smem + C::TILE_BYTES * (4 + kStages);   // kStages tiles

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int q_tiles = (p.S + kBM - 1) / kBM;
  const int q_pairs = (q_tiles + 1) / 2;
  const int n_items = q_pairs * p.B * p.H;
  const unsigned kid = 0x80u + HD;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 4);
      mbar_init(&o_full[g], 1);
      mbar_init(&o_free[g], 4);
      mbar_init(&pv_done[g], 1);
      mbar_init(&s_free[g], 4);
    }
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

  // Register split: every warp of a warpgroup executes the same setmaxnreg,
  // which dominates that warpgroup's role code.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == 0) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_k);
        prefetch_tensormap(&map_v);
        int kv_count = 0;  // KV tiles loaded so far (ring position)
        int qn = 0;        // items with work loaded so far (Q buffer set = qn & 1)
        bool ok = true;
        for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
          const Item it = make_item(p, idx, q_tiles, q_pairs);
          if (it.n_kv == 0) continue;
          const int qs = qn & 1;
          const uint32_t q_phase = (qn >> 1) & 1;
          ++qn;
          if (!mbar_wait(&q_empty[qs], q_phase ^ 1u, &abort_flag, p.wait_limit_ns)) {
            report_error(kDevWaitTimeout, kid * 256 + kSiteQEmpty);
            abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* q_dst = sQ + qs * 2 * C::TILE_BYTES;
          mbar_arrive_expect_tx(&q_full[qs], C::TILE_BYTES * (it.has1 ? 2 : 1));
          load_tile(q_dst, &map_q, &q_full[qs], p, it.tq0 * kBM, it.h, it.b);
          if (it.has1) load_tile(q_dst + C::TILE_BYTES, &map_q, &q_full[qs], p, it.tq1 * kBM, it.h, it.b);
          for (int j = 0; j < it.n_kv; ++j, ++kv_count) {
            const int s = kv_count % kStages;
            const uint32_t ph = (kv_count / kStages) & 1;
            if (!mbar_wait(&kv_empty[s], ph ^ 1u, &abort_flag, p.wait_limit_ns)) {
              report_error(kDevWaitTimeout, kid * 256 + kSiteEmpty);
              abort_flag = 1;
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&kv_full[s], 2 * C::TILE_BYTES);
            load_tile(sK + s * C::TILE_BYTES, &map_k, &kv_full[s], p, j * kBN, it.h, it.b);
            load_tile(sV + s * C::TILE_BYTES, &map_v, &kv_full[s], p, j * kBN, it.h, it.b);
          }
        }
        // all of this CTA's loads are issued: the next kernel may be scheduled
        grid_dep_launch();
        if (!ok) {
          // let copies already in flight land before the CTA can exit
          for (int t = max(0, kv_count - kStages); t < kv_count; ++t)
            mbar_wait(&kv_full[t % kStages], (t / kStages) & 1, nullptr, kDrainLimitNs);
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        constexpr uint32_t idesc_s = idesc_f16_f32(kBM, kBN, false, false);
        constexpr uint32_t idesc_o = idesc_f16_f32(kBM, HD, false, true);
        // Per-group counters live in named scalars and every per-group step is
        // expanded for g = 0 and g = 1 separately, so nothing on this
        // single-thread critical path is indexed dynamically (local memory).
        struct Group {
          int tiles = 0;     // tiles handed over by the softmax (p_full phases)
          int o_uses = 0;    // items in which O_g was accumulated (o_full / o_free phases)
          int s_issued = 0;  // S_g MMAs issued (s_free phases)
        };
        Group grp0, grp1;
        int kv_count = 0;  // KV tiles consumed so far (ring position)
        int qn = 0;        // items with work consumed so far (Q buffer set = qn & 1)
        bool ok = true;
        auto fail = [&](unsigned site) {
          report_error(kDevWaitTimeout, kid * 256 + site);
          ok = false;
        };
        for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
          const Item it = make_item(p, idx, q_tiles, q_pairs);
          if (it.n_kv == 0) continue;
          const int last0 = it.last[0], last1 = it.last[1];
          const int qs = qn & 1;
          const uint32_t q_phase = (qn >> 1) & 1;
          ++qn;
          if (!mbar_wait(&q_full[qs], q_phase, &abort_flag, p.wait_limit_ns)) {
            fail(kSiteQ);
            break;
          }
          const int kv_base = kv_count;
          int kv_ready = -1;
          auto wait_kv = [&](int j) -> bool {
            if (j <= kv_ready) return true;
            const int t = kv_base + j;
            if (!mbar_wait(&kv_full[t % kStages], (t / kStages) & 1, &abort_flag, p.wait_limit_ns)) {
              fail(kSiteKV);
              return false;
            }
            kv_ready = j;
            return true;
          };
          // S_g(j) overwrites S_g: the softmax must have pulled the previous
          // scores of group g into registers (s_free) first.
          auto issue_s = [&](Group& gs, const int g, int j) {
            if (!ok) return;
            if (!wait_kv(j)) return;
            if (gs.s_issued > 0 && !mbar_wait(&s_free[g], (gs.s_issued - 1) & 1, &abort_flag, p.wait_limit_ns)) {
              fail(kSiteSFree);
              return;
            }
            ++gs.s_issued;
            tc_fence_after();
            const uint32_t q_addr = smem_u32(sQ + (qs * 2 + g) * C::TILE_BYTES);
            const uint32_t k_addr = smem_u32(sK + ((kv_base + j) % kStages) * C::TILE_BYTES);
  #pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t dq = smem_desc(q_addr + kk * 32, 16, C::SBO, C::LAYOUT);
              const uint64_t dk = smem_desc(k_addr + kk * 32, 16, C::SBO, C::LAYOUT);
              mma_f16_ss(tmem_base + g * kBN, dq, dk, idesc_s, kk > 0 ? 1u : 0u);
            }
            mma_commit(&s_full[g]);
          };
          // O_g += P_g(j) V_j once group g has written P_g(j) (p_full).
          auto issue_pv = [&](Group& gs, const int g, int j, int last_g, bool last_reader) {
            if (!ok) return;
            if (!mbar_wait(&p_full[g], gs.tiles & 1, &abort_flag, p.wait_limit_ns)) {
              fail(kSiteP);
              return;
            }
            ++gs.tiles;
            if (j == 0 && gs.o_uses > 0 &&
                !mbar_wait(&o_free[g], (gs.o_uses - 1) & 1, &abort_flag, p.wait_limit_ns)) {
              // the previous item's epilogue of group g must be done reading O_g
              fail(kSiteOFree);
              return;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(sV + ((kv_base + j) % kStages) * C::TILE_BYTES);
  #pragma unroll
            for (int ks = 0; ks < kBN / 16; ++ks) {
              const uint64_t dv = smem_desc(v_addr + ks * 16 * C::ROW_BYTES, C::TILE_BYTES, C::SBO, C::LAYOUT);
              mma_f16_ts(tmem_base + kColO + g * 64, tmem_base + kColP + g * 64 + ks * 8, dv, idesc_o,
                         (j > 0 || ks > 0) ? 1u : 0u);
            }
            mma_commit(&pv_done[g]);  // P_g and O_g free for the softmax of tile j+1
            if (last_reader) mma_commit(&kv_empty[(kv_base + j) % kStages]);  // K_j / V_j released
            if (j + 1 == last_g) {
              mma_commit(&o_full[g]);
              ++gs.o_uses;
            }
          };
          if (last0 > 0) issue_s(grp0, 0, 0);
          if (last1 > 0) issue_s(grp1, 1, 0);
          for (int j = 0; j < it.n_kv && ok; ++j) {
            // S_g(j+1) as soon as group g has pulled S_g(j) into registers, so the
            // next scores are computed during tile j's exponentials.
            if (j + 1 < last0) issue_s(grp0, 0, j + 1);
            if (j + 1 < last1) issue_s(grp1, 1, j + 1);
            // the last reader of K_j / V_j (group 1 when it attends tile j) releases the stage
            if (j < last0) issue_pv(grp0, 0, j, last0, j >= last1);
            if (j < last1) issue_pv(grp1, 1, j, last1, true);
          }
          if (!ok) break;
          mma_commit(&q_empty[qs]);  // every S of this item read its Q set
          kv_count += it.n_kv;
        }
        // everything issued is complete before TMEM can be released
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, nullptr, ok ? p.wait_limit_ns : kDrainLimitNs);
        if (!ok) abort_flag = 1;
      }
      __syncwarp();
    }  // warps 2 and 3: no role
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ---------------- softmax, group g, one query row per thread ----------------
    const int g = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + static_cast<int>(lane);
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_s = t_lane + g * kBN;
    const uint32_t t_p = t_lane + kColP + g * 64;
    const uint32_t t_o = t_lane + kColO + g * 64;
    const float sl = p.scale_log2;
    int tiles = 0, o_uses = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
      const Item it = make_item(p, idx, q_tiles, q_pairs);
      const int tq = g == 0 ? it.tq0 : it.tq1;
      const int n_g = g == 0 ? it.last[0] : it.last[1];  // no runtime index: Item stays in registers
      const int q_idx = tq * kBM + r;
      float m = -INFINITY;  // running max, raw score units
      float l = 0.f;
      for (int j = 0; j < n_g; ++j, ++tiles) {
        if (!mbar_wait_warp(&s_full[g], tiles & 1, &abort_flag, p.wait_limit_ns)) {
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

        // The whole 128-column score row is pulled into registers with one
        // TMEM read and S_g is released to the MMA warp at once, so S_g(j+1)
        // is computed during this tile's exponentials. Then: row max, lazy
        // rescale decision, exponentials, fp16 packing with the row sums,
        // and P_g stored once PV_g(j-1) has read the previous P.
        const bool full = lim >= kBN;  // masking only on the causal diagonal / kv-bound tile
        uint32_t sv[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, sv[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_wait(sv[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[g]);
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (full) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int t = 0; t < 32; t += 2)
              mx4[(t >> 1) & 3] = max3(mx4[(t >> 1) & 3], __uint_as_float(sv[c][t]), __uint_as_float(sv[c][t + 1]));
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
          if (m == -INFINITY || (mx - m) * sl > kLazyRescaleLog2) {
            alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - mx) * sl);
            m_use = mx;
          }
        }
        const float neg_mc = (m_use == -INFINITY) ? 0.f : -m_use * sl;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            float x0, x1;
            fma2(x0, x1, __uint_as_float(sv[c][t]), __uint_as_float(sv[c][t + 1]), sl, neg_mc);
            sv[c][t] = __float_as_uint(x0);
            sv[c][t + 1] = __float_as_uint(x1);
          }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) exp2_cols(sv[c][t], sv[c][t + 1], t);
        if (!full) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (c * 32 + t >= lim) sv[c][t] = 0u;
        }
        float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t pk[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            const float p0 = __uint_as_float(sv[c][t]), p1 = __uint_as_float(sv[c][t + 1]);
            const int a = ((t >> 1) & 3) * 2;
            add2(rs[a], rs[a + 1], p0, p1);
            pk[c][t / 2] = pack_half2(p0, p1);
          }
        // PV_g of the previous tile reads P_g and writes O_g: it must be
        // complete before P_g is overwritten or O_g rescaled.
        if (tiles > 0) {
          if (!mbar_wait_warp(&pv_done[g], (tiles - 1) & 1, &abort_flag, p.wait_limit_ns)) {
            report_error(kDevWaitTimeout, kid * 256 + kSitePv);
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_st16(t_p + c * 16, pk[c]);
        const float row_sum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
        const bool need = (j > 0) && (alpha != 1.f);
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
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
        if (lane == 0) mbar_arrive(&p_full[g]);
      }
      if (!ok) break;
      // epilogue: O / l -> fp16 [b, q, h*HD + c]
      if (n_g > 0) {
        if (!mbar_wait_warp(&o_full[g], o_uses & 1, &abort_flag, p.wait_limit_ns)) {
          report_error(kDevWaitTimeout, kid * 256 + kSiteO);
          abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (tq < q_tiles) {
        const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
        __half* dst = p.out + (static_cast<int64_t>(it.b) * p.S + q_idx) * p.ld_out + it.h * p.hd;
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          uint32_t o[16];
          if (n_g > 0) {
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
            if (c + 16 <= p.hd) reinterpret_cast<uint4*>(dst + c)[1] = w1;  // head_dim 8: columns 8..15 are padding
          }
        }
      }
      if (n_g > 0) {
        ++o_uses;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[g]);
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
