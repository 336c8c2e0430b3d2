// Tensor-core tree attention on CTA pairs (tcgen05 cta_group::2) for sm_100a.
//
// Unit of work: 256 packed query rows of one (sequence b, kv head) -- a
// "unit", the rows g * n + i for query head g of the kv head's group and
// tree node i -- run by a cluster of two CTAs: CTA rank r holds rows
// r * 128 .. r * 128 + 127 in its TMEM lanes.  Key/value tiles are 128 rows.
// One tcgen05.mma.cta_group::2 instruction, issued by the even CTA, computes
// M = 256 rows at once, each CTA supplying its own 128 rows of the A operand
// and half of B:
//
//   S = Q K^T   M 256, N 128 keys, K 16: CTA r holds keys r*64 .. r*64+63 of
//               the tile (K-major), the result lands in both CTAs' TMEM.
//   O += P V    M 256, N 128 (head_dim), K 16 keys: P from each CTA's TMEM,
//               CTA r holds V's columns r*64 .. r*64+63 of all 128 keys.
//
// Per SM this is the single-CTA kernel's work per key and query row, but
// Q.K^T runs at N = 128 with half of B per CTA (6 KB of shared-memory
// operands per 64 cycles of math, against 6 KB per 32 for the single CTA's
// N = 64 tiles, where the tensor pipe waits on shared memory), and every CTA
// stages half a K/V tile per 128 keys.
//
// The even CTA's producers load both CTAs' halves (non-multicast
// cta_group::2 tile loads into either CTA's shared memory, completing on the
// even CTA's barriers); its two issuer threads issue every MMA and commit
// each result to the barriers of both CTAs.  Each CTA runs two softmax
// warpgroups: warpgroup j takes the tiles of parity j (tile i uses S buffer
// i & 1 and accumulates into O_j), so the two keep independent running
// maxima and sums and never wait for each other inside a unit; the epilogue
// merges O_0 and O_1 once per unit.
//
// TMEM (512 columns per CTA): S_0, S_1 (128 columns each, fp32 scores; P as
// 16-bit pairs overwrites columns 0-31 for keys 0-63 and 64-95 for keys
// 64-127 of its own S buffer) and O_0, O_1 (128 columns each).
//
// Warp roles (384 threads per CTA):
//   warp 0       (even CTA) TMA producer for K, both CTAs' halves
//   warp 3       (even CTA) TMA producer for V, both CTAs' halves
//   warp 1       (even CTA) Q.K^T issuer (one thread)
//   warp 2       (even CTA) P.V issuer (one thread); in both CTAs it
//                allocates and frees the pair's TMEM
//   warps 4-7    softmax of the even tiles (warpgroup 0)
//   warps 8-11   softmax of the odd tiles (warpgroup 1)
//
// Every wait is bounded (wait_limit_ns()); a CTA whose wait runs out sets
// its own and its partner's abort flag, so both stop, drain what they
// issued, free TMEM and raise kErrTimeout.  Whole units only.  It runs when
// asked for (backend GORGON_BACKEND_TCGEN05_PAIR): measured on B200 it is
// slower than the single-CTA kernel, so the planner does not pick it.
#include <cuda.h>

#include <mutex>
#include <utility>
#include <vector>

#include "attn.cuh"
#include "sm100.cuh"
#include "attn_tc_common.cuh"

namespace gorgon {
namespace {
using namespace sm100;

constexpr int kPRows = 256;                     // packed query rows per unit (both CTAs)
constexpr int kPBN = 128;                       // keys per tile
constexpr int kPStages = 5;                     // K and V ring depth
constexpr int kPThreads = 384;
constexpr uint32_t kPKBox = 64 * 128;           // K box: 64 rows x 64 columns = 8 KB
constexpr uint32_t kPKStage = 2 * kPKBox;       // this CTA's 64 keys x 128 columns
constexpr uint32_t kPVStage = kPBN * 128;       // 128 keys x this CTA's 64 columns
constexpr uint32_t kPOffQ = 0;                  // 2 halves x 16 KB
constexpr uint32_t kPOffK = 2 * kQHalf;
constexpr uint32_t kPOffV = kPOffK + kPStages * kPKStage;
constexpr uint32_t kPOffBar = kPOffV + kPStages * kPVStage;
constexpr uint32_t kPOffMl = kPOffBar + 512;    // [2 warpgroups][128 rows] (m, l)
constexpr uint32_t kPSmem = kPOffMl + 2 * 128 * 8 + 1024;  // + alignment slack
static_assert(kPSmem <= 232448, "shared memory per block");
constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPColS = 0;                  // + j * 128
constexpr uint32_t kPColO = 256;                // + j * 128

struct PairArgs {
  AttnArgs a;
  int qgroups;         // units per (b, kv head)
  int units;           // batch * hkv * qgroups
  int tiles;           // 128-key tiles per unit
  int ab_fmt;          // 0 f16, 1 bf16
  int out_bf16;        // 1: bf16 output rows, 0: f16 (16-byte aligned rows)
  uint64_t wait_ns;
};

struct PairBars {
  uint64_t k_full[kPStages];   // even CTA: both halves of a K stage landed
  uint64_t k_empty[kPStages];  // even CTA: the stage's Q.K^T completed
  uint64_t v_full[kPStages];
  uint64_t v_empty[kPStages];
  uint64_t q_full;             // even CTA: 16 softmax warps (8 per CTA) stored the unit's Q
  uint64_t s_full[2];          // each CTA: S_j of the current tile of parity j is in TMEM
  uint64_t p_full[2];          // even CTA: 8 warps (warpgroup j of both CTAs) stored P_j
  uint64_t p_free[2];          // each CTA: P.V of the tile of parity j completed
  uint64_t ml_ready;           // each CTA: both warpgroups posted (m, l) of the unit
  uint64_t unit_done;          // each CTA: both warpgroups finished the unit's epilogue
  uint64_t drain[2];           // even CTA: the issuers' last MMAs completed
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(PairBars) <= 512, "barrier block");

struct UnitInfo {
  int b, kvh, qg;
};
__device__ __forceinline__ UnitInfo unit_info(const PairArgs& t, int u) {
  UnitInfo ui;
  ui.qg = u % t.qgroups;
  ui.kvh = (u / t.qgroups) % t.a.hkv;
  ui.b = u / (t.qgroups * t.a.hkv);
  return ui;
}

// Stops both CTAs of the pair: this CTA's flag (set by the wait that ran
// out) and the partner's.
__device__ __forceinline__ void abort_pair(PairBars* bars, uint32_t peer) {
  bars->abort = 1;
  st_cluster_u32(map_shared(&bars->abort, peer), 1u);
}

__device__ __forceinline__ bool pair_wait(const PairArgs& t, PairBars* bars, uint64_t* bar, uint32_t parity,
                                          uint32_t peer) {
  if (bounded_wait(bar, parity, &bars->abort, t.wait_ns)) return true;
  abort_pair(bars, peer);
  return false;
}
template <bool kCluster>
__device__ __forceinline__ bool pair_spin(const PairArgs& t, PairBars* bars, uint64_t* bar, uint32_t parity,
                                          uint32_t peer) {
  if (spin_wait<kCluster>(bar, parity, &bars->abort, t.wait_ns)) return true;
  abort_pair(bars, peer);
  return false;
}
__device__ __forceinline__ bool pair_warp_wait(const PairArgs& t, PairBars* bars, uint64_t* bar, uint32_t parity,
                                               uint32_t peer) {
  const bool ok = __all_sync(0xffffffffu, bounded_wait(bar, parity, &bars->abort, t.wait_ns));
  if (!ok && (threadIdx.x & 31) == 0) abort_pair(bars, peer);
  return ok;
}

// ------------------------------------------------------------ producers
// Streams K (is_v == 0) or V of every tile of the pair's units: both CTAs'
// halves, completing on this (the even) CTA's full barrier of the stage.
__device__ void pair_producer(const PairArgs& t, const CUtensorMap* map, uint8_t* smem, PairBars* bars, int is_v) {
  uint64_t* full = is_v ? bars->v_full : bars->k_full;
  uint64_t* empty = is_v ? bars->v_empty : bars->k_empty;
  const uint32_t ring = is_v ? kPOffV : kPOffK;
  const uint32_t stage_bytes = is_v ? kPVStage : kPKStage;
  const uint32_t own = map_shared(smem + ring, 0), peer = map_shared(smem + ring, 1);
  // A unit's K/V feed only its own CTA pair when each (b, kv head) is one
  // unit: keep them from pushing other data out of L2.  With several units
  // per (b, kv head) the pairs that share K/V run side by side (units are
  // dealt out in order), and the later ones should find it in L2.
  const uint64_t policy = t.qgroups > 1 ? l2_policy_evict_last() : l2_policy_evict_first();
  const int pairs = gridDim.x / 2;
  uint32_t issued = 0;
  bool ok = true;
  for (int u = blockIdx.x / 2; ok && u < t.units; u += pairs) {
    const UnitInfo ui = unit_info(t, u);
    for (int tile = 0; tile < t.tiles; ++tile, ++issued) {
      const uint32_t stage = issued % kPStages;
      const uint32_t ph = (issued / kPStages) & 1u;
      if (!pair_wait(t, bars, &empty[stage], ph ^ 1u, 1)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[stage], 2 * stage_bytes);
      const uint32_t bar = map_shared(&full[stage], 0);
      const uint32_t off = stage * stage_bytes;
      const int row = tile * kPBN;
      if (is_v) {
        // this CTA's V half: columns 0-63 of all 128 keys; the partner's: 64-127
        tma_load_4d_pair(own + off, map, bar, 0, row, ui.kvh, ui.b, policy);
        tma_load_4d_pair(peer + off, map, bar, 64, row, ui.kvh, ui.b, policy);
      } else {
        // this CTA's K half: keys 0-63 of the tile; the partner's: keys 64-127
        tma_load_4d_pair(own + off, map, bar, 0, row, ui.kvh, ui.b, policy);
        tma_load_4d_pair(own + off + kPKBox, map, bar, 64, row, ui.kvh, ui.b, policy);
        tma_load_4d_pair(peer + off, map, bar, 0, row + 64, ui.kvh, ui.b, policy);
        tma_load_4d_pair(peer + off + kPKBox, map, bar, 64, row + 64, ui.kvh, ui.b, policy);
      }
    }
  }
  // Every issued load must land (in both CTAs) before the pair leaves.
  for (uint32_t k = (issued > kPStages ? issued - kPStages : 0); k < issued; ++k)
    drain_wait(&full[k % kPStages], (k / kPStages) & 1u);
}

// ------------------------------------------------------------ issuers
__device__ __forceinline__ uint64_t pair_desc(uint8_t* smem, uint32_t off, uint32_t lbo) {
  return umma_desc_sw128(smem_u32(smem + off), lbo, 1024);
}

// Every Q.K^T: tile i into S buffer i & 1, once its K stage has landed and
// the P.V that last read that buffer (tile i - 2) has completed.
__device__ void pair_qk_issuer(const PairArgs& t, uint8_t* smem, PairBars* bars, uint32_t tmem) {
  const uint64_t q0 = pair_desc(smem, kPOffQ, 16);
  const uint64_t k0 = pair_desc(smem, kPOffK, 16);
  const uint32_t idesc = umma_idesc_f16(t.ab_fmt, kPRows, kPBN, 0, 0);
  const int pairs = gridDim.x / 2;
  uint32_t i = 0, seg = 0, stage = 0, phase = 0;
  bool ok = true;
  for (int u = blockIdx.x / 2; ok && u < t.units; u += pairs, ++seg) {
    if (!pair_spin<true>(t, bars, &bars->q_full, seg & 1u, 1)) break;
    for (int tile = 0; tile < t.tiles; ++tile, ++i) {
      const uint32_t buf = i & 1u;
      if (!pair_spin<true>(t, bars, &bars->k_full[stage], phase, 1) ||
          (i >= 2 && !pair_spin<false>(t, bars, &bars->p_free[buf], ((i - 2) >> 1) & 1u, 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t kst = k0 + static_cast<uint64_t>(stage * (kPKStage >> 4));
      const uint32_t d_tmem = tmem + kPColS + buf * 128;
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        const uint64_t a = q0 + static_cast<uint64_t>((ks >> 2) * (kQHalf >> 4) + (ks & 3) * 2);
        const uint64_t b = kst + static_cast<uint64_t>((ks >> 2) * (kPKBox >> 4) + (ks & 3) * 2);
        umma_f16_ss_pair(d_tmem, a, b, idesc, ks > 0 ? 1u : 0u);
      }
      umma_commit_pair(map_shared(&bars->s_full[buf], 0));
      umma_commit_pair(map_shared(&bars->s_full[buf], 1));
      umma_commit_pair(map_shared(&bars->k_empty[stage], 0));
      if (++stage == kPStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  umma_commit_pair(map_shared(&bars->drain[0], 0));
  drain_wait(&bars->drain[0], 0);
}

// Every P.V: O_{i&1} += P_i V_i once both CTAs' warpgroup i & 1 stored P_i.
// P for keys 0-63 sits in columns 0-31 of the S buffer, keys 64-127 in 64-95.
__device__ void pair_pv_issuer(const PairArgs& t, uint8_t* smem, PairBars* bars, uint32_t tmem) {
  const uint64_t v0 = pair_desc(smem, kPOffV, kPVStage);
  const uint32_t idesc = umma_idesc_f16(t.ab_fmt, kPRows, kD, 0, 1);
  const int pairs = gridDim.x / 2;
  uint32_t i = 0, stage = 0, phase = 0;
  bool ok = true;
  for (int u = blockIdx.x / 2; ok && u < t.units; u += pairs) {
    for (int tile = 0; tile < t.tiles; ++tile, ++i) {
      const uint32_t buf = i & 1u;
      if (!pair_spin<true>(t, bars, &bars->v_full[stage], phase, 1) ||
          !pair_spin<true>(t, bars, &bars->p_full[buf], (i >> 1) & 1u, 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t vst = v0 + static_cast<uint64_t>(stage * (kPVStage >> 4));
      const uint32_t d_tmem = tmem + kPColO + buf * 128;
      const uint32_t p_tmem = tmem + kPColS + buf * 128;
      const bool first = tile < 2;  // the unit's first tile of this parity starts O_buf afresh
#pragma unroll
      for (int ks = 0; ks < kPBN / 16; ++ks)
        umma_f16_ts_pair(d_tmem, p_tmem + ks * 8 + (ks >= 4 ? 32 : 0), vst + static_cast<uint64_t>(ks * (2048 >> 4)),
                         idesc, (ks > 0 || !first) ? 1u : 0u);
      umma_commit_pair(map_shared(&bars->p_free[buf], 0));
      umma_commit_pair(map_shared(&bars->p_free[buf], 1));
      umma_commit_pair(map_shared(&bars->v_empty[stage], 0));
      if (++stage == kPStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  umma_commit_pair(map_shared(&bars->drain[1], 0));
  drain_wait(&bars->drain[1], 0);
}

// ------------------------------------------------------------ softmax + epilogue
// Arrives on a barrier of the even CTA from either CTA (one arrival per warp).
__device__ __forceinline__ void arrive_even(uint64_t* bar, uint32_t rank) {
  if (rank == 0) mbar_arrive(bar);
  else mbar_arrive_cluster(map_shared(bar, 0));
}

template <int ANCW, bool BF16>
__device__ void pair_softmax(const PairArgs& t, uint8_t* smem, PairBars* bars, uint32_t tmem, uint32_t rank) {
  const AttnArgs& a = t.a;
  const uint32_t peer = rank ^ 1u;
  const int j = (threadIdx.x >> 7) - 1;        // warpgroup = tile parity
  const int r = threadIdx.x & 127;             // row within this CTA = TMEM lane
  const int wq = (threadIdx.x >> 5) & 3;       // warp quarter: TMEM lanes 32*wq ..
  const int lane = threadIdx.x & 31;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  uint8_t* q_tile = smem + kPOffQ;
  float2* ml = reinterpret_cast<float2*>(smem + kPOffMl);
  const int R = a.group * a.n;
  const float sl2 = a.scale_log2;
  const int pairs = gridDim.x / 2;
  uint32_t i = 0, seg = 0;
  for (int u = blockIdx.x / 2; u < t.units; u += pairs, ++seg) {
    const UnitInfo ui = unit_info(t, u);
    const int row0 = ui.qg * kPRows + static_cast<int>(rank) * kBM;  // packed row of TMEM lane 0
    const int pr = row0 + r;
    const bool row_ok = pr < R;
    const int node = row_ok ? pr % a.n : 0;
    const int L = a.kv_len;
    const int P = L - a.n;
    const bool len_ok = L >= a.n;

    // ---- Q rows -> shared memory (SW128 K-major): warp (j, wq) fills rows
    // 32 wq + 16 j .. + 15, a half-warp per 256-byte row, all 8 row loads of a
    // half-warp in flight at once.  The unit_done wait of the previous unit
    // (below) guarantees both warpgroups are done with the staging rows.
    {
      const int sub = lane >> 4, jc = lane & 15;
      const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(a.q) + static_cast<int64_t>(ui.b) * a.q_sb +
                                static_cast<int64_t>(ui.kvh) * a.group * a.q_sh;
      uint4 qv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int rr = wq * 32 + j * 16 + sub + 2 * k;
        const int prr = row0 + rr;
        if (prr < R) {
          const int gq = prr / a.n, nd = prr - (prr / a.n) * a.n;
          qv[k] = __ldg(reinterpret_cast<const uint4*>(qb + static_cast<int64_t>(gq) * a.q_sh +
                                                       static_cast<int64_t>(nd) * a.q_sn) + jc);
        } else {
          qv[k] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<uint4*>(stage_at(q_tile, wq, j * 16 + sub + 2 * k, jc)) = qv[k];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) arrive_even(&bars->q_full, rank);
    }
    // ---- ancestor bits of this row's node (the walk of fused_tree_verify_triton.py:52-63)
    uint32_t anc[ANCW];
#pragma unroll
    for (int k = 0; k < ANCW; ++k) anc[k] = 0;
    if (a.mask_kind == GORGON_MASK_PARENTS) {
      const int32_t* par = a.parents + static_cast<int64_t>(ui.b) * a.par_sb;
      int pv[ANCW];
#pragma unroll
      for (int k = 0; k < ANCW; ++k) {
        const int idx = lane + 32 * k;
        pv[k] = (len_ok && idx < a.n) ? __ldg(par + idx) : -1;
      }
      int cur = (row_ok && len_ok) ? node : -1;
      bool bad = false;
      for (int hop = -1; hop < a.max_depth; ++hop) {
        if (!__any_sync(0xffffffffu, cur >= 0)) break;
        if (cur >= a.n) {
          bad = true;
          cur = -1;
        }
#pragma unroll
        for (int k = 0; k < ANCW; ++k)
          if (cur >= 0 && (cur >> 5) == k) anc[k] |= 1u << (cur & 31);
        int nxt = -1;
#pragma unroll
        for (int k = 0; k < ANCW; ++k) {
          const int v = __shfl_sync(0xffffffffu, pv[k], cur & 31);
          if ((cur >> 5) == k) nxt = v;
        }
        cur = cur >= 0 ? nxt : -1;
      }
      if (bad && j == 0) raise_device_error(a.err, kErrBadParent);
    } else if (row_ok && len_ok) {
      const uint8_t* mrow = a.mask + static_cast<int64_t>(ui.b) * a.mask_sb + static_cast<int64_t>(node) * a.mask_sn;
      for (int c = 0; c < a.n; ++c)
        if (mrow[c]) {
#pragma unroll
          for (int k = 0; k < ANCW; ++k)
            if ((c >> 5) == k) anc[k] |= 1u << (c & 31);
        }
    }
    if (!len_ok && r == 0 && j == 0 && rank == 0) raise_device_error(a.err, kErrBadSeqlen);

    float m_used = -INFINITY, l = 0.f;
    const uint32_t i0 = i;
    const uint32_t my_first = i0 + ((i0 & 1u) == static_cast<uint32_t>(j) ? 0u : 1u);  // this parity's first tile
    const uint32_t s_addr = lane_base + kPColS + j * 128;
    const int plain_end = len_ok ? P / kPBN : 0;  // tiles whose 128 keys all precede the tree
    // One tile of this warpgroup's parity: S -> P against the lazy running max
    // (moved only when a tile exceeds it by more than 8, log2 units).  Scores
    // come out of TMEM twice: 32 columns at a time for the row max, then 64
    // at a time for the exponentials, the second half first (its P goes over
    // its own columns 64-95), then the first (P over columns 0-31).
    auto tile = [&](int tix, bool masked) -> bool {
      uint32_t vw[4] = {~0u, ~0u, ~0u, ~0u};
      if (masked) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint64_t w = len_ok ? vis_window<ANCW>(anc, tix * kPBN + 64 * hh - P) : 0ull;
          vw[2 * hh] = static_cast<uint32_t>(w);
          vw[2 * hh + 1] = static_cast<uint32_t>(w >> 32);
        }
      }
      if (!pair_warp_wait(t, bars, &bars->s_full[j], (i >> 1) & 1u, peer)) return false;
      tc_fence_after();
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      // max pass, 32 columns at a time
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t rr[32];
        tmem_ld32(s_addr + 32 * q4, rr);
        tmem_wait_ld();
        const uint32_t vb = vw[q4];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float s0 = (!masked || ((vb >> c) & 1u)) ? __uint_as_float(rr[c]) : -INFINITY;
          const float s1 = (!masked || ((vb >> (c + 1)) & 1u)) ? __uint_as_float(rr[c + 1]) : -INFINITY;
          mx[(c >> 1) & 3] = fmax3(mx[(c >> 1) & 3], s0, s1);
        }
      }
      const float tmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * sl2;
      float alpha = 1.f;
      bool need = false;
      if (i == my_first) {
        m_used = tmax;
      } else if (tmax > m_used + 8.f) {
        alpha = ex2_approx(m_used - tmax);  // 0 while nothing was visible yet
        m_used = tmax;
        need = true;
      }
      const float nmb = m_used == -INFINITY ? 0.f : -m_used;
      const uint64_t sl2_2 = f2_pack(sl2, sl2), nmb_2 = f2_pack(nmb, nmb);
      uint64_t acc2[2] = {0, 0};
      // exponentials 32 columns at a time: keys 64-127 first (P over their
      // own columns 64-95), then keys 0-63 (P over columns 0-31)
#pragma unroll
      for (int q4i = 0; q4i < 4; ++q4i) {
        const int q4 = (q4i + 2) & 3;
        uint32_t rr[32];
        tmem_ld32(s_addr + 32 * q4, rr);
        tmem_wait_ld();
        const uint32_t vb = vw[q4];
        uint32_t packed[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float s0 = (!masked || ((vb >> c) & 1u)) ? __uint_as_float(rr[c]) : -INFINITY;
          const float s1 = (!masked || ((vb >> (c + 1)) & 1u)) ? __uint_as_float(rr[c + 1]) : -INFINITY;
          float a0, a1;
          f2_unpack(f2_fma(f2_pack(s0, s1), sl2_2, nmb_2), a0, a1);
          const float p0 = ex2_approx(a0);
          const float p1 = ex2_approx(a1);
          acc2[(c >> 1) & 1] = f2_add(acc2[(c >> 1) & 1], f2_pack(p0, p1));
          packed[c >> 1] = pack16x2(p0, p1, BF16);
        }
        tmem_st16(s_addr + (q4 < 2 ? 16 * q4 : 64 + 16 * (q4 - 2)), packed);
      }
      {
        const uint64_t s2 = f2_add(acc2[0], acc2[1]);
        float s0, s1;
        f2_unpack(s2, s0, s1);
        l = l * alpha + (s0 + s1);
      }
      // rescale O_j (warp-uniform) once the P.V of this parity's previous tile has landed
      if (__any_sync(0xffffffffu, need)) {
        if (!pair_warp_wait(t, bars, &bars->p_free[j], ((i - 2) >> 1) & 1u, peer)) return false;
        tc_fence_after();
        const uint32_t o_addr = lane_base + kPColO + j * 128;
#pragma unroll 1
        for (int ch = 0; ch < kD / 32; ++ch) {
          uint32_t ov[32];
          tmem_ld32(o_addr + ch * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
          tmem_st32(o_addr + ch * 32, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_even(&bars->p_full[j], rank);
      return true;
    };
    bool ok = true;
    for (int tix = 0; tix < t.tiles; ++tix, ++i) {
      if ((i & 1u) != static_cast<uint32_t>(j)) continue;
      if (!tile(tix, tix >= plain_end)) {
        ok = false;
        break;
      }
    }
    if (!ok) return;

    // ---- epilogue: merge O_0 and O_1 of every row, once both parities' last
    // P.V has landed.  A parity with no tile in this unit contributes nothing.
    const uint32_t n_tiles = static_cast<uint32_t>(t.tiles);
    bool has[2];
    uint32_t last[2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const uint32_t first = i0 + ((i0 & 1u) == static_cast<uint32_t>(jj) ? 0u : 1u);
      has[jj] = first < i0 + n_tiles;
      last[jj] = has[jj] ? first + ((i0 + n_tiles - 1 - first) & ~1u) : 0u;
      if (has[jj] && !pair_warp_wait(t, bars, &bars->p_free[jj], (last[jj] >> 1) & 1u, peer)) return;
    }
    tc_fence_after();
    ml[j * 128 + r] = make_float2(m_used, l);
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->ml_ready);
    if (!pair_warp_wait(t, bars, &bars->ml_ready, seg & 1u, peer)) return;
    const float2 other = ml[(j ^ 1) * 128 + r];
    const float m_of[2] = {j == 0 ? m_used : other.x, j == 0 ? other.x : m_used};
    const float l_of[2] = {j == 0 ? l : other.y, j == 0 ? other.y : l};
    const float M = fmaxf(m_of[0], m_of[1]);
    float w[2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) w[jj] = (has[jj] && l_of[jj] > 0.f) ? ex2_approx(m_of[jj] - M) : 0.f;
    const float den = l_of[0] * w[0] + l_of[1] * w[1];
    const float inv = 1.f / den;  // no visible key: 0 * inf = NaN, as softmax gives
    // this warpgroup's 64 output columns, 16-bit, into its half of the staging rows
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const uint32_t col = static_cast<uint32_t>(64 * j + 32 * ch);
      uint32_t o0[32], o1[32];
      tmem_ld32(lane_base + kPColO + col, o0);
      tmem_ld32(lane_base + kPColO + 128 + col, o1);
      tmem_wait_ld();
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        uint32_t wd[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v2[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            const int c = 8 * u4 + 2 * e + z;
            const float a0 = w[0] > 0.f ? __uint_as_float(o0[c]) * w[0] : 0.f;
            const float a1 = w[1] > 0.f ? __uint_as_float(o1[c]) * w[1] : 0.f;
            v2[z] = (a0 + a1) * inv;
          }
          wd[e] = pack16x2(v2[0], v2[1], t.out_bf16 != 0);
        }
        *reinterpret_cast<uint4*>(stage_at(q_tile, wq, lane, 8 * j + 4 * ch + u4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
    }
    if (a.lse && row_ok && j == 0) {
      const int gq = pr / a.n;
      const int64_t orow = (static_cast<int64_t>(ui.b) * a.hq + ui.kvh * a.group + gq) * a.n + node;
      a.lse[orow] = den > 0.f ? (M + __log2f(den)) * 0.6931471805599453f : -INFINITY;
    }
    __syncwarp();
    // the warp's 32 rows, this warpgroup's 128-byte half of each: 8 lanes per row
    {
      const int sub = lane >> 3, ch = lane & 7;
      uint16_t* ob = static_cast<uint16_t*>(a.out) + static_cast<int64_t>(ui.b) * a.o_sb +
                     static_cast<int64_t>(ui.kvh) * a.group * a.o_sh + 64 * j + ch * 8;
#pragma unroll 4
      for (int k = 0; k < 8; ++k) {
        const int rr = 4 * k + sub;
        const int prr = row0 + wq * 32 + rr;
        const uint4 v = *reinterpret_cast<const uint4*>(stage_at(q_tile, wq, rr, 8 * j + ch));
        if (prr < R) {
          const int gq = prr / a.n, nd = prr - (prr / a.n) * a.n;
          *reinterpret_cast<uint4*>(ob + static_cast<int64_t>(gq) * a.o_sh + static_cast<int64_t>(nd) * a.o_sn) = v;
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->unit_done);
    if (!pair_warp_wait(t, bars, &bars->unit_done, seg & 1u, peer)) return;
    tc_fence_after();
  }
}

template <int ANCW, bool BF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
attn_pair_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                 const __grid_constant__ PairArgs t) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + kPOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->q_full, 16);  // 8 softmax warps in each CTA
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 8);  // warpgroup b of both CTAs
      mbar_init(&bars->p_free[b], 1);
    }
    mbar_init(&bars->ml_ready, 8);
    mbar_init(&bars->unit_done, 8);
    mbar_init(&bars->drain[0], 1);
    mbar_init(&bars->drain[1], 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0 && rank == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  // both CTAs' barriers exist before either CTA touches the other's
  cluster_sync();
  if (warp == 2) {
    tmem_alloc_pair(&bars->tmem_base, kPTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp >= 4) {
    pair_softmax<ANCW, BF16>(t, smem, bars, tmem, rank);
  } else if (rank == 0 && lane == 0) {
    if (warp == 0) pair_producer(t, &kmap, smem, bars, 0);
    else if (warp == 3) pair_producer(t, &vmap, smem, bars, 1);
    else if (warp == 1) pair_qk_issuer(t, smem, bars, tmem);
    else pair_pv_issuer(t, smem, bars, tmem);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // the even CTA's loads into this CTA and MMAs on its TMEM are complete
  cluster_sync();
  if (bars->abort && threadIdx.x == 0) raise_device_error(t.a.err, kErrTimeout);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kPTmemCols);
  }
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn pair_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

template <int ANCW, bool BF16>
const void* pair_kernel_ptr() {
  return reinterpret_cast<const void*>(attn_pair_kernel<ANCW, BF16>);
}

const void* pick_pair_kernel(const AttnArgs& a, int dtype) {
  const bool bf = dtype == GORGON_BF16;
  if (a.n <= 64) return bf ? pair_kernel_ptr<2, true>() : pair_kernel_ptr<2, false>();
  return bf ? pair_kernel_ptr<8, true>() : pair_kernel_ptr<8, false>();
}

// Shared-memory limit raised once per (kernel, device); the number of CTA
// pairs that fit on the device at once, cached likewise.
int pair_setup(const void* fn, int* max_pairs) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<const void*, int>, int>> done;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "tcgen05 pair: current device");
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : done)
    if (e.first.first == fn && e.first.second == dev) {
      *max_pairs = e.second;
      return GORGON_OK;
    }
  rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kPSmem)),
                  "tcgen05 pair: smem attribute");
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 148);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmem;
  int n = 0;  // the kernel's compile-time cluster shape (2 x 1 x 1) applies
  rc = check_cuda(cudaOccupancyMaxActiveClusters(&n, fn, &cfg), "tcgen05 pair: cluster occupancy");
  if (rc) return rc;
  if (n < 1) return set_error(GORGON_ERR_UNSUPPORTED, "tcgen05 pair: no CTA pair fits on this device");
  done.push_back({{fn, dev}, n});
  *max_pairs = n;
  return GORGON_OK;
}

bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool attn_pair_supported(const AttnArgs& a, int dtype) {
  if (dtype != GORGON_BF16 && dtype != GORGON_F16) return false;
  if (a.d != kD || a.n < 1 || a.n > 256 || a.cu_seqlens) return false;
  if (a.mask_kind != GORGON_MASK_PARENTS && a.mask_kind != GORGON_MASK_DENSE_TREE) return false;
  if (!a.vec_ok || !aligned16p(a.q) || !aligned16p(a.k) || !aligned16p(a.v)) return false;
  // 16-bit output rows of whole 16-byte chunks
  if (a.out_dtype != dtype || !aligned16p(a.out) || a.o_sb % 8 || a.o_sh % 8 || a.o_sn % 8) return false;
  return pair_encode_fn() != nullptr;
}

int attn_pair_plan(const AttnArgs& a, int dtype, int* pairs, int* units) {
  int max_pairs = 0;
  const int rc = pair_setup(pick_pair_kernel(a, dtype), &max_pairs);
  if (rc) return rc;
  const int qgroups = (a.group * a.n + kPRows - 1) / kPRows;
  const int64_t u = static_cast<int64_t>(a.batch) * a.hkv * qgroups;
  const int64_t waves = (u + max_pairs - 1) / max_pairs;
  *units = static_cast<int>(u);
  *pairs = static_cast<int>(std::max<int64_t>(1, (u + waves - 1) / std::max<int64_t>(waves, 1)));
  return GORGON_OK;
}

int launch_attn_pair(const AttnArgs& a, int dtype, cudaStream_t st) {
  int pairs = 0, units = 0;
  int rc = attn_pair_plan(a, dtype, &pairs, &units);
  if (rc) return rc;
  EncodeTiledFn enc = pair_encode_fn();
  if (!enc) return set_error(GORGON_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType tdt = dtype == GORGON_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap kmap, vmap;
  const void* srcs[2] = {a.k, a.v};
  const int64_t ss[2] = {a.k_ss, a.v_ss}, sh[2] = {a.k_sh, a.v_sh}, sb[2] = {a.k_sb, a.v_sb};
  const cuuint32_t rows[2] = {64, 128};  // K boxes: 64 keys; V boxes: 128 keys
  CUtensorMap* maps[2] = {&kmap, &vmap};
  for (int m = 0; m < 2; ++m) {
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.kv_len),
                                static_cast<cuuint64_t>(a.hkv), static_cast<cuuint64_t>(a.batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss[m]) * 2, static_cast<cuuint64_t>(sh[m]) * 2,
                                   static_cast<cuuint64_t>(sb[m]) * 2};
    const cuuint32_t box[4] = {64, rows[m], 1, 1};
    const CUresult r = enc(maps[m], tdt, 4, const_cast<void*>(srcs[m]), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return set_error(GORGON_ERR_INVALID, "tcgen05 pair: cuTensorMapEncodeTiled rejected the K/V layout "
                                           "(strides must be multiples of 16 bytes)");
  }
  PairArgs t{};
  t.a = a;
  t.qgroups = (a.group * a.n + kPRows - 1) / kPRows;
  t.units = units;
  t.tiles = (a.kv_len + kPBN - 1) / kPBN;
  t.ab_fmt = dtype == GORGON_BF16 ? 1 : 0;
  t.out_bf16 = a.out_dtype == GORGON_BF16 ? 1 : 0;
  t.wait_ns = wait_limit_ns();
  const bool bf = dtype == GORGON_BF16;
  auto kern = a.n <= 64 ? (bf ? attn_pair_kernel<2, true> : attn_pair_kernel<2, false>)
                        : (bf ? attn_pair_kernel<8, true> : attn_pair_kernel<8, false>);
  kern<<<2 * pairs, kPThreads, kPSmem, st>>>(kmap, vmap, t);
  return check_cuda(cudaGetLastError(), "tcgen05 pair tree attention launch");
}

}  // namespace gorgon
