// Tensor-core (tcgen05) tree attention for sm_100a.
//
// Unit of work: MT 128-row M-tiles of one (sequence b, kv head) — a "unit".
// The packed query rows of a (b, kv head) are (query head in the GQA group,
// tree node): row g * n + i; a unit takes MT * 128 consecutive packed rows.
// Those rows share every key/value row of the sequence, so each K/V tile a
// CTA fetches feeds all MT of its MMA tiles.  Two shapes, chosen per launch:
//
//   MT = 2: 256 rows per unit, 64-row K/V tiles, 384 threads (two softmax
//           warpgroups), 5-stage K and V rings.
//   MT = 1: 128 rows per unit, 128-row K/V tiles, 256 threads (one softmax
//           warpgroup), 3-stage rings.  Q.K^T runs at N = 128 (the tensor
//           pipe's full rate; N = 64 takes ~57 cycles per K step for 32 of
//           math), the softmax thread keeps a 128-column row in registers
//           (255 per thread at 256 threads), and the two units of a 256-row
//           group run on neighbouring CTAs that share K/V through L2.
//
// Schedule: a grid of at most one CTA per SM.  When whole units roughly fill
// the SMs, CTA c takes units c, c + grid, ... (so the units that share K/V run
// at the same time).  With room for two or more CTAs per unit (uniform
// lengths), each unit is cut into equal tile ranges over the CTAs of one
// thread-block cluster: every piece leaves its normalised rows and
// log-sum-exp in the workspace, and after a cluster barrier each CTA merges
// a slice of the unit's rows from L2 (one launch, no merge kernel).  Otherwise (stream-K)
// the unit-major list of K/V tiles is split into equal contiguous ranges: a
// unit that falls inside one CTA is finished there; a unit cut between CTAs
// leaves normalised partials plus log-sum-exp in the workspace, and
// attn_tc_combine, launched right after, merges them with one warp per row.
//
// Warp roles:
//   warp 0       TMA producer for K tiles (two 64-column SW128 boxes)
//   warp 3       TMA producer for V tiles, its own ring
//   warp 1       Q.K^T issuer (one thread): S = Q K^T into TMEM
//   warp 2       P.V issuer (one thread): O += P V with P read from TMEM; the
//                warp also allocates and releases TMEM
//   warps 4-7    softmax + epilogue of M-tile 0 (TMEM lanes 0-127)
//   warps 8-11   (MT = 2) softmax + epilogue of M-tile 1
// TMEM (512 columns): S double-buffered (2 buffers x MT M-tiles x BN
// columns, 256 in all) and O (MT x 128 columns).  P (16-bit pairs)
// overwrites the first BN / 2 columns of its own S buffer and is the TMEM A
// operand of P.V.  A K stage is released as soon as its Q.K^T completes, a V
// stage after P.V.
//
// Softmax per row is owned by one thread (TMEM lane = row), so row max and
// sum need no shuffles.  Rescaling of O is lazy: the running max only moves
// when a tile's max exceeds it by more than 8 (log2 units), which bounds P by
// 2^8 and makes O corrections rare.  Every mbarrier wait is bounded; on
// timeout the CTA raises kErrTimeout, drains its copies and MMAs, frees TMEM
// and returns.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <utility>
#include <vector>

#include "attn.cuh"
#include "sm100.cuh"
#include "attn_tc_common.cuh"

namespace gorgon {
namespace {
using namespace sm100;

constexpr uint32_t kOffQ = 0;                          // [mtile][half]
constexpr int kMaxPeers = 8;                           // GORGON_MAX_PEERS
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // + (buf * MT + mtile) * BN
constexpr uint32_t kColO = 256;  // + mtile * 128

// The constants that follow from MT, the 128-row M-tiles per CTA.
template <int MT>
struct Cfg {
  static_assert(MT == 1 || MT == 2, "one or two M-tiles per CTA");
  static constexpr int kQRows = MT * kBM;          // packed query rows per unit
  static constexpr int kBN = MT == 2 ? 64 : 128;   // key/value rows per tile
  static constexpr int kStages = MT == 2 ? 5 : 3;  // per ring (K and V)
  static constexpr int kThreads = 128 + MT * 128;
  static constexpr uint32_t kKVHalf = kBN * 128;   // BN rows x 64 cols bf16
  static constexpr uint32_t kTileBytes = 2 * kKVHalf;
  static constexpr uint32_t kOffK = kOffQ + MT * 2 * kQHalf;  // [stage][half]
  static constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
  static constexpr uint32_t kOffBar = kOffV + kStages * kTileBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;  // + alignment slack
  // Who frees a K stage: with two M-tiles (a 5-stage ring) each softmax
  // warpgroup arrives once it has seen its S, which takes a barrier
  // operation off the Q.K^T issuer, the busiest thread; with one M-tile
  // (a 3-stage ring) the issuer commits the release as soon as its MMAs
  // complete, so the shorter ring refills sooner.
  static constexpr bool kSoftmaxFreesK = MT == 2;
  static_assert(kSmemBytes <= 232448, "shared memory per block");
  static_assert(2 * MT * kBN <= kColO, "S buffers below O");
};

struct TcArgs {
  AttnArgs a;
  int varlen;
  int qgroups;        // units per (b, kv head)
  int pairs;          // units: batch * hkv * qgroups
  int tiles_per_pair; // tiles per unit (uniform lengths only)
  int grid;
  int pair_align;     // whole units per CTA, strided by the grid (no partials to merge)
  int cluster;        // > 1: each unit cut between the CTAs of a cluster of this size, merged in DSMEM
  int q_tma;          // Q M-tiles come by TMA (tree size divides 128 or is a multiple of it)
  // Output gather over NVLink (gorgon_tree_attn_gather): every output chunk
  // is also stored at peer_out[p] + (its offset from a.out), for npeers
  // other ranks; sig / peer_sig are the ranks' signal words
  // {arrived, done, calls completed, done expected}.
  int npeers;
  void* peer_out[kMaxPeers - 1];
  uint64_t* peer_sig[kMaxPeers - 1];
  uint64_t* sig;
  int ab_fmt;         // 0 f16, 1 bf16
  int out_vec;        // 16-byte aligned output rows: kOutBf16 / kOutF16 / kOutF32, else 0
  float* part_o;      // [grid * 2][rows per unit][128]
  float* part_lse;    // [grid * 2][rows per unit]
  int* tile_start;    // varlen: [units + 1] tile prefix (written by attn_tc_prologue)
  int* order;         // varlen whole units: unit ids, most tiles first (attn_tc_prologue_sorted); else null
  uint64_t wait_ns;   // bound on every wait (wait_limit_ns())
};

template <int MT>
struct Barriers {
  uint64_t k_full[Cfg<MT>::kStages];
  uint64_t k_empty[Cfg<MT>::kStages];
  uint64_t v_full[Cfg<MT>::kStages];
  uint64_t v_empty[Cfg<MT>::kStages];
  uint64_t q_full;
  uint64_t q_empty;         // (Q by TMA) the softmax warps are done with the Q tile as output staging
  // per (S buffer, M-tile): index buf * MT + mtile
  uint64_t s_full[2 * MT];
  uint64_t p_full[2 * MT];
  uint64_t p_free[2];       // P.V of every M-tile of the tile in this buffer has completed
  uint64_t drain[2];        // all MMAs of the Q.K^T / P.V issuer complete
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Barriers<2>) <= 512 && sizeof(Barriers<1>) <= 512, "barrier block");

// ------------------------------------------------------------ schedule
__device__ __forceinline__ int64_t total_tiles(const TcArgs& t) {
  return t.varlen ? static_cast<int64_t>(t.tile_start[t.pairs])
                  : static_cast<int64_t>(t.pairs) * t.tiles_per_pair;
}
__device__ __forceinline__ int64_t pair_start(const TcArgs& t, int p) {
  return t.varlen ? static_cast<int64_t>(t.tile_start[p]) : static_cast<int64_t>(p) * t.tiles_per_pair;
}
__device__ __forceinline__ int pair_of(const TcArgs& t, int64_t g) {
  if (!t.varlen) return static_cast<int>(g / t.tiles_per_pair);
  int lo = 0, hi = t.pairs - 1;  // largest p with start(p) <= g
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t.tile_start[mid] <= g) lo = mid; else hi = mid - 1;
  }
  return lo;
}
__device__ __forceinline__ int64_t range_start(int64_t c, int64_t T, int64_t G) { return c * T / G; }
__device__ __forceinline__ int64_t cta_of(int64_t g, int64_t T, int64_t G) {
  return ((g + 1) * G + T - 1) / T - 1;
}

struct PairInfo {
  int b, kvh, qg;
  int L;          // kv rows of the sequence
  int row0;       // first kv row (varlen: cu_seqlens[b]; else 0)
  int64_t start;  // first global tile
  int64_t end;    // one past the last global tile
};

__device__ __forceinline__ PairInfo pair_info(const TcArgs& t, int p) {
  PairInfo pi;
  pi.qg = p % t.qgroups;
  pi.kvh = (p / t.qgroups) % t.a.hkv;
  pi.b = p / (t.qgroups * t.a.hkv);
  if (t.a.cu_seqlens) {
    pi.row0 = t.a.cu_seqlens[pi.b];
    pi.L = t.a.cu_seqlens[pi.b + 1] - pi.row0;
  } else {
    pi.row0 = 0;
    pi.L = t.a.kv_len;
  }
  pi.start = pair_start(t, p);
  pi.end = t.varlen ? static_cast<int64_t>(t.tile_start[p + 1]) : pi.start + t.tiles_per_pair;
  return pi;
}

// The segments (the tiles of one unit each) a CTA works through, the same
// sequence for every role: whole units blockIdx.x, blockIdx.x + grid, ...
// when t.pair_align, else the pieces of units inside the CTA's tile range
// [g0, g1) (stream-K).
struct Segments {
  int64_t g0, g1;
  int unit, round = 0;
  __device__ Segments(int64_t r0, int64_t r1) : g0(r0), g1(r1), unit(blockIdx.x) {}
  __device__ bool next(const TcArgs& t, int64_t& g, int64_t& e, PairInfo& pi) {
    if (t.pair_align) {
      while (true) {
        int u;
        if (t.order) {
          // units sorted by tile count, dealt out in snake order: CTA c takes
          // sorted unit c in round 0, grid - 1 - c in round 1, and so on
          const int i = round * t.grid + ((round & 1) ? t.grid - 1 - static_cast<int>(blockIdx.x)
                                                      : static_cast<int>(blockIdx.x));
          if (i >= t.pairs) return false;
          u = t.order[i];
          ++round;
        } else {
          if (unit >= t.pairs) return false;
          u = unit;
          unit += t.grid;
        }
        pi = pair_info(t, u);
        if (pi.end > pi.start) {
          g = pi.start;
          e = pi.end;
          return true;
        }
      }
    }
    if (g0 >= g1) return false;
    pi = pair_info(t, pair_of(t, g0));
    g = g0;
    e = min(g1, pi.end);
    g0 = e;
    return true;
  }
};

// ------------------------------------------------------------ output gather
// True once every peer's stream has reached this call (each adds 1 to our
// `arrived` word when its kernel starts, after the earlier work on its
// stream), so their buffers are free for this call's rows; false, with the
// timeout bit raised, if that wait runs out.
__device__ bool peers_ready(const TcArgs& t) {
  const uint64_t calls = *reinterpret_cast<volatile const uint64_t*>(t.sig + 2);
  const uint64_t need = (calls + 1) * static_cast<uint64_t>(t.npeers);
  if (ld_acquire_sys(t.sig) >= need) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(t.sig) < need) {
    if (globaltimer_ns() - t0 > t.wait_ns) {
      raise_device_error(t.a.err, kErrTimeout);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}
// The warp's answer (lane 0 waits); the warp barrier orders the lanes'
// stores to the peers after lane 0's acquire.
__device__ __forceinline__ bool warp_peers_ready(const TcArgs& t) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = peers_ready(t) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ------------------------------------------------------------ roles
// Streams one operand (K when is_v == 0, else V) of every tile of the CTA's
// segments through its ring.
// The Q rows of one unit (MT M-tiles, two 64-column SW128 boxes each) by
// TMA: a box of 128 / n heads x n nodes (or 128 of the nodes) is 128
// consecutive packed rows.  Rows past the unit's real rows read the next
// heads' rows (or zeros past the last head); nothing reads their results.
template <int MT>
__device__ __forceinline__ void load_q_tma(const TcArgs& t, const CUtensorMap* qmap, uint8_t* smem,
                                           Barriers<MT>* bars, const PairInfo& pi) {
  const AttnArgs& a = t.a;
  mbar_arrive_expect_tx(&bars->q_full, MT * 2 * kQHalf);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int pr0 = pi.qg * Cfg<MT>::kQRows + mt * kBM;
    const int gq = pr0 / a.n, node = pr0 - gq * a.n;
    const int head = pi.kvh * a.group + gq;
    uint8_t* dst = smem + kOffQ + mt * 2 * kQHalf;
    tma_load_4d_hint(dst, qmap, &bars->q_full, 0, node, head, pi.b, l2_policy_evict_first());
    tma_load_4d_hint(dst + kQHalf, qmap, &bars->q_full, 64, node, head, pi.b, l2_policy_evict_first());
  }
}

template <int MT>
__device__ void producer(const TcArgs& t, const CUtensorMap* map, const CUtensorMap* qmap, uint8_t* smem,
                         Barriers<MT>* bars, int64_t g0, int64_t g1, int is_v) {
  using C = Cfg<MT>;
  volatile int* abort = &bars->abort;
  uint64_t* full = is_v ? bars->v_full : bars->k_full;
  uint64_t* empty = is_v ? bars->v_empty : bars->k_empty;
  uint8_t* ring = smem + (is_v ? C::kOffV : C::kOffK);
  int64_t issued = 0;
  // With one unit per (sequence, kv head) K/V are read once: keep them from
  // pushing the partial results out of L2.  With several, the units' CTAs run
  // side by side over the same K/V, and the later ones should find it in L2.
  const uint64_t policy = t.qgroups > 1 ? l2_policy_evict_last() : l2_policy_evict_first();
  Segments sg(g0, g1);
  int64_t g, e;
  PairInfo pi;
  bool ok = true;
  uint32_t q_loads = 0;  // Q tiles issued by TMA (K producer only)
  while (ok && sg.next(t, g, e, pi)) {
    if (t.q_tma && !is_v) {
      // the previous unit's epilogue has finished with the Q tile
      if (q_loads > 0 && !bounded_wait(&bars->q_empty, (q_loads - 1) & 1u, abort, t.wait_ns)) break;
      load_q_tma<MT>(t, qmap, smem, bars, pi);
      ++q_loads;
    }
    for (; g < e; ++g) {
      const int tile = static_cast<int>(g - pi.start);
      const int stage = static_cast<int>(issued % C::kStages);
      const uint32_t ph = static_cast<uint32_t>(issued / C::kStages) & 1u;
      if (!bounded_wait(&empty[stage], ph ^ 1u, abort, t.wait_ns)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[stage], C::kTileBytes);
      uint8_t* st = ring + stage * C::kTileBytes;
      const int row = tile * C::kBN;
      if (t.varlen) {
        const int r = pi.row0 + row;
        tma_load_3d_hint(st, map, &full[stage], 0, pi.kvh, r, policy);
        tma_load_3d_hint(st + C::kKVHalf, map, &full[stage], 64, pi.kvh, r, policy);
      } else {
        tma_load_4d_hint(st, map, &full[stage], 0, row, pi.kvh, pi.b, policy);
        tma_load_4d_hint(st + C::kKVHalf, map, &full[stage], 64, row, pi.kvh, pi.b, policy);
      }
      ++issued;
    }
  }
  // Every issued load must land before the CTA leaves.
  for (int64_t k = (issued > C::kStages ? issued - C::kStages : 0); k < issued; ++k)
    drain_wait(&full[k % C::kStages], static_cast<uint32_t>(k / C::kStages) & 1u);
  if (q_loads > 0) drain_wait(&bars->q_full, (q_loads - 1) & 1u);
}

// Ring position of a tile counter, advanced without divisions.
template <int N>
struct Ring {
  uint32_t stage = 0, phase = 0;
  __device__ __forceinline__ void next() {
    if (++stage == N) {
      stage = 0;
      phase ^= 1u;
    }
  }
};

// The MMA issuers keep every operand descriptor in registers and only add
// constant offsets (in the descriptor's 16-byte address units) per K step.
struct MmaDescs {
  uint64_t q0;  // Q M-tile 0, d half 0 ([mtile][half] at 16 KB steps), SW128 K-major, SBO 1 KB
  uint64_t k0;  // K ring stage 0, half 0
  uint64_t v0;  // V ring stage 0: MN-major, LBO = one d half of a tile, SBO 1 KB
  uint32_t idesc_qk, idesc_pv;
};

// S_mt = Q_mt K^T of one tile into S buffer `buf` (M 128, N BN, K 128).
template <int MT>
__device__ __forceinline__ void issue_qk(const MmaDescs& md, uint32_t tmem, uint32_t stage, uint32_t buf, int mt) {
  using C = Cfg<MT>;
  const uint64_t kst = md.k0 + static_cast<uint64_t>(stage * (C::kTileBytes >> 4));
  const uint32_t d_tmem = tmem + kColS + (buf * MT + mt) * C::kBN;
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    const uint64_t a = md.q0 + static_cast<uint64_t>((mt * 2 + (ks >> 2)) * (kQHalf >> 4) + (ks & 3) * 2);
    const uint64_t b = kst + static_cast<uint64_t>((ks >> 2) * (C::kKVHalf >> 4) + (ks & 3) * 2);
    umma_f16_ss(d_tmem, a, b, md.idesc_qk, ks > 0 ? 1u : 0u);
  }
}

// O_mt += P_mt (TMEM, over S buffer `buf`) * V (smem stage): M 128, N 128, K BN.
template <int MT>
__device__ __forceinline__ void issue_pv(const MmaDescs& md, uint32_t tmem, uint32_t stage, uint32_t buf, int mt,
                                         uint32_t first) {
  using C = Cfg<MT>;
  const uint64_t vst = md.v0 + static_cast<uint64_t>(stage * (C::kTileBytes >> 4));
  const uint32_t d_tmem = tmem + kColO + mt * kD;
  const uint32_t p_tmem = tmem + kColS + (buf * MT + mt) * C::kBN;
#pragma unroll
  for (int ks = 0; ks < C::kBN / 16; ++ks) {
    umma_f16_ts(d_tmem, p_tmem + ks * 8, vst + static_cast<uint64_t>(ks * (2048 >> 4)), md.idesc_pv,
                (ks > 0 || !first) ? 1u : 0u);
  }
}

template <int MT>
__device__ __forceinline__ void make_descs(const TcArgs& t, uint8_t* smem, MmaDescs& md) {
  using C = Cfg<MT>;
  md.q0 = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
  md.k0 = umma_desc_sw128(smem_u32(smem + C::kOffK), 16, 1024);
  md.v0 = umma_desc_sw128(smem_u32(smem + C::kOffV), C::kKVHalf, 1024);
  md.idesc_qk = umma_idesc_f16(t.ab_fmt, kBM, C::kBN, 0, 0);
  md.idesc_pv = umma_idesc_f16(t.ab_fmt, kBM, kD, 0, 1);
}

// Two threads (in different warps) feed the tensor pipe: one issues every
// Q.K^T, the other every P.V, so neither group waits behind the other's
// bookkeeping.  S buffer i & 1 doubles as P's storage, so Q.K^T(i) waits for
// P.V(i - 2) to complete before overwriting it.  Both spin on their barriers
// (they have nothing else to do) to start the moment their inputs land.
template <int MT>
__device__ void qk_issuer(const TcArgs& t, uint8_t* smem, Barriers<MT>* bars, uint32_t tmem, int64_t g0,
                          int64_t g1) {
  volatile int* abort = &bars->abort;
  MmaDescs md;
  make_descs<MT>(t, smem, md);
  Ring<Cfg<MT>::kStages> kr;
  uint32_t i = 0, seg = 0;
  Segments sg(g0, g1);
  int64_t g, e;
  PairInfo pi;
  bool ok = true;
  while (ok && sg.next(t, g, e, pi)) {
    const uint32_t n_tiles = static_cast<uint32_t>(e - g);
    if (!spin_wait(&bars->q_full, seg & 1u, abort, t.wait_ns)) break;
    for (uint32_t j = 0; j < n_tiles; ++j, ++i) {
      // Both probes are issued before either result is used, so when the K
      // tile and the S buffer are already there (the usual case) the two
      // barrier round trips overlap; otherwise fall back to bounded spins.
      const uint32_t pf_par = ((i - 2) >> 1) & 1u;
      const bool k_ready = mbar_test_wait(&bars->k_full[kr.stage], kr.phase);
      const bool p_ready = i < 2 || mbar_test_wait(&bars->p_free[i & 1u], pf_par);
      if (!(k_ready && p_ready) &&
          (!spin_wait(&bars->k_full[kr.stage], kr.phase, abort, t.wait_ns) ||
           (i >= 2 && !spin_wait(&bars->p_free[i & 1u], pf_par, abort, t.wait_ns)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // per M-tile: each softmax warpgroup starts as soon as its own S lands
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        issue_qk<MT>(md, tmem, kr.stage, i & 1u, mt);
        umma_commit(&bars->s_full[(i & 1u) * MT + mt]);
      }
      if (!Cfg<MT>::kSoftmaxFreesK) umma_commit(&bars->k_empty[kr.stage]);
      kr.next();
    }
    ++seg;
  }
  umma_commit(&bars->drain[0]);
  drain_wait(&bars->drain[0], 0);
}

template <int MT>
__device__ void pv_issuer(const TcArgs& t, uint8_t* smem, Barriers<MT>* bars, uint32_t tmem, int64_t g0,
                          int64_t g1) {
  volatile int* abort = &bars->abort;
  MmaDescs md;
  make_descs<MT>(t, smem, md);
  Ring<Cfg<MT>::kStages> vr;
  uint32_t i = 0;
  Segments sg(g0, g1);
  int64_t g, e;
  PairInfo pi;
  bool ok = true;
  while (ok && sg.next(t, g, e, pi)) {
    const uint32_t n_tiles = static_cast<uint32_t>(e - g);
    for (uint32_t j = 0; j < n_tiles; ++j, ++i) {
      const uint32_t buf = i & 1u;
      if (!spin_wait(&bars->v_full[vr.stage], vr.phase, abort, t.wait_ns)) {
        ok = false;
        break;
      }
      for (int mt = 0; mt < MT && ok; ++mt) {
        const uint32_t bi = buf * MT + mt;
        if (!spin_wait(&bars->p_full[bi], (i >> 1) & 1u, abort, t.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv<MT>(md, tmem, vr.stage, buf, mt, j == 0);
      }
      if (!ok) break;
      umma_commit(&bars->p_free[buf]);
      umma_commit(&bars->v_empty[vr.stage]);
      vr.next();
    }
  }
  umma_commit(&bars->drain[1]);
  drain_wait(&bars->drain[1], 0);
}


template <int MT, int ANCW, bool BF16, bool QTMA>
__device__ void softmax_epilogue(const TcArgs& t, uint8_t* smem, Barriers<MT>* bars, uint32_t tmem, int64_t g0,
                                 int64_t g1, int cta) {
  using C = Cfg<MT>;
  constexpr int kBN = C::kBN;
  const AttnArgs& a = t.a;
  volatile int* abort = &bars->abort;
  const int wg = (threadIdx.x >> 7) - 1;       // M-tile: 0 .. MT - 1
  const int r = threadIdx.x & 127;              // row within the M-tile = TMEM lane
  const int wq = (threadIdx.x >> 5) & 3;        // warp quarter: TMEM lanes 32*wq..
  const int lane = threadIdx.x & 31;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  uint8_t* q_tile = smem + kOffQ + wg * 2 * kQHalf;
  const int R = a.group * a.n;
  const float sl2 = a.scale_log2;
  constexpr bool ab_bf16 = BF16;  // P's 16-bit type (that of Q, K and V)
  const int qrow = wg * kBM + r;                // row within the unit
  int64_t i = 0;
  // (Q by TMA) the warp hands the Q tile back to the producer once its
  // output staging in it is done: generic-proxy accesses before the TMA writes
  auto q_done = [&]() {
    if (QTMA) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->q_empty);
    }
  };
  Segments sg(g0, g1);
  int64_t g, e;
  PairInfo pi;
  while (sg.next(t, g, e, pi)) {
    const bool whole = !t.cluster && g == pi.start && e == pi.end;
    const int64_t i_first = i;
    const int pr = pi.qg * C::kQRows + qrow;  // packed row
    const bool row_ok = pr < R;
    const int gq = row_ok ? pr / a.n : 0;
    const int node = row_ok ? pr % a.n : 0;
    const int h = pi.kvh * a.group + gq;
    const int P = pi.L - a.n;
    const bool len_ok = pi.L >= a.n;

    // ---- Q rows -> shared memory (SW128 K-major), then hand them to the MMA
    // warp.  Each warp fills its own 32 rows, a half-warp per 256-byte row, so
    // a load instruction reads two whole rows (a row per thread would touch 32
    // cache lines per instruction and keep the load unit busy for
    // microseconds); 8 rows per half-warp are in flight per round trip.
    const bool walk = a.mask_kind == GORGON_MASK_PARENTS;
    if (!QTMA) {
      const int sub = lane >> 4, jc = lane & 15;  // row parity and 16-byte chunk
      const int prow0 = pi.qg * C::kQRows + wg * kBM + wq * 32 + sub;  // packed row of the first pass
      const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(a.q) + static_cast<int64_t>(pi.b) * a.q_sb +
                                static_cast<int64_t>(pi.kvh) * a.group * a.q_sh;
      constexpr int kBatch = 8;  // rows in flight per half-warp
      RowCursor rc(prow0, a.n);
#pragma unroll 1
      for (int hh = 0; hh < 16 / kBatch; ++hh) {
        uint4 qv[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
          const uint4* src = reinterpret_cast<const uint4*>(qb + static_cast<int64_t>(rc.gq) * a.q_sh +
                                                            static_cast<int64_t>(rc.node) * a.q_sn) + jc;
          qv[k] = rc.pr < R ? __ldg(src) : make_uint4(0, 0, 0, 0);
          rc.next2(a.n);
        }
#pragma unroll
        for (int k = 0; k < kBatch; ++k)
          *reinterpret_cast<uint4*>(stage_at(q_tile, wq, sub + 2 * (hh * kBatch + k), jc)) = qv[k];
      }
      fence_proxy_async_smem();
      tc_fence_before();  // the previous segment's O reads precede the next MMAs
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->q_full);
    }
    // ---- ancestor bits of this row's node
    uint32_t anc[ANCW];
#pragma unroll
    for (int k = 0; k < ANCW; ++k) anc[k] = 0;
    if (walk) {
      // The warp keeps parents[] in registers (lane l holds entries l, l + 32,
      // ...) and every lane walks its own node's chain through shuffles, so
      // the walk costs one coalesced load instead of a chain of dependent ones.
      const int32_t* par = a.parents + static_cast<int64_t>(pi.b) * a.par_sb;
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
      if (bad) raise_device_error(a.err, kErrBadParent);
    } else if (row_ok && len_ok) {
      const uint8_t* mrow =
          a.mask + static_cast<int64_t>(pi.b) * a.mask_sb + static_cast<int64_t>(node) * a.mask_sn;
      for (int j = 0; j < a.n; ++j)
        if (mrow[j]) {
#pragma unroll
          for (int k = 0; k < ANCW; ++k)
            if ((j >> 5) == k) anc[k] |= 1u << (j & 31);
        }
    }
    if (!len_ok && qrow == 0) raise_device_error(a.err, kErrBadSeqlen);

    float m_used = -INFINITY, l = 0.f;
    // One tile of this row: S -> P against the lazy running max.  Masked
    // tiles reach the tree rows or the sequence end and hide the columns this
    // row may not see; the others (all but the last one or two of a unit) run
    // a loop without that code, which keeps the hot loop's register
    // allocation and schedule tight.
    auto tile = [&](auto mask_tag) -> bool {
      constexpr bool kMask = decltype(mask_tag)::value;
      const uint32_t buf = static_cast<uint32_t>(i & 1);
      const uint32_t bi = buf * MT + wg;
      // masked tiles: the row's visibility words, before S fills the registers
      // (columns past the sequence are tree indices >= n, whose ancestor bits are 0)
      uint32_t vw[kBN / 32];
      if (kMask) {
        const int o = static_cast<int>(g - pi.start) * kBN - P;
#pragma unroll
        for (int hh = 0; hh < kBN / 64; ++hh) {
          const uint64_t w = len_ok ? vis_window<ANCW>(anc, o + 64 * hh) : 0ull;
          vw[2 * hh] = static_cast<uint32_t>(w);
          vw[2 * hh + 1] = static_cast<uint32_t>(w >> 32);
        }
      }
      if (!warp_wait(&bars->s_full[bi], static_cast<uint32_t>(i >> 1) & 1u, abort, t.wait_ns)) return false;
      // this M-tile's Q.K^T of the tile has completed: the K stage is free
      // once every warpgroup has seen its S (kSoftmaxFreesK)
      if (C::kSoftmaxFreesK && wq == 0 && lane == 0) mbar_arrive(&bars->k_empty[static_cast<uint32_t>(i % C::kStages)]);
      tc_fence_after();
      const uint32_t s_addr = lane_base + kColS + bi * kBN;
      float x[kBN];
      {
        uint32_t rr[kBN / 32][32];
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q) tmem_ld32(s_addr + 32 * q, rr[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q)
#pragma unroll
          for (int c = 0; c < 32; ++c) x[32 * q + c] = __uint_as_float(rr[q][c]);
      }
      if (kMask) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) x[c] = ((vw[c >> 5] >> (c & 31)) & 1u) ? x[c] : -INFINITY;
      }
      // row max of the raw scores (scale > 0, so it commutes with max)
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kBN; c += 2) mx[(c >> 1) & 3] = fmax3(mx[(c >> 1) & 3], x[c], x[c + 1]);
      const float tmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * sl2;
      // lazy running max: move it only when this tile exceeds it by > 8
      float alpha = 1.f;
      bool need = false;
      if (i == i_first) {
        m_used = tmax;
      } else if (tmax > m_used + 8.f) {
        alpha = ex2_approx(m_used - tmax);  // 0 while nothing was visible yet
        m_used = tmax;
        need = true;
      }
      const float nmb = m_used == -INFINITY ? 0.f : -m_used;
      const uint64_t sl2_2 = f2_pack(sl2, sl2), nmb_2 = f2_pack(nmb, nmb);
      uint64_t acc2[4] = {0, 0, 0, 0};  // bit pattern of (0.f, 0.f)
      uint32_t packed[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        float a0, a1;
        f2_unpack(f2_fma(f2_pack(x[c], x[c + 1]), sl2_2, nmb_2), a0, a1);
        const float p0 = ex2_approx(a0);
        const float p1 = ex2_approx(a1);
        const uint64_t pp = f2_pack(p0, p1);
        acc2[(c >> 1) & 3] = f2_add(acc2[(c >> 1) & 3], pp);
        if (ab_bf16) {
          const __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
          packed[c >> 1] = *reinterpret_cast<const uint32_t*>(&v2);
        } else {
          const __half2 v2 = __floats2half2_rn(p0, p1);
          packed[c >> 1] = *reinterpret_cast<const uint32_t*>(&v2);
        }
      }
      float sum;
      {
        const uint64_t s2 = f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3]));
        float s0, s1;
        f2_unpack(s2, s0, s1);
        sum = s0 + s1;
      }
      l = l * alpha + sum;
      // rescale O (warp-uniform) once the P.V of tile i - 1 has landed
      if (__any_sync(0xffffffffu, need)) {
        const int64_t pv = i - 1;
        if (!warp_wait(&bars->p_free[pv & 1], static_cast<uint32_t>(pv >> 1) & 1u, abort, t.wait_ns))
          return false;
        tc_fence_after();
        const uint32_t o_addr = lane_base + kColO + wg * kD;
#pragma unroll
        for (int ch = 0; ch < kD / 32; ++ch) {
          uint32_t ov[32];
          tmem_ld32(o_addr + ch * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
          tmem_st32(o_addr + ch * 32, ov);
        }
        tmem_wait_st();
      }
      // P row (16-bit pairs) -> the first BN / 2 columns of this tile's S buffer
#pragma unroll
      for (int q = 0; q < kBN / 64; ++q) {
        uint32_t pq[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) pq[c] = packed[32 * q + c];
        tmem_st32(s_addr + 32 * q, pq);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[bi]);
      return true;
    };
    // tiles whose BN columns all lie in the prefix before the tree rows
    const int64_t plain_end = len_ok ? pi.start + P / kBN : pi.start;
    for (; g < min(e, plain_end); ++g, ++i)
      if (!tile(std::integral_constant<bool, false>())) return;
    for (; g < e; ++g, ++i)
      if (!tile(std::integral_constant<bool, true>())) return;

    // ---- epilogue: O / l for this row, once the last P.V has landed
    const int64_t lastv = i - 1;
    if (!warp_wait(&bars->p_free[lastv & 1], static_cast<uint32_t>(lastv >> 1) & 1u, abort, t.wait_ns)) return;
    tc_fence_after();
    const int64_t orow = (static_cast<int64_t>(pi.b) * a.hq + h) * a.n + node;
    const int64_t ob = static_cast<int64_t>(pi.b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh +
                       static_cast<int64_t>(node) * a.o_sn;
    const uint32_t o_addr = lane_base + kColO + wg * kD;
    const float lse2 = (l > 0.f) ? m_used + __log2f(l) : -INFINITY;
    // The rows go out through the warp's staging rows (its slice of the Q
    // tile, free now that the segment's last Q.K^T has completed) so that
    // every store instruction writes whole rows.  A piece of a unit cut
    // between CTAs writes fp32 partials (0 where nothing was visible) into
    // slot 0 when it starts the CTA's range, else slot 1.
    const int64_t slot = static_cast<int64_t>(cta) * 2 + ((pi.start <= g0) ? 0 : 1);
    const int sub = lane >> 4, jc = lane & 15;
    const int prow0 = pi.qg * C::kQRows + wg * kBM + wq * 32 + sub;
    const int mode = whole ? t.out_vec : kOutF32;
    const float inv = 1.f / l;  // whole, l == 0: no visible key, NaN like softmax
    const bool zero = !whole && !(l > 0.f);
    if (mode == kOutBf16 || mode == kOutF16) {
#pragma unroll
      for (int ch = 0; ch < kD / 32; ++ch) {
        uint32_t ov[32];
        tmem_ld32(o_addr + ch * 32, ov);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack16x2(__uint_as_float(ov[8 * u + 2 * e]) * inv, __uint_as_float(ov[8 * u + 2 * e + 1]) * inv,
                            mode == kOutBf16);
          *reinterpret_cast<uint4*>(stage_at(q_tile, wq, lane, ch * 4 + u)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      __syncwarp();
      const int64_t ob0 = static_cast<int64_t>(pi.b) * a.o_sb + static_cast<int64_t>(pi.kvh) * a.group * a.o_sh;
      uint16_t* ob16 = static_cast<uint16_t*>(a.out) + ob0;
      RowCursor rc(prow0, a.n);
      if (t.npeers == 0) {
#pragma unroll 4
        for (int k = 0; k < 16; ++k) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage_at(q_tile, wq, sub + 2 * k, jc));
          if (rc.pr < R)
            *reinterpret_cast<uint4*>(ob16 + static_cast<int64_t>(rc.gq) * a.o_sh +
                                      static_cast<int64_t>(rc.node) * a.o_sn + jc * 8) = v;
          rc.next2(a.n);
        }
      } else {
        // the same rows into every peer's buffer too, once the peers are ready
        const int np = warp_peers_ready(t) ? t.npeers : 0;
#pragma unroll 1
        for (int k = 0; k < 16; ++k) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage_at(q_tile, wq, sub + 2 * k, jc));
          if (rc.pr < R) {
            const int64_t off = static_cast<int64_t>(rc.gq) * a.o_sh + static_cast<int64_t>(rc.node) * a.o_sn + jc * 8;
            *reinterpret_cast<uint4*>(ob16 + off) = v;
            for (int p = 0; p < np; ++p)
              *reinterpret_cast<uint4*>(static_cast<uint16_t*>(t.peer_out[p]) + ob0 + off) = v;
          }
          rc.next2(a.n);
        }
      }
      __syncwarp();
    } else if (mode == kOutF32) {
      // fp32 rows are 512 bytes: two passes of 64 columns through the staging rows
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t ov[32];
          tmem_ld32(o_addr + (ps * 2 + c2) * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(stage_at(q_tile, wq, lane, c2 * 8 + u)) =
                zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                     : make_float4(__uint_as_float(ov[4 * u]) * inv, __uint_as_float(ov[4 * u + 1]) * inv,
                                   __uint_as_float(ov[4 * u + 2]) * inv, __uint_as_float(ov[4 * u + 3]) * inv);
        }
        __syncwarp();
        if (whole) {
          float* of = static_cast<float*>(a.out) + static_cast<int64_t>(pi.b) * a.o_sb +
                      static_cast<int64_t>(pi.kvh) * a.group * a.o_sh + ps * 64 + jc * 4;
          RowCursor rc(prow0, a.n);
#pragma unroll 4
          for (int k = 0; k < 16; ++k) {
            const float4 v = *reinterpret_cast<const float4*>(stage_at(q_tile, wq, sub + 2 * k, jc));
            if (rc.pr < R)
              *reinterpret_cast<float4*>(of + static_cast<int64_t>(rc.gq) * a.o_sh +
                                         static_cast<int64_t>(rc.node) * a.o_sn) = v;
            rc.next2(a.n);
          }
        } else {
          float* po = t.part_o + (slot * C::kQRows + wg * kBM + wq * 32) * kD + ps * 64 + jc * 4;
#pragma unroll 4
          for (int k = 0; k < 16; ++k)
            *reinterpret_cast<float4*>(po + (sub + 2 * k) * kD) =
                *reinterpret_cast<const float4*>(stage_at(q_tile, wq, sub + 2 * k, jc));
        }
        __syncwarp();
      }
    } else {
#pragma unroll
      for (int ch = 0; ch < kD / 32; ++ch) {
        uint32_t ov[32];
        tmem_ld32(o_addr + ch * 32, ov);
        tmem_wait_ld();
        float vals[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) vals[c] = __uint_as_float(ov[c]) * inv;
        if (row_ok) store_cols32(t.a, ob, ch * 32, vals);
      }
    }
    if (whole) {
      if (row_ok && a.lse) a.lse[orow] = lse2 * 0.6931471805599453f;
    } else {
      t.part_lse[slot * C::kQRows + qrow] = lse2;  // attn_tc_combine merges the pieces
    }
    q_done();
  }
}

template <int MT>
__device__ void cluster_merge(const TcArgs& t);

// QTMA: the Q M-tiles come by TMA from the K producer (t.q_tma), so the
// softmax warps skip their own Q loads (a compile-time switch: as a run-time
// branch it cost the hot loop registers).
template <int MT, int ANCW, bool BF16, bool QTMA>
__global__ void __launch_bounds__(Cfg<MT>::kThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
               const __grid_constant__ CUtensorMap qmap, const __grid_constant__ TcArgs t) {
  using C = Cfg<MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers<MT>* bars = reinterpret_cast<Barriers<MT>*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], C::kSoftmaxFreesK ? MT : 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->q_full, t.q_tma ? 1 : 4 * MT);  // the K producer's expect-tx, else every softmax warp
    mbar_init(&bars->q_empty, 4 * MT);
    for (int b = 0; b < 2 * MT; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 4);  // the four warps of one softmax warpgroup
    }
    mbar_init(&bars->p_free[0], 1);
    mbar_init(&bars->p_free[1], 1);
    mbar_init(&bars->drain[0], 1);
    mbar_init(&bars->drain[1], 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    if (t.q_tma) prefetch_tensormap(&qmap);
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // (output gather) this rank's stream has reached the call: peers may write here
  if (t.npeers && blockIdx.x == 0 && threadIdx.x == 0)
    for (int p = 0; p < t.npeers; ++p) red_add_release_sys(t.peer_sig[p], 1);

  int64_t g0 = 0, g1 = 0;
  bool work;
  if (t.pair_align) {
    work = static_cast<int>(blockIdx.x) < t.pairs;
  } else if (t.cluster) {
    // unit blockIdx.x / cluster, cut into equal tile ranges, one per CTA of its cluster
    const int c = static_cast<int>(blockIdx.x) % t.cluster;
    const PairInfo pu = pair_info(t, static_cast<int>(blockIdx.x) / t.cluster);
    const int64_t n = pu.end - pu.start;
    g0 = pu.start + n * c / t.cluster;
    g1 = pu.start + n * (c + 1) / t.cluster;
    work = g0 < g1;
  } else {
    const int64_t T = total_tiles(t);
    g0 = range_start(blockIdx.x, T, t.grid);
    g1 = range_start(blockIdx.x + 1, T, t.grid);
    work = g0 < g1;
  }

  if (work) {
    if (warp == 0) {
      if (lane == 0) producer<MT>(t, &kmap, &qmap, smem, bars, g0, g1, 0);
    } else if (warp == 3) {
      if (lane == 0) producer<MT>(t, &vmap, &qmap, smem, bars, g0, g1, 1);
    } else if (warp == 1) {
      if (lane == 0) qk_issuer<MT>(t, smem, bars, tmem, g0, g1);
    } else if (warp == 2) {
      if (lane == 0) pv_issuer<MT>(t, smem, bars, tmem, g0, g1);
    } else if (warp >= 4) {
      softmax_epilogue<MT, ANCW, BF16, QTMA>(t, smem, bars, tmem, g0, g1, blockIdx.x);
    }
  }
  __syncwarp();  // role warps ran their loop on lane 0: reconverge before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (t.cluster) {
    // Every thread of every CTA of the cluster passes the barrier (the roles
    // return here on every path, a timeout included).
    __threadfence();  // the piece's rows (written by its softmax warps) before the barrier's release
    __syncwarp();
    cluster_sync();   // every piece of the cluster's unit is in the workspace
    cluster_merge<MT>(t);
  }
  if (t.npeers) {
    // (output gather) one count per CTA in every peer's `done` word, after
    // the CTA barrier: the release is cumulative, so it orders every
    // thread's stores to the peers that the barrier ordered before it
    __syncthreads();
    if (threadIdx.x == 0)
      for (int p = 0; p < t.npeers; ++p) red_add_release_sys(t.peer_sig[p] + 1, 1);
  }
  if (bars->abort && threadIdx.x == 0) raise_device_error(t.a.err, kErrTimeout);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Varlen schedule: tile prefix over units (one thread; units are few).
template <int MT>
__global__ void attn_tc_prologue(const TcArgs t) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  constexpr int kBN = Cfg<MT>::kBN;
  int acc = 0;
  int p = 0;
  for (int b = 0; b < t.a.batch; ++b) {
    const int L = t.a.cu_seqlens[b + 1] - t.a.cu_seqlens[b];
    const int nt = L > 0 ? (L + kBN - 1) / kBN : 0;
    for (int k = 0; k < t.a.hkv * t.qgroups; ++k, ++p) {
      t.tile_start[p] = acc;
      acc += nt;
    }
  }
  t.tile_start[p] = acc;
}

// Varlen schedule for whole units (one CTA of 1024 threads, at most
// kMaxSortedUnits units): the tile prefix as above, and the unit ids ordered
// by tile count, most first (ties by id), for the snake deal of Segments.
constexpr int kMaxSortedUnits = 1024;
template <int MT>
__global__ void __launch_bounds__(1024) attn_tc_prologue_sorted(const TcArgs t) {
  constexpr int kBN = Cfg<MT>::kBN;
  __shared__ int cnt[kMaxSortedUnits];
  const int U = t.pairs;
  const int per_b = t.a.hkv * t.qgroups;
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int b = u / per_b;
    const int L = t.a.cu_seqlens[b + 1] - t.a.cu_seqlens[b];
    cnt[u] = L > 0 ? (L + kBN - 1) / kBN : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int u = 0; u < U; ++u) {
      t.tile_start[u] = acc;
      acc += cnt[u];
    }
    t.tile_start[U] = acc;
  }
  for (int u = threadIdx.x; u < U; u += blockDim.x) {
    const int c = cnt[u];
    int r = 0;
    for (int v = 0; v < U; ++v) {
      const int cv = cnt[v];
      r += (cv > c || (cv == c && v < u)) ? 1 : 0;
    }
    t.order[r] = u;
  }
}

// Merges the pieces of every unit that the stream-K schedule cut between
// CTAs: out = sum_k 2^(lse_k - M) o_k / sum_k 2^(lse_k - M) with M = max_k
// lse_k (log2 units) and o_k each piece's normalised output.  Grid (units,
// rows per unit / 32), 8 warps of 4 rows each.  One thread works out the
// unit's pieces (their CTAs and workspace slots) for the block.  With at most
// kCombineFast pieces (every unit of a batch large enough to fill the GPU) a
// warp issues the lse values of its 4 rows in one round trip (8 lanes per
// row) and then every piece's 512-byte row of all 4 rows in another, a lane
// holding four columns; more pieces go row by row, 32 lse values and 8
// pieces' rows in flight at a time.  Units that one CTA finished are skipped.
constexpr int kCombineWarps = 8;
constexpr int kCombineThreads = kCombineWarps * 32;
constexpr int kCombineRowsPerWarp = 4;
constexpr int kCombineRows = kCombineWarps * kCombineRowsPerWarp;  // rows per CTA
constexpr int kCombineFast = 4;                                    // pieces per row on the fast path

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Writes four consecutive output columns of one row.
// np: peers whose buffers also get the values (the output gather; 16-bit
// outputs only, and only after warp_peers_ready).
__device__ __forceinline__ void store4(const TcArgs& t, int64_t idx, float x, float y, float z, float w,
                                       int np = 0) {
  if (t.out_vec == kOutBf16 || t.out_vec == kOutF16) {
    const bool bf = t.out_vec == kOutBf16;
    const uint2 v = make_uint2(pack16x2(x, y, bf), pack16x2(z, w, bf));
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(t.a.out) + idx) = v;
    for (int p = 0; p < np; ++p) *reinterpret_cast<uint2*>(static_cast<uint16_t*>(t.peer_out[p]) + idx) = v;
  } else if (t.out_vec == kOutF32) {
    *reinterpret_cast<float4*>(static_cast<float*>(t.a.out) + idx) = make_float4(x, y, z, w);
  } else {
    store_as(t.a.out, t.a.out_dtype, idx, x);
    store_as(t.a.out, t.a.out_dtype, idx + 1, y);
    store_as(t.a.out, t.a.out_dtype, idx + 2, z);
    store_as(t.a.out, t.a.out_dtype, idx + 3, w);
  }
}

// The merge of a unit cut between the CTAs of a cluster: every piece leaves
// its normalised fp32 rows and log-sum-exp in its workspace slot (like a
// stream-K piece), and after the cluster barrier CTA c of the cluster
// finishes packed rows [c * rows / size, (c + 1) * rows / size) of the unit,
// a warp per row, reading the pieces' rows from L2.  out = sum_j w_j o_j /
// sum_j w_j with w_j = 2^(lse_j - max lse); pieces that saw no key weigh 0
// (their rows are never multiplied in), and a row no piece saw is NaN with
// log-sum-exp -inf, like the single-CTA path.  A warp issues the loads of
// 16 / size of its rows before it uses any, one round trip per batch.
// Measured against reading the pieces from the other CTAs' shared memory
// (distributed shared memory): ~64 KB per CTA took 3.3-3.5 us that way.
constexpr int kMaxCluster = 8;
constexpr int kMergeSlots = 16;  // (row, piece) loads in flight per lane

template <int MT, int NC>
__device__ void cluster_merge_n(const TcArgs& t) {
  using C = Cfg<MT>;
  constexpr int kWarps = C::kThreads / 32;
  constexpr int kRows = kMergeSlots / NC;  // rows per batch
  const AttnArgs& a = t.a;
  const int c = static_cast<int>(blockIdx.x) % NC;
  const int unit = static_cast<int>(blockIdx.x) / NC;
  const PairInfo pi = pair_info(t, unit);
  const int R = a.group * a.n;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // piece j of the unit is CTA unit * NC + j, workspace slot 2 * (unit * NC + j)
  const int64_t slot0 = static_cast<int64_t>(unit) * NC * 2;
  // this CTA's rows that are real packed rows: [r0, r1)
  const int r0 = c * C::kQRows / NC;
  const int r1 = min((c + 1) * C::kQRows / NC, R - pi.qg * C::kQRows);
  const int np = (t.npeers && r0 + warp < r1 && warp_peers_ready(t)) ? t.npeers : 0;
#pragma unroll 1
  for (int rb = r0 + warp; rb < r1; rb += kWarps * kRows) {
    // lane k * NC + j holds piece j's log-sum-exp of batch row k (-inf for a
    // piece with no tiles, which wrote nothing: the planner gives every CTA
    // at least one tile, but the merge does not rely on it)
    float lj = -INFINITY;
    {
      const int k = lane / NC, j = lane - (lane / NC) * NC;
      const int row = rb + kWarps * k;
      const int64_t nt = pi.end - pi.start;
      if (k < kRows && row < r1 && nt * (j + 1) / NC > nt * j / NC)
        lj = __ldcg(t.part_lse + (slot0 + 2 * j) * C::kQRows + row);
    }
    float4 v[kRows][NC];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int row = rb + kWarps * k;
      if (row < r1) {
#pragma unroll
        for (int j = 0; j < NC; ++j)
          v[k][j] = __ldcg(reinterpret_cast<const float4*>(t.part_o + ((slot0 + 2 * j) * C::kQRows + row) * kD) + lane);
      }
    }
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int row = rb + kWarps * k;
      float lk[NC];
      float M = -INFINITY;
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        lk[j] = __shfl_sync(0xffffffffu, lj, k * NC + j);
        M = fmaxf(M, lk[j]);
      }
      if (row >= r1) continue;  // warp-uniform
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float wsum = 0.f;
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const float w = (lk[j] == -INFINITY) ? 0.f : ex2_approx(lk[j] - M);
        wsum += w;
        if (w > 0.f) {
          acc.x = fmaf(w, v[k][j].x, acc.x);
          acc.y = fmaf(w, v[k][j].y, acc.y);
          acc.z = fmaf(w, v[k][j].z, acc.z);
          acc.w = fmaf(w, v[k][j].w, acc.w);
        }
      }
      const int pr = pi.qg * C::kQRows + row;
      const int gq = pr / a.n, node = pr - gq * a.n;
      const int h = pi.kvh * a.group + gq;
      const int64_t orow = (static_cast<int64_t>(pi.b) * a.hq + h) * a.n + node;
      const int64_t ob = static_cast<int64_t>(pi.b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh +
                         static_cast<int64_t>(node) * a.o_sn;
      if (M == -INFINITY) {
        store4(t, ob + lane * 4, NAN, NAN, NAN, NAN, np);
        if (a.lse && lane == 0) a.lse[orow] = -INFINITY;
      } else {
        const float winv = 1.f / wsum;
        store4(t, ob + lane * 4, acc.x * winv, acc.y * winv, acc.z * winv, acc.w * winv, np);
        if (a.lse && lane == 0) a.lse[orow] = (M + __log2f(wsum)) * 0.6931471805599453f;
      }
    }
  }
}

template <int MT>
__device__ void cluster_merge(const TcArgs& t) {
  switch (t.cluster) {
    case 2: cluster_merge_n<MT, 2>(t); break;
    case 3: cluster_merge_n<MT, 3>(t); break;
    case 4: cluster_merge_n<MT, 4>(t); break;
    case 5: cluster_merge_n<MT, 5>(t); break;
    case 6: cluster_merge_n<MT, 6>(t); break;
    case 7: cluster_merge_n<MT, 7>(t); break;
    case 8: cluster_merge_n<MT, 8>(t); break;
    default: break;
  }
}

template <int MT>
__global__ void __launch_bounds__(kCombineThreads) attn_tc_combine(const TcArgs t) {
  constexpr int kQRows = Cfg<MT>::kQRows;
  __shared__ long long s_slot0, s_first;
  __shared__ int s_parts;
  const PairInfo pi = pair_info(t, blockIdx.x);
  if (threadIdx.x == 0) {
    int parts = 0;
    if (pi.end > pi.start) {
      const int64_t T = total_tiles(t);
      const int64_t first = cta_of(pi.start, T, t.grid);
      parts = static_cast<int>(cta_of(pi.end - 1, T, t.grid) - first + 1);
      s_first = first;
      // slot 1 when the unit is the second one in its first CTA's range
      s_slot0 = first * 2 + (pi.start > range_start(first, T, t.grid) ? 1 : 0);
    }
    s_parts = parts;
  }
  __syncthreads();
  const int parts = s_parts;
  if (parts <= 1) return;
  const int64_t first = s_first, slot0 = s_slot0;
  auto slot = [&](int j) -> int64_t { return j == 0 ? slot0 : (first + j) * 2; };
  const AttnArgs& a = t.a;
  const int R = a.group * a.n;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrow0 = blockIdx.y * kCombineRows + warp * kCombineRowsPerWarp;
  const int pr0 = pi.qg * kQRows + qrow0;  // packed row of the warp's first row
  // Finishes row k from its weighted sum: NaN (and lse -inf) when no piece saw a key.
  auto finish = [&](int k, float M, float wsum, float4 acc) {
    const int pr = pr0 + k;
    const int gq = pr / a.n, node = pr - gq * a.n;
    const int h = pi.kvh * a.group + gq;
    const int64_t orow = (static_cast<int64_t>(pi.b) * a.hq + h) * a.n + node;
    const int64_t ob =
        static_cast<int64_t>(pi.b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh + static_cast<int64_t>(node) * a.o_sn;
    if (M == -INFINITY) {
      store4(t, ob + lane * 4, NAN, NAN, NAN, NAN);
      if (a.lse && lane == 0) a.lse[orow] = -INFINITY;
      return;
    }
    const float winv = 1.f / wsum;
    store4(t, ob + lane * 4, acc.x * winv, acc.y * winv, acc.z * winv, acc.w * winv);
    if (a.lse && lane == 0) a.lse[orow] = (M + __log2f(wsum)) * 0.6931471805599453f;
  };

  if (parts <= kCombineFast) {
    // lanes 8k .. 8k + 7 hold row k's piece lse values
    const int kr = lane >> 3, jp = lane & 7;
    float lj = -INFINITY;
#pragma unroll
    for (int k = 0; k < kCombineRowsPerWarp; ++k)
      if (k == kr && pr0 + k < R && jp < parts) lj = __ldcg(t.part_lse + slot(jp) * kQRows + qrow0 + k);
    float4 v[kCombineRowsPerWarp][kCombineFast];
#pragma unroll
    for (int k = 0; k < kCombineRowsPerWarp; ++k)
#pragma unroll
      for (int j = 0; j < kCombineFast; ++j)
        v[k][j] = (pr0 + k < R && j < parts)
                      ? __ldcg(reinterpret_cast<const float4*>(t.part_o + (slot(j) * kQRows + qrow0 + k) * kD) + lane)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    float M = lj;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wj = M == -INFINITY ? 0.f : ex2_approx(lj - M);  // 0 for missing pieces
#pragma unroll
    for (int k = 0; k < kCombineRowsPerWarp; ++k) {
      const float Mk = __shfl_sync(0xffffffffu, M, 8 * k);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float wsum = 0.f;
#pragma unroll
      for (int j = 0; j < kCombineFast; ++j) {
        const float w = __shfl_sync(0xffffffffu, wj, 8 * k + j);
        wsum += w;
        acc.x = fmaf(w, v[k][j].x, acc.x);
        acc.y = fmaf(w, v[k][j].y, acc.y);
        acc.z = fmaf(w, v[k][j].z, acc.z);
        acc.w = fmaf(w, v[k][j].w, acc.w);
      }
      if (pr0 + k < R) finish(k, Mk, wsum, acc);
    }
    return;
  }

#pragma unroll 1
  for (int k = 0; k < kCombineRowsPerWarp; ++k) {
    if (pr0 + k >= R) continue;
    const int qrow = qrow0 + k;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float M = -INFINITY, wsum = 0.f;
    for (int c0 = 0; c0 < parts; c0 += 32) {
      // lane j holds piece c0 + j's lse; the group's max rescales what came before
      const int cj = c0 + lane;
      const float lj = cj < parts ? __ldcg(t.part_lse + slot(cj) * kQRows + qrow) : -INFINITY;
      const float Mn = fmaxf(M, warp_max(lj));
      if (Mn == -INFINITY) continue;  // nothing visible yet
      const float r = ex2_approx(M - Mn);  // 0 while M was -inf
      acc.x *= r; acc.y *= r; acc.z *= r; acc.w *= r;
      wsum *= r;
      M = Mn;
      const float wj = ex2_approx(lj - M);  // 0 for pieces past the end or with nothing visible
      const int n_here = min(32, parts - c0);
      for (int j0 = 0; j0 < n_here; j0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = j0 + j < n_here
                     ? __ldcg(reinterpret_cast<const float4*>(t.part_o + (slot(c0 + j0 + j) * kQRows + qrow) * kD) +
                              lane)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float w = __shfl_sync(0xffffffffu, wj, (j0 + j) & 31);
          if (j0 + j < n_here) {
            wsum += w;
            acc.x = fmaf(w, v[j].x, acc.x);
            acc.y = fmaf(w, v[j].y, acc.y);
            acc.z = fmaf(w, v[j].z, acc.z);
            acc.w = fmaf(w, v[j].w, acc.w);
          }
        }
      }
    }
    finish(k, M, wsum, acc);
  }
}

// (output gather) Ends the call on this rank's stream: waits until every
// peer CTA of the call has counted in our `done` word (a running total:
// npeers x grid more than after the last call), then records the call.
__global__ void attn_peer_wait(uint64_t* sig, int npeers, int grid, uint64_t wait_ns, uint32_t* err) {
  if (threadIdx.x != 0) return;
  const uint64_t expected = sig[3] + static_cast<uint64_t>(npeers) * static_cast<uint64_t>(grid);
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(sig + 1) < expected) {
    if (globaltimer_ns() - t0 > wait_ns) {
      raise_device_error(err, kErrTimeout);
      break;
    }
    __nanosleep(100);
  }
  sig[3] = expected;
  sig[2] = sig[2] + 1;
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

struct Plan {
  int mt;  // 128-row M-tiles per CTA
  int qgroups, pairs, tiles_per_pair, grid;
  bool varlen, pair_align;
  int cluster;  // > 1: CTAs per unit in a thread-block cluster (no workspace partials, no merge launch)
  bool sorted;  // varlen whole units, longest first (attn_tc_prologue_sorted)
};

template <int MT>
int cluster_capacity(int size);

// Units cut between the CTAs of a cluster: as many CTAs per unit as the SMs
// allow (at most 8, the portable cluster size, and no more than the unit has
// tiles), shrunk until every cluster is resident at once; 0 when fewer than
// two CTAs per unit fit.
template <int MT>
int cluster_size(int pairs, int tiles_per_pair, int sms) {
  int cl = std::min({kMaxCluster, sms / std::max(1, pairs), tiles_per_pair});
  while (cl >= 2 && cluster_capacity<MT>(cl) < pairs) --cl;
  return cl >= 2 ? cl : 0;
}

template <int MT>
Plan make_plan_mt(const AttnArgs& a) {
  using C = Cfg<MT>;
  Plan pl{};
  pl.mt = MT;
  const int R = a.group * a.n;
  pl.qgroups = (R + C::kQRows - 1) / C::kQRows;
  pl.pairs = a.batch * a.hkv * pl.qgroups;
  pl.varlen = a.cu_seqlens != nullptr;
  const int sms = sm_count();
  pl.pair_align = false;
  if (pl.varlen) {
    pl.tiles_per_pair = 0;
    pl.grid = a.splits > 0 ? a.splits : sms;
    if (a.splits <= 0 && pl.pairs >= sms && pl.pairs <= kMaxSortedUnits) {
      // enough units to fill the GPU: whole units, longest first, dealt out
      // in snake order (no partials, no merge launch)
      pl.pair_align = true;
      pl.sorted = true;
    }
  } else {
    pl.tiles_per_pair = (a.kv_len + C::kBN - 1) / C::kBN;
    const int64_t T = static_cast<int64_t>(pl.pairs) * pl.tiles_per_pair;
    if (a.splits > 0) {
      pl.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(a.splits, T)));
    } else {
      // Whole units per CTA avoid the partial write and the merge, which cost
      // about a fifth of a unit's time on a loaded GPU (measured on the 16 x
      // 8192-row Llama-3-8B layer); take them unless stream-K's even split is
      // more than that much shorter.
      const int64_t per_cta = (pl.pairs + sms - 1) / sms;
      const int64_t cost_pairs = per_cta * pl.tiles_per_pair;
      if (cost_pairs * 5 <= ((T + sms - 1) / sms) * 6) {
        pl.pair_align = true;
        pl.grid = static_cast<int>(std::min<int64_t>(sms, pl.pairs));
      } else if (const int cl = cluster_size<MT>(pl.pairs, pl.tiles_per_pair, sms)) {
        pl.cluster = cl;
        pl.grid = pl.pairs * cl;
      } else {
        // at least 4 tiles per CTA so partials stay a small share of the work
        const int64_t g0 = std::max<int64_t>(1, std::min<int64_t>(sms, (T + 3) / 4));
        // With room for two or more CTAs per unit, a grid that is a multiple
        // of the unit count cuts every unit into equal pieces, one per CTA
        // (range c * T / grid never straddles a unit boundary).  Otherwise
        // some CTAs start two units and write two sets of partials, and with
        // few tiles per CTA those run about twice as long as the rest:
        // measured on one sequence with a 2048-token prefix, 64 CTAs take
        // 28.3 us against 35.8 for 68, and 2-4 sequences or an 8192-token
        // prefix gain 14-20 %.
        const int64_t per_unit = g0 / pl.pairs;
        pl.grid = static_cast<int>(per_unit >= 2 ? per_unit * pl.pairs : g0);
      }
    }
  }
  return pl;
}

// The CTA shape: two M-tiles (K/V staged once for 256 rows) or one (128-key
// tiles, twice the units).  Whole units filling the GPU beat any split, so a
// shape whose plan is whole units wins, MT = 2 first; between two split
// plans, MT = 2 once the work per SM is large (its K/V staging pays), MT = 1
// below (less fixed work per piece): the MT = 2 tile count per SM crosses
// over between 14 and 28.  Measured on B200 (bf16, 32 q / 8 kv heads,
// 64-node trees, CUDA graphs, us, MT = 1 against MT = 2): 8 x 2048 28.5 /
// 38.6 and 8 x 4096 46.7 / 54.7 (MT = 1 whole units); 2 x 8192 34.3 / 37.2
// and 1 x 2048 19.3 / 22.3 (split, few tiles); 4 x 8192 53.4 / 50.7 and
// 2 x 16384 53.0 / 51.1 (split, many tiles); 16 x 8192 159.4 / 148.4 and
// 256-node trees over 8 x 32k 1351 / 1142 (MT = 2 whole units).
Plan make_plan(const AttnArgs& a) {
  const Plan p2 = make_plan_mt<2>(a);
  if (p2.pair_align) return p2;
  const Plan p1 = make_plan_mt<1>(a);
  if (p1.pair_align) return p1;
  const int64_t units2 = static_cast<int64_t>(a.batch) * a.hkv * ((a.group * a.n + 2 * kBM - 1) / (2 * kBM));
  const int64_t tiles2 = units2 * ((static_cast<int64_t>(a.kv_len) + Cfg<2>::kBN - 1) / Cfg<2>::kBN);
  return tiles2 <= 20LL * sm_count() ? p1 : p2;
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct WsLayout {
  size_t part_o, part_lse, tile_start, order, total;
};

WsLayout ws_layout(const Plan& pl) {
  const size_t rows = static_cast<size_t>(pl.mt) * kBM;
  WsLayout w{};
  size_t off = 0;
  w.tile_start = off; off += align_up(static_cast<size_t>(pl.pairs + 1) * sizeof(int));
  w.order = off;      off += align_up(static_cast<size_t>(pl.sorted ? pl.pairs : 0) * sizeof(int));
  const size_t slots = static_cast<size_t>(pl.grid) * 2;
  w.part_lse = off;   off += align_up(slots * rows * sizeof(float));
  w.part_o = off;     off += align_up(slots * rows * kD * sizeof(float));
  w.total = off;
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raises a kernel's dynamic shared-memory limit once per (kernel, device)
// rather than on every launch.
int ensure_smem_limit(const void* fn, uint32_t bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "tcgen05 current device");
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : done)
    if (e.first == fn && e.second == dev) return GORGON_OK;
  rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                  "tcgen05 smem attribute");
  if (!rc) done.emplace_back(fn, dev);
  return rc;
}

// How many clusters of `size` CTAs of the MT kernel can be resident at once
// (thread-block clusters sit inside one GPC, so this is below SMs / size when
// the GPCs' SM counts are not multiples of it); once per (device, MT, size).
template <int MT>
int cluster_capacity(int size) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, int>, int>> cache;  // ((device, size), clusters)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& e : cache)
      if (e.first.first == dev && e.first.second == size) return e.second;
  }
  using C = Cfg<MT>;
  const void* fn = reinterpret_cast<const void*>(attn_tc_kernel<MT, 2, true, true>);
  int n = 0;
  if (ensure_smem_limit(fn, C::kSmemBytes) == GORGON_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(size));
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(size);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();  // not sticky: clear it, plan without clusters, ask again next time
      return 0;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({{dev, size}, n});
  return n;
}

template <int MT>
int launch_mt(const AttnArgs& a, int dtype, const Plan& pl, const CUtensorMap& kmap, const CUtensorMap& vmap,
              const CUtensorMap& qmap, TcArgs& t, cudaStream_t st) {
  using C = Cfg<MT>;
  int rc = GORGON_OK;
  if (pl.varlen) {
    if (pl.sorted)
      attn_tc_prologue_sorted<MT><<<1, 1024, 0, st>>>(t);
    else
      attn_tc_prologue<MT><<<1, 32, 0, st>>>(t);
    rc = check_cuda(cudaGetLastError(), "tcgen05 prologue launch");
    if (rc) return rc;
  }
  using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const TcArgs);
  Kern kern;
  const bool bf = dtype == GORGON_BF16;
  if (t.q_tma)
    kern = a.n <= 64 ? (bf ? attn_tc_kernel<MT, 2, true, true> : attn_tc_kernel<MT, 2, false, true>)
                     : (bf ? attn_tc_kernel<MT, 8, true, true> : attn_tc_kernel<MT, 8, false, true>);
  else
    kern = a.n <= 64 ? (bf ? attn_tc_kernel<MT, 2, true, false> : attn_tc_kernel<MT, 2, false, false>)
                     : (bf ? attn_tc_kernel<MT, 8, true, false> : attn_tc_kernel<MT, 8, false, false>);
  rc = ensure_smem_limit(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (rc) return rc;
  if (pl.cluster) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(pl.cluster);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, kern, kmap, vmap, qmap, t), "tcgen05 tree attention cluster launch");
  }
  kern<<<pl.grid, C::kThreads, C::kSmemBytes, st>>>(kmap, vmap, qmap, t);
  rc = check_cuda(cudaGetLastError(), "tcgen05 tree attention launch");
  if (rc || pl.pair_align) return rc;
  attn_tc_combine<MT><<<dim3(pl.pairs, C::kQRows / kCombineRows), kCombineThreads, 0, st>>>(t);
  return check_cuda(cudaGetLastError(), "tcgen05 combine launch");
}

}  // namespace

bool attn_tc_supported(const AttnArgs& a, int dtype) {
  if (dtype != GORGON_BF16 && dtype != GORGON_F16) return false;
  if (a.d != kD || a.n < 1 || a.n > 256) return false;
  if (a.mask_kind != GORGON_MASK_PARENTS && a.mask_kind != GORGON_MASK_DENSE_TREE) return false;
  if (!a.vec_ok || !aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v)) return false;
  if (a.cu_seqlens && a.kv_rows <= 0) return false;
  // TMA strides are byte multiples of 16 (vec_ok already makes element strides multiples of 8)
  if (!encode_fn()) return false;
  return true;
}

size_t attn_tc_workspace(const AttnArgs& a) { return ws_layout(make_plan(a)).total; }

void attn_tc_plan(const AttnArgs& a, int32_t* splits, int32_t* launches) {
  const Plan pl = make_plan(a);
  *splits = pl.grid;
  *launches = 1 + (pl.varlen ? 1 : 0) + (pl.pair_align || pl.cluster ? 0 : 1);
}

int launch_attn_tc(const AttnArgs& a, int dtype, void* workspace, size_t ws_bytes, cudaStream_t st,
                   const PeerLaunch* peers) {
  const Plan pl = make_plan(a);
  const WsLayout w = ws_layout(pl);
  if (!workspace || ws_bytes < w.total)
    return set_error(GORGON_ERR_WORKSPACE, "tcgen05 tree attention: workspace too small");
  if (peers && !pl.pair_align && !pl.cluster)
    return set_error(GORGON_ERR_UNSUPPORTED, "tree attention gather: this shape's plan merges pieces in a second "
                                             "launch (stream-K); the fused gather needs whole units or a cluster plan");
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GORGON_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType tdt = dtype == GORGON_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint32_t bn = pl.mt == 1 ? Cfg<1>::kBN : Cfg<2>::kBN;  // box rows = K/V tile rows
  CUtensorMap kmap, vmap;
  const void* srcs[2] = {a.k, a.v};
  const int64_t ss[2] = {a.k_ss, a.v_ss}, sh[2] = {a.k_sh, a.v_sh}, sb[2] = {a.k_sb, a.v_sb};
  CUtensorMap* maps[2] = {&kmap, &vmap};
  for (int m = 0; m < 2; ++m) {
    CUresult r;
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (pl.varlen) {
      const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.hkv),
                                  static_cast<cuuint64_t>(a.kv_rows)};
      const cuuint64_t strides[2] = {static_cast<cuuint64_t>(sh[m]) * 2, static_cast<cuuint64_t>(ss[m]) * 2};
      const cuuint32_t box[3] = {64, 1, bn};
      r = enc(maps[m], tdt, 3, const_cast<void*>(srcs[m]), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.kv_len),
                                  static_cast<cuuint64_t>(a.hkv), static_cast<cuuint64_t>(a.batch)};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss[m]) * 2, static_cast<cuuint64_t>(sh[m]) * 2,
                                     static_cast<cuuint64_t>(sb[m]) * 2};
      const cuuint32_t box[4] = {64, bn, 1, 1};
      r = enc(maps[m], tdt, 4, const_cast<void*>(srcs[m]), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS)
      return set_error(GORGON_ERR_INVALID, "tcgen05 tree attention: cuTensorMapEncodeTiled rejected the K/V layout "
                                           "(strides must be multiples of 16 bytes)");
  }
  TcArgs t{};
  t.a = a;
  t.varlen = pl.varlen;
  t.qgroups = pl.qgroups;
  t.pairs = pl.pairs;
  t.tiles_per_pair = pl.tiles_per_pair;
  t.grid = pl.grid;
  t.pair_align = pl.pair_align;
  t.cluster = pl.cluster;
  t.ab_fmt = dtype == GORGON_BF16 ? 1 : 0;
  t.wait_ns = wait_limit_ns();
  char* ws = static_cast<char*>(workspace);
  t.tile_start = reinterpret_cast<int*>(ws + w.tile_start);
  t.order = pl.sorted ? reinterpret_cast<int*>(ws + w.order) : nullptr;
  t.part_lse = reinterpret_cast<float*>(ws + w.part_lse);
  t.part_o = reinterpret_cast<float*>(ws + w.part_o);
  {
    // rows of whole 16-byte chunks: strides in elements that are multiples of 16 bytes
    const int per16 = a.out_dtype == GORGON_F32 ? 4 : 8;
    const bool rows16 = aligned16(a.out) && a.o_sb % per16 == 0 && a.o_sh % per16 == 0 && a.o_sn % per16 == 0;
    t.out_vec = !rows16 ? 0
                        : a.out_dtype == GORGON_BF16 ? kOutBf16
                                                     : (a.out_dtype == GORGON_F16 ? kOutF16 : kOutF32);
  }
  // Q by TMA when a 128-row M-tile is whole heads (n divides 128) or part of
  // one (n a multiple of 128): a 4-D box (64 columns, nodes, heads, 1) over
  // q [B, Hq, n, D] is then 128 consecutive packed rows.  Cluster plans only:
  // their CTAs have few tiles, so the earlier first Q.K^T shows (one
  // sequence over 2048 tokens 16.3 -> 15.4 us, two over 8192 32.7 -> 31.6);
  // whole-unit plans measured ~1 % slower with it.
  CUtensorMap qmap;
  std::memset(&qmap, 0, sizeof(qmap));
  if (pl.cluster && (kBM % a.n == 0 || a.n % kBM == 0) && a.q_sn > 0) {
    const int nb = a.n < kBM ? a.n : kBM;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.n),
                                static_cast<cuuint64_t>(a.hq), static_cast<cuuint64_t>(a.batch)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.q_sn) * 2, static_cast<cuuint64_t>(a.q_sh) * 2,
                                   static_cast<cuuint64_t>(a.q_sb) * 2};
    const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(nb), static_cast<cuuint32_t>(kBM / nb), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    t.q_tma = enc(&qmap, tdt, 4, const_cast<void*>(a.q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (peers) {
    if (t.out_vec != kOutBf16 && t.out_vec != kOutF16)
      return set_error(GORGON_ERR_UNSUPPORTED, "tree attention gather: needs bf16/f16 output rows of whole 16-byte chunks");
    t.npeers = peers->npeers;
    for (int p = 0; p < peers->npeers; ++p) {
      t.peer_out[p] = peers->peer_out[p];
      t.peer_sig[p] = peers->peer_sig[p];
    }
    t.sig = peers->sig;
  }
  const int rc = pl.mt == 1 ? launch_mt<1>(a, dtype, pl, kmap, vmap, qmap, t, st)
                            : launch_mt<2>(a, dtype, pl, kmap, vmap, qmap, t, st);
  if (rc || !peers) return rc;
  attn_peer_wait<<<1, 32, 0, st>>>(peers->sig, peers->npeers, pl.grid, t.wait_ns, a.err);
  return check_cuda(cudaGetLastError(), "tree attention gather: wait launch");
}

}  // namespace gorgon
