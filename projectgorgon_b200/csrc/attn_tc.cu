// Tensor-core (tcgen05) tree attention for sm_100a.
//
// Unit of work: a "pair" = (sequence b, kv head, query group).  A query group
// packs up to 256 rows of (query head in the GQA group, tree node): row
// g * n + i.  Those rows share every key/value row of the pair, so each K/V
// tile is fetched from HBM once and used by two 128-row MMA tiles.
//
// Schedule: a persistent grid (at most one CTA per SM) splits the global list
// of 64-row key/value tiles, pair-major, into equal contiguous ranges.  A pair
// that falls inside one CTA is finished there; a pair cut between CTAs leaves
// normalised partials plus log-sum-exp in the workspace and the CTA that
// finishes it last merges them (no spinning: an atomic arrival count).
//
// Warp roles (384 threads):
//   warp 0       TMA producer: K and V tiles (two 64-column SW128 boxes each)
//                into a 3-stage ring
//   warp 1       MMA issuer (one thread): S = Q K^T into TMEM, O += P V
//   warp 2       TMEM allocation / release
//   warps 4-7    softmax + epilogue of M-tile 0 (TMEM lanes 0-127)
//   warps 8-11   softmax + epilogue of M-tile 1
// TMEM (512 columns): S double-buffered (2 buffers x 2 M-tiles x 64 columns),
// O (2 M-tiles x 128 columns).  P goes back through shared memory (bf16,
// SW128 K-major) as the A operand of the P.V MMA.
//
// Softmax per row is owned by one thread (TMEM lane = row), so row max and
// sum need no shuffles.  Rescaling of O is lazy: the running max only moves
// when a tile's max exceeds it by more than 8 (log2 units), which bounds P by
// 2^8 and makes O corrections rare.  Every mbarrier wait is bounded; on
// timeout the CTA raises kErrTimeout, drains its copies and MMAs, frees TMEM
// and returns.
#include <cuda.h>

#include <mutex>

#include "attn.cuh"
#include "sm100.cuh"

namespace gorgon {

constexpr uint32_t kErrTimeout = 1u << 4;

namespace {
using namespace sm100;

constexpr int kBM = 128;              // rows per MMA tile
constexpr int kQRows = 2 * kBM;       // packed query rows per pair
constexpr int kBN = 64;               // key/value rows per tile
constexpr int kD = 128;               // head_dim
constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// shared memory layout (bytes from a 1024-aligned base)
constexpr uint32_t kQHalf = kBM * 128;                 // 128 rows x 64 cols bf16 = 16 KB
constexpr uint32_t kKVHalf = kBN * 128;                // 64 rows x 64 cols = 8 KB
constexpr uint32_t kStageBytes = 4 * kKVHalf;          // K and V, two halves each
constexpr uint32_t kPTile = kBM * kBN * 2;             // 128 x 64 bf16 = 16 KB
constexpr uint32_t kOffQ = 0;                          // [mtile][half]
constexpr uint32_t kOffKV = kOffQ + 4 * kQHalf;        // [stage][K0 K1 V0 V1]
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;  // [buf][mtile]
constexpr uint32_t kOffBar = kOffP + 4 * kPTile;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + alignment slack

// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // + (buf * 2 + mtile) * 64
constexpr uint32_t kColO = 256;  // + mtile * 128

struct TcArgs {
  AttnArgs a;
  int varlen;
  int qgroups;        // query groups per (b, kv head)
  int pairs;          // batch * hkv * qgroups
  int tiles_per_pair; // uniform lengths only
  int grid;
  int ab_fmt;         // 0 f16, 1 bf16
  int out_vec;        // bf16 output with 16-byte aligned rows
  int* counters;      // [pairs][8] arrivals of partial pairs, per softmax warp
  float* part_o;      // [grid * 2][256][128]
  float* part_lse;    // [grid * 2][256]
  int* tile_start;    // varlen: [pairs + 1] tile prefix (written by attn_tc_prologue)
};

struct Barriers {
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t p_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

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

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in an SW128 K-major
// tile whose rows are 128 bytes.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  return mbar_wait(bar, parity, abort, kWaitLimitNs);
}

// Wait used on the way out: ignores the abort flag, gives up after 100 ms.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 100000000ull) break;
  }
}

// ------------------------------------------------------------ roles
__device__ void producer(const TcArgs& t, const CUtensorMap* kmap, const CUtensorMap* vmap, uint8_t* smem,
                         Barriers* bars, int64_t g0, int64_t g1) {
  volatile int* abort = &bars->abort;
  int64_t issued = 0;
  int cur_pair = -1;
  PairInfo pi{};
  for (int64_t g = g0; g < g1; ++g) {
    const int p = pair_of(t, g);
    if (p != cur_pair) {
      cur_pair = p;
      pi = pair_info(t, p);
    }
    const int tile = static_cast<int>(g - pi.start);
    const int stage = static_cast<int>(issued % kStages);
    const uint32_t ph = static_cast<uint32_t>(issued / kStages) & 1u;
    if (!bounded_wait(&bars->kv_empty[stage], ph ^ 1u, abort)) break;
    mbar_arrive_expect_tx(&bars->kv_full[stage], kStageBytes);
    uint8_t* st = smem + kOffKV + stage * kStageBytes;
    const int row = tile * kBN;
    if (t.varlen) {
      const int r = pi.row0 + row;
      tma_load_3d(st + 0 * kKVHalf, kmap, &bars->kv_full[stage], 0, pi.kvh, r);
      tma_load_3d(st + 1 * kKVHalf, kmap, &bars->kv_full[stage], 64, pi.kvh, r);
      tma_load_3d(st + 2 * kKVHalf, vmap, &bars->kv_full[stage], 0, pi.kvh, r);
      tma_load_3d(st + 3 * kKVHalf, vmap, &bars->kv_full[stage], 64, pi.kvh, r);
    } else {
      tma_load_4d(st + 0 * kKVHalf, kmap, &bars->kv_full[stage], 0, row, pi.kvh, pi.b);
      tma_load_4d(st + 1 * kKVHalf, kmap, &bars->kv_full[stage], 64, row, pi.kvh, pi.b);
      tma_load_4d(st + 2 * kKVHalf, vmap, &bars->kv_full[stage], 0, row, pi.kvh, pi.b);
      tma_load_4d(st + 3 * kKVHalf, vmap, &bars->kv_full[stage], 64, row, pi.kvh, pi.b);
    }
    ++issued;
  }
  // Every issued load must land before the CTA leaves.
  for (int64_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k)
    drain_wait(&bars->kv_full[k % kStages], static_cast<uint32_t>(k / kStages) & 1u);
}

__device__ void mma_issuer(const TcArgs& t, uint8_t* smem, Barriers* bars, uint32_t tmem, int64_t g0,
                           int64_t g1) {
  volatile int* abort = &bars->abort;
  const uint32_t idesc_qk = umma_idesc_f16(t.ab_fmt, kBM, kBN, 0, 0);
  const uint32_t idesc_pv = umma_idesc_f16(t.ab_fmt, kBM, kD, 0, 1);
  const uint32_t q_base = smem_u32(smem + kOffQ);
  const uint32_t kv_base = smem_u32(smem + kOffKV);
  const uint32_t p_base = smem_u32(smem + kOffP);
  int64_t i = 0;    // tiles consumed by this CTA
  int seg = 0;
  bool ok = true;
  auto issue_qk = [&](int64_t ti) {
    const int stage = static_cast<int>(ti % kStages);
    const uint32_t buf = static_cast<uint32_t>(ti & 1);
    const uint32_t kst = kv_base + stage * kStageBytes;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t d_tmem = tmem + kColS + (buf * 2 + mt) * kBN;
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        const uint32_t half = ks >> 2, off = (ks & 3) * 32;
        const uint64_t a = umma_desc_sw128(q_base + (mt * 2 + half) * kQHalf + off, 16, 1024);
        const uint64_t b = umma_desc_sw128(kst + half * kKVHalf + off, 16, 1024);
        umma_f16_ss(d_tmem, a, b, idesc_qk, ks > 0 ? 1u : 0u);
      }
    }
    umma_commit(&bars->s_full[buf]);
  };
  for (int64_t g = g0; g < g1 && ok;) {
    const PairInfo pi = pair_info(t, pair_of(t, g));
    const int64_t e = min(g1, pi.end);
    if (!bounded_wait(&bars->q_full, static_cast<uint32_t>(seg) & 1u, abort)) { ok = false; break; }
    tc_fence_after();
    // first tile of the segment
    if (!bounded_wait(&bars->kv_full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u, abort)) {
      ok = false;
      break;
    }
    tc_fence_after();
    issue_qk(i);
    const int64_t i_first = i;
    for (; g < e; ++g, ++i) {
      if (g + 1 < e) {
        const int64_t n = i + 1;
        if (!bounded_wait(&bars->kv_full[n % kStages], static_cast<uint32_t>(n / kStages) & 1u, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_qk(n);
      }
      const uint32_t buf = static_cast<uint32_t>(i & 1);
      if (!bounded_wait(&bars->p_full[buf], static_cast<uint32_t>(i >> 1) & 1u, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int stage = static_cast<int>(i % kStages);
      const uint32_t vst = kv_base + stage * kStageBytes + 2 * kKVHalf;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t d_tmem = tmem + kColO + mt * kD;
        const uint32_t pa = p_base + (buf * 2 + mt) * kPTile;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          const uint64_t a = umma_desc_sw128(pa + ks * 32, 16, 1024);
          // V tile: MN-major (d contiguous); d halves 8 KB apart, 8-row groups 1 KB apart
          const uint64_t b = umma_desc_sw128(vst + ks * 2048, kKVHalf, 1024);
          umma_f16_ss(d_tmem, a, b, idesc_pv, (i > i_first || ks > 0) ? 1u : 0u);
        }
      }
      umma_commit(&bars->p_free[buf]);
      umma_commit(&bars->kv_empty[stage]);
    }
    ++seg;
  }
  // all MMAs complete before TMEM is released
  umma_commit(&bars->drain);
  drain_wait(&bars->drain, 0);
}

template <int ANCW>
__device__ __forceinline__ bool anc_bit(const uint32_t (&anc)[ANCW], int t) {
  uint32_t w = 0;
#pragma unroll
  for (int k = 0; k < ANCW; ++k)
    if ((t >> 5) == k) w = anc[k];
  return (w >> (t & 31)) & 1u;
}

// All 32 lanes wait; the result is the same on every lane.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = bounded_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

template <int ANCW>
__device__ void softmax_epilogue(const TcArgs& t, uint8_t* smem, Barriers* bars, uint32_t tmem, int64_t g0,
                                 int64_t g1, int64_t T, int cta) {
  const AttnArgs& a = t.a;
  volatile int* abort = &bars->abort;
  const int wg = (threadIdx.x >> 7) - 1;       // 0 or 1: M-tile
  const int r = threadIdx.x & 127;              // row within the M-tile = TMEM lane
  const int wq = (threadIdx.x >> 5) & 3;        // warp quarter: TMEM lanes 32*wq..
  const int lane = threadIdx.x & 31;
  const int wslot = wg * 4 + wq;                // softmax warp 0..7
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  uint8_t* q_tile = smem + kOffQ + wg * 2 * kQHalf;
  const int R = a.group * a.n;
  const float sl2 = a.scale_log2;
  const int qrow = wg * kBM + r;                // row within the pair's 256
  int64_t i = 0;
  for (int64_t g = g0; g < g1;) {
    const int p = pair_of(t, g);
    const PairInfo pi = pair_info(t, p);
    const int64_t e = min(g1, pi.end);
    const int64_t i_first = i;
    const int pr = pi.qg * kQRows + qrow;  // packed row
    const bool row_ok = pr < R;
    const int gq = row_ok ? pr / a.n : 0;
    const int node = row_ok ? pr % a.n : 0;
    const int h = pi.kvh * a.group + gq;
    const int P = pi.L - a.n;
    const bool len_ok = pi.L >= a.n;

    // ---- Q row -> shared memory (SW128 K-major), then hand it to the MMA warp
    {
      const uint4* src = reinterpret_cast<const uint4*>(
          static_cast<const __nv_bfloat16*>(a.q) + static_cast<int64_t>(pi.b) * a.q_sb +
          static_cast<int64_t>(h) * a.q_sh + static_cast<int64_t>(node) * a.q_sn);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = row_ok ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(q_tile + (c >> 3) * kQHalf + sw128(r, c & 7)) = v;
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
    if (row_ok && len_ok) {
      if (a.mask_kind == GORGON_MASK_PARENTS) {
        const int32_t* par = a.parents + static_cast<int64_t>(pi.b) * a.par_sb;
        int cur = node;
        for (int hop = -1; hop < a.max_depth && cur >= 0; ++hop) {
          if (cur >= a.n) {
            raise_device_error(a.err, kErrBadParent);
            break;
          }
#pragma unroll
          for (int k = 0; k < ANCW; ++k)
            if ((cur >> 5) == k) anc[k] |= 1u << (cur & 31);
          cur = par[cur];
        }
      } else {
        const uint8_t* mrow =
            a.mask + static_cast<int64_t>(pi.b) * a.mask_sb + static_cast<int64_t>(node) * a.mask_sn;
        for (int j = 0; j < a.n; ++j)
          if (mrow[j]) {
#pragma unroll
            for (int k = 0; k < ANCW; ++k)
              if ((j >> 5) == k) anc[k] |= 1u << (j & 31);
          }
      }
    }
    if (!len_ok && qrow == 0) raise_device_error(a.err, kErrBadSeqlen);

    float m_used = -INFINITY, l = 0.f;
    for (; g < e; ++g, ++i) {
      const uint32_t buf = static_cast<uint32_t>(i & 1);
      if (!warp_wait(&bars->s_full[buf], static_cast<uint32_t>(i >> 1) & 1u, abort)) return;
      tc_fence_after();
      float x[kBN];
      {
        uint32_t r0[32], r1[32];
        const uint32_t s_addr = lane_base + kColS + (buf * 2 + wg) * kBN;
        tmem_ld32(s_addr, r0);
        tmem_ld32(s_addr + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x[c] = __uint_as_float(r0[c]);
          x[32 + c] = __uint_as_float(r1[c]);
        }
      }
      const int c0 = static_cast<int>(g - pi.start) * kBN;
      float tmax = -INFINITY;
      if (len_ok && c0 + kBN <= P) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          x[c] *= sl2;
          tmax = fmaxf(tmax, x[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int col = c0 + c;
          const int tt = col - P;
          const bool vis = len_ok && col < pi.L && (tt < 0 || anc_bit<ANCW>(anc, tt));
          x[c] = vis ? x[c] * sl2 : -INFINITY;
          tmax = fmaxf(tmax, x[c]);
        }
      }
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
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      float sum = 0.f;
      uint32_t packed[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = ex2_approx(x[c] - mb);
        const float p1 = ex2_approx(x[c + 1] - mb);
        sum += p0 + p1;
        if (t.ab_fmt) {
          const __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
          packed[c >> 1] = *reinterpret_cast<const uint32_t*>(&v2);
        } else {
          const __half2 v2 = __floats2half2_rn(p0, p1);
          packed[c >> 1] = *reinterpret_cast<const uint32_t*>(&v2);
        }
      }
      l = l * alpha + sum;
      // this P buffer was last read by the P.V MMA of tile i - 2
      if (i >= 2 && !warp_wait(&bars->p_free[buf], static_cast<uint32_t>((i - 2) >> 1) & 1u, abort)) return;
      // rescale O (warp-uniform) once the P.V of tile i - 1 has landed
      if (__any_sync(0xffffffffu, need)) {
        const int64_t pv = i - 1;
        if (!warp_wait(&bars->p_free[pv & 1], static_cast<uint32_t>(pv >> 1) & 1u, abort)) return;
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
      // P row -> shared memory (SW128 K-major, 64 columns = one 128-byte row)
      uint8_t* pt = smem + kOffP + (buf * 2 + wg) * kPTile;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        *reinterpret_cast<uint4*>(pt + sw128(r, c)) =
            make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[buf]);
    }

    // ---- epilogue: O / l for this row, once the last P.V has landed
    const int64_t lastv = i - 1;
    if (!warp_wait(&bars->p_free[lastv & 1], static_cast<uint32_t>(lastv >> 1) & 1u, abort)) return;
    tc_fence_after();
    const bool whole = pi.start >= g0 && pi.end <= g1;
    const int64_t orow = (static_cast<int64_t>(pi.b) * a.hq + h) * a.n + node;
    const int64_t ob = static_cast<int64_t>(pi.b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh +
                       static_cast<int64_t>(node) * a.o_sn;
    const uint32_t o_addr = lane_base + kColO + wg * kD;
    const float inv = 1.f / l;  // l == 0: no visible key, NaN like softmax
    const float lse2 = (l > 0.f) ? m_used + __log2f(l) : -INFINITY;
    if (whole) {
#pragma unroll
      for (int ch = 0; ch < kD / 32; ++ch) {
        uint32_t ov[32];
        tmem_ld32(o_addr + ch * 32, ov);
        tmem_wait_ld();
        if (row_ok) {
          if (t.out_vec) {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) + ob + ch * 32;
#pragma unroll
            for (int c = 0; c < 32; c += 8) {
              uint32_t w[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const __nv_bfloat162 v2 = __floats2bfloat162_rn(__uint_as_float(ov[c + 2 * u]) * inv,
                                                                __uint_as_float(ov[c + 2 * u + 1]) * inv);
                w[u] = *reinterpret_cast<const uint32_t*>(&v2);
              }
              *reinterpret_cast<uint4*>(dst + c) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              store_as(a.out, a.out_dtype, ob + ch * 32 + c, __uint_as_float(ov[c]) * inv);
          }
        }
      }
      if (row_ok && a.lse) a.lse[orow] = lse2 * 0.6931471805599453f;
      continue;
    }
    // partial: slot 0 when this piece of the pair starts the CTA's range, else slot 1
    const int which = (pi.start <= g0) ? 0 : 1;
    const int64_t slot = static_cast<int64_t>(cta) * 2 + which;
    float* po = t.part_o + (slot * kQRows + qrow) * kD;
    const bool any = l > 0.f;
#pragma unroll
    for (int ch = 0; ch < kD / 32; ++ch) {
      uint32_t ov[32];
      tmem_ld32(o_addr + ch * 32, ov);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<float4*>(po + ch * 32 + c) =
            make_float4(any ? __uint_as_float(ov[c]) * inv : 0.f, any ? __uint_as_float(ov[c + 1]) * inv : 0.f,
                        any ? __uint_as_float(ov[c + 2]) * inv : 0.f, any ? __uint_as_float(ov[c + 3]) * inv : 0.f);
    }
    t.part_lse[slot * kQRows + qrow] = lse2;
    __threadfence();
    __syncwarp();
    // per-warp arrival count: the warp that completes the set of parts merges them
    const int64_t first = cta_of(pi.start, T, t.grid);
    const int64_t last = cta_of(pi.end - 1, T, t.grid);
    int is_last = 0;
    if (lane == 0) {
      const int prev = atomicAdd(t.counters + static_cast<int64_t>(p) * 8 + wslot, 1);
      is_last = prev == static_cast<int>(last - first);
    }
    is_last = __shfl_sync(0xffffffffu, is_last, 0);
    if (!is_last) continue;
    __threadfence();
    float M = -INFINITY;
    for (int64_t c = first; c <= last; ++c) {
      const int wh = (c == first && pi.start > range_start(c, T, t.grid)) ? 1 : 0;
      M = fmaxf(M, __ldcg(t.part_lse + (c * 2 + wh) * kQRows + qrow));
    }
    if (!row_ok) continue;
    if (M == -INFINITY) {
      for (int c = 0; c < kD; ++c) store_as(a.out, a.out_dtype, ob + c, NAN);
      if (a.lse) a.lse[orow] = -INFINITY;
      continue;
    }
    float wsum = 0.f;
    for (int64_t c = first; c <= last; ++c) {
      const int wh = (c == first && pi.start > range_start(c, T, t.grid)) ? 1 : 0;
      wsum += ex2_approx(__ldcg(t.part_lse + (c * 2 + wh) * kQRows + qrow) - M);
    }
    const float winv = 1.f / wsum;
    for (int ch = 0; ch < kD; ch += 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t c = first; c <= last; ++c) {
        const int wh = (c == first && pi.start > range_start(c, T, t.grid)) ? 1 : 0;
        const int64_t sl = c * 2 + wh;
        const float w = ex2_approx(__ldcg(t.part_lse + sl * kQRows + qrow) - M);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(t.part_o + (sl * kQRows + qrow) * kD + ch));
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      store_as(a.out, a.out_dtype, ob + ch, acc.x * winv);
      store_as(a.out, a.out_dtype, ob + ch + 1, acc.y * winv);
      store_as(a.out, a.out_dtype, ob + ch + 2, acc.z * winv);
      store_as(a.out, a.out_dtype, ob + ch + 3, acc.w * winv);
    }
    if (a.lse) a.lse[orow] = (M + __log2f(wsum)) * 0.6931471805599453f;
  }
}

template <int ANCW>
__global__ void __launch_bounds__(kThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
               const TcArgs t) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->q_full, 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 8);
      mbar_init(&bars->p_free[b], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  const int64_t T = total_tiles(t);
  const int64_t G = t.grid;
  const int64_t g0 = range_start(blockIdx.x, T, G);
  const int64_t g1 = range_start(blockIdx.x + 1, T, G);

  if (g0 < g1) {
    if (warp == 0) {
      if (lane == 0) producer(t, &kmap, &vmap, smem, bars, g0, g1);
    } else if (warp == 1) {
      if (lane == 0) mma_issuer(t, smem, bars, tmem, g0, g1);
    } else if (warp >= 4) {
      softmax_epilogue<ANCW>(t, smem, bars, tmem, g0, g1, T, blockIdx.x);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (bars->abort && threadIdx.x == 0) raise_device_error(t.a.err, kErrTimeout);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Varlen schedule: tile prefix over pairs (one thread; pairs are few).
__global__ void attn_tc_prologue(const TcArgs t) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
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
  int qgroups, pairs, tiles_per_pair, grid;
  bool varlen;
};

Plan make_plan(const AttnArgs& a) {
  Plan pl{};
  const int R = a.group * a.n;
  pl.qgroups = (R + kQRows - 1) / kQRows;
  pl.pairs = a.batch * a.hkv * pl.qgroups;
  pl.varlen = a.cu_seqlens != nullptr;
  const int sms = sm_count();
  if (pl.varlen) {
    pl.tiles_per_pair = 0;
    pl.grid = sms;
  } else {
    pl.tiles_per_pair = (a.kv_len + kBN - 1) / kBN;
    const int64_t T = static_cast<int64_t>(pl.pairs) * pl.tiles_per_pair;
    // at least 4 tiles per CTA so partials stay a small share of the work
    pl.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sms, (T + 3) / 4)));
  }
  return pl;
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct WsLayout {
  size_t counters, part_o, part_lse, tile_start, total;
};

WsLayout ws_layout(const Plan& pl) {
  WsLayout w{};
  size_t off = 0;
  w.counters = off;   off += align_up(static_cast<size_t>(pl.pairs) * 8 * sizeof(int));
  w.tile_start = off; off += align_up(static_cast<size_t>(pl.pairs + 1) * sizeof(int));
  w.part_lse = off;   off += align_up(static_cast<size_t>(pl.grid) * 2 * kQRows * sizeof(float));
  w.part_o = off;     off += align_up(static_cast<size_t>(pl.grid) * 2 * kQRows * kD * sizeof(float));
  w.total = off;
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

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
  *launches = pl.varlen ? 2 : 1;
}

int launch_attn_tc(const AttnArgs& a, int dtype, void* workspace, size_t ws_bytes, cudaStream_t st) {
  const Plan pl = make_plan(a);
  const WsLayout w = ws_layout(pl);
  if (!workspace || ws_bytes < w.total)
    return set_error(GORGON_ERR_WORKSPACE, "tcgen05 tree attention: workspace too small");
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(GORGON_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType tdt = dtype == GORGON_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
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
      const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kBN)};
      r = enc(maps[m], tdt, 3, const_cast<void*>(srcs[m]), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(a.kv_len),
                                  static_cast<cuuint64_t>(a.hkv), static_cast<cuuint64_t>(a.batch)};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss[m]) * 2, static_cast<cuuint64_t>(sh[m]) * 2,
                                     static_cast<cuuint64_t>(sb[m]) * 2};
      const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(kBN), 1, 1};
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
  t.ab_fmt = dtype == GORGON_BF16 ? 1 : 0;
  char* ws = static_cast<char*>(workspace);
  t.counters = reinterpret_cast<int*>(ws + w.counters);
  t.tile_start = reinterpret_cast<int*>(ws + w.tile_start);
  t.part_lse = reinterpret_cast<float*>(ws + w.part_lse);
  t.part_o = reinterpret_cast<float*>(ws + w.part_o);
  t.out_vec = a.out_dtype == GORGON_BF16 && aligned16(a.out) && a.o_sb % 8 == 0 && a.o_sh % 8 == 0 &&
              a.o_sn % 8 == 0;
  int rc = check_cuda(cudaMemsetAsync(t.counters, 0, static_cast<size_t>(pl.pairs) * 8 * sizeof(int), st),
                      "tcgen05 counters reset");
  if (rc) return rc;
  if (pl.varlen) {
    attn_tc_prologue<<<1, 32, 0, st>>>(t);
    rc = check_cuda(cudaGetLastError(), "tcgen05 prologue launch");
    if (rc) return rc;
  }
  auto kern = a.n <= 64 ? attn_tc_kernel<2> : attn_tc_kernel<8>;
  rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                  "tcgen05 smem attribute");
  if (rc) return rc;
  kern<<<pl.grid, kThreads, kSmemBytes, st>>>(kmap, vmap, t);
  return check_cuda(cudaGetLastError(), "tcgen05 tree attention launch");
}

}  // namespace gorgon
