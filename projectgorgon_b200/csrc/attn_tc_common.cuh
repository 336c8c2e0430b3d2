// Device helpers shared by the two tensor-core tree-attention kernels (one
// CTA per unit in attn_tc.cu, a CTA pair per unit in attn_pair.cu): tile
// constants, the SW128 shared-memory layout, output staging, packed-row
// cursors and the visibility words of masked tiles.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attn.cuh"
#include "sm100.cuh"

namespace gorgon {

namespace {

constexpr int kBM = 128;               // rows per MMA tile (per CTA)
constexpr int kD = 128;                // head_dim
constexpr uint32_t kQHalf = kBM * 128;  // 128 rows x 64 cols bf16 = 16 KB
constexpr int kOutBf16 = 1, kOutF16 = 2, kOutF32 = 3;  // 16-byte output rows of this dtype

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in an SW128 K-major
// tile whose rows are 128 bytes.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// Packed query row -> (query head within the kv group, tree node), advanced
// two rows at a time (the rows a half-warp visits in the coalesced Q load and
// output store).
struct RowCursor {
  int pr, gq, node;
  __device__ __forceinline__ RowCursor(int p, int n) : pr(p), gq(p / n), node(p - (p / n) * n) {}
  __device__ __forceinline__ void next2(int n) {
    pr += 2;
    node += 2;
    while (node >= n) {  // at most twice: n >= 1
      node -= n;
      ++gq;
    }
  }
};

// A softmax warp's 32 rows of its M-tile's Q buffer (two 4 KB pieces, one per
// d half) double as the warp's staging area for output rows: row rr (0..31)
// holds 16 chunks of 16 bytes in the same SW128 order as Q, so a thread
// writing its own row and a half-warp reading one row are both free of bank
// conflicts.
__device__ __forceinline__ uint8_t* stage_at(uint8_t* q_tile, int wq, int rr, int j) {
  return q_tile + (j >> 3) * kQHalf + sw128(static_cast<uint32_t>(wq * 32 + rr), static_cast<uint32_t>(j & 7));
}

__device__ __forceinline__ uint32_t pack16x2(float x, float y, bool bf16) {
  if (bf16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  const __half2 v = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Visibility of 64 consecutive key columns for one row: bit j is set when
// column (tree index o + j) is visible -- a prefix column (tree index < 0) or
// an ancestor of the row's node (bit set in anc).  Built once per masked
// tile with a funnel shift of the ancestor words, so that masking a column
// costs a constant-bit test instead of a run-time compare-and-select chain
// per column (the per-column form made the masked tile the slowest tile of
// a unit by several microseconds).
template <int ANCW>
__device__ __forceinline__ uint64_t vis_window(const uint32_t (&anc)[ANCW], int o) {
  if (o <= -64) return ~0ull;
  // word w of the extended bit array: all ones before the tree, 0 after the last word
  auto word = [&](int w) -> uint32_t {
    uint32_t r = w < 0 ? 0xffffffffu : 0u;
#pragma unroll
    for (int k = 0; k < ANCW; ++k) r = (w == k) ? anc[k] : r;
    return r;
  };
  const int w0 = o >> 5;  // floor(o / 32), also for negative o
  const int sh = o & 31;
  const uint64_t lo = static_cast<uint64_t>(word(w0)) | (static_cast<uint64_t>(word(w0 + 1)) << 32);
  const uint64_t hi = word(w0 + 2);
  return sh == 0 ? lo : (lo >> sh) | (hi << (64 - sh));
}

// Writes 32 finished output columns of one row in any output dtype or layout
// (the path for rows that are not 16-byte aligned).
__device__ __forceinline__ void store_cols32(const AttnArgs& a, int64_t ob, int col0, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 32; ++c) store_as(a.out, a.out_dtype, ob + col0 + c, v[c]);
}

// ---------------------------------------------------------------- waits
// Every wait of the tensor-core kernels is bounded by `limit_ns` of
// %globaltimer (wait_limit_ns() on the host, 2 s unless changed through
// gorgon_set_wait_limit_ns).  A wait that runs out sets the CTA's abort flag,
// which ends every other wait of the CTA; the kernel then drains its copies
// and MMAs, frees its tensor memory and raises kErrTimeout.
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit_ns) {
  return sm100::mbar_wait_ns(bar, parity, abort, limit_ns);
}

// Wait of a thread that does nothing else (the MMA issuers): spins on the
// non-blocking test so it resumes the moment the phase completes, instead of
// sleeping in try_wait.  Bounded like bounded_wait.  With `cluster`, the
// probe acquires at cluster scope (the arrivals come from the other CTA of a
// pair too).
template <bool kCluster = false>
__device__ __forceinline__ bool spin_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit_ns) {
  auto probe = [&]() { return kCluster ? sm100::mbar_test_wait_cluster(bar, parity) : sm100::mbar_test_wait(bar, parity); };
  if (probe()) return true;
  const uint64_t t0 = sm100::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (probe()) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (sm100::globaltimer_ns() - t0 > limit_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// Wait used on the way out: ignores the abort flag, gives up after 200 ms.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = sm100::globaltimer_ns();
  while (!sm100::mbar_try_wait(bar, parity)) {
    if (sm100::globaltimer_ns() - t0 > 200000000ull) break;
  }
}

// All 32 lanes wait; the result is the same on every lane.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit_ns) {
  const bool ok = bounded_wait(bar, parity, abort, limit_ns);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace
}  // namespace gorgon
