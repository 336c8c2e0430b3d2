// Candidate-tree builder on the device: the per-head statistics and the tree
// assembly of build_candidate_tree (src/gorgon/inference/tree_candidates.py:
// 92-245, with _topk_per_head :42-81) for a batch of sequences, with no host
// synchronisation.  The reference runs both on the host: one softmax, one
// entropy `.item()` and one top-k per head, then Python loops over the nodes.
//
// cand_segment_kernel — one CTA per segment of a (sequence, level) row of
//   logits: 256 threads x 8 vectors of 16 bytes, all copied at once into
//   shared memory (cp.async).  Both passes then run as short loops over the
//   thread's own vectors: a CTA executes its code once, so straight-line
//   unrolled passes spent most of their time fetching instructions.  Pass 1:
//   every thread's online
//   (max m, Z = sum e^(x-m), T = sum e^(x-m) (x-m)) and its maximum.  A bound
//   follows from the thread maxima (warp w's k-th largest leaves k logits at
//   or above it, so the segment's top k are all >= the largest such value).
//   Pass 2 appends every logit at or above the bound to a
//   shared-memory buffer, from which one warp picks the segment's top k;
//   segments with more ties at the bound than the buffer holds merge
//   per-thread top-K lists instead.  Writes (m, Z, T) and the list.
// cand_merge_kernel — one warp per row: merges the segments' statistics
//   (entropy = ln Z - T / Z) and lists into the row's top k (descending;
//   equal values by ascending id, a total order independent of the thread
//   layout) and the softmax over them.
// cand_tree_kernel — one warp per sequence.  The reference's expansion, level
//   by level: a level's (parent, candidate) pairs are taken in the reference's
//   order (parents sorted by their own logit, descending and stable, when a
//   budget is set; candidates in top-k order), 32 at a time; each lane tests
//   its pair against the thresholds, a ballot gives every passing pair its
//   rank, and pairs are kept while the budget lasts.  Path probabilities and
//   thresholds are in double precision, as the reference's Python floats.
// head_segment_kernel — the heads' last Linear fused with the segment
//   statistics (gorgon_head_candidate_tree): the logits are computed from the
//   lm_head inputs and weights in the kernel and never stored.
#include <climits>
#include <cmath>
#include <cstdio>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace gorgon {


namespace {
using namespace sm100;

constexpr int kSegThreads = 256;                 // per segment CTA
constexpr int kSegWarps = kSegThreads / 32;
constexpr int kSegVecs = 8;                      // 16-byte vectors per thread
constexpr int kSegBuf = 1024;                    // logits at or above the bound kept per segment
template <typename T>
constexpr int seg_elems() { return kSegThreads * kSegVecs * (16 / static_cast<int>(sizeof(T))); }
constexpr float kLog2e = 1.4426950408889634f;

struct CandArgs {
  const void* logits;
  int64_t lsb, lsl;
  int batch, levels, vocab, top_k, kk;  // kk = min(top_k, vocab)
  int max_candidates;
  double threshold;
  int use_path, entropy_weighted;
  int cap;
  int segs;            // segments per row
  float* part_m;       // [rows * segs][3]: m, Z, T of each segment
  float* part_v;       // [rows * segs][K]: each segment's top K values ...
  int32_t* part_i;     // ... and ids
  int kmax;            // K, the list length of the launch
  int64_t* tokens;
  int32_t* parents;
  float* probs;
  int32_t* n_nodes;
  int32_t* topk_ids;
  float* topk_scores;
  float* topk_probs;
  float* entropy;
  uint32_t* err;
};

// Strict total order of (value, id): larger value first, equal values by
// smaller id; an empty slot (id < 0) comes last.
__device__ __forceinline__ bool ahead(float a, int ia, float b, int ib) {
  if (ib < 0) return ia >= 0;
  if (ia < 0) return false;
  return a > b || (a == b && ia < ib);
}

// Inserts (v, id) into a sorted register list of K entries (the last drops out).
template <int K>
__device__ __forceinline__ void list_insert(float (&kv)[K], int (&ki)[K], float v, int id) {
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const bool take = ahead(v, id, kv[j], ki[j]);
    const float tv = kv[j];
    const int ti = ki[j];
    kv[j] = take ? v : tv;
    ki[j] = take ? id : ti;
    v = take ? tv : v;
    id = take ? ti : id;
  }
}

// Merges the 32 lanes' sorted lists into the first K entries of the order,
// returned in lane 0's list (the other lanes' lists are consumed).
template <int K>
__device__ __forceinline__ void warp_merge(float (&kv)[K], int (&ki)[K]) {
  const int lane = threadIdx.x & 31;
  float ov[K];
  int oi[K];
#pragma unroll
  for (int r = 0; r < K; ++r) {
    float bv = kv[0];
    int bi = ki[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ahead(v2, i2, bv, bi)) {
        bv = v2;
        bi = i2;
      }
    }
    ov[r] = bv;
    oi[r] = bi;
    // the lane whose head won pops it (ids are unique, so exactly one lane)
    if (bi >= 0 && ki[0] == bi) {
#pragma unroll
      for (int j = 0; j + 1 < K; ++j) {
        kv[j] = kv[j + 1];
        ki[j] = ki[j + 1];
      }
      kv[K - 1] = -INFINITY;
      ki[K - 1] = -1;
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < K; ++r) {
      kv[r] = ov[r];
      ki[r] = oi[r];
    }
  }
}

// 16-byte copy from global to shared memory that bypasses registers (and L1).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Online softmax statistics of one thread.
struct Stats {
  float m = -INFINITY, z = 0.f, t = 0.f;
  __device__ __forceinline__ void rebase(float nm) {  // nm >= m
    if (z > 0.f) {
      const float d = m - nm;
      const float c = sm100::ex2_approx(d * kLog2e);
      t = c * (t + z * d);
      z *= c;
    }
    m = nm;
  }
  __device__ __forceinline__ void add(float x) {
    const float d = fmaxf(x - m, -1e30f);  // -inf logits add nothing (and no 0 * inf)
    const float e = sm100::ex2_approx(d * kLog2e);
    z += e;
    t = fmaf(e, d, t);
  }
  __device__ __forceinline__ void merge(const Stats& o) {
    if (o.z <= 0.f) return;
    if (z <= 0.f) {
      *this = o;
      return;
    }
    const float nm = fmaxf(m, o.m);
    const float d1 = m - nm, d2 = o.m - nm;
    const float c1 = sm100::ex2_approx(d1 * kLog2e), c2 = sm100::ex2_approx(d2 * kLog2e);
    t = c1 * (t + z * d1) + c2 * (o.t + o.z * d2);
    z = c1 * z + c2 * o.z;
    m = nm;
  }
};

// 16-byte streaming load that the compiler keeps where it is written, so a
// batch of them is in flight before the first is used.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The 16-byte vector of a row's logits that starts at element i0: one load
// when the row is 16-byte aligned and the vector lies inside it, else
// element by element with -inf past the end.
template <typename T>
__device__ __forceinline__ uint4 load_vec(const T* src, int i0, int V, bool aligned) {
  constexpr int kVec = 16 / sizeof(T);
  if (aligned && i0 + kVec <= V) return ld_stream(reinterpret_cast<const uint4*>(src + i0));
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if constexpr (sizeof(T) == 4) {
      w[q] = __float_as_uint(i0 + q < V ? Cvt<T>::to_f(src[i0 + q]) : -INFINITY);
    } else {
      const T lo = i0 + 2 * q < V ? src[i0 + 2 * q] : Cvt<T>::from_f(-INFINITY);
      const T hi = i0 + 2 * q + 1 < V ? src[i0 + 2 * q + 1] : Cvt<T>::from_f(-INFINITY);
      w[q] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
             (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// k-th largest (1 <= k <= 32) of the warp's 32 values: bitonic sort across
// the lanes, descending, then lane k - 1's value.
__device__ __forceinline__ float warp_kth_largest(float x, int k) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, x, stride);
      const bool lower = (lane & stride) == 0;  // first lane of the compared pair
      const bool desc = (lane & size) == 0;     // this run is sorted descending
      x = (lower == desc) ? fmaxf(x, y) : fminf(x, y);
    }
  }
  return __shfl_sync(0xffffffffu, x, k - 1);
}

template <typename T, int K>
__global__ void __launch_bounds__(kSegThreads, K <= 16 ? 2 : 1) cand_segment_kernel(const CandArgs a) {
  constexpr int kVec = 16 / sizeof(T);
  const int S = a.segs;
  const int row = blockIdx.x / S, seg = blockIdx.x - row * S;
  const int b = row / a.levels, l = row - b * a.levels;
  const T* src = static_cast<const T*>(a.logits) + static_cast<int64_t>(b) * a.lsb + static_cast<int64_t>(l) * a.lsl;
  const int V = a.vocab;
  const int e0 = seg * seg_elems<T>();
  const bool aligned = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_m[kSegWarps], s_z[kSegWarps], s_t[kSegWarps], s_bound[kSegWarps];
  __shared__ float s_kv[kSegWarps][K];
  __shared__ int s_ki[kSegWarps][K];
  __shared__ float s_bv[kSegBuf];
  __shared__ int s_bi[kSegBuf];
  __shared__ int s_count;
  if (threadIdx.x == 0) s_count = 0;

  // the whole segment in flight at once; vector u of this thread starts at
  // element i0(u) and lands in s_seg[u][thread] (past the row's end: -inf)
  __shared__ uint4 s_seg[kSegVecs][kSegThreads];
  auto i0_of = [&](int u) { return e0 + (u * kSegThreads + static_cast<int>(threadIdx.x)) * kVec; };
#pragma unroll
  for (int u = 0; u < kSegVecs; ++u) {
    const int i0 = i0_of(u);
    if (aligned && i0 + kVec <= V) cp_async16(&s_seg[u][threadIdx.x], src + i0);
    else s_seg[u][threadIdx.x] = load_vec<T>(src, i0, V, aligned);
  }
  cp_async_wait_all();  // each thread reads only its own vectors: no CTA barrier needed

  // ---- pass 1: online softmax statistics (pairs in packed f32x2 arithmetic),
  // each vector's maximum, and this thread's maximum
  Stats st;
  uint64_t z2 = 0, t2 = 0;  // (0.f, 0.f): the sums of the current base st.m
  float vmax[kSegVecs];
  const uint64_t l2e2 = f2_pack(kLog2e, kLog2e);
#pragma unroll
  for (int u = 0; u < kSegVecs; ++u) {
    const uint4 raw = s_seg[u][threadIdx.x];
    const T* e = reinterpret_cast<const T*>(&raw);
    float x[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = fmaxf(Cvt<T>::to_f(e[j]), -1e30f);  // -inf adds nothing
    float cm = x[0];
#pragma unroll
    for (int j = 1; j < kVec; j += 2) cm = fmax3(cm, x[j], j + 1 < kVec ? x[j + 1] : x[j]);
    vmax[u] = cm;
    if (cm > st.m) {  // new base: fold the packed sums in, rescale
      float z0, z1, t0, t1;
      f2_unpack(z2, z0, z1);
      f2_unpack(t2, t0, t1);
      st.z += z0 + z1;
      st.t += t0 + t1;
      st.rebase(cm);
      z2 = t2 = 0;
    }
    const uint64_t nm2 = f2_pack(-st.m, -st.m);
#pragma unroll
    for (int j = 0; j < kVec; j += 2) {
      const uint64_t d = f2_add(f2_pack(x[j], x[j + 1]), nm2);
      float a0, a1;
      f2_unpack(f2_mul(d, l2e2), a0, a1);
      const uint64_t ee = f2_pack(ex2_approx(a0), ex2_approx(a1));
      z2 = f2_add(z2, ee);
      t2 = f2_fma(ee, d, t2);
    }
  }
  {
    float z0, z1, t0, t1;
    f2_unpack(z2, z0, z1);
    f2_unpack(t2, t0, t1);
    st.z += z0 + z1;
    st.t += t0 + t1;
  }
  float tmax = vmax[0];
#pragma unroll
  for (int u = 1; u < kSegVecs; ++u) tmax = fmaxf(tmax, vmax[u]);
  if (tmax <= -1e30f) tmax = -INFINITY;  // nothing but padding
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    other.z = __shfl_xor_sync(0xffffffffu, st.z, o);
    other.t = __shfl_xor_sync(0xffffffffu, st.t, o);
    st.merge(other);
  }
  // warp w's kk-th largest thread maximum leaves kk logits of warp w at or
  // above it (a thread without logits reports -inf)
  const float wk = warp_kth_largest(tmax, a.kk);
  if (lane == 0) {
    s_m[warp] = st.m;
    s_z[warp] = st.z;
    s_t[warp] = st.t;
    s_bound[warp] = wk;
  }
  __syncthreads();
  float bound = s_bound[0];
#pragma unroll
  for (int w = 1; w < kSegWarps; ++w) bound = fmaxf(bound, s_bound[w]);

  // ---- pass 2: the vectors whose maximum reaches the bound (rare) give their
  // logits at or above it to the buffer, read back from shared memory
  unsigned need = 0;
#pragma unroll
  for (int u = 0; u < kSegVecs; ++u) need |= (vmax[u] >= bound ? 1u : 0u) << u;
  while (need) {
    const int u = __ffs(need) - 1;
    need &= need - 1;
    const int i0 = i0_of(u);
    const T* e = reinterpret_cast<const T*>(&s_seg[u][threadIdx.x]);
    for (int j = 0; j < kVec; ++j) {
      const float xv = Cvt<T>::to_f(e[j]);
      if (xv >= bound && i0 + j < V) {
        const int slot = atomicAdd(&s_count, 1);
        if (slot < kSegBuf) {
          s_bv[slot] = xv;
          s_bi[slot] = i0 + j;
        }
      }
    }
  }
  __syncthreads();
  const int count = s_count;

  float kv[K];
  int ki[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    kv[j] = -INFINITY;
    ki[j] = -1;
  }
  if (count <= kSegBuf) {
    if (warp == 0) {  // one warp picks the top K of the buffer
      for (int j = lane; j < count; j += 32) list_insert<K>(kv, ki, s_bv[j], s_bi[j]);
      warp_merge<K>(kv, ki);
    }
  } else {
    // More ties at the bound than the buffer holds: per-thread lists over the
    // segment, merged per warp and then across warps.
#pragma unroll 1
    for (int u = 0; u < kSegVecs; ++u) {
      const int i0 = i0_of(u);
      const T* e = reinterpret_cast<const T*>(&s_seg[u][threadIdx.x]);
      for (int j = 0; j < kVec; ++j) {
        const float xv = Cvt<T>::to_f(e[j]);
        if (xv >= bound && i0 + j < V && (ki[K - 1] < 0 || xv > kv[K - 1])) list_insert<K>(kv, ki, xv, i0 + j);
      }
    }
    warp_merge<K>(kv, ki);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        s_kv[warp][j] = kv[j];
        s_ki[warp][j] = ki[j];
      }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < K; ++j) {
        kv[j] = lane < kSegWarps ? s_kv[lane][j] : -INFINITY;
        ki[j] = lane < kSegWarps ? s_ki[lane][j] : -1;
      }
      warp_merge<K>(kv, ki);
    }
  }
  if (warp != 0) return;

  // ---- this segment's statistics and list
  Stats all;
  if (lane < kSegWarps) {
    all.m = s_m[lane];
    all.z = s_z[lane];
    all.t = s_t[lane];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffffu, all.m, o);
    other.z = __shfl_xor_sync(0xffffffffu, all.z, o);
    other.t = __shfl_xor_sync(0xffffffffu, all.t, o);
    all.merge(other);
  }
  const int64_t p = blockIdx.x;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const float v = __shfl_sync(0xffffffffu, kv[j], 0);
    const int i = __shfl_sync(0xffffffffu, ki[j], 0);
    if (lane == j) {
      a.part_v[p * K + j] = v;
      a.part_i[p * K + j] = i;
    }
  }
  if (lane == 0) {
    a.part_m[p * 3] = all.m;
    a.part_m[p * 3 + 1] = all.z;
    a.part_m[p * 3 + 2] = all.t;
  }
}

// Per lane: statistics and a top-K list over segments [s0, s1) of the row
// whose partials start at p0.  Loads go out in batches (4 segments'
// statistics, then 8 list entries per lane) before any is used: with
// hundreds of segments per row (the fused heads) a load per loop trip would
// leave the warp waiting on memory each time.
template <int K>
__device__ __forceinline__ void scan_segments(const CandArgs& a, int64_t p0, int s0, int s1, Stats& all,
                                              float (&kv)[K], int (&ki)[K]) {
  const int lane = threadIdx.x & 31;
  for (int sg0 = s0; sg0 < s1; sg0 += 32 * 4) {
    float m[4], z[4], t[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int sg = sg0 + u * 32 + lane;
      const bool ok = sg < s1;
      m[u] = ok ? a.part_m[(p0 + sg) * 3] : -INFINITY;
      z[u] = ok ? a.part_m[(p0 + sg) * 3 + 1] : 0.f;
      t[u] = ok ? a.part_m[(p0 + sg) * 3 + 2] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      Stats o;
      o.m = m[u];
      o.z = z[u];
      o.t = t[u];
      all.merge(o);
    }
  }
  const int e1 = s1 * K;
  for (int e0 = s0 * K; e0 < e1; e0 += 32 * 8) {
    float v[8];
    int id[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * 32 + lane;
      const bool ok = e < e1;
      id[u] = ok ? a.part_i[p0 * K + e] : -1;
      v[u] = ok ? a.part_v[p0 * K + e] : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (ahead(v[u], id[u], kv[K - 1], ki[K - 1])) list_insert<K>(kv, ki, v[u], id[u]);
  }
}

template <int K>
__device__ __forceinline__ void empty_list(float (&kv)[K], int (&ki)[K]) {
#pragma unroll
  for (int j = 0; j < K; ++j) {
    kv[j] = -INFINITY;
    ki[j] = -1;
  }
}

__device__ __forceinline__ void warp_reduce_stats(Stats& all) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffffu, all.m, o);
    other.z = __shfl_xor_sync(0xffffffffu, all.z, o);
    other.t = __shfl_xor_sync(0xffffffffu, all.t, o);
    all.merge(other);
  }
}

// One warp, from every lane's partial statistics and top-K list: row `row`'s
// top k and entropy.  Writes them to the statistics outputs and returns this
// lane's entry (lane j < kk: the j-th candidate's id, logit and probability).
template <int K>
__device__ __forceinline__ float finish_row(const CandArgs& a, int row, Stats all, float (&kv)[K], int (&ki)[K],
                                            int& id_out, float& score_out, float& prob_out) {
  const int lane = threadIdx.x & 31;
  warp_reduce_stats(all);
  warp_merge<K>(kv, ki);
  // lane 0 holds the top K; hand entry j to lane j
  float myv = -INFINITY;
  int myi = -1;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const float v = __shfl_sync(0xffffffffu, kv[j], 0);
    const int i = __shfl_sync(0xffffffffu, ki[j], 0);
    if (lane == j) {
      myv = v;
      myi = i;
    }
  }
  const float top = __shfl_sync(0xffffffffu, myv, 0);
  const bool mine = lane < a.kk;
  // softmax over the kept logits, relative to the largest
  const float e = mine ? expf(myv - top) : 0.f;
  const float es = warp_sum(e);
  const int64_t o = static_cast<int64_t>(row) * a.top_k + lane;
  id_out = mine ? myi : -1;
  score_out = mine ? myv : -INFINITY;
  prob_out = mine ? e / es : 0.f;
  if (lane < a.top_k) {  // past min(top_k, vocab): empty slots
    a.topk_ids[o] = id_out;
    a.topk_scores[o] = score_out;
    a.topk_probs[o] = prob_out;
  }
  const float ent = all.z > 0.f ? logf(all.z) - all.t / all.z : 0.f;
  if (lane == 0) a.entropy[row] = ent;
  return ent;
}

// One warp: row `row`'s top k and entropy from all of its segments.
template <int K>
__device__ __forceinline__ float merge_row(const CandArgs& a, int row, int& id_out, float& score_out,
                                           float& prob_out) {
  Stats all;
  float kv[K];
  int ki[K];
  empty_list<K>(kv, ki);
  scan_segments<K>(a, static_cast<int64_t>(row) * a.segs, 0, a.segs, all, kv, ki);
  return finish_row<K>(a, row, all, kv, ki, id_out, score_out, prob_out);
}

__device__ __forceinline__ unsigned lanes_below() {
  unsigned r;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(r));
  return r;
}

// One warp builds one sequence's tree.  Shared memory: path probability per
// node, the current and next level's (node, logit) lists, the expansion order
// of the current level, and the sequence's per-level statistics (read once,
// coalesced, so the level loops wait on no global load).
// One warp per row: the row's statistics from its segments (all rows at once,
// rather than level after level inside the tree kernel, which measured 4x
// slower).
template <int K>
__global__ void __launch_bounds__(256) cand_merge_kernel(const CandArgs a) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.batch * a.levels) return;
  int id;
  float sc, pr;
  merge_row<K>(a, row, id, sc, pr);
}

// Rows with many segments (the fused heads: hundreds): one CTA per row, each
// of its 8 warps scans an eighth of the segments, warp 0 merges the eight
// results through shared memory.
constexpr int kWideMergeSegs = 64;  // segments per row above which the wide merge runs

template <int K>
__global__ void __launch_bounds__(256) cand_merge_wide_kernel(const CandArgs a) {
  __shared__ float s_m[8], s_z[8], s_t[8];
  __shared__ float s_v[8][K];
  __shared__ int s_i[8][K];
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.segs;
  const int per = (S + 7) / 8;
  const int s0 = min(S, warp * per), s1 = min(S, s0 + per);
  Stats st;
  float kv[K];
  int ki[K];
  empty_list<K>(kv, ki);
  scan_segments<K>(a, static_cast<int64_t>(row) * S, s0, s1, st, kv, ki);
  warp_reduce_stats(st);
  warp_merge<K>(kv, ki);
  if (lane == 0) {
    s_m[warp] = st.m;
    s_z[warp] = st.z;
    s_t[warp] = st.t;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      s_v[warp][j] = kv[j];
      s_i[warp][j] = ki[j];
    }
  }
  __syncthreads();
  if (warp != 0) return;
  Stats all;
  if (lane < 8) {
    all.m = s_m[lane];
    all.z = s_z[lane];
    all.t = s_t[lane];
  }
  empty_list<K>(kv, ki);
  for (int e = lane; e < 8 * K; e += 32) {
    const int w = e / K, j = e - w * K;
    if (ahead(s_v[w][j], s_i[w][j], kv[K - 1], ki[K - 1])) list_insert<K>(kv, ki, s_v[w][j], s_i[w][j]);
  }
  int id;
  float sc, pr;
  finish_row<K>(a, row, all, kv, ki, id, sc, pr);
}

// ------------------------------------------------------------ fused heads
// head_segment_kernel — the last Linear of every Medusa head fused with the
// segment statistics: CTA (segment s, level l) computes the logits of vocab
// rows [R s, R s + R) of head l (R <= 256, chosen so that the launch is a
// whole number of waves of resident CTAs) for every sequence of the batch
// (at most 4) and leaves the same per-segment (m, Z, T) and top-K list as
// cand_segment_kernel, so the merge and tree kernels run unchanged.  The
// head inputs of level l (batch x hidden, 16-bit) sit in shared memory; each
// warp takes one weight row at a time, a lane holding 16 of its 16-byte
// vectors (the whole row of a 4096-wide head in flight per warp), and
// accumulates the batch's dot products in packed fp32 pairs.  Each logit is
// rounded to the head's output dtype before the statistics, as the logits of
// the Linear would be.  The weights stream from HBM once per launch; the
// logits never leave the SM.
constexpr int kHeadThreads = 256;
constexpr int kHeadWarps = kHeadThreads / 32;
constexpr int kHeadRows = 256;       // most vocab rows per segment
constexpr int kHeadCtasPerSm = 2;    // resident segment CTAs per SM (the launch bounds)
constexpr int kHeadChunk = 16;       // 16-byte weight vectors per lane in flight
constexpr int kHeadMaxBatch = 4;
constexpr int kHeadMaxLevels = 64;
constexpr int kHeadMaxHidden = 8192;

struct HeadArgs {
  const void* x;  // [batch, levels, hidden]
  int64_t xsb, xsl;
  const void* w[kHeadMaxLevels];  // per level: [vocab, hidden], rows wsv elements apart
  int64_t wsv;
  int hidden;       // a multiple of 8
  int seg_rows;     // vocab rows per segment (<= kHeadRows)
  int logit_dtype;  // rounding of each logit
};

__device__ __forceinline__ float round_logit(float x, int dt) {
  if (dt == GORGON_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dt == GORGON_F16) return __half2float(__float2half_rn(x));
  return x;
}

// Eight 16-bit values -> four packed fp32 pairs (element order kept).
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, uint64_t (&p)[4]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      p[k] = sm100::f2_pack(__uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xffff0000u));
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      p[k] = sm100::f2_pack(f.x, f.y);
    }
  }
}

template <typename T, int NB, int K>
__global__ void __launch_bounds__(kHeadThreads, kHeadCtasPerSm) head_segment_kernel(const CandArgs a, const HeadArgs h) {
  extern __shared__ uint4 s_x[];  // [NB][hidden / 8]
  __shared__ float s_lg[NB][kHeadRows];
  const int S = a.segs;
  const int seg = blockIdx.x, l = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H8 = h.hidden >> 3;
  const int B = a.batch;
  for (int i = threadIdx.x; i < NB * H8; i += kHeadThreads) {
    const int b = i / H8, j = i - b * H8;
    s_x[i] = b < B ? *reinterpret_cast<const uint4*>(static_cast<const T*>(h.x) + b * h.xsb + l * h.xsl + j * 8)
                   : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const T* W = static_cast<const T*>(h.w[l]);
  const int v0 = seg * h.seg_rows;
  const int nrows = min(h.seg_rows, a.vocab - v0);
  for (int r = warp; r < nrows; r += kHeadWarps) {
    const uint4* wrow = reinterpret_cast<const uint4*>(W + static_cast<int64_t>(v0 + r) * h.wsv);
    uint64_t acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0;  // (0.f, 0.f)
    for (int j0 = 0; j0 < H8; j0 += 32 * kHeadChunk) {
      uint4 wv[kHeadChunk];
#pragma unroll
      for (int u = 0; u < kHeadChunk; ++u) {
        const int j = j0 + u * 32 + lane;
        wv[u] = j < H8 ? ld_stream(wrow + j) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kHeadChunk; ++u) {
        const int j = j0 + u * 32 + lane;
        if (j < H8) {
          uint64_t wp[4];
          unpack8<T>(wv[u], wp);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            uint64_t xp[4];
            unpack8<T>(s_x[b * H8 + j], xp);
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[b] = sm100::f2_fma(wp[k], xp[k], acc[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float lo, hi;
      sm100::f2_unpack(acc[b], lo, hi);
      const float s = warp_sum(lo + hi);
      if (lane == 0) s_lg[b][r] = round_logit(s, h.logit_dtype);
    }
  }
  __syncthreads();
  if (warp >= B) return;
  // warp b: the segment's statistics and top K for sequence b
  const int b = warp;
  const float* lg = s_lg[b];
  float mx = -INFINITY;
  for (int i = lane; i < nrows; i += 32) mx = fmaxf(mx, lg[i]);
  Stats st;
  if (mx > -INFINITY) {
    st.rebase(mx);
    for (int i = lane; i < nrows; i += 32) st.add(lg[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    other.z = __shfl_xor_sync(0xffffffffu, st.z, o);
    other.t = __shfl_xor_sync(0xffffffffu, st.t, o);
    st.merge(other);
  }
  float kv[K];
  int ki[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    kv[j] = -INFINITY;
    ki[j] = -1;
  }
  for (int i = lane; i < nrows; i += 32) list_insert<K>(kv, ki, lg[i], v0 + i);
  warp_merge<K>(kv, ki);
  if (lane == 0) {
    const int64_t p = (static_cast<int64_t>(b) * a.levels + l) * S + seg;
    a.part_m[p * 3] = st.m;
    a.part_m[p * 3 + 1] = st.z;
    a.part_m[p * 3 + 2] = st.t;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      a.part_v[p * K + j] = kv[j];
      a.part_i[p * K + j] = ki[j];
    }
  }
}

__global__ void __launch_bounds__(32) cand_tree_kernel(const CandArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int cap = a.cap;
  double* path = reinterpret_cast<double*>(smem);
  int* lvl_node = reinterpret_cast<int*>(path + cap);               // [2][cap]
  float* lvl_score = reinterpret_cast<float*>(lvl_node + 2 * cap);  // [2][cap]
  int* order = reinterpret_cast<int*>(lvl_score + 2 * cap);         // [cap]
  const int LK = a.levels * a.top_k;
  int* s_ids = order + cap;                                          // [levels][top_k]
  float* s_score = reinterpret_cast<float*>(s_ids + LK);
  float* s_prob = s_score + LK;
  float* s_ent = s_prob + LK;                                        // [levels]
  const int b = blockIdx.x, lane = threadIdx.x;
  {
    const int64_t base = static_cast<int64_t>(b) * LK;
    for (int j = lane; j < LK; j += 32) {
      s_ids[j] = a.topk_ids[base + j];
      s_score[j] = a.topk_scores[base + j];
      s_prob[j] = a.topk_probs[base + j];
    }
    for (int j = lane; j < a.levels; j += 32) s_ent[j] = a.entropy[static_cast<int64_t>(b) * a.levels + j];
    __syncwarp();
  }
  const int kk = a.kk;
  const bool thr_on = a.threshold > 0.0;
  int64_t* tokens = a.tokens + static_cast<int64_t>(b) * cap;
  int32_t* parents = a.parents + static_cast<int64_t>(b) * cap;
  float* probs = a.probs + static_cast<int64_t>(b) * cap;
  // the level's threshold: scaled by 1 - entropy / ln(top_k) when entropy-weighted
  auto level_threshold = [&](int l) -> double {
    if (thr_on && a.entropy_weighted) {
      const double max_ent = a.top_k > 1 ? log(static_cast<double>(a.top_k)) : 1.0;
      const double ent = static_cast<double>(s_ent[l]);
      return a.threshold * (1.0 - ent / max_ent);
    }
    return a.threshold;
  };
  int n = 0;  // nodes so far
  int budget = a.max_candidates < 0 ? INT_MAX : a.max_candidates;
  bool overflow = false;  // the capacity, not the budget, cut a level
  // Keeps the passing pairs of one 32-pair chunk, in lane order, while the
  // budget and the capacity last.  Returns how many were kept; `slot` is this
  // lane's rank among them (-1 if its pair is not kept).
  auto take = [&](bool pass, int& slot) -> int {
    const unsigned bal = __ballot_sync(0xffffffffu, pass);
    const int pos = __popc(bal & lanes_below());
    const int want = __popc(bal);
    const int room = cap - n;
    const int lim = budget < room ? budget : room;
    if (want > lim && room < budget) overflow = true;
    slot = (pass && pos < lim) ? pos : -1;
    const int cnt = want < lim ? want : lim;
    n += cnt;
    budget -= cnt;
    return cnt;
  };

  // ---- level 0: head 0's candidates become roots (tree_candidates.py:149-172)
  int cur = 0, cur_n = 0;
  {
    const double thr = level_threshold(0);
    const int s0 = 0;
    for (int base = 0; base < kk && budget > 0; base += 32) {
      const int i = base + lane;
      const bool valid = i < kk;
      const float pr = valid ? s_prob[s0 + i] : 0.f;
      const bool pass = valid && !(thr_on && static_cast<double>(pr) < thr);
      const int n0 = n;
      int slot;
      const int cnt = take(pass, slot);
      if (slot >= 0) {
        const int node = n0 + slot;
        tokens[node] = s_ids[s0 + i];
        parents[node] = -1;
        probs[node] = pr;
        path[node] = static_cast<double>(pr);
        lvl_node[cur * cap + cur_n + slot] = node;
        lvl_score[cur * cap + cur_n + slot] = s_score[s0 + i];
      }
      cur_n += cnt;
    }
  }
  __syncwarp();

  // ---- later levels: every node of the level above x the level's candidates (:175-226)
  for (int l = 1; l < a.levels && budget > 0; ++l) {
    const double thr = level_threshold(l);
    const int sl = l * a.top_k;
    // expansion order: by the parent's own logit, descending and stable, under a budget
    for (int p = lane; p < cur_n; p += 32) {
      int rank = p;
      if (a.max_candidates >= 0) {
        const float sp = lvl_score[cur * cap + p];
        rank = 0;
        for (int q = 0; q < cur_n; ++q) {
          const float sq = lvl_score[cur * cap + q];
          rank += (sq > sp || (sq == sp && q < p)) ? 1 : 0;
        }
      }
      order[rank] = p;
    }
    __syncwarp();
    const int nxt = cur ^ 1;
    int nxt_n = 0;
    const int total = cur_n * kk;
    for (int base = 0; base < total && budget > 0; base += 32) {
      const int j = base + lane;
      const bool valid = j < total;
      int i = 0, pnode = 0;
      float pr = 0.f;
      double cp = 0.0;
      if (valid) {
        const int pj = j / kk;
        i = j - pj * kk;
        pnode = lvl_node[cur * cap + order[pj]];
        pr = s_prob[sl + i];
        cp = path[pnode] * static_cast<double>(pr);
      }
      const bool pass = valid && !(thr_on && static_cast<double>(pr) < thr) &&
                        !(a.use_path && thr_on && cp < thr);
      const int n0 = n;
      int slot;
      const int cnt = take(pass, slot);
      if (slot >= 0) {
        const int node = n0 + slot;
        tokens[node] = s_ids[sl + i];
        parents[node] = pnode;
        probs[node] = pr;
        path[node] = cp;
        lvl_node[nxt * cap + nxt_n + slot] = node;
        lvl_score[nxt * cap + nxt_n + slot] = s_score[sl + i];
      }
      nxt_n += cnt;
    }
    __syncwarp();
    cur = nxt;
    cur_n = nxt_n;
  }

  if (lane == 0) {
    a.n_nodes[b] = n;
    if (overflow) raise_device_error(a.err, kErrCandCapacity);
  }
  for (int s = n + lane; s < cap; s += 32) {
    tokens[s] = -1;
    parents[s] = -1;
    probs[s] = 0.f;
  }
}

template <typename T, int K>
int launch_stats_k(const CandArgs& a, int rows, cudaStream_t st) {
  cand_segment_kernel<T, K><<<static_cast<unsigned>(rows) * a.segs, kSegThreads, 0, st>>>(a);
  return check_cuda(cudaGetLastError(), "candidate-tree segment launch");
}

template <int K>
int launch_merge_k(const CandArgs& a, cudaStream_t st) {
  if (a.segs > kWideMergeSegs)
    cand_merge_wide_kernel<K><<<static_cast<unsigned>(a.batch * a.levels), 256, 0, st>>>(a);
  else
    cand_merge_kernel<K><<<static_cast<unsigned>((a.batch * a.levels + 7) / 8), 256, 0, st>>>(a);
  return check_cuda(cudaGetLastError(), "candidate-tree merge launch");
}

template <typename T>
int launch_stats_t(const CandArgs& a, int rows, cudaStream_t st) {
  if (a.kmax == 4) return launch_stats_k<T, 4>(a, rows, st);
  if (a.kmax == 8) return launch_stats_k<T, 8>(a, rows, st);
  if (a.kmax == 16) return launch_stats_k<T, 16>(a, rows, st);
  return launch_stats_k<T, 32>(a, rows, st);
}

inline int list_len(int kk) { return kk <= 4 ? 4 : (kk <= 8 ? 8 : (kk <= 16 ? 16 : 32)); }
inline int64_t segments(int dtype, int64_t vocab) {
  const int64_t per = dtype == GORGON_F32 ? seg_elems<float>() : seg_elems<__nv_bfloat16>();
  return (vocab + per - 1) / per;
}

constexpr size_t kWsAlign = 256;
inline size_t ws_align(size_t x) { return (x + kWsAlign - 1) / kWsAlign * kWsAlign; }

// Segments per level of the fused heads: at least vocab / 256, rounded up so
// that segments x levels fills whole waves of resident CTAs (a launch of 6.8
// waves leaves most SMs idle for the last 0.8).
inline int64_t head_seg_rows(int64_t vocab, int64_t levels) {
  const int64_t slots = static_cast<int64_t>(sm_count()) * kHeadCtasPerSm;
  const int64_t min_segs = (vocab + kHeadRows - 1) / kHeadRows;
  const int64_t waves = (min_segs * levels + slots - 1) / slots;
  const int64_t segs = (waves * slots + levels - 1) / levels;
  const int64_t rows = (vocab + segs - 1) / segs;
  return rows < 1 ? 1 : rows;
}
inline int64_t head_segments(int64_t vocab, int64_t levels) {
  const int64_t rows = head_seg_rows(vocab, levels);
  return (vocab + rows - 1) / rows;
}

// Workspace: the per-row statistics (unless the caller takes them), then the
// segments' (m, Z, T) and top-K lists.
size_t workspace_bytes(const gorgon_candidate_tree_params* p, int64_t segs) {
  const size_t rows = static_cast<size_t>(p->batch) * static_cast<size_t>(p->levels);
  const size_t per = rows * static_cast<size_t>(p->top_k);
  const size_t parts = rows * static_cast<size_t>(segs);
  const size_t K = static_cast<size_t>(list_len(static_cast<int>(p->vocab < p->top_k ? p->vocab : p->top_k)));
  return ws_align(per * sizeof(int32_t)) + 2 * ws_align(per * sizeof(float)) + ws_align(rows * sizeof(float)) +
         ws_align(parts * 3 * sizeof(float)) + ws_align(parts * K * sizeof(float)) +
         ws_align(parts * K * sizeof(int32_t));
}

// Checks the tree parameters that both entry points share; 1 when there is
// nothing to do (an empty batch), 0 to go on, else the error code.
int check_tree(const gorgon_candidate_tree_params* p, int64_t segs, const char* who) {
  char msg[160];
  auto fail = [&](int code, const char* what) {
    snprintf(msg, sizeof(msg), "%s: %s", who, what);
    return set_error(code, msg);
  };
  if (!dtype_ok(p->dtype)) return fail(GORGON_ERR_INVALID, "unknown dtype");
  if (p->batch < 0 || p->levels < 0 || p->vocab < 0) return fail(GORGON_ERR_INVALID, "negative size");
  if (p->batch == 0) return 1;
  if (p->levels < 1) return fail(GORGON_ERR_INVALID, "levels must be >= 1");
  if (p->vocab < 1 || p->vocab > INT_MAX - 16) return fail(GORGON_ERR_INVALID, "vocab outside [1, 2^31)");
  if (p->top_k < 1 || p->top_k > 32) return fail(GORGON_ERR_UNSUPPORTED, "top_k must be in [1, 32]");
  if (p->max_nodes < 1 || p->max_nodes > 4096) return fail(GORGON_ERR_UNSUPPORTED, "max_nodes must be in [1, 4096]");
  if (p->levels > 64) return fail(GORGON_ERR_UNSUPPORTED, "levels must be <= 64");
  if (p->batch > INT_MAX / p->levels) return fail(GORGON_ERR_UNSUPPORTED, "batch * levels too large");
  if (!(p->confidence_threshold == p->confidence_threshold))
    return fail(GORGON_ERR_INVALID, "confidence_threshold is NaN");
  if (!p->tokens || !p->parents || !p->probs || !p->n_nodes) return fail(GORGON_ERR_INVALID, "null pointer");
  if (segs * p->batch * p->levels > INT_MAX) return fail(GORGON_ERR_UNSUPPORTED, "batch * levels * vocab too large");
  return 0;
}

// The kernels' arguments over a checked parameter block and its workspace.
CandArgs make_args(const gorgon_candidate_tree_params* p, int64_t segs, char* ws) {
  const int rows = static_cast<int>(p->batch * p->levels);
  const size_t per = static_cast<size_t>(rows) * static_cast<size_t>(p->top_k);
  CandArgs a{};
  a.logits = p->logits;
  a.lsb = p->logits_stride_b;
  a.lsl = p->logits_stride_l;
  a.batch = static_cast<int>(p->batch);
  a.levels = static_cast<int>(p->levels);
  a.vocab = static_cast<int>(p->vocab);
  a.top_k = p->top_k;
  a.kk = static_cast<int>(p->vocab < p->top_k ? p->vocab : p->top_k);
  a.max_candidates = p->max_candidates;
  a.threshold = static_cast<double>(p->confidence_threshold);
  a.use_path = p->use_path_confidence != 0;
  a.entropy_weighted = p->entropy_weighted != 0;
  a.cap = static_cast<int>(p->max_nodes);
  a.tokens = p->tokens;
  a.parents = p->parents;
  a.probs = p->probs;
  a.n_nodes = p->n_nodes;
  a.topk_ids = p->topk_ids ? p->topk_ids : reinterpret_cast<int32_t*>(ws);
  a.topk_scores = p->topk_scores ? p->topk_scores : reinterpret_cast<float*>(ws + ws_align(per * 4));
  a.topk_probs = p->topk_probs ? p->topk_probs : reinterpret_cast<float*>(ws + ws_align(per * 4) + ws_align(per * 4));
  a.entropy = p->entropy ? p->entropy
                         : reinterpret_cast<float*>(ws + ws_align(per * 4) + 2 * ws_align(per * 4));
  a.segs = static_cast<int>(segs);
  a.kmax = list_len(a.kk);
  const size_t parts = static_cast<size_t>(rows) * a.segs;
  char* q = ws + 3 * ws_align(per * 4) + ws_align(static_cast<size_t>(rows) * 4);
  a.part_m = reinterpret_cast<float*>(q);
  q += ws_align(parts * 3 * sizeof(float));
  a.part_v = reinterpret_cast<float*>(q);
  q += ws_align(parts * a.kmax * sizeof(float));
  a.part_i = reinterpret_cast<int32_t*>(q);
  a.err = device_error_word();
  return a;
}

// The segments' partials -> per-row statistics -> trees.
int launch_merge_and_tree(const CandArgs& a, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(a.cap) * (sizeof(double) + 2 * sizeof(int) + 2 * sizeof(float) + sizeof(int)) +
                      static_cast<size_t>(a.levels) * (static_cast<size_t>(a.top_k) * 12 + 4);
  int rc = a.kmax == 4 ? launch_merge_k<4>(a, st)
                        : a.kmax == 8 ? launch_merge_k<8>(a, st)
                                      : a.kmax == 16 ? launch_merge_k<16>(a, st) : launch_merge_k<32>(a, st);
  if (rc) return rc;
  if (smem > 48 * 1024) {
    rc = check_cuda(cudaFuncSetAttribute(cand_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)),
                    "candidate-tree smem attribute");
    if (rc) return rc;
  }
  cand_tree_kernel<<<static_cast<unsigned>(a.batch), 32, smem, st>>>(a);
  return check_cuda(cudaGetLastError(), "candidate-tree launch");
}

template <typename T, int NB, int K>
int launch_head_k(const CandArgs& a, const HeadArgs& h, cudaStream_t st) {
  auto kern = head_segment_kernel<T, NB, K>;
  const size_t smem = static_cast<size_t>(NB) * h.hidden * sizeof(T);
  if (smem > 48 * 1024) {
    const int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem)),
                              "fused head smem attribute");
    if (rc) return rc;
  }
  kern<<<dim3(static_cast<unsigned>(a.segs), static_cast<unsigned>(a.levels)), kHeadThreads, smem, st>>>(a, h);
  return check_cuda(cudaGetLastError(), "fused head segment launch");
}

template <typename T, int NB>
int launch_head_nb(const CandArgs& a, const HeadArgs& h, cudaStream_t st) {
  if (a.kmax == 4) return launch_head_k<T, NB, 4>(a, h, st);
  if (a.kmax == 8) return launch_head_k<T, NB, 8>(a, h, st);
  if (a.kmax == 16) return launch_head_k<T, NB, 16>(a, h, st);
  return launch_head_k<T, NB, 32>(a, h, st);
}

template <typename T>
int launch_head_t(const CandArgs& a, const HeadArgs& h, cudaStream_t st) {
  if (a.batch == 1) return launch_head_nb<T, 1>(a, h, st);
  if (a.batch == 2) return launch_head_nb<T, 2>(a, h, st);
  return launch_head_nb<T, 4>(a, h, st);
}

}  // namespace
}  // namespace gorgon

extern "C" size_t gorgon_candidate_tree_workspace_size(const gorgon_candidate_tree_params* p) {
  using namespace gorgon;
  if (!p || p->batch <= 0 || p->levels <= 0 || p->top_k <= 0 || p->vocab <= 0 || !dtype_ok(p->dtype)) return 0;
  return workspace_bytes(p, segments(p->dtype, p->vocab));
}

extern "C" int gorgon_candidate_tree(const gorgon_candidate_tree_params* p, void* workspace, size_t workspace_bytes_,
                                     void* stream) {
  using namespace gorgon;
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: params is null");
  const int64_t segs = p->vocab > 0 && dtype_ok(p->dtype) ? segments(p->dtype, p->vocab) : 0;
  int rc = check_tree(p, segs, "gorgon_candidate_tree");
  if (rc) return rc == 1 ? GORGON_OK : rc;
  if (!p->logits) return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: null pointer");
  if (!workspace || workspace_bytes_ < workspace_bytes(p, segs))
    return set_error(GORGON_ERR_WORKSPACE, "gorgon_candidate_tree: workspace too small");
  const CandArgs a = make_args(p, segs, static_cast<char*>(workspace));
  const int rows = a.batch * a.levels;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->dtype == GORGON_F32) rc = launch_stats_t<float>(a, rows, st);
  else if (p->dtype == GORGON_BF16) rc = launch_stats_t<__nv_bfloat16>(a, rows, st);
  else rc = launch_stats_t<__half>(a, rows, st);
  if (rc) return rc;
  return launch_merge_and_tree(a, st);
}

extern "C" size_t gorgon_head_candidate_tree_workspace_size(const gorgon_head_candidate_params* p) {
  using namespace gorgon;
  if (!p) return 0;
  const gorgon_candidate_tree_params* t = &p->tree;
  if (t->batch <= 0 || t->levels <= 0 || t->top_k <= 0 || t->vocab <= 0 || !dtype_ok(t->dtype)) return 0;
  return workspace_bytes(t, head_segments(t->vocab, t->levels));
}

extern "C" int gorgon_head_candidate_tree(const gorgon_head_candidate_params* p, void* workspace,
                                          size_t workspace_bytes_, void* stream) {
  using namespace gorgon;
  constexpr const char* kWho = "gorgon_head_candidate_tree";
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_head_candidate_tree: params is null");
  const gorgon_candidate_tree_params* t = &p->tree;
  const int64_t segs = t->vocab > 0 && t->levels > 0 ? head_segments(t->vocab, t->levels) : 0;
  int rc = check_tree(t, segs, kWho);
  if (rc) return rc == 1 ? GORGON_OK : rc;
  if (p->x_dtype != GORGON_BF16 && p->x_dtype != GORGON_F16)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_head_candidate_tree: hidden and lm_head must be bf16 or f16");
  if (t->batch > kHeadMaxBatch)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_head_candidate_tree: batch must be <= 4");
  if (p->hidden_size < 8 || p->hidden_size > kHeadMaxHidden || p->hidden_size % 8)
    return set_error(GORGON_ERR_UNSUPPORTED,
                     "gorgon_head_candidate_tree: hidden_size must be a multiple of 8 in [8, 8192]");
  if (!p->hidden || !p->lm_head) return set_error(GORGON_ERR_INVALID, "gorgon_head_candidate_tree: null pointer");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al16(p->hidden) || p->hidden_stride_b % 8 || p->hidden_stride_l % 8 || p->lm_head_stride_v % 8 ||
      p->lm_head_stride_v < p->hidden_size)
    return set_error(GORGON_ERR_INVALID,
                     "gorgon_head_candidate_tree: hidden and lm_head rows must be 16-byte aligned, strides "
                     "multiples of 8 elements, lm_head rows at least hidden_size apart");
  HeadArgs h{};
  for (int64_t l = 0; l < t->levels; ++l) {
    if (!p->lm_head[l] || !al16(p->lm_head[l]))
      return set_error(GORGON_ERR_INVALID, "gorgon_head_candidate_tree: an lm_head pointer is null or unaligned");
    h.w[l] = p->lm_head[l];
  }
  if (!workspace || workspace_bytes_ < workspace_bytes(t, segs))
    return set_error(GORGON_ERR_WORKSPACE, "gorgon_head_candidate_tree: workspace too small");
  h.x = p->hidden;
  h.xsb = p->hidden_stride_b;
  h.xsl = p->hidden_stride_l;
  h.wsv = p->lm_head_stride_v;
  h.hidden = static_cast<int>(p->hidden_size);
  h.seg_rows = static_cast<int>(head_seg_rows(t->vocab, t->levels));
  h.logit_dtype = t->dtype;
  const CandArgs a = make_args(t, segs, static_cast<char*>(workspace));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = p->x_dtype == GORGON_BF16 ? launch_head_t<__nv_bfloat16>(a, h, st) : launch_head_t<__half>(a, h, st);
  if (rc) return rc;
  return launch_merge_and_tree(a, st);
}
