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
#include <climits>
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace gorgon {

constexpr uint32_t kErrCandCapacity = 1u << 3;

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

// One warp: row `row`'s top k and entropy from its segments' lists and
// (m, Z, T).  Writes them to the statistics outputs and returns this lane's
// entry (lane j < kk: the j-th candidate's id, logit and probability).
template <int K>
__device__ __forceinline__ float merge_row(const CandArgs& a, int row, int& id_out, float& score_out,
                                           float& prob_out) {
  const int lane = threadIdx.x & 31;
  const int S = a.segs;
  const int64_t p0 = static_cast<int64_t>(row) * S;
  Stats all;
  for (int sg = lane; sg < S; sg += 32) {
    Stats o;
    o.m = a.part_m[(p0 + sg) * 3];
    o.z = a.part_m[(p0 + sg) * 3 + 1];
    o.t = a.part_m[(p0 + sg) * 3 + 2];
    all.merge(o);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stats other;
    other.m = __shfl_xor_sync(0xffffffffu, all.m, o);
    other.z = __shfl_xor_sync(0xffffffffu, all.z, o);
    other.t = __shfl_xor_sync(0xffffffffu, all.t, o);
    all.merge(other);
  }
  float kv[K];
  int ki[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    kv[j] = -INFINITY;
    ki[j] = -1;
  }
  const int n_entries = S * K;
  for (int e = lane; e < n_entries; e += 32) {
    const int id = a.part_i[p0 * K + e];
    if (id >= 0) list_insert<K>(kv, ki, a.part_v[p0 * K + e], id);
  }
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

}  // namespace
}  // namespace gorgon

// Workspace: the per-row statistics (unless the caller takes them), then the
// segments' (m, Z, T) and top-K lists.
extern "C" size_t gorgon_candidate_tree_workspace_size(const gorgon_candidate_tree_params* p) {
  using namespace gorgon;
  if (!p || p->batch <= 0 || p->levels <= 0 || p->top_k <= 0 || p->vocab <= 0 || !dtype_ok(p->dtype)) return 0;
  const size_t rows = static_cast<size_t>(p->batch) * static_cast<size_t>(p->levels);
  const size_t per = rows * static_cast<size_t>(p->top_k);
  const size_t parts = rows * static_cast<size_t>(segments(p->dtype, p->vocab));
  const size_t K = static_cast<size_t>(list_len(static_cast<int>(p->vocab < p->top_k ? p->vocab : p->top_k)));
  return ws_align(per * sizeof(int32_t)) + 2 * ws_align(per * sizeof(float)) + ws_align(rows * sizeof(float)) +
         ws_align(parts * 3 * sizeof(float)) + ws_align(parts * K * sizeof(float)) +
         ws_align(parts * K * sizeof(int32_t));
}

extern "C" int gorgon_candidate_tree(const gorgon_candidate_tree_params* p, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  using namespace gorgon;
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: params is null");
  if (!dtype_ok(p->dtype)) return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: unknown dtype");
  if (p->batch < 0 || p->levels < 0 || p->vocab < 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: negative size");
  if (p->batch == 0) return GORGON_OK;
  if (p->levels < 1) return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: levels must be >= 1");
  if (p->vocab < 1 || p->vocab > INT_MAX - 16)
    return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: vocab outside [1, 2^31)");
  if (p->top_k < 1 || p->top_k > 32)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_candidate_tree: top_k must be in [1, 32]");
  if (p->max_nodes < 1 || p->max_nodes > 4096)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_candidate_tree: max_nodes must be in [1, 4096]");
  if (p->levels > 64) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_candidate_tree: levels must be <= 64");
  if (p->batch > INT_MAX / p->levels)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_candidate_tree: batch * levels too large");
  if (!(p->confidence_threshold == p->confidence_threshold))
    return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: confidence_threshold is NaN");
  if (!p->logits || !p->tokens || !p->parents || !p->probs || !p->n_nodes)
    return set_error(GORGON_ERR_INVALID, "gorgon_candidate_tree: null pointer");
  if (segments(p->dtype, p->vocab) * p->batch * p->levels > INT_MAX)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_candidate_tree: batch * levels * vocab too large");
  const size_t need = gorgon_candidate_tree_workspace_size(p);
  if (!workspace || workspace_bytes < need)
    return set_error(GORGON_ERR_WORKSPACE, "gorgon_candidate_tree: workspace too small");
  const int rows = static_cast<int>(p->batch * p->levels);
  const size_t per = static_cast<size_t>(rows) * static_cast<size_t>(p->top_k);
  char* ws = static_cast<char*>(workspace);
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
  a.segs = static_cast<int>(segments(p->dtype, p->vocab));
  a.kmax = list_len(a.kk);
  {
    const size_t parts = static_cast<size_t>(rows) * a.segs;
    char* q = ws + 3 * ws_align(per * 4) + ws_align(static_cast<size_t>(rows) * 4);
    a.part_m = reinterpret_cast<float*>(q);
    q += ws_align(parts * 3 * sizeof(float));
    a.part_v = reinterpret_cast<float*>(q);
    q += ws_align(parts * a.kmax * sizeof(float));
    a.part_i = reinterpret_cast<int32_t*>(q);
  }
  a.err = device_error_word();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (p->dtype == GORGON_F32) rc = launch_stats_t<float>(a, rows, st);
  else if (p->dtype == GORGON_BF16) rc = launch_stats_t<__nv_bfloat16>(a, rows, st);
  else rc = launch_stats_t<__half>(a, rows, st);
  if (rc) return rc;
  const size_t smem = static_cast<size_t>(a.cap) * (sizeof(double) + 2 * sizeof(int) + 2 * sizeof(float) + sizeof(int)) +
                      static_cast<size_t>(a.levels) * (static_cast<size_t>(a.top_k) * 12 + 4);
  rc = a.kmax == 4 ? launch_merge_k<4>(a, st)
                    : a.kmax == 8 ? launch_merge_k<8>(a, st)
                                  : a.kmax == 16 ? launch_merge_k<16>(a, st) : launch_merge_k<32>(a, st);
  if (rc) return rc;
  if (smem > 48 * 1024) {
    rc = check_cuda(cudaFuncSetAttribute(cand_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)),
                    "candidate-tree smem attribute");
    if (rc) return rc;
  }
  cand_tree_kernel<<<static_cast<unsigned>(p->batch), 32, smem, st>>>(a);
  return check_cuda(cudaGetLastError(), "candidate-tree launch");
}
