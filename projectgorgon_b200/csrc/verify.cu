// Fused tree verifier: argmax over the vocabulary for every needed logits row,
// draft match and longest-accepted-path selection, in one launch.
//
// Grid (n + 1, batch): CTA j computes the argmax of row prompt_len - 1 + j of
// sequence b with 16-byte vector loads, writes it to pred[b, j], and bumps a
// per-sequence arrival counter.  The CTA that arrives last for a sequence
// selects the winner, with no host synchronisation:
//
//   match(t)  = draft[t] == pred[row of parent(t)]   (root: row prompt_len - 1)
//   accepted  = match holds on t and every ancestor of t
//   winner    = among accepted nodes of greatest depth, the first in DFS
//               preorder (roots ascending, children in index order)
//
// which is the node where the reference's first longest accepted path ends
// (src/gorgon/inference/gorgon_loop.py:336-371: paths in DFS order, strict >
// keeps the earliest).  Two nodes of equal depth are ordered by walking both
// up to the level where their ancestors share a parent and comparing the two
// sibling indices there.  Nodes that never reach a root (a cycle) belong to no
// path, as in the reference's get_tree_paths, and are never accepted.
#include <climits>
#include <mutex>

#include "common.cuh"

namespace gorgon {
namespace {

constexpr int kThreads = 256;

struct VerifyArgs {
  const void* logits;
  int64_t lsb, lsr;
  int64_t rows, vocab;
  int n, prompt_len;
  const int32_t* draft;
  int64_t dsb;
  const int32_t* parents;
  int64_t psb;
  int32_t* pred;
  int32_t* accepted_len;
  int32_t* path;
  int32_t* bonus;
  int32_t* best_node;
  int32_t* hidden_row;
  int32_t* counters;
  uint32_t* err;
  int vec_ok;
};

// (v1, i1) ranks before (v2, i2): larger value first, NaN above everything,
// lower index on ties -- torch.argmax's choice.
__device__ __forceinline__ bool arg_better(float v1, int i1, float v2, int i2) {
  const bool n1 = isnan(v1), n2 = isnan(v2);
  if (n1 || n2) {
    if (n1 && n2) return i1 < i2;
    return n1;
  }
  if (v1 != v2) return v1 > v2;
  return i1 < i2;
}

// 16-bit logits: packed pair types and their NaN-propagating max.
template <typename T> struct Pair16;
template <> struct Pair16<__nv_bfloat16> {
  using P = __nv_bfloat162;
  static __device__ __forceinline__ P max_nan(P a, P b) { return __hmax2_nan(a, b); }
  static __device__ __forceinline__ float lo(P p) { return __low2float(p); }
  static __device__ __forceinline__ float hi(P p) { return __high2float(p); }
};
template <> struct Pair16<__half> {
  using P = __half2;
  static __device__ __forceinline__ P max_nan(P a, P b) { return __hmax2_nan(a, b); }
  static __device__ __forceinline__ float lo(P p) { return __low2float(p); }
  static __device__ __forceinline__ float hi(P p) { return __high2float(p); }
};

// Thread's argmax over its 16-byte chunks of a 16-bit row (chunks v, v +
// kThreads, ...; the caller handles the vocabulary tail).  Per chunk the 8
// values fold into one with packed NaN-propagating maxima; the thread keeps
// the largest chunk maximum and the first chunk that reached it (NaN above
// everything, ties to the earlier chunk), then reads that chunk again (an L2
// hit) for the first element equal to its maximum.  Same result as ranking
// every element with arg_better, at about one instruction per element pair.
template <typename T>
__device__ __forceinline__ void scan_chunks16(const uint4* __restrict__ rv, int64_t nvec, float& bv, int& bi) {
  using PT = Pair16<T>;
  using P = typename PT::P;
  float rm = -INFINITY;
  int64_t rc = -1;
  constexpr int U = 8;
  int64_t v = threadIdx.x;
  auto fold = [&](const uint4& raw, int64_t idx) {
    const P* p = reinterpret_cast<const P*>(&raw);
    const P m = PT::max_nan(PT::max_nan(p[0], p[1]), PT::max_nan(p[2], p[3]));
    const float a = PT::lo(m), b = PT::hi(m);
    const float cm = (isnan(a) || isnan(b)) ? NAN : fmaxf(a, b);
    const bool better = rc < 0 || (isnan(cm) ? !isnan(rm) : cm > rm);
    if (better) {
      rm = cm;
      rc = idx;
    }
  };
  for (; v + (U - 1) * kThreads < nvec; v += U * kThreads) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = __ldcs(rv + v + u * kThreads);
#pragma unroll
    for (int u = 0; u < U; ++u) fold(raw[u], v + u * kThreads);
  }
  for (; v < nvec; v += kThreads) fold(__ldcs(rv + v), v);
  if (rc < 0) return;
  const uint4 raw = rv[rc];
  const T* e = reinterpret_cast<const T*>(&raw);
  int q = 0;
  float x = rm;
#pragma unroll
  for (int k = 7; k >= 0; --k) {
    const float xk = Cvt<T>::to_f(e[k]);
    if (isnan(rm) ? isnan(xk) : xk == rm) {
      q = k;
      x = xk;
    }
  }
  const int idx = static_cast<int>(rc * 8 + q);
  if (arg_better(x, idx, bv, bi)) {
    bv = x;
    bi = idx;
  }
}

template <typename T>
__device__ __forceinline__ void scan_row(const T* __restrict__ row, int64_t vocab, bool vec_ok,
                                         float& bv, int& bi) {
  if constexpr (sizeof(T) == 2) {
    if (vec_ok) {
      const int64_t nvec = vocab / 8;
      scan_chunks16<T>(reinterpret_cast<const uint4*>(row), nvec, bv, bi);
      for (int64_t c = nvec * 8 + threadIdx.x; c < vocab; c += kThreads) {
        const float x = Cvt<T>::to_f(row[c]);
        if (arg_better(x, static_cast<int>(c), bv, bi)) { bv = x; bi = static_cast<int>(c); }
      }
      return;
    }
  }
  constexpr int EV = 16 / sizeof(T);
  int64_t start = 0;
  if (vec_ok) {
    const int64_t nvec = vocab / EV;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    constexpr int U = 8;
    int64_t v = threadIdx.x;
    for (; v + (U - 1) * kThreads < nvec; v += U * kThreads) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = __ldcs(rv + v + u * kThreads);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T* e = reinterpret_cast<const T*>(&raw[u]);
        const int base = static_cast<int>((v + u * kThreads) * EV);
#pragma unroll
        for (int q = 0; q < EV; ++q) {
          const float x = Cvt<T>::to_f(e[q]);
          if (arg_better(x, base + q, bv, bi)) { bv = x; bi = base + q; }
        }
      }
    }
    for (; v < nvec; v += kThreads) {
      const uint4 raw = __ldcs(rv + v);
      const T* e = reinterpret_cast<const T*>(&raw);
      const int base = static_cast<int>(v * EV);
#pragma unroll
      for (int q = 0; q < EV; ++q) {
        const float x = Cvt<T>::to_f(e[q]);
        if (arg_better(x, base + q, bv, bi)) { bv = x; bi = base + q; }
      }
    }
    start = nvec * EV;
  }
  for (int64_t c = start + threadIdx.x; c < vocab; c += kThreads) {
    const float x = Cvt<T>::to_f(row[c]);
    if (arg_better(x, static_cast<int>(c), bv, bi)) { bv = x; bi = static_cast<int>(c); }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) verify_kernel(const VerifyArgs a) {
  extern __shared__ int32_t sm[];
  __shared__ float red_v[kThreads / 32];
  __shared__ int red_i[kThreads / 32];
  __shared__ int s_last;

  const int j = blockIdx.x;
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(a.prompt_len) - 1 + j;
  const int np1 = a.n + 1;

  // ---- phase 1: argmax of one row ----
  if (r < a.rows) {
    float bv = -INFINITY;
    int bi = INT_MAX;
    const T* row = static_cast<const T*>(a.logits) + static_cast<int64_t>(b) * a.lsb + r * a.lsr;
    scan_row<T>(row, a.vocab, a.vec_ok != 0, bv, bi);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kThreads / 32; ++w)
        if (arg_better(red_v[w], red_i[w], bv, bi)) { bv = red_v[w]; bi = red_i[w]; }
      a.pred[static_cast<int64_t>(b) * np1 + j] = bi == INT_MAX ? -1 : bi;
    }
  } else if (threadIdx.x == 0) {
    a.pred[static_cast<int64_t>(b) * np1 + j] = -1;
  }

  // ---- arrival: the last CTA of sequence b goes on to select ----
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(a.counters + b, 1);
    s_last = (prev == np1 - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- phase 2: selection (one CTA per sequence) ----
  const int n = a.n;
  int32_t* s_par = sm;               // [n]
  int32_t* s_pred = s_par + n;       // [n + 1]
  int32_t* s_depth = s_pred + np1;   // [n]  hop depth if accepted, -1 otherwise
  int32_t* s_draft = s_depth + n;    // [n]
  __shared__ int s_best_depth;
  __shared__ int s_winner;
  const int32_t* par = a.parents + static_cast<int64_t>(b) * a.psb;
  const int32_t* drf = a.draft + static_cast<int64_t>(b) * a.dsb;
  for (int t = threadIdx.x; t < n; t += kThreads) {
    int p = par[t];
    if (p < -1 || p >= n) {
      raise_device_error(a.err, kErrBadVerifyInput);
      p = -2;  // marks a node outside every path
    }
    s_par[t] = p;
    s_draft[t] = drf[t];
  }
  for (int t = threadIdx.x; t < np1; t += kThreads) s_pred[t] = __ldcg(a.pred + static_cast<int64_t>(b) * np1 + t);
  if (threadIdx.x == 0) { s_best_depth = -1; s_winner = -1; }
  __syncthreads();

  // accepted iff every node on the chain up to a root matches its row
  for (int t = threadIdx.x; t < n; t += kThreads) {
    int u = t, depth = 0;
    bool ok = false;
    for (int hop = 0; hop <= n; ++hop) {
      const int p = s_par[u];
      if (p == -2) break;
      const int want = s_pred[p < 0 ? 0 : p + 1];
      if (want < 0 || want != s_draft[u]) break;
      if (p < 0) { ok = true; break; }  // reached a root with every node matching
      u = p;
      ++depth;
    }
    s_depth[t] = ok ? depth : -1;
    if (ok) atomicMax(&s_best_depth, depth);
  }
  __syncthreads();

  if (threadIdx.x == 0) {
    const int bd = s_best_depth;
    int win = -1;
    if (bd >= 0) {
      for (int t = 0; t < n; ++t) {
        if (s_depth[t] != bd) continue;
        if (win < 0) { win = t; continue; }
        // equal depth: climb both until they are siblings (or both roots)
        int x = t, y = win;
        while (s_par[x] != s_par[y]) { x = s_par[x]; y = s_par[y]; }
        if (x < y) win = t;
      }
    }
    s_winner = win;
    const int64_t ob = static_cast<int64_t>(b);
    int len = 0;
    if (win >= 0) {
      len = bd + 1;
      int u = win;
      for (int k = len - 1; k >= 0; --k) {
        a.path[ob * n + k] = u;
        u = s_par[u];
      }
    }
    a.accepted_len[ob] = len;
    a.best_node[ob] = win;
    a.bonus[ob] = s_pred[win >= 0 ? win + 1 : 0];
    if (a.hidden_row) a.hidden_row[ob] = win >= 0 ? a.prompt_len + win : a.prompt_len - 1;
  }
  __syncthreads();
  const int len = s_winner >= 0 ? s_best_depth + 1 : 0;
  for (int k = len + threadIdx.x; k < n; k += kThreads) a.path[static_cast<int64_t>(b) * n + k] = -1;
}

template <typename T>
int launch_verify_t(const VerifyArgs& a, int batch, cudaStream_t st) {
  const size_t smem = (static_cast<size_t>(a.n) * 4 + 1) * sizeof(int32_t);
  auto kern = verify_kernel<T>;
  if (smem > 48 * 1024) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)), "verify smem attribute");
    if (rc) return rc;
  }
  dim3 grid(a.n + 1, batch);
  kern<<<grid, kThreads, smem, st>>>(a);
  return check_cuda(cudaGetLastError(), "verify launch");
}

}  // namespace
}  // namespace gorgon

extern "C" size_t gorgon_verify_workspace_size(const gorgon_verify_params* p) {
  if (!p || p->batch <= 0) return 0;
  return static_cast<size_t>(p->batch) * sizeof(int32_t);
}

extern "C" int gorgon_verify(const gorgon_verify_params* p, void* workspace, size_t workspace_bytes,
                             void* stream) {
  using namespace gorgon;
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_verify: params is null");
  if (!dtype_ok(p->dtype)) return set_error(GORGON_ERR_INVALID, "gorgon_verify: unknown dtype");
  if (p->batch < 0 || p->rows < 0 || p->vocab < 0 || p->n < 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_verify: negative size");
  if (p->batch == 0) return GORGON_OK;
  if (p->n < 1 || p->n > 4096) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_verify: n must be in [1, 4096]");
  if (p->prompt_len < 1) return set_error(GORGON_ERR_INVALID, "gorgon_verify: prompt_len must be >= 1");
  if (p->vocab < 1 || p->vocab > INT_MAX - 16) return set_error(GORGON_ERR_INVALID, "gorgon_verify: vocab outside [1, 2^31)");
  if (p->rows < p->prompt_len) return set_error(GORGON_ERR_INVALID, "gorgon_verify: rows < prompt_len");
  if (p->batch > 65535) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_verify: batch > 65535");
  if (!p->logits || !p->draft || !p->parents || !p->pred || !p->accepted_len || !p->path ||
      !p->bonus || !p->best_node)
    return set_error(GORGON_ERR_INVALID, "gorgon_verify: null pointer");
  const size_t need = gorgon_verify_workspace_size(p);
  if (!workspace || workspace_bytes < need)
    return set_error(GORGON_ERR_WORKSPACE, "gorgon_verify: workspace smaller than gorgon_verify_workspace_size()");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(workspace, 0, need, st), "gorgon_verify counter reset");
  if (rc) return rc;
  VerifyArgs a{};
  a.logits = p->logits; a.lsb = p->logits_stride_b; a.lsr = p->logits_stride_r;
  a.rows = p->rows; a.vocab = p->vocab;
  a.n = static_cast<int>(p->n); a.prompt_len = static_cast<int>(p->prompt_len);
  a.draft = p->draft; a.dsb = p->draft_stride_b;
  a.parents = p->parents; a.psb = p->parents_stride_b;
  a.pred = p->pred; a.accepted_len = p->accepted_len; a.path = p->path; a.bonus = p->bonus;
  a.best_node = p->best_node; a.hidden_row = p->hidden_row;
  a.counters = static_cast<int32_t*>(workspace);
  a.err = device_error_word();
  const int64_t ev = static_cast<int64_t>(16 / dtype_bytes(p->dtype));
  a.vec_ok = (reinterpret_cast<uintptr_t>(p->logits) % 16 == 0) && p->logits_stride_b % ev == 0 &&
             p->logits_stride_r % ev == 0;
  const int batch = static_cast<int>(p->batch);
  switch (p->dtype) {
    case GORGON_F32: return launch_verify_t<float>(a, batch, st);
    case GORGON_BF16: return launch_verify_t<__nv_bfloat16>(a, batch, st);
    default: return launch_verify_t<__half>(a, batch, st);
  }
}

// ---------------------------------------------------------------------------
// gorgon_verify_noalloc: the same fused verifier for callers that cannot
// allocate device memory.  Its only scratch, one arrival counter per sequence,
// lives in a fixed array compiled into the library instead of a caller
// workspace.  Every GPU that loads the library holds this array until the
// process exits.
namespace gorgon {
namespace {

constexpr int kNoAllocMaxBatch = 4096;  // 16 KiB of counters per device

static __device__ __align__(256) int32_t g_verify_noalloc_counters[kNoAllocMaxBatch];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
int32_t* g_noalloc_counters[kNoAllocMaxDevices] = {};

// Device address of the counter array on the current device.  Host code only
// sees a stand-in for a __device__ symbol, so the address is looked up once
// per device (with that device current) and cached for the life of the
// process: a device reset (cudaDeviceReset, or a primary context destroyed
// and created again) would leave the cached address stale, so the library
// must not be used across one.
int noalloc_counters(int32_t** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "gorgon_verify_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_verify_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_counters[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_verify_noalloc_counters),
                    "gorgon_verify_noalloc: cudaGetSymbolAddress");
    if (rc) return rc;
    g_noalloc_counters[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_counters[dev];
  return GORGON_OK;
}

}  // namespace
}  // namespace gorgon

extern "C" int gorgon_verify_noalloc(const gorgon_verify_params* p, void* stream) {
  using namespace gorgon;
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: params is null");
  if (!dtype_ok(p->dtype)) return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: unknown dtype");
  if (p->batch < 0 || p->rows < 0 || p->vocab < 0 || p->n < 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: negative size");
  if (p->batch == 0) return GORGON_OK;
  if (p->batch > kNoAllocMaxBatch)
    return set_error(GORGON_ERR_UNSUPPORTED,
                     "gorgon_verify_noalloc: batch > 4096; its fixed scratch holds 4096 sequence counters "
                     "(use gorgon_verify with a workspace for larger batches)");
  if (p->n < 1 || p->n > 4096) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_verify_noalloc: n must be in [1, 4096]");
  if (p->prompt_len < 1) return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: prompt_len must be >= 1");
  if (p->vocab < 1 || p->vocab > INT_MAX - 16)
    return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: vocab outside [1, 2^31)");
  if (p->rows < p->prompt_len) return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: rows < prompt_len");
  if (!p->logits || !p->draft || !p->parents || !p->pred || !p->accepted_len || !p->path || !p->bonus ||
      !p->best_node)
    return set_error(GORGON_ERR_INVALID, "gorgon_verify_noalloc: null pointer");
  int32_t* counters = nullptr;
  int rc = noalloc_counters(&counters);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's counts: clear the ones this call uses.
  rc = check_cuda(cudaMemsetAsync(counters, 0, static_cast<size_t>(p->batch) * sizeof(int32_t), st),
                  "gorgon_verify_noalloc counter reset");
  if (rc) return rc;
  VerifyArgs a{};
  a.logits = p->logits; a.lsb = p->logits_stride_b; a.lsr = p->logits_stride_r;
  a.rows = p->rows; a.vocab = p->vocab;
  a.n = static_cast<int>(p->n); a.prompt_len = static_cast<int>(p->prompt_len);
  a.draft = p->draft; a.dsb = p->draft_stride_b;
  a.parents = p->parents; a.psb = p->parents_stride_b;
  a.pred = p->pred; a.accepted_len = p->accepted_len; a.path = p->path; a.bonus = p->bonus;
  a.best_node = p->best_node; a.hidden_row = p->hidden_row;
  a.counters = counters;
  a.err = device_error_word();
  const int64_t ev = static_cast<int64_t>(16 / dtype_bytes(p->dtype));
  a.vec_ok = (reinterpret_cast<uintptr_t>(p->logits) % 16 == 0) && p->logits_stride_b % ev == 0 &&
             p->logits_stride_r % ev == 0;
  const int batch = static_cast<int>(p->batch);
  switch (p->dtype) {
    case GORGON_F32: return launch_verify_t<float>(a, batch, st);
    case GORGON_BF16: return launch_verify_t<__nv_bfloat16>(a, batch, st);
    default: return launch_verify_t<__half>(a, batch, st);
  }
}
