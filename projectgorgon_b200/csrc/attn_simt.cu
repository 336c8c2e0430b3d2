// CUDA-core (SIMT) tree attention: split-K over the key/value rows,
// grouped-query packing, warp-shuffle online softmax.
//
// Work split: grid (split, batch * heads_kv, query tile).  A query tile holds
// 32 rows of the packed (query head in the group, tree node) space, so the
// key/value rows a CTA stages in shared memory serve every query head of its
// group.  Each of the 4 warps owns 8 query rows; lane j scores key row j of
// the 32-row tile against those 8 rows, the warp reduces max and sum with
// shuffles, then lanes switch to owning output columns for P.V.  With several
// splits each CTA leaves a normalised partial output and its log-sum-exp in
// the caller's workspace and attn_combine_kernel merges them.
//
// This path serves fp32 (the reference's tree_attention_cuda computes in fp32,
// src/gorgon/kernels/cuda/tree_attention.cu:7-51), any head_dim up to 256, and
// dense masks; the tcgen05 kernel takes bf16/f16 trees of 64+ nodes.
#include "attn.cuh"

namespace gorgon {
namespace {

constexpr int kQT = 32;      // query rows per CTA
constexpr int kKT = 32;      // key/value rows per tile
constexpr int kWarps = 4;
constexpr int kRPW = kQT / kWarps;  // query rows per warp
constexpr int kThreads = kWarps * 32;
constexpr float kLn2 = 0.6931471805599453f;

template <int DMAX>
struct SimtSmem {
  static constexpr int kPad = DMAX + 4;
  static constexpr size_t q_floats = size_t(kQT) * DMAX;
  static constexpr size_t k_floats = size_t(kKT) * kPad;
  static constexpr size_t v_floats = size_t(kKT) * DMAX;
  static constexpr size_t p_floats = size_t(kWarps) * kKT * kRPW;
  static size_t bytes(int anc_words) {
    return (q_floats + k_floats + v_floats + p_floats) * sizeof(float) +
           size_t(kQT) * anc_words * sizeof(uint32_t);
  }
};

__device__ __forceinline__ bool kv_visible(const AttnArgs& a, int b, int node, int c, int L,
                                           const uint32_t* anc_row) {
  if (a.mask_kind == GORGON_MASK_DENSE) {
    return a.mask[static_cast<int64_t>(b) * a.mask_sb + static_cast<int64_t>(node) * a.mask_sn + c] != 0;
  }
  const int t = c - (L - a.n);
  if (t < 0) return true;
  if (a.mask_kind == GORGON_MASK_PARENTS) return (anc_row[t >> 5] >> (t & 31)) & 1u;
  return a.mask[static_cast<int64_t>(b) * a.mask_sb + static_cast<int64_t>(node) * a.mask_sn + t] != 0;
}

// Loads `count` consecutive elements of a row into float smem, zero-padding to DMAX.
template <typename T, int DMAX>
__device__ __forceinline__ void load_rows(float* dst, int dst_stride, const T* __restrict__ src,
                                          int64_t row0_off, int64_t row_stride, int rows_valid,
                                          int rows, int d, bool vec_ok, float mul) {
  constexpr int EV = 16 / sizeof(T);
  if (vec_ok) {
    constexpr int VPR = DMAX / EV;  // vectors per row
    // Up to 8 vectors per thread are requested before any is converted and
    // stored, so a tile costs one or two memory round trips instead of one
    // per vector (31-node bf16 trees over 16 x 8192: 4611 -> 3265 us).  The
    // 256-wide variant keeps one at a time: its accumulators leave no
    // registers for more without losing a resident CTA (68 -> 81 us with 8).
    constexpr int kBatch = DMAX > 128 ? 1 : 8;
    const int total = rows * VPR;
    for (int base = 0; base < total; base += kBatch * kThreads) {
      uint4 raw[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int idx = base + i * kThreads + threadIdx.x;
        const int r = idx / VPR;
        const int c0 = (idx % VPR) * EV;
        raw[i] = (idx < total && r < rows_valid && c0 < d)
                     ? *reinterpret_cast<const uint4*>(src + row0_off + r * row_stride + c0)
                     : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int idx = base + i * kThreads + threadIdx.x;
        if (idx >= total) continue;
        const int r = idx / VPR;
        const int c0 = (idx % VPR) * EV;
        const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
        for (int u = 0; u < EV; ++u) dst[r * dst_stride + c0 + u] = Cvt<T>::to_f(e[u]) * mul;
      }
    }
  } else {
    for (int idx = threadIdx.x; idx < rows * DMAX; idx += kThreads) {
      const int r = idx / DMAX;
      const int c = idx % DMAX;
      float x = 0.f;
      if (r < rows_valid && c < d) x = Cvt<T>::to_f(src[row0_off + r * row_stride + c]) * mul;
      dst[r * dst_stride + c] = x;
    }
  }
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
attn_simt_kernel(const AttnArgs a) {
  using S = SimtSmem<DMAX>;
  constexpr int NC = DMAX / 32;
  extern __shared__ float4 smem_f4[];
  float* qs = reinterpret_cast<float*>(smem_f4);
  float* ks = qs + S::q_floats;
  float* vs = ks + S::k_floats;
  float* ps = vs + S::v_floats;
  uint32_t* anc = reinterpret_cast<uint32_t*>(ps + S::p_floats);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y / a.hkv;
  const int kvh = blockIdx.y % a.hkv;
  const int R = a.group * a.n;
  const int row0 = blockIdx.z * kQT;
  const T* __restrict__ qp = static_cast<const T*>(a.q);
  const T* __restrict__ kp = static_cast<const T*>(a.k);
  const T* __restrict__ vp = static_cast<const T*>(a.v);

  const SeqExtent ext = seq_extent(a, b, kvh);
  const int L = ext.L;
  const bool tree_mode = a.mask_kind != GORGON_MASK_DENSE;
  const bool bad_len = tree_mode && L < a.n;
  if (bad_len && threadIdx.x == 0 && split == 0 && blockIdx.z == 0) raise_device_error(a.err, kErrBadSeqlen);

  // This split's key/value rows [lo, hi).
  const int per = (L + a.splits - 1) / a.splits;
  const int chunk = ((per + kKT - 1) / kKT) * kKT;
  const int lo = min(L, split * chunk);
  const int hi = bad_len ? lo : min(L, lo + chunk);

  // Query tile, pre-scaled by softmax scale * log2(e).  Row r of the tile is
  // packed row row0 + r = g * n + i (group member g, tree node i).
  {
    constexpr int EV = 16 / sizeof(T);
    for (int idx = threadIdx.x; idx < kQT * (DMAX / EV); idx += kThreads) {
      const int r = idx / (DMAX / EV);
      const int c0 = (idx % (DMAX / EV)) * EV;
      const int rg = row0 + r;
      float vals[EV];
#pragma unroll
      for (int u = 0; u < EV; ++u) vals[u] = 0.f;
      if (rg < R) {
        const int g = rg / a.n, i = rg % a.n;
        const int64_t off = static_cast<int64_t>(b) * a.q_sb +
                            static_cast<int64_t>(kvh * a.group + g) * a.q_sh +
                            static_cast<int64_t>(i) * a.q_sn;
        if (a.vec_ok) {
          if (c0 < a.d) {
            const uint4 raw = *reinterpret_cast<const uint4*>(qp + off + c0);
            const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int u = 0; u < EV; ++u) vals[u] = Cvt<T>::to_f(e[u]) * a.scale_log2;
          }
        } else {
#pragma unroll
          for (int u = 0; u < EV; ++u)
            if (c0 + u < a.d) vals[u] = Cvt<T>::to_f(qp[off + c0 + u]) * a.scale_log2;
        }
      }
#pragma unroll
      for (int u = 0; u < EV; ++u) qs[r * DMAX + c0 + u] = vals[u];
    }
  }
  const int aw = (a.n + 31) >> 5;
  if (a.mask_kind == GORGON_MASK_PARENTS) {
    for (int idx = threadIdx.x; idx < kQT * aw; idx += kThreads) anc[idx] = 0u;
    __syncthreads();
    if (threadIdx.x < kQT) {
      const int rg = row0 + threadIdx.x;
      if (rg < R) {
        const int32_t* par = a.parents + static_cast<int64_t>(b) * a.par_sb;
        ancestor_bits(par, a.n, rg % a.n, a.max_depth, anc + threadIdx.x * aw, a.err);
      }
    }
  }
  __syncthreads();

  float m[kRPW], l[kRPW], acc[kRPW][NC];
#pragma unroll
  for (int r = 0; r < kRPW; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[r][c] = 0.f;
  }

  for (int t0 = lo; t0 < hi; t0 += kKT) {
    const int rows_valid = min(kKT, hi - t0);
    load_rows<T, DMAX>(ks, S::kPad, kp, ext.base_k + static_cast<int64_t>(t0) * a.k_ss, a.k_ss,
                       rows_valid, kKT, a.d, a.vec_ok, 1.f);
    load_rows<T, DMAX>(vs, DMAX, vp, ext.base_v + static_cast<int64_t>(t0) * a.v_ss, a.v_ss,
                       rows_valid, kKT, a.d, a.vec_ok, 1.f);
    __syncthreads();

    float s[kRPW];
#pragma unroll
    for (int r = 0; r < kRPW; ++r) s[r] = 0.f;
#pragma unroll 4
    for (int dd = 0; dd < DMAX; dd += 4) {
      const float4 kf = *reinterpret_cast<const float4*>(&ks[lane * S::kPad + dd]);
#pragma unroll
      for (int r = 0; r < kRPW; ++r) {
        const float4 qf = *reinterpret_cast<const float4*>(&qs[(warp * kRPW + r) * DMAX + dd]);
        s[r] = fmaf(qf.x, kf.x, s[r]);
        s[r] = fmaf(qf.y, kf.y, s[r]);
        s[r] = fmaf(qf.z, kf.z, s[r]);
        s[r] = fmaf(qf.w, kf.w, s[r]);
      }
    }

    const int c = t0 + lane;
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
      const int lr = warp * kRPW + r;
      const int rg = row0 + lr;
      bool vis = (lane < rows_valid) && (rg < R);
      if (vis) vis = kv_visible(a, b, rg % a.n, c, L, anc + lr * aw);
      const float sv = vis ? s[r] : -INFINITY;
      const float mt = warp_max(sv);
      const float mn = fmaxf(m[r], mt);
      float p = 0.f, alpha = 1.f;
      if (mn != -INFINITY) {
        alpha = exp2f(m[r] - mn);
        p = vis ? exp2f(sv - mn) : 0.f;
      }
      l[r] = l[r] * alpha + warp_sum(p);
      m[r] = mn;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) acc[r][cc] *= alpha;
      ps[(warp * kKT + lane) * kRPW + r] = p;
    }
    __syncwarp();
#pragma unroll 4
    for (int j = 0; j < kKT; ++j) {
      const float4 p0 = *reinterpret_cast<const float4*>(&ps[(warp * kKT + j) * kRPW]);
      const float4 p1 = *reinterpret_cast<const float4*>(&ps[(warp * kKT + j) * kRPW + 4]);
      const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        const float vv = vs[j * DMAX + lane + 32 * cc];
#pragma unroll
        for (int r = 0; r < kRPW; ++r) acc[r][cc] = fmaf(pr[r], vv, acc[r][cc]);
      }
    }
    __syncthreads();
  }

  const int64_t total = static_cast<int64_t>(a.batch) * a.hq * a.n;
#pragma unroll
  for (int r = 0; r < kRPW; ++r) {
    const int rg = row0 + warp * kRPW + r;
    if (rg >= R) continue;
    const int g = rg / a.n, i = rg % a.n;
    const int h = kvh * a.group + g;
    const int64_t orow = (static_cast<int64_t>(b) * a.hq + h) * a.n + i;
    if (a.splits == 1) {
      const float inv = 1.f / l[r];  // l == 0 (nothing visible): 0 * inf = NaN, as softmax
      const int64_t ob = static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh +
                         static_cast<int64_t>(i) * a.o_sn;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        const int col = lane + 32 * cc;
        if (col < a.d) store_as(a.out, a.out_dtype, ob + col, acc[r][cc] * inv);
      }
      if (a.lse && lane == 0) a.lse[orow] = (m[r] + log2f(l[r])) * kLn2;
    } else {
      const int64_t prow = static_cast<int64_t>(split) * total + orow;
      const bool any = l[r] > 0.f;
      const float inv = any ? 1.f / l[r] : 0.f;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        const int col = lane + 32 * cc;
        if (col < a.d) a.part_o[prow * a.d + col] = acc[r][cc] * inv;
      }
      if (lane == 0) a.part_lse[prow] = any ? m[r] + log2f(l[r]) : -INFINITY;
    }
  }
}

// Merges split partials: out = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M).
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnArgs a) {
  const int64_t total = static_cast<int64_t>(a.batch) * a.hq * a.n;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= total) return;
  const int i = static_cast<int>(row % a.n);
  const int h = static_cast<int>((row / a.n) % a.hq);
  const int b = static_cast<int>(row / (static_cast<int64_t>(a.n) * a.hq));
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.part_lse[s * total + row]);
  const int64_t ob = static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(h) * a.o_sh +
                     static_cast<int64_t>(i) * a.o_sn;
  if (M == -INFINITY) {
    for (int col = lane; col < a.d; col += 32) store_as(a.out, a.out_dtype, ob + col, NAN);
    if (a.lse && lane == 0) a.lse[row] = -INFINITY;
    return;
  }
  float wsum = 0.f;
  for (int s = 0; s < a.splits; ++s) wsum += exp2f(a.part_lse[s * total + row] - M);
  const float inv = 1.f / wsum;
  for (int col = lane; col < a.d; col += 32) {
    float o = 0.f;
    // Every split's row is loaded (the workspace holds them all) and a zero
    // weight selects it away, rather than branching around the load, so the
    // unrolled splits' loads are in flight together; an empty split's row
    // never reaches the sum.
#pragma unroll 4
    for (int s = 0; s < a.splits; ++s) {
      const float w = exp2f(a.part_lse[s * total + row] - M);
      const float v = a.part_o[(s * total + row) * a.d + col];
      o = w > 0.f ? fmaf(w, v, o) : o;
    }
    store_as(a.out, a.out_dtype, ob + col, o * inv);
  }
  if (a.lse && lane == 0) a.lse[row] = (M + log2f(wsum)) * kLn2;
}

template <typename T, int DMAX>
int launch_simt_t(const AttnArgs& a, cudaStream_t st) {
  const int aw = a.mask_kind == GORGON_MASK_PARENTS ? (a.n + 31) / 32 : 0;
  const size_t smem = SimtSmem<DMAX>::bytes(aw);
  auto kern = attn_simt_kernel<T, DMAX>;
  int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem)),
                      "attn_simt smem attribute");
  if (rc) return rc;
  const int R = a.group * a.n;
  dim3 grid(a.splits, a.batch * a.hkv, (R + kQT - 1) / kQT);
  kern<<<grid, kThreads, smem, st>>>(a);
  return check_cuda(cudaGetLastError(), "attn_simt launch");
}

template <typename T>
int launch_simt_d(const AttnArgs& a, cudaStream_t st) {
  if (a.d <= 32) return launch_simt_t<T, 32>(a, st);
  if (a.d <= 64) return launch_simt_t<T, 64>(a, st);
  if (a.d <= 128) return launch_simt_t<T, 128>(a, st);
  return launch_simt_t<T, 256>(a, st);
}

}  // namespace

int launch_attn_simt(const AttnArgs& a, int dtype, cudaStream_t st) {
  switch (dtype) {
    case GORGON_F32: return launch_simt_d<float>(a, st);
    case GORGON_BF16: return launch_simt_d<__nv_bfloat16>(a, st);
    case GORGON_F16: return launch_simt_d<__half>(a, st);
    default: return set_error(GORGON_ERR_INVALID, "attn_simt: bad dtype");
  }
}

int launch_attn_combine(const AttnArgs& a, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(a.batch) * a.hq * a.n;
  const int64_t blocks = (total + 3) / 4;
  if (blocks > 0x7fffffff) return set_error(GORGON_ERR_UNSUPPORTED, "attn_combine: too many rows");
  attn_combine_kernel<<<static_cast<unsigned>(blocks), 128, 0, st>>>(a);
  return check_cuda(cudaGetLastError(), "attn_combine launch");
}

}  // namespace gorgon
