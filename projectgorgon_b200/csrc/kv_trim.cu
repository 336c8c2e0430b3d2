// KV-cache trim-on-reject: gathers the accepted rows of every (layer, batch
// row, kv head) slice into contiguous slots, all layers in one launch.
//
// Grid (heads, batch, 2 * layers): z picks the layer and K or V.  A CTA first
// checks every index of its slice, then copies the slice's lens[b] source rows
// into shared memory, synchronises, and only then writes them out, so an
// in-place gather whose destination slots overlap later source rows (slot 1
// <- row 2 while row 2 <- row 4) reads every source before it is overwritten.
// This is apply_cache_slice (src/gorgon/inference/kv_cache.py:89-108,
// new[:L] = old[idx]) per slice, with the destination start per batch row.
#include "common.cuh"

namespace gorgon {
namespace {

constexpr int kThreads = 128;
constexpr int kLayersPerLaunch = 32;

struct TrimArgs {
  void* src[2][kLayersPerLaunch];
  void* dst[2][kLayersPerLaunch];
  int64_t sb, sh, ss;   // element strides
  int64_t row_bytes;    // head_dim * elem_bytes
  int64_t elem_bytes;
  int64_t seq;
  const int32_t* idx;
  int64_t idx_sb;
  int max_len;
  const int32_t* lens;
  const int32_t* dst_start;
  uint32_t* err;
  int vec_ok;
};

__global__ void __launch_bounds__(kThreads) kv_trim_kernel(const TrimArgs a) {
  extern __shared__ uint4 stage[];
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int layer = blockIdx.z >> 1;
  const int kv = blockIdx.z & 1;
  const int len = a.lens[b];
  const int d0 = a.dst_start ? a.dst_start[b] : 0;
  const int32_t* ib = a.idx + static_cast<int64_t>(b) * a.idx_sb;
  int bad = (len < 0 || len > a.max_len || d0 < 0 || static_cast<int64_t>(d0) + max(len, 0) > a.seq);
  if (!bad) {
    for (int r = threadIdx.x; r < len; r += kThreads) {
      const int s = ib[r];
      if (s < 0 || s >= a.seq) bad = 1;
    }
  }
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0 && h == 0 && blockIdx.z == 0) raise_device_error(a.err, kErrBadTrimIndex);
    return;
  }
  if (len == 0) return;
  const int64_t slice = (static_cast<int64_t>(b) * a.sb + static_cast<int64_t>(h) * a.sh) * a.elem_bytes;
  const char* src = static_cast<const char*>(a.src[kv][layer]) + slice;
  char* dst = static_cast<char*>(a.dst[kv][layer]) + slice;
  const int64_t rs = a.ss * a.elem_bytes;  // row stride in bytes
  if (a.vec_ok) {
    const int vpr = static_cast<int>(a.row_bytes / 16);
    for (int e = threadIdx.x; e < len * vpr; e += kThreads) {
      const int r = e / vpr, c = e % vpr;
      stage[e] = *reinterpret_cast<const uint4*>(src + ib[r] * rs + c * 16);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < len * vpr; e += kThreads) {
      const int r = e / vpr, c = e % vpr;
      *reinterpret_cast<uint4*>(dst + (d0 + r) * rs + c * 16) = stage[e];
    }
  } else {
    uint8_t* sb = reinterpret_cast<uint8_t*>(stage);
    const int rb = static_cast<int>(a.row_bytes);
    for (int e = threadIdx.x; e < len * rb; e += kThreads) {
      const int r = e / rb, c = e % rb;
      sb[e] = static_cast<const uint8_t*>(reinterpret_cast<const void*>(src + ib[r] * rs))[c];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < len * rb; e += kThreads) {
      const int r = e / rb, c = e % rb;
      dst[(d0 + r) * rs + c] = static_cast<char>(sb[e]);
    }
  }
}

// Fast path for the common case (16-byte aligned rows, at most kChunks * 32
// 16-byte chunks per slice, e.g. 8 rows of 256 bytes with kChunks = 4): one
// warp per (layer, batch row, head), moving both its K and its V slice, kWarps
// heads per CTA.  Lengths, destination starts and indices are fetched once
// for both (indices up to max_len, unconditionally in range of the index row),
// both slices' source rows go to registers in one batch of loads, a warp
// barrier orders every lane's loads before any lane's stores (in-place moves
// whose slots overlap later sources stay correct), then the rows are written.
// The register array is sized to the slice (kChunks), so short paths leave
// room for more resident warps: the whole trim of a decode step is then one
// wave of round trips.
constexpr int kWarps = 8;

template <int kChunks>
__global__ void __launch_bounds__(kWarps * 32) kv_trim_warp_kernel(const TrimArgs a, int heads) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * kWarps + warp;
  const int b = blockIdx.y;
  const int layer = blockIdx.z;
  if (h >= heads) return;
  const int32_t* ib = a.idx + static_cast<int64_t>(b) * a.idx_sb;
  const int len = a.lens[b];
  const int d0 = a.dst_start ? a.dst_start[b] : 0;
  const int my_src = lane < a.max_len ? ib[lane] : 0;  // max_len <= 32 on this path
  int bad = (len < 0 || len > a.max_len || d0 < 0 || static_cast<int64_t>(d0) + max(len, 0) > a.seq);
  if (!bad && lane < len && (my_src < 0 || my_src >= a.seq)) bad = 1;
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0 && h == 0 && blockIdx.z == 0) raise_device_error(a.err, kErrBadTrimIndex);
    return;
  }
  if (len == 0) return;
  const int64_t slice = (static_cast<int64_t>(b) * a.sb + static_cast<int64_t>(h) * a.sh) * a.elem_bytes;
  const char* src0 = static_cast<const char*>(a.src[0][layer]) + slice;
  const char* src1 = static_cast<const char*>(a.src[1][layer]) + slice;
  const int64_t rs = a.ss * a.elem_bytes;
  const int vpr = static_cast<int>(a.row_bytes / 16);
  const int total = len * vpr;
  uint4 v0[kChunks], v1[kChunks];
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int e = lane + 32 * k;
    const int r = e / vpr;
    const int s = __shfl_sync(0xffffffffu, my_src, min(r, 31));  // every lane, one program point
    if (e < total) {
      const int64_t off = s * rs + (e - r * vpr) * 16;
      v0[k] = __ldcs(reinterpret_cast<const uint4*>(src0 + off));
      v1[k] = __ldcs(reinterpret_cast<const uint4*>(src1 + off));
    }
  }
  __syncwarp();
  char* dst0 = static_cast<char*>(a.dst[0][layer]) + slice;
  char* dst1 = static_cast<char*>(a.dst[1][layer]) + slice;
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int e = lane + 32 * k;
    if (e < total) {
      const int r = e / vpr, c = e - r * vpr;
      const int64_t off = (d0 + r) * rs + c * 16;
      *reinterpret_cast<uint4*>(dst0 + off) = v0[k];
      *reinterpret_cast<uint4*>(dst1 + off) = v1[k];
    }
  }
}

}  // namespace
}  // namespace gorgon

extern "C" int gorgon_kv_trim(const gorgon_kv_trim_params* p, void* stream) {
  using namespace gorgon;
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_kv_trim: params is null");
  if (p->layers < 0 || p->batch < 0 || p->heads < 0 || p->seq_capacity < 0 || p->head_dim < 0 ||
      p->max_len < 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_kv_trim: negative size");
  if (p->layers == 0 || p->batch == 0 || p->heads == 0 || p->head_dim == 0) return GORGON_OK;
  if (p->elem_bytes != 1 && p->elem_bytes != 2 && p->elem_bytes != 4 && p->elem_bytes != 8)
    return set_error(GORGON_ERR_INVALID, "gorgon_kv_trim: elem_bytes must be 1, 2, 4 or 8");
  if (p->max_len > 256) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_kv_trim: max_len > 256");
  if (p->batch > 65535 || p->heads > 65535 || p->seq_capacity > INT32_MAX)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_kv_trim: batch, heads or seq_capacity too large");
  if (!p->k_src || !p->v_src || !p->src_idx || !p->lens)
    return set_error(GORGON_ERR_INVALID, "gorgon_kv_trim: null pointer");
  const int64_t row_bytes = p->head_dim * p->elem_bytes;
  const size_t smem = static_cast<size_t>(p->max_len) * static_cast<size_t>(row_bytes);
  if (smem > 200 * 1024) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_kv_trim: max_len * row bytes > 200 KiB");
  TrimArgs a{};
  a.sb = p->stride_b; a.sh = p->stride_h; a.ss = p->stride_s;
  a.row_bytes = row_bytes; a.elem_bytes = p->elem_bytes; a.seq = p->seq_capacity;
  a.idx = p->src_idx; a.idx_sb = p->idx_stride_b; a.max_len = static_cast<int>(p->max_len);
  a.lens = p->lens; a.dst_start = p->dst_start;
  a.err = device_error_word();
  bool vec = row_bytes % 16 == 0 && (p->stride_b * p->elem_bytes) % 16 == 0 &&
             (p->stride_h * p->elem_bytes) % 16 == 0 && (p->stride_s * p->elem_bytes) % 16 == 0;
  for (int64_t l = 0; l < p->layers; ++l) {
    const void* ptrs[4] = {p->k_src[l], p->v_src[l], p->k_dst ? p->k_dst[l] : p->k_src[l],
                           p->v_dst ? p->v_dst[l] : p->v_src[l]};
    for (const void* q : ptrs) {
      if (!q) return set_error(GORGON_ERR_INVALID, "gorgon_kv_trim: null layer pointer");
      if (reinterpret_cast<uintptr_t>(q) % 16) vec = false;
    }
  }
  a.vec_ok = vec;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t chunks = p->max_len * (row_bytes / 16);  // 16-byte chunks of the longest slice
  if (vec && p->max_len <= 32 && chunks <= 32 * 8) {
    for (int64_t l0 = 0; l0 < p->layers; l0 += kLayersPerLaunch) {
      const int nl = static_cast<int>(std::min<int64_t>(kLayersPerLaunch, p->layers - l0));
      for (int i = 0; i < nl; ++i) {
        a.src[0][i] = p->k_src[l0 + i];
        a.src[1][i] = p->v_src[l0 + i];
        a.dst[0][i] = p->k_dst ? p->k_dst[l0 + i] : p->k_src[l0 + i];
        a.dst[1][i] = p->v_dst ? p->v_dst[l0 + i] : p->v_src[l0 + i];
      }
      dim3 grid(static_cast<unsigned>((p->heads + kWarps - 1) / kWarps), static_cast<unsigned>(p->batch),
                static_cast<unsigned>(nl));
      if (chunks <= 32 * 4)
        kv_trim_warp_kernel<4><<<grid, kWarps * 32, 0, st>>>(a, static_cast<int>(p->heads));
      else
        kv_trim_warp_kernel<8><<<grid, kWarps * 32, 0, st>>>(a, static_cast<int>(p->heads));
      int rc = check_cuda(cudaGetLastError(), "kv_trim launch");
      if (rc) return rc;
    }
    return GORGON_OK;
  }
  auto kern = kv_trim_kernel;
  if (smem > 48 * 1024) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)), "kv_trim smem attribute");
    if (rc) return rc;
  }
  for (int64_t l0 = 0; l0 < p->layers; l0 += kLayersPerLaunch) {
    const int nl = static_cast<int>(std::min<int64_t>(kLayersPerLaunch, p->layers - l0));
    for (int i = 0; i < nl; ++i) {
      a.src[0][i] = p->k_src[l0 + i];
      a.src[1][i] = p->v_src[l0 + i];
      a.dst[0][i] = p->k_dst ? p->k_dst[l0 + i] : p->k_src[l0 + i];
      a.dst[1][i] = p->v_dst ? p->v_dst[l0 + i] : p->v_src[l0 + i];
    }
    dim3 grid(static_cast<unsigned>(p->heads), static_cast<unsigned>(p->batch), 2u * nl);
    kern<<<grid, kThreads, smem, st>>>(a);
    int rc = check_cuda(cudaGetLastError(), "kv_trim launch");
    if (rc) return rc;
  }
  return GORGON_OK;
}
