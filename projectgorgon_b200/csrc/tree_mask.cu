// Ancestor mask from a compact parents[] array (build_tree_mask).
//
// One CTA per (tree, row i): a single thread walks at most `depth` parent hops
// from i and marks each ancestor in a shared-memory byte row, then the whole
// CTA streams the row out with coalesced stores.  The walk is the reference's
// pointer jumping (src/gorgon/kernels/tree_mask.py:33-42) seen from one row:
// round r of the reference marks the r-th ancestor of every row at once.
#include "common.cuh"

namespace gorgon {
namespace {

constexpr int kMaskThreads = 256;

__global__ void __launch_bounds__(kMaskThreads)
tree_mask_kernel(const int32_t* __restrict__ parents, int64_t n, int64_t parents_stride_b,
                 int64_t depth, uint8_t* __restrict__ out, uint32_t* err) {
  extern __shared__ uint8_t row[];
  const int64_t i = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int32_t* par = parents + b * parents_stride_b;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) row[j] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    row[i] = 1;
    int64_t cur = par[i];
    for (int64_t hop = 0; hop < depth && cur >= 0; ++hop) {
      if (cur >= n) {
        raise_device_error(err, kErrBadParent);
        break;
      }
      row[cur] = 1;
      cur = par[cur];
    }
  }
  __syncthreads();
  uint8_t* dst = out + (b * n + i) * n;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) dst[j] = row[j];
}

}  // namespace
}  // namespace gorgon

extern "C" int gorgon_tree_mask(const int32_t* parents, int64_t batch, int64_t n,
                                int64_t parents_stride_b, int64_t depth, uint8_t* out,
                                void* stream) {
  using namespace gorgon;
  if (n < 0 || batch < 0) return set_error(GORGON_ERR_INVALID, "gorgon_tree_mask: negative size");
  if (n == 0 || batch == 0) return GORGON_OK;
  if (!parents || !out) return set_error(GORGON_ERR_INVALID, "gorgon_tree_mask: null pointer");
  if (n > 32768) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_mask: n > 32768");
  if (batch > 65535) return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_mask: batch > 65535");
  if (parents_stride_b < 0) return set_error(GORGON_ERR_INVALID, "gorgon_tree_mask: negative stride");
  const int64_t hops = depth < 0 ? n : depth;
  dim3 grid(static_cast<unsigned>(n), static_cast<unsigned>(batch));
  tree_mask_kernel<<<grid, kMaskThreads, static_cast<size_t>(n), static_cast<cudaStream_t>(stream)>>>(
      parents, n, parents_stride_b, hops, out, device_error_word());
  return check_cuda(cudaGetLastError(), "gorgon_tree_mask launch");
}
