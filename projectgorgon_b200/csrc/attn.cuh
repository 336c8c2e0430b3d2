// Internal description of one tree-attention launch, shared by the CUDA-core
// (SIMT) and tensor-core (tcgen05) kernels.
#pragma once

#include "common.cuh"

namespace gorgon {

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t q_sb, q_sh, q_sn;
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t o_sb, o_sh, o_sn;
  const int32_t* cu_seqlens;
  const int32_t* parents;
  int64_t par_sb;
  const uint8_t* mask;
  int64_t mask_sb, mask_sn;
  float* lse;
  float* part_o;    // [splits, batch*hq*n, d] when splits > 1
  float* part_lse;  // [splits, batch*hq*n]   (log2 domain)
  uint32_t* err;
  int64_t kv_rows;   // rows of k/v with cu_seqlens (0 = unknown)
  int batch, hq, hkv, group, n, kv_len, d;
  int mask_kind, max_depth, out_dtype, splits;
  int vec_ok;        // 16-byte vector loads of q/k/v rows are legal
  float scale_log2;  // softmax scale * log2(e)
};

// Key/value extent of sequence b: rows [0, L) starting at element offsets
// base_k / base_v of kv head `kvh`.
struct SeqExtent {
  int64_t base_k, base_v;
  int L;
};

__device__ __forceinline__ SeqExtent seq_extent(const AttnArgs& a, int b, int kvh) {
  SeqExtent e;
  if (a.cu_seqlens) {
    const int s0 = a.cu_seqlens[b];
    const int s1 = a.cu_seqlens[b + 1];
    e.L = s1 - s0;
    e.base_k = static_cast<int64_t>(s0) * a.k_ss + static_cast<int64_t>(kvh) * a.k_sh;
    e.base_v = static_cast<int64_t>(s0) * a.v_ss + static_cast<int64_t>(kvh) * a.v_sh;
  } else {
    e.L = a.kv_len;
    e.base_k = static_cast<int64_t>(b) * a.k_sb + static_cast<int64_t>(kvh) * a.k_sh;
    e.base_v = static_cast<int64_t>(b) * a.v_sb + static_cast<int64_t>(kvh) * a.v_sh;
  }
  return e;
}

// Fills anc[0 .. ceil(n/32)) with the ancestor-or-self bits of tree node i:
// node i itself plus at most max_depth parent hops (the walk of
// src/gorgon/kernels/fused_tree_verify_triton.py:52-63).
__device__ __forceinline__ void ancestor_bits(const int32_t* __restrict__ par, int n, int i,
                                              int max_depth, uint32_t* anc, uint32_t* err) {
  anc[i >> 5] |= 1u << (i & 31);
  int cur = par[i];
  for (int hop = 0; hop < max_depth && cur >= 0; ++hop) {
    if (cur >= n) {
      raise_device_error(err, kErrBadParent);
      break;
    }
    anc[cur >> 5] |= 1u << (cur & 31);
    cur = par[cur];
  }
}

// The output gather of gorgon_tree_attn_gather: the other ranks' copies of
// a.out (same byte offset in their buffers), their signal words and ours.
struct PeerLaunch {
  int npeers;
  void* peer_out[7];
  uint64_t* peer_sig[7];
  uint64_t* sig;
};

// Host launchers (defined in attn_simt.cu / attn_tc.cu).
int launch_attn_simt(const AttnArgs& a, int dtype, cudaStream_t st);
int launch_attn_combine(const AttnArgs& a, cudaStream_t st);
bool attn_tc_supported(const AttnArgs& a, int dtype);
int launch_attn_tc(const AttnArgs& a, int dtype, void* workspace, size_t ws_bytes, cudaStream_t st,
                   const PeerLaunch* peers = nullptr);
size_t attn_tc_workspace(const AttnArgs& a);
void attn_tc_plan(const AttnArgs& a, int32_t* splits, int32_t* launches);
// CTA-pair kernel (attn_pair.cu): whole units only, no workspace.
bool attn_pair_supported(const AttnArgs& a, int dtype);
int attn_pair_plan(const AttnArgs& a, int dtype, int* pairs, int* units);
int launch_attn_pair(const AttnArgs& a, int dtype, cudaStream_t st);

}  // namespace gorgon
