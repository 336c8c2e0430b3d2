// gorgon_tree_attn: argument checking, kernel choice and workspace layout.
#include <string>

#include "attn.cuh"

namespace gorgon {
namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Fills `a` from the public parameters; returns GORGON_OK or an error code.
int make_args(const gorgon_tree_attn_params* p, AttnArgs* a) {
  if (!p) return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: params is null");
  if (!dtype_ok(p->dtype) || !dtype_ok(p->out_dtype))
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: unknown dtype");
  if (p->batch < 0 || p->heads_q < 0 || p->heads_kv < 0 || p->n_tree < 0 || p->kv_len < 0 ||
      p->head_dim < 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: negative size");
  if (p->heads_kv == 0 || p->heads_q % p->heads_kv != 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: heads_q must be a multiple of heads_kv");
  if (p->head_dim > 256)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: head_dim > 256");
  if (p->batch > 65535 || p->batch * p->heads_kv > 65535 || p->heads_q > 4096)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: batch * heads_kv > 65535");
  if (p->kv_len > (int64_t(1) << 30) || p->n_tree > 65536)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: sequence too long");
  if (p->mask_kind != GORGON_MASK_PARENTS && p->mask_kind != GORGON_MASK_DENSE &&
      p->mask_kind != GORGON_MASK_DENSE_TREE)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: unknown mask_kind");
  const bool tree_mode = p->mask_kind != GORGON_MASK_DENSE;
  if ((p->heads_q / p->heads_kv) * p->n_tree > int64_t(65535) * 32)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: (heads_q / heads_kv) * n_tree > 2097120");
  if (tree_mode && p->n_tree > 1024)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: trees above 1024 nodes need a dense mask");
  if (tree_mode && !p->cu_seqlens && p->kv_len < p->n_tree)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: kv_len < n_tree (the tree rows are the last n_tree kv rows)");
  const int64_t work = p->batch * p->heads_q * p->n_tree * p->head_dim;
  if (work > 0) {
    if (!p->q || !p->k || !p->v || !p->out)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: null q/k/v/out");
    if (p->mask_kind == GORGON_MASK_PARENTS && !p->parents)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: mask_kind PARENTS needs parents");
    if (p->mask_kind != GORGON_MASK_PARENTS && !p->mask)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: dense mask_kind needs mask");
    if (p->kv_len == 0 && !p->cu_seqlens)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: kv_len == 0");
  }
  if (p->backend < GORGON_BACKEND_AUTO || p->backend > GORGON_BACKEND_TCGEN05_CTA)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: unknown backend");
  if (p->num_splits < 0 || p->num_splits > 1024)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn: num_splits outside [0, 1024]");

  AttnArgs& x = *a;
  x = AttnArgs{};
  x.q = p->q; x.k = p->k; x.v = p->v; x.out = p->out;
  x.q_sb = p->q_stride_b; x.q_sh = p->q_stride_h; x.q_sn = p->q_stride_n;
  x.k_sb = p->k_stride_b; x.k_sh = p->k_stride_h; x.k_ss = p->k_stride_s;
  x.v_sb = p->v_stride_b; x.v_sh = p->v_stride_h; x.v_ss = p->v_stride_s;
  x.o_sb = p->o_stride_b; x.o_sh = p->o_stride_h; x.o_sn = p->o_stride_n;
  x.cu_seqlens = p->cu_seqlens;
  x.kv_rows = p->cu_seqlens ? p->kv_rows : 0;
  x.parents = p->parents; x.par_sb = p->parents_stride_b;
  x.mask = p->mask; x.mask_sb = p->mask_stride_b; x.mask_sn = p->mask_stride_n;
  x.lse = p->lse;
  x.err = device_error_word();
  x.batch = static_cast<int>(p->batch);
  x.hq = static_cast<int>(p->heads_q);
  x.hkv = static_cast<int>(p->heads_kv);
  x.group = x.hkv ? x.hq / x.hkv : 1;
  x.n = static_cast<int>(p->n_tree);
  x.kv_len = static_cast<int>(p->kv_len);
  x.d = static_cast<int>(p->head_dim);
  x.mask_kind = p->mask_kind;
  x.max_depth = p->max_depth < 0 ? x.n : p->max_depth;
  x.out_dtype = p->out_dtype;
  x.splits = p->num_splits;  // tensor-core grid request; the CUDA-core path sets its own
  const float scale = p->scale != 0.f ? p->scale : (x.d > 0 ? 1.f / std::sqrt(static_cast<float>(x.d)) : 1.f);
  x.scale_log2 = scale * 1.4426950408889634f;
  const int ev = static_cast<int>(16 / dtype_bytes(p->dtype));
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  x.vec_ok = al(p->q) && al(p->k) && al(p->v) && x.d % ev == 0 && p->q_stride_b % ev == 0 &&
             p->q_stride_h % ev == 0 && p->q_stride_n % ev == 0 && p->k_stride_b % ev == 0 &&
             p->k_stride_h % ev == 0 && p->k_stride_s % ev == 0 && p->v_stride_b % ev == 0 &&
             p->v_stride_h % ev == 0 && p->v_stride_s % ev == 0;
  return GORGON_OK;
}

enum class Kernel { kSimt, kTcCta, kTcPair, kNone };

// The planner does not pick the CTA-pair kernel: measured on B200 it is
// slower than the single-CTA kernel on every shape tried (16 x 8192 layer
// 205 us against 144; 2 x 8192 102 against 34), because each of its
// 128-key tiles puts a 16K-score softmax on four warps and a cross-SM
// arrival on the critical path.  It stays available as backend
// GORGON_BACKEND_TCGEN05_PAIR.
bool pair_preferred(const AttnArgs&, int) { return false; }

Kernel choose(const gorgon_tree_attn_params* p, const AttnArgs& a) {
  switch (p->backend) {
    case GORGON_BACKEND_SIMT:
      return Kernel::kSimt;
    case GORGON_BACKEND_TCGEN05_PAIR:
      return attn_pair_supported(a, p->dtype) ? Kernel::kTcPair : Kernel::kNone;
    case GORGON_BACKEND_TCGEN05_CTA:
      return attn_tc_supported(a, p->dtype) ? Kernel::kTcCta : Kernel::kNone;
    default:
      break;
  }
  const bool tc = attn_tc_supported(a, p->dtype);
  // Auto: tensor cores once the packed (group x tree) rows fill an MMA tile.
  if (p->backend == GORGON_BACKEND_AUTO && !(tc && a.n >= 64)) return Kernel::kSimt;
  if (!tc) return p->backend == GORGON_BACKEND_TCGEN05 ? Kernel::kNone : Kernel::kSimt;
  return pair_preferred(a, p->dtype) ? Kernel::kTcPair : Kernel::kTcCta;
}

int simt_splits(const gorgon_tree_attn_params* p, const AttnArgs& a) {
  if (p->num_splits > 0) return static_cast<int>(p->num_splits);
  const int64_t qtiles = (static_cast<int64_t>(a.group) * a.n + 31) / 32;
  const int64_t base = static_cast<int64_t>(a.batch) * a.hkv * qtiles;
  const int64_t target = 4LL * sm_count();
  int64_t s = (target + base - 1) / std::max<int64_t>(base, 1);
  const int64_t max_by_len = std::max<int64_t>(1, (static_cast<int64_t>(a.kv_len) + 63) / 64);
  s = std::min<int64_t>(s, max_by_len);
  s = std::min<int64_t>(s, 64);
  return static_cast<int>(std::max<int64_t>(s, 1));
}

size_t simt_workspace(const AttnArgs& a, int splits) {
  if (splits <= 1) return 0;
  const size_t rows = static_cast<size_t>(a.batch) * a.hq * a.n;
  return align_up(static_cast<size_t>(splits) * rows * a.d * sizeof(float)) +
         align_up(static_cast<size_t>(splits) * rows * sizeof(float));
}

}  // namespace
}  // namespace gorgon

extern "C" size_t gorgon_tree_attn_workspace_size(const gorgon_tree_attn_params* p) {
  using namespace gorgon;
  AttnArgs a;
  if (make_args(p, &a) != GORGON_OK) return 0;
  switch (choose(p, a)) {
    case Kernel::kTcCta: return attn_tc_workspace(a);
    case Kernel::kTcPair:
    case Kernel::kNone: return 0;
    default: return simt_workspace(a, simt_splits(p, a));
  }
}

extern "C" int gorgon_tree_attn_plan(const gorgon_tree_attn_params* p, int32_t* backend,
                                     int32_t* splits, int32_t* launches) {
  using namespace gorgon;
  AttnArgs a;
  int rc = make_args(p, &a);
  if (rc) return rc;
  int32_t be, sp, ln;
  switch (choose(p, a)) {
    case Kernel::kTcCta:
      be = GORGON_BACKEND_TCGEN05;
      attn_tc_plan(a, &sp, &ln);
      break;
    case Kernel::kTcPair: {
      int pairs = 0, units = 0;
      rc = attn_pair_plan(a, p->dtype, &pairs, &units);
      if (rc) return rc;
      be = GORGON_BACKEND_TCGEN05_PAIR;
      sp = 2 * pairs;  // CTAs
      ln = 1;
      break;
    }
    case Kernel::kNone:
      return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn_plan: the requested tcgen05 kernel does not take this shape");
    default:
      be = GORGON_BACKEND_SIMT;
      sp = simt_splits(p, a);
      ln = sp > 1 ? 2 : 1;
  }
  if (backend) *backend = be;
  if (splits) *splits = sp;
  if (launches) *launches = ln;
  return GORGON_OK;
}

extern "C" int gorgon_tree_attn(const gorgon_tree_attn_params* p, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace gorgon;
  AttnArgs a;
  int rc = make_args(p, &a);
  if (rc) return rc;
  if (static_cast<int64_t>(a.batch) * a.hq * a.n * a.d == 0) return GORGON_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Kernel k = choose(p, a);
  if (k == Kernel::kTcPair) return launch_attn_pair(a, p->dtype, st);
  if (k == Kernel::kTcCta) {
    const size_t need = attn_tc_workspace(a);
    if (need > 0 && (!workspace || workspace_bytes < need))
      return set_error(GORGON_ERR_WORKSPACE, "gorgon_tree_attn: workspace smaller than gorgon_tree_attn_workspace_size()");
    return launch_attn_tc(a, p->dtype, workspace, workspace_bytes, st);
  }
  if (k == Kernel::kNone) {
    if (p->backend == GORGON_BACKEND_TCGEN05_PAIR)
      return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: the tcgen05 pair kernel needs bf16/f16, head_dim 128, a tree mask, "
                                               "one kv length (no cu_seqlens) and 16-bit output rows of whole 16-byte chunks");
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn: tcgen05 backend needs bf16/f16, head_dim 128, a tree mask and f32/bf16/f16 output");
  }
  a.splits = simt_splits(p, a);
  const size_t need = simt_workspace(a, a.splits);
  if (need > 0) {
    if (!workspace || workspace_bytes < need)
      return set_error(GORGON_ERR_WORKSPACE, "gorgon_tree_attn: workspace smaller than gorgon_tree_attn_workspace_size()");
    const size_t rows = static_cast<size_t>(a.batch) * a.hq * a.n;
    a.part_o = static_cast<float*>(workspace);
    a.part_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                          align_up(static_cast<size_t>(a.splits) * rows * a.d * sizeof(float)));
  }
  rc = launch_attn_simt(a, p->dtype, st);
  if (rc) return rc;
  if (a.splits > 1) rc = launch_attn_combine(a, st);
  return rc;
}

extern "C" int gorgon_tree_attn_gather(const gorgon_tree_attn_params* p, const gorgon_peer_group* g,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  using namespace gorgon;
  if (!p || !g) return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: null argument");
  if (g->world < 1 || g->world > GORGON_MAX_PEERS || g->rank < 0 || g->rank >= g->world)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: world must be 1..8 and rank in [0, world)");
  if (g->world == 1) return gorgon_tree_attn(p, workspace, workspace_bytes, stream);
  if (g->signal_offset < 0 || g->signal_offset % 8 != 0)
    return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: signal_offset must be a non-negative multiple of 8");
  for (int r = 0; r < g->world; ++r)
    if (!g->base[r]) return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: a rank's buffer is null");
  const char* own = static_cast<const char*>(g->base[g->rank]);
  const char* out = static_cast<const char*>(p->out);
  if (out < own) return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: out does not point into this rank's buffer");
  const int64_t off = out - own;
  {
    // every output element (and so its copy in each peer's buffer) must lie
    // in the data region, before the signal words
    const int64_t esz = p->out_dtype == GORGON_F32 ? 4 : 2;
    if (p->o_stride_b < 0 || p->o_stride_h < 0 || p->o_stride_n < 0)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: negative output strides");
    const int64_t last = (p->batch - 1) * p->o_stride_b + (p->heads_q - 1) * p->o_stride_h +
                         (p->n_tree - 1) * p->o_stride_n + p->head_dim;
    if (p->batch > 0 && p->heads_q > 0 && p->n_tree > 0 && off + last * esz > g->signal_offset)
      return set_error(GORGON_ERR_INVALID, "gorgon_tree_attn_gather: out reaches past the buffer's data region "
                                           "(signal_offset)");
  }
  AttnArgs a;
  int rc = make_args(p, &a);
  if (rc) return rc;
  if (static_cast<int64_t>(a.batch) * a.hq * a.n * a.d == 0) return GORGON_OK;
  if (choose(p, a) != Kernel::kTcCta)
    return set_error(GORGON_ERR_UNSUPPORTED, "gorgon_tree_attn_gather: the fused gather runs on the tcgen05 "
                                             "single-CTA kernel (bf16/f16, head_dim 128, a tree mask)");
  const size_t need = attn_tc_workspace(a);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return set_error(GORGON_ERR_WORKSPACE, "gorgon_tree_attn_gather: workspace smaller than gorgon_tree_attn_workspace_size()");
  PeerLaunch pl{};
  for (int r = 0; r < g->world; ++r) {
    char* b = static_cast<char*>(g->base[r]);
    uint64_t* sig = reinterpret_cast<uint64_t*>(b + g->signal_offset);
    if (r == g->rank) {
      pl.sig = sig;
    } else {
      pl.peer_out[pl.npeers] = b + off;
      pl.peer_sig[pl.npeers] = sig;
      ++pl.npeers;
    }
  }
  return launch_attn_tc(a, p->dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), &pl);
}
