/*
 * gorgon_b200.h - C ABI of the B200 (sm_100a) tree-verification library.
 *
 * One shared library (libgorgon_b200.so) exports the entry points below.  They
 * take plain device pointers, element strides and sizes, and a CUDA stream
 * passed as `void*` (a cudaStream_t; NULL is the legacy default stream).  Every
 * entry point is stream-ordered and asynchronous unless stated otherwise, and
 * returns a gorgon_status (0 = ok).  On error, gorgon_last_error() returns a
 * message for the calling thread.  The library never allocates device memory
 * behind the caller's back: kernels that need scratch space take a caller-owned
 * workspace whose size the matching *_workspace_size() function reports.
 *
 * Each entry point replaces one operator of ProjectGorgon's Python surface;
 * the reference interface is cited beside it (paths are inside that project).
 */
#ifndef GORGON_B200_H_
#define GORGON_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GORGON_API __attribute__((visibility("default")))
#else
#define GORGON_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GORGON_ABI_VERSION 1

typedef enum {
  GORGON_OK = 0,
  GORGON_ERR_INVALID = 1,     /* bad argument: shape, stride, dtype, null pointer */
  GORGON_ERR_UNSUPPORTED = 2, /* valid request this build cannot run */
  GORGON_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  GORGON_ERR_WORKSPACE = 4    /* workspace missing or smaller than required */
} gorgon_status;

typedef enum {
  GORGON_F32 = 0,
  GORGON_BF16 = 1,
  GORGON_F16 = 2
} gorgon_dtype;

/* How the tree rows of each sequence are masked. */
typedef enum {
  GORGON_MASK_PARENTS = 0,   /* ancestor walk over parents[]; prefix rows visible */
  GORGON_MASK_DENSE = 1,     /* mask[n, mask_cols]; mask_cols == kv length of the sequence */
  GORGON_MASK_DENSE_TREE = 2 /* mask[n, n] over the tree rows; prefix rows visible */
} gorgon_mask_kind;

typedef enum {
  GORGON_BACKEND_AUTO = 0,   /* tensor cores when the shape allows, else CUDA cores */
  GORGON_BACKEND_SIMT = 1,   /* CUDA-core split-K kernel (any head_dim <= 256, f32/bf16/f16) */
  GORGON_BACKEND_TCGEN05 = 2, /* tcgen05 kernels (bf16/f16, head_dim 128); the planner picks the shape */
  GORGON_BACKEND_TCGEN05_PAIR = 3, /* tcgen05 on CTA pairs (cta_group::2): whole 256-row units, uniform
                                      kv length, 16-bit output rows of whole 16-byte chunks */
  GORGON_BACKEND_TCGEN05_CTA = 4   /* tcgen05 on single CTAs (any tcgen05-capable shape) */
} gorgon_backend;

/* ABI version compiled into the library (GORGON_ABI_VERSION). */
GORGON_API int gorgon_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
GORGON_API const char* gorgon_last_error(void);

/* Reads (synchronously) the device-side error word of the current device:
 * bit 0 = a parents[] entry outside [-1, n) was met, bit 1 = a KV-trim index
 * outside the cache, bit 2 = a verifier tree/draft entry out of range, bit 3 =
 * a sequence shorter than its tree, bit 4 = a bounded wait inside a
 * tensor-core kernel ran out (the kernel stopped early and its outputs are
 * incomplete), bit 5 = a candidate tree was cut at max_nodes.  The offending
 * element is skipped, never dereferenced.  clear != 0 resets it. */
GORGON_API int gorgon_device_error(uint32_t* out_flags, int clear);

/* Sets the bound on every wait inside the tensor-core kernels (mbarrier
 * waits on copies, MMAs and other warps), in nanoseconds of the GPU's global
 * timer, for the whole process; ns <= 0 leaves it unchanged.  Returns the
 * previous bound.  Default 2 s: far above any wait of a working kernel, so
 * that only a stuck wait (a lost copy, a broken barrier) runs out; the CTA
 * then stops, drains what it issued, frees its tensor memory and raises
 * bit 4 of the device error word instead of hanging.  A very short bound
 * makes ordinary waits run out too, which is how the test suite exercises
 * that path.  No counterpart in the reference (its kernels have no waits). */
GORGON_API int64_t gorgon_set_wait_limit_ns(int64_t ns);

/* ------------------------------------------------------------------------
 * Tree mask.  Replaces build_tree_mask(parents, depth)
 * (src/gorgon/kernels/tree_mask.py:16-44) and candidate_tree_to_mask
 * (src/gorgon/inference/tree_candidates.py:248-279).
 * out[b, i, j] = 1 iff j == i or j is within `depth` parent hops above i
 * (depth < 0 means n hops, the reference's default).  parents: int32
 * [batch, n] with row stride parents_stride_b (0 = one tree for all rows);
 * out: uint8 [batch, n, n] contiguous.  n <= 32768.
 * ---------------------------------------------------------------------- */
GORGON_API int gorgon_tree_mask(const int32_t* parents, int64_t batch, int64_t n,
                     int64_t parents_stride_b, int64_t depth, uint8_t* out,
                     void* stream);

/* ------------------------------------------------------------------------
 * Tree attention over [prefix | tree] key/value rows.
 *
 * Replaces tree_attention_ref / tree_attention_triton / tree_attention_cuda
 * (src/gorgon/kernels/tree_attention_ref.py:8-18,
 * tree_attention_triton.py:86-127, tree_attention_cuda.py:24-38 ->
 * kernels/cuda/tree_attention.cpp:12-46) when mask_kind is DENSE or
 * DENSE_TREE, and fused_tree_verify (fused_tree_verify_triton.py:110-172)
 * when mask_kind is PARENTS.  The reference is one 2-D head; this call adds
 * batch, grouped-query heads (query head h reads kv head h / (heads_q /
 * heads_kv)), a key/value prefix and ragged sequences.
 *
 * Layouts (strides in elements, head_dim contiguous):
 *   q   [batch, heads_q,  n_tree, head_dim]
 *   k,v [batch, heads_kv, kv_len, head_dim]    (kv_len = prefix + n_tree)
 *   out [batch, heads_q,  n_tree, head_dim]    (dtype out_dtype)
 * With cu_seqlens (int32 [batch+1], device) sequence b owns kv rows
 * [cu_seqlens[b], cu_seqlens[b+1]) addressed as row * k_stride_s (the batch
 * stride is ignored); kv_len is then the largest sequence length.  The tree
 * is always the last n_tree rows of a sequence.
 *
 * out = softmax(q k^T * scale + mask) v, scale = 1/sqrt(head_dim) when
 * scale == 0.  A row with no visible key yields NaN (as torch.softmax does).
 * lse (optional, float [batch, heads_q, n_tree]) receives the natural-log
 * sum of exponentials of the scaled, masked scores.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t dtype;      /* gorgon_dtype of q, k, v */
  int32_t out_dtype;  /* gorgon_dtype of out */
  int64_t batch, heads_q, heads_kv, n_tree, kv_len, head_dim;
  const void* q;  int64_t q_stride_b, q_stride_h, q_stride_n;
  const void* k;  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v;  int64_t v_stride_b, v_stride_h, v_stride_s;
  void* out;      int64_t o_stride_b, o_stride_h, o_stride_n;
  const int32_t* cu_seqlens;      /* nullable */
  int32_t mask_kind;              /* gorgon_mask_kind */
  const int32_t* parents;         /* PARENTS: int32 [batch, n_tree] */
  int64_t parents_stride_b;       /*   0 = one tree shared by the batch */
  int32_t max_depth;              /*   hops walked; < 0 = n_tree */
  const uint8_t* mask;            /* DENSE*: uint8/bool [batch, n_tree, mask_cols] */
  int64_t mask_stride_b, mask_stride_n;
  float scale;
  float* lse;                     /* nullable */
  int32_t backend;                /* gorgon_backend */
  int32_t num_splits;             /* key/value splits (CUDA-core kernel) or CTAs
                                     (tcgen05 kernel); 0 = chosen by the library */
  int64_t kv_rows;                /* with cu_seqlens: rows of k and v (0 = unknown, which
                                     keeps ragged batches on the CUDA-core kernel) */
} gorgon_tree_attn_params;

GORGON_API size_t gorgon_tree_attn_workspace_size(const gorgon_tree_attn_params* p);
GORGON_API int gorgon_tree_attn(const gorgon_tree_attn_params* p, void* workspace,
                     size_t workspace_bytes, void* stream);
/* The launch plan gorgon_tree_attn would use for `p`: backend (gorgon_backend
 * value actually run), key/value splits, and kernel launches per call. */
GORGON_API int gorgon_tree_attn_plan(const gorgon_tree_attn_params* p, int32_t* backend,
                          int32_t* splits, int32_t* launches);

/* ------------------------------------------------------------------------
 * A layer split by kv head over the GPUs of one node (NVLink peers), with the
 * output gather fused into the attention kernel.  No counterpart in the
 * reference, which runs on one GPU; this replaces an all-gather of the
 * layer's output after tree attention.
 *
 * Every rank allocates a buffer of the same size with
 * gorgon_peer_buffer_alloc (device memory of the current device, zeroed), passes the
 * 64-byte handle to the other ranks (any host channel), and opens theirs with
 * gorgon_peer_buffer_open.  Each buffer holds the layer's output (the same
 * layout on every rank) and, at signal_offset, four zeroed uint64 words of
 * signal state.  A gorgon_peer_group lists every rank's buffer
 * as seen from this rank (base[rank] is this rank's own).
 *
 * gorgon_tree_attn_gather runs gorgon_tree_attn with p->out pointing into
 * base[rank].  The tensor-core kernel's epilogue writes each output row there
 * and, at the same byte offset, into every other rank's buffer (stores over
 * NVLink).  It writes into a peer's buffer only once that peer's stream has
 * reached the same call, so the peer's earlier readers of the buffer are done.
 * A one-CTA kernel then waits on the stream, without the host, until every
 * peer's rows have landed here.  All ranks
 * must make the same calls with the same shapes, in the same order.  The
 * counters only grow, so the calls can be captured in a CUDA graph and
 * replayed.  Every wait is bounded (gorgon_set_wait_limit_ns).  A wait that
 * runs out (a peer that never calls) raises bit 4 of the device error word.
 * The outputs are then incomplete and the group must be rebuilt.
 * Needs the tcgen05 single-CTA kernel, bf16/f16 output rows of whole
 * 16-byte chunks, and a plan without a separate merge launch (whole units
 * or cluster plans).  Otherwise it returns GORGON_ERR_UNSUPPORTED, and the
 * caller gathers some other way.
 * ---------------------------------------------------------------------- */
#define GORGON_MAX_PEERS 8
typedef struct {
  unsigned char bytes[64];
} gorgon_ipc_handle;

GORGON_API int gorgon_peer_buffer_alloc(size_t bytes, void** ptr, gorgon_ipc_handle* handle);
GORGON_API int gorgon_peer_buffer_open(const gorgon_ipc_handle* handle, void** ptr);
GORGON_API int gorgon_peer_buffer_close(void* peer_ptr);
GORGON_API int gorgon_peer_buffer_free(void* ptr);

typedef struct {
  int32_t world;                    /* ranks, 1 .. GORGON_MAX_PEERS */
  int32_t rank;                     /* this rank */
  void* base[GORGON_MAX_PEERS];     /* every rank's buffer as mapped here */
  int64_t signal_offset;            /* byte offset of the 4 signal words (8-byte aligned); the
                                       output must lie wholly before it, or the call is refused */
} gorgon_peer_group;

GORGON_API int gorgon_tree_attn_gather(const gorgon_tree_attn_params* p, const gorgon_peer_group* g,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Fused tree verifier: per-row argmax over the vocabulary, draft match and
 * longest accepted path in one launch, with no host synchronisation.
 * Replaces the vectorised verifier of _verify_tree_candidates
 * (src/gorgon/inference/gorgon_loop.py:328-392, paths from
 * get_tree_paths, src/gorgon/inference/tree_candidates.py:282-311) and, for a
 * chain tree, accept_draft_tokens (gorgon_loop.py:161-184).
 *
 * Rows: node t is checked against the argmax of row prompt_len - 1 when it is
 * a root (parent -1) and of row prompt_len + parent otherwise.  The winner is
 * the first root-to-leaf path in DFS order (roots ascending, children in index
 * order) with the longest accepted prefix; bonus = argmax of row
 * prompt_len + last accepted node, or of row prompt_len - 1 when nothing is
 * accepted (-1 if that row is beyond `rows`).  argmax returns the first index
 * of the maximum; NaN counts as the maximum.
 *
 * logits [batch, rows, vocab] (vocab contiguous); draft, parents int32
 * [batch, n] (parents_stride_b 0 = shared tree).  Outputs (int32, device):
 * pred [batch, n + 1] = argmax of rows prompt_len - 1 + j (-1 past `rows`),
 * accepted_len [batch], path [batch, n] (winning nodes from the root, -1
 * padded), bonus [batch], best_node [batch] (-1 if none), hidden_row [batch]
 * (nullable).  n <= 4096.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t dtype;  /* gorgon_dtype of logits */
  const void* logits; int64_t logits_stride_b, logits_stride_r;
  int64_t batch, rows, vocab, n, prompt_len;
  const int32_t* draft;   int64_t draft_stride_b;
  const int32_t* parents; int64_t parents_stride_b;
  int32_t* pred;
  int32_t* accepted_len;
  int32_t* path;
  int32_t* bonus;
  int32_t* best_node;
  int32_t* hidden_row;
} gorgon_verify_params;

GORGON_API size_t gorgon_verify_workspace_size(const gorgon_verify_params* p);
GORGON_API int gorgon_verify(const gorgon_verify_params* p, void* workspace,
                  size_t workspace_bytes, void* stream);

/* The fused verifier above for callers that cannot allocate device memory.
 * No counterpart in the reference (its verifier is torch code).
 *
 * Some callers cannot call cudaMalloc: host runtimes that only receive the
 * buffers an owning framework hands them (a cgo/JNI host, a serving engine
 * whose memory comes from a fixed arena), or code that must not add a
 * synchronising allocation to its decode step.  This entry point takes the
 * same inputs and outputs as gorgon_verify but no workspace: its scratch (one
 * arrival counter per sequence) is a 16 KiB array compiled into the library,
 * held by every GPU that loads it until the process exits.
 *
 * - batch may be at most 4096; larger batches return GORGON_ERR_UNSUPPORTED.
 * - The first call on a device looks up the array's address on that device
 *   (with it current); make that first call before any stream capture.
 * - Every call clears the counters it uses on `stream` first.  All calls
 *   share the one array, so calls that overlap on the GPU (on different
 *   streams at the same time) race; keep them ordered on one stream.
 * - The looked-up address is kept for the life of the process: the library
 *   must not outlive a reset of the device (cudaDeviceReset, or the primary
 *   context torn down and created again); call nothing here after one.
 * - It allocates nothing: no cudaMalloc, cudaFree or allocating routine. */
GORGON_API int gorgon_verify_noalloc(const gorgon_verify_params* p, void* stream);

/* ------------------------------------------------------------------------
 * KV-cache trim-on-reject for all layers in one launch.  Replaces
 * apply_cache_slice (src/gorgon/inference/kv_cache.py:89-108) and the
 * cache crop after verification (src/gorgon/inference/gorgon_loop.py:569-570,
 * kv_cache.py:72-80):
 *   dst[l][b, h, dst_start[b] + r] = src[l][b, h, src_idx[b, r]],  r < lens[b]
 * for every layer l, batch row b, kv head h, on caches laid out
 * [batch, heads, seq_capacity, head_dim] (strides in elements, head_dim
 * contiguous, identical for every layer and for K and V).  k_src / v_src are
 * HOST arrays of `layers` device pointers; k_dst / v_dst likewise, or NULL to
 * trim in place (all rows of a (layer, b, h) slice are read before any is
 * written, so in-place gathers whose source and destination rows overlap
 * are safe).  src_idx int32 [batch, max_len] (row stride idx_stride_b),
 * lens int32 [batch], dst_start int32 [batch] or NULL for 0: device arrays,
 * so a verifier's output can feed this call without a host round trip.
 * max_len <= 256.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t elem_bytes;  /* 1, 2, 4 or 8 */
  int64_t layers, batch, heads, seq_capacity, head_dim;
  int64_t stride_b, stride_h, stride_s;
  void* const* k_src; void* const* v_src;
  void* const* k_dst; void* const* v_dst;
  const int32_t* src_idx; int64_t idx_stride_b, max_len;
  const int32_t* lens;
  const int32_t* dst_start;
} gorgon_kv_trim_params;

GORGON_API int gorgon_kv_trim(const gorgon_kv_trim_params* p, void* stream);

/* ------------------------------------------------------------------------
 * Candidate-tree builder.  Replaces build_candidate_tree
 * (src/gorgon/inference/tree_candidates.py:92-245) with its per-head
 * statistics _topk_per_head (:42-81), once the Medusa heads have produced
 * their logits: logits[b, l, :] is the vocabulary row of head l (tree level
 * l + 1) for sequence b.
 *
 * Per row: the min(top_k, vocab) largest logits (descending; equal logits by
 * ascending id), the softmax over them, and the entropy of the softmax over
 * the whole row.  Per sequence, the reference's expansion: head 0's
 * candidates become roots; each later level gives every node of the level
 * above (in order of that node's own logit, descending and stable, when
 * max_candidates >= 0; in node order otherwise) one child per candidate of
 * the level's head, in top-k order.  A candidate is skipped when its
 * probability -- or, with use_path_confidence, the product of probabilities
 * along its path -- is below the level's threshold: confidence_threshold
 * (0 = off), times 1 - entropy / ln(top_k) when entropy_weighted.  Nodes are
 * added until max_candidates exist (< 0: no budget).
 *
 * logits [batch, levels, vocab] (vocab contiguous; finite values).  Outputs,
 * in node order: tokens int64 [batch, max_nodes], parents int32 [batch,
 * max_nodes] (-1 = root), probs float [batch, max_nodes], n_nodes int32
 * [batch]; slots from n_nodes[b] on hold -1 / -1 / 0.  A tree that would
 * outgrow max_nodes is cut there and sets device error bit 3.  topk_ids
 * int32, topk_scores and topk_probs float [batch, levels, top_k] and entropy
 * float [batch, levels] receive the per-row statistics when non-NULL (the
 * workspace holds them otherwise).  The workspace of
 * gorgon_candidate_tree_workspace_size() bytes is always required: it also
 * holds every vocabulary segment's partial results.  The entropy is
 * ln Z - sum(e^x (x - max)) / Z, the reference's -sum p log(p + 1e-10)
 * without the 1e-10 (at most ~1e-5 apart for a 128k vocabulary).
 * top_k <= 32, levels <= 64, max_nodes <= 4096.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t dtype;  /* gorgon_dtype of logits */
  const void* logits; int64_t logits_stride_b, logits_stride_l;
  int64_t batch, levels, vocab;
  int32_t top_k;
  int32_t max_candidates;
  float confidence_threshold;
  int32_t use_path_confidence, entropy_weighted;
  int64_t max_nodes;
  int64_t* tokens;
  int32_t* parents;
  float* probs;
  int32_t* n_nodes;
  int32_t* topk_ids;
  float* topk_scores;
  float* topk_probs;
  float* entropy;
} gorgon_candidate_tree_params;

GORGON_API size_t gorgon_candidate_tree_workspace_size(const gorgon_candidate_tree_params* p);
GORGON_API int gorgon_candidate_tree(const gorgon_candidate_tree_params* p, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Candidate trees straight from the Medusa heads' last Linear.  Replaces
 * MedusaHead.forward's lm_head (src/gorgon/models/medusa_heads.py:42-47)
 * followed by _topk_per_head (src/gorgon/inference/tree_candidates.py:42-81)
 * and the expansion of build_candidate_tree (:92-245): the outputs and rules
 * are gorgon_candidate_tree's, with
 *   logits[b, l, v] = sum_i hidden[b, l, i] * lm_head[l][v, i]
 * accumulated in fp32 and rounded to tree.dtype (the dtype the Linear would
 * return) inside the kernel; the logits are never written to memory, and
 * tree.logits and its strides are ignored.  A logit may differ from a
 * library GEMM's by one rounding step of tree.dtype (summation order).
 *
 * hidden [batch, levels, hidden_size]: the input of head l's lm_head (after
 * its norm and residual blocks) for sequence b.  lm_head: a HOST array of
 * `levels` device pointers, head l's weight [vocab, hidden_size] with rows
 * lm_head_stride_v elements apart.  hidden and the weights are x_dtype
 * (GORGON_BF16 or GORGON_F16), 16-byte aligned, with hidden_size and every
 * stride a multiple of 8.  batch <= 4 (above that the dot products outrun
 * the CUDA cores: use a GEMM and gorgon_candidate_tree), hidden_size <= 8192,
 * levels <= 64.  The workspace of gorgon_head_candidate_tree_workspace_size()
 * bytes is always required.
 * ---------------------------------------------------------------------- */
typedef struct {
  gorgon_candidate_tree_params tree;
  int32_t x_dtype;
  const void* hidden; int64_t hidden_stride_b, hidden_stride_l;
  int64_t hidden_size;
  const void* const* lm_head; int64_t lm_head_stride_v;
} gorgon_head_candidate_params;

GORGON_API size_t gorgon_head_candidate_tree_workspace_size(const gorgon_head_candidate_params* p);
GORGON_API int gorgon_head_candidate_tree(const gorgon_head_candidate_params* p, void* workspace,
                                          size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GORGON_B200_H_ */
