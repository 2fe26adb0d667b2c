/*
 * cast_b200: C ABI of the B200 (sm_100a) ragged tree-verification path.
 *
 * Replaces, behind a plain C interface (device pointers, sizes, a stream):
 *   - cast_trees/tree_attn.py:116-139  varlen_tree_attention (host wrapper)
 *   - cast_trees/tree_attn.py:17-92    _tree_attn_fwd (the Triton kernel)
 *   - cast_trees/tree_attn.py:104-113  _tile_schedule (host tile list + D2H sync)
 *   - cast_trees/tree.py:20-26         block_topk
 *   - cast_trees/tree.py:29-49         build_tree
 *   - cast_trees/serving.py:213-222    packed tok/pos/ancestor layout of one verify pass
 *   - cast_trees/serving.py:60-71      per-layer ragged K/V assembly (store-mode attention)
 *   - cast_trees/decode.py:85-103      walk_tree at temperature 0 (greedy walk)
 *   - cast_trees/tree.py:63-82         select_global_topk
 *   - cast_trees/serving.py:264-289    BatchedServer._append_store
 *   - cast_trees/verify.py:48-60       gather_cache
 *
 * Conventions shared by every entry point:
 *   - All array arguments are DEVICE pointers owned by the caller. The library
 *     allocates nothing per call; scratch space is passed in as `workspace`.
 *   - Work is enqueued on `stream` (a cudaStream_t / CUstream; NULL = the legacy
 *     default stream) and is asynchronous: a return of CAST_OK means the
 *     launch was accepted.
 *   - Negative return codes are argument errors found on the host before any
 *     launch. Kernels that find inconsistent device-side metadata skip the bad
 *     unit and record a positive code in a per-device error word; read (and
 *     clear) it with cast_device_error(), which synchronises the stream.
 *   - No entry point aborts, traps or prints.
 *   - Entry points are re-entrant; concurrent calls on different streams must
 *     use different workspaces.
 */
#ifndef CAST_B200_H
#define CAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* cast_stream_t;  /* cudaStream_t */

/*
 * element types of q / k / v / out. CAST_F32_SPLIT (no counterpart in the
 * reference) is fp32 data computed on the tensor cores: q, k, v and the
 * softmax probabilities are carried as bf16 hi + lo pairs and every product
 * takes the three significant terms (hi*hi + hi*lo + lo*hi), which keeps the
 * output within ~1e-5 of exact fp32 arithmetic at unit-scale inputs (the
 * reference's fp32 path, tree_attn.py with fp32 copies from serving.py:68-71,
 * is held to 1e-4). CAST_F32 is the exact CUDA-core path.
 */
enum cast_dtype { CAST_F32 = 0, CAST_BF16 = 1, CAST_F16 = 2, CAST_F32_SPLIT = 3 };

enum cast_status {
  CAST_OK = 0,
  CAST_ERR_NULL = -1,         /* a required pointer is NULL */
  CAST_ERR_SHAPE = -2,        /* non-positive size, or H_q % H_kv != 0 */
  CAST_ERR_DTYPE = -3,        /* unknown dtype */
  CAST_ERR_HEAD_DIM = -4,     /* head dim not in {64, 128} */
  CAST_ERR_PACK = -5,         /* max_pack above CAST_MAX_PACK, or anc words too few */
  CAST_ERR_WORKSPACE = -6,    /* workspace smaller than cast_tree_attn_workspace_size() (CAST_F32_SPLIT: _size_kv(), base 256-byte aligned) */
  CAST_ERR_ALIGN = -7,        /* a pointer or stride breaks the kernel's alignment rule */
  CAST_ERR_TOPK = -8,         /* k out of range [1, CAST_MAX_TOPK] or V < k */
  CAST_ERR_LAUNCH = -9,       /* the CUDA launch itself failed */
  CAST_ERR_DEVICE = -10,      /* no usable CUDA device */
  CAST_ERR_MASK_MODE = -11,   /* both or neither of anc_words / parent given */
  CAST_ERR_SCRATCH_LIMIT = -12, /* cast_tree_attn_fwd_noalloc: problem needs more than CAST_NOALLOC_SCRATCH_BYTES */
  /* device-side codes (positive), reported by cast_device_error() */
  CAST_DEV_BAD_LAYOUT = 1,    /* cu/prefix/pack arrays out of range or above max_pack/max_kv */
  CAST_DEV_BAD_PARENT = 2,    /* parent[i] >= i or < -1 (or parent[0] != -1) */
  CAST_DEV_TIMEOUT = 4,       /* a bounded wait inside a kernel gave up */
  CAST_DEV_TREE_OVERFLOW = 5  /* build_tree budget above max_budget */
};

#define CAST_MAX_PACK 1024    /* largest pack (1 + N) the attention kernels accept */
#define CAST_MAX_TOPK 24      /* largest k of block_topk / build_tree */
#define CAST_MAX_DEPTH 64     /* largest L of build_tree */
#define CAST_MAX_SELECT_TREES 12288  /* largest forest of cast_select_global_topk */
#define CAST_MAX_SELECT_NODES 1024   /* largest tree (row width) of cast_select_global_topk */

/* Human-readable text for a status code (never NULL). */
const char* cast_strerror(int status);

/* Library ABI version: 100 * major + minor. */
int cast_version(void);

/*
 * Reads and clears the device error word of the current device after
 * synchronising `stream`. Returns 0 (CAST_OK), a positive CAST_DEV_* code,
 * or CAST_ERR_LAUNCH if the CUDA runtime itself reports an error.
 */
int cast_device_error(cast_stream_t stream);

/*
 * Testing hook (no counterpart in the reference). Sets, for every launch of
 * the tensor-core attention kernel this process makes afterwards, the limit
 * in nanoseconds of the kernel's pipeline waits (a TMA copy or MMA it waits
 * for, a ring slot, a softmax hand-off); 0 restores the default (1 s). With a
 * limit shorter than a copy takes, a wait runs out: the CTA records
 * CAST_DEV_TIMEOUT (read with cast_device_error), lets its in-flight copies
 * and MMAs finish under the full limit, frees its tensor memory and returns,
 * so the failure path can be tested without a hang or a fault. Results of a
 * call that timed out are undefined; later calls are unaffected once the
 * default is restored.
 */
void cast_test_set_wait_limit_ns(uint64_t ns);

/*
 * Testing hook (no counterpart in the reference). Chooses the 16-bit
 * tensor-core attention kernel of the regular-layout cast_tree_attn_fwd calls
 * this process makes afterwards: 1 (default) = CTA pairs (tcgen05
 * cta_group::2, one 256-row block over the two SMs of a TPC) whenever
 * (H_q / H_kv) * max_pack is a multiple of 256; pairs for the full 256-row
 * blocks and single CTAs for the last blocks when it is larger than 256,
 * ends in a one-tile block and the key chunks are long; single CTAs
 * otherwise; 0 = single CTAs always (two 128-row query tiles per SM, the
 * kernel store mode always uses); -1 = the CUDA-core kernel for every dtype
 * (to measure the dispatch). All compute the same function; tests run each
 * against the oracle.
 */
void cast_test_set_tc_kernel(int kernel);

/*
 * Ragged ancestor-masked GQA tree attention, forward.
 * Replaces cast_trees/tree_attn.py:116 varlen_tree_attention and the kernel
 * it launches (tree_attn.py:17-92).
 *
 * Sequence b owns the packed query rows [cu_q[b], cu_q[b] + pack_len[b]) and
 * the key/value rows [cu_kv[b], cu_kv[b] + prefix_len[b] + pack_len[b]): its
 * prefix first, then its pack (tree_attn.py:39-41,71). Query row i of the pack
 * sees every prefix key and pack key j iff bit j of its ancestor bitset is set.
 *
 * q: [total_q, H_q, D], k/v: [total_kv, H_kv, D], out: [total_q, H_q, D]; all
 *   of `dtype` (float32 for CAST_F32_SPLIT); strides[12] = element strides
 *   (row, head, dim) of q, k, v, out. The dim stride must be 1.
 *   CAST_F32_SPLIT needs D = 128, H_q / H_kv dividing 128, row / head strides
 *   that are multiples of 4 and 16-byte aligned bases, and a workspace of
 *   cast_tree_attn_workspace_size_kv() bytes (it holds the bf16 hi / lo copies
 *   of q, k and v, 4 bytes per element of each).
 * anc_words: int64 [total_q, anc_words_per_row] ancestor bitsets (bit j of word
 *   j/64), the reference's `ancestor_mask` when anc_words_per_row == 1; or NULL.
 * parent: int32 [total_q] pack-local parents (-1 for the root, parent[i] < i),
 *   from which the kernel builds the bitsets in shared memory; or NULL.
 *   Exactly one of anc_words / parent is given.
 * max_pack / max_kv: host-side upper bounds of pack_len[b] and
 *   prefix_len[b] + pack_len[b]; they size the launch so no device-to-host
 *   read is needed (the reference reads cu_q back every call, tree_attn.py:128).
 * sm_scale: softmax scale; pass a value <= 0 for the default 1/sqrt(D)
 *   (tree_attn.py:125-126).
 * Rows that see no key are written as 0 (tree_attn.py:89).
 */
int cast_tree_attn_fwd(const void* q, const void* k, const void* v, void* out, int dtype,
                       const int64_t* strides,
                       const int32_t* cu_q, const int32_t* cu_kv,
                       const int32_t* prefix_len, const int32_t* pack_len,
                       const int64_t* anc_words, int anc_words_per_row,
                       const int32_t* parent,
                       int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                       float sm_scale, int max_pack, int max_kv,
                       void* workspace, size_t workspace_bytes, cast_stream_t stream);

/*
 * No counterpart in the reference: an added variant for callers that cannot
 * allocate device memory.
 *
 * Same arguments, meaning and results as cast_tree_attn_fwd, minus the
 * workspace: when the launch splits the key range, the fp32 partial results
 * go to a fixed scratch array that the library itself holds in device memory
 * (CAST_NOALLOC_SCRATCH_BYTES, reserved on every GPU that loads the library
 * and kept until the process exits). It is meant for callers that are not
 * allowed to call cudaMalloc or an allocator at this point: code running
 * under a strict memory budget or a pre-reserved pool, plugin hosts that own
 * all device allocations, or callers on a path where an allocation could
 * block or fail. This call allocates nothing and calls no allocating routine.
 *
 * Limits and rules:
 *   - Problems whose split partials need more than CAST_NOALLOC_SCRATCH_BYTES
 *     (cast_tree_attn_workspace_size() above it) are rejected with
 *     CAST_ERR_SCRATCH_LIMIT before anything is launched.
 *   - The first call on each device looks up the scratch array's device
 *     address (cudaGetSymbolAddress) with that device current; make that first
 *     call before any stream capture begins. The address is kept per context:
 *     after cudaDeviceReset (which unloads the library's module with the
 *     context) the next call sees the new context and looks the address up
 *     again, so that call, too, belongs before any capture.
 *   - Every call on a device shares the one scratch array, which keeps the
 *     last call's contents. Calls whose kernels may overlap on the GPU (other
 *     streams, other host threads) race on it: issue them on one stream, or
 *     order them with events. Nothing in it needs to start at zero: each call
 *     writes every partial it later reads.
 */
#define CAST_NOALLOC_SCRATCH_BYTES (64u << 20) /* 64 MiB */
int cast_tree_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* out, int dtype,
                               const int64_t* strides,
                               const int32_t* cu_q, const int32_t* cu_kv,
                               const int32_t* prefix_len, const int32_t* pack_len,
                               const int64_t* anc_words, int anc_words_per_row,
                               const int32_t* parent,
                               int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                               float sm_scale, int max_pack, int max_kv, cast_stream_t stream);

/*
 * Bytes of workspace cast_tree_attn_fwd needs for these sizes (0 is possible).
 * Pure host arithmetic; the same arguments must be passed to the call.
 */
size_t cast_tree_attn_workspace_size(int dtype, int B, int total_q, int H_q, int H_kv, int D,
                                     int max_pack, int max_kv);

/*
 * The same, exact for CAST_F32_SPLIT, whose workspace grows with total_kv
 * (cast_tree_attn_workspace_size bounds total_kv by B * max_kv there). Equal to
 * cast_tree_attn_workspace_size for the other dtypes. No counterpart in the
 * reference.
 */
size_t cast_tree_attn_workspace_size_kv(int dtype, int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                                        int max_pack, int max_kv);

/*
 * Tree attention reading the prefix straight from a per-request KV store.
 * Replaces the ragged K/V assembly of cast_trees/serving.py:60-71 (every layer
 * copies each request's prefix from its store into one buffer, k_rag/v_rag,
 * and casts q/k/v to fp32) together with the attention call it feeds.
 *
 * Sequence b's prefix keys are rows [0, prefix_len[b]) of request b of the
 * stores k_store / v_store [store_batch, H_kv, store_rows, D] (the per-layer
 * stores the serving loop keeps, cast_trees/serving.py:190-205); its pack keys
 * are rows [cu_q[b], cu_q[b] + pack_len[b]) of k_pack / v_pack [total_q, H_kv, D]
 * (the current pass's keys, already in pack order). Visibility, output and
 * parent / ancestor conventions are those of cast_tree_attn_fwd.
 * 16-bit inputs (CAST_BF16 / CAST_F16), or fp32 inputs and output with
 * CAST_F32_SPLIT; D = 128, H_q / H_kv dividing 128.
 * strides[20] = element strides of q (row, head, dim), k_store (batch, head,
 * row, dim), v_store (same), k_pack (row, head, dim), v_pack, out; dim strides
 * 1, every other stride a multiple of 16 bytes (8 16-bit or 4 fp32 elements),
 * bases 16-byte aligned. CAST_F32_SPLIT reads the stores once in its split pass
 * (prefix rows from the store, pack rows from k_pack / v_pack) into ragged
 * bf16 hi / lo copies in the workspace (256-byte aligned), then runs the
 * tensor-core kernel on them.
 * max_prefix bounds prefix_len[b] (<= store_rows); workspace as returned by
 * cast_tree_attn_store_workspace_size(). Store rows past prefix_len[b] are
 * never part of the result, whatever they hold (non-finite values included).
 * Returns CAST_ERR_DTYPE / CAST_ERR_HEAD_DIM / CAST_ERR_SHAPE / CAST_ERR_ALIGN
 * for inputs outside that form (the Python wrapper then assembles the ragged
 * layout and calls cast_tree_attn_fwd).
 */
int cast_tree_attn_store_fwd(const void* q, const void* k_store, const void* v_store, const void* k_pack,
                             const void* v_pack, void* out, int dtype, const int64_t* strides,
                             const int32_t* cu_q, const int32_t* prefix_len, const int32_t* pack_len,
                             const int64_t* anc_words, int anc_words_per_row, const int32_t* parent,
                             int B, int total_q, int store_batch, int store_rows, int H_q, int H_kv, int D,
                             float sm_scale, int max_pack, int max_prefix,
                             void* workspace, size_t workspace_bytes, cast_stream_t stream);

/* Bytes of workspace cast_tree_attn_store_fwd needs for these sizes (0 is possible). */
size_t cast_tree_attn_store_workspace_size(int dtype, int B, int total_q, int H_q, int H_kv, int D, int max_pack,
                                           int max_prefix);

/*
 * The ragged K/V assembly of cast_trees/serving.py:60-69 on the device, for
 * store-mode calls the tensor-core kernels do not take (other head dims or
 * group sizes, strides that are not 16-byte multiples): k_out / v_out
 * [rows_cap, H, D] (contiguous, elem_bytes 2 or 4) receive, for sequence b at
 * rows [cu_kv[b], cu_kv[b + 1]), its prefix rows [0, prefix_len[b]) of store
 * row b followed by its pack rows [cu_q[b], cu_q[b] + pack_len[b]) of k_pack /
 * v_pack; cu_kv_out [B + 1] receives the offsets (a scan of the lengths, on
 * the device: no host read). Rows from cu_kv[B] to rows_cap are zero.
 * rows_cap >= sum of prefix_len + pack_len, e.g. B * (max_prefix + max_pack).
 * strides[14] = element strides of k_store, v_store (batch, head, row, dim) and
 * k_pack, v_pack (row, head, dim); dim strides 1. Lengths outside
 * [0, store_rows] / [0, max_pack] are reported as CAST_DEV_BAD_LAYOUT and their
 * rows written as zeros. No counterpart in the reference's API.
 */
int cast_kv_ragged_gather(const void* k_store, const void* v_store, const void* k_pack, const void* v_pack,
                          int elem_bytes, const int64_t* strides, const int32_t* cu_q, const int32_t* prefix_len,
                          const int32_t* pack_len, int B, int total_q, int store_batch, int store_rows, int H, int D,
                          int max_pack, int64_t rows_cap, void* k_out, void* v_out, int32_t* cu_kv_out,
                          cast_stream_t stream);

/*
 * How cast_tree_attn_fwd would run for these arguments (pure host arithmetic):
 * plan[0] = 1 for the tcgen05 tensor-core kernel, 0 for the CUDA-core kernel,
 * 2 for the tcgen05 kernel of CAST_F32_SPLIT (after its split pass);
 * plan[1] = number of key-range splits; plan[2] = kernel launches per call
 * (2 when split partials are merged by the combine kernel; CAST_F32_SPLIT adds
 * its split pass).
 */
int cast_tree_attn_plan(int dtype, int B, int total_q, int H_q, int H_kv, int D, int max_pack, int max_kv,
                        const int64_t* strides, const void* q, const void* k, const void* v, const void* out,
                        int* plan);

/*
 * Per-row fp64 log-softmax and top-k, bit-compatible with
 * cast_trees/tree.py:20-26 block_topk: ties keep the lower index first.
 * logits: float64 [n_rows, V] with row stride `row_stride` (elements).
 * top_idx: int64 [n_rows, k]; top_lp: float64 [n_rows, k], best first.
 */
int cast_block_topk(const double* logits, int64_t n_rows, int64_t V, int64_t row_stride, int k,
                    int64_t* top_idx, double* top_lp, cast_stream_t stream);

/*
 * Best-first prefix-closed trees, node order identical to
 * cast_trees/tree.py:29-49 build_tree (pop order of the heap keyed by
 * (-path_logprob, depth, parent, rank)).
 * top_idx / top_lp: [B, L, k_cols] (row-major), k = min(k, k_cols) is used.
 * budget: int32 [B] non-root node count per tree (<= max_budget).
 * Outputs [B, max_budget] (row b holds count[b] nodes): token (int32),
 * depth (int32, 1..L), parent (int32, -1 = root) and score (float64).
 * Optional pack layout of cast_trees/serving.py:213-222 (pass NULL to skip):
 *   cu_q (int32 [B+1]) gives each pack's first row; then
 *   pack_parent[cu_q[b] + 0] = -1, pack_parent[cu_q[b] + 1 + i] = parent_i + 1,
 *   pack_token (needs root_token int32 [B]) = root, then node tokens,
 *   pack_pos (needs seq_len int32 [B]) = seq_len, then seq_len + depth_i.
 */
int cast_build_tree(const int64_t* top_idx, const double* top_lp, int B, int L, int k_cols, int k,
                    const int32_t* budget, int max_budget,
                    int32_t* token, int32_t* depth, int32_t* parent, double* score, int32_t* count,
                    const int32_t* cu_q, int32_t* pack_parent,
                    const int32_t* root_token, int32_t* pack_token,
                    const int32_t* seq_len, int32_t* pack_pos,
                    cast_stream_t stream);

/*
 * Greedy tree walk of a verify pass, cast_trees/decode.py:85-103 at
 * temperature 0, for every sequence at once (the per-request loop of
 * cast_trees/serving.py:326-336). From the root (pack row 0) the walk picks
 * argmax(logits[row]) (torch.argmax order: NaN first, then the larger value,
 * then the lower index); if a child of the current node carries that token
 * (lowest pack index first) it moves there, else that token is the bonus.
 * logits: [total_q, V] rows in pack order (dtype CAST_F32/BF16/F16, row stride
 * in elements); cu_q int32 [B+1]; pack_parent int32 [total_q] (pack-local,
 * -1 = root); pack_token int32 [total_q] (the token each packed row carries).
 * Outputs: path int32 [B, path_cap] (accepted node indices = pack row - 1,
 * -1 padded), accepted int32 [B] (= len(path) + 1), bonus int64 [B];
 * optional keep int32 [B, path_cap + 1] (0, then path + 1: the reference's
 * keep list) and tokens int64 [B, path_cap + 1] (the committed tokens: path
 * tokens, then the bonus), -1 padded. Only the rows on each accepted path are
 * read. A path longer than path_cap records CAST_DEV_TREE_OVERFLOW.
 */
int cast_tree_walk_greedy(const void* logits, int dtype, int64_t row_stride, int V, const int32_t* cu_q,
                          const int32_t* pack_parent, const int32_t* pack_token, int B, int total_q, int path_cap,
                          int32_t* path, int32_t* accepted, int64_t* bonus, int32_t* keep, int64_t* tokens,
                          cast_stream_t stream);

/*
 * Shared-budget split of a forest, cast_trees/tree.py:63-82
 * select_global_topk: the first `total` nodes of the pool sorted by
 * (-score, tree, node) are kept (total < 0 acts like Python's pool[:total]),
 * each tree keeps its nodes in their original order and parents are
 * renumbered (-1 when the parent is not kept).
 * Inputs [B, max_nodes] (row b holds count[b] nodes, as cast_build_tree writes
 * them): token, depth, parent (tree-local), score. Outputs of the same shape
 * and out_count [B]; they must not be the input arrays.
 * Optional packed layout of the selected trees (cast_trees/serving.py:213-222):
 * cu_q int32 [B+1] (written), pack_parent / pack_token (needs root_token) /
 * pack_pos (needs seq_len), each with room for pack_capacity rows.
 */
int cast_select_global_topk(const int32_t* token, const int32_t* depth, const int32_t* parent, const double* score,
                            const int32_t* count, int B, int max_nodes, int64_t total,
                            int32_t* out_token, int32_t* out_depth, int32_t* out_parent, double* out_score,
                            int32_t* out_count, int32_t* cu_q, const int32_t* root_token, const int32_t* seq_len,
                            int32_t* pack_parent, int32_t* pack_token, int32_t* pack_pos, int64_t pack_capacity,
                            cast_stream_t stream);

/*
 * Accepted-path append into the per-request KV stores, every layer in one
 * call: cast_trees/serving.py:264-289 BatchedServer._append_store.
 * src_kv / dst_kv / pack_kv are HOST arrays of 2 * n_layers device pointers
 * (layer l's K at [2l], V at [2l + 1]). Stores are [B, H, cap, D] (strides
 * batch, head, row in elements; dim stride 1); pack K/V are the verify pass's
 * [H, total_q, D] per-layer tensors (pack_strides = batch (0), head, row).
 * For destination row nb (source row b = rows[nb], or nb when rows is NULL),
 * head h, layer l: rows store_len[b] + j (j < accepted[b]) take pack row
 * cu_q[b] + keep[b * keep_stride + j]; every other row below src_cap copies
 * source row b and rows from src_cap to dst_cap are zero (the reference's
 * gather of whole store rows, zero growth, then the append). append_only = 1
 * writes only the appended rows of a store in place (dst_kv == src_kv, rows
 * NULL, same shape).
 */
int cast_append_store(int n_layers, const void* const* src_kv, void* const* dst_kv, const void* const* pack_kv,
                      int elem_bytes, int H, int D, int B_src, int64_t src_cap, const int64_t* src_strides,
                      int B_dst, int64_t dst_cap, const int64_t* dst_strides, int64_t pack_rows,
                      const int64_t* pack_strides, const int32_t* rows, const int32_t* store_len,
                      const int32_t* accepted, const int32_t* keep, int keep_stride, const int32_t* cu_q,
                      int append_only, cast_stream_t stream);

/*
 * cast_trees/verify.py:48-60 gather_cache for every layer in one call: the
 * destination [B, H, n_prefix + n_keep, D] gets the first n_prefix rows of the
 * source [B, H, src_len, D] and then its rows n_prefix + keep[j]. src_kv /
 * dst_kv as in cast_append_store; keep is a device int32 array; the
 * destination must not overlap the source.
 */
int cast_gather_cache(int n_layers, const void* const* src_kv, void* const* dst_kv, int elem_bytes, int B, int H,
                      int D, int64_t src_len, const int64_t* src_strides, const int64_t* dst_strides, int n_prefix,
                      const int32_t* keep, int n_keep, cast_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CAST_B200_H */
