// The steps of a verify round around the attention pass, on the device:
//   walk::  greedy tree walk (cast_trees/decode.py:85-103 at temperature 0,
//           serving.py:326-336's keep / accepted / bonus lists)
//   sel::   shared-budget selection over a forest (cast_trees/tree.py:63-82
//           select_global_topk), optionally writing the pack layout
//   kvg::   KV-store append / compaction (serving.py:264-289 _append_store) and
//           cache gather (verify.py:48-60 gather_cache): one row-gather kernel
#pragma once

#include <cooperative_groups.h>
#include <limits.h>

#include "common.cuh"

namespace cast {

// ---------------------------------------------------------------------------
// Greedy tree walk. One cluster of CS CTAs per sequence: each CTA takes the
// argmax of its slice of the current packed row's logits, CTA 0 of the cluster
// merges the slices through distributed shared memory, looks for the child of
// the current node carrying that token (lowest pack index first, which is the
// reference's child order), and broadcasts the next row. Only rows on the
// accepted path are read: (accepted + 1) rows of V logits per sequence.
// ---------------------------------------------------------------------------
namespace walk {
constexpr int NT = 256;
constexpr int UNROLL = 8;

struct WalkArgs {
  const void* logits;    // [total_q, V] rows of the packed verify pass
  int64_t row_stride;    // elements
  int V;
  const int32_t* cu_q;         // [B+1]
  const int32_t* pack_parent;  // [total_q] pack-local parent, -1 = root
  const int32_t* pack_token;   // [total_q] token of every packed row
  int B, total_q, path_cap;
  int32_t* path;      // [B, path_cap] accepted node indices (pack row - 1), -1 padded
  int32_t* accepted;  // [B] len(path) + 1 (0 for a sequence with a bad layout)
  int64_t* bonus;     // [B] token picked after the path (-1 for a bad layout)
  int32_t* keep;      // optional [B, path_cap + 1]: 0, path + 1, then -1
  int64_t* tokens;    // optional [B, path_cap + 1]: path tokens, bonus, then -1
};

// torch.argmax order: NaN above everything, then the larger value, then the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

// Packed 16-bit helpers: NaN-propagating max and per-half equality masks.
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using P2 = __nv_bfloat162;
  static __device__ __forceinline__ P2 lowest() { return __bfloat162bfloat162(__float2bfloat16_rn(-INFINITY)); }
  static __device__ __forceinline__ P2 max2(P2 a, P2 b) { return __hmax2_nan(a, b); }
  static __device__ __forceinline__ float hmax(P2 a) { return __bfloat162float(__hmax_nan(a.x, a.y)); }
  static __device__ __forceinline__ P2 splat(float v) { return __bfloat162bfloat162(__float2bfloat16_rn(v)); }
  static __device__ __forceinline__ unsigned eq(P2 a, P2 b) { return __heq2_mask(a, b); }
  static __device__ __forceinline__ unsigned nan(P2 a) { return __hne2_mask(a, a); }
};
template <> struct Pair<__half> {
  using P2 = __half2;
  static __device__ __forceinline__ P2 lowest() { return __half2half2(__float2half_rn(-INFINITY)); }
  static __device__ __forceinline__ P2 max2(P2 a, P2 b) { return __hmax2_nan(a, b); }
  static __device__ __forceinline__ float hmax(P2 a) { return __half2float(__hmax_nan(a.x, a.y)); }
  static __device__ __forceinline__ P2 splat(float v) { return __half2half2(__float2half_rn(v)); }
  static __device__ __forceinline__ unsigned eq(P2 a, P2 b) { return __heq2_mask(a, b); }
  static __device__ __forceinline__ unsigned nan(P2 a) { return __hne2_mask(a, a); }
};

// 16-bit rows: per batch of UNROLL vectors a packed NaN-propagating max, and the index
// search only for a batch that beats the running best (batches rise in index, so a
// batch's lowest index stands in for its argmax in the comparison).
template <typename T>
__device__ __forceinline__ void scan_slice16(const T* row, int lo, int hi, float& bv, int& bi) {
  using PT = Pair<T>;
  using P2 = typename PT::P2;
  constexpr int PER = 8;
  const int nvec = (hi - lo) / PER;
  const uint4* p = reinterpret_cast<const uint4*>(row + lo);
  for (int base = threadIdx.x; base < nvec; base += NT * UNROLL) {
    uint4 buf[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int vi = base + u * NT;
      if (vi < nvec) buf[u] = __ldg(p + vi);
    }
    P2 m2 = PT::lowest();
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      if (base + u * NT < nvec) {
        const P2* e = reinterpret_cast<const P2*>(&buf[u]);
        m2 = PT::max2(PT::max2(m2, e[0]), PT::max2(e[1], PT::max2(e[2], e[3])));
      }
    }
    const float mv = PT::hmax(m2);
    if (!better(mv, lo + base * PER, bv, bi)) continue;
    const bool want_nan = mv != mv;
    const P2 mm = PT::splat(mv);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int vi = base + u * NT;
      if (vi < nvec) {
        const P2* e = reinterpret_cast<const P2*>(&buf[u]);
        int hit = -1;
#pragma unroll
        for (int x = 3; x >= 0; --x) {
          const unsigned msk = want_nan ? PT::nan(e[x]) : PT::eq(e[x], mm);
          if (msk) hit = 2 * x + ((msk & 0xffffu) ? 0 : 1);
        }
        if (hit >= 0) { bv = mv; bi = lo + vi * PER + hit; break; }
      }
    }
  }
  for (int i = lo + nvec * PER + threadIdx.x; i < hi; i += NT) {
    const float v = Elem<T>::to_f(row[i]);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
}

template <typename T>
__device__ __forceinline__ void scan_slice(const T* row, int lo, int hi, bool vec, float& bv, int& bi) {
  constexpr int PER = 16 / sizeof(T);
  if constexpr (sizeof(T) == 2) {
    if (vec) { scan_slice16<T>(row, lo, hi, bv, bi); return; }
  }
  int tail = lo;
  if (vec) {
    const int nvec = (hi - lo) / PER;
    const uint4* p = reinterpret_cast<const uint4*>(row + lo);
    for (int base = threadIdx.x; base < nvec; base += NT * UNROLL) {
      uint4 buf[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int vi = base + u * NT;
        if (vi < nvec) buf[u] = __ldg(p + vi);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int vi = base + u * NT;
        if (vi < nvec) {
          const T* e = reinterpret_cast<const T*>(&buf[u]);
#pragma unroll
          for (int x = 0; x < PER; ++x) {
            const float v = Elem<T>::to_f(e[x]);
            const int i = lo + vi * PER + x;
            if (better(v, i, bv, bi)) { bv = v; bi = i; }
          }
        }
      }
    }
    tail = lo + nvec * PER;
  }
  for (int i = tail + threadIdx.x; i < hi; i += NT) {
    const float v = Elem<T>::to_f(row[i]);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
}

// Block-wide argmax; the result lands in (*out_v, *out_i) (written by thread 0).
__device__ __forceinline__ void block_argmax(float bv, int bi, float* s_v, int* s_i, float* out_v, int* out_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_down_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_down_sync(0xffffffffu, bi, o);
    if (better(v2, i2, bv, bi)) { bv = v2; bi = i2; }
  }
  if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < NT / 32 ? s_v[lane] : -INFINITY;
    bi = lane < NT / 32 ? s_i[lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_down_sync(0xffffffffu, bv, o);
      const int i2 = __shfl_down_sync(0xffffffffu, bi, o);
      if (better(v2, i2, bv, bi)) { bv = v2; bi = i2; }
    }
    if (lane == 0) { *out_v = bv; *out_i = bi; }
  }
}

constexpr int SMEM_PACK = 1024;   // packs up to this size keep parent / token / first child in shared memory
__device__ __forceinline__ bool in_smem_tokens(int P) { return P <= SMEM_PACK; }

// L2 prefetch of this CTA's slice of a row the walk is likely to read next.
template <typename T>
__device__ __forceinline__ void prefetch_slice(const T* row, int lo, int hi) {
  const char* p0 = reinterpret_cast<const char*>(row + lo);
  const char* p1 = reinterpret_cast<const char*>(row + hi);
  for (const char* p = p0 + (size_t)threadIdx.x * 128; p < p1; p += (size_t)NT * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

template <typename T, int CS>
__global__ void __launch_bounds__(NT) tree_walk_kernel(const WalkArgs a, bool vec) {
  namespace cg = cooperative_groups;
  __shared__ int s_par[SMEM_PACK], s_tkn[SMEM_PACK], s_fc[SMEM_PACK];
  __shared__ float s_v[NT / 32];
  __shared__ int s_i[NT / 32];
  __shared__ float s_pv[2];   // this CTA's slice argmax, double-buffered by step parity
  __shared__ int s_pi[2];
  __shared__ int s_tok, s_child;
  const int b = blockIdx.x / CS;
  int rank = 0;
  if constexpr (CS > 1) rank = (int)cg::this_cluster().block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // every CTA of the cluster reads the same metadata and takes the same branches:
  // each one merges all slices and decides the step itself (no broadcast needed)
  const int q0 = a.cu_q[b], q1 = a.cu_q[b + 1];
  const int P = q1 - q0;
  const bool ok = q0 >= 0 && q1 <= a.total_q && P >= 1;
  int n = 0;
  long long bonus = -1;
  if (ok) {
    constexpr int PER = 16 / sizeof(T);
    const int per = ((a.V + CS - 1) / CS + PER - 1) / PER * PER;
    const int lo = min(a.V, rank * per), hi = min(a.V, lo + per);
    const T* base = static_cast<const T*>(a.logits);
    // the pack's parents and tokens, and each node's first child (the drafter's most
    // likely continuation: children are stored in decreasing score order)
    const bool in_smem = P <= SMEM_PACK;
    if (in_smem) {
      for (int c = tid; c < P; c += NT) {
        s_par[c] = a.pack_parent[q0 + c];
        s_tkn[c] = a.pack_token[q0 + c];
        s_fc[c] = INT_MAX;
      }
      __syncthreads();
      for (int c = 1 + tid; c < P; c += NT) {
        const int p = s_par[c];
        if (p >= 0 && p < c) atomicMin(&s_fc[p], c);
      }
      __syncthreads();
    }
    int cur = 0;
    for (int step = 0;; ++step) {
      if (in_smem && s_fc[cur] != INT_MAX)
        prefetch_slice<T>(base + (int64_t)(q0 + s_fc[cur]) * a.row_stride, lo, hi);
      float bv = -INFINITY;
      int bi = INT_MAX;
      scan_slice<T>(base + (int64_t)(q0 + cur) * a.row_stride, lo, hi, vec, bv, bi);
      block_argmax(bv, bi, s_v, s_i, &s_pv[step & 1], &s_pi[step & 1]);
      if constexpr (CS > 1) cg::this_cluster().sync(); else __syncthreads();
      if (warp == 0) {
        float v = -INFINITY;
        int i = INT_MAX;
        if (lane < CS) {
          if constexpr (CS > 1) {
            auto cl = cg::this_cluster();
            v = *cl.map_shared_rank(&s_pv[step & 1], lane);
            i = *cl.map_shared_rank(&s_pi[step & 1], lane);
          } else {
            v = s_pv[step & 1];
            i = s_pi[step & 1];
          }
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
          const float v2 = __shfl_down_sync(0xffffffffu, v, o);
          const int i2 = __shfl_down_sync(0xffffffffu, i, o);
          if (better(v2, i2, v, i)) { v = v2; i = i2; }
        }
        if (lane == 0) { s_tok = i; s_child = INT_MAX; }
      }
      __syncthreads();
      const int tok = s_tok;
      int best = INT_MAX;
      if (in_smem) {
        for (int c = cur + 1 + tid; c < P; c += NT)
          if (s_par[c] == cur && s_tkn[c] == tok) { best = c; break; }
      } else {
        for (int c = cur + 1 + tid; c < P; c += NT)
          if (a.pack_parent[q0 + c] == cur && a.pack_token[q0 + c] == tok) { best = c; break; }
      }
      if (best != INT_MAX) atomicMin(&s_child, best);
      __syncthreads();
      const int c = s_child;
      if (c == INT_MAX) { bonus = tok; break; }
      if (n >= a.path_cap) {
        if (rank == 0 && tid == 0) report(CAST_DEV_TREE_OVERFLOW);
        break;
      }
      if (rank == 0 && tid == 0) a.path[(int64_t)b * a.path_cap + n] = c - 1;
      ++n;
      cur = c;
    }
    // no CTA leaves while another may still read its partials
    if constexpr (CS > 1) cg::this_cluster().sync();
  } else if (rank == 0 && tid == 0) {
    report(CAST_DEV_BAD_LAYOUT);
  }
  if (rank != 0) return;
  // rank 0 writes the outputs: path padding, accepted, bonus, keep / token rows
  const int acc = ok && bonus >= 0 ? n + 1 : 0;
  if (tid == 0) { a.accepted[b] = acc; a.bonus[b] = bonus; }
  for (int j = n + tid; j < a.path_cap; j += NT) a.path[(int64_t)b * a.path_cap + j] = -1;
  __syncthreads();   // path entries written by thread 0 are read below
  const int w = a.path_cap + 1;
  for (int j = tid; j < w; j += NT) {
    if (a.keep) {
      int kj = -1;
      if (j == 0 && acc > 0) kj = 0;
      else if (j > 0 && j < acc) kj = a.path[(int64_t)b * a.path_cap + j - 1] + 1;
      a.keep[(int64_t)b * w + j] = kj;
    }
    if (a.tokens) {
      int64_t t = -1;
      if (j < n && acc > 0) {
        const int c = a.path[(int64_t)b * a.path_cap + j] + 1;
        t = in_smem_tokens(P) ? s_tkn[c] : a.pack_token[q0 + c];
      }
      else if (j == n && acc > 0) t = bonus;
      a.tokens[(int64_t)b * w + j] = t;
    }
  }
}
}  // namespace walk

// ---------------------------------------------------------------------------
// select_global_topk. One CTA: a radix select finds the `total`-th smallest
// pooled key (-score, b, j), then one warp per tree keeps the nodes at or
// below it in node order and renumbers their parents.
// ---------------------------------------------------------------------------
namespace sel {
constexpr int NT = 1024;
constexpr int NW = NT / 32;
constexpr int MAX_NODES = 1024;   // per tree (32 keep words per warp)
constexpr size_t MAX_DYN_SMEM = 180 * 1024;   // dynamic shared memory beside the static arrays

struct SelArgs {
  const int32_t* token; const int32_t* depth; const int32_t* parent; const double* score; const int32_t* count;
  int B, mb;
  int cache_keys;                // 1: the pooled keys [B * mb] are staged in shared memory
  int64_t total;
  int32_t* o_token; int32_t* o_depth; int32_t* o_parent; double* o_score; int32_t* o_count;
  int32_t* cu_q;                 // optional out [B+1]
  const int32_t* root_token;     // optional (pack tokens)
  const int32_t* seq_len;        // optional (pack positions)
  int32_t* pack_parent; int32_t* pack_token; int32_t* pack_pos;
  int64_t pack_cap;
};

__device__ __forceinline__ uint64_t pool_key(double score) { return ordered_key(-score); }

__device__ __forceinline__ int block_sum(int v, int* s_w) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  __syncthreads();
  if (lane == 0) s_w[warp] = v;
  __syncthreads();
  int t = lane < NW ? s_w[lane] : 0;
  return __reduce_add_sync(0xffffffffu, t);
}

// Exclusive scan of s[0..n) in place (n <= any); returns the total.
__device__ int block_exclusive_scan(int* s, int n, int* s_w) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int carry = 0;
  for (int base = 0; base < n; base += NT) {
    const int i = base + threadIdx.x;
    const int v = i < n ? s[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) s_w[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = lane < NW ? s_w[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < NW) s_w[lane] = w;
    }
    __syncthreads();
    const int before = (warp > 0 ? s_w[warp - 1] : 0) + x - v;
    if (i < n) s[i] = carry + before;
    carry += s_w[NW - 1];
  }
  __syncthreads();
  return carry;
}

__global__ void __launch_bounds__(NT, 1) select_kernel(const SelArgs a) {
  extern __shared__ __align__(8) int s_dyn[];  // [B] tie offsets, [B+1] pack offsets, then (optional) keys
  __shared__ unsigned s_whist[NW][256];
  __shared__ int s_w[NW];
  __shared__ uint32_t s_keep[NW][MAX_NODES / 32];
  __shared__ uint64_t s_prefix;
  __shared__ long long s_rank;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int* tie_off = s_dyn;
  int* pack_off = s_dyn + a.B;
  int* s_cnt = s_dyn + 2 * a.B + 1;             // [B] clamped node counts
  uint64_t* s_key = reinterpret_cast<uint64_t*>(s_dyn + ((3 * a.B + 1 + 1) & ~1));
  for (int b = tid; b < a.B; b += NT) s_cnt[b] = max(0, min(a.count[b], a.mb));
  if (a.cache_keys) {
    const int64_t n_slots = (int64_t)a.B * a.mb;
    for (int64_t f = tid; f < n_slots; f += NT) s_key[f] = pool_key(a.score[f]);
  }
  auto key_of = [&](int64_t f) -> uint64_t { return a.cache_keys ? s_key[f] : pool_key(a.score[f]); };
  // pooled node count (counts are clamped to the row width)
  int part = 0;
  for (int b = tid; b < a.B; b += NT) part += s_cnt[b];
  const int n_all = block_sum(part, s_w);
  long long total = a.total < 0 ? max(0ll, (long long)n_all + a.total) : a.total;   // Python slice pool[:total]
  const bool keep_all = total >= n_all;
  // radix select of the total-th smallest key: threshold key and ties to take
  uint64_t thr = ~0ull;
  long long need = 0;
  if (!keep_all && total > 0) {
    if (tid == 0) { s_prefix = 0; s_rank = total; }
    uint64_t mask = 0;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = tid; i < NW * 256; i += NT) (&s_whist[0][0])[i] = 0;
      __syncthreads();
      const uint64_t prefix = s_prefix;
      for (int b = warp; b < a.B; b += NW) {
        const int n = s_cnt[b];
        for (int j = lane; j < n; j += 32) {
          const uint64_t key = key_of((int64_t)b * a.mb + j);
          if ((key & mask) == prefix) atomicAdd(&s_whist[warp][(key >> shift) & 255u], 1u);   // per-warp copy
        }
      }
      __syncthreads();
      // merge the warp copies (thread t < 256 owns bin t), then warp 0 finds the digit
      if (tid < 256) {
        unsigned c = 0;
#pragma unroll 8
        for (int w = 0; w < NW; ++w) c += s_whist[w][tid];
        s_whist[0][tid] = c;
      }
      __syncthreads();
      if (warp == 0) {
        // lane l holds bins [8l, 8l + 8): inclusive scan of the lane totals, then the lane
        // whose range crosses the rank finds the digit inside its 8 bins
        unsigned cnt[8], tot = 0;
#pragma unroll
        for (int x = 0; x < 8; ++x) { cnt[x] = s_whist[0][lane * 8 + x]; tot += cnt[x]; }
        unsigned incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const long long k = s_rank;
        const long long before = (long long)incl - tot;
        if (before < k && k <= (long long)incl) {
          long long cum = before;
          int d = lane * 8;
          for (int x = 0; x < 8; ++x, ++d) {
            if (cum + cnt[x] >= k) break;
            cum += cnt[x];
          }
          s_rank = k - cum;
          s_prefix = prefix | ((uint64_t)d << shift);
        }
      }
      mask |= 0xffull << shift;
      __syncthreads();
    }
    thr = s_prefix;
    need = s_rank;
  }
  const bool none = !keep_all && total <= 0;
  // ties at the threshold are taken in (b, j) order: per-tree tie counts, then offsets
  if (!keep_all && !none) {
    for (int b = warp; b < a.B; b += NW) {
      const int n = s_cnt[b];
      int t = 0;
      for (int j = lane; j < n; j += 32) t += key_of((int64_t)b * a.mb + j) == thr;
      t = __reduce_add_sync(0xffffffffu, t);
      if (lane == 0) tie_off[b] = t;
    }
    __syncthreads();
    block_exclusive_scan(tie_off, a.B, s_w);
  }
  // per tree: keep bits, then the compacted, renumbered node list
  for (int b = warp; b < a.B; b += NW) {
    const int n = s_cnt[b];
    const int64_t row = (int64_t)b * a.mb;
    int ties_before = keep_all || none ? 0 : tie_off[b];
    for (int c = 0; c < (n + 31) / 32; ++c) {
      const int j = c * 32 + lane;
      bool kept = false, tie = false;
      if (j < n) {
        if (keep_all) {
          kept = true;
        } else if (!none) {
          const uint64_t key = key_of(row + j);
          kept = key < thr;
          tie = key == thr;
        }
      }
      const unsigned tmask = __ballot_sync(0xffffffffu, tie);
      if (tie) kept = ties_before + __popc(tmask & ((1u << lane) - 1u)) < need;
      ties_before += __popc(tmask);
      const unsigned km = __ballot_sync(0xffffffffu, kept);
      if (lane == 0) s_keep[warp][c] = km;
    }
    __syncwarp();
    int kept_total = 0;
    for (int c = 0; c < (n + 31) / 32; ++c) {
      const unsigned km = s_keep[warp][c];
      const int j = c * 32 + lane;
      if ((km >> lane) & 1u) {
        const int nj = kept_total + __popc(km & ((1u << lane) - 1u));
        const int p = a.parent[row + j];
        int np = -1;
        if (p >= 0 && p < n && ((s_keep[warp][p >> 5] >> (p & 31)) & 1u)) {
          np = 0;
          for (int w = 0; w < (p >> 5); ++w) np += __popc(s_keep[warp][w]);
          np += __popc(s_keep[warp][p >> 5] & ((1u << (p & 31)) - 1u));
        }
        a.o_token[row + nj] = a.token[row + j];
        a.o_depth[row + nj] = a.depth[row + j];
        a.o_parent[row + nj] = np;
        a.o_score[row + nj] = a.score[row + j];
      }
      kept_total += __popc(km);
    }
    if (lane == 0) {
      a.o_count[b] = kept_total;
      if (a.cu_q) pack_off[b] = 1 + kept_total;
    }
    __syncwarp();
  }
  if (!a.cu_q) return;
  // packed layout of the selected trees (cast_trees/serving.py:213-222)
  __syncthreads();
  const int tot = block_exclusive_scan(pack_off, a.B, s_w);
  for (int b = tid; b < a.B; b += NT) a.cu_q[b] = pack_off[b];
  if (tid == 0) a.cu_q[a.B] = tot;
  if (tot > a.pack_cap) {
    if (tid == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  for (int b = warp; b < a.B; b += NW) {
    const int q0 = pack_off[b];
    const int n = a.o_count[b];
    const int64_t row = (int64_t)b * a.mb;
    for (int i = lane; i <= n; i += 32) {
      if (a.pack_parent) a.pack_parent[q0 + i] = i == 0 ? -1 : a.o_parent[row + i - 1] + 1;
      if (a.pack_token && a.root_token) a.pack_token[q0 + i] = i == 0 ? a.root_token[b] : a.o_token[row + i - 1];
      if (a.pack_pos && a.seq_len) a.pack_pos[q0 + i] = a.seq_len[b] + (i == 0 ? 0 : a.o_depth[row + i - 1]);
    }
  }
}
}  // namespace sel

// ---------------------------------------------------------------------------
// KV row gather. Destination row r of (layer l, batch row nb, head h), with
// b = rows[nb] its source batch row, S = store_len[b], A = accepted[b]:
//   S <= r < S + A : pack row cu_q[b] + keep[b][r - S]
//   r < src_cap    : source store row r          (copy mode only)
//   otherwise      : zeros                       (copy mode only)
// which is the reference's order: gather the surviving store rows whole, grow
// with zeros, then write the appended rows.
// Copy mode writes rows [0, dst_cap) of a new store; append mode writes only
// rows [S, S + A) of the store in place.
// ---------------------------------------------------------------------------
namespace kvg {
constexpr int NT = 256;
constexpr int MAXL = 64;
constexpr int ROWS_PER_CTA = 64;

struct Layers {
  const void* src[MAXL][2];
  void* dst[MAXL][2];
  const void* pack[MAXL][2];
};

struct KvArgs {
  int L, H, row_bytes, append_only;
  int B_src, B_dst;
  int64_t src_cap, dst_cap, pack_rows;
  int64_t src_sb, src_sh, src_sr;      // bytes
  int64_t dst_sb, dst_sh, dst_sr;
  int64_t pk_sb, pk_sh, pk_st;
  const int32_t* rows;       // [B_dst] or NULL (identity)
  const int32_t* store_len;  // [B_src], or NULL: every row has s_const
  const int32_t* accepted;   // [B_src], or NULL: every row has a_const
  int s_const, a_const;
  const int32_t* keep;       // keep[b * keep_stride + j]
  int keep_stride;
  const int32_t* cu_q;       // [B_src] pack offsets or NULL (0)
};

template <typename W>
__global__ void __launch_bounds__(NT) kv_gather_kernel(const KvArgs a, const Layers ly) {
  const int l = blockIdx.z;
  const int nb = blockIdx.y / a.H, h = blockIdx.y % a.H;
  const int b = a.rows ? a.rows[nb] : nb;
  if (b < 0 || b >= a.B_src) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int S = a.store_len ? a.store_len[b] : a.s_const;
  const int A = a.accepted ? a.accepted[b] : a.a_const;
  if (S < 0 || A < 0 || (int64_t)S + A > a.dst_cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int64_t r_begin = a.append_only ? S : 0;
  const int64_t r_end = a.append_only ? (int64_t)S + A : a.dst_cap;
  const int64_t r0 = r_begin + (int64_t)blockIdx.x * ROWS_PER_CTA;
  if (r0 >= r_end) return;
  const int64_t r1 = min(r_end, r0 + ROWS_PER_CTA);
  const int wpr = a.row_bytes / (int)sizeof(W);       // words per row
  const int64_t qb = a.cu_q ? a.cu_q[b] : 0;
  for (int kv = 0; kv < 2; ++kv) {
    const char* src = static_cast<const char*>(ly.src[l][kv]) + b * a.src_sb + h * a.src_sh;
    char* dst = static_cast<char*>(ly.dst[l][kv]) + nb * a.dst_sb + h * a.dst_sh;
    const char* pack = static_cast<const char*>(ly.pack[l][kv]) + b * a.pk_sb + h * a.pk_sh;
    for (int64_t e = threadIdx.x; e < (r1 - r0) * wpr; e += NT) {
      const int64_t r = r0 + e / wpr;
      const int w = (int)(e % wpr);
      W val;
      if (r >= S && r < (int64_t)S + A) {
        const int pk = a.keep[(int64_t)b * a.keep_stride + (r - S)];
        const int64_t t = qb + pk;
        if (pk < 0 || t < 0 || t >= a.pack_rows) {
          if (w == 0) report(CAST_DEV_BAD_LAYOUT);
          continue;
        }
        val = reinterpret_cast<const W*>(pack + t * a.pk_st)[w];
      } else if (r < a.src_cap) {
        val = reinterpret_cast<const W*>(src + r * a.src_sr)[w];
      } else {
        val = W{};
      }
      reinterpret_cast<W*>(dst + r * a.dst_sr)[w] = val;
    }
  }
}
// Append-only form: CTA (nb, layer group) writes the accepted rows of request nb
// for every head of LAYERS_PER_CTA layers (a few rows each: one CTA per head and
// layer would leave the GPU launch-bound).
constexpr int LAYERS_PER_CTA = 4;

template <typename W>
__global__ void __launch_bounds__(NT) kv_append_kernel(const KvArgs a, const Layers ly) {
  const int nb = blockIdx.x;
  const int l0 = blockIdx.y * LAYERS_PER_CTA;
  const int nl = min(LAYERS_PER_CTA, a.L - l0);
  const int b = nb;
  const int S = a.store_len[b], A = a.accepted[b];
  if (S < 0 || A < 0 || (int64_t)S + A > a.dst_cap || A > a.keep_stride) {
    if (threadIdx.x == 0 && blockIdx.y == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  if (A == 0) return;
  const int wpr = a.row_bytes / (int)sizeof(W);
  const int64_t qb = a.cu_q ? a.cu_q[b] : 0;
  const int64_t per_kv = (int64_t)a.H * A * wpr;       // words of one layer's K (or V)
  const int64_t total = per_kv * 2 * nl;
  for (int64_t e = threadIdx.x; e < total; e += NT) {
    const int w = (int)(e % wpr);
    int64_t rest = e / wpr;
    const int j = (int)(rest % A);
    rest /= A;
    const int h = (int)(rest % a.H);
    rest /= a.H;
    const int kv = (int)(rest & 1);
    const int l = l0 + (int)(rest >> 1);
    const int pk = a.keep[(int64_t)b * a.keep_stride + j];
    const int64_t t = qb + pk;
    if (pk < 0 || t < 0 || t >= a.pack_rows) {
      if (w == 0) report(CAST_DEV_BAD_LAYOUT);
      continue;
    }
    const char* pack = static_cast<const char*>(ly.pack[l][kv]) + h * a.pk_sh + t * a.pk_st;
    char* dst = static_cast<char*>(ly.dst[l][kv]) + nb * a.dst_sb + h * a.dst_sh + (S + j) * a.dst_sr;
    reinterpret_cast<W*>(dst)[w] = reinterpret_cast<const W*>(pack)[w];
  }
}
}  // namespace kvg

}  // namespace cast
