// Tree construction on the GPU: per-row top-k of fp64 log-softmax, then the
// best-first tree of each sequence, node for node the reference's pop order.
#pragma once

#include "common.cuh"
#include "tc_common.cuh"

namespace cast {

// ---------------------------------------------------------------------------
// block_topk (cast_trees/tree.py:20-26).
//
// One CTA per row of V logits; the common case reads the row once. Each
// thread keeps
//  * the exact running max (the reference's x.max()),
//  * sum_t = sum of exp(x - ref_t) against a reference ref_t that moves only
//    when an element exceeds it by more than 2^8 nats worth of headroom (so
//    the sum never overflows; fp64 keeps its relative precision at any scale),
//  * its 8 best (x, index) candidates, sorted by x descending; a thread visits
//    its elements in increasing index order, so an equal x never displaces an
//    earlier one (the stable sort's lower-index-first rule).
// The CTA merges the thread lists into its KC best by (x desc, index asc).
// That set is exactly the row's KC best unless some thread's 8th candidate is
// itself among them (the thread may have dropped a 9th): such rows take the
// exact path below. The row max M is the best candidate. With M the max and lse = log(sum exp(x - M)), the KC
// candidates get lp = (x - M) - lse (the reference's operation order) and are
// re-sorted by (lp desc, index asc); rounding in that subtraction can map
// distinct x to one lp, so when the k-th and KC-th lp are equal an element
// outside the candidates could tie into the top k, and the row also takes the
// exact path: a second read that selects the top k on lp itself.
// ---------------------------------------------------------------------------
namespace topk {
constexpr int NT = 128;
constexpr int NW = NT / 32;
constexpr int TL = 8;  // candidates per thread in the common path
}

// exp(t) in float64 for t <= 709, written from the mathematics: Cody-Waite
// reduction t = k ln2 + r with ln 2 split into a 33-bit head (k * head exact
// for |k| < 2^20) and its tail, |r| <= ln2/2, then the degree-10 Taylor
// polynomial of e^r by Horner's rule (truncation < 2.3e-13 relative: the
// log-sum it feeds is then within 2.3e-13 absolute, far inside the 1e-12
// relative bound on log-probs) and an exponent-field scale by 2^k. Results
// below 2^-1022 are returned as 0: such terms are more than 700 nats below the
// running reference and cannot move a sum that includes a term of size 1.
// The kernel is bound by the float64 pipe, so the degree is kept minimal.
__device__ __forceinline__ double exp_fast(double t) {
  constexpr double kLog2e = 1.4426950408889634;
  constexpr double kLn2Hi = 0.6931471803691238;        // 0x1.62e42fee00000p-1
  constexpr double kLn2Lo = 1.9082149292705877e-10;    // ln 2 - kLn2Hi
  constexpr double kShift = 6755399441055744.0;        // 1.5 * 2^52: rounds to an integer in the low bits
  const double kd = fma(t, kLog2e, kShift);
  const int k = (int)(__double_as_longlong(kd) & 0xFFFFFFFFll);
  const double kf = kd - kShift;
  const double r = fma(-kf, kLn2Lo, fma(-kf, kLn2Hi, t));
  double p = 2.755731922398589e-07;                   // 1/10!
  p = fma(p, r, 2.7557319223985893e-06);              // 1/9!
  p = fma(p, r, 2.48015873015873e-05);                // 1/8!
  p = fma(p, r, 0.0001984126984126984);               // 1/7!
  p = fma(p, r, 0.001388888888888889);                // 1/6!
  p = fma(p, r, 0.008333333333333333);                // 1/5!
  p = fma(p, r, 0.041666666666666664);                // 1/4!
  p = fma(p, r, 0.16666666666666666);                 // 1/3!
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  if (k < -1022) return 0.0;
  return p * __longlong_as_double((long long)(k + 1023) << 52);
}

// exp_fast for t >= -708 (callers clamp): no underflow check, 2^k is always a normal number.
__device__ __forceinline__ double exp_fast_clamped(double t) {
  constexpr double kLog2e = 1.4426950408889634;
  constexpr double kLn2Hi = 0.6931471803691238;
  constexpr double kLn2Lo = 1.9082149292705877e-10;
  constexpr double kShift = 6755399441055744.0;
  const double kd = fma(t, kLog2e, kShift);
  const int k = __double2loint(kd);
  const double kf = kd - kShift;
  const double r = fma(-kf, kLn2Lo, fma(-kf, kLn2Hi, t));
  double p = 2.755731922398589e-07;
  p = fma(p, r, 2.7557319223985893e-06);
  p = fma(p, r, 2.48015873015873e-05);
  p = fma(p, r, 0.0001984126984126984);
  p = fma(p, r, 0.001388888888888889);
  p = fma(p, r, 0.008333333333333333);
  p = fma(p, r, 0.041666666666666664);
  p = fma(p, r, 0.16666666666666666);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return p * __hiloint2double((k + 1023) << 20, 0);
}

// exp(t) in float64 for -708 <= t <= 709 from a 64-entry table (callers clamp): t = (64 n + i) ln2/64 + r
// with |r| <= ln2/128 (Cody-Waite with the split ln 2 of exp_fast, scaled by 1/64, exact for |64 n + i|
// < 2^20), e^t = 2^n * 2^(i/64) * e^r, e^r by its degree-5 Taylor polynomial (truncation < 4e-17
// relative) and 2^n added to the exponent field of the table entry. Ten float64 operations against
// exp_fast's sixteen; `tab` holds 2^(i/64), i = 0..63 (exp2_table_init).
// The constants live in the constant bank, where an fp64 instruction reads them as an operand: as
// literals they were rebuilt from two 32-bit moves at every use under the kernel's register budget.
__constant__ double c_exp_tab[9] = {
    92.33248261689366,             // 64 / ln 2
    6755399441055744.0,            // 1.5 * 2^52
    -0.6931471803691238 / 64.0,    // -(ln 2 head) / 64, exact: a power-of-two scale of exp_fast's split
    -1.9082149292705877e-10 / 64.0,
    1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0, 0.5, 1.0};
__device__ __forceinline__ double exp_tab(double t, const double* tab) {
  const double kd = fma(t, c_exp_tab[0], c_exp_tab[1]);
  const int m = __double2loint(kd);
  const double kf = kd - c_exp_tab[1];
  const double r = fma(kf, c_exp_tab[3], fma(kf, c_exp_tab[2], t));
  double p = c_exp_tab[4];
  p = fma(p, r, c_exp_tab[5]);
  p = fma(p, r, c_exp_tab[6]);
  p = fma(p, r, c_exp_tab[7]);
  p = fma(p, r, c_exp_tab[8]);
  p = fma(p, r, c_exp_tab[8]);
  const double tv = tab[m & 63];
  return p * __hiloint2double(__double2hiint(tv) + ((m >> 6) << 20), __double2loint(tv));
}

__device__ __forceinline__ void exp2_table_init(double* tab) {
  for (int i = threadIdx.x; i < 64; i += blockDim.x) tab[i] = exp2((double)i / 64.0);
}

// Folds one element into a thread's (reference, sum of exp(x - reference)).
__device__ __forceinline__ void lse_add(double& ref, double& s, double v) {
  if (v == -INFINITY) return;
  double t = v - ref;
  if (!(t <= 256.0)) {
    s = (ref == -INFINITY) ? 0.0 : s * exp_fast(ref - v);
    ref = v;
    t = 0.0;
  }
  s += exp_fast(t);
}

template <int KC>
struct CandList {
  double x[KC];
  int idx[KC];  // -1 = empty slot (ranks below every real element)

  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < KC; ++i) { x[i] = -INFINITY; idx[i] = -1; }
  }
  __device__ __forceinline__ bool wants(double v) const { return idx[KC - 1] < 0 || v > x[KC - 1]; }
  // j is larger than every index already held (increasing visit order).
  __device__ __forceinline__ void insert(double v, int j) {
    x[KC - 1] = v;
    idx[KC - 1] = j;
#pragma unroll
    for (int i = KC - 1; i > 0; --i) {
      const bool up = idx[i - 1] < 0 || x[i] > x[i - 1];
      if (up) {
        const double tx = x[i]; x[i] = x[i - 1]; x[i - 1] = tx;
        const int ti = idx[i]; idx[i] = idx[i - 1]; idx[i - 1] = ti;
      }
    }
  }
  __device__ __forceinline__ void offer(double v, int j) {
    if (wants(v)) insert(v, j);
  }
  __device__ __forceinline__ void pop_front() {
#pragma unroll
    for (int i = 0; i < KC - 1; ++i) { x[i] = x[i + 1]; idx[i] = idx[i + 1]; }
    x[KC - 1] = -INFINITY;
    idx[KC - 1] = -1;
  }
};

// (a_x, a_i) ranks before (b_x, b_i): larger value, then smaller index; empty last.
__device__ __forceinline__ bool cand_before(double ax, int ai, double bx, int bi) {
  if (ai < 0) return false;
  if (bi < 0) return true;
  return ax > bx || (ax == bx && ai < bi);
}

// Visits the row in each thread's increasing index order: f(value, index).
template <bool VEC2, typename F>
__device__ __forceinline__ void scan_row(const double* x, int64_t V, F&& f) {
  using namespace topk;
  const int tid = threadIdx.x;
  if (VEC2) {
    const double2* x2 = reinterpret_cast<const double2*>(x);
    const int64_t n2 = V >> 1;
    int64_t i = tid;
    for (; i + 3 * NT < n2; i += 4 * NT) {
      double2 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(x2 + i + u * NT);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = (int)(2 * (i + u * NT));
        f(v[u].x, j);
        f(v[u].y, j + 1);
      }
    }
    for (; i < n2; i += NT) {
      const double2 v = __ldcs(x2 + i);
      const int j = (int)(2 * i);
      f(v.x, j);
      f(v.y, j + 1);
    }
    if ((V & 1) && tid == 0) f(x[V - 1], (int)(V - 1));
  } else {
    for (int64_t i = tid; i < V; i += NT) f(x[i], (int)i);
  }
}

template <int KC>
__device__ __forceinline__ void merge_warp_lists(double* s_cx, int* s_ci, double* s_out_x, int* s_out_i);

// Merges every thread's sorted list into s_out_* (the CTA's KC best, best first).
template <int KC, int TLN>
__device__ __forceinline__ void merge_lists(CandList<TLN>& cl, double* s_cx, int* s_ci, double* s_out_x,
                                            int* s_out_i) {
  using namespace topk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int rnd = 0; rnd < KC; ++rnd) {       // warp level: KC rounds of an arg-best
    double bx = cl.x[0];
    int bi = cl.idx[0];
    int bl = lane;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const double ox = __shfl_xor_sync(0xffffffffu, bx, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, off);
      if (cand_before(ox, oi, bx, bi) || (oi == bi && ol < bl)) { bx = ox; bi = oi; bl = ol; }
    }
    if (lane == bl && bi >= 0) cl.pop_front();
    if (lane == 0) { s_cx[warp * KC + rnd] = bx; s_ci[warp * KC + rnd] = bi; }
  }
  merge_warp_lists<KC>(s_cx, s_ci, s_out_x, s_out_i);
}

// CTA level: the KC best of the NW warp lists in s_cx / s_ci (index -1 = empty) into s_out_*.
template <int KC>
__device__ __forceinline__ void merge_warp_lists(double* s_cx, int* s_ci, double* s_out_x, int* s_out_i) {
  using namespace topk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (warp == 0) {                            // CTA level, over the NW warp lists
    for (int rnd = 0; rnd < KC; ++rnd) {
      double bx = -INFINITY;
      int bi = -1, bslot = -1;
      for (int c = lane; c < NW * KC; c += 32) {
        if (cand_before(s_cx[c], s_ci[c], bx, bi)) { bx = s_cx[c]; bi = s_ci[c]; bslot = c; }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const double ox = __shfl_xor_sync(0xffffffffu, bx, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        const int os = __shfl_xor_sync(0xffffffffu, bslot, off);
        if (cand_before(ox, oi, bx, bi)) { bx = ox; bi = oi; bslot = os; }
      }
      if (lane == 0) {
        s_out_x[rnd] = bx;
        s_out_i[rnd] = bi;
        if (bslot >= 0) s_ci[bslot] = -1;  // taken
      }
      __syncwarp();
    }
  }
  __syncthreads();
}

// Warp-level candidate set of the fast path: the warp's KC best (x desc, index
// asc) seen so far live in a shared-memory buffer behind a threshold (the KC-th
// of them); an element enters the buffer only if it beats the threshold, which
// after the first few hundred elements is rare, so the common per-element cost
// is one comparison and a ballot. When the buffer passes CAP - 32 entries it is
// cut back to its KC best.
namespace topk {
constexpr int CAP = 64;
}

template <int KC>
struct WarpCands {
  double* x;   // [CAP] of this warp
  int* i;
  int n;       // entries held (warp-uniform)
  double tx;   // threshold: the KC-th best held (valid once n >= KC after a cut)
  int ti;
  bool full;

  // Keeps the KC best of the n entries, in order, and sets the threshold.
  __device__ __forceinline__ void cut() {
    const int lane = threadIdx.x & 31;
    __syncwarp();
    double vx[topk::CAP / 32];
    int vi[topk::CAP / 32], rk[topk::CAP / 32];
#pragma unroll
    for (int u = 0; u < topk::CAP / 32; ++u) {
      const int e = lane + 32 * u;
      vx[u] = e < n ? x[e] : -INFINITY;
      vi[u] = e < n ? i[e] : -1;
      int r = 0;
      if (e < n)
        for (int f = 0; f < n; ++f) r += cand_before(x[f], i[f], vx[u], vi[u]);
      rk[u] = r;
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < topk::CAP / 32; ++u)
      if (vi[u] >= 0 && rk[u] < KC) { x[rk[u]] = vx[u]; i[rk[u]] = vi[u]; }
    __syncwarp();
    n = min(n, KC);
    full = n >= KC;
    if (full) { tx = x[KC - 1]; ti = i[KC - 1]; }
  }

  // One element per lane (valid = inside the row); every lane of the warp calls it.
  __device__ __forceinline__ void offer(double v, int j, bool valid) {
    const int lane = threadIdx.x & 31;
    // v >= tx admits a superset (equal values the cut then ranks by index): one comparison
    const bool pass = valid && (!full || v >= tx);
    const unsigned mask = __ballot_sync(0xffffffffu, pass);
    if (mask) {
      if (pass) {
        const int pos = n + __popc(mask & ((1u << lane) - 1u));
        x[pos] = v;
        i[pos] = j;
      }
      n += __popc(mask);
      if (n > topk::CAP - 32) cut();
    }
  }
};

// Shared memory of one row's top-k: warp candidate buffers, the merge lists and the exp table.
template <int KC>
struct TopkSmem {
  double r[topk::NW], sum[topk::NW];
  double cx[topk::NW * KC];
  int ci[topk::NW * KC];
  double fx[KC], flp[KC];
  int fi[KC];
  double wx[topk::NW][topk::CAP];
  int wi[topk::NW][topk::CAP];
  double tab[64];
};

// One thread's share of a row: its warp's candidate buffer and its lazily rescaled fp64 sum of
// exp(x - ref). The reference moves once per batch of 8 elements: when the batch max exceeds it by
// more than 256, so every exp argument is at most 256.
template <int KC>
struct TopkRow {
  WarpCands<KC> wc;
  double ref, s;
  const double* tab;

  // A batch of up to 8 elements (nb valid slots; ok[u] marks elements inside the row, ALL_OK that all
  // are; elements past the row are -inf). Every lane of the warp calls it the same number of times.
  // index(u) gives element u's index; it is evaluated only when an element enters the buffer.
  template <bool ALL_OK, typename IndexF>
  __device__ __forceinline__ void add8(const double (&v)[8], IndexF&& index, const bool (&ok)[8], int nb) {
    constexpr bool all_ok = ALL_OK;
    double mv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mv[u] = (u < nb && (all_ok || ok[u])) ? v[u] : -INFINITY;
    const double bm = fmax(fmax(fmax(mv[0], mv[1]), fmax(mv[2], mv[3])), fmax(fmax(mv[4], mv[5]), fmax(mv[6], mv[7])));
    if (bm != -INFINITY && !(bm - ref <= 256.0)) {
      s = (ref == -INFINITY) ? 0.0 : s * exp_fast(ref - bm);
      ref = bm;
    }
    // an argument clamped at -708 (elements past the row are -inf) adds at most 2^-1022,
    // nothing next to a sum that holds a term of 1
    double e[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) e[u] = u < nb ? exp_tab(fmax(v[u] - ref, -708.0), tab) : 0.0;
    s += ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));   // a tree: short dependency chain
    // candidates: one vote per batch on its max; the per-element offers (a ballot each, in element
    // order) run only when some lane's batch max clears the threshold as it stands at the batch start
    // (the threshold only rises, so this admits a superset of what the offers take in)
    if (__any_sync(0xffffffffu, !wc.full || bm >= wc.tx)) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < nb) wc.offer(v[u], index(u), all_ok || ok[u]);
    }
  }
};

// After the row: the CTA's KC best, M = the best, lse = log of the merged sums, lp = (x - M) - lse in
// the reference's order, sorted by (lp desc, index asc); a tie at the k-th / KC-th lp hands the row
// to block_topk_exact_kernel (top_idx[row][0] = -1).
template <int KC>
__device__ __forceinline__ void topk_finish(TopkRow<KC>& rw, TopkSmem<KC>& sm, int64_t V, int k, int64_t row,
                                            int64_t* __restrict__ top_idx, double* __restrict__ top_lp) {
  using namespace topk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  rw.wc.cut();   // the warp's KC best, in order
  double ref = rw.ref, s = rw.s;
  // (reference, sum): warp, then CTA
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double orf = __shfl_xor_sync(0xffffffffu, ref, off);
    const double os = __shfl_xor_sync(0xffffffffu, s, off);
    const double nr = fmax(ref, orf);
    if (nr != -INFINITY) {
      s = (ref == -INFINITY ? 0.0 : s * exp_fast(ref - nr)) + (orf == -INFINITY ? 0.0 : os * exp_fast(orf - nr));
    }
    ref = nr;
  }
  if (lane == 0) { sm.r[warp] = ref; sm.sum[warp] = s; }
  for (int c = lane; c < KC; c += 32) {
    sm.cx[warp * KC + c] = c < rw.wc.n ? rw.wc.x[c] : -INFINITY;
    sm.ci[warp * KC + c] = c < rw.wc.n ? rw.wc.i[c] : -1;
  }
  merge_warp_lists<KC>(sm.cx, sm.ci, sm.fx, sm.fi);

  if (tid == 0) {
    const double M = sm.fi[0] >= 0 ? sm.fx[0] : -INFINITY;   // the row max is the best candidate
    double S = 0.0;
    for (int w = 0; w < NW; ++w)
      if (sm.r[w] != -INFINITY) S += sm.sum[w] * exp_fast(sm.r[w] - M);
    const double lse = log(S);
    int n = 0;
    for (int c = 0; c < KC; ++c) {
      if (sm.fi[c] < 0) break;
      sm.flp[c] = (sm.fx[c] - M) - lse;
      ++n;
    }
    // stable insertion sort by (lp desc, index asc)
    for (int a = 1; a < n; ++a) {
      const double lv = sm.flp[a];
      const int iv = sm.fi[a];
      int c = a - 1;
      while (c >= 0 && (sm.flp[c] < lv || (sm.flp[c] == lv && sm.fi[c] > iv))) {
        sm.flp[c + 1] = sm.flp[c];
        sm.fi[c + 1] = sm.fi[c];
        --c;
      }
      sm.flp[c + 1] = lv;
      sm.fi[c + 1] = iv;
    }
    const bool tie = V > KC && n == KC && sm.flp[k - 1] == sm.flp[KC - 1];
    if (tie) {
      top_idx[row * k] = -1;  // hands the row to block_topk_exact_kernel
    } else {
      for (int c = 0; c < k; ++c) {
        top_idx[row * k + c] = c < n ? (int64_t)sm.fi[c] : (int64_t)0;
        top_lp[row * k + c] = c < n ? sm.flp[c] : -INFINITY;
      }
    }
  }
}

// Rows read with plain loads (any alignment): each thread loads 8 elements per batch.
template <int KC, bool VEC2>
__global__ void __launch_bounds__(topk::NT, 8)   // eight CTAs per SM (64 registers): one wave of rows
block_topk_kernel(const double* __restrict__ logits, int64_t V, int64_t row_stride, int k,
                  int64_t* __restrict__ top_idx, double* __restrict__ top_lp) {
  using namespace topk;
  __shared__ TopkSmem<KC> sm;
  const int64_t row = blockIdx.x;
  const double* x = logits + row * row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  exp2_table_init(sm.tab);
  __syncthreads();
  TopkRow<KC> rw{WarpCands<KC>{sm.wx[warp], sm.wi[warp], 0, -INFINITY, -1, false}, -INFINITY, 0.0, sm.tab};
  if (VEC2) {
    const double2* x2 = reinterpret_cast<const double2*>(x);
    const int64_t n2 = V >> 1;
    const int64_t n2_full = n2 - n2 % (4 * NT);   // batches every lane's loads stay inside
    int64_t base = 0;
    for (; base < n2_full; base += 4 * NT) {
      double v[8];
      const bool ok[8] = {true, true, true, true, true, true, true, true};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const double2 d = __ldcs(x2 + base + u * NT + tid);
        v[2 * u] = d.x; v[2 * u + 1] = d.y;
      }
      rw.template add8<true>(v, [&](int u) { return (int)(2 * (base + (u >> 1) * NT + tid)) + (u & 1); }, ok, 8);
    }
    if (base < n2) {   // the last, partial batch
      double v[8];
      bool ok[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t ii = base + u * NT + tid;
        const bool in = ii < n2;
        const double2 d = in ? __ldcs(x2 + ii) : make_double2(-INFINITY, -INFINITY);
        v[2 * u] = d.x; v[2 * u + 1] = d.y;
        ok[2 * u] = in; ok[2 * u + 1] = in;
      }
      rw.template add8<false>(v, [&](int u) { return (int)(2 * (base + (u >> 1) * NT + tid)) + (u & 1); }, ok, 8);
    }
    if (V & 1) {   // the odd last element: lane 0 of warp 0, the warp calls together
      if (warp == 0) {
        double v[8] = {lane == 0 ? x[V - 1] : -INFINITY};
        bool ok[8] = {lane == 0};
        rw.template add8<false>(v, [&](int) { return (int)(V - 1); }, ok, 1);
      }
    }
  } else {
    for (int64_t base = 0; base < V; base += 8 * NT) {
      double v[8];
      bool ok[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t ii = base + u * NT + tid;
        ok[u] = ii < V;
        v[u] = ok[u] ? x[ii] : -INFINITY;
      }
      rw.template add8<false>(v, [&](int u) { return (int)(base + u * NT + tid); }, ok, 8);
    }
  }
  topk_finish<KC>(rw, sm, V, k, row, top_idx, top_lp);
}

// Exact path of rows block_topk_kernel flagged (top_idx[row][0] == -1): one
// read for the max and log-sum, a second that selects the k best on
// lp = (x - M) - lse itself. Other rows exit at once.
template <int KC, bool VEC2>
__global__ void __launch_bounds__(topk::NT)
block_topk_exact_kernel(const double* __restrict__ logits, int64_t V, int64_t row_stride, int k,
                        int64_t* __restrict__ top_idx, double* __restrict__ top_lp) {
  using namespace topk;
  __shared__ double s_m[NW], s_r[NW], s_s[NW];
  __shared__ double s_cx[NW * KC];
  __shared__ int s_ci[NW * KC];
  __shared__ double s_flp[KC];
  __shared__ int s_fi[KC];
  __shared__ double s_M, s_lse;
  const int64_t row = blockIdx.x;
  if (top_idx[row * k] >= 0) return;
  const double* x = logits + row * row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  double mx = -INFINITY, ref = -INFINITY, s = 0.0;
  scan_row<VEC2>(x, V, [&](double v, int) {
    mx = fmax(mx, v);
    lse_add(ref, s, v);
  });
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const double orf = __shfl_xor_sync(0xffffffffu, ref, off);
    const double os = __shfl_xor_sync(0xffffffffu, s, off);
    const double nr = fmax(ref, orf);
    if (nr != -INFINITY)
      s = (ref == -INFINITY ? 0.0 : s * exp_fast(ref - nr)) + (orf == -INFINITY ? 0.0 : os * exp_fast(orf - nr));
    ref = nr;
  }
  if (lane == 0) { s_m[warp] = mx; s_r[warp] = ref; s_s[warp] = s; }
  __syncthreads();
  if (tid == 0) {
    double M = s_m[0];
    for (int w = 1; w < NW; ++w) M = fmax(M, s_m[w]);
    double S = 0.0;
    for (int w = 0; w < NW; ++w)
      if (s_r[w] != -INFINITY) S += s_s[w] * exp_fast(s_r[w] - M);
    s_M = M;
    s_lse = log(S);
  }
  __syncthreads();
  const double M = s_M, lse = s_lse;
  CandList<KC> full;
  full.init();
  scan_row<VEC2>(x, V, [&](double v, int j) { full.offer((v - M) - lse, j); });
  merge_lists<KC, KC>(full, s_cx, s_ci, s_flp, s_fi);
  if (tid == 0) {
    for (int c = 0; c < k; ++c) {
      top_idx[row * k + c] = s_fi[c] >= 0 ? (int64_t)s_fi[c] : (int64_t)0;
      top_lp[row * k + c] = s_fi[c] >= 0 ? s_flp[c] : -INFINITY;
    }
  }
}

// ---------------------------------------------------------------------------
// build_tree (cast_trees/tree.py:29-49), one warp per tree.
//
// The reference pops a heap keyed by (neg, depth, parent, rank) and pushes all
// k children of every popped node. Siblings share depth and parent, so a
// node's children leave that heap in the order of (neg_child, rank). Keeping
// only each expanded node's next unpopped child in the candidate set therefore
// never changes the minimum: any pushed-but-unpopped child has a sibling of
// equal or smaller key in the set. The set holds at most budget + 1 entries;
// each pop is a warp arg-min over it, the popped slot takes the next sibling,
// and the new node's first child is appended. Keys compare exactly like
// Python tuples: neg as an ordered 64-bit pattern (with -0.0 folded into
// +0.0, which Python treats as equal), then (depth, parent + 1, rank) packed
// into a second word. Scores use the reference's float64 operations:
// -lp[0, r] at depth 1, neg_parent - lp[d, r] below.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ordered_key(double v) {
  const uint64_t u = (uint64_t)__double_as_longlong(v + 0.0);
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

struct TreeArgs {
  const int64_t* top_idx;
  const double* top_lp;
  int B, L, k_cols, k;
  const int32_t* budget;
  int max_budget;
  int32_t* token;
  int32_t* depth;
  int32_t* parent;
  double* score;
  int32_t* count;
  const int32_t* cu_q;
  int32_t* pack_parent;
  const int32_t* root_token;
  int32_t* pack_token;
  const int32_t* seq_len;
  int32_t* pack_pos;
};

__host__ __device__ inline size_t tree_smem_bytes(int max_budget, int L, int k) {
  const size_t nc = (size_t)max_budget + 1;
  return nc * (2 * sizeof(uint64_t) + sizeof(double) + 4 * sizeof(int)) +  // candidates
         (size_t)max_budget * (sizeof(double) + sizeof(int32_t)) +        // node neg and (parent, depth, rank)
         ((size_t)max_budget + 1) * k * sizeof(unsigned char) +            // child order per node (+root)
         (size_t)L * k * sizeof(double) +                                  // lp rows
         (size_t)L * k * sizeof(int32_t) + 64;                             // token rows
}

// Warp-wide arg-min of a 128-bit key (hi, lo); every lane returns the winner's
// slot (-1 if no lane has one). Up to four 32-bit redux.sync rounds, most
// significant word first (one when a single lane holds the least first word),
// then the one lane left holding the minimum.
__device__ __forceinline__ int warp_argmin128(uint64_t hi, uint64_t lo, int slot) {
  unsigned live = 0xffffffffu;
  bool mine = slot >= 0;
  // every lane takes part in each reduction (computed before it is compared)
  const uint32_t w0 = (uint32_t)(hi >> 32);
  const uint32_t m0 = __reduce_min_sync(0xffffffffu, mine ? w0 : 0xffffffffu);
  mine = mine && w0 == m0;
  // usually one lane is left after the first word: the other words cannot change the winner
  if (__popc(__ballot_sync(0xffffffffu, mine)) != 1) {
    const uint32_t w1 = (uint32_t)hi, w2 = (uint32_t)(lo >> 32), w3 = (uint32_t)lo;
    const uint32_t m1 = __reduce_min_sync(0xffffffffu, mine ? w1 : 0xffffffffu);
    mine = mine && w1 == m1;
    const uint32_t m2 = __reduce_min_sync(0xffffffffu, mine ? w2 : 0xffffffffu);
    mine = mine && w2 == m2;
    const uint32_t m3 = __reduce_min_sync(0xffffffffu, mine ? w3 : 0xffffffffu);
    mine = mine && w3 == m3;
  }
  live = __ballot_sync(0xffffffffu, mine);
  if (live == 0) return -1;
  return __shfl_sync(0xffffffffu, slot, __ffs(live) - 1);
}

__global__ void __launch_bounds__(32) build_tree_kernel(const TreeArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  const int k = a.k, L = a.L;
  const int nc_max = a.max_budget + 1;
  uint64_t* c_hi = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* c_lo = c_hi + nc_max;
  double* c_neg = reinterpret_cast<double*>(c_lo + nc_max);
  int* c_par = reinterpret_cast<int*>(c_neg + nc_max);  // parent node (-1 = root)
  int* c_j = c_par + nc_max;                            // position in the parent's child order
  int* c_d = c_j + nc_max;                              // depth of the candidate
  int* c_r = c_d + nc_max;                              // rank
  double* n_neg = reinterpret_cast<double*>(c_r + nc_max);
  double* s_lp = n_neg + a.max_budget;
  int32_t* s_tok = reinterpret_cast<int32_t*>(s_lp + (size_t)L * k);                // token of each (row, rank)
  int32_t* n_info = s_tok + (size_t)L * k;                     // popped node: (parent + 1) | depth << 16 | rank << 24
  unsigned char* order = reinterpret_cast<unsigned char*>(n_info + a.max_budget);  // [(1 + max_budget)][k], row 0 = root

  int budget = a.budget[b];
  if (budget > a.max_budget || budget < 0) {
    if (lane == 0) { report(CAST_DEV_TREE_OVERFLOW); a.count[b] = 0; }
    return;
  }
  const double* lp_g = a.top_lp + (size_t)b * L * a.k_cols;
  const int64_t* idx_g = a.top_idx + (size_t)b * L * a.k_cols;
  bool sorted_rows = true;
  // the tree's lp and token tables, staged once: no global load on the pop loop's dependency chain
  for (int e = lane; e < L * k; e += 32) {
    const double v = lp_g[(e / k) * a.k_cols + (e % k)];
    s_lp[e] = v;
    s_tok[e] = (int32_t)idx_g[(e / k) * a.k_cols + (e % k)];
    if (e % k != k - 1 && !(v >= lp_g[(e / k) * a.k_cols + (e % k) + 1])) sorted_rows = false;
  }
  // Rows sorted best-first (block_topk's output): fl(neg - lp[d, r]) is then
  // non-decreasing in r, so every node's children leave the heap in rank
  // order and the sibling order needs no sorting.
  sorted_rows = __all_sync(0xffffffffu, sorted_rows);
  __syncwarp();

  // child order of a node whose own neg is `base` (root: children neg = -lp[0, r])
  auto child_order = [&](int slot, bool root, double base, int d) {
    if (sorted_rows) return;
    uint64_t hi = ~0ull;
    if (lane < k) hi = ordered_key(root ? -s_lp[lane] : base - s_lp[d * k + lane]);
    int rank = 0;
    for (int r2 = 0; r2 < k; ++r2) {
      const uint64_t h2 = __shfl_sync(0xffffffffu, hi, r2);
      if (lane < k && (h2 < hi || (h2 == hi && r2 < lane))) ++rank;
    }
    if (lane < k) order[(size_t)slot * k + rank] = (unsigned char)lane;
    __syncwarp();
  };
  auto nth_child = [&](int slot, int j) -> int { return sorted_rows ? j : (int)order[(size_t)slot * k + j]; };

  int ncand = 0;
  if (budget > 0 && k > 0 && L > 0) {
    child_order(0, true, 0.0, 0);
    if (lane == 0) {
      const int r = nth_child(0, 0);
      const double neg = -s_lp[r];
      c_hi[0] = ordered_key(neg);
      c_lo[0] = (1ull << 40) | (0ull << 8) | (uint64_t)r;
      c_neg[0] = neg; c_par[0] = -1; c_j[0] = 0; c_d[0] = 1; c_r[0] = r;
    }
    ncand = 1;
    __syncwarp();
  }

  int n = 0;
  const int q0 = a.cu_q ? a.cu_q[b] : 0;
  const int pos0 = (a.cu_q && a.pack_pos) ? a.seq_len[b] : 0;
  bool pack_ok = true;
  if (a.cu_q && lane == 0) {
    pack_ok = q0 >= 0 && (long long)q0 + 1 + budget <= (long long)a.cu_q[b + 1];
    if (!pack_ok) report(CAST_DEV_BAD_LAYOUT);
  }
  pack_ok = __shfl_sync(0xffffffffu, pack_ok ? 1 : 0, 0) != 0;

  while (n < budget && ncand > 0) {
    // arg-min over the candidate set: a scan of this lane's slots, then the warp
    uint64_t bh = ~0ull, bl = ~0ull;
    int bs = -1;
    for (int c = lane; c < ncand; c += 32) {
      const uint64_t h = c_hi[c], l = c_lo[c];
      if (bs < 0 || h < bh || (h == bh && l < bl)) { bh = h; bl = l; bs = c; }
    }
    const int slot = warp_argmin128(bh, bl, bs);
    const double neg = c_neg[slot];
    const int par = c_par[slot], j = c_j[slot], d = c_d[slot], r = c_r[slot];
    const int me = n;
    __syncwarp();  // every lane has read the slot before lane 0 rewrites it
    if (lane == 0) {   // the outputs are written after the loop, all lanes together
      n_neg[me] = neg;
      n_info[me] = (par + 1) | (d << 16) | (r << 24);
      // the popped slot takes the next sibling, or the last candidate
      if (j + 1 < k) {
        const int r2 = nth_child(par + 1, j + 1);
        const double sneg = (par < 0) ? -s_lp[r2] : n_neg[par] - s_lp[(size_t)(d - 1) * k + r2];
        c_hi[slot] = ordered_key(sneg);
        c_lo[slot] = ((uint64_t)d << 40) | ((uint64_t)(par + 1) << 8) | (uint64_t)r2;
        c_neg[slot] = sneg; c_j[slot] = j + 1; c_r[slot] = r2;
      } else {
        const int last = ncand - 1;
        c_hi[slot] = c_hi[last]; c_lo[slot] = c_lo[last]; c_neg[slot] = c_neg[last];
        c_par[slot] = c_par[last]; c_j[slot] = c_j[last]; c_d[slot] = c_d[last]; c_r[slot] = c_r[last];
      }
    }
    if (j + 1 >= k) --ncand;
    __syncwarp();
    if (d < L) {
      child_order(me + 1, false, neg, d);
      if (lane == 0) {
        const int r2 = nth_child(me + 1, 0);
        const double cneg = neg - s_lp[(size_t)d * k + r2];
        const int c = ncand;
        c_hi[c] = ordered_key(cneg);
        c_lo[c] = ((uint64_t)(d + 1) << 40) | ((uint64_t)(me + 1) << 8) | (uint64_t)r2;
        c_neg[c] = cneg; c_par[c] = me; c_j[c] = 0; c_d[c] = d + 1; c_r[c] = r2;
      }
      ++ncand;
    }
    ++n;
    __syncwarp();
  }
  for (int me = lane; me < n; me += 32) {
    const int info = n_info[me];
    const int par = (info & 0xffff) - 1, d = (info >> 16) & 0xff, r = info >> 24;
    const int tok = s_tok[(size_t)(d - 1) * k + r];
    const size_t o = (size_t)b * a.max_budget + me;
    a.token[o] = tok;
    a.depth[o] = d;
    a.parent[o] = par;
    a.score[o] = -n_neg[me];
    if (a.cu_q && pack_ok) {
      if (a.pack_parent) a.pack_parent[q0 + 1 + me] = par + 1;
      if (a.pack_token) a.pack_token[q0 + 1 + me] = tok;
      if (a.pack_pos) a.pack_pos[q0 + 1 + me] = pos0 + d;
    }
  }
  if (lane == 0) {
    a.count[b] = n;
    if (a.cu_q && pack_ok) {
      if (a.pack_parent) a.pack_parent[q0] = -1;
      if (a.pack_token) a.pack_token[q0] = a.root_token[b];
      if (a.pack_pos) a.pack_pos[q0] = pos0;
    }
  }
}


// build_tree with the candidate set in registers: candidate c sits in lane c % 32, register slot
// c / 32 (SLOTS slots per lane, so budget + 1 <= 32 * SLOTS). Each key carries its whole payload:
// hi = the ordered pattern of neg, lo = depth << 46 | (parent + 1) << 14 | rank << 6 | j << 1 | z
// (j = position in the parent's child order, z = neg is -0.0). Candidates never share (depth,
// parent, rank), so the bits below rank never decide an order, and (hi, lo) compares exactly like
// the reference's (neg, depth, parent, rank). A pop is a scan of the lane's slots, a warp arg-min
// (one 32-bit reduction over hi's upper word when a single lane holds its minimum, else over all of hi
// and, on a tie, over lo), and an in-register replacement: no shared-memory round trip sits on the pop
// chain except the neg of the popped node's parent. The output arrays are written after the last pop.
__device__ __forceinline__ double key_to_neg(uint64_t hi, uint64_t lo) {
  if (lo & 1ull) return -0.0;
  const uint64_t u = (hi >> 63) ? (hi & 0x7fffffffffffffffull) : ~hi;
  return __longlong_as_double((long long)u);
}
__device__ __forceinline__ uint64_t cand_lo(int d, int par, int r, int j, double neg) {
  const bool z = (uint64_t)__double_as_longlong(neg) == 0x8000000000000000ull;
  return ((uint64_t)d << 46) | ((uint64_t)(uint32_t)(par + 1) << 14) | ((uint64_t)r << 6) | ((uint64_t)j << 1) |
         (z ? 1ull : 0ull);
}
// warp-wide minimum of a 64-bit value (every lane gets it)
__device__ __forceinline__ uint64_t warp_min64(uint64_t x, bool& mine) {
  const uint32_t m0 = __reduce_min_sync(0xffffffffu, (uint32_t)(x >> 32));
  mine = (uint32_t)(x >> 32) == m0;
  const uint32_t m1 = __reduce_min_sync(0xffffffffu, mine ? (uint32_t)x : 0xffffffffu);
  mine = mine && (uint32_t)x == m1;
  return ((uint64_t)m0 << 32) | m1;
}

// candidate index c := (h, l): lane c % 32, slot c / 32 (compile-time slot indices only)
template <int SLOTS>
__device__ __forceinline__ void cand_put(uint64_t (&ch)[SLOTS], uint64_t (&cl)[SLOTS], int lane, int c, uint64_t h,
                                         uint64_t l) {
  const bool here = lane == (c & 31);
  const int cs = c >> 5;
#pragma unroll
  for (int s = 0; s < SLOTS; ++s) {
    const bool w = here && s == cs;
    ch[s] = w ? h : ch[s];
    cl[s] = w ? l : cl[s];
  }
}

template <int SLOTS>
__global__ void __launch_bounds__(32) build_tree_reg_kernel(const TreeArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  const int k = a.k, L = a.L;
  double* n_neg = reinterpret_cast<double*>(smem_raw);                                  // neg of popped nodes
  double* s_lp = n_neg + a.max_budget;
  int32_t* s_tok = reinterpret_cast<int32_t*>(s_lp + (size_t)L * k);                  // token of each (row, rank)
  int32_t* n_info = s_tok + (size_t)L * k;                     // popped node: (parent + 1) | depth << 16 | rank << 24
  unsigned char* order = reinterpret_cast<unsigned char*>(n_info + a.max_budget);    // [(1 + max_budget)][k], row 0 = root

  int budget = a.budget[b];
  if (budget > a.max_budget || budget < 0) {
    if (lane == 0) { report(CAST_DEV_TREE_OVERFLOW); a.count[b] = 0; }
    return;
  }
  const double* lp_g = a.top_lp + (size_t)b * L * a.k_cols;
  const int64_t* idx_g = a.top_idx + (size_t)b * L * a.k_cols;
  bool sorted_rows = true;
  for (int e = lane; e < L * k; e += 32) {
    const double v = lp_g[(e / k) * a.k_cols + (e % k)];
    s_lp[e] = v;
    s_tok[e] = (int32_t)idx_g[(e / k) * a.k_cols + (e % k)];
    if (e % k != k - 1 && !(v >= lp_g[(e / k) * a.k_cols + (e % k) + 1])) sorted_rows = false;
  }
  sorted_rows = __all_sync(0xffffffffu, sorted_rows);
  __syncwarp();
  auto child_order = [&](int slot, bool root, double base, int d) {
    if (sorted_rows) return;
    uint64_t hi = ~0ull;
    if (lane < k) hi = ordered_key(root ? -s_lp[lane] : base - s_lp[d * k + lane]);
    int rank = 0;
    for (int r2 = 0; r2 < k; ++r2) {
      const uint64_t h2 = __shfl_sync(0xffffffffu, hi, r2);
      if (lane < k && (h2 < hi || (h2 == hi && r2 < lane))) ++rank;
    }
    if (lane < k) order[(size_t)slot * k + rank] = (unsigned char)lane;
    __syncwarp();
  };
  auto nth_child = [&](int slot, int j) -> int { return sorted_rows ? j : (int)order[(size_t)slot * k + j]; };

  uint64_t ch[SLOTS], cl[SLOTS];
#pragma unroll
  for (int s = 0; s < SLOTS; ++s) ch[s] = cl[s] = ~0ull;
  int ncand = 0;
  if (budget > 0 && k > 0 && L > 0) {
    child_order(0, true, 0.0, 0);
    const int r = nth_child(0, 0);
    const double neg = -s_lp[r];
    const uint64_t h0 = ordered_key(neg), l0 = cand_lo(1, -1, r, 0, neg);
    cand_put<SLOTS>(ch, cl, lane, 0, h0, l0);
    ncand = 1;
  }

  int n = 0;
  const int q0 = a.cu_q ? a.cu_q[b] : 0;
  const int pos0 = (a.cu_q && a.pack_pos) ? a.seq_len[b] : 0;
  bool pack_ok = true;
  if (a.cu_q && lane == 0) {
    pack_ok = q0 >= 0 && (long long)q0 + 1 + budget <= (long long)a.cu_q[b + 1];
    if (!pack_ok) report(CAST_DEV_BAD_LAYOUT);
  }
  pack_ok = __shfl_sync(0xffffffffu, pack_ok ? 1 : 0, 0) != 0;

  while (n < budget && ncand > 0) {
    // this lane's least candidate (empty slots hold all ones) and its slot, then the warp's
    uint64_t bh = ch[0], bl = cl[0];
    int bs = 0;
#pragma unroll
    for (int s = 1; s < SLOTS; ++s)
      if (ch[s] < bh || (ch[s] == bh && cl[s] < bl)) { bh = ch[s]; bl = cl[s]; bs = s; }
    // usually one lane alone holds the least upper word of hi: its candidate is the minimum
    const uint32_t top = (uint32_t)(bh >> 32);
    const unsigned first = __ballot_sync(0xffffffffu, top == __reduce_min_sync(0xffffffffu, top));
    uint64_t wh, wl;
    bool win;   // this lane holds the popped candidate, in slot bs (keys are unique)
    if (__popc(first) == 1) {
      const int src = __ffs(first) - 1;
      wh = __shfl_sync(0xffffffffu, bh, src);
      wl = __shfl_sync(0xffffffffu, bl, src);
      win = lane == src;
    } else {
      bool mine;
      wh = warp_min64(bh, mine);
      const unsigned tied = __ballot_sync(0xffffffffu, mine);
      if (__popc(tied) == 1) {
        wl = __shfl_sync(0xffffffffu, bl, __ffs(tied) - 1);
        win = mine;
      } else {
        bool m2;
        wl = warp_min64(mine ? bl : ~0ull, m2);
        win = mine && m2;
      }
    }
    const int d = (int)(wl >> 46);
    const int par = (int)(uint32_t)((wl >> 14) & 0xffffffffull) - 1;
    const int r = (int)((wl >> 6) & 0xff);
    const int j = (int)((wl >> 1) & 31);
    const double neg = key_to_neg(wh, wl);
    const int me = n;
    if (lane == 0) {   // the outputs are written after the loop, all lanes together
      n_neg[me] = neg;
      n_info[me] = (par + 1) | (d << 16) | (r << 24);
    }
    if (j + 1 < k) {
      // the popped candidate becomes its next sibling
      const int r2 = nth_child(par + 1, j + 1);
      const double sneg = (par < 0) ? -s_lp[r2] : n_neg[par] - s_lp[(size_t)(d - 1) * k + r2];
      const uint64_t nh = ordered_key(sneg), nl = cand_lo(d, par, r2, j + 1, sneg);
#pragma unroll
      for (int s = 0; s < SLOTS; ++s) {
        const bool w = win && s == bs;
        ch[s] = w ? nh : ch[s];
        cl[s] = w ? nl : cl[s];
      }
    } else {
      // no sibling left: the last candidate moves into the popped one's place
      const int last = ncand - 1;
      // (a shuffle per slot: a select over slots by a run-time index would put the slots in memory)
      uint64_t lh = ~0ull, ll = ~0ull;
#pragma unroll
      for (int s = 0; s < SLOTS; ++s) {
        if (s <= (ncand - 1) >> 5) {
          const uint64_t th = __shfl_sync(0xffffffffu, ch[s], last & 31);
          const uint64_t tl = __shfl_sync(0xffffffffu, cl[s], last & 31);
          lh = s == (last >> 5) ? th : lh;
          ll = s == (last >> 5) ? tl : ll;
        }
      }
      const bool last_here = lane == (last & 31);
#pragma unroll
      for (int s = 0; s < SLOTS; ++s) {
        const bool w = win && s == bs;                 // the popped candidate: takes the last one's key
        const bool e = last_here && s == (last >> 5);  // the last candidate's place: emptied
        ch[s] = e ? ~0ull : (w ? lh : ch[s]);
        cl[s] = e ? ~0ull : (w ? ll : cl[s]);
      }
      --ncand;
    }
    __syncwarp();   // n_neg[me] (lane 0) before any lane reads it
    if (d < L) {
      child_order(me + 1, false, neg, d);
      const int r2 = nth_child(me + 1, 0);
      const double cneg = neg - s_lp[(size_t)d * k + r2];
      const uint64_t hc = ordered_key(cneg), lc = cand_lo(d + 1, me, r2, 0, cneg);
      cand_put<SLOTS>(ch, cl, lane, ncand, hc, lc);
      ++ncand;
    }
    ++n;
  }
  __syncwarp();
  for (int me = lane; me < n; me += 32) {
    const int info = n_info[me];
    const int par = (info & 0xffff) - 1, d = (info >> 16) & 0xff, r = info >> 24;
    const int tok = s_tok[(size_t)(d - 1) * k + r];
    const size_t o = (size_t)b * a.max_budget + me;
    a.token[o] = tok;
    a.depth[o] = d;
    a.parent[o] = par;
    a.score[o] = -n_neg[me];
    if (a.cu_q && pack_ok) {
      if (a.pack_parent) a.pack_parent[q0 + 1 + me] = par + 1;
      if (a.pack_token) a.pack_token[q0 + 1 + me] = tok;
      if (a.pack_pos) a.pack_pos[q0 + 1 + me] = pos0 + d;
    }
  }
  if (lane == 0) {
    a.count[b] = n;
    if (a.cu_q && pack_ok) {
      if (a.pack_parent) a.pack_parent[q0] = -1;
      if (a.pack_token) a.pack_token[q0] = a.root_token[b];
      if (a.pack_pos) a.pack_pos[q0] = pos0;
    }
  }
}

__host__ __device__ inline size_t tree_reg_smem_bytes(int max_budget, int L, int k) {
  return (size_t)max_budget * (sizeof(double) + sizeof(int32_t)) +  // node neg and (parent, depth, rank)
         ((size_t)max_budget + 1) * k * sizeof(unsigned char) +      // child order per node (+root)
         (size_t)L * k * sizeof(double) +                            // lp rows
         (size_t)L * k * sizeof(int32_t) + 64;                       // token rows
}
}  // namespace cast
