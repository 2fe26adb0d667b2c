// Split-KV CUDA-core tree attention (any dtype, head dim 64/128, any pack size).
//
// This is the exact-fp32 path: q/k/v are widened to fp32 in shared memory and
// every product is an fp32 FMA, so fp32 inputs meet a 1e-4 bound against the
// fp32 oracle. It also serves fp16 inputs and any shape the tensor-core kernel
// does not take.
//
// Work unit (one CTA): sequence b, KV head h, a 64-row tile of the G*P_b query
// rows of that head group (row r = token r / G, query head h*G + r % G), and a
// chunk of the key range [0, S_b + P_b). Keys < S_b are the prefix and always
// visible; key S_b + j is pack token j, visible iff bit j of the row token's
// ancestor bitset is set (cast_trees/tree_attn.py:50-87). The bitsets of the
// tile's tokens live in shared memory, built from `parent` or copied from the
// caller's words. With one key chunk the CTA writes the output; with several
// it writes fp32 partials (unnormalised O, running max m in log2 units, sum l)
// that attn_combine_kernel merges.
#pragma once

#include "common.cuh"

namespace cast {

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t sq_m, sq_h, sk_m, sk_h, sv_m, sv_h, so_m, so_h;
  const int32_t* cu_q;
  const int32_t* cu_kv;
  const int32_t* prefix_len;
  const int32_t* pack_len;
  const int64_t* anc_words;
  int anc_wpr;
  const int32_t* parent;
  int B, total_q, total_kv, H_q, H_kv, G, D;
  float scale_log2;
  int max_pack, max_kv;
  int n_split, chunk, m_tiles, W;
  float* ws_o;   // [n_split, total_q, H_q, D]
  float* ws_ml;  // [n_split, total_q, H_q, 2]
  // Store mode (tensor-core kernel only): the prefix of sequence b is rows
  // [0, S_b) of a per-request store [store_batch, H_kv, store_rows, D], the
  // pack K/V rows [cu_q[b], cu_q[b] + P_b) of [total_q, H_kv, D] tensors; the
  // key tiles are ceil(S_b/128) prefix tiles then ceil(P_b/128) pack tiles.
  int store_mode;
  int store_rows, store_batch;
  // Limit of the tensor-core kernel's pipeline waits (ns). The waits that let
  // in-flight copies and MMAs drain before a CTA exits keep the full limit.
  uint64_t wait_ns;
  // fp32 split path: flags[0..2] != 0 when the bf16 low parts of q / k / v hold any non-zero value
  const int* split_flags;
  // Single-CTA tensor-core kernel: 1 when the largest head group ends in a one-tile block (G * max_pack
  // mod 256 in (0, 128]): the launch then runs every other row block first and the last blocks after.
  int tail_last;
  // Row-block selection when one call runs on both tensor-core kernels: the CTA-pair kernel takes
  // only full 256-row blocks (pair_full_only), the single-CTA kernel only each sequence's partial
  // last block (tail_only; its grid then holds one row block per (sequence, KV head, key chunk)).
  int pair_full_only, tail_only;
};

// Key tiles of one sequence: the whole range for the regular layout, the
// prefix tiles plus the pack tiles for the store layout.
__device__ __forceinline__ int seq_key_tiles(const AttnParams& p, int S, int P, int bn) {
  return p.store_mode ? (S + bn - 1) / bn + (P + bn - 1) / bn : (S + P + bn - 1) / bn;
}

namespace simt {
constexpr int BM = 64, BN = 64, NT = 256;
template <int D> __host__ __device__ constexpr int qk_stride() { return D + 4; }
template <int D> __host__ __device__ constexpr size_t smem_bytes(int W) {
  return sizeof(float) * (2 * BM * qk_stride<D>() + BN * D + BM * (BN + 1)) +
         sizeof(uint64_t) * (BM + 1) * W;
}
}  // namespace simt

// Largest bitset width (64-bit words per token) for which the tensor-core kernels stage the
// pack's parents in shared memory before building the bitsets (W * 64 ints).
constexpr int kStageParentMaxW = 8;
__host__ __device__ inline size_t parent_stage_bytes(int W) {
  return W <= kStageParentMaxW ? (size_t)W * 64 * sizeof(int) : 0;
}

// Builds the ancestor bitsets of pack tokens [i_lo, i_lo + nt) into s_anc
// ([nt][W] words). One thread per token; each walks its own ancestor chain
// (parent[j] < j, so the walk ends within j + 1 steps), reading the parents
// from `par` (the pack's parents staged in shared memory) when given, else
// from global memory. Bits are gathered one word at a time (the chain only
// descends) and each word is stored once.
__device__ __forceinline__ void build_tile_bitsets(const AttnParams& p, const SeqMeta& m, int i_lo,
                                                   int nt, uint64_t* s_anc, const int* par = nullptr) {
  const int W = p.W;
  const int wn = (m.P + 63) >> 6;
  for (int li = threadIdx.x; li < nt; li += blockDim.x) {
    uint64_t* row = s_anc + (size_t)li * W;
    for (int w = 0; w < W; ++w) row[w] = 0ull;
    const int i = i_lo + li;
    if (p.anc_words != nullptr) {
      const int64_t* src = p.anc_words + (int64_t)(m.q0 + i) * p.anc_wpr;
      const int wc = min(wn, p.anc_wpr);
      for (int w = 0; w < wc; ++w) row[w] = (uint64_t)src[w];
    } else {
      int j = i;
      int guard = 0;
      int cw = j >> 6;
      uint64_t acc = 0ull;
      while (j >= 0 && guard <= i) {
        if ((j >> 6) != cw) {
          row[cw] = acc;
          acc = 0ull;
          cw = j >> 6;
        }
        acc |= 1ull << (j & 63);
        const int pj = par != nullptr ? par[j] : p.parent[m.q0 + j];
        if (pj >= j || pj < -1 || (j == 0 && pj != -1)) {
          report(CAST_DEV_BAD_PARENT);
          break;
        }
        j = pj;
        ++guard;
      }
      row[cw] = acc;
    }
  }
}

// Visibility of keys [nb, nb + 32) for one query row, bit i for key nb + i: prefix keys (< S) are
// visible, pack key S + j iff bit j of the row token's bitset `anc` (W words), and keys at or past
// `klim` are not. A shifted window of the bitset words, so a masked tile costs a few instructions
// per 32 keys.
__device__ __forceinline__ uint32_t visible32(const uint64_t* anc, int W, int nb, int S, int klim) {
  uint32_t bits;
  const int rel = nb - S;   // pack index of key nb (negative inside the prefix)
  if (rel >= 0) {
    const int w = rel >> 6, sh = rel & 63;
    const uint64_t lo = w < W ? anc[w] : 0ull;
    const uint64_t hi = (sh != 0 && w + 1 < W) ? anc[w + 1] : 0ull;
    bits = (uint32_t)(sh != 0 ? (lo >> sh) | (hi << (64 - sh)) : lo);
  } else if (rel > -32) {
    bits = ((uint32_t)anc[0] << -rel) | ((1u << -rel) - 1u);   // -rel prefix keys, then pack bits 0..
  } else {
    bits = ~0u;
  }
  const int lim = klim - nb;
  return lim >= 32 ? bits : (lim <= 0 ? 0u : bits & ((1u << lim) - 1u));
}

template <typename T, int D>
__global__ void __launch_bounds__(simt::NT)
attn_simt_kernel(const AttnParams p) {
  using namespace simt;
  constexpr int QS = qk_stride<D>();
  constexpr int CPT = D / 16;  // output columns per thread (4 or 8)
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sQ = reinterpret_cast<float*>(smem_raw);
  float* sK = sQ + BM * QS;
  float* sV = sK + BN * QS;
  float* sP = sV + BN * D;
  uint64_t* sAnc = reinterpret_cast<uint64_t*>(sP + BM * (BN + 1));

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int b = blockIdx.y / p.H_kv, h = blockIdx.y % p.H_kv;
  const SeqMeta m = load_seq(p.cu_q, p.cu_kv, p.prefix_len, p.pack_len, b, p.total_q, p.total_kv,
                             p.max_pack, p.max_kv);
  if (!m.ok) {
    if (tid == 0 && blockIdx.x == 0 && blockIdx.z == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int G = p.G;
  const int rows = G * m.P;
  const int r0 = blockIdx.x * BM;
  if (r0 >= rows) return;
  const int nkeys = m.S + m.P;
  const int k_begin = blockIdx.z * p.chunk;
  if (k_begin >= nkeys) return;
  const int k_end = min(nkeys, k_begin + p.chunk);

  const T* Q = static_cast<const T*>(p.q);
  const T* K = static_cast<const T*>(p.k);
  const T* V = static_cast<const T*>(p.v);

  // Q tile, pre-scaled into log2 units; rows past the pack are zero.
  for (int e = tid; e < BM * (D / 4); e += NT) {
    const int rr = e / (D / 4), c4 = (e % (D / 4)) * 4;
    const int r = r0 + rr;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) {
      const int i = r / G, g = r % G;
      x = load4<T>(Q + (int64_t)(m.q0 + i) * p.sq_m + (int64_t)(h * G + g) * p.sq_h + c4);
      x.x *= p.scale_log2; x.y *= p.scale_log2; x.z *= p.scale_log2; x.w *= p.scale_log2;
    }
    *reinterpret_cast<float4*>(sQ + rr * QS + c4) = x;
  }
  const int i_lo = r0 / G;
  const int i_hi = min(m.P - 1, (r0 + BM - 1) / G);
  if (k_end > m.S) build_tile_bitsets(p, m, i_lo, i_hi - i_lo + 1, sAnc);

  float o[4][CPT];
  float mrow[4], lrow[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    mrow[a] = -INFINITY;
    lrow[a] = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) o[a][c] = 0.f;
  }

  for (int kb = k_begin; kb < k_end; kb += BN) {
    __syncthreads();  // previous tile's sK/sV/sP reads are done (and sQ/sAnc writes on entry)
    for (int e = tid; e < BN * (D / 4); e += NT) {
      const int rr = e / (D / 4), c4 = (e % (D / 4)) * 4;
      const int n = kb + rr;
      float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
      if (n < k_end) {
        const int64_t row = m.kv0 + n;
        kx = load4<T>(K + row * p.sk_m + (int64_t)h * p.sk_h + c4);
        vx = load4<T>(V + row * p.sv_m + (int64_t)h * p.sv_h + c4);
      }
      *reinterpret_cast<float4*>(sK + rr * QS + c4) = kx;
      *reinterpret_cast<float4*>(sV + rr * D + c4) = vx;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[a][c] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d += 4) {
      float4 qa[4], kc[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(sQ + (ty + 16 * a) * QS + d);
#pragma unroll
      for (int c = 0; c < 4; ++c) kc[c] = *reinterpret_cast<const float4*>(sK + (tx + 16 * c) * QS + d);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[a][c] = fmaf(qa[a].x, kc[c].x, s[a][c]);
          s[a][c] = fmaf(qa[a].y, kc[c].y, s[a][c]);
          s[a][c] = fmaf(qa[a].z, kc[c].z, s[a][c]);
          s[a][c] = fmaf(qa[a].w, kc[c].w, s[a][c]);
        }
    }

    // visibility: prefix keys always, pack keys by ancestor bit, nothing past k_end
    const bool full = (kb + BN <= m.S) && (kb + BN <= k_end);
    if (!full) {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int r = r0 + ty + 16 * a;
        const int li = min(r / G, m.P - 1) - i_lo;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int n = kb + tx + 16 * c;
          bool vis = n < k_end;
          if (vis && n >= m.S) {
            const int j = n - m.S;
            vis = (sAnc[(size_t)li * p.W + (j >> 6)] >> (j & 63)) & 1ull;
          }
          if (!vis) s[a][c] = -INFINITY;
        }
      }
    }

#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float mx = fmaxf(fmaxf(s[a][0], s[a][1]), fmaxf(s[a][2], s[a][3]));
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off, 16));
      const float m_new = fmaxf(mrow[a], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(mrow[a] - m_use);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float pv = exp2f(s[a][c] - m_use);
        rs += pv;
        sP[(ty + 16 * a) * (BN + 1) + tx + 16 * c] = pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off, 16);
      lrow[a] = lrow[a] * alpha + rs;
      mrow[a] = m_new;
#pragma unroll
      for (int c = 0; c < CPT; ++c) o[a][c] *= alpha;
    }
    __syncthreads();

#pragma unroll 4
    for (int kk = 0; kk < BN; ++kk) {
      float4 v0 = *reinterpret_cast<const float4*>(sV + kk * D + tx * 4);
      float4 v1 = v0;
      if constexpr (CPT == 8) v1 = *reinterpret_cast<const float4*>(sV + kk * D + 64 + tx * 4);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float pa = sP[(ty + 16 * a) * (BN + 1) + kk];
        o[a][0] = fmaf(pa, v0.x, o[a][0]);
        o[a][1] = fmaf(pa, v0.y, o[a][1]);
        o[a][2] = fmaf(pa, v0.z, o[a][2]);
        o[a][3] = fmaf(pa, v0.w, o[a][3]);
        if constexpr (CPT == 8) {
          o[a][4] = fmaf(pa, v1.x, o[a][4]);
          o[a][5] = fmaf(pa, v1.y, o[a][5]);
          o[a][6] = fmaf(pa, v1.z, o[a][6]);
          o[a][7] = fmaf(pa, v1.w, o[a][7]);
        }
      }
    }
  }

  // epilogue: each of the 16 threads of a row holds CPT of its D columns
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int r = r0 + ty + 16 * a;
    if (r >= rows) continue;
    const int i = r / G, hq = h * G + r % G;
    const int64_t t = m.q0 + i;
    if (p.n_split == 1) {
      const float inv = lrow[a] > 0.f ? 1.f / lrow[a] : 0.f;
      T* O = static_cast<T*>(p.out) + t * p.so_m + (int64_t)hq * p.so_h;
      store4<T>(O + tx * 4, make_float4(o[a][0] * inv, o[a][1] * inv, o[a][2] * inv, o[a][3] * inv));
      if constexpr (CPT == 8)
        store4<T>(O + 64 + tx * 4, make_float4(o[a][4] * inv, o[a][5] * inv, o[a][6] * inv, o[a][7] * inv));
    } else {
      const int64_t slot = ((int64_t)blockIdx.z * p.total_q + t) * p.H_q + hq;
      float* O = p.ws_o + slot * D;
      *reinterpret_cast<float4*>(O + tx * 4) = make_float4(o[a][0], o[a][1], o[a][2], o[a][3]);
      if constexpr (CPT == 8)
        *reinterpret_cast<float4*>(O + 64 + tx * 4) = make_float4(o[a][4], o[a][5], o[a][6], o[a][7]);
      if (tx == 0) {
        p.ws_ml[slot * 2 + 0] = mrow[a];
        p.ws_ml[slot * 2 + 1] = lrow[a];
      }
    }
  }
}

// Merges the key-chunk partials of one (query row, query head) per warp.
template <typename T>
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.total_q * p.H_q) return;
  const int t = warp / p.H_q, hq = warp % p.H_q;
  // sequence of row t: last b with cu_q[b] <= t
  int lo = 0, hi = p.B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  SeqMeta m;
  if (p.store_mode) {
    m.q0 = p.cu_q[b]; m.kv0 = 0; m.S = p.prefix_len[b]; m.P = p.pack_len[b];
    m.ok = m.q0 >= 0 && m.S >= 0 && m.P >= 0 && m.P <= p.max_pack && m.S <= p.store_rows &&
           (long long)m.q0 + m.P <= p.total_q;
  } else {
    m = load_seq(p.cu_q, p.cu_kv, p.prefix_len, p.pack_len, b, p.total_q, p.total_kv, p.max_pack, p.max_kv);
  }
  if (!m.ok || t < m.q0 || t >= m.q0 + m.P) return;
  const int tiles_per_chunk = p.chunk / 128;
  const int nsplit = p.store_mode ? min(p.n_split, (seq_key_tiles(p, m.S, m.P, 128) + tiles_per_chunk - 1) / tiles_per_chunk)
                                  : min(p.n_split, (m.S + m.P + p.chunk - 1) / p.chunk);
  float M = -INFINITY;
  for (int z = 0; z < nsplit; ++z)
    M = fmaxf(M, p.ws_ml[(((int64_t)z * p.total_q + t) * p.H_q + hq) * 2]);
  const float m_use = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  const int nv = p.D / 128 + (p.D % 128 ? 1 : 0);  // float4 groups per lane: D/128 (1 for D=64 uses half the lanes)
  for (int z = 0; z < nsplit; ++z) {
    const int64_t slot = ((int64_t)z * p.total_q + t) * p.H_q + hq;
    const float w = exp2f(p.ws_ml[slot * 2] - m_use);
    L += w * p.ws_ml[slot * 2 + 1];
    const float* O = p.ws_o + slot * p.D;
    for (int g = 0; g < nv; ++g) {
      const int c = (g * 32 + lane) * 4;
      if (c < p.D) {
        const float4 x = *reinterpret_cast<const float4*>(O + c);
        acc[g].x += w * x.x; acc[g].y += w * x.y; acc[g].z += w * x.z; acc[g].w += w * x.w;
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* out = static_cast<T*>(p.out) + (int64_t)t * p.so_m + (int64_t)hq * p.so_h;
  for (int g = 0; g < nv; ++g) {
    const int c = (g * 32 + lane) * 4;
    if (c < p.D)
      store4<T>(out + c, make_float4(acc[g].x * inv, acc[g].y * inv, acc[g].z * inv, acc[g].w * inv));
  }
}

}  // namespace cast
