// Tensor-core (tcgen05 / TMEM / TMA) ragged tree attention for 16-bit inputs, D = 128.
//
// Work unit (one CTA, one per SM): sequence b, KV head h, up to two 128-row
// query tiles of the G*P_b rows of that head group (row r = pack token r / G,
// query head h*G + r % G; both tiles share every K/V tile), and a chunk of the
// key range [0, S_b + P_b) (the whole range unless the launch splits keys).
//
// Roles (12 warps):
//   warp 0      TMEM allocation; one lane issues the TMA loads of the Q tiles (once)
//               and of the 128-key K tiles into a 2-stage ring.
//   warp 2      one lane issues the TMA loads of the V tiles into their 2-stage ring.
//   warp 1      lane 0 issues every tcgen05.mma:
//                 S_q  = Q_q K_j^T    (A, B in shared memory, K-major)
//                 O_q += P_q V_j      (A = P in tensor memory, B = V MN-major)
//               in the order QK0_j, PV1_{j-1}, QK1_j, PV0_j, so that the
//               softmax of one tile overlaps the tensor core on the other.
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: thread t owns
//               TMEM lane t (query row t). Per key tile: row max from S, lazy
//               rescale of O (only when the max grew by more than 2^8), then
//               P = exp2(S*c - m) rounded to 16 bits and stored into the first
//               64 columns of S (tcgen05.st), which the PV MMA reads.
// A CTA with one query tile and two or more key tiles runs "dual": its even key
// tiles go through S_0/O_0 (warps 4-7) and its odd ones through S_1/O_1 (warps
// 8-11), both on query tile 0, and the epilogue merges the two partial softmaxes.
// Tensor memory (512 columns): S_0, S_1 (128 fp32 columns each), O_0, O_1.
// Visibility: keys < S_b always; pack key S_b + j iff bit j of the row token's
// ancestor bitset (shared memory; built from `parent` or copied); keys past
// the chunk end are masked (TMA fills rows past the tensor with zeros and the
// next sequence's rows are masked out). Every mbarrier wait is bounded; on
// expiry the CTA records CAST_DEV_TIMEOUT, lets in-flight copies and MMAs
// drain, frees its tensor memory and returns.
#pragma once

#include "attn_simt.cuh"
#include "tc_common.cuh"

namespace cast {
namespace tca {

constexpr int BM = 128;           // rows per query tile
constexpr int QT = 2;             // query tiles per CTA
constexpr int BN = 128;           // keys per K/V tile
constexpr int D = 128;
constexpr int NST = 2;            // K/V ring stages
constexpr int NT = 384;           // threads
constexpr int TILE_BYTES = BN * D * 2;        // 32 KB: one 128 x 128 16-bit tile
constexpr int HALF_BYTES = TILE_BYTES / 2;    // 16 KB: 64-column half (one 128B-swizzle panel)
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = SMEM_Q + QT * TILE_BYTES;
constexpr int SMEM_V = SMEM_K + NST * TILE_BYTES;
constexpr int SMEM_ANC = SMEM_V + NST * TILE_BYTES;   // 196608
constexpr float kRescaleLog2 = 8.0f;          // lazy O rescale threshold (factor 256)
// Registers: launched at 168 per thread (384 x 168 = 64512, the whole file);
// warpgroup 0 (TMA, MMA, two idle warps) gives back to 104, the two softmax
// warpgroups take 200: 128 x 104 + 256 x 200 = 64512.
constexpr int kRegsLow = 104, kRegsHigh = 200;
// Largest batch whose sequences the CTAs rank by length (longest first); larger
// batches run in sequence order. Every CTA ranks the whole batch (O(B^2 / threads)):
// at 512 sequences that took ~5 us per CTA and the ranked order was slower overall
// than sequence order (configuration 5, one GPU: 3.06 against 3.25 ms at N = 16,
// 12.9-13.3 against 13.6-13.8 ms at N = 128). The keys take 4 bytes each of the K ring.
constexpr int kMaxRankedSeqs = 128;

__host__ __device__ inline int anc_tokens(int G) { return QT * BM / G + 2; }
__host__ __device__ inline size_t smem_bytes(int G, int W) {
  return 1024 + SMEM_ANC + (size_t)anc_tokens(G) * W * sizeof(uint64_t) + parent_stage_bytes(W);
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[NST], k_empty[NST], v_full[NST], v_empty[NST];
  uint64_t s_full[QT], p_full[QT];
  uint64_t o_full;
  uint64_t comb;   // dual mode: the odd-tile half's (m, l) are in shared memory
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// The sequence of the given length rank (S + P descending, lower index first), computed by the
// whole CTA from prefix_len / pack_len with `keys` (p.B ints of shared memory not yet used by any
// TMA copy) as scratch; batches above kMaxRankedSeqs keep sequence order. Every CTA computes the
// same permutation, so the launch covers each sequence exactly once.
__device__ __forceinline__ int ranked_sequence(const AttnParams& p, int rank, int* keys) {
  __shared__ int seq_of_rank;
  const int tid = threadIdx.x, nt = blockDim.x;
  if (p.B <= kMaxRankedSeqs) {
    for (int i = tid; i < p.B; i += nt) {
      const long long k = (long long)p.prefix_len[i] + p.pack_len[i];
      keys[i] = (int)max(-1LL, min(k, 0x7fffffffLL));
    }
    __syncthreads();
    for (int i = tid; i < p.B; i += nt) {
      const int ki = keys[i];
      int r = 0;
      for (int j = 0; j < p.B; ++j) {
        const int kj = keys[j];
        r += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
      }
      if (r == rank) seq_of_rank = i;
    }
  } else if (tid == 0) {
    seq_of_rank = rank;
  }
  tc::fence_proxy_async_smem();   // the keys' generic-proxy writes are ordered before later TMA copies there
  __syncthreads();
  return seq_of_rank;
}

// STORE = false: K/V are [total_kv, H_kv, D] (tmK, tmV; tmKp/tmVp unused).
// STORE = true: tmK/tmV map the per-request prefix stores [B, H_kv, S_max, D]
// (4-D), tmKp/tmVp the pack K/V [total_q, H_kv, D].
template <bool BF16, bool STORE>
__global__ void __launch_bounds__(NT, 1)
attn_tc_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKp,
               const __grid_constant__ CUtensorMap tmVp) {
  using namespace tc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* sAnc = reinterpret_cast<uint64_t*>(smem + SMEM_ANC);
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  __shared__ float comb_m[BM], comb_l[BM];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Work unit of this CTA, longest sequences first. CTAs start in launch order (linear block
  // index), so the launch-order index L is decoded as (rank of the sequence, KV head, key chunk,
  // row block), row blocks fastest (the blocks of one head share its K/V tiles through L2), and
  // the sequence of that rank is found by ranking every sequence by S + P (descending, lower
  // index first): the longest units start first and the last wave holds the shortest ones.
  // When the largest head group ends in a one-tile block (tail_last), that last row block of every
  // (sequence, KV head, key chunk) goes after all the others: it costs about half a two-tile block,
  // and with it interleaved the last wave held long two-tile units.
  const int L = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nb_first = (p.tail_last && gridDim.x > 1) ? gridDim.x - 1 : gridDim.x;
  const int n_first = nb_first * gridDim.y * gridDim.z;
  const bool late = L >= n_first;
  const int Lr = late ? L - n_first : L;
  const int nb = late ? 1 : nb_first;
  int mblk = late ? gridDim.x - 1 : Lr % nb;
  int rest = Lr / nb;
  const int split = rest % gridDim.z;
  rest /= gridDim.z;
  const int h = rest % p.H_kv;
  const int rank = rest / p.H_kv;
  const int b = ranked_sequence(p, rank, reinterpret_cast<int*>(smem + SMEM_K));  // K ring as scratch
  SeqMeta m;
  if constexpr (STORE) {
    m.q0 = p.cu_q[b]; m.kv0 = 0; m.S = p.prefix_len[b]; m.P = p.pack_len[b];
    m.ok = m.q0 >= 0 && m.S >= 0 && m.P >= 0 && m.P <= p.max_pack && m.S <= p.store_rows && b < p.store_batch &&
           (long long)m.q0 + m.P <= p.total_q;
  } else {
    m = load_seq(p.cu_q, p.cu_kv, p.prefix_len, p.pack_len, b, p.total_q, p.total_kv, p.max_pack, p.max_kv);
  }
  if (!m.ok) {
    if (tid == 0 && mblk == 0 && split == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int G = p.G;
  const int rows = G * m.P;
  if (p.tail_only) {   // only the sequence's partial last 256-row block (the CTA-pair launch runs the rest)
    if (rows % (QT * BM) == 0) return;
    mblk = rows / (QT * BM);
  }
  const int r_base = mblk * (QT * BM);
  if (r_base >= rows) return;
  const int n_qt = (rows - r_base > BM) ? 2 : 1;
  const int nkeys = m.S + m.P;
  // Key tiles of this CTA. Regular layout: keys [k_begin, k_end) of concat(prefix, pack),
  // tile j at key k_begin + 128 j. Store layout: tiles [t_begin, t_begin + n_kt) of the
  // list (prefix tiles, then pack tiles).
  int k_begin, k_end, t_begin = 0, nt_pre = 0, n_kt;
  if constexpr (STORE) {
    nt_pre = (m.S + BN - 1) / BN;
    const int nt_all = nt_pre + (m.P + BN - 1) / BN;
    const int ct = p.chunk / BN;
    t_begin = split * ct;
    if (t_begin >= nt_all) return;
    n_kt = min(nt_all, t_begin + ct) - t_begin;
    k_begin = 0;
    k_end = nkeys;
  } else {
    k_begin = split * p.chunk;
    if (k_begin >= nkeys) return;
    k_end = min(nkeys, k_begin + p.chunk);
    n_kt = (k_end - k_begin + BN - 1) / BN;
  }
  // Tile j: its first key (position in concat(prefix, pack)) and the end of the visible range.
  auto tile_keys = [&](int j, int& n0, int& klim) {
    if constexpr (STORE) {
      const int t = t_begin + j;
      if (t < nt_pre) { n0 = t * BN; klim = m.S; }
      else { n0 = m.S + (t - nt_pre) * BN; klim = nkeys; }
    } else {
      n0 = k_begin + j * BN;
      klim = k_end;
    }
  };
  const bool has_pack_tile = STORE ? (t_begin + n_kt > nt_pre) : (k_end > m.S);
  // A CTA with a single query tile runs it as two interleaved key streams (even key tiles on
  // S_0/O_0, odd ones on S_1/O_1, each with its own softmax warpgroup) and merges the two
  // partial softmaxes at the end: the same overlap as two query tiles, on half the key tiles each.
  const bool dual = n_qt == 1 && n_kt >= 2;
  volatile int* abort_flag = &abort_sh;

  if (tid == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(smem_u32(&bars.k_full[s]), 1);
      mbar_init(smem_u32(&bars.k_empty[s]), 1);
      mbar_init(smem_u32(&bars.v_full[s]), 1);
      mbar_init(smem_u32(&bars.v_empty[s]), 1);
    }
    for (int q = 0; q < QT; ++q) {
      mbar_init(smem_u32(&bars.s_full[q]), 1);
      mbar_init(smem_u32(&bars.p_full[q]), BM / 32);   // one arrival per softmax warp
    }
    mbar_init(smem_u32(&bars.o_full), 1);
    mbar_init(smem_u32(&bars.comb), BM);
    abort_sh = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 0) tmem_alloc(smem_u32(&tmem_base_sh), 512);
  const int i_lo = r_base / G;
  const int i_hi = min(m.P - 1, (r_base + QT * BM - 1) / G);
  // the pack's parents up to the last token of the block, staged for the bitset walks
  int* sPar = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(sAnc) + (size_t)anc_tokens(G) * p.W * sizeof(uint64_t));
  const bool stage = has_pack_tile && p.anc_words == nullptr && p.W <= kStageParentMaxW;
  if (stage)
    for (int j = tid; j <= i_hi; j += NT) sPar[j] = p.parent[m.q0 + j];
  __syncthreads();   // barriers initialised, parents staged

  // TMA producers: warp 0 loads the Q tiles and the K ring, warp 2 the V ring (a K slot frees up
  // after the second QK of its tile, a V slot only after the second PV, so one loop over both would
  // hold every K copy back behind the previous V slot).
  const bool is_k = warp == 0;
  const uint32_t qf = smem_u32(&bars.q_full);
  uint64_t* full = is_k ? bars.k_full : bars.v_full;
  uint64_t* empty = is_k ? bars.k_empty : bars.v_empty;
  const uint32_t ring = smem_u32(smem + (is_k ? SMEM_K : SMEM_V));
  const CUtensorMap* m_reg = is_k ? &tmK : &tmV;
  const CUtensorMap* m_pack = is_k ? &tmKp : &tmVp;
  // one 128-key tile (two 64-column halves) into ring slot j % NST
  auto issue_tile = [&](int j) {
    if (elect_one()) {
      const uint32_t dst = ring + (j % NST) * TILE_BYTES, bar = smem_u32(&full[j % NST]);
      mbar_expect_tx(bar, TILE_BYTES);
      for (int hf = 0; hf < 2; ++hf) {
        if constexpr (STORE) {
          const int t = t_begin + j;
          if (t < nt_pre) tma_load_4d(dst + hf * HALF_BYTES, m_reg, hf * 64, t * BN, h, b, bar);
          else tma_load_3d(dst + hf * HALF_BYTES, m_pack, hf * 64, h, m.q0 + (t - nt_pre) * BN, bar);
        } else {
          tma_load_3d(dst + hf * HALF_BYTES, m_reg, hf * 64, h, m.kv0 + k_begin + j * BN, bar);
        }
      }
    }
    __syncwarp();
  };
  // The Q tiles and the first NST key tiles need no free slot: their copies go out before the
  // ancestor bitsets are built.
  const int n_early = min(NST, n_kt);
  if (warp == 0 || warp == 2) {
    if (is_k && elect_one()) {
      mbar_expect_tx(qf, n_qt * TILE_BYTES);
      for (int q = 0; q < n_qt; ++q) {
        const int tok = m.q0 + (r_base + q * BM) / G;
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem_u32(smem + SMEM_Q + q * TILE_BYTES + hf * HALF_BYTES), &tmQ, hf * 64, h * G, tok, qf);
      }
    }
    __syncwarp();
    for (int j = 0; j < n_early; ++j) issue_tile(j);
  }
  if (has_pack_tile) build_tile_bitsets(p, m, i_lo, i_hi - i_lo + 1, sAnc, stage ? sPar : nullptr);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base_sh;
  if (warp < 4) {
  regs_dec<kRegsLow>();
  // Warps 0 and 1 walk their schedules converged, so warp-uniform values (loop
  // counters, shared-memory addresses, descriptors) stay in uniform registers;
  // one elected lane issues each TMA copy / MMA / commit.
  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ TMA producers (continued)
    int issued = n_early;   // tiles whose copies were issued
    for (int j = n_early; j < n_kt; ++j) {
      const int s = j % NST;
      const uint32_t use = (uint32_t)(j / NST);
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&empty[s]), (use - 1) & 1, abort_flag, p.wait_ns))) break;
      issue_tile(j);
      issued = j + 1;
    }
    // let the last copies land before the CTA can exit (immediate on the normal path); only
    // copies that were issued are waited for
    for (int j = max(0, issued - NST); j < issued; ++j)
      mbar_wait(smem_u32(&full[j % NST]), (uint32_t)(j / NST) & 1, nullptr);
    if (is_k) mbar_wait(qf, 0, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_f16(BF16, BM, BN, false, false);
    constexpr uint32_t idesc_pv = idesc_f16(BF16, BM, D, false, true);
    const uint32_t sQ = smem_u32(smem + SMEM_Q), sK = smem_u32(smem + SMEM_K), sV = smem_u32(smem + SMEM_V);
    // descriptors of every tile base; a K step adds its byte offset / 16 to the start-address field
    const uint64_t dQ0 = desc_kmajor(sQ), dQ1 = desc_kmajor(sQ + TILE_BYTES);
    const uint64_t dK0 = desc_kmajor(sK), dK1 = desc_kmajor(sK + TILE_BYTES);
    const uint64_t dV0 = desc_mnmajor(sV, HALF_BYTES), dV1 = desc_mnmajor(sV + TILE_BYTES, HALF_BYTES);
    // S_q = Q_qa K(slot s)^T
    auto qk_ = [&](int q, int qa, int s) {
      const uint64_t a = qa ? dQ1 : dQ0, b = s ? dK1 : dK0;
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t off = (uint64_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
          mma_ss(tmem + q * 128, a + off, b + off, idesc_qk, k > 0 ? 1u : 0u);
        }
      }
      __syncwarp();
    };
    // O_q (+)= P_q V(slot s); `first` starts the accumulator
    auto pv_ = [&](int q, int s, bool first) {
      const uint64_t b = s ? dV1 : dV0;
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          mma_ts(tmem + 256 + q * 128, tmem + q * 128 + k * 8, b + (uint64_t)((k * 2048) >> 4), idesc_pv,
                 (!first || k > 0) ? 1u : 0u);
      }
      __syncwarp();
    };
    auto qk = [&](int q, int j) { qk_(q, q, j % NST); };
    auto pv = [&](int q, int j) { pv_(q, j % NST, j == 0); };
    auto commit = [&](uint64_t& bar) {
      if (elect_one()) mma_commit(smem_u32(&bar));
      __syncwarp();
    };
    auto wait_all = [&](uint64_t& bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(&bar), parity, abort_flag, p.wait_ns));
    };
    // Store mode: the last prefix tile also holds store rows past the prefix; their scores
    // are masked, but 0 x (a non-finite stale value) would still poison P V, so those V rows
    // are zeroed (whole 128-byte rows: the swizzle only permutes inside a row).
    auto zero_tail = [&](int j, int s) {
      if constexpr (STORE) {
        int n0, klim;
        tile_keys(j, n0, klim);
        if (n0 < m.S && n0 + BN > m.S) {
          uint8_t* vt = smem + SMEM_V + s * TILE_BYTES;
          for (int e = lane; e < (n0 + BN - m.S) * 16; e += 32) {
            const int r = m.S - n0 + (e >> 4), c = e & 15;
            *reinterpret_cast<uint4*>(vt + (c >> 3) * HALF_BYTES + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
      }
    };
    bool ok = wait_all(bars.q_full, 0);
    if (dual) {
      // step i: QK of key tile 2i on S_0, PV of key tile 2i-1 (S_1), QK of key tile 2i+1 on S_1,
      // PV of key tile 2i (S_0); both QKs read query tile 0
      const int n_pairs = (n_kt + 1) / 2;
      for (int i = 0; ok && i < n_pairs; ++i) {
        const int j0 = 2 * i, j1 = 2 * i + 1;
        const int s0 = j0 % NST, s1 = j1 % NST;
        if (!(ok = wait_all(bars.k_full[s0], (uint32_t)(j0 / NST) & 1))) break;
        fence_after_sync();
        qk_(0, 0, s0);
        commit(bars.s_full[0]);
        commit(bars.k_empty[s0]);
        if (i > 0) {
          const int jp = j1 - 2, sp = jp % NST;
          if (!(ok = wait_all(bars.v_full[sp], (uint32_t)(jp / NST) & 1))) break;
          zero_tail(jp, sp);
          if (!(ok = wait_all(bars.p_full[1], (uint32_t)(i - 1) & 1))) break;
          fence_after_sync();
          pv_(1, sp, i == 1);
          commit(bars.v_empty[sp]);
        }
        if (j1 < n_kt) {
          if (!(ok = wait_all(bars.k_full[s1], (uint32_t)(j1 / NST) & 1))) break;
          fence_after_sync();
          qk_(1, 0, s1);
          commit(bars.s_full[1]);
          commit(bars.k_empty[s1]);
        }
        if (!(ok = wait_all(bars.v_full[s0], (uint32_t)(j0 / NST) & 1))) break;
        zero_tail(j0, s0);
        if (!(ok = wait_all(bars.p_full[0], (uint32_t)i & 1))) break;
        fence_after_sync();
        pv_(0, s0, i == 0);
        commit(bars.v_empty[s0]);
      }
      const int jl = 2 * n_pairs - 1;   // the last odd key tile, if there is one
      if (ok && jl < n_kt) {
        const int sl = jl % NST;
        if (wait_all(bars.v_full[sl], (uint32_t)(jl / NST) & 1)) {
          zero_tail(jl, sl);
          if (wait_all(bars.p_full[1], (uint32_t)(n_pairs - 1) & 1)) {
            fence_after_sync();
            pv_(1, sl, n_pairs == 1);
            commit(bars.v_empty[sl]);
          }
        }
      }
    }
    for (int j = 0; ok && !dual && j < n_kt; ++j) {
      const int s = j % NST;
      const uint32_t ph = (uint32_t)(j / NST) & 1;
      if (!(ok = wait_all(bars.k_full[s], ph))) break;
      fence_after_sync();
      qk(0, j);
      commit(bars.s_full[0]);
      if (n_qt == 2) {
        if (j > 0) {
          if (!(ok = wait_all(bars.p_full[1], (uint32_t)(j - 1) & 1))) break;
          fence_after_sync();
          pv(1, j - 1);
          commit(bars.v_empty[(j - 1) % NST]);
        }
        qk(1, j);
        commit(bars.s_full[1]);
      }
      commit(bars.k_empty[s]);
      if (!(ok = wait_all(bars.v_full[s], ph))) break;
      zero_tail(j, s);
      if (!(ok = wait_all(bars.p_full[0], (uint32_t)j & 1))) break;
      fence_after_sync();
      pv(0, j);
      if (n_qt == 1) commit(bars.v_empty[s]);
    }
    if (ok && !dual && n_qt == 2) {
      if (wait_all(bars.p_full[1], (uint32_t)(n_kt - 1) & 1)) {
        fence_after_sync();
        pv(1, n_kt - 1);
        commit(bars.v_empty[(n_kt - 1) % NST]);
      }
    }
    commit(bars.o_full);  // also on abort: tracks whatever was issued
  }
  } else {
    regs_inc<kRegsHigh>();
    // ------------------------------------------------------------ softmax / epilogue
    const int q = (warp - 4) >> 2;
    const int t = tid - 128 - q * BM;  // == TMEM lane
    if (q < n_qt || dual) {
      const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
      const uint32_t S_t = tmem + lane_off + q * 128;
      const uint32_t O_t = tmem + lane_off + 256 + q * 128;
      const int r = r_base + (dual ? 0 : q * BM) + t;
      // key tiles of this warpgroup: all of them, or every other one in dual mode
      const int n_steps = dual ? (n_kt + 1 - q) / 2 : n_kt;
      const int li = min(r / G, m.P - 1) - i_lo;
      const uint64_t* anc = sAnc + (size_t)li * p.W;
      const float c = p.scale_log2;
      float m_ref = -INFINITY, l = 0.f;
      bool ok = true;
      uint32_t v[32];
      // Every tcgen05.ld/st below is .sync.aligned: control flow around them is
      // kept warp-uniform (waits are followed by a warp vote, per-row choices
      // are made with per-lane values inside uniform branches).
      uint32_t sv[BN];
      for (int j = 0; j < n_steps; ++j) {
        ok = mbar_wait(smem_u32(&bars.s_full[q]), (uint32_t)j & 1, abort_flag, p.wait_ns);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        fence_after_sync();
        int n0, klim;
        tile_keys(dual ? 2 * j + q : j, n0, klim);
        const bool full = (n0 + BN <= m.S) && (n0 + BN <= klim);
        // visibility bits of the 128 keys (only tiles that reach the pack or the chunk end)
        uint32_t vis[4] = {~0u, ~0u, ~0u, ~0u};
        if (!full) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) vis[c4] = visible32(anc, p.W, n0 + 32 * c4, m.S, klim);
        }
        // the whole 128-column row of S in one round trip
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) tmem_ld32(S_t + cc * 32, sv + cc * 32);
        tmem_ld_wait();
        if (!full) {
          // invisible keys become -inf: the max ignores them and exp2 gives 0
#pragma unroll
          for (int i = 0; i < BN; ++i)
            sv[i] = ((vis[i >> 5] >> (i & 31)) & 1u) ? sv[i] : 0xff800000u;
        }
        // row max (raw scores; the scale c > 0 is applied once): three-input max, 4 chains
        float mm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < BN / 2; ++i)
          mm[i & 3] = max3(mm[i & 3], __uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
        const float mx = fmaxf(max3(mm[0], mm[1], mm[2]), mm[3]);
        const float m_tile = (mx == -INFINITY) ? -INFINITY : mx * c;
        const bool grow = m_tile > m_ref + kRescaleLog2 || (m_ref == -INFINITY && m_tile != -INFINITY);
        const bool rescale = grow && m_ref != -INFINITY;
        const float alpha = rescale ? ex2(m_ref - m_tile) : 1.f;
        if (grow) m_ref = m_tile;
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
        // P = exp2(S*c - m) in packed pairs (f32x2 FMA / add), 16-bit, into the first 64 columns of S
        const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
        float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = cc * 32 + 2 * i;
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nm2);
            const float p0 = ex2(x.x);
            const float p1 = ex2(x.y);
            acc[i & 1] = __fadd2_rn(acc[i & 1], make_float2(p0, p1));
            pk[i] = pack2<BF16>(p0, p1);
          }
          tmem_st16(S_t + cc * 16, pk);
        }
        l = l * alpha + ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y));
        // lazy correction of O (rows whose max grew by more than 2^8); PV_{j-1} is complete
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            tmem_ld32(O_t + cc * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st32(O_t + cc * 32, v);
          }
        }
        tmem_st_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars.p_full[q]));
      }
      // epilogue: O / l, or the unnormalised partial of this key chunk
      bool done = ok ? mbar_wait(smem_u32(&bars.o_full), 0, abort_flag, p.wait_ns) : mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
      done = __all_sync(0xffffffffu, done && ok);
      fence_after_sync();
      // dual mode: the odd-tile warpgroup hands its (m, l) over; the even one merges the two
      // partials (O_1 sits in the same TMEM lanes, columns 384..511) and writes the rows
      float a0 = 1.f, a1 = 0.f;
      if (dual) {
        if (q == 1) {
          comb_m[t] = m_ref;
          comb_l[t] = l;
          mbar_arrive(smem_u32(&bars.comb));
          done = false;
        } else {
          done = __all_sync(0xffffffffu, done && mbar_wait(smem_u32(&bars.comb), 0, abort_flag, p.wait_ns));
          if (done) {
            const float m1 = comb_m[t], l1 = comb_l[t];
            const float mx = fmaxf(m_ref, m1);
            a0 = m_ref == -INFINITY ? 0.f : ex2(m_ref - mx);
            a1 = m1 == -INFINITY ? 0.f : ex2(m1 - mx);
            l = l * a0 + l1 * a1;
            m_ref = mx;
          }
        }
      }
      const uint32_t O1_t = tmem + lane_off + 256 + 128;
      auto load_o = [&](int cc) {
        tmem_ld32(O_t + cc * 32, v);
        tmem_ld_wait();
        if (dual) {
          uint32_t w[32];
          tmem_ld32(O1_t + cc * 32, w);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = __float_as_uint(__uint_as_float(v[i]) * a0 + __uint_as_float(w[i]) * a1);
        }
      };
      if (done) {
        const bool store = r < rows;
        const int i = min(r / G, m.P - 1), hq = h * G + r % G;
        const int64_t tq = m.q0 + i;
        if (p.n_split == 1) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
          T* out = static_cast<T*>(p.out) + tq * p.so_m + (int64_t)hq * p.so_h;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            load_o(cc);
            uint32_t pk[16];
#pragma unroll
            for (int i2 = 0; i2 < 16; ++i2)
              pk[i2] = pack2<BF16>(__uint_as_float(v[2 * i2]) * inv, __uint_as_float(v[2 * i2 + 1]) * inv);
            if (store) {
              uint4* dst = reinterpret_cast<uint4*>(out + cc * 32);
#pragma unroll
              for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            }
          }
        } else {
          const int64_t slot = ((int64_t)split * p.total_q + tq) * p.H_q + hq;
          float* O = p.ws_o + slot * D;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            load_o(cc);
            if (store) {
              float4* dst = reinterpret_cast<float4*>(O + cc * 32);
#pragma unroll
              for (int u = 0; u < 8; ++u)
                dst[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                                     __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
            }
          }
          if (store) {
            p.ws_ml[slot * 2 + 0] = m_ref;
            p.ws_ml[slot * 2 + 1] = l;
          }
        }
      }
    }
  }

  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) {
    // on the normal path every MMA has completed (o_full); after an abort, wait (bounded) for them
    mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
    __syncwarp();
    tmem_dealloc(tmem, 512);
    tmem_relinquish();
  }
}

}  // namespace tca
}  // namespace cast
