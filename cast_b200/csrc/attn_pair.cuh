// Tensor-core ragged tree attention on CTA pairs (tcgen05 cta_group::2), 16-bit inputs, D = 128.
//
// Work unit (one cluster of two CTAs on the two SMs of a TPC): sequence b, KV head h, a 256-row
// block of the G*P_b rows of that head group (row r = pack token r / G, query head h*G + r % G)
// and a chunk of the key range [0, S_b + P_b). CTA c of the pair owns rows [256 m + 128 c, +128):
// its query tile, its S buffers and its O live in its own SM.
//
// Every MMA is a pair MMA issued by the even CTA: M = 256 (128 rows per SM), N = 128.
//   S_j  = Q K_j^T   A = each CTA's Q tile, B = K_j split by keys: CTA c holds keys [64 c, +64)
//                    of the tile, K-major
//   O   += P_j V_j   A = P_j in each CTA's tensor memory, B = V_j split by dims: CTA c holds dims
//                    [64 c, +64) of all 128 keys, MN-major
// so each SM reads half of every K/V tile from L2 and half the B operand from its own shared
// memory, and every K/V tile serves 256 query rows.
//
// Tensor memory of each CTA (512 columns): three S buffers (key tile j uses buffer j % 3; P_j,
// 16-bit, overwrites its first 64 columns) and one O. With three buffers the tensor core computes
// S_{j+1} and S_{j+2} while the softmax of tile j runs; the MMA order is QK_j, PV_{j-2}, QK_{j+1},
// PV_{j-1}, ..., so the softmax of a tile has four MMA groups' time before its PV is due.
//
// Roles (12 warps per CTA):
//   warp 0      TMA producer of Q (once) and of this CTA's halves of the K tiles; warp 2 of its
//               halves of the V tiles; NST-stage rings; every copy completes on the even CTA's
//               full barriers (the copy's `.cta_group::2` form lets the barrier be the peer's).
//   warp 1      (even CTA) MMA issuer; commits multicast to both CTAs' barriers.
//   warps 4-7   softmax of the even key tiles, warps 8-11 of the odd ones, thread t = TMEM lane t =
//               query row t of this CTA. Both accumulate into the one O: the row max passes from one
//               warpgroup to the other every tile (per warp, through shared memory, bounded waits),
//               O is rescaled lazily (only when the max grows by more than 2^8, after the previous PV
//               completed), each warpgroup keeps its own partial sum l with the max it last used,
//               and the epilogue merges the two sums. Each warpgroup writes 64 of the 128 dims.
// Visibility is that of the single-CTA kernel: keys < S_b always; pack key S_b + j iff bit j of the
// row token's ancestor bitset (shared memory); keys past the chunk end are masked. Every mbarrier
// wait is bounded; on expiry the CTA records CAST_DEV_TIMEOUT and winds down. Both CTAs of a pair
// take the same exits before the first cluster barrier and reach the last one on every path; the
// even CTA's producers wait for every copy they counted before they arrive there, so no copy or MMA
// of the pair is in flight when either CTA exits.
#pragma once

#include "attn_tc.cuh"

namespace cast {
namespace tcp {

constexpr int BM = 128;                       // rows per CTA; a pair covers 256
constexpr int BN = 128;                       // keys per tile
constexpr int D = 128;
constexpr int NSB = 3;                        // S buffers in tensor memory
constexpr int NT = 384;
constexpr int Q_BYTES = BM * D * 2;           // 32 KB: 128 rows x 128 dims
constexpr int Q_PANEL = BM * 128;             // 16 KB: 128 rows x 64 dims (one 128-byte swizzle panel)
constexpr int KH_BYTES = (BN / 2) * D * 2;    // 16 KB: 64 keys x 128 dims
constexpr int K_PANEL = (BN / 2) * 128;       // 8 KB: 64 keys x 64 dims
constexpr int VH_BYTES = BN * (D / 2) * 2;    // 16 KB: 128 keys x 64 dims (one panel)
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = SMEM_Q + Q_BYTES;
constexpr int TM_O = NSB * 128;               // O columns [384, 512)
constexpr float kRescaleLog2 = 8.0f;
constexpr int kRegsLow = 104, kRegsHigh = 200;      // 128 x 104 + 256 x 200 = 384 x 168
constexpr int NST = 4;                        // K/V ring stages (5 measured no faster: 824 against 815 us)

__host__ __device__ constexpr int smem_v(int nst) { return SMEM_K + nst * KH_BYTES; }
__host__ __device__ constexpr int smem_anc(int nst) { return smem_v(nst) + nst * VH_BYTES; }
__host__ __device__ inline int anc_tokens(int G) { return BM / G + 2; }
__host__ __device__ inline size_t smem_bytes(int nst, int G, int W) {
  return 1024 + smem_anc(nst) + (size_t)anc_tokens(G) * W * sizeof(uint64_t) + parent_stage_bytes(W);
}

struct Bars {
  uint64_t q_full;                              // even CTA: both Q tiles landed
  uint64_t k_full[NST], v_full[NST];            // even CTA: both halves of the K / V tile landed
  uint64_t k_empty[NST], v_empty[NST];          // both: the MMAs reading the slot completed
  uint64_t s_full[NSB];                         // both: S of the buffer is computed
  uint64_t p_full[NSB];                         // even CTA: P of the buffer written in both CTAs (8 warps)
  uint64_t pv_done[2];                          // both: PV of the even / odd key tiles completed
  uint64_t o_full;                              // both: every MMA of the pair completed
  uint64_t m_ready[2][4];                       // local: row max after an even / odd tile, per warp
  uint64_t comb;                                // local: both warpgroups' (m, l) published
};

template <bool BF16, int NSTAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NT, 1)
attn_pair_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV) {
  using namespace tc;
  static_assert(NSTAGES == NST, "the barrier arrays are sized by NST");
  constexpr int SMEM_V = smem_v(NST);
  constexpr int SMEM_ANC = smem_anc(NST);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* sAnc = reinterpret_cast<uint64_t*>(smem + SMEM_ANC);
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  __shared__ float m_sh[2][BM];
  __shared__ float comb_m[2][BM], comb_l[2][BM];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = cluster_ctarank();
  const bool lead = crank == 0;
  // Pair index in launch order (a cluster is two consecutive CTAs along x), decoded as (rank of the
  // sequence by length, KV head, key chunk, row block), row blocks fastest.
  const int L = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int U = L >> 1;
  const int nblk = gridDim.x >> 1;
  const int mblk = U % nblk;
  int rest = U / nblk;
  const int split = rest % gridDim.z;
  rest /= gridDim.z;
  const int h = rest % p.H_kv;
  const int rank = rest / p.H_kv;
  const int b = tca::ranked_sequence(p, rank, reinterpret_cast<int*>(smem + SMEM_K));   // K ring as scratch
  // Everything up to the first cluster barrier depends only on the pair's unit, so both CTAs take
  // the same early exits.
  const SeqMeta m = load_seq(p.cu_q, p.cu_kv, p.prefix_len, p.pack_len, b, p.total_q, p.total_kv, p.max_pack,
                             p.max_kv);
  if (!m.ok) {
    if (tid == 0 && lead && mblk == 0 && split == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int G = p.G;
  const int rows = G * m.P;
  const int r_pair = mblk * (2 * BM);
  if (r_pair >= rows) return;
  if (p.pair_full_only && r_pair + 2 * BM > rows) return;   // a partial block: the single-CTA launch takes it
  const int nkeys = m.S + m.P;
  const int k_begin = split * p.chunk;
  if (k_begin >= nkeys) return;
  const int k_end = min(nkeys, k_begin + p.chunk);
  const int n_kt = (k_end - k_begin + BN - 1) / BN;
  const bool has_pack_tile = k_end > m.S;
  const int r_cta = r_pair + (int)crank * BM;        // this CTA's first row (may be past `rows`)
  volatile int* abort_flag = &abort_sh;

  if (tid == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(smem_u32(&bars.k_full[s]), 1);
      mbar_init(smem_u32(&bars.v_full[s]), 1);
      mbar_init(smem_u32(&bars.k_empty[s]), 1);
      mbar_init(smem_u32(&bars.v_empty[s]), 1);
    }
    for (int i = 0; i < NSB; ++i) {
      mbar_init(smem_u32(&bars.s_full[i]), 1);
      mbar_init(smem_u32(&bars.p_full[i]), 2 * BM / 32);   // one arrival per softmax warp of both CTAs
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars.pv_done[i]), 1);
      for (int w = 0; w < 4; ++w) mbar_init(smem_u32(&bars.m_ready[i][w]), 1);   // one arrival per warp
    }
    mbar_init(smem_u32(&bars.o_full), 1);
    mbar_init(smem_u32(&bars.comb), 2 * BM);
    abort_sh = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 0) tmem_alloc_pair(smem_u32(&tmem_base_sh), 512);
  // ancestor bitsets of this CTA's tokens (rows past the pack read the last token's); the pack's
  // parents up to the last of them are staged for the walks
  const int i_lo = min(r_cta / G, m.P - 1);
  const int i_hi = min(m.P - 1, (r_cta + BM - 1) / G);
  int* sPar = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(sAnc) + (size_t)anc_tokens(G) * p.W * sizeof(uint64_t));
  const bool stage = has_pack_tile && p.anc_words == nullptr && p.W <= kStageParentMaxW;
  if (stage)
    for (int j = tid; j <= i_hi; j += NT) sPar[j] = p.parent[m.q0 + j];
  fence_before_sync();
  cluster_sync();   // barriers initialised and tensor memory allocated in both CTAs, parents staged
  fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  // TMA producers: warp 0 loads Q and the K ring, warp 2 the V ring (a V slot frees only when its
  // PV completes, two tiles after its QK). Every copy of the pair completes on the even CTA's
  // barrier, which expects both CTAs' bytes.
  const bool is_k = warp == 0;
  uint64_t* full = is_k ? bars.k_full : bars.v_full;
  uint64_t* empty = is_k ? bars.k_empty : bars.v_empty;
  auto issue_tile = [&](int j) {
    const int s = j % NST;
    const int key0 = m.kv0 + k_begin + j * BN;
    if (elect_one()) {
      if (lead) mbar_expect_tx(smem_u32(&full[s]), 2 * (is_k ? KH_BYTES : VH_BYTES));
      const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
      if (is_k) {
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d_pair(smem_u32(smem + SMEM_K + s * KH_BYTES + hf * K_PANEL), &tmK, hf * 64, h,
                           key0 + (int)crank * (BN / 2), fb);
      } else {
        tma_load_3d_pair(smem_u32(smem + SMEM_V + s * VH_BYTES), &tmV, (int)crank * 64, h, key0, fb);
      }
    }
    __syncwarp();
  };
  // Q and the first NST key tiles need no free slot: their copies go out before the bitsets are built.
  const int n_early = min(NST, n_kt);
  if (warp == 0 || warp == 2) {
    if (is_k && elect_one()) {
      if (lead) mbar_expect_tx(smem_u32(&bars.q_full), 2 * Q_BYTES);
      const uint32_t qf = mapa_shared(smem_u32(&bars.q_full), 0);
      const int tok = m.q0 + r_cta / G;
      for (int hf = 0; hf < 2; ++hf)
        tma_load_3d_pair(smem_u32(smem + SMEM_Q + hf * Q_PANEL), &tmQ, hf * 64, h * G, tok, qf);
    }
    __syncwarp();
    for (int j = 0; j < n_early; ++j) issue_tile(j);
  }
  if (has_pack_tile) build_tile_bitsets(p, m, i_lo, i_hi - i_lo + 1, sAnc, stage ? sPar : nullptr);
  __syncthreads();   // bitsets built

  if (warp < 4) {
    regs_dec<kRegsLow>();
    if (warp == 0 || warp == 2) {
      // ---------------------------------------------------------------- TMA producers (continued)
      // In each ring slot j % NST is refilled once the MMAs of use j - NST completed.
      int issued = n_early;
      for (int j = n_early; j < n_kt; ++j) {
        const int s = j % NST;
        const uint32_t use = (uint32_t)(j / NST);
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&empty[s]), (use - 1) & 1, abort_flag, p.wait_ns)))
          break;
        issue_tile(j);
        issued = j + 1;
      }
      if (lead) {
        // Every copy of the pair completes on these barriers: wait for the ones counted here
        // (immediate on the normal path, where the MMAs consumed them all). After an abort a phase
        // may never complete (the other CTA stopped issuing): short limit.
        const uint64_t lim = *abort_flag ? 50000000ull : kWaitLimitNs;
        for (int j = max(0, issued - NST); j < issued; ++j)
          mbar_wait(smem_u32(&full[j % NST]), (uint32_t)(j / NST) & 1, nullptr, lim);
        if (is_k) mbar_wait(smem_u32(&bars.q_full), 0, nullptr, lim);
      }
      if (*abort_flag) {
        // After an abort this CTA cannot see when its last copies land (the odd CTA's complete on the
        // even CTA's barriers, and the even CTA may not have counted them): give every copy already
        // issued a bounded 200 us to land before the CTA can reach the final cluster barrier.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
      }
    } else if (warp == 1 && lead) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_qk = idesc_f16(BF16, 2 * BM, BN, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(BF16, 2 * BM, D, false, true);
      const uint32_t sQ = smem_u32(smem + SMEM_Q), sK = smem_u32(smem + SMEM_K), sV = smem_u32(smem + SMEM_V);
      const uint64_t dQ = desc_kmajor(sQ);
      constexpr uint16_t kBoth = 0x3;
      auto commit = [&](uint64_t& bar) {
        if (elect_one()) mma_commit_pair(smem_u32(&bar), kBoth);
        __syncwarp();
      };
      auto wait_all = [&](uint64_t& bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(smem_u32(&bar), parity, abort_flag, p.wait_ns));
      };
      // O (+)= P_i V_i
      auto pv = [&](int i) -> bool {
        const int s = i % NST, bi = i % NSB;
        if (!wait_all(bars.v_full[s], (uint32_t)(i / NST) & 1)) return false;
        if (!wait_all(bars.p_full[bi], (uint32_t)(i / NSB) & 1)) return false;
        fence_after_sync();
        const uint64_t dv = desc_mnmajor(sV + s * VH_BYTES, VH_BYTES);
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            mma_ts_pair(tmem + TM_O, tmem + bi * 128 + k * 8, dv + (uint64_t)((k * 2048) >> 4), idesc_pv,
                        (i > 0 || k > 0) ? 1u : 0u);
        }
        __syncwarp();
        commit(bars.v_empty[s]);
        commit(bars.pv_done[i & 1]);
        return true;
      };
      bool ok = wait_all(bars.q_full, 0);
      for (int j = 0; ok && j < n_kt; ++j) {
        const int s = j % NST, bj = j % NSB;
        if (!(ok = wait_all(bars.k_full[s], (uint32_t)(j / NST) & 1))) break;
        fence_after_sync();
        const uint64_t dk = desc_kmajor(sK + s * KH_BYTES);
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t oq = (uint64_t)(((k >> 2) * Q_PANEL + (k & 3) * 32) >> 4);
            const uint64_t okk = (uint64_t)(((k >> 2) * K_PANEL + (k & 3) * 32) >> 4);
            mma_ss_pair(tmem + bj * 128, dQ + oq, dk + okk, idesc_qk, k > 0 ? 1u : 0u);
          }
        }
        __syncwarp();
        commit(bars.s_full[bj]);
        commit(bars.k_empty[s]);
        // S buffer (j + 1) % 3 held P_{j-2}: its PV goes before QK_{j+1}
        if (j >= 2) ok = pv(j - 2);
      }
      for (int i = max(0, n_kt - 2); ok && i < n_kt; ++i) ok = pv(i);
      commit(bars.o_full);   // also after an abort: tracks whatever was issued
    }
  } else {
    regs_inc<kRegsHigh>();
    // ---------------------------------------------------------------- softmax / epilogue
    const int wg = (warp - 4) >> 2;
    const int t = tid - 128 - wg * BM;                 // == TMEM lane == query row of this CTA
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int r = r_cta + t;
    const int li = min(r / G, m.P - 1) - i_lo;
    const uint64_t* anc = sAnc + (size_t)li * p.W;
    const float c = p.scale_log2;
    const uint32_t pf_lead = mapa_shared(smem_u32(&bars.p_full[0]), 0);
    float m_w = -INFINITY, l_w = 0.f;                  // this warpgroup's last max and partial sum
    bool ok = true;
    uint32_t sv[BN];
    uint32_t v[32];
    for (int j = wg; j < n_kt; j += 2) {
      const int bj = j % NSB;
      ok = mbar_wait(smem_u32(&bars.s_full[bj]), (uint32_t)(j / NSB) & 1, abort_flag, p.wait_ns);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      fence_after_sync();
      const uint32_t S_t = tmem + lane_off + bj * 128;
      const int n0 = k_begin + j * BN;
      const bool full = (n0 + BN <= m.S) && (n0 + BN <= k_end);
      uint32_t vis[4] = {~0u, ~0u, ~0u, ~0u};
      if (!full) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) vis[c4] = visible32(anc, p.W, n0 + 32 * c4, m.S, k_end);
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(S_t + cc * 32, sv + cc * 32);
      tmem_ld_wait();
      if (!full) {
#pragma unroll
        for (int i = 0; i < BN; ++i) sv[i] = ((vis[i >> 5] >> (i & 31)) & 1u) ? sv[i] : 0xff800000u;
      }
      float mm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN / 2; ++i)
        mm[i & 3] = tca::max3(mm[i & 3], __uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
      const float mx = fmaxf(tca::max3(mm[0], mm[1], mm[2]), mm[3]);
      const float m_tile = (mx == -INFINITY) ? -INFINITY : mx * c;
      // the running max after tile j - 1 comes from the same rows' warp of the other warpgroup
      float m_prev = -INFINITY;
      if (j > 0) {
        ok = mbar_wait(smem_u32(&bars.m_ready[(j - 1) & 1][warp & 3]), (uint32_t)((j - 1) >> 1) & 1, abort_flag,
                       p.wait_ns);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        m_prev = m_sh[(j - 1) & 1][t];
      }
      const bool grow = m_tile > m_prev + kRescaleLog2 || (m_prev == -INFINITY && m_tile != -INFINITY);
      const float m_new = grow ? m_tile : m_prev;
      m_sh[j & 1][t] = m_new;
      __syncwarp();   // the warp's m_sh writes are ordered before its lane 0's (releasing) arrival
      if (lane == 0) mbar_arrive(smem_u32(&bars.m_ready[j & 1][warp & 3]));
      const bool rescale = grow && m_prev != -INFINITY;
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = cc * 32 + 2 * i;
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nm2);
          const float p0 = tca::ex2(x.x);
          const float p1 = tca::ex2(x.y);
          acc[i & 1] = __fadd2_rn(acc[i & 1], make_float2(p0, p1));
          pk[i] = tca::pack2<BF16>(p0, p1);
        }
        tmem_st16(S_t + cc * 16, pk);
      }
      if (m_w != m_new) l_w = (m_w == -INFINITY) ? 0.f : l_w * tca::ex2(m_w - m_new);
      l_w += (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
      m_w = m_new;
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds the tiles before j in the scale of m_prev once PV_{j-1} has completed; PV_j waits
        // for this warpgroup's P, so nothing writes O while it is rescaled
        ok = mbar_wait(smem_u32(&bars.pv_done[(j - 1) & 1]), (uint32_t)((j - 1) >> 1) & 1, abort_flag, p.wait_ns);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        fence_after_sync();
        const float alpha = rescale ? tca::ex2(m_prev - m_new) : 1.f;
        const uint32_t O_t = tmem + lane_off + TM_O;
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
      if (lane == 0) mbar_arrive_cluster(pf_lead + (uint32_t)(bj * sizeof(uint64_t)));
    }
    // ---- epilogue: O (scale: the last tile's max) / (l_0 + l_1 in that scale)
    bool done = ok ? mbar_wait(smem_u32(&bars.o_full), 0, abort_flag, p.wait_ns)
                   : mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
    done = __all_sync(0xffffffffu, done && ok);
    fence_after_sync();
    comb_m[wg][t] = m_w;
    comb_l[wg][t] = l_w;
    mbar_arrive(smem_u32(&bars.comb));
    done = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars.comb), 0, abort_flag, p.wait_ns) && done);
    if (done) {
      const float m0 = comb_m[0][t], m1 = comb_m[1][t];
      const float mf = fmaxf(m0, m1);
      const float l = (m0 == -INFINITY ? 0.f : comb_l[0][t] * tca::ex2(m0 - mf)) +
                      (m1 == -INFINITY ? 0.f : comb_l[1][t] * tca::ex2(m1 - mf));
      const bool store = r < rows;
      const int i = min(r / G, m.P - 1), hq = h * G + r % G;
      const int64_t tq = m.q0 + i;
      const uint32_t O_t = tmem + lane_off + TM_O + wg * 64;
      if (p.n_split == 1) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        T* out = static_cast<T*>(p.out) + tq * p.so_m + (int64_t)hq * p.so_h + wg * 64;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          tmem_ld32(O_t + cc * 32, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2)
            pk[i2] = tca::pack2<BF16>(__uint_as_float(v[2 * i2]) * inv, __uint_as_float(v[2 * i2 + 1]) * inv);
          if (store) {
            uint4* dst = reinterpret_cast<uint4*>(out + cc * 32);
#pragma unroll
            for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
          }
        }
      } else {
        const int64_t slot = ((int64_t)split * p.total_q + tq) * p.H_q + hq;
        float* O = p.ws_o + slot * D + wg * 64;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          tmem_ld32(O_t + cc * 32, v);
          tmem_ld_wait();
          if (store) {
            float4* dst = reinterpret_cast<float4*>(O + cc * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u)
              dst[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                                   __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
          }
        }
        if (store && wg == 0) {
          p.ws_ml[slot * 2 + 0] = mf;
          p.ws_ml[slot * 2 + 1] = l;
        }
      }
    }
  }

  // ---- wind-down: no MMA of the pair in flight (o_full), every copy landed (the even CTA's
  // producers waited above), then both CTAs leave together and free the pair's tensor memory
  if (warp == 0) mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
  fence_before_sync();
  cluster_sync();
  fence_after_sync();
  if (warp == 0) {
    tmem_dealloc_pair(tmem, 512);
    tmem_relinquish_pair();
  }
}

}  // namespace tcp
}  // namespace cast
