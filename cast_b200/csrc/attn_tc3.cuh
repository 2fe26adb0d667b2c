// fp32 ragged tree attention on the tensor cores, from a three-term bf16 split.
//
// A float x is carried as hi + lo with hi = bf16(x) and lo = bf16(x - hi): about 16
// significant bits, a relative error near 2^-17. Products drop only the lo * lo term:
//   S  = Qh Kh^T + Qh Kl^T + Ql Kh^T
//   O += Ph Vh   + Pl Vh   + Ph Vl        (P = exp2(S c - m) in fp32, split the same way)
// so the output stays within ~1e-5 of the fp32 reference at unit-scale inputs, against
// the 1e-3 a single bf16 (or tf32) pass gives. split3_kernel writes the hi / lo copies of
// q, k and v (contiguous [rows, heads, 128] bf16) into the caller's workspace and raises a
// flag per tensor when any lo is non-zero; the attention kernel reads the flags and skips
// the MMAs of all-zero lo parts, so fp32 copies of 16-bit data (the reference hook's
// .float() inputs, cast_trees/serving.py:68-71) cost one QK and two PV MMAs per tile.
//
// Work unit (one CTA per SM): sequence b, KV head h, one 128-row query tile of the G*P_b rows
// of that head group, a chunk of the key range; units start longest sequence first.
// Roles (8 warps): warp 0 TMA producer (Q once, then one 128-key K and V tile at a time, hi
// and lo), warp 1 MMA issuer, warps 4-7 softmax (thread t = TMEM lane t = query row t;
// Ph goes to columns 0-63 of S, Pl to 64-127). Tensor memory: S (128 columns), O (128).
// Shared memory: Qh, Ql, Kh, Kl, Vh, Vl (32 KB each) and the ancestor bitsets. Waits are
// bounded as in the 16-bit kernel; on expiry the CTA reports CAST_DEV_TIMEOUT, drains and exits.
#pragma once

#include "attn_tc.cuh"

namespace cast {
namespace tc3 {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int D = 128;
constexpr int NT = 256;
constexpr int TILE_BYTES = BN * D * 2;
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int SMEM_QH = 0;
constexpr int SMEM_QL = SMEM_QH + TILE_BYTES;
constexpr int SMEM_KH = SMEM_QL + TILE_BYTES;
constexpr int SMEM_KL = SMEM_KH + TILE_BYTES;
constexpr int SMEM_VH = SMEM_KL + TILE_BYTES;
constexpr int SMEM_VL = SMEM_VH + TILE_BYTES;
constexpr int SMEM_ANC = SMEM_VL + TILE_BYTES;   // 196608
constexpr float kRescaleLog2 = 8.0f;

__host__ __device__ inline int anc_tokens(int G) { return BM / G + 2; }
__host__ __device__ inline size_t smem_bytes(int G, int W) {
  return 1024 + SMEM_ANC + (size_t)anc_tokens(G) * W * sizeof(uint64_t) + parent_stage_bytes(W);
}

// ---- split pass -----------------------------------------------------------------
struct SplitSrc {
  const float* src;      // [rows, heads, 128], dim stride 1 (store layout: [batch, heads, store_rows, 128])
  int64_t rows, s_row, s_head;
  int heads;
  __nv_bfloat16* hi;     // [rows, heads, 128] contiguous
  __nv_bfloat16* lo;
  // Store layout (the store entry point's k and v): output row r is position s = r - cu_kv[b] of
  // sequence b, read from the store at [b, h, s] for s < prefix_len[b] and from `pack`
  // [cu_q[b] + s - prefix_len[b], h] after it; rows past cu_kv[B] are written as zeros.
  int store;
  const float* pack;
  int64_t s_b, pk_row, pk_head;
  int B, store_rows, max_pack, total_q;
  const int32_t* cu_kv;
  const int32_t* cu_q;
  const int32_t* prefix_len;
  const int32_t* pack_len;
};

// Largest b in [0, B) with cu[b] <= r (cu non-decreasing, cu[0] = 0).
__device__ __forceinline__ int seq_of_row(const int32_t* cu, int B, int64_t r) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Source row (nullptr: write zeros) of ragged row r, head h of a store-layout tensor.
__device__ __forceinline__ const float* store_row(const SplitSrc& t, int64_t r, int h) {
  if (r >= t.cu_kv[t.B]) return nullptr;
  const int b = seq_of_row(t.cu_kv, t.B, r);
  const int64_t s = r - t.cu_kv[b];
  const int S = t.prefix_len[b], P = t.pack_len[b], q0 = t.cu_q[b];
  if (S < 0 || S > t.store_rows || P < 0 || P > t.max_pack || q0 < 0 || (int64_t)q0 + P > t.total_q || s < 0 ||
      s >= (int64_t)S + P) {
    report(CAST_DEV_BAD_LAYOUT);
    return nullptr;
  }
  return s < S ? t.src + b * t.s_b + h * t.s_head + s * t.s_row : t.pack + (q0 + s - S) * t.pk_row + h * t.pk_head;
}

// cu_kv[b] = sum over b' < b of prefix_len[b'] + pack_len[b'] (negative lengths count as 0,
// the sum saturates at INT32_MAX). One block of 1024 threads.
__global__ void __launch_bounds__(1024) cu_kv_scan_kernel(const int32_t* prefix_len, const int32_t* pack_len, int B,
                                                          int32_t* cu_kv) {
  __shared__ long long warp_sum[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  long long carry = 0;
  for (int base = 0; base < B; base += 1024) {
    const int i = base + threadIdx.x;
    long long x = i < B ? (long long)max(0, prefix_len[i]) + max(0, pack_len[i]) : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sum[wid] = x;
    __syncthreads();
    if (wid == 0) {
      long long w = warp_sum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sum[lane] = w;
    }
    __syncthreads();
    const long long incl = carry + x + (wid > 0 ? warp_sum[wid - 1] : 0);
    if (i < B) cu_kv[i + 1] = (int32_t)min(incl, 0x7fffffffLL);
    carry += warp_sum[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) cu_kv[0] = 0;
}
// ---- ragged assembly -------------------------------------------------------------
// K and V of the store layout copied into the ragged layout [rows_cap, H, D] (contiguous),
// for the shapes the tensor-core kernels do not take (the CUDA-core kernel reads only the
// ragged layout). One warp per (row, head); rows past cu_kv[B] are zeros.
struct GatherArgs {
  const void* store[2];
  const void* pack[2];
  void* out[2];
  int64_t st_b[2], st_h[2], st_r[2], pk_t[2], pk_h[2];
  int B, H, D, store_rows, max_pack, total_q;
  int64_t rows_cap;
  const int32_t* cu_kv;
  const int32_t* cu_q;
  const int32_t* prefix_len;
  const int32_t* pack_len;
};

template <typename T>
__global__ void __launch_bounds__(256) kv_ragged_gather_kernel(const GatherArgs a) {
  const int kv = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int64_t n = a.rows_cap * a.H;
  T* out = static_cast<T*>(a.out[kv]);
  for (int64_t rh = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; rh < n;
       rh += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t r = rh / a.H;
    const int h = (int)(rh - r * a.H);
    const T* src = nullptr;
    if (r < a.cu_kv[a.B]) {
      const int b = seq_of_row(a.cu_kv, a.B, r);
      const int64_t s = r - a.cu_kv[b];
      const int S = a.prefix_len[b], P = a.pack_len[b], q0 = a.cu_q[b];
      if (S < 0 || S > a.store_rows || P < 0 || P > a.max_pack || q0 < 0 || (int64_t)q0 + P > a.total_q || s < 0 ||
          s >= (int64_t)S + P) {
        if (lane == 0) report(CAST_DEV_BAD_LAYOUT);
      } else if (s < S) {
        src = static_cast<const T*>(a.store[kv]) + b * a.st_b[kv] + h * a.st_h[kv] + s * a.st_r[kv];
      } else {
        src = static_cast<const T*>(a.pack[kv]) + (q0 + s - S) * a.pk_t[kv] + h * a.pk_h[kv];
      }
    }
    T* dst = out + rh * a.D;
    for (int c = lane; c < a.D; c += 32) dst[c] = src ? src[c] : T(0);
  }
}

struct SplitArgs {
  SplitSrc t[3];         // q, k, v
  int* flags;            // [3], zeroed before the launch
};

// blockIdx.y picks the tensor; a grid-stride loop over its float4 groups.
__global__ void __launch_bounds__(256) split3_kernel(const SplitArgs a) {
  const SplitSrc& t = a.t[blockIdx.y];
  const int64_t n4 = t.rows * t.heads * 32;
  uint32_t any = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rh = i >> 5;
    const int c = (int)(i & 31) * 4;
    const int64_t r = rh / t.heads;
    const int h = (int)(rh - r * t.heads);
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t.store) {
      const float* row = store_row(t, r, h);   // warp-uniform: the 32 lanes of a warp share (r, h)
      if (row != nullptr) x = __ldg(reinterpret_cast<const float4*>(row + c));
    } else {
      x = __ldg(reinterpret_cast<const float4*>(t.src + r * t.s_row + h * t.s_head + c));
    }
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(x.x - f01.x, x.y - f01.y);
    const __nv_bfloat162 l23 = __floats2bfloat162_rn(x.z - f23.x, x.w - f23.y);
    uint2 hv, lv;
    hv.x = *reinterpret_cast<const uint32_t*>(&h01);
    hv.y = *reinterpret_cast<const uint32_t*>(&h23);
    lv.x = *reinterpret_cast<const uint32_t*>(&l01);
    lv.y = *reinterpret_cast<const uint32_t*>(&l23);
    *reinterpret_cast<uint2*>(t.hi + i * 4) = hv;
    *reinterpret_cast<uint2*>(t.lo + i * 4) = lv;
    any |= (lv.x | lv.y) & 0x7fff7fffu;   // -0.0 counts as zero
  }
  if (__any_sync(0xffffffffu, any != 0) && (threadIdx.x & 31) == 0) atomicOr(a.flags + blockIdx.y, 1);
}

// ---- attention ----------------------------------------------------------------------
struct Bars {
  uint64_t q_full, k_full, k_empty, v_full, v_empty, s_full, p_full, o_full;
};

__global__ void __launch_bounds__(NT, 1)
attn_tc3_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl) {
  using namespace tc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* sAnc = reinterpret_cast<uint64_t*>(smem + SMEM_ANC);
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int mblk = L % gridDim.x;
  int rest = L / gridDim.x;
  const int split = rest % gridDim.z;
  rest /= gridDim.z;
  const int h = rest % p.H_kv;
  const int rank = rest / p.H_kv;
  const int b = tca::ranked_sequence(p, rank, reinterpret_cast<int*>(smem + SMEM_KH));
  const SeqMeta m = load_seq(p.cu_q, p.cu_kv, p.prefix_len, p.pack_len, b, p.total_q, p.total_kv, p.max_pack,
                             p.max_kv);
  if (!m.ok) {
    if (tid == 0 && mblk == 0 && split == 0) report(CAST_DEV_BAD_LAYOUT);
    return;
  }
  const int G = p.G;
  const int rows = G * m.P;
  const int r_base = mblk * BM;
  if (r_base >= rows) return;
  const int nkeys = m.S + m.P;
  const int k_begin = split * p.chunk;
  if (k_begin >= nkeys) return;
  const int k_end = min(nkeys, k_begin + p.chunk);
  const int n_kt = (k_end - k_begin + BN - 1) / BN;
  const bool has_pack_tile = k_end > m.S;
  const bool q_lo = p.split_flags[0] != 0, k_lo = p.split_flags[1] != 0, v_lo = p.split_flags[2] != 0;
  volatile int* abort_flag = &abort_sh;

  if (tid == 0) {
    mbar_init(smem_u32(&bars.q_full), 1);
    mbar_init(smem_u32(&bars.k_full), 1);
    mbar_init(smem_u32(&bars.k_empty), 1);
    mbar_init(smem_u32(&bars.v_full), 1);
    mbar_init(smem_u32(&bars.v_empty), 1);
    mbar_init(smem_u32(&bars.s_full), 1);
    mbar_init(smem_u32(&bars.p_full), BM / 32);   // one arrival per softmax warp
    mbar_init(smem_u32(&bars.o_full), 1);
    abort_sh = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQh);
    tma_prefetch_desc(&tmKh);
    tma_prefetch_desc(&tmVh);
  }
  if (warp == 0) tmem_alloc(smem_u32(&tmem_base_sh), 256);
  const int i_lo = r_base / G;
  const int i_hi = min(m.P - 1, (r_base + BM - 1) / G);
  // the pack's parents up to the last token of the tile, staged for the bitset walks
  int* sPar = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(sAnc) + (size_t)anc_tokens(G) * p.W * sizeof(uint64_t));
  const bool stage = has_pack_tile && p.anc_words == nullptr && p.W <= kStageParentMaxW;
  if (stage) {
    for (int j = tid; j <= i_hi; j += NT) sPar[j] = p.parent[m.q0 + j];
    __syncthreads();
  }
  if (has_pack_tile) build_tile_bitsets(p, m, i_lo, i_hi - i_lo + 1, sAnc, stage ? sPar : nullptr);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    const uint32_t qf = smem_u32(&bars.q_full);
    if (elect_one()) {
      mbar_expect_tx(qf, (q_lo ? 2 : 1) * TILE_BYTES);
      const int tok = m.q0 + r_base / G;
      for (int hf = 0; hf < 2; ++hf) {
        tma_load_3d(smem_u32(smem + SMEM_QH + hf * HALF_BYTES), &tmQh, hf * 64, h * G, tok, qf);
        if (q_lo) tma_load_3d(smem_u32(smem + SMEM_QL + hf * HALF_BYTES), &tmQl, hf * 64, h * G, tok, qf);
      }
    }
    __syncwarp();
    int issued_k = 0, issued_v = 0;
    for (int j = 0; j < n_kt; ++j) {
      const int row = m.kv0 + k_begin + j * BN;
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars.k_empty), (uint32_t)(j - 1) & 1, abort_flag,
                                                       p.wait_ns)))
        break;
      if (elect_one()) {
        const uint32_t bar = smem_u32(&bars.k_full);
        mbar_expect_tx(bar, (k_lo ? 2 : 1) * TILE_BYTES);
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_3d(smem_u32(smem + SMEM_KH + hf * HALF_BYTES), &tmKh, hf * 64, h, row, bar);
          if (k_lo) tma_load_3d(smem_u32(smem + SMEM_KL + hf * HALF_BYTES), &tmKl, hf * 64, h, row, bar);
        }
      }
      __syncwarp();
      issued_k = j + 1;
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars.v_empty), (uint32_t)(j - 1) & 1, abort_flag,
                                                       p.wait_ns)))
        break;
      if (elect_one()) {
        const uint32_t bar = smem_u32(&bars.v_full);
        mbar_expect_tx(bar, (v_lo ? 2 : 1) * TILE_BYTES);
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_3d(smem_u32(smem + SMEM_VH + hf * HALF_BYTES), &tmVh, hf * 64, h, row, bar);
          if (v_lo) tma_load_3d(smem_u32(smem + SMEM_VL + hf * HALF_BYTES), &tmVl, hf * 64, h, row, bar);
        }
      }
      __syncwarp();
      issued_v = j + 1;
    }
    // the last issued copies land before the CTA can exit (earlier ones were consumed)
    if (issued_k > 0) mbar_wait(smem_u32(&bars.k_full), (uint32_t)(issued_k - 1) & 1, nullptr);
    if (issued_v > 0) mbar_wait(smem_u32(&bars.v_full), (uint32_t)(issued_v - 1) & 1, nullptr);
    mbar_wait(qf, 0, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_f16(true, BM, BN, false, false);
    constexpr uint32_t idesc_pv = idesc_f16(true, BM, D, false, true);
    const uint64_t dQh = desc_kmajor(smem_u32(smem + SMEM_QH)), dQl = desc_kmajor(smem_u32(smem + SMEM_QL));
    const uint64_t dKh = desc_kmajor(smem_u32(smem + SMEM_KH)), dKl = desc_kmajor(smem_u32(smem + SMEM_KL));
    const uint64_t dVh = desc_mnmajor(smem_u32(smem + SMEM_VH), HALF_BYTES);
    const uint64_t dVl = desc_mnmajor(smem_u32(smem + SMEM_VL), HALF_BYTES);
    const uint32_t S_t = tmem, O_t = tmem + 128;
    auto wait_all = [&](uint64_t& bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(&bar), parity, abort_flag, p.wait_ns));
    };
    auto commit = [&](uint64_t& bar) {
      if (elect_one()) mma_commit(smem_u32(&bar));
      __syncwarp();
    };
    bool ok = wait_all(bars.q_full, 0);
    for (int j = 0; ok && j < n_kt; ++j) {
      const uint32_t ph = (uint32_t)j & 1;
      if (!(ok = wait_all(bars.k_full, ph))) break;
      fence_after_sync();
      if (elect_one()) {
        // S = Qh Kh^T (+ Qh Kl^T) (+ Ql Kh^T), 16 dims per MMA
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t off = (uint64_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
          mma_ss(S_t, dQh + off, dKh + off, idesc_qk, k > 0 ? 1u : 0u);
        }
        if (k_lo) {
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t off = (uint64_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
            mma_ss(S_t, dQh + off, dKl + off, idesc_qk, 1u);
          }
        }
        if (q_lo) {
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t off = (uint64_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
            mma_ss(S_t, dQl + off, dKh + off, idesc_qk, 1u);
          }
        }
      }
      __syncwarp();
      commit(bars.s_full);
      commit(bars.k_empty);
      if (!(ok = wait_all(bars.v_full, ph))) break;
      if (!(ok = wait_all(bars.p_full, ph))) break;
      fence_after_sync();
      if (elect_one()) {
        // O += Ph Vh + Pl Vh (+ Ph Vl), 16 keys per MMA; Ph in S columns 0-63, Pl in 64-127
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t voff = (uint64_t)((k * 2048) >> 4);
          mma_ts(O_t, S_t + k * 8, dVh + voff, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
          mma_ts(O_t, S_t + 64 + k * 8, dVh + voff, idesc_pv, 1u);
          if (v_lo) mma_ts(O_t, S_t + k * 8, dVl + voff, idesc_pv, 1u);
        }
      }
      __syncwarp();
      commit(bars.v_empty);
    }
    commit(bars.o_full);  // also on abort: tracks whatever was issued
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / epilogue
    const int t = tid - 128;   // == TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t S_t = tmem + lane_off, O_t = tmem + lane_off + 128;
    const int r = r_base + t;
    const int li = min(r / G, m.P - 1) - i_lo;
    const uint64_t* anc = sAnc + (size_t)li * p.W;
    const float c = p.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    uint32_t sv[BN];
    uint32_t v[32];
    for (int j = 0; j < n_kt; ++j) {
      ok = mbar_wait(smem_u32(&bars.s_full), (uint32_t)j & 1, abort_flag, p.wait_ns);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      fence_after_sync();
      const int n0 = k_begin + j * BN, klim = k_end;
      const bool full = (n0 + BN <= m.S) && (n0 + BN <= klim);
      uint32_t vis[4] = {~0u, ~0u, ~0u, ~0u};
      if (!full) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) vis[c4] = visible32(anc, p.W, n0 + 32 * c4, m.S, klim);
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
      const bool grow = m_tile > m_ref + kRescaleLog2 || (m_ref == -INFINITY && m_tile != -INFINITY);
      const bool rescale = grow && m_ref != -INFINITY;
      const float alpha = rescale ? tca::ex2(m_ref - m_tile) : 1.f;
      if (grow) m_ref = m_tile;
      const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
      // P in fp32, then Ph = bf16(P) to columns [0, 64) and Pl = bf16(P - Ph) to [64, 128)
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = cc * 32 + 2 * i;
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nm2);
          const float p0 = tca::ex2(x.x), p1 = tca::ex2(x.y);
          acc[i & 1] = __fadd2_rn(acc[i & 1], make_float2(p0, p1));
          const __nv_bfloat162 hb = __floats2bfloat162_rn(p0, p1);
          const float2 hf = __bfloat1622float2(hb);
          const __nv_bfloat162 lb = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
          ph[i] = *reinterpret_cast<const uint32_t*>(&hb);
          pl[i] = *reinterpret_cast<const uint32_t*>(&lb);
        }
        tmem_st16(S_t + cc * 16, ph);
        tmem_st16(S_t + 64 + cc * 16, pl);
      }
      l = l * alpha + ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y));
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
      if (lane == 0) mbar_arrive(smem_u32(&bars.p_full));
    }
    bool done = ok ? mbar_wait(smem_u32(&bars.o_full), 0, abort_flag, p.wait_ns)
                   : mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
    done = __all_sync(0xffffffffu, done && ok);
    fence_after_sync();
    if (done) {
      const bool store = r < rows;
      const int i = min(r / G, m.P - 1), hq = h * G + r % G;
      const int64_t tq = m.q0 + i;
      if (p.n_split == 1) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float* out = static_cast<float*>(p.out) + tq * p.so_m + (int64_t)hq * p.so_h;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          tmem_ld32(O_t + cc * 32, v);
          tmem_ld_wait();
          if (store) {
            float4* dst = reinterpret_cast<float4*>(out + cc * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u)
              dst[u] = make_float4(__uint_as_float(v[4 * u]) * inv, __uint_as_float(v[4 * u + 1]) * inv,
                                   __uint_as_float(v[4 * u + 2]) * inv, __uint_as_float(v[4 * u + 3]) * inv);
          }
        }
      } else {
        const int64_t slot = ((int64_t)split * p.total_q + tq) * p.H_q + hq;
        float* O = p.ws_o + slot * D;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
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
        if (store) {
          p.ws_ml[slot * 2 + 0] = m_ref;
          p.ws_ml[slot * 2 + 1] = l;
        }
      }
    }
  }

  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (warp == 0) {
    mbar_wait(smem_u32(&bars.o_full), 0, nullptr);
    __syncwarp();
    tmem_dealloc(tmem, 256);
    tmem_relinquish();
  }
}

}  // namespace tc3
}  // namespace cast
