// C ABI of cast_b200 (declared in include/cast_b200.h): argument checks, launch
// planning and kernel dispatch. Everything the library launches is in this
// translation unit, so the per-device error word is one symbol.
#include <cudaTypedefs.h>
#include <math.h>
#include <stdio.h>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "attn_simt.cuh"
#include "attn_tc.cuh"
#include "attn_tc3.cuh"
#include "attn_pair.cuh"
#include "tree_build.cuh"
#include "verify_ops.cuh"

namespace cast {
namespace {

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
// Limit of the tensor-core kernel's pipeline waits for the launches that follow
// (cast_test_set_wait_limit_ns); the default is the library-wide wait limit.
std::atomic<uint64_t> g_pipeline_wait_ns{tc::kWaitLimitNs};
// 16-bit kernel of the regular-layout launches that follow (cast_test_set_tc_kernel): 1 = CTA pairs
// (attn_pair_kernel) where they apply, the default; 0 = single CTAs (attn_tc_kernel); -1 = the
// CUDA-core kernel (attn_simt_kernel), for measuring the dispatch.
std::atomic<int> g_tc_kernel{1};

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return -1;
  if (dev < kMaxDevices) {
    const int cached = g_sm_count[dev].load(std::memory_order_relaxed);
    if (cached > 0) return cached;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return -1;
  if (dev < kMaxDevices) g_sm_count[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Launch plan of the CUDA-core kernel: the key range of every sequence is cut
// into `chunk`-key pieces until the grid covers the GPU about twice.
struct SimtPlan {
  int m_tiles, n_split, chunk, W;
  size_t ws_bytes;
};

SimtPlan plan_simt(int B, int total_q, int H_q, int H_kv, int D, int max_pack, int max_kv, int sms) {
  SimtPlan pl;
  const int G = H_q / H_kv;
  pl.m_tiles = (G * max_pack + simt::BM - 1) / simt::BM;
  if (pl.m_tiles < 1) pl.m_tiles = 1;
  pl.W = (max_pack + 63) / 64;
  if (pl.W < 1) pl.W = 1;
  const long long base = (long long)B * H_kv * pl.m_tiles;
  const long long target = 2LL * (sms > 0 ? sms : 148);
  const int kv = max_kv > 0 ? max_kv : 1;
  int chunk = ((kv + simt::BN - 1) / simt::BN) * simt::BN;
  int n_split = 1;
  while (base * n_split < target && chunk > 4 * simt::BN) {
    n_split *= 2;
    chunk = (((kv + n_split - 1) / n_split + simt::BN - 1) / simt::BN) * simt::BN;
  }
  n_split = (kv + chunk - 1) / chunk;
  pl.n_split = n_split;
  pl.chunk = chunk;
  pl.ws_bytes = n_split > 1 ? (size_t)n_split * total_q * H_q * (D + 2) * sizeof(float) : 0;
  return pl;
}

template <typename T>
int launch_simt(AttnParams& p, const SimtPlan& pl, cudaStream_t st) {
  p.n_split = pl.n_split;
  p.chunk = pl.chunk;
  p.m_tiles = pl.m_tiles;
  p.W = pl.W;
  dim3 grid(pl.m_tiles, p.B * p.H_kv, pl.n_split);
  if (p.D == 128) {
    const size_t smem = simt::smem_bytes<128>(pl.W);
    cudaFuncSetAttribute(attn_simt_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_simt_kernel<T, 128><<<grid, simt::NT, smem, st>>>(p);
  } else {
    const size_t smem = simt::smem_bytes<64>(pl.W);
    cudaFuncSetAttribute(attn_simt_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_simt_kernel<T, 64><<<grid, simt::NT, smem, st>>>(p);
  }
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  if (pl.n_split > 1) {
    const long long warps = (long long)p.total_q * p.H_q;
    const int blocks = (int)((warps * 32 + 255) / 256);
    attn_combine_kernel<T><<<blocks, 256, 0, st>>>(p);
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  }
  return CAST_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- tensor-core path ---------------------------------------------------------
// Launch plan: 256-row blocks of each (sequence, KV head); the key range is
// split only when the grid would not hold two CTAs per SM (measured: four per
// SM split configuration 2's 16 sequences in two for 99.5 us a call against 74
// us unsplit, with no change on configurations 3 and 4).
struct TcPlan {
  int m_blocks, n_split, chunk, W;
  size_t ws_bytes;
};

TcPlan plan_tc(int B, int total_q, int H_q, int H_kv, int max_pack, int max_kv, int sms) {
  TcPlan pl;
  const int G = H_q / H_kv;
  pl.m_blocks = (G * max_pack + tca::QT * tca::BM - 1) / (tca::QT * tca::BM);
  if (pl.m_blocks < 1) pl.m_blocks = 1;
  pl.W = (max_pack + 63) / 64;
  if (pl.W < 1) pl.W = 1;
  const long long base = (long long)B * H_kv * pl.m_blocks;
  const long long target = 2LL * (sms > 0 ? sms : 148);
  const int kv = max_kv > 0 ? max_kv : 1;
  int chunk = ((kv + tca::BN - 1) / tca::BN) * tca::BN;
  int n_split = 1;
  while (base * n_split < target && chunk > 16 * tca::BN) {
    n_split *= 2;
    chunk = (((kv + n_split - 1) / n_split + tca::BN - 1) / tca::BN) * tca::BN;
  }
  n_split = (kv + chunk - 1) / chunk;
  pl.n_split = n_split;
  pl.chunk = chunk;
  pl.ws_bytes = n_split > 1 ? (size_t)n_split * total_q * H_q * (tca::D + 2) * sizeof(float) : 0;
  return pl;
}

// Store layout: key tiles per sequence are ceil(S/128) + ceil(P/128); plan on
// that tile count (chunks stay whole numbers of tiles).
TcPlan plan_tc_store(int B, int total_q, int H_q, int H_kv, int max_pack, int max_prefix, int sms) {
  const int tiles = (max_prefix + tca::BN - 1) / tca::BN + (max_pack + tca::BN - 1) / tca::BN;
  return plan_tc(B, total_q, H_q, H_kv, max_pack, tiles * tca::BN, sms);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load(std::memory_order_acquire);
  if (f) return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || f == nullptr)
    return nullptr;
  fn.store(f, std::memory_order_release);
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// 3-D map over a [rows, heads, 128] 16-bit tensor: box = 64 dims x `box_heads` x `box_rows`, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int dtype, int64_t rows, int heads, int64_t s_row, int64_t s_head,
              int box_heads, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)s_head * 2, (cuuint64_t)s_row * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_heads, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == CAST_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor-core kernel takes 16-bit inputs with D = 128, G dividing 128,
// 16-byte aligned bases and row/head strides that are multiples of 8 elements.
bool tc_eligible(int dtype, int D, int G, const int64_t* st, const void* q, const void* k, const void* v,
                 const void* out) {
  if (dtype == CAST_F32 || D != 128 || G < 1 || 128 % G != 0) return false;
  for (int t = 0; t < 4; ++t)
    if (st[3 * t] % 8 != 0 || st[3 * t + 1] % 8 != 0 || st[3 * t + 2] != 1) return false;
  return aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16);
}

// 4-D map over a per-request store [batch, heads, rows, 128] (strides in elements,
// dim stride 1): box = 64 dims x 128 rows of one head of one request, 128-byte swizzle.
bool make_store_map(CUtensorMap* map, const void* base, int dtype, int batch, int heads, int64_t rows, int64_t s_b,
                    int64_t s_h, int64_t s_r) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {128, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)s_r * 2, (cuuint64_t)s_h * 2, (cuuint64_t)s_b * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)tca::BN, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == CAST_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool STORE>
int launch_tc_maps(AttnParams& p, const TcPlan& pl, int dtype, cudaStream_t st, const CUtensorMap& mq,
                   const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mkp, const CUtensorMap& mvp,
                   bool combine = true) {
  p.n_split = pl.n_split;
  p.chunk = pl.chunk;
  p.m_tiles = pl.m_blocks;
  p.W = pl.W;
  {
    const long long last = ((long long)p.G * p.max_pack) % (tca::QT * tca::BM);
    p.tail_last = (last > 0 && last <= tca::BM) ? 1 : 0;
  }
  const size_t smem = tca::smem_bytes(p.G, pl.W);
  dim3 grid(p.tail_only ? 1 : pl.m_blocks, p.B * p.H_kv, pl.n_split);
  if (dtype == CAST_BF16) {
    cudaFuncSetAttribute(tca::attn_tc_kernel<true, STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tca::attn_tc_kernel<true, STORE><<<grid, tca::NT, smem, st>>>(p, mq, mk, mv, mkp, mvp);
  } else {
    cudaFuncSetAttribute(tca::attn_tc_kernel<false, STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tca::attn_tc_kernel<false, STORE><<<grid, tca::NT, smem, st>>>(p, mq, mk, mv, mkp, mvp);
  }
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  if (combine && pl.n_split > 1) {
    const long long warps = (long long)p.total_q * p.H_q;
    const int blocks = (int)((warps * 32 + 255) / 256);
    if (dtype == CAST_BF16) attn_combine_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
    else attn_combine_kernel<__half><<<blocks, 256, 0, st>>>(p);
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  }
  return CAST_OK;
}

// ---- fp32 through the tensor cores (three-term bf16 split) --------------------------
// Launch plan: 128-row query tiles (one per CTA); keys split as for the 16-bit kernel.
TcPlan plan_tc3(int B, int total_q, int H_q, int H_kv, int max_pack, int max_kv, int sms) {
  TcPlan pl;
  const int G = H_q / H_kv;
  pl.m_blocks = (G * max_pack + tc3::BM - 1) / tc3::BM;
  if (pl.m_blocks < 1) pl.m_blocks = 1;
  pl.W = (max_pack + 63) / 64;
  if (pl.W < 1) pl.W = 1;
  const long long base = (long long)B * H_kv * pl.m_blocks;
  const long long target = 4LL * (sms > 0 ? sms : 148);
  const int kv = max_kv > 0 ? max_kv : 1;
  int chunk = ((kv + tc3::BN - 1) / tc3::BN) * tc3::BN;
  int n_split = 1;
  while (base * n_split < target && chunk > 16 * tc3::BN) {
    n_split *= 2;
    chunk = (((kv + n_split - 1) / n_split + tc3::BN - 1) / tc3::BN) * tc3::BN;
  }
  n_split = (kv + chunk - 1) / chunk;
  pl.n_split = n_split;
  pl.chunk = chunk;
  pl.ws_bytes = n_split > 1 ? (size_t)n_split * total_q * H_q * (tc3::D + 2) * sizeof(float) : 0;
  return pl;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace of the split path: [partials][q hi][q lo][k hi][k lo][v hi][v lo][flags].
struct Split3Layout {
  size_t part, q_hi, q_lo, k_hi, k_lo, v_hi, v_lo, flags, total;
};
Split3Layout split3_layout(size_t part_bytes, long long total_q, long long total_kv, int H_q, int H_kv) {
  Split3Layout w;
  const size_t qb = align256((size_t)total_q * H_q * 128 * 2), kb = align256((size_t)total_kv * H_kv * 128 * 2);
  w.part = 0;
  w.q_hi = align256(part_bytes);
  w.q_lo = w.q_hi + qb;
  w.k_hi = w.q_lo + qb;
  w.k_lo = w.k_hi + kb;
  w.v_hi = w.k_lo + kb;
  w.v_lo = w.v_hi + kb;
  w.flags = w.v_lo + kb;
  w.total = w.flags + 256;
  return w;
}

// Split sources of the regular layout: q, k and v read as [rows, heads, 128].
tc3::SplitArgs plain_split_args(const AttnParams& p, const Split3Layout& lay, char* ws) {
  auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
  tc3::SplitArgs sa{};
  sa.t[0] = {static_cast<const float*>(p.q), p.total_q, p.sq_m, p.sq_h, p.H_q, bf(lay.q_hi), bf(lay.q_lo)};
  sa.t[1] = {static_cast<const float*>(p.k), p.total_kv, p.sk_m, p.sk_h, p.H_kv, bf(lay.k_hi), bf(lay.k_lo)};
  sa.t[2] = {static_cast<const float*>(p.v), p.total_kv, p.sv_m, p.sv_h, p.H_kv, bf(lay.v_hi), bf(lay.v_lo)};
  return sa;
}

// Split pass then the attention kernel (and the combine when the keys are split). p describes
// the ragged layout the hi / lo copies are in (p.cu_kv, p.total_kv rows).
int launch_tc3(AttnParams& p, const TcPlan& pl, const Split3Layout& lay, char* ws, tc3::SplitArgs sa, int sms,
               cudaStream_t st) {
  int* flags = reinterpret_cast<int*>(ws + lay.flags);
  if (cudaMemsetAsync(flags, 0, 16, st) != cudaSuccess) return CAST_ERR_LAUNCH;
  sa.flags = flags;
  const long long n4 = std::max((long long)p.total_q * p.H_q, (long long)p.total_kv * p.H_kv) * 32;
  const unsigned gx = (unsigned)std::max(1LL, std::min((n4 + 255) / 256, 8LL * (sms > 0 ? sms : 148)));
  tc3::split3_kernel<<<dim3(gx, 3), 256, 0, st>>>(sa);
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
  const int G = p.G;
  const int64_t qr = (int64_t)p.H_q * 128, kr = (int64_t)p.H_kv * 128;
  if (!make_map(&mqh, ws + lay.q_hi, CAST_BF16, p.total_q, p.H_q, qr, 128, G, tc3::BM / G) ||
      !make_map(&mql, ws + lay.q_lo, CAST_BF16, p.total_q, p.H_q, qr, 128, G, tc3::BM / G) ||
      !make_map(&mkh, ws + lay.k_hi, CAST_BF16, p.total_kv, p.H_kv, kr, 128, 1, tc3::BN) ||
      !make_map(&mkl, ws + lay.k_lo, CAST_BF16, p.total_kv, p.H_kv, kr, 128, 1, tc3::BN) ||
      !make_map(&mvh, ws + lay.v_hi, CAST_BF16, p.total_kv, p.H_kv, kr, 128, 1, tc3::BN) ||
      !make_map(&mvl, ws + lay.v_lo, CAST_BF16, p.total_kv, p.H_kv, kr, 128, 1, tc3::BN))
    return CAST_ERR_LAUNCH;
  p.split_flags = flags;
  p.n_split = pl.n_split;
  p.chunk = pl.chunk;
  p.m_tiles = pl.m_blocks;
  p.W = pl.W;
  const size_t smem = tc3::smem_bytes(G, pl.W);
  cudaFuncSetAttribute(tc3::attn_tc3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  tc3::attn_tc3_kernel<<<dim3(pl.m_blocks, p.B * p.H_kv, pl.n_split), tc3::NT, smem, st>>>(p, mqh, mql, mkh, mkl,
                                                                                           mvh, mvl);
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  if (pl.n_split > 1) {
    const long long warps = (long long)p.total_q * p.H_q;
    attn_combine_kernel<float><<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(p);
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  }
  return CAST_OK;
}

bool split3_strides_ok(const int64_t* st, const void* q, const void* k, const void* v, const void* out) {
  for (int t = 0; t < 4; ++t)
    if (st[3 * t + 2] != 1 || st[3 * t] % 4 != 0 || st[3 * t + 1] % 4 != 0) return false;
  return aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16);
}

int launch_tc(AttnParams& p, const TcPlan& pl, int dtype, cudaStream_t st, bool combine = true) {
  CUtensorMap mq, mk, mv;
  const int G = p.G;
  if (!make_map(&mq, p.q, dtype, p.total_q, p.H_q, p.sq_m, p.sq_h, G, tca::BM / G) ||
      !make_map(&mk, p.k, dtype, p.total_kv, p.H_kv, p.sk_m, p.sk_h, 1, tca::BN) ||
      !make_map(&mv, p.v, dtype, p.total_kv, p.H_kv, p.sv_m, p.sv_h, 1, tca::BN))
    return CAST_ERR_LAUNCH;
  return launch_tc_maps<false>(p, pl, dtype, st, mq, mk, mv, mk, mv, combine);
}

// CTA-pair kernel: a cluster of two CTAs per 256-row block; K tiles arrive in 64-key halves (one
// per CTA of the pair), V tiles in 64-dim halves of all 128 keys.
bool pair_fits(int G, int W) {
  constexpr size_t kMaxSmem = 227 * 1024 - 8 * 1024;   // the kernel's static shared memory takes the rest
  return tcp::smem_bytes(tcp::NST, G, W) <= kMaxSmem;
}

int launch_pair(AttnParams& p, const TcPlan& pl, int dtype, cudaStream_t st, bool combine = true) {
  CUtensorMap mq, mk, mv;
  const int G = p.G;
  if (!make_map(&mq, p.q, dtype, p.total_q, p.H_q, p.sq_m, p.sq_h, G, tcp::BM / G) ||
      !make_map(&mk, p.k, dtype, p.total_kv, p.H_kv, p.sk_m, p.sk_h, 1, tcp::BN / 2) ||
      !make_map(&mv, p.v, dtype, p.total_kv, p.H_kv, p.sv_m, p.sv_h, 1, tcp::BN))
    return CAST_ERR_LAUNCH;
  p.n_split = pl.n_split;
  p.chunk = pl.chunk;
  p.m_tiles = pl.m_blocks;
  p.W = pl.W;
  constexpr size_t kMaxSmem = 227 * 1024 - 8 * 1024;   // the kernel's static shared memory takes the rest
  const size_t smem = tcp::smem_bytes(tcp::NST, G, pl.W);
  if (smem > kMaxSmem) return CAST_ERR_PACK;
  dim3 grid(2 * pl.m_blocks, p.B * p.H_kv, pl.n_split);
  auto go = [&](auto bf16_c, auto nst_c) {
    auto kern = tcp::attn_pair_kernel<decltype(bf16_c)::value, decltype(nst_c)::value>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, tcp::NT, smem, st>>>(p, mq, mk, mv);
  };
  if (dtype == CAST_BF16) go(std::true_type{}, std::integral_constant<int, tcp::NST>{});
  else go(std::false_type{}, std::integral_constant<int, tcp::NST>{});
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  if (combine && pl.n_split > 1) {
    const long long warps = (long long)p.total_q * p.H_q;
    const int blocks = (int)((warps * 32 + 255) / 256);
    if (dtype == CAST_BF16) attn_combine_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
    else attn_combine_kernel<__half><<<blocks, 256, 0, st>>>(p);
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  }
  return CAST_OK;
}


}  // namespace
}  // namespace cast

using namespace cast;

// Scratch of cast_tree_attn_fwd_noalloc: one fixed array per device, part of
// the library image, so that entry point never allocates. In host code this
// name is only a stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress, looked up once per device by noalloc_scratch().
static __device__ __align__(256) unsigned char g_noalloc_scratch[CAST_NOALLOC_SCRATCH_BYTES];

namespace cast {
namespace {
// Per device: the context the cached address belongs to, and the address.
struct NoallocSlot {
  std::mutex mu;
  CUcontext ctx = nullptr;
  void* ptr = nullptr;
};
NoallocSlot g_noalloc[kMaxDevices];

PFN_cuCtxGetCurrent_v4000 ctx_get_current() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load(std::memory_order_acquire);
  if (f) return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || f == nullptr)
    return nullptr;
  fn.store(f, std::memory_order_release);
  return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
}

// Device address of g_noalloc_scratch on the current device (nullptr on failure).
// The address is looked up once per context: a device reset (cudaDeviceReset)
// destroys the context and the library's module with it, so a call after a reset
// sees a new current context and looks the address up again in it.
void* noalloc_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  auto get_ctx = ctx_get_current();
  if (!get_ctx) return nullptr;
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return nullptr;
  NoallocSlot& slot = g_noalloc[dev];
  std::lock_guard<std::mutex> lock(slot.mu);
  if (ctx != nullptr && slot.ptr != nullptr && slot.ctx == ctx) return slot.ptr;
  // (no current context yet: the lookup below makes the device's primary context current)
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    return nullptr;
  }
  if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return nullptr;
  slot.ctx = ctx;
  slot.ptr = ptr;
  return ptr;
}
}  // namespace
}  // namespace cast

extern "C" {

const char* cast_strerror(int status) {
  switch (status) {
    case CAST_OK: return "ok";
    case CAST_ERR_NULL: return "a required pointer is NULL";
    case CAST_ERR_SHAPE: return "invalid shape (non-positive size, or H_q not a multiple of H_kv)";
    case CAST_ERR_DTYPE: return "unsupported dtype (expected float32, bfloat16 or float16)";
    case CAST_ERR_HEAD_DIM: return "unsupported head dim (expected 64 or 128)";
    case CAST_ERR_PACK: return "pack too large (max_pack above CAST_MAX_PACK) or too few ancestor words per row";
    case CAST_ERR_WORKSPACE: return "workspace smaller than cast_tree_attn_workspace_size() (CAST_F32_SPLIT: _size_kv(), 256-byte aligned)";
    case CAST_ERR_ALIGN: return "misaligned pointer or stride (base 16-byte aligned, row/head strides multiples of 4 elements, dim stride 1)";
    case CAST_ERR_TOPK: return "k out of range (1 <= k <= CAST_MAX_TOPK, k <= V) or L out of range";
    case CAST_ERR_LAUNCH: return "CUDA launch failed";
    case CAST_ERR_DEVICE: return "no usable CUDA device";
    case CAST_ERR_MASK_MODE: return "pass exactly one of anc_words and parent";
    case CAST_ERR_SCRATCH_LIMIT: return "problem needs more scratch than the no-alloc entry point's fixed array (CAST_NOALLOC_SCRATCH_BYTES); use cast_tree_attn_fwd with a workspace";
    case CAST_DEV_BAD_LAYOUT: return "device: cu_q/cu_kv/prefix_len/pack_len out of range or above max_pack/max_kv";
    case CAST_DEV_BAD_PARENT: return "device: parent array is not a forest in pack order (need -1 <= parent[i] < i, parent[0] = -1)";
    case CAST_DEV_TIMEOUT: return "device: a bounded wait gave up";
    case CAST_DEV_TREE_OVERFLOW: return "device: budget above max_budget, or an accepted path longer than path_cap";
    default: return "unknown status";
  }
}

int cast_version(void) { return 100; }

void cast_test_set_wait_limit_ns(uint64_t ns) {
  g_pipeline_wait_ns.store(ns == 0 ? tc::kWaitLimitNs : ns, std::memory_order_relaxed);
}

void cast_test_set_tc_kernel(int kernel) {
  g_tc_kernel.store(kernel < 0 ? -1 : (kernel == 0 ? 0 : 1), std::memory_order_relaxed);
}

int cast_device_error(cast_stream_t stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(&h, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return CAST_ERR_LAUNCH;
  if (cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return CAST_ERR_LAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return CAST_ERR_LAUNCH;
  return h;
}

size_t cast_tree_attn_workspace_size_kv(int dtype, int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                                        int max_pack, int max_kv) {
  if (dtype != CAST_F32_SPLIT)
    return cast_tree_attn_workspace_size(dtype, B, total_q, H_q, H_kv, D, max_pack, max_kv);
  if (B <= 0 || total_q <= 0 || total_kv < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0 || D != 128) return 0;
  const TcPlan tp = plan_tc3(B, total_q, H_q, H_kv, max_pack, max_kv, sm_count());
  return split3_layout(tp.ws_bytes, total_q, total_kv, H_q, H_kv).total;
}

size_t cast_tree_attn_workspace_size(int dtype, int B, int total_q, int H_q, int H_kv, int D,
                                     int max_pack, int max_kv) {
  if (B <= 0 || total_q <= 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0) return 0;
  if (dtype == CAST_F32_SPLIT)
    return cast_tree_attn_workspace_size_kv(dtype, B, total_q, (int)std::min<long long>((long long)B * max_kv, 0x7fffffffLL),
                                            H_q, H_kv, D, max_pack, max_kv);
  const int sms = sm_count();
  const SimtPlan pl = plan_simt(B, total_q, H_q, H_kv, D, max_pack, max_kv, sms);
  size_t ws = pl.ws_bytes;
  if (dtype != CAST_F32 && D == 128) {
    const TcPlan tp = plan_tc(B, total_q, H_q, H_kv, max_pack, max_kv, sms);
    if (tp.ws_bytes > ws) ws = tp.ws_bytes;
  }
  return ws;
}

int cast_tree_attn_plan(int dtype, int B, int total_q, int H_q, int H_kv, int D, int max_pack, int max_kv,
                        const int64_t* strides, const void* q, const void* k, const void* v, const void* out,
                        int* plan) {
  if (!strides || !plan) return CAST_ERR_NULL;
  if (dtype != CAST_F32 && dtype != CAST_BF16 && dtype != CAST_F16 && dtype != CAST_F32_SPLIT) return CAST_ERR_DTYPE;
  if (B < 0 || total_q < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0) return CAST_ERR_SHAPE;
  if (D != 64 && D != 128) return CAST_ERR_HEAD_DIM;
  const int sms = sm_count();
  if (dtype == CAST_F32_SPLIT) {
    if (D != 128 || 128 % (H_q / H_kv) != 0) return CAST_ERR_HEAD_DIM;
    if (!split3_strides_ok(strides, q, k, v, out)) return CAST_ERR_ALIGN;
    const TcPlan tp = plan_tc3(B, total_q, H_q, H_kv, max_pack, max_kv, sms);
    plan[0] = 2;
    plan[1] = tp.n_split;
    plan[2] = tp.n_split > 1 ? 3 : 2;
    return CAST_OK;
  }
  if (tc_eligible(dtype, D, H_q / H_kv, strides, q, k, v, out) && g_tc_kernel.load(std::memory_order_relaxed) >= 0) {
    const TcPlan tp = plan_tc(B, total_q, H_q, H_kv, max_pack, max_kv, sms);
    plan[0] = 1;
    plan[1] = tp.n_split;
  } else {
    const SimtPlan sp = plan_simt(B, total_q, H_q, H_kv, D, max_pack, max_kv, sms);
    plan[0] = 0;
    plan[1] = sp.n_split;
  }
  plan[2] = plan[1] > 1 ? 2 : 1;
  return CAST_OK;
}

int cast_tree_attn_fwd(const void* q, const void* k, const void* v, void* out, int dtype,
                       const int64_t* strides,
                       const int32_t* cu_q, const int32_t* cu_kv,
                       const int32_t* prefix_len, const int32_t* pack_len,
                       const int64_t* anc_words, int anc_words_per_row,
                       const int32_t* parent,
                       int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                       float sm_scale, int max_pack, int max_kv,
                       void* workspace, size_t workspace_bytes, cast_stream_t stream) {
  if (dtype != CAST_F32 && dtype != CAST_BF16 && dtype != CAST_F16 && dtype != CAST_F32_SPLIT) return CAST_ERR_DTYPE;
  if (B < 0 || total_q < 0 || total_kv < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0 || max_pack < 0 ||
      max_kv < 0)
    return CAST_ERR_SHAPE;
  if (D != 64 && D != 128) return CAST_ERR_HEAD_DIM;
  if (dtype == CAST_F32_SPLIT && (D != 128 || 128 % (H_q / H_kv) != 0)) return CAST_ERR_HEAD_DIM;
  if (max_pack > CAST_MAX_PACK) return CAST_ERR_PACK;
  if (B == 0 || total_q == 0 || max_pack == 0) return CAST_OK;  // nothing to compute
  if (!q || !k || !v || !out || !strides || !cu_q || !cu_kv || !prefix_len || !pack_len) return CAST_ERR_NULL;
  if ((anc_words == nullptr) == (parent == nullptr)) return CAST_ERR_MASK_MODE;
  if (anc_words && anc_words_per_row < 1) return CAST_ERR_PACK;
  for (int t = 0; t < 4; ++t) {
    if (strides[3 * t + 2] != 1) return CAST_ERR_ALIGN;
    if (strides[3 * t + 0] % 4 != 0 || strides[3 * t + 1] % 4 != 0) return CAST_ERR_ALIGN;
  }
  const size_t ab = 16;
  if (!aligned(q, ab) || !aligned(k, ab) || !aligned(v, ab) || !aligned(out, ab)) return CAST_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return CAST_ERR_DEVICE;

  AttnParams p{};
  p.q = q; p.k = k; p.v = v; p.out = out;
  p.sq_m = strides[0]; p.sq_h = strides[1];
  p.sk_m = strides[3]; p.sk_h = strides[4];
  p.sv_m = strides[6]; p.sv_h = strides[7];
  p.so_m = strides[9]; p.so_h = strides[10];
  p.cu_q = cu_q; p.cu_kv = cu_kv; p.prefix_len = prefix_len; p.pack_len = pack_len;
  p.anc_words = anc_words; p.anc_wpr = anc_words_per_row; p.parent = parent;
  p.B = B; p.total_q = total_q; p.total_kv = total_kv; p.H_q = H_q; p.H_kv = H_kv; p.G = H_q / H_kv; p.D = D;
  const float scale = sm_scale > 0.f ? sm_scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = scale * kLog2e;
  p.max_pack = max_pack; p.max_kv = max_kv;
  p.wait_ns = g_pipeline_wait_ns.load(std::memory_order_relaxed);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == CAST_F32_SPLIT) {
    if (!split3_strides_ok(strides, q, k, v, out)) return CAST_ERR_ALIGN;
    const TcPlan tp = plan_tc3(B, total_q, H_q, H_kv, max_pack, max_kv, sms);
    const Split3Layout lay = split3_layout(tp.ws_bytes, total_q, total_kv, H_q, H_kv);
    if (!workspace || workspace_bytes < lay.total || !aligned(workspace, 256)) return CAST_ERR_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    if (tp.ws_bytes > 0) {
      p.ws_o = reinterpret_cast<float*>(ws);
      p.ws_ml = p.ws_o + (size_t)tp.n_split * total_q * H_q * D;
    }
    return launch_tc3(p, tp, lay, ws, plain_split_args(p, lay, ws), sms, st);
  }
  if (tc_eligible(dtype, D, p.G, strides, q, k, v, out) && g_tc_kernel.load(std::memory_order_relaxed) >= 0) {
    const TcPlan tp = plan_tc(B, total_q, H_q, H_kv, max_pack, max_kv, sms);
    if (tp.ws_bytes > 0) {
      if (!workspace || workspace_bytes < tp.ws_bytes || !aligned(workspace, 16)) return CAST_ERR_WORKSPACE;
      p.ws_o = static_cast<float*>(workspace);
      p.ws_ml = p.ws_o + (size_t)tp.n_split * total_q * H_q * D;
    }
    // CTA pairs run the head groups' full 256-row blocks; a pair whose second CTA has few or no rows
    // would stream every key tile on two SMs, so partial blocks go to the single-CTA kernel. When the
    // largest head group fills whole pairs (G * max_pack a multiple of 256 rows) the pair kernel runs
    // everything (a shorter group's partial block included). When it is longer than one pair, ends in
    // a one-tile block and the units are long (key chunks of 64 tiles or more), the pair launch takes
    // the full blocks and a single-CTA launch the partial last blocks, then the combine (if the keys
    // are split) runs over both: configuration 4 714 -> 689 us, configuration 5 at N = 64, 128, 256
    // 3-4 % faster. With short units (configuration 2: 74 -> 104 us) or a two-tile last block
    // (configuration 5 at N = 96: 3 % slower) the two launches' tails cost more than the pairs save.
    const long long gmp = (long long)p.G * max_pack;
    const long long last = gmp % (tca::QT * tca::BM);
    const bool pairs_on = g_tc_kernel.load(std::memory_order_relaxed) != 0 && pair_fits(p.G, tp.W);
    if (pairs_on && last == 0) return launch_pair(p, tp, dtype, st);
    if (pairs_on && gmp > tca::QT * tca::BM && last <= tca::BM && tp.chunk >= 64 * tca::BN) {
      AttnParams pp = p;
      pp.pair_full_only = 1;
      const int rc = launch_pair(pp, tp, dtype, st, false);
      if (rc != CAST_OK) return rc;
      AttnParams ps = p;
      ps.tail_only = 1;
      return launch_tc(ps, tp, dtype, st);
    }
    return launch_tc(p, tp, dtype, st);
  }
  const SimtPlan pl = plan_simt(B, total_q, H_q, H_kv, D, max_pack, max_kv, sms);
  if (pl.ws_bytes > 0) {
    if (!workspace || workspace_bytes < pl.ws_bytes || !aligned(workspace, 16)) return CAST_ERR_WORKSPACE;
    p.ws_o = static_cast<float*>(workspace);
    p.ws_ml = p.ws_o + (size_t)pl.n_split * total_q * H_q * D;
  }
  switch (dtype) {
    case CAST_F32: return launch_simt<float>(p, pl, st);
    case CAST_BF16: return launch_simt<__nv_bfloat16>(p, pl, st);
    default: return launch_simt<__half>(p, pl, st);
  }
}

int cast_tree_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* out, int dtype,
                               const int64_t* strides,
                               const int32_t* cu_q, const int32_t* cu_kv,
                               const int32_t* prefix_len, const int32_t* pack_len,
                               const int64_t* anc_words, int anc_words_per_row,
                               const int32_t* parent,
                               int B, int total_q, int total_kv, int H_q, int H_kv, int D,
                               float sm_scale, int max_pack, int max_kv, cast_stream_t stream) {
  // Same checks and launches as cast_tree_attn_fwd; only the scratch differs.
  const size_t need = cast_tree_attn_workspace_size(dtype, B, total_q, H_q, H_kv, D, max_pack, max_kv);
  if (need > (size_t)CAST_NOALLOC_SCRATCH_BYTES) return CAST_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    scratch = noalloc_scratch();
    if (scratch == nullptr) return CAST_ERR_DEVICE;
  }
  return cast_tree_attn_fwd(q, k, v, out, dtype, strides, cu_q, cu_kv, prefix_len, pack_len, anc_words,
                            anc_words_per_row, parent, B, total_q, total_kv, H_q, H_kv, D, sm_scale, max_pack,
                            max_kv, scratch, need > 0 ? (size_t)CAST_NOALLOC_SCRATCH_BYTES : 0, stream);
}

size_t cast_tree_attn_store_workspace_size(int dtype, int B, int total_q, int H_q, int H_kv, int D, int max_pack,
                                           int max_prefix) {
  if (dtype == CAST_F32 || D != 128 || B <= 0 || total_q <= 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0) return 0;
  if (dtype == CAST_F32_SPLIT) {
    const long long rows_cap = (long long)B * ((long long)max_prefix + max_pack);
    const TcPlan tp = plan_tc3(B, total_q, H_q, H_kv, max_pack, max_prefix + max_pack, sm_count());
    return align256((size_t)(B + 1) * sizeof(int32_t)) + split3_layout(tp.ws_bytes, total_q, rows_cap, H_q, H_kv).total;
  }
  return plan_tc_store(B, total_q, H_q, H_kv, max_pack, max_prefix, sm_count()).ws_bytes;
}

int cast_tree_attn_store_fwd(const void* q, const void* k_store, const void* v_store, const void* k_pack,
                             const void* v_pack, void* out, int dtype, const int64_t* strides,
                             const int32_t* cu_q, const int32_t* prefix_len, const int32_t* pack_len,
                             const int64_t* anc_words, int anc_words_per_row, const int32_t* parent,
                             int B, int total_q, int store_batch, int store_rows, int H_q, int H_kv, int D,
                             float sm_scale, int max_pack, int max_prefix,
                             void* workspace, size_t workspace_bytes, cast_stream_t stream) {
  if (dtype != CAST_BF16 && dtype != CAST_F16 && dtype != CAST_F32_SPLIT) return CAST_ERR_DTYPE;
  if (B < 0 || total_q < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0 || max_pack < 0 || max_prefix < 0 ||
      store_batch < 0 || store_rows < 0)
    return CAST_ERR_SHAPE;
  if (D != 128) return CAST_ERR_HEAD_DIM;
  if (max_pack > CAST_MAX_PACK) return CAST_ERR_PACK;
  if (B == 0 || total_q == 0 || max_pack == 0) return CAST_OK;
  if (!q || !k_store || !v_store || !k_pack || !v_pack || !out || !strides || !cu_q || !prefix_len || !pack_len)
    return CAST_ERR_NULL;
  if ((anc_words == nullptr) == (parent == nullptr)) return CAST_ERR_MASK_MODE;
  if (anc_words && anc_words_per_row < 1) return CAST_ERR_PACK;
  if (store_batch < B || (max_prefix > 0 && store_rows < 1)) return CAST_ERR_SHAPE;
  const int G = H_q / H_kv;
  if (G < 1 || 128 % G != 0) return CAST_ERR_SHAPE;
  // strides: q (3), k_store (4), v_store (4), k_pack (3), v_pack (3), out (3); dims innermost last
  const int64_t* sq = strides;
  const int64_t* sks = strides + 3;
  const int64_t* svs = strides + 7;
  const int64_t* skp = strides + 11;
  const int64_t* svp = strides + 14;
  const int64_t* so = strides + 17;
  const int sm = dtype == CAST_F32_SPLIT ? 4 : 8;   // stride multiple: 16 bytes either way
  for (const int64_t* t3 : {sq, skp, svp, so})
    if (t3[2] != 1 || t3[0] % sm != 0 || t3[1] % sm != 0) return CAST_ERR_ALIGN;
  for (const int64_t* t4 : {sks, svs})
    if (t4[3] != 1 || t4[0] % sm != 0 || t4[1] % sm != 0 || t4[2] % sm != 0) return CAST_ERR_ALIGN;
  if (!aligned(q, 16) || !aligned(k_store, 16) || !aligned(v_store, 16) || !aligned(k_pack, 16) ||
      !aligned(v_pack, 16) || !aligned(out, 16))
    return CAST_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return CAST_ERR_DEVICE;

  AttnParams p{};
  p.q = q; p.k = k_pack; p.v = v_pack; p.out = out;
  p.sq_m = sq[0]; p.sq_h = sq[1];
  p.sk_m = skp[0]; p.sk_h = skp[1];
  p.sv_m = svp[0]; p.sv_h = svp[1];
  p.so_m = so[0]; p.so_h = so[1];
  p.cu_q = cu_q; p.cu_kv = nullptr; p.prefix_len = prefix_len; p.pack_len = pack_len;
  p.anc_words = anc_words; p.anc_wpr = anc_words_per_row; p.parent = parent;
  p.B = B; p.total_q = total_q; p.total_kv = 0; p.H_q = H_q; p.H_kv = H_kv; p.G = G; p.D = D;
  const float scale = sm_scale > 0.f ? sm_scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = scale * kLog2e;
  p.max_pack = max_pack; p.max_kv = max_prefix + max_pack;
  p.store_mode = 1; p.store_rows = store_rows; p.store_batch = store_batch;
  p.wait_ns = g_pipeline_wait_ns.load(std::memory_order_relaxed);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (dtype == CAST_F32_SPLIT) {
    // fp32: the split pass reads each prefix from its store and the pack rows from the pack
    // tensors and writes the hi / lo copies in the ragged layout (cu_kv from a scan of the
    // lengths, rows_cap = B * (max_prefix + max_pack) rows, unused rows zero); the attention
    // kernel then runs on that layout.
    const long long rows_cap = (long long)B * ((long long)max_prefix + max_pack);
    if (rows_cap > 0x7fffffffLL) return CAST_ERR_SHAPE;
    const TcPlan tp = plan_tc3(B, total_q, H_q, H_kv, max_pack, max_prefix + max_pack, sms);
    const size_t cu_bytes = align256((size_t)(B + 1) * sizeof(int32_t));
    const Split3Layout lay = split3_layout(tp.ws_bytes, total_q, rows_cap, H_q, H_kv);
    if (!workspace || workspace_bytes < cu_bytes + lay.total || !aligned(workspace, 256)) return CAST_ERR_WORKSPACE;
    int32_t* cu_kv = static_cast<int32_t*>(workspace);
    char* ws = static_cast<char*>(workspace) + cu_bytes;
    tc3::cu_kv_scan_kernel<<<1, 1024, 0, st>>>(prefix_len, pack_len, B, cu_kv);
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
    p.store_mode = 0;
    p.cu_kv = cu_kv;
    p.total_kv = (int)rows_cap;
    if (tp.ws_bytes > 0) {
      p.ws_o = reinterpret_cast<float*>(ws);
      p.ws_ml = p.ws_o + (size_t)tp.n_split * total_q * H_q * D;
    }
    tc3::SplitArgs sa{};
    auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
    sa.t[0] = {static_cast<const float*>(q), total_q, sq[0], sq[1], H_q, bf(lay.q_hi), bf(lay.q_lo)};
    const void* stores[2] = {k_store, v_store};
    const void* packs[2] = {k_pack, v_pack};
    const int64_t* sst[2] = {sks, svs};
    const int64_t* spk[2] = {skp, svp};
    const size_t his[2] = {lay.k_hi, lay.v_hi}, los[2] = {lay.k_lo, lay.v_lo};
    for (int kv = 0; kv < 2; ++kv) {
      tc3::SplitSrc& t = sa.t[1 + kv];
      t.src = static_cast<const float*>(stores[kv]);
      t.rows = rows_cap;
      t.s_b = sst[kv][0]; t.s_head = sst[kv][1]; t.s_row = sst[kv][2];
      t.heads = H_kv;
      t.hi = bf(his[kv]); t.lo = bf(los[kv]);
      t.store = 1;
      t.pack = static_cast<const float*>(packs[kv]);
      t.pk_row = spk[kv][0]; t.pk_head = spk[kv][1];
      t.B = B; t.store_rows = store_rows; t.max_pack = max_pack; t.total_q = total_q;
      t.cu_kv = cu_kv; t.cu_q = cu_q; t.prefix_len = prefix_len; t.pack_len = pack_len;
    }
    return launch_tc3(p, tp, lay, ws, sa, sms, st);
  }

  const TcPlan pl = plan_tc_store(B, total_q, H_q, H_kv, max_pack, max_prefix, sms);
  if (pl.ws_bytes > 0) {
    if (!workspace || workspace_bytes < pl.ws_bytes || !aligned(workspace, 16)) return CAST_ERR_WORKSPACE;
    p.ws_o = static_cast<float*>(workspace);
    p.ws_ml = p.ws_o + (size_t)pl.n_split * total_q * H_q * D;
  }
  CUtensorMap mq, mks, mvs, mkp, mvp;
  if (!make_map(&mq, q, dtype, total_q, H_q, sq[0], sq[1], G, tca::BM / G) ||
      !make_store_map(&mks, k_store, dtype, store_batch, H_kv, store_rows > 0 ? store_rows : 1, sks[0], sks[1], sks[2]) ||
      !make_store_map(&mvs, v_store, dtype, store_batch, H_kv, store_rows > 0 ? store_rows : 1, svs[0], svs[1], svs[2]) ||
      !make_map(&mkp, k_pack, dtype, total_q, H_kv, skp[0], skp[1], 1, tca::BN) ||
      !make_map(&mvp, v_pack, dtype, total_q, H_kv, svp[0], svp[1], 1, tca::BN))
    return CAST_ERR_LAUNCH;
  return launch_tc_maps<true>(p, pl, dtype, st, mq, mks, mvs, mkp, mvp);
}

int cast_kv_ragged_gather(const void* k_store, const void* v_store, const void* k_pack, const void* v_pack,
                          int elem_bytes, const int64_t* strides, const int32_t* cu_q, const int32_t* prefix_len,
                          const int32_t* pack_len, int B, int total_q, int store_batch, int store_rows, int H, int D,
                          int max_pack, int64_t rows_cap, void* k_out, void* v_out, int32_t* cu_kv_out,
                          cast_stream_t stream) {
  if (elem_bytes != 2 && elem_bytes != 4) return CAST_ERR_DTYPE;
  if (B < 0 || total_q < 0 || store_batch < B || store_rows < 0 || H < 1 || D < 1 || max_pack < 0 || rows_cap < 0)
    return CAST_ERR_SHAPE;
  if (!cu_kv_out) return CAST_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0) return cudaMemsetAsync(cu_kv_out, 0, sizeof(int32_t), st) == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
  if (!k_store || !v_store || !k_pack || !v_pack || !strides || !cu_q || !prefix_len || !pack_len ||
      (rows_cap > 0 && (!k_out || !v_out)))
    return CAST_ERR_NULL;
  // strides: k_store (4), v_store (4), k_pack (3), v_pack (3); dim strides 1
  if (strides[3] != 1 || strides[7] != 1 || strides[10] != 1 || strides[13] != 1) return CAST_ERR_ALIGN;
  tc3::cu_kv_scan_kernel<<<1, 1024, 0, st>>>(prefix_len, pack_len, B, cu_kv_out);
  if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  if (rows_cap == 0) return CAST_OK;
  tc3::GatherArgs a{};
  a.store[0] = k_store; a.store[1] = v_store;
  a.pack[0] = k_pack; a.pack[1] = v_pack;
  a.out[0] = k_out; a.out[1] = v_out;
  for (int kv = 0; kv < 2; ++kv) {
    const int64_t* s4 = strides + 4 * kv;
    const int64_t* s3 = strides + 8 + 3 * kv;
    a.st_b[kv] = s4[0]; a.st_h[kv] = s4[1]; a.st_r[kv] = s4[2];
    a.pk_t[kv] = s3[0]; a.pk_h[kv] = s3[1];
  }
  a.B = B; a.H = H; a.D = D; a.store_rows = store_rows; a.max_pack = max_pack; a.total_q = total_q;
  a.rows_cap = rows_cap; a.cu_kv = cu_kv_out; a.cu_q = cu_q; a.prefix_len = prefix_len; a.pack_len = pack_len;
  const int sms = sm_count();
  const long long warps = rows_cap * H;
  const unsigned gx = (unsigned)std::max(1LL, std::min((warps * 32 + 255) / 256, 16LL * (sms > 0 ? sms : 148)));
  if (elem_bytes == 2) tc3::kv_ragged_gather_kernel<uint16_t><<<dim3(gx, 2), 256, 0, st>>>(a);
  else tc3::kv_ragged_gather_kernel<uint32_t><<<dim3(gx, 2), 256, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
}

int cast_block_topk(const double* logits, int64_t n_rows, int64_t V, int64_t row_stride, int k,
                    int64_t* top_idx, double* top_lp, cast_stream_t stream) {
  if (!logits || !top_idx || !top_lp) return CAST_ERR_NULL;
  if (n_rows < 0 || V <= 0 || row_stride < V || V > 0x7fffffffLL || n_rows > 0x7fffffffLL) return CAST_ERR_SHAPE;
  if (k < 1 || k > CAST_MAX_TOPK || k > V) return CAST_ERR_TOPK;
  if (n_rows == 0) return CAST_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = aligned(logits, 16) && (row_stride % 2 == 0);
  const dim3 grid((unsigned)n_rows);
#define CAST_TOPK_LAUNCH(KC, VEC)                                                                        \
  block_topk_kernel<KC, VEC><<<grid, topk::NT, 0, st>>>(logits, V, row_stride, k, top_idx, top_lp);       \
  block_topk_exact_kernel<KC, VEC><<<grid, topk::NT, 0, st>>>(logits, V, row_stride, k, top_idx, top_lp);
  if (k <= 8) {
    if (vec) { CAST_TOPK_LAUNCH(16, true) } else { CAST_TOPK_LAUNCH(16, false) }
  } else {
    if (vec) { CAST_TOPK_LAUNCH(32, true) } else { CAST_TOPK_LAUNCH(32, false) }
  }
#undef CAST_TOPK_LAUNCH
  return cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
}

int cast_build_tree(const int64_t* top_idx, const double* top_lp, int B, int L, int k_cols, int k,
                    const int32_t* budget, int max_budget,
                    int32_t* token, int32_t* depth, int32_t* parent, double* score, int32_t* count,
                    const int32_t* cu_q, int32_t* pack_parent,
                    const int32_t* root_token, int32_t* pack_token,
                    const int32_t* seq_len, int32_t* pack_pos,
                    cast_stream_t stream) {
  if (!top_idx || !top_lp || !budget || !token || !depth || !parent || !score || !count) return CAST_ERR_NULL;
  if (B < 0 || L < 1 || L > CAST_MAX_DEPTH || k_cols < 1 || max_budget < 0 || max_budget >= CAST_MAX_PACK)
    return CAST_ERR_SHAPE;
  if (k < 1) return CAST_ERR_TOPK;
  if (k > k_cols) k = k_cols;
  if (k > CAST_MAX_TOPK) return CAST_ERR_TOPK;
  if ((pack_token && !root_token) || (pack_pos && !seq_len)) return CAST_ERR_NULL;
  if (!cu_q && (pack_parent || pack_token || pack_pos)) return CAST_ERR_NULL;
  if (B == 0) return CAST_OK;
  TreeArgs a{top_idx, top_lp, B, L, k_cols, k, budget, max_budget, token, depth, parent, score, count,
             cu_q, pack_parent, root_token, pack_token, seq_len, pack_pos};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // candidate sets of up to 256 entries live in registers; larger budgets keep them in shared memory
  const int mb = max_budget > 0 ? max_budget : 1;
  if (mb + 1 <= 256) {
    const size_t smem = tree_reg_smem_bytes(mb, L, k);
    auto kern = mb + 1 <= 128 ? build_tree_reg_kernel<4> : build_tree_reg_kernel<8>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<B, 32, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
  }
  const size_t smem = tree_smem_bytes(mb, L, k);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(build_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  build_tree_kernel<<<B, 32, smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
}

int cast_tree_walk_greedy(const void* logits, int dtype, int64_t row_stride, int V, const int32_t* cu_q,
                          const int32_t* pack_parent, const int32_t* pack_token, int B, int total_q, int path_cap,
                          int32_t* path, int32_t* accepted, int64_t* bonus, int32_t* keep, int64_t* tokens,
                          cast_stream_t stream) {
  if (dtype != CAST_F32 && dtype != CAST_BF16 && dtype != CAST_F16) return CAST_ERR_DTYPE;
  if (B < 0 || total_q < 0 || V < 1 || row_stride < V || path_cap < 1) return CAST_ERR_SHAPE;
  if (B == 0) return CAST_OK;
  if (!logits || !cu_q || !pack_parent || !pack_token || !path || !accepted || !bonus) return CAST_ERR_NULL;
  const int es = dtype == CAST_F32 ? 4 : 2;
  const bool vec = aligned(logits, 16) && (row_stride * es) % 16 == 0;
  const int sms = sm_count();
  if (sms <= 0) return CAST_ERR_DEVICE;
  // one cluster per sequence, wide enough for about two CTAs per SM
  int cs = 1;
  while (cs < 8 && (int64_t)B * cs < 2 * sms) cs *= 2;
  walk::WalkArgs a{logits, row_stride, V, cu_q, pack_parent, pack_token, B, total_q, path_cap,
                   path, accepted, bonus, keep, tokens};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * cs));
  cfg.blockDim = dim3(walk::NT);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
#define CAST_WALK_LAUNCH(T)                                                          \
  switch (cs) {                                                                      \
    case 1: e = cudaLaunchKernelEx(&cfg, walk::tree_walk_kernel<T, 1>, a, vec); break; \
    case 2: e = cudaLaunchKernelEx(&cfg, walk::tree_walk_kernel<T, 2>, a, vec); break; \
    case 4: e = cudaLaunchKernelEx(&cfg, walk::tree_walk_kernel<T, 4>, a, vec); break; \
    default: e = cudaLaunchKernelEx(&cfg, walk::tree_walk_kernel<T, 8>, a, vec); break; \
  }
  if (dtype == CAST_F32) { CAST_WALK_LAUNCH(float) }
  else if (dtype == CAST_BF16) { CAST_WALK_LAUNCH(__nv_bfloat16) }
  else { CAST_WALK_LAUNCH(__half) }
#undef CAST_WALK_LAUNCH
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
}

int cast_select_global_topk(const int32_t* token, const int32_t* depth, const int32_t* parent, const double* score,
                            const int32_t* count, int B, int max_nodes, int64_t total,
                            int32_t* out_token, int32_t* out_depth, int32_t* out_parent, double* out_score,
                            int32_t* out_count, int32_t* cu_q, const int32_t* root_token, const int32_t* seq_len,
                            int32_t* pack_parent, int32_t* pack_token, int32_t* pack_pos, int64_t pack_capacity,
                            cast_stream_t stream) {
  if (B < 0 || max_nodes < 1 || max_nodes > sel::MAX_NODES || B > CAST_MAX_SELECT_TREES) return CAST_ERR_SHAPE;
  if (B == 0) return CAST_OK;
  if (!token || !depth || !parent || !score || !count || !out_token || !out_depth || !out_parent || !out_score ||
      !out_count)
    return CAST_ERR_NULL;
  if ((pack_parent || pack_token || pack_pos) && !cu_q) return CAST_ERR_NULL;
  if ((pack_token && !root_token) || (pack_pos && !seq_len)) return CAST_ERR_NULL;
  if (cu_q && pack_capacity < 0) return CAST_ERR_SHAPE;
  if ((const void*)out_token == token || (const void*)out_depth == depth || (const void*)out_parent == parent ||
      (const void*)out_score == score)
    return CAST_ERR_ALIGN;
  // pooled keys go to shared memory when they fit beside the offset arrays
  const size_t base_smem = (size_t)((3 * B + 1 + 1) & ~1) * sizeof(int);
  const size_t key_smem = (size_t)B * max_nodes * sizeof(uint64_t);
  const int cache_keys = base_smem + key_smem <= sel::MAX_DYN_SMEM ? 1 : 0;
  sel::SelArgs a{token, depth, parent, score, count, B, max_nodes, cache_keys, total, out_token, out_depth,
                 out_parent, out_score, out_count, cu_q, root_token, seq_len, pack_parent, pack_token, pack_pos,
                 pack_capacity};
  const size_t smem = base_smem + (cache_keys ? key_smem : 0);
  // the static arrays already take ~37 KB, so any dynamic size needs the opt-in
  if (cudaFuncSetAttribute(sel::select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return CAST_ERR_LAUNCH;
  sel::select_kernel<<<1, sel::NT, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? CAST_OK : CAST_ERR_LAUNCH;
}

}  // extern "C"

namespace cast {
namespace {
// One row-gather launch per block of up to kvg::MAXL layers.
int kv_gather(int n_layers, const void* const* src_kv, void* const* dst_kv, const void* const* pack_kv,
              int64_t pack_offset_bytes, kvg::KvArgs a, int64_t grid_rows, cudaStream_t st) {
  const bool v16 = a.row_bytes % 16 == 0 && a.src_sb % 16 == 0 && a.src_sh % 16 == 0 && a.src_sr % 16 == 0 &&
                   a.dst_sb % 16 == 0 && a.dst_sh % 16 == 0 && a.dst_sr % 16 == 0 && a.pk_sb % 16 == 0 &&
                   a.pk_sh % 16 == 0 && a.pk_st % 16 == 0 && pack_offset_bytes % 16 == 0;
  const bool v4 = a.row_bytes % 4 == 0 && a.src_sb % 4 == 0 && a.src_sh % 4 == 0 && a.src_sr % 4 == 0 &&
                  a.dst_sb % 4 == 0 && a.dst_sh % 4 == 0 && a.dst_sr % 4 == 0 && a.pk_sb % 4 == 0 &&
                  a.pk_sh % 4 == 0 && a.pk_st % 4 == 0 && pack_offset_bytes % 4 == 0;
  bool p16 = v16, p4 = v4;
  for (int i = 0; i < 2 * n_layers; ++i) {
    for (const void* p : {(const void*)src_kv[i], (const void*)dst_kv[i], (const void*)pack_kv[i]}) {
      p16 = p16 && aligned(p, 16);
      p4 = p4 && aligned(p, 4);
    }
  }
  const unsigned gx = (unsigned)((grid_rows + kvg::ROWS_PER_CTA - 1) / kvg::ROWS_PER_CTA);
  if (gx == 0) return CAST_OK;
  for (int l0 = 0; l0 < n_layers; l0 += kvg::MAXL) {
    const int nl = std::min(kvg::MAXL, n_layers - l0);
    kvg::Layers ly{};
    for (int l = 0; l < nl; ++l)
      for (int kv = 0; kv < 2; ++kv) {
        ly.src[l][kv] = src_kv[2 * (l0 + l) + kv];
        ly.dst[l][kv] = dst_kv[2 * (l0 + l) + kv];
        ly.pack[l][kv] = static_cast<const char*>(pack_kv[2 * (l0 + l) + kv]) + pack_offset_bytes;
      }
    a.L = nl;
    if (a.append_only) {
      dim3 grid((unsigned)a.B_dst, (unsigned)((nl + kvg::LAYERS_PER_CTA - 1) / kvg::LAYERS_PER_CTA));
      if (p16) kvg::kv_append_kernel<uint4><<<grid, kvg::NT, 0, st>>>(a, ly);
      else if (p4) kvg::kv_append_kernel<uint32_t><<<grid, kvg::NT, 0, st>>>(a, ly);
      else kvg::kv_append_kernel<uint16_t><<<grid, kvg::NT, 0, st>>>(a, ly);
    } else {
      dim3 grid(gx, (unsigned)(a.B_dst * a.H), (unsigned)nl);
      if (p16) kvg::kv_gather_kernel<uint4><<<grid, kvg::NT, 0, st>>>(a, ly);
      else if (p4) kvg::kv_gather_kernel<uint32_t><<<grid, kvg::NT, 0, st>>>(a, ly);
      else kvg::kv_gather_kernel<uint16_t><<<grid, kvg::NT, 0, st>>>(a, ly);
    }
    if (cudaGetLastError() != cudaSuccess) return CAST_ERR_LAUNCH;
  }
  return CAST_OK;
}
}  // namespace
}  // namespace cast

extern "C" {

int cast_append_store(int n_layers, const void* const* src_kv, void* const* dst_kv, const void* const* pack_kv,
                      int elem_bytes, int H, int D, int B_src, int64_t src_cap, const int64_t* src_strides,
                      int B_dst, int64_t dst_cap, const int64_t* dst_strides, int64_t pack_rows,
                      const int64_t* pack_strides, const int32_t* rows, const int32_t* store_len,
                      const int32_t* accepted, const int32_t* keep, int keep_stride, const int32_t* cu_q,
                      int append_only, cast_stream_t stream) {
  if (elem_bytes != 2 && elem_bytes != 4) return CAST_ERR_DTYPE;
  if (n_layers < 0 || H < 1 || D < 1 || B_src < 0 || B_dst < 0 || src_cap < 0 || dst_cap < 0 || pack_rows < 0 ||
      keep_stride < 0 || (int64_t)B_dst * H > 65535)
    return CAST_ERR_SHAPE;
  if (n_layers == 0 || B_dst == 0) return CAST_OK;
  if (!src_kv || !dst_kv || !pack_kv || !src_strides || !dst_strides || !pack_strides || !store_len || !accepted ||
      !keep)
    return CAST_ERR_NULL;
  for (int i = 0; i < 2 * n_layers; ++i)
    if (!src_kv[i] || !dst_kv[i] || !pack_kv[i]) return CAST_ERR_NULL;
  if (append_only) {
    if (rows || B_dst != B_src || dst_cap != src_cap) return CAST_ERR_SHAPE;
    for (int i = 0; i < 2 * n_layers; ++i)
      if (src_kv[i] != dst_kv[i]) return CAST_ERR_SHAPE;
    for (int i = 0; i < 3; ++i)
      if (src_strides[i] != dst_strides[i]) return CAST_ERR_SHAPE;
  }
  const int64_t e = elem_bytes;
  kvg::KvArgs a{};
  a.H = H; a.row_bytes = D * elem_bytes; a.append_only = append_only ? 1 : 0;
  a.B_src = B_src; a.B_dst = B_dst; a.src_cap = src_cap; a.dst_cap = dst_cap; a.pack_rows = pack_rows;
  a.src_sb = src_strides[0] * e; a.src_sh = src_strides[1] * e; a.src_sr = src_strides[2] * e;
  a.dst_sb = dst_strides[0] * e; a.dst_sh = dst_strides[1] * e; a.dst_sr = dst_strides[2] * e;
  a.pk_sb = pack_strides[0] * e; a.pk_sh = pack_strides[1] * e; a.pk_st = pack_strides[2] * e;
  a.rows = rows; a.store_len = store_len; a.accepted = accepted; a.keep = keep; a.keep_stride = keep_stride;
  a.cu_q = cu_q;
  const int64_t grid_rows = append_only ? keep_stride : dst_cap;
  return kv_gather(n_layers, src_kv, dst_kv, pack_kv, 0, a, grid_rows, static_cast<cudaStream_t>(stream));
}

int cast_gather_cache(int n_layers, const void* const* src_kv, void* const* dst_kv, int elem_bytes, int B, int H,
                      int D, int64_t src_len, const int64_t* src_strides, const int64_t* dst_strides, int n_prefix,
                      const int32_t* keep, int n_keep, cast_stream_t stream) {
  if (elem_bytes != 2 && elem_bytes != 4) return CAST_ERR_DTYPE;
  if (n_layers < 0 || B < 0 || H < 1 || D < 1 || src_len < 0 || n_prefix < 0 || n_keep < 0 ||
      n_prefix > src_len || (int64_t)B * H > 65535)
    return CAST_ERR_SHAPE;
  if (n_layers == 0 || B == 0 || n_prefix + n_keep == 0) return CAST_OK;
  if (!src_kv || !dst_kv || !src_strides || !dst_strides || (n_keep > 0 && !keep)) return CAST_ERR_NULL;
  for (int i = 0; i < 2 * n_layers; ++i)
    if (!src_kv[i] || !dst_kv[i]) return CAST_ERR_NULL;
  const int64_t e = elem_bytes;
  kvg::KvArgs a{};
  a.H = H; a.row_bytes = D * elem_bytes; a.append_only = 0;
  a.B_src = B; a.B_dst = B; a.src_cap = src_len; a.dst_cap = (int64_t)n_prefix + n_keep;
  a.pack_rows = src_len - n_prefix;
  a.src_sb = src_strides[0] * e; a.src_sh = src_strides[1] * e; a.src_sr = src_strides[2] * e;
  a.dst_sb = dst_strides[0] * e; a.dst_sh = dst_strides[1] * e; a.dst_sr = dst_strides[2] * e;
  a.pk_sb = a.src_sb; a.pk_sh = a.src_sh; a.pk_st = a.src_sr;
  a.rows = nullptr; a.store_len = nullptr; a.accepted = nullptr; a.s_const = n_prefix; a.a_const = n_keep;
  a.keep = n_keep > 0 ? keep : nullptr;   // with no kept rows the kernel never reads it
  a.keep_stride = 0; a.cu_q = nullptr;
  return kv_gather(n_layers, src_kv, dst_kv, src_kv, (int64_t)n_prefix * a.src_sr, a, a.dst_cap,
                   static_cast<cudaStream_t>(stream));
}

}  // extern "C"
