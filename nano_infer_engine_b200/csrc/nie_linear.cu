// (f) Weight-streaming linear for decode-size batches:
//     y[M, N] = x[M, K] . W[N, K]^T,  bf16 in and out, fp32 accumulation, M <= 16.
//
// A decode step multiplies 16 activation rows by each projection matrix, so
// the work is a stream of the weights (2 bytes per weight, ~16 flops per
// weight byte pair): the bound is HBM, not the tensor pipe.  cuBLAS runs the
// small-N shapes at 1.1-2.6 TB/s (too few CTAs for N = 2048-3072, no K split
// for the long K of down_proj), so this kernel puts every SM on the stream:
//
//  * An n-tile is 128 weight rows.  The K range of a tile is split over the
//    CTAs of one thread-block cluster (cs = 1..8 CTAs, chosen so that all
//    clusters are resident at once), each streaming its share of 128 x 64
//    k-steps (16 KiB, one 128-byte swizzled TMA box) through an 8-deep ring.
//  * One producer warp issues the TMA loads (weight tile + the matching 16 x 64
//    slice of x); four consumer warps each own 32 weight rows and run m16n8k16
//    bf16 MMAs (x rows are M, weight rows are N) into fp32 registers.  The
//    tensor work is a few percent of the stream time, so the legacy MMA is not
//    the bound.
//  * The partial sums of a tile meet in distributed shared memory: each CTA
//    stores its 16 x 128 fp32 partial, the cluster synchronises, and CTA r
//    sums 1/cs of the outputs over the cluster's partials in rank order (a
//    fixed order: results do not depend on timing) and writes them as bf16.
//    No global workspace, counter or atomic is involved.
//
// Replaces the nn.Linear calls of the decoder layers at decode time
// (reference layers/attention.py:121-145 projections, layers/mlp.py:18-22)
// when the batch has at most 16 rows; torch's cuBLAS GEMM handles the rest.
#include <map>
#include <mutex>
#include <tuple>

#include "nie_attn.cuh"

namespace nie {
namespace {

constexpr int kLnK = 64;                // K elements per k-step (one 128-byte swizzle row)
constexpr int kLnStages = 8;            // ring depth
constexpr int kLnConsumerWarps = 4;
constexpr int kLnThreads = (kLnConsumerWarps + 1) * 32;
constexpr int kLnXRows = 16;            // MMA M: activation rows (zero-filled past M)
constexpr int kLnXBytes = kLnXRows * kLnK * 2;
constexpr int kLnMaxCluster = 8;
constexpr uint32_t kLnWaitProbes = 1u << 22;

// Shared-memory layout of a CTA working on ROWS-row tiles.
template <int ROWS>
struct LnLayout {
  static constexpr int kWBytes = ROWS * kLnK * 2;
  static constexpr int kStageBytes = kWBytes + kLnXBytes;      // a multiple of 1024
  static constexpr int kPairs = kLnXRows * ROWS / 2;           // output pairs of one tile
  static constexpr int kRecvBytes = (kPairs + kLnMaxCluster) * 8;
  static constexpr size_t kUsed =
      1024 + (size_t)kLnStages * kStageBytes + kRecvBytes + 2 * kLnStages * sizeof(uint64_t);
  // Requested per CTA: more than half an SM's shared memory, so that CTAs
  // never pair up on one SM (each SM streams for one CTA).
  static constexpr size_t kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
};

struct LinearArgs {
  __nv_bfloat16* y;
  int64_t ldy;
  int m;
  int ksteps;  // k-steps per n-tile (K / 64)
  int32_t* err;
  int early_weights;  // issue the first ring of weight loads before waiting for the previous kernel
  uint32_t wait_probes;  // bound of every mbarrier wait (kLnWaitProbes outside the timeout test hook)
  int withhold;          // timeout test hook: the producer issues no copy, so every consumer wait runs out
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster arrives; shared-memory writes
// (local or remote) before it are visible to the cluster after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Split cluster barrier: every thread arrives once its CTA has started (after
// the mbarrier set-up) and waits before its first remote shared-memory store,
// so no CTA writes into a peer that has not started yet.  The wait sits after
// the streaming loop, where all peers have long arrived.
__device__ __forceinline__ void cluster_arrive_started() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_started() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Store two floats at `local_addr` (an address in this CTA's shared window)
// in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ void st_cluster_f2(uint32_t local_addr, uint32_t rank, float x, float y) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(remote), "f"(x), "f"(y) : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// First output pair owned by cluster CTA r (of cs) and the owner of pair p.
__device__ __forceinline__ int pair_begin(int r, int cs, int pairs) { return (int)((int64_t)pairs * r / cs); }
__device__ __forceinline__ int pair_owner(int p, int cs, int pairs) {
  return (int)((((int64_t)p + 1) * cs - 1) / pairs);
}

// grid = n_tiles * cs CTAs in clusters of cs (consecutive blockIdx.x); CTA
// rank r of a cluster streams k-steps [ksteps*r/cs, ksteps*(r+1)/cs) of tile
// blockIdx.x / cs.  Weight map boxes are ROWS x 64.
template <int ROWS>
__global__ void __launch_bounds__(kLnThreads, 1)
    linear_stream_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                         LinearArgs a) {
  using Lay = LnLayout<ROWS>;
  constexpr int NT = ROWS / 32;  // n8 tiles per consumer warp (ROWS / 4 weight rows)
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  float2* recv = reinterpret_cast<float2*>(dsm + kLnStages * Lay::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + kLnStages * Lay::kStageBytes + Lay::kRecvBytes);
  uint64_t* empty = full + kLnStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();  // the kernel after this one may be staged now
  const int cs = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
  const int tile = (int)(blockIdx.x / (unsigned)cs);
  const int s0 = (int)((int64_t)a.ksteps * rank / cs), s1 = (int)((int64_t)a.ksteps * (rank + 1) / cs);
  const int steps = s1 - s0;
  const int per = (Lay::kPairs + cs - 1) / cs;  // receive slots per source CTA
  if (threadIdx.x == 0) {
    for (int i = 0; i < kLnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kLnConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive_started();

  if (warp == kLnConsumerWarps) {
    // ---------------- producer: one lane keeps the ring full
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      const uint64_t stream_once = l2_policy_evict_first();
      // Dependent launch: x (and y's memory) belong to the kernel before until it
      // completes, so x is loaded only after this wait (the consumers write y
      // only after their stages, x included, have landed).  With early_weights
      // the caller guarantees that kernel does not write w: the first ring of
      // weight tiles is already streaming while it finishes.
      int k = 0;
      if (a.withhold) {
        pdl_wait();
        k = steps;  // nothing issued: nothing in flight, no drain below
      } else if (a.early_weights) {
        for (; k < steps && k < kLnStages; ++k) {
          mbar_arrive_expect_tx(&full[k], Lay::kStageBytes);
          tma_load_2d_hint(dsm + k * Lay::kStageBytes, &wmap, &full[k], (s0 + k) * kLnK, tile * ROWS, stream_once);
        }
        pdl_wait();
        for (int j = 0; j < k; ++j)
          tma_load_2d(dsm + j * Lay::kStageBytes + Lay::kWBytes, &xmap, &full[j], (s0 + j) * kLnK, 0);
      } else {
        pdl_wait();
      }
      for (; k < steps; ++k) {
        const int st = k % kLnStages;
        if (k >= kLnStages && !mbar_wait_bounded(&empty[st], (uint32_t)((k / kLnStages) - 1) & 1u, a.wait_probes)) {
          raise_flag(a.err, NIE_DEV_ERR_TIMEOUT);
          break;
        }
        uint8_t* stage = dsm + st * Lay::kStageBytes;
        const int kk = s0 + k;
        mbar_arrive_expect_tx(&full[st], Lay::kStageBytes);
        tma_load_2d_hint(stage, &wmap, &full[st], kk * kLnK, tile * ROWS, stream_once);
        tma_load_2d(stage + Lay::kWBytes, &xmap, &full[st], kk * kLnK, 0);
      }
      // Copies of the last issued stages may still be landing if a consumer
      // gave up early: wait (bounded) for them before the CTA moves on.
      if (!a.withhold)
        for (int j = k > kLnStages ? k - kLnStages : 0; j < k; ++j)
          mbar_wait_bounded(&full[j % kLnStages], (uint32_t)(j / kLnStages) & 1u, a.wait_probes);
    }
    __syncwarp();
    cluster_wait_started();
  } else {
    // ---------------- consumers: warp w owns weight rows [w*ROWS/4, (w+1)*ROWS/4) of the tile
    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, rr = lane & 7;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    for (int k = 0; k < steps; ++k) {
      const int st = k % kLnStages;
      if (!mbar_wait_bounded(&full[st], (uint32_t)(k / kLnStages) & 1u, a.wait_probes)) {
        if (lane == 0) raise_flag(a.err, NIE_DEV_ERR_TIMEOUT);
        break;
      }
      const uint32_t wb = smem_u32(dsm + st * Lay::kStageBytes);
      const uint32_t xb = wb + Lay::kWBytes;
      uint32_t af[4][4];
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int row = (mi & 1) * 8 + rr;
        const int chunk = ks * 2 + (mi >> 1);
        ldmatrix_x4(af[ks][0], af[ks][1], af[ks][2], af[ks][3], xb + row * 128 + ((chunk ^ (row & 7)) << 4));
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int row = warp * (ROWS / 4) + nt * 8 + rr;
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          const int chunk = kp * 4 + mi;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3, wb + row * 128 + ((chunk ^ (row & 7)) << 4));
          mma_bf16_16816(acc[nt], af[2 * kp], b0, b1);
          mma_bf16_16816(acc[nt], af[2 * kp + 1], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // send each output pair's partial to the cluster CTA that owns it (every
    // cluster CTA has started: see cluster_wait_started)
    cluster_wait_started();
    const uint32_t rbase = smem_u32(recv);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = warp * (ROWS / 4) + nt * 8 + 2 * t;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = g + 8 * h;
        if (row >= a.m) continue;
        const int p = row * (ROWS / 2) + col / 2;
        const int owner = pair_owner(p, cs, Lay::kPairs);
        const int slot = rank * per + (p - pair_begin(owner, cs, Lay::kPairs));
        st_cluster_f2(rbase + (uint32_t)slot * 8u, (uint32_t)owner, acc[nt][2 * h], acc[nt][2 * h + 1]);
      }
    }
  }

  // ---------------- every partial of this CTA's pairs has arrived: sum in rank order
  cluster_sync_all();
  const int p0 = pair_begin(rank, cs, Lay::kPairs), p1 = pair_begin(rank + 1, cs, Lay::kPairs);
  for (int p = p0 + (int)threadIdx.x; p < p1; p += kLnThreads) {
    const int row = p / (ROWS / 2), col = (p % (ROWS / 2)) * 2;
    if (row >= a.m) continue;
    float sx = 0.f, sy = 0.f;
    for (int q = 0; q < cs; ++q) {
      const float2 v = recv[q * per + (p - p0)];
      sx += v.x;
      sy += v.y;
    }
    *reinterpret_cast<uint32_t*>(a.y + (int64_t)row * a.ldy + (int64_t)tile * ROWS + col) = pack_bf16x2(sx, sy);
  }
}

// Tensor maps of weight matrices, keyed by (device, address, N, K, box rows):
// a map depends only on those, so reuse is always valid.
std::mutex g_ln_mu;
std::map<std::tuple<int, uintptr_t, int64_t, int64_t, int>, CUtensorMap> g_wmaps;
// Per device and tile height: the number of clusters of each size (1..8)
// resident at once (-1: that size cannot be launched).
int g_max_clusters[64][2][kLnMaxCluster + 1];

template <int ROWS>
int max_active_clusters(int dev, int cs) {
  int& slot = g_max_clusters[dev][ROWS == 128 ? 0 : 1][cs];
  if (slot == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(cs * 1024));
    cfg.blockDim = dim3(kLnThreads);
    cfg.dynamicSmemBytes = LnLayout<ROWS>::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, linear_stream_kernel<ROWS>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;
    }
    slot = n;
  }
  return slot;
}

// The widest K split (cluster size) whose clusters of `tiles` tiles are all
// resident at once without more CTAs than SMs; 0 when the tiles alone do not fit.
template <int ROWS>
int pick_cluster(int dev, int tiles, int ksteps, int sms) {
  for (int c = kLnMaxCluster; c >= 1; --c) {
    if (c > ksteps || tiles * c > sms) continue;
    const int fit = max_active_clusters<ROWS>(dev, c);
    if (fit > 0 && tiles <= fit) return c;
  }
  return 0;
}

// Per-device set-up on the first call: the shared-memory opt-in of both
// kernel instances and the whole resident-cluster table, so that later calls
// (a new shape, or a call inside a CUDA-graph capture) only read the table.
int opt_in_both(int dev) {
  int rc = opt_in_smem(kSmemLinear, (const void*)linear_stream_kernel<128>, LnLayout<128>::kSmem);
  if (rc != NIE_OK) return rc;
  rc = opt_in_smem(kSmemLinear64, (const void*)linear_stream_kernel<64>, LnLayout<64>::kSmem);
  if (rc != NIE_OK) return rc;
  for (int c = 1; c <= kLnMaxCluster; ++c) {
    max_active_clusters<128>(dev, c);
    max_active_clusters<64>(dev, c);
  }
  return NIE_OK;
}

}  // namespace
}  // namespace nie

using namespace nie;

static int linear_impl(const void* x, int64_t ldx, const void* w, int64_t n, int64_t k, int64_t m, void* y,
                       int64_t ldy, int32_t dtype, int32_t* err_flag, void* stream, bool early_weights,
                       bool withhold = false, uint32_t wait_probes = kLnWaitProbes) {
  NIE_REQUIRE(x && w && y, "null pointer argument");
  NIE_REQUIRE(m >= 0 && n > 0 && k > 0, "bad shape m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
  if (dtype != NIE_DTYPE_BF16 || m > kLnXRows || n % 64 != 0 || k % kLnK != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(y) & 3) != 0 || (ldx * 2) % 16 != 0 || ldx < k || ldy % 2 != 0 || ldy < n ||
      n >= (int64_t(1) << 30) || k >= (int64_t(1) << 30))
    return fail(NIE_ERR_UNSUPPORTED,
                "nie_linear takes bf16, m <= 16, n %% 64 == 0, k %% 64 == 0, 16-byte aligned x and w rows");
  if (m == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int dev = stream_device(s);
  NIE_REQUIRE(dev >= 0 && dev < 64, "cannot resolve the current device");
  const int sms = sm_count(dev);
  NIE_REQUIRE(sms > 0, "cannot query the SM count of device %d", dev);
  const int ksteps = (int)(k / kLnK);

  // Tile height and K split: as many CTAs as possible, at most one per SM,
  // every cluster resident at once (128-row tiles on a tie: fewer partials).
  int rows = 0, cs = 0;
  {
    std::lock_guard<std::mutex> lk(g_ln_mu);
    const int rc = opt_in_both(dev);
    if (rc != NIE_OK) return rc;
    const int c128 = n % 128 == 0 ? pick_cluster<128>(dev, (int)(n / 128), ksteps, sms) : 0;
    const int c64 = pick_cluster<64>(dev, (int)(n / 64), ksteps, sms);
    if (c128 > 0 && (n / 128) * c128 >= (n / 64) * c64) {
      rows = 128;
      cs = c128;
    } else if (c64 > 0) {
      rows = 64;
      cs = c64;
    }
  }
  if (rows == 0)
    return fail(NIE_ERR_UNSUPPORTED, "nie_linear: n = %lld needs more than one CTA per SM; use a library GEMM",
                (long long)n);
  const int tiles = (int)(n / rows);
  CUtensorMap wmap, xmap;
  {
    std::lock_guard<std::mutex> lk(g_ln_mu);
    const auto key = std::make_tuple(dev, reinterpret_cast<uintptr_t>(w), n, k, rows);
    auto it = g_wmaps.find(key);
    if (it == g_wmaps.end()) {
      const uint64_t dims[2] = {(uint64_t)k, (uint64_t)n};
      const uint64_t strides[1] = {(uint64_t)k * 2};
      const uint32_t box[2] = {(uint32_t)kLnK, (uint32_t)rows};
      const int rc = encode_tiled(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides,
                                  box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != NIE_OK) return rc;
      if (g_wmaps.size() > 4096) g_wmaps.clear();
      g_wmaps.emplace(key, wmap);
    } else {
      wmap = it->second;
    }
  }
  {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)m};
    const uint64_t strides[1] = {(uint64_t)ldx * 2};
    const uint32_t box[2] = {(uint32_t)kLnK, (uint32_t)kLnXRows};
    const int rc = encode_tiled(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NIE_OK) return rc;
  }
  LinearArgs la{};
  la.y = reinterpret_cast<__nv_bfloat16*>(y);
  la.ldy = ldy;
  la.m = (int)m;
  la.ksteps = ksteps;
  la.err = err_flag;
  la.early_weights = early_weights ? 1 : 0;
  la.wait_probes = wait_probes;
  la.withhold = withhold ? 1 : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(tiles * cs));
  cfg.blockDim = dim3(kLnThreads);
  cfg.dynamicSmemBytes = rows == 128 ? LnLayout<128>::kSmem : LnLayout<64>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = rows == 128 ? cudaLaunchKernelEx(&cfg, linear_stream_kernel<128>, wmap, xmap, la)
                              : cudaLaunchKernelEx(&cfg, linear_stream_kernel<64>, wmap, xmap, la);
  if (e != cudaSuccess) return fail(NIE_ERR_CUDA, "linear_stream_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("linear_stream_kernel");
}

extern "C" int nie_linear(const void* x, int64_t ldx, const void* w, int64_t n, int64_t k, int64_t m, void* y,
                          int64_t ldy, int32_t dtype, int32_t* err_flag, void* stream) {
  return linear_impl(x, ldx, w, n, k, m, y, ldy, dtype, err_flag, stream, false);
}

extern "C" int nie_linear_overlapped(const void* x, int64_t ldx, const void* w, int64_t n, int64_t k, int64_t m,
                                     void* y, int64_t ldy, int32_t dtype, int32_t* err_flag, void* stream) {
  return linear_impl(x, ldx, w, n, k, m, y, ldy, dtype, err_flag, stream, true);
}

extern "C" int nie_linear_timeout_test(const void* x, int64_t ldx, const void* w, int64_t n, int64_t k, int64_t m,
                                       void* y, int64_t ldy, int32_t dtype, int32_t* err_flag, void* stream,
                                       uint32_t wait_probes) {
  NIE_REQUIRE(wait_probes > 0 && wait_probes <= kLnWaitProbes, "wait_probes must be in [1, %u]", kLnWaitProbes);
  return linear_impl(x, ldx, w, n, k, m, y, ldy, dtype, err_flag, stream, false, true, wait_probes);
}
