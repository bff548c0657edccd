// (d) Varlen causal attention over the paged cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), bf16 / head_dim 64 / block_size 16.
//
// Work decomposition (persistent, stream-K).  A "segment" is one (128-query
// tile of one request, query head) pair; it owns ceil(keys / 64) key tiles.
// All segments are laid end to end (query tile major, head minor, so the
// heads sharing a kv head are neighbours), each weighted as its key tiles plus
// kPfSegCost for its fixed work (first and diagonal tiles, epilogue, pipeline
// drain), and the resulting cost list is cut into equal contiguous ranges,
// one per CTA, with two CTAs per SM and one wave: every SM does the same
// amount of work whatever the length mix (short segments cost more per tile),
// and each CTA pays its prologue once.  A segment that lies wholly in one
// CTA's range is normalised and written by that CTA.  A segment cut by range
// boundaries begins in the range of one CTA (its last segment, processed at
// the end) and continues into the next ones (their first segment, processed
// at their start): those later CTAs leave (max, sum, unnormalised O) partials
// in the workspace and raise one flag per softmax warp, and the CTA where the
// segment begins waits for the flags (bounded), merges in CTA order and
// writes the rows.  All CTAs of the grid are resident at once (two per SM,
// one wave), so the wait always ends.  Without a workspace each CTA takes
// exactly one segment instead.
//
// Roles of the 6 warps of a CTA (all iterate the same segments / tiles):
//   warp 4  TMA producer   per segment the Q tile (128 rows x 128 B) into one
//                          of two Q buffers, then per 64-key tile 4+4 block
//                          loads of K and V rows of the kv head (2 KiB each,
//                          128-byte swizzle) into a 4-stage ring; blocks past
//                          the needed keys are fetched out of bounds (zeros).
//   warp 5  MMA issuer     one thread issues S_g = Q K_g^T (M=128, N=64,
//                          4 x K=16, operands in shared memory) into one of
//                          two TMEM S buffers, then O += P_{g-1} V_{g-1}
//                          (M=128, N=64, 4 x K=16, A = P read from TMEM, V as
//                          an MN-major operand) into the segment's TMEM O
//                          buffer (two O buffers alternate between segments).
//   warps 0-3 softmax      thread t owns query row t: its S row (64 values
//                          in registers) rounded as the reference does
//                          (score = bf16(bf16(q.k) * scale); exact as one
//                          rounding when scale is a power of two) straight
//                          into bf16 pairs, causal mask on diagonal tiles
//                          only, row max on the pairs (max.bf16x2), exp2
//                          arguments and row sums two lanes per instruction
//                          (f32x2), P as bf16 pairs over the S columns.  The
//                          running max is only raised when a tile exceeds it
//                          by more than 2^8 (lazy rescale: O in TMEM and l are
//                          then scaled once); otherwise P is taken against the
//                          stale max, which stays exact because the final
//                          O / l uses the same reference.  Segment end: O / l
//                          (or the partial), then the O buffer is released.
//
// TMEM (256 columns per CTA): S0 0-63, S1 64-127, O0 128-191, O1 192-255.
// Waits are bounded: a wait that runs out raises NIE_DEV_ERR_TIMEOUT, the
// CTA stops issuing work, drains what is in flight and frees its TMEM.
#include "nie_attn.cuh"

namespace nie {

constexpr int kPfBM = 128;
constexpr int kPfBN = 64;
constexpr int kPfHD = 64;
constexpr int kPfBS = 16;
constexpr int kPfBlocksPerTile = kPfBN / kPfBS;
constexpr int kPfStages = 4;
constexpr int kPfThreads = 192;
constexpr uint32_t kPfTmemCols = 256;
constexpr uint32_t kPfWait = 1u << 22;
constexpr uint32_t kPfMergeWait = 1u << 20;  // polls of a producer's flag (each an L2 round trip)
constexpr int kPfTileQ = kPfBM * kPfHD * 2;       // 16 KiB
constexpr int kPfTileKV = kPfBN * kPfHD * 2;      // 8 KiB
constexpr int kPfBlockBytes = kPfBS * kPfHD * 2;  // 2 KiB
constexpr uint32_t kSCol0 = 0, kSCol1 = 64, kOCol0 = 128;  // O buffer b at kOCol0 + 64 b
constexpr float kPfLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;
// Work of one segment beyond its key tiles (first tile, diagonal tiles, the
// O epilogue, the pipeline drain and refill), in key tiles: the persistent
// grid splits key tiles plus this much per segment evenly over the CTAs.
constexpr int kPfSegCost = 3;
constexpr int kPfMaxUnits = 2048;  // 128-query tiles per call (larger calls use the generic kernel)
constexpr int kPfMaxCtas = 320;    // persistent grid bound (2 per SM)
constexpr int kPfPartialFloats = (2 + kPfHD) * kPfBM;  // m[128], l[128], O[64][128]
// workspace: [flags: kPfMaxCtas x 4 int32, zeroed by the host before each call | partials]
constexpr size_t kPfFlagBytes = ((size_t)kPfMaxCtas * 4 * sizeof(int32_t) + 255) & ~size_t(255);

struct PrefillArgs {
  __nv_bfloat16* out;
  int64_t out_stride;
  int64_t nb;
  int hkv, hq, group;
  const int32_t* tables;
  int64_t tstride;
  const int32_t* table_rows;
  const int32_t* seq_lens;
  const int64_t* qsl;
  const int32_t* req_list;
  int tiles_per_req;
  int units;        // num_requests * tiles_per_req query tiles
  int stream;       // 1: equal tile ranges per CTA + partials; 0: one segment per CTA
  float* partials;  // [grid] x kPfPartialFloats (stream mode): a CTA's first segment when cut
  int32_t* flags;   // [grid][4] (stream mode): softmax warp w of CTA c has written its rows of c's partial
  float scale;
  float scale_log2e;
  int scale_pow2;
  int32_t* err;
};

struct PfBars {
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t kv_full[kPfStages];
  uint64_t kv_empty[kPfStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;      // every P V product (global tile order)
  uint64_t o_full[2];   // a segment's last P V product, per O buffer
  uint64_t o_free[2];   // the softmax warps have read an O buffer
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int red[kPfThreads];
  int cum[kPfMaxUnits + 1];
};

// Bounded wait that also gives up once another warp aborted the CTA.
__device__ __forceinline__ bool pf_wait(PfBars* b, uint64_t* bar, uint32_t parity, int32_t* err) {
  for (uint32_t i = 0; i < kPfWait; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *reinterpret_cast<volatile int*>(&b->abort)) return false;
  }
  *reinterpret_cast<volatile int*>(&b->abort) = 1;
  raise_flag(err, NIE_DEV_ERR_TIMEOUT);
  return false;
}

// Flag store / load with gpu-scope release / acquire ordering.
__device__ __forceinline__ void st_release_gpu(int32_t* p, int32_t v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_gpu(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The two halves of a bf16 pair as fp32 (exact).
__device__ __forceinline__ float bf16_lo(uint32_t r) { return __uint_as_float(r << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t r) { return __uint_as_float(r & 0xffff0000u); }

// Lane-wise maximum of two bf16 pairs (exact, as the fp32 maximum of the values).
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// d = a * b + c on two fp32 lanes in one instruction (sm_100 f32x2): each lane
// is an IEEE fma, so the results equal two fmaf calls.
__device__ __forceinline__ void fma_f32x2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                          float c1) {
  asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// d += b on two fp32 lanes in one instruction.
__device__ __forceinline__ void add_f32x2(float& d0, float& d1, float b0, float b1) {
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(d0), "f"(d1), "f"(b0), "f"(b1));
}

// Geometry of one 128-query tile ("unit").
struct PfUnit {
  int64_t qs;   // first query row of the request
  int q0, nq;   // tile offset in the request, rows in the tile
  int ctx;      // cached tokens before the request's queries
  int seq_len;
  int trow;     // block-table row
  int n_kt;     // key tiles (0: the tile is past the request's queries)
};

__device__ __forceinline__ PfUnit pf_unit(const PrefillArgs& a, int u) {
  PfUnit x;
  const int item = u / a.tiles_per_req, tile = u % a.tiles_per_req;
  const int r = a.req_list ? a.req_list[item] : item;
  x.qs = a.qsl[r];
  const int qlen = (int)(a.qsl[r + 1] - x.qs);
  x.q0 = tile * kPfBM;
  x.nq = min(kPfBM, qlen - x.q0);
  x.seq_len = a.seq_lens[r];
  x.ctx = x.seq_len - qlen;
  x.trow = a.table_rows ? a.table_rows[r] : r;
  x.n_kt = x.q0 < qlen ? (x.ctx + x.q0 + x.nq + kPfBN - 1) / kPfBN : 0;
  return x;
}

// Cost of a unit per query head: its key tiles plus kPfSegCost when it has any.
__device__ __forceinline__ int pf_unit_cost(int n_kt) { return n_kt > 0 ? n_kt + kPfSegCost : 0; }

// The global work list: segments (unit major, head minor), each occupying a
// cost interval of kPfSegCost followed by its key tiles; cum[u] = the cost of
// one head of every unit < u, so segment (u, h) starts at hq cum[u] + h d_u
// with d_u = cum[u + 1] - cum[u].  A CTA owns the cost range [lo, hi) and
// processes the key tiles that lie in it.  Walks the segments with tiles in
// that range; identical in every warp.
struct PfSegIter {
  const int* cum;
  int units, hq;
  int64_t lo, hi;
  int u, h;        // current segment
  int d;           // cost of one segment of unit u
  int64_t start;   // cost position of its first key tile
  int n;           // its key tiles

  __device__ void set_unit() {
    d = cum[u + 1] - cum[u];
    n = d > 0 ? d - kPfSegCost : 0;
  }
  __device__ void init(const int* c, int U, int H, int64_t a_lo, int64_t a_hi) {
    cum = c;
    units = U;
    hq = H;
    lo = a_lo;
    hi = a_hi;
    // largest unit with hq * cum[u] <= lo (it has cost since lo < total)
    int l = 0, r = U - 1;
    while (l < r) {
      const int m = (l + r + 1) >> 1;
      if ((int64_t)hq * cum[m] <= lo) l = m; else r = m - 1;
    }
    u = l;
    set_unit();
    h = d > 0 ? (int)((lo - (int64_t)hq * cum[u]) / d) : 0;
    start = (int64_t)hq * cum[u] + (int64_t)h * d + kPfSegCost;
  }
  // a segment whose tiles start at or past hi belongs to the next CTA
  __device__ bool valid() const { return lo < hi && start < hi; }
  __device__ int t_lo() const { return (int)(max(lo, start) - start); }
  __device__ int t_hi() const { return (int)(min(hi, start + n) - start); }
  __device__ void next() {
    if (++h < hq) {
      start += d;
      return;
    }
    h = 0;
    do {
      ++u;
    } while (u < units && cum[u + 1] == cum[u]);
    if (u >= units) {
      start = hi;
      return;
    }
    set_unit();
    start = (int64_t)hq * cum[u] + kPfSegCost;
  }
};

__global__ void __launch_bounds__(kPfThreads, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm;                     // two Q buffers
  uint8_t* skv = sm + 2 * kPfTileQ;     // K/V ring
  PfBars* b = reinterpret_cast<PfBars*>(skv + kPfStages * 2 * kPfTileKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = a.units;

  // ---- cost per unit and head, and their prefix sums (the whole CTA)
  {
    const int per = (U + kPfThreads - 1) / kPfThreads;
    const int u0 = threadIdx.x * per, u1 = min(U, u0 + per);
    int local = 0;
    for (int u = u0; u < u1; ++u) {
      const int n = pf_unit_cost(pf_unit(a, u).n_kt);
      b->cum[u] = n;
      local += n;
    }
    b->red[threadIdx.x] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0;
      for (int i = 0; i < kPfThreads; ++i) {
        const int v = b->red[i];
        b->red[i] = run;
        run += v;
      }
      b->cum[U] = run;
    }
    __syncthreads();
    int run = b->red[threadIdx.x];
    for (int u = u0; u < u1; ++u) {
      const int v = b->cum[u];
      b->cum[u] = run;
      run += v;
    }
    __syncthreads();
  }
  const int64_t total = (int64_t)a.hq * b->cum[U];
  int64_t lo, hi;
  int64_t W = 0;
  if (a.stream) {
    W = (total + gridDim.x - 1) / gridDim.x;
    lo = (int64_t)blockIdx.x * W;
    hi = min(total, lo + W);
  } else {
    // one segment per CTA: blockIdx.x = unit * hq + head
    const int u = blockIdx.x / a.hq, h = blockIdx.x % a.hq;
    const int d = b->cum[u + 1] - b->cum[u];
    lo = (int64_t)a.hq * b->cum[u] + (int64_t)h * d;
    hi = lo + d;
  }
  // a dependent launch after this kernel may be staged now (every CTA of this
  // grid is resident once all have passed here)
  pdl_trigger();
  if (lo >= hi) return;  // uniform: nothing to do for this CTA

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b->q_full[i], 1);
      mbar_init(&b->q_empty[i], 1);
      mbar_init(&b->s_full[i], 1);
      mbar_init(&b->p_full[i], kPfBM);
      mbar_init(&b->o_full[i], 1);
      mbar_init(&b->o_free[i], kPfBM);
    }
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&b->kv_full[s], 1);
      mbar_init(&b->kv_empty[s], 1);
    }
    mbar_init(&b->o_done, 1);
    mbar_init(&b->done, 1);
    b->abort = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&b->tmem_base, kPfTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = b->tmem_base;
  PfSegIter seg;
  seg.init(b->cum, U, a.hq, lo, hi);

  if (warp == 4) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    int k = 0;        // segments of this CTA so far
    int64_t g = 0;    // key tiles of this CTA so far
    int64_t issued = 0;
    int q_issued = 0;
    bool ok = true;
    for (; ok && seg.valid(); seg.next(), ++k) {
      const PfUnit x = pf_unit(a, seg.u);
      const int qb = k & 1;
      if (k >= 2 && !pf_wait(b, &b->q_empty[qb], (uint32_t)((k - 2) >> 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&b->q_full[qb], kPfTileQ);
        tma_load_3d(sq + qb * kPfTileQ, &qmap, &b->q_full[qb], 0, seg.h, (int)(x.qs + x.q0));
      }
      q_issued = k + 1;
      const int kvh = seg.h / a.group;
      const int n_keys = x.ctx + x.q0 + x.nq;
      for (int kt = seg.t_lo(); kt < seg.t_hi(); ++kt, ++g) {
        const int st = (int)(g % kPfStages);
        if (g >= kPfStages && !pf_wait(b, &b->kv_empty[st], (uint32_t)((g - kPfStages) / kPfStages) & 1u, a.err)) {
          ok = false;
          break;
        }
        int coord = (int)(a.nb * kPfBS);  // out of bounds: zero fill
        if (lane < kPfBlocksPerTile) {
          const int lb = kt * kPfBlocksPerTile + lane;
          if (lb * kPfBS < n_keys) {
            int64_t blk = (lb < a.tstride) ? (int64_t)a.tables[(int64_t)x.trow * a.tstride + lb] : -1;
            if (blk < 0 || blk >= a.nb) {
              raise_flag(a.err, NIE_DEV_ERR_BLOCK_RANGE);
              blk = 0;
            }
            coord = (int)(blk * kPfBS);
          }
        }
        if (lane == 0) mbar_arrive_expect_tx(&b->kv_full[st], 2 * kPfTileKV);
        __syncwarp();
        if (lane < kPfBlocksPerTile) {
          uint8_t* dst = skv + st * 2 * kPfTileKV + lane * kPfBlockBytes;
          tma_load_3d(dst, &kmap, &b->kv_full[st], 0, kvh, coord);
          tma_load_3d(dst + kPfTileKV, &vmap, &b->kv_full[st], 0, kvh, coord);
        }
        issued = g + 1;
      }
    }
    if (*reinterpret_cast<volatile int*>(&b->abort)) {
      // drain copies still in flight before the CTA exits
      for (int kq = max(0, q_issued - 2); kq < q_issued; ++kq)
        mbar_wait_bounded(&b->q_full[kq & 1], (uint32_t)(kq >> 1) & 1u, kPfWait);
      for (int64_t gg = max((int64_t)0, issued - kPfStages); gg < issued; ++gg)
        mbar_wait_bounded(&b->kv_full[gg % kPfStages], (uint32_t)(gg / kPfStages) & 1u, kPfWait);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------- MMA issuer
    const uint32_t id_s = idesc_bf16_f32(kPfBM, kPfBN, false, false);
    const uint32_t id_pv = idesc_bf16_f32(kPfBM, kPfHD, false, true);
    bool ok = true;
    // the P V product still to issue (one tile behind S)
    struct Pend {
      bool live = false;
      int64_t g;
      int ob;           // O buffer of its segment
      int k;            // its segment's index in this CTA
      bool first, last; // first / last tile of that segment in this CTA
      int seq_len;      // its sequence: stale V rows past the end are zeroed
      int kt;           // its key tile index within the segment
    } pend;

    auto issue_pv = [&](const Pend& p) -> bool {
      if (!pf_wait(b, &b->p_full[p.g & 1], (uint32_t)(p.g >> 1) & 1u, a.err)) return false;
      if (p.first && p.k >= 2 &&
          !pf_wait(b, &b->o_free[p.ob], (uint32_t)((p.k - 2) >> 1) & 1u, a.err))
        return false;  // the softmax warps still read this O buffer's previous segment
      const int st = (int)(p.g % kPfStages);
      uint8_t* vt = skv + st * 2 * kPfTileKV + kPfTileKV;
      const int last_lb = (p.seq_len - 1) / kPfBS;
      const int tail = p.seq_len % kPfBS;
      if (tail != 0 && last_lb / kPfBlocksPerTile == p.kt) {
        // stale rows past the sequence end (possibly NaN) must not meet P = 0
        uint4* z = reinterpret_cast<uint4*>(vt + (last_lb % kPfBlocksPerTile) * kPfBlockBytes + tail * (kPfHD * 2));
        for (int c = lane; c < (kPfBS - tail) * 8; c += 32) z[c] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
      }
      __syncwarp();
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(vt);
        const uint32_t pcol = tbase + ((p.g & 1) ? kSCol1 : kSCol0);
        const uint32_t ocol = tbase + kOCol0 + 64u * (uint32_t)p.ob;
#pragma unroll
        for (int kk = 0; kk < kPfBN / 16; ++kk)
          tc_mma_ts(ocol, pcol + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kPfTileKV, 1024), id_pv,
                    (!p.first || kk > 0) ? 1u : 0u);
        tc_commit(&b->o_done);
        tc_commit(&b->kv_empty[st]);
        if (p.last) tc_commit(&b->o_full[p.ob]);
      }
      __syncwarp();
      return true;
    };

    int k = 0;
    int64_t g = 0;
    for (; ok && seg.valid(); seg.next(), ++k) {
      const PfUnit x = pf_unit(a, seg.u);
      const int qb = k & 1;
      if (!pf_wait(b, &b->q_full[qb], (uint32_t)(k >> 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      const uint32_t q_addr = smem_u32(sq + qb * kPfTileQ);
      const int tlo = seg.t_lo(), thi = seg.t_hi();
      for (int kt = tlo; ok && kt < thi; ++kt, ++g) {
        const int st = (int)(g % kPfStages);
        if (!pf_wait(b, &b->kv_full[st], (uint32_t)(g / kPfStages) & 1u, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t k_addr = smem_u32(skv + st * 2 * kPfTileKV);
          const uint32_t d = tbase + ((g & 1) ? kSCol1 : kSCol0);
#pragma unroll
          for (int kk = 0; kk < kPfHD / 16; ++kk)
            tc_mma_ss(d, smem_desc_sw128(q_addr + kk * 32, 16, 1024), smem_desc_sw128(k_addr + kk * 32, 16, 1024),
                      id_s, kk > 0 ? 1u : 0u);
          tc_commit(&b->s_full[g & 1]);
          // the Q buffer is free once this segment's last S product completes
          if (kt + 1 == thi) tc_commit(&b->q_empty[qb]);
        }
        __syncwarp();
        if (pend.live) ok = issue_pv(pend);
        pend.live = true;
        pend.g = g;
        pend.ob = k & 1;
        pend.k = k;
        pend.first = kt == tlo;
        pend.last = kt + 1 == thi;
        pend.seq_len = x.seq_len;
        pend.kt = kt;
      }
    }
    if (ok && pend.live) issue_pv(pend);
    if (lane == 0) tc_commit(&b->done);
    __syncwarp();
    mbar_wait_bounded(&b->done, 0, kPfWait);
  } else {
    // -------------------------------------------------- softmax warps
    const int t = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    uint32_t v[64];
    // exp2 argument per unit of the stored score: the stored scores are raw
    // (scale not applied) when the scale is a power of two
    const float coef = a.scale_pow2 ? a.scale_log2e : kPfLog2e;
    int k = 0;
    int64_t g = 0;
    for (; ok && seg.valid(); seg.next(), ++k) {
      const PfUnit x = pf_unit(a, seg.u);
      const int ob = k & 1;
      const uint32_t ocol = kOCol0 + 64u * (uint32_t)ob;
      const int qpos = x.ctx + x.q0 + t;
      const int diag_from = x.ctx + x.q0;  // smallest query position of the tile
      const int tlo = seg.t_lo(), thi = seg.t_hi();
      float m_ref = -INFINITY, l = 0.f;
      for (int kt = tlo; kt < thi; ++kt, ++g) {
        const int sb = (int)(g & 1);
        if (!pf_wait(b, &b->s_full[sb], (uint32_t)(g >> 1) & 1u, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_addr = tbase + lane_off + (sb ? kSCol1 : kSCol0);
        tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        // r[e]: the rounded scores of keys 2e, 2e+1 as a bf16 pair.  With a
        // power-of-two scale bf16(bf16(acc) * 2^k) == bf16(acc) * 2^k, so one
        // rounding gives the raw-domain score and the scale rides in coef;
        // otherwise r holds bf16(bf16(acc) * scale) itself.
        uint32_t r[32];
        if (a.scale_pow2) {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t h = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
            r[e] = pack_bf16x2(bf16_lo(h) * a.scale, bf16_hi(h) * a.scale);
          }
        }
        const int key0 = kt * kPfBN;
        if (key0 + kPfBN - 1 > diag_from) {
          // causal mask (diagonal tiles only): keys past the row's position
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (key0 + 2 * e > qpos) r[e] = (r[e] & 0xffff0000u) | 0xff80u;
            if (key0 + 2 * e + 1 > qpos) r[e] = (r[e] & 0x0000ffffu) | 0xff800000u;
          }
        }
        // row max of the bf16 scores (coef > 0, so it is taken before scaling):
        // eight independent packed chains
        uint32_t mx2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx2[i] = r[i];
#pragma unroll
        for (int e = 8; e < 32; ++e) mx2[e & 7] = max_bf16x2(mx2[e & 7], r[e]);
        const uint32_t mxp = max_bf16x2(max_bf16x2(max_bf16x2(mx2[0], mx2[1]), max_bf16x2(mx2[2], mx2[3])),
                                        max_bf16x2(max_bf16x2(mx2[4], mx2[5]), max_bf16x2(mx2[6], mx2[7])));
        const float mx = fmaxf(bf16_lo(mxp), bf16_hi(mxp)) * coef;
        const bool raise = mx > m_ref + kRescaleLog2;
        if (__any_sync(0xffffffffu, raise)) {
          const float alpha = raise ? fast_exp2(m_ref - mx) : 1.f;
          if (raise) {
            l *= alpha;
            m_ref = mx;
          }
          if (kt > tlo) {
            // O must hold P_{g-1} V_{g-1} (this segment's previous tile) before
            // it is rescaled.  S_g was issued after P_{g-2} V_{g-2} and its
            // commit covers every earlier MMA, so o_done has completed g-1 or g
            // phases here: the parity wait for phase g-1 is unambiguous
            // although earlier phases were not waited on.
            if (!pf_wait(b, &b->o_done, (uint32_t)(g - 1) & 1u, a.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            uint32_t o[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              tmem_ld32(tbase + lane_off + ocol + 32 * half, o);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st32(tbase + lane_off + ocol + 32 * half, o);
            }
          }
        }
        // p = exp2(score * coef - m_ref) two lanes at a time; a row whose keys
        // in this range are all masked keeps m_ref = -inf: its p must come out
        // 0, not exp2(-inf + inf)
        float rs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs[i] = 0.f;
        const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float y0, y1;
          fma_f32x2(y0, y1, bf16_lo(r[e]), bf16_hi(r[e]), coef, coef, neg_m, neg_m);
          const float p0 = fast_exp2(y0), p1 = fast_exp2(y1);
          add_f32x2(rs[2 * (e & 3)], rs[2 * (e & 3) + 1], p0, p1);
          pk[e] = pack_bf16x2(p0, p1);
        }
        const float row_sum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
        tmem_st32(s_addr, pk);
        tmem_wait_st();
        l += row_sum;
        tc_fence_before();
        mbar_arrive(&b->p_full[sb]);
      }
      if (!ok) break;
      // the segment's last P V product has completed once o_full fires (one
      // phase per use of the buffer)
      if (!pf_wait(b, &b->o_full[ob], (uint32_t)(k >> 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_ld32(tbase + lane_off + ocol, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tbase + lane_off + ocol + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&b->o_free[ob]);
      const bool whole = tlo == 0 && thi == seg.n;
      // the three cases are uniform across the CTA (they depend on the
      // segment and the range only), so whole warps take each branch
      if (whole) {
        if (t < x.nq) {
        const float inv = 1.f / l;
        __nv_bfloat16* op = a.out + (x.qs + x.q0 + t) * a.out_stride + (int64_t)seg.h * kPfHD;
#pragma unroll
        for (int c = 0; c < kPfHD / 8; ++c) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[8 * c + 0]) * inv, __uint_as_float(v[8 * c + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[8 * c + 2]) * inv, __uint_as_float(v[8 * c + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[8 * c + 4]) * inv, __uint_as_float(v[8 * c + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[8 * c + 6]) * inv, __uint_as_float(v[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(op + 8 * c) = w;
        }
        }
      } else if (tlo > 0) {
        // the segment began in an earlier CTA's range (so it is this CTA's
        // first segment): leave the partial (d-major, so that a warp's stores
        // and the merging warp's loads are contiguous) and raise this warp's flag
        float* ps = a.partials + (int64_t)blockIdx.x * kPfPartialFloats;
        if (t < x.nq) {
          ps[t] = m_ref;
          ps[kPfBM + t] = l;
#pragma unroll
          for (int d = 0; d < kPfHD; ++d) ps[2 * kPfBM + d * kPfBM + t] = __uint_as_float(v[d]);
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(a.flags + blockIdx.x * 4 + warp, 1);
      } else {
        // the segment begins here and continues into CTAs c+1 .. c1: wait for
        // their partials of this warp's rows, merge in CTA order, write
        const int64_t c1 = (seg.start + seg.n - 1) / W;
        for (int64_t c = blockIdx.x + 1; ok && c <= c1; ++c) {
          const int32_t* flag = a.flags + c * 4 + warp;
          uint32_t i = 0;
          while (ld_acquire_gpu(flag) == 0) {
            if (++i == kPfMergeWait || ((i & 1023u) == 0 && *reinterpret_cast<volatile int*>(&b->abort))) {
              if (i == kPfMergeWait) {
                *reinterpret_cast<volatile int*>(&b->abort) = 1;
                raise_flag(a.err, NIE_DEV_ERR_TIMEOUT);
              }
              ok = false;
              break;
            }
          }
        }
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        if (t < x.nq) {
          float M = m_ref;
          for (int64_t c = blockIdx.x + 1; c <= c1; ++c) M = fmaxf(M, a.partials[c * kPfPartialFloats + t]);
          const float w0 = (m_ref == -INFINITY) ? 0.f : fast_exp2(m_ref - M);
          float L = l * w0;
#pragma unroll
          for (int d = 0; d < kPfHD; ++d) v[d] = __float_as_uint(__uint_as_float(v[d]) * w0);
          for (int64_t c = blockIdx.x + 1; c <= c1; ++c) {
            const float* ps = a.partials + c * kPfPartialFloats;
            const float m = ps[t];
            const float w = (m == -INFINITY) ? 0.f : fast_exp2(m - M);
            L += ps[kPfBM + t] * w;
#pragma unroll
            for (int d = 0; d < kPfHD; ++d)
              v[d] = __float_as_uint(fmaf(ps[2 * kPfBM + d * kPfBM + t], w, __uint_as_float(v[d])));
          }
          const float inv = 1.f / L;
          __nv_bfloat16* op = a.out + (x.qs + x.q0 + t) * a.out_stride + (int64_t)seg.h * kPfHD;
#pragma unroll
          for (int c = 0; c < kPfHD / 8; ++c) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * c + 0]) * inv, __uint_as_float(v[8 * c + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[8 * c + 2]) * inv, __uint_as_float(v[8 * c + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[8 * c + 4]) * inv, __uint_as_float(v[8 * c + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[8 * c + 6]) * inv, __uint_as_float(v[8 * c + 7]) * inv);
            *reinterpret_cast<uint4*>(op + 8 * c) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kPfTmemCols);
  }
}

size_t prefill_workspace_bytes(int32_t num_requests, int32_t max_query_len, int32_t max_seq_len, int32_t q_heads) {
  (void)max_seq_len;
  (void)q_heads;
  if (num_requests <= 0 || max_query_len <= 0) return 0;
  return kPfFlagBytes + (size_t)kPfMaxCtas * kPfPartialFloats * sizeof(float);
}

static size_t prefill_smem_bytes() {
  return 1024 + 2 * kPfTileQ + (size_t)kPfStages * 2 * kPfTileKV + sizeof(PfBars);
}

static bool is_pow2_float(float x) {
  if (!(x > 0.f)) return false;
  int e = 0;
  return frexpf(x, &e) == 0.5f;
}

// Returns NIE_ERR_UNSUPPORTED when the shape is not the tensor-core one, so
// the caller can use the generic kernel.
int launch_prefill_tc(const void* q, void* out, int64_t row_stride, int64_t num_q_rows, const void* key_cache,
                      const void* value_cache, int32_t layer, int64_t num_blocks, int32_t kv_heads, int32_t q_heads,
                      const int32_t* block_tables, int64_t table_stride, const int32_t* table_rows,
                      const int32_t* seq_lens, const int64_t* qsl, const int32_t* req_list, int32_t num_requests,
                      int32_t max_query_len, int32_t max_seq_len, float scale, void* workspace,
                      size_t workspace_bytes, int32_t* err_flag, cudaStream_t s) {
  (void)max_seq_len;
  const int tiles_per_req = (max_query_len + kPfBM - 1) / kPfBM;
  const int64_t units = (int64_t)num_requests * tiles_per_req;
  if (num_blocks * kPfBS >= (int64_t(1) << 31) || num_q_rows >= (int64_t(1) << 31) || (row_stride % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(q) % 16) != 0 || (reinterpret_cast<uintptr_t>(out) % 16) != 0 ||
      (reinterpret_cast<uintptr_t>(key_cache) % 16) != 0 || (reinterpret_cast<uintptr_t>(value_cache) % 16) != 0 ||
      q_heads > 65535 || num_q_rows <= 0 || units <= 0 || units > kPfMaxUnits || units * q_heads >= (int64_t(1) << 31))
    return NIE_ERR_UNSUPPORTED;
  const int64_t row_bytes = (int64_t)kv_heads * kPfHD * 2;
  const int64_t layer_bytes = num_blocks * kPfBS * row_bytes;
  CUtensorMap qmap, kmap, vmap;
  {
    const uint64_t dims[3] = {(uint64_t)kPfHD, (uint64_t)q_heads, (uint64_t)num_q_rows};
    const uint64_t strides[2] = {(uint64_t)kPfHD * 2, (uint64_t)row_stride * 2};
    const uint32_t box[3] = {(uint32_t)kPfHD, 1u, (uint32_t)kPfBM};
    int rc = encode_tiled(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NIE_OK) return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)kPfHD, (uint64_t)kv_heads, (uint64_t)(num_blocks * kPfBS)};
    const uint64_t strides[2] = {(uint64_t)kPfHD * 2, (uint64_t)row_bytes};
    const uint32_t box[3] = {(uint32_t)kPfHD, 1u, (uint32_t)kPfBS};
    int rc = encode_tiled(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                          (void*)((const char*)key_cache + layer * layer_bytes), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NIE_OK) return rc;
    rc = encode_tiled(&vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void*)((const char*)value_cache + layer * layer_bytes),
                      dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NIE_OK) return rc;
  }
  PrefillArgs pa{};
  pa.out = (__nv_bfloat16*)out;
  pa.out_stride = row_stride;
  pa.nb = num_blocks;
  pa.hkv = kv_heads;
  pa.hq = q_heads;
  pa.group = q_heads / kv_heads;
  pa.tables = block_tables;
  pa.tstride = table_stride;
  pa.table_rows = table_rows;
  pa.seq_lens = seq_lens;
  pa.qsl = qsl;
  pa.req_list = req_list;
  pa.tiles_per_req = tiles_per_req;
  pa.units = (int)units;
  const size_t need = prefill_workspace_bytes(num_requests, max_query_len, max_seq_len, q_heads);
  pa.stream = workspace != nullptr && workspace_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) % 256) == 0;
  if (pa.stream) {
    pa.flags = (int32_t*)workspace;
    pa.partials = (float*)((char*)workspace + kPfFlagBytes);
  }
  pa.scale = scale;
  pa.scale_log2e = scale * kPfLog2e;
  pa.scale_pow2 = is_pow2_float(scale) ? 1 : 0;
  pa.err = err_flag;
  const size_t smem = prefill_smem_bytes();
  const int orc = opt_in_smem(kSmemPrefill, (const void*)prefill_tc_kernel, smem);
  if (orc != NIE_OK) return orc;
  int grid;
  if (pa.stream) {
    const int sms = sm_count(stream_device(s));
    if (sms <= 0) return fail(NIE_ERR_CUDA, "cannot query the SM count");
    grid = std::min(2 * sms, kPfMaxCtas);
  } else {
    grid = (int)(units * q_heads);  // one segment per CTA
  }
  if (pa.stream && cudaMemsetAsync(pa.flags, 0, kPfFlagBytes, s) != cudaSuccess)
    return fail(NIE_ERR_CUDA, "cannot clear the prefill flags");
  prefill_tc_kernel<<<grid, kPfThreads, smem, s>>>(qmap, kmap, vmap, pa);
  return check_launch("prefill_tc_kernel");
}

}  // namespace nie
