// (d) Varlen causal attention over the paged cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), bf16 / head_dim 64 / block_size 16.
//
// One CTA computes one (128-query tile of one request, one query head); two
// CTAs share an SM (256 TMEM columns, <= 168 registers and ~98 KiB of shared
// memory each), so each SM sub-partition has two softmax warps in flight.
//
//   warp 4  TMA producer   Q tile once (128 rows x 128 B), then per 64-key
//                          tile 4+4 block loads of K and V rows of the kv head
//                          (2 KiB each, 128-byte swizzle) into a 5-stage ring;
//                          blocks past the needed keys are fetched out of
//                          bounds, i.e. as zeros.
//   warp 5  MMA issuer     one thread issues S_j = Q K_j^T (M=128, N=64,
//                          4 x K=16, both operands from shared memory) into one
//                          of two TMEM S buffers, and O += P_j V_j (M=128,
//                          N=64, 4 x K=16, A = P read from TMEM, V as an
//                          MN-major operand) into a TMEM O accumulator that
//                          lives across all key tiles.
//   warps 0-3 softmax      thread t owns query row t: one pass over its S row
//                          (64 values in registers): reference rounding
//                          (score = bf16(bf16(q.k) * scale); exact as one
//                          rounding when scale is a power of two), causal mask
//                          on diagonal tiles only, row max, exp2, row sum, P
//                          as bf16 pairs written over the S columns.  The
//                          running max is only raised when a tile exceeds it
//                          by more than 2^8 (lazy rescale: O in TMEM and l are
//                          then scaled once); otherwise P is taken against the
//                          stale max, which stays exact because the final
//                          O / l uses the same reference.  Epilogue: O / l.
//
// Waits are bounded: a wait that runs out raises NIE_DEV_ERR_TIMEOUT, the
// CTA stops issuing work, drains what is in flight and frees its TMEM.
#include "nie_attn.cuh"

namespace nie {

constexpr int kPfBM = 128;
constexpr int kPfBN = 64;
constexpr int kPfHD = 64;
constexpr int kPfBS = 16;
constexpr int kPfBlocksPerTile = kPfBN / kPfBS;
constexpr int kPfStages = 5;
constexpr int kPfThreads = 192;
constexpr uint32_t kPfTmemCols = 256;
constexpr uint32_t kPfWait = 1u << 22;
constexpr int kPfTileQ = kPfBM * kPfHD * 2;   // 16 KiB
constexpr int kPfTileKV = kPfBN * kPfHD * 2;  // 8 KiB
constexpr int kPfBlockBytes = kPfBS * kPfHD * 2;  // 2 KiB
constexpr uint32_t kSCol0 = 0, kSCol1 = 64, kOCol = 128;
constexpr float kPfLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;

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
  int chunks;       // key chunks per query tile (grid bound); 1 = no split
  int chunk_tiles;  // key tiles per chunk
  float* partials;  // [grid.x][hq] x {m[128], l[128], O[64][128]} when chunks > 1
  float scale;
  float scale_log2e;
  int scale_pow2;
  int32_t* err;
};

constexpr int kPfChunkTiles = 16;                   // 1024 keys per CTA at most
constexpr int kPfPartialFloats = (2 + kPfHD) * kPfBM;  // one (unit, head) partial

struct PfBars {
  uint64_t q_full;
  uint64_t kv_full[kPfStages];
  uint64_t kv_empty[kPfStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t done;
  uint32_t tmem_base;
  int abort;
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

// Round two fp32 values to bf16 and back (one packed conversion).
__device__ __forceinline__ void round_bf16_pair(float& a, float& b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  a = __low2float(h);
  b = __high2float(h);
}

__global__ void __launch_bounds__(kPfThreads, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm;
  uint8_t* skv = sm + kPfTileQ;
  PfBars* b = reinterpret_cast<PfBars*>(skv + kPfStages * 2 * kPfTileKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item (uniform across the CTA, decided before any barrier)
  const int chunk = blockIdx.x % a.chunks, unit = blockIdx.x / a.chunks;
  const int item = unit / a.tiles_per_req, tile = unit % a.tiles_per_req;
  const int r = a.req_list ? a.req_list[item] : item;
  const int64_t qs = a.qsl[r];
  const int qlen = (int)(a.qsl[r + 1] - qs);
  const int q0 = tile * kPfBM;
  if (q0 >= qlen) return;
  const int nq = min(kPfBM, qlen - q0);
  const int h = blockIdx.y, kvh = h / a.group;
  const int seq_len = a.seq_lens[r];
  const int ctx = seq_len - qlen;
  const int n_keys = ctx + q0 + nq;
  const int n_kt_all = (n_keys + kPfBN - 1) / kPfBN;
  const int kt0 = chunk * a.chunk_tiles;  // first key tile of this CTA
  if (kt0 >= n_kt_all) return;
  const int n_kt = min(a.chunk_tiles, n_kt_all - kt0);  // key tiles of this CTA
  const bool split = (n_kt_all + a.chunk_tiles - 1) / a.chunk_tiles > 1;
  const int trow = a.table_rows ? a.table_rows[r] : r;

  if (threadIdx.x == 0) {
    mbar_init(&b->q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&b->kv_full[s], 1);
      mbar_init(&b->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b->s_full[i], 1);
      mbar_init(&b->p_full[i], kPfBM);
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

  if (warp == 4) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(&b->q_full, kPfTileQ);
      tma_load_3d(sq, &qmap, &b->q_full, 0, h, (int)(qs + q0));
    }
    int issued = 0;
    for (int kt = 0; kt < n_kt; ++kt) {
      const int st = kt % kPfStages;
      if (kt >= kPfStages && !pf_wait(b, &b->kv_empty[st], (uint32_t)((kt - kPfStages) / kPfStages) & 1u, a.err))
        break;
      int coord = (int)(a.nb * kPfBS);  // out of bounds: zero fill
      if (lane < kPfBlocksPerTile) {
        const int lb = (kt0 + kt) * kPfBlocksPerTile + lane;
        if (lb * kPfBS < n_keys) {
          int64_t blk = (lb < a.tstride) ? (int64_t)a.tables[(int64_t)trow * a.tstride + lb] : -1;
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
      issued = kt + 1;
    }
    if (*reinterpret_cast<volatile int*>(&b->abort)) {
      // drain copies still in flight before the CTA exits
      mbar_wait_bounded(&b->q_full, 0, kPfWait);
      for (int kt = max(0, issued - kPfStages); kt < issued; ++kt)
        mbar_wait_bounded(&b->kv_full[kt % kPfStages], (uint32_t)(kt / kPfStages) & 1u, kPfWait);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------- MMA issuer
    const uint32_t id_s = idesc_bf16_f32(kPfBM, kPfBN, false, false);
    const uint32_t id_pv = idesc_bf16_f32(kPfBM, kPfHD, false, true);
    const uint32_t q_addr = smem_u32(sq);
    const int last_lb = (seq_len - 1) / kPfBS;
    const int tail = seq_len % kPfBS;
    bool ok = pf_wait(b, &b->q_full, 0, a.err);

    auto issue_s = [&](int j) -> bool {
      const int st = j % kPfStages;
      if (!pf_wait(b, &b->kv_full[st], (uint32_t)(j / kPfStages) & 1u, a.err)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(skv + st * 2 * kPfTileKV);
        const uint32_t d = tbase + ((j & 1) ? kSCol1 : kSCol0);
#pragma unroll
        for (int k = 0; k < kPfHD / 16; ++k)
          tc_mma_ss(d, smem_desc_sw128(q_addr + k * 32, 16, 1024), smem_desc_sw128(k_addr + k * 32, 16, 1024), id_s,
                    k > 0 ? 1u : 0u);
        tc_commit(&b->s_full[j & 1]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int j) -> bool {
      if (!pf_wait(b, &b->p_full[j & 1], (uint32_t)(j >> 1) & 1u, a.err)) return false;
      const int st = j % kPfStages;
      uint8_t* vt = skv + st * 2 * kPfTileKV + kPfTileKV;
      if (tail != 0 && last_lb / kPfBlocksPerTile == kt0 + j && last_lb * kPfBS < n_keys) {
        // stale rows past the sequence end (possibly NaN) must not meet P = 0
        uint4* z = reinterpret_cast<uint4*>(vt + (last_lb % kPfBlocksPerTile) * kPfBlockBytes + tail * (kPfHD * 2));
        for (int c = lane; c < (kPfBS - tail) * 8; c += 32) z[c] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
      }
      __syncwarp();
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(vt);
        const uint32_t p = tbase + ((j & 1) ? kSCol1 : kSCol0);
#pragma unroll
        for (int k = 0; k < kPfBN / 16; ++k)
          tc_mma_ts(tbase + kOCol, p + k * 8, smem_desc_sw128(v_addr + k * 2048, kPfTileKV, 1024), id_pv,
                    (j > 0 || k > 0) ? 1u : 0u);
        tc_commit(&b->o_done);
        tc_commit(&b->kv_empty[st]);
      }
      __syncwarp();
      return true;
    };

    if (ok && n_kt > 0) ok = issue_s(0);
    for (int j = 1; ok && j < n_kt; ++j) {
      ok = issue_s(j);
      if (ok) ok = issue_pv(j - 1);
    }
    if (ok && n_kt > 0) issue_pv(n_kt - 1);
    if (lane == 0) tc_commit(&b->done);
    __syncwarp();
    mbar_wait_bounded(&b->done, 0, kPfWait);
  } else {
    // -------------------------------------------------- softmax warps
    const int t = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int qpos = ctx + q0 + t;
    const int diag_from = ctx + q0;  // smallest query position of the tile
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    uint32_t v[64];

    for (int j = 0; j < n_kt; ++j) {
      const int sb = j & 1;
      if (!pf_wait(b, &b->s_full[sb], (uint32_t)(j >> 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tbase + lane_off + (sb ? kSCol1 : kSCol0);
      tmem_ld32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      const int key0 = (kt0 + j) * kPfBN;
      const bool masked = key0 + kPfBN - 1 > diag_from;
      // v holds the rounded scores in the "raw" domain (before * scale*log2e,
      // a positive factor, so the max can be taken before scaling)
      // eight independent max chains (a single chain is 32 dependent ops)
      float mxa[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxa[i] = -INFINITY;
      if (a.scale_pow2) {
        // bf16(bf16(acc) * 2^k) == bf16(acc) * 2^k: one rounding
#pragma unroll
        for (int e = 0; e < 64; e += 2) {
          float x0 = __uint_as_float(v[e]), x1 = __uint_as_float(v[e + 1]);
          round_bf16_pair(x0, x1);
          if (masked) {
            if (key0 + e > qpos) x0 = -INFINITY;
            if (key0 + e + 1 > qpos) x1 = -INFINITY;
          }
          v[e] = __float_as_uint(x0);
          v[e + 1] = __float_as_uint(x1);
          mxa[(e >> 1) & 7] = fmaxf(mxa[(e >> 1) & 7], fmaxf(x0, x1));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 64; e += 2) {
          float x0 = __uint_as_float(v[e]), x1 = __uint_as_float(v[e + 1]);
          round_bf16_pair(x0, x1);
          x0 *= a.scale;
          x1 *= a.scale;
          round_bf16_pair(x0, x1);
          x0 /= a.scale;  // exact: undoes a multiply whose result is representable
          x1 /= a.scale;
          if (masked) {
            if (key0 + e > qpos) x0 = -INFINITY;
            if (key0 + e + 1 > qpos) x1 = -INFINITY;
          }
          v[e] = __float_as_uint(x0);
          v[e + 1] = __float_as_uint(x1);
          mxa[(e >> 1) & 7] = fmaxf(mxa[(e >> 1) & 7], fmaxf(x0, x1));
        }
      }
      const float mx_raw = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                                 fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
      const float mx = mx_raw * a.scale_log2e;
      const bool raise = mx > m_ref + kRescaleLog2;
      if (__any_sync(0xffffffffu, raise)) {
        const float alpha = raise ? fast_exp2(m_ref - mx) : 1.f;
        if (raise) {
          l *= alpha;
          m_ref = mx;
        }
        if (j >= 1) {
          // O must hold P_{j-1} V_{j-1} before it is rescaled.  S_j was issued
          // after P_{j-2} V_{j-2} and its commit covers every earlier MMA, so
          // o_done has completed j-1 or j phases here: the parity wait for
          // phase j-1 is unambiguous although earlier phases were not waited on.
          if (!pf_wait(b, &b->o_done, (uint32_t)(j - 1) & 1u, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t o[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tmem_ld32(tbase + lane_off + kOCol + 32 * half, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(tbase + lane_off + kOCol + 32 * half, o);
          }
        }
      }
      float rsa[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) rsa[i] = 0.f;
      uint32_t pk[32];
      // a row whose keys in this chunk are all masked keeps m_ref = -inf: its
      // p must come out 0, not exp2(-inf + inf)
      const float sl2e = a.scale_log2e, neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float p0 = fast_exp2(fmaf(__uint_as_float(v[2 * e]), sl2e, neg_m));
        const float p1 = fast_exp2(fmaf(__uint_as_float(v[2 * e + 1]), sl2e, neg_m));
        rsa[e & 7] += p0 + p1;
        pk[e] = pack_bf16x2(p0, p1);
      }
      const float rs = ((rsa[0] + rsa[1]) + (rsa[2] + rsa[3])) + ((rsa[4] + rsa[5]) + (rsa[6] + rsa[7]));
      tmem_st32(s_addr, pk);
      tmem_wait_st();
      l += rs;
      tc_fence_before();
      mbar_arrive(&b->p_full[sb]);
    }
    // every MMA of the CTA has completed once `done` fires (its single phase is
    // unambiguous; o_done may be any number of phases behind the last tile)
    if (ok && n_kt > 0) ok = pf_wait(b, &b->done, 0u, a.err);
    if (ok) {
      tc_fence_after();
      tmem_ld32(tbase + lane_off + kOCol, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tbase + lane_off + kOCol + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      if (t < nq && !split) {
        const float inv = 1.f / l;
        __nv_bfloat16* op = a.out + (qs + q0 + t) * a.out_stride + (int64_t)h * kPfHD;
#pragma unroll
        for (int c = 0; c < kPfHD / 8; ++c) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[8 * c + 0]) * inv, __uint_as_float(v[8 * c + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[8 * c + 2]) * inv, __uint_as_float(v[8 * c + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[8 * c + 4]) * inv, __uint_as_float(v[8 * c + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[8 * c + 6]) * inv, __uint_as_float(v[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(op + 8 * c) = w;
        }
      } else if (t < nq) {
        // partial of this key chunk: m, l, unnormalised O (d-major so that a
        // warp's stores and the combine kernel's loads are contiguous)
        float* ps = a.partials + ((int64_t)blockIdx.x * a.hq + h) * kPfPartialFloats;
        ps[t] = m_ref;
        ps[kPfBM + t] = l;
#pragma unroll
        for (int d = 0; d < kPfHD; ++d) ps[2 * kPfBM + d * kPfBM + t] = __uint_as_float(v[d]);
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

// Merge the key-chunk partials of query tiles that were split across CTAs.
// grid = (units, q_heads), one thread per query row.
__global__ void __launch_bounds__(kPfBM) prefill_combine_kernel(PrefillArgs a) {
  const int unit = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  const int item = unit / a.tiles_per_req, tile = unit % a.tiles_per_req;
  const int r = a.req_list ? a.req_list[item] : item;
  const int64_t qs = a.qsl[r];
  const int qlen = (int)(a.qsl[r + 1] - qs);
  const int q0 = tile * kPfBM;
  if (q0 >= qlen) return;
  const int nq = min(kPfBM, qlen - q0);
  const int ctx = a.seq_lens[r] - qlen;
  const int n_kt_all = (ctx + q0 + nq + kPfBN - 1) / kPfBN;
  const int n_chunks = (n_kt_all + a.chunk_tiles - 1) / a.chunk_tiles;
  if (n_chunks <= 1 || t >= nq) return;
  auto slot = [&](int c) { return a.partials + ((int64_t)(unit * a.chunks + c) * a.hq + h) * kPfPartialFloats; };
  float M = -INFINITY;
  for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, slot(c)[t]);
  float L = 0.f;
  float o[kPfHD];
#pragma unroll
  for (int d = 0; d < kPfHD; ++d) o[d] = 0.f;
  for (int c = 0; c < n_chunks; ++c) {
    const float* ps = slot(c);
    const float m = ps[t];
    const float w = (m == -INFINITY) ? 0.f : fast_exp2(m - M);
    L += ps[kPfBM + t] * w;
#pragma unroll
    for (int d = 0; d < kPfHD; ++d) o[d] += ps[2 * kPfBM + d * kPfBM + t] * w;
  }
  const float inv = 1.f / L;
  __nv_bfloat16* op = a.out + (qs + q0 + t) * a.out_stride + (int64_t)h * kPfHD;
#pragma unroll
  for (int c = 0; c < kPfHD / 8; ++c) {
    uint4 w;
    w.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
    w.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
    w.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
    w.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
    *reinterpret_cast<uint4*>(op + 8 * c) = w;
  }
}

// Key chunks per 128-query tile for sequences of at most max_seq_len tokens.
static int prefill_chunks(int32_t max_seq_len) {
  if (max_seq_len <= 0) return 1;
  const int tiles = (max_seq_len + kPfBN - 1) / kPfBN;
  return max(1, (tiles + kPfChunkTiles - 1) / kPfChunkTiles);
}

size_t prefill_workspace_bytes(int32_t num_requests, int32_t max_query_len, int32_t max_seq_len, int32_t q_heads) {
  const int chunks = prefill_chunks(max_seq_len);
  if (chunks <= 1 || num_requests <= 0 || max_query_len <= 0) return 0;
  const int64_t units = (int64_t)num_requests * ((max_query_len + kPfBM - 1) / kPfBM);
  return (size_t)(units * chunks * q_heads) * kPfPartialFloats * sizeof(float);
}

static size_t prefill_smem_bytes() {
  return 1024 + kPfTileQ + (size_t)kPfStages * 2 * kPfTileKV + sizeof(PfBars);
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
  if (num_blocks * kPfBS >= (int64_t(1) << 31) || num_q_rows >= (int64_t(1) << 31) || (row_stride % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(q) % 16) != 0 || (reinterpret_cast<uintptr_t>(out) % 16) != 0 ||
      (reinterpret_cast<uintptr_t>(key_cache) % 16) != 0 || (reinterpret_cast<uintptr_t>(value_cache) % 16) != 0 ||
      q_heads > 65535 || num_q_rows <= 0)
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
  pa.tiles_per_req = (max_query_len + kPfBM - 1) / kPfBM;
  pa.chunks = prefill_chunks(max_seq_len);
  pa.chunk_tiles = kPfChunkTiles;
  pa.partials = nullptr;
  if (pa.chunks > 1) {
    const size_t need = prefill_workspace_bytes(num_requests, max_query_len, max_seq_len, q_heads);
    if (workspace != nullptr && workspace_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) % 16) == 0) {
      pa.partials = (float*)workspace;
    } else {
      // no scratch: one CTA per query tile walks all of its keys
      pa.chunks = 1;
      pa.chunk_tiles = 1 << 30;
    }
  } else {
    pa.chunk_tiles = 1 << 30;
  }
  pa.scale = scale;
  pa.scale_log2e = scale * kPfLog2e;
  pa.scale_pow2 = is_pow2_float(scale) ? 1 : 0;
  pa.err = err_flag;
  const size_t smem = prefill_smem_bytes();
  static thread_local bool s_attr = false;
  if (!s_attr) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NIE_ERR_CUDA, "prefill smem %zu: %s", smem, cudaGetErrorString(e));
    s_attr = true;
  }
  const int64_t units = (int64_t)num_requests * pa.tiles_per_req;
  const int64_t gx = units * pa.chunks;
  if (gx >= (int64_t(1) << 31)) return NIE_ERR_UNSUPPORTED;
  dim3 grid((unsigned)gx, (unsigned)q_heads);
  prefill_tc_kernel<<<grid, kPfThreads, smem, s>>>(qmap, kmap, vmap, pa);
  int rc = check_launch("prefill_tc_kernel");
  if (rc != NIE_OK || pa.chunks <= 1) return rc;
  prefill_combine_kernel<<<dim3((unsigned)units, (unsigned)q_heads), kPfBM, 0, s>>>(pa);
  return check_launch("prefill_combine_kernel");
}

}  // namespace nie
