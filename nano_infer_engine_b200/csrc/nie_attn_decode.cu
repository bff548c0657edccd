// (c) Paged decode attention, bf16 / head_dim 64 / block_size 16 (the
// Llama-3.2-1B cache shape), as a balanced split-K ("stream-K") kernel:
//
//  * The blocks of all requests form one global list (prefix sums of
//    ceil(seq_len / 16)); CTA c of a fixed grid (one per SM) takes the
//    contiguous range [c*W, (c+1)*W), so every SM streams the same number of
//    KV bytes whatever the length mix.  A range may span several requests; a
//    request covered by one CTA is finished in place, a request split over
//    CTAs leaves (max, sum, unnormalised O) partials that a small combine
//    kernel merges.
//  * Warp w owns kv head w (the CTA has kv_heads warps) and runs its own
//    NSTAGE-deep pipeline: lane 0 issues two 2 KiB TMA tile loads (K and V
//    rows of that head for one 16-token block, 128-byte swizzled) per block on
//    a per-stage mbarrier; no CTA-wide barrier is taken inside the loop.
//  * The G = q_heads / kv_heads query heads of the group are the M rows of
//    m16n8k16 bf16 MMAs (rows >= G are zero): S = Q K^T (8 MMAs / block),
//    online softmax on the accumulator fragments with quad shuffles, and
//    O += P V (8 MMAs / block) reusing the S fragments as the A operand.
//    The tensor-core work is ~10x below the HBM time, so the legacy MMA is
//    not the bound; the kernel is HBM-bound by design.
//
// Numerics follow nano_infer_engine/layers/paged_attention.py:95-114: the
// q.k dot is rounded to bf16, scaled, rounded again; softmax runs in fp32
// (base-2 with the log2(e) factor folded in); probabilities enter the PV
// product as bf16 and the output is rounded once.  The one difference from
// the reference is that p is normalised after the PV product instead of
// before its cast to bf16 (online softmax), a < 2^-8 relative effect.
#include <mutex>

#include "nie_attn.cuh"

namespace nie {

constexpr int kDecBS = 16;
constexpr int kDecHD = 64;
constexpr int kTileBytes = kDecBS * kDecHD * 2;  // one (block, head) tile: 2 KiB
constexpr int kDecStages = 4;       // pipeline depth per warp for kv_heads <= 8
constexpr int kDecStagesWide = 3;   // kv_heads 9..16 (shared memory bound)
constexpr int kDecCtasPerSm = 1;
constexpr int kDecMaxReq = 8192;
constexpr uint32_t kWaitProbes = 1u << 22;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t q_stride;
  __nv_bfloat16* out;
  int64_t out_stride;
  int64_t nb;
  int hkv, hq, group;
  const int32_t* tables;
  int64_t tstride;
  const int32_t* table_rows;
  const int32_t* seq_lens;
  const int64_t* q_rows;
  const int32_t* req_list;
  int num_req;
  float scale;
  float* partials;  // [slots][hq * (64 + 2)]: m[hq], l[hq], O[hq][64]
  int32_t* cum_out; // [num_req + 2]: block prefix sums, then W
  int32_t* err;
};

// Exclusive scan of vals[0..n) in place by the whole CTA; returns the total.
__device__ int cta_exclusive_scan(int* vals, int n, int* warp_tot) {
  const int nt = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int per = (n + nt - 1) / nt;
  const int b = tid * per, e = min(n, b + per);
  int local = 0;
  for (int i = b; i < e; ++i) local += vals[i];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < nw) ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < nw) warp_tot[lane] = wi - w;
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  int run = warp_tot[warp] + incl - local;
  for (int i = b; i < e; ++i) {
    int v = vals[i];
    vals[i] = run;
    run += v;
  }
  const int total = warp_tot[32];
  __syncthreads();
  return total;
}

__device__ __forceinline__ uint32_t ld_u32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int NST>
__global__ void __launch_bounds__(512, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                      DecodeArgs a) {
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ int warp_tot[33];
  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* tiles = dsm;
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsm + nw * NST * 2 * kTileBytes);
  int* cum = reinterpret_cast<int*>(bars + nw * NST);
  const int R = a.num_req;
  int* reqs = cum + R + 1;   // request index of list entry i
  int* trows = reqs + R;     // its block-table row
  if (threadIdx.x == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }

  // Per-request metadata into shared memory up front: one dependent global
  // load (the request list) before the lengths and table rows, which load in
  // parallel; the block walk below then reads only the block tables.
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int r = a.req_list ? a.req_list[i] : i;
    const int n = a.seq_lens[r];
    const int trow = a.table_rows ? a.table_rows[r] : r;
    reqs[i] = r;
    trows[i] = trow;
    cum[i] = n > 0 ? (n + kDecBS - 1) / kDecBS : 0;
  }
  __syncthreads();
  const int total = cta_exclusive_scan(cum, R, warp_tot);
  if (threadIdx.x == 0) cum[R] = total;
  if (lane == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&bars[warp * NST + s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int W = (total + (int)gridDim.x - 1) / (int)gridDim.x;
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i <= R; i += blockDim.x) a.cum_out[i] = cum[i];
    if (threadIdx.x == 0) a.cum_out[R + 1] = W;
  }
  if (total == 0) return;
  const int gb0 = (int)blockIdx.x * W;
  const int gb1 = min(total, gb0 + W);
  if (gb0 >= gb1) return;

  uint8_t* my_tiles = tiles + warp * NST * 2 * kTileBytes;
  uint64_t* my_bars = bars + warp * NST;
  const uint64_t policy = l2_policy_evict_first();

  auto locate = [&](int g) {
    int lo = 0, hi = R;  // cum[lo] <= g < cum[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cum[mid] <= g) lo = mid; else hi = mid;
    }
    return lo;
  };

  // ---- producer side: a window of 32 physical block ids, one per lane
  int win_base = gb0, win_blk = 0;
  auto refill = [&](int base) {
    win_base = base;
    const int g = base + lane;
    int blk = 0;
    if (g < gb1) {
      const int i = locate(g);
      const int trow = trows[i];
      const int64_t lb = g - cum[i];
      int64_t b = (lb < a.tstride) ? (int64_t)a.tables[(int64_t)trow * a.tstride + lb] : -1;
      if (b < 0 || b >= a.nb) {
        raise_flag(a.err, NIE_DEV_ERR_BLOCK_RANGE);
        b = 0;  // stay in bounds; the host reports the flag
      }
      blk = (int)b;
    }
    win_blk = blk;
  };
  auto issue = [&](int g, int st) {
    if (g - win_base >= 32) refill(g);
    const int blk = __shfl_sync(0xffffffffu, win_blk, g - win_base);
    if (lane == 0) {
      uint64_t* bar = my_bars + st;
      uint8_t* kt = my_tiles + st * 2 * kTileBytes;
      mbar_arrive_expect_tx(bar, 2 * kTileBytes);
      tma_load_3d_hint(kt, &kmap, bar, 0, warp, blk * kDecBS, policy);
      tma_load_3d_hint(kt + kTileBytes, &vmap, bar, 0, warp, blk * kDecBS, policy);
    }
  };
  refill(gb0);
  // Everything above reads step metadata written before the previous kernel
  // (RoPE + KV write) was launched; q and the newest cache rows come from that
  // kernel, so wait for it before the first load of either.
  pdl_wait();
  int iss = gb0;
  for (int st = 0; st < NST && iss < gb1; ++st, ++iss) issue(iss, st);

  // ---- consumer side
  const int G = a.group;
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  uint32_t qa[4][4];
  float m0, m1, l0, l1;
  float o[8][4];
  int n_tok = 0;
  int64_t qrow = 0;

  auto begin_request = [&](int i) {
    const int req = reqs[i];
    n_tok = a.seq_lens[req];
    qrow = a.q_rows ? a.q_rows[req] : (int64_t)req;
    const __nv_bfloat16* qp = a.q + qrow * a.q_stride + (int64_t)warp * G * kDecHD;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int c = ks * 16 + 2 * t;
      qa[ks][0] = (g < G) ? ld_u32(qp + g * kDecHD + c) : 0u;
      qa[ks][1] = (g + 8 < G) ? ld_u32(qp + (g + 8) * kDecHD + c) : 0u;
      qa[ks][2] = (g < G) ? ld_u32(qp + g * kDecHD + c + 8) : 0u;
      qa[ks][3] = (g + 8 < G) ? ld_u32(qp + (g + 8) * kDecHD + c + 8) : 0u;
    }
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  };

  auto finalize = [&](int i, bool whole) {
    float L0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
    float L1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
    if (whole) {
      if (g < G) {
        __nv_bfloat16* op = a.out + qrow * a.out_stride + (int64_t)(warp * G + g) * kDecHD;
        const float inv = 1.f / L0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<uint32_t*>(op + j * 8 + 2 * t) = pack_bf16x2(o[j][0] * inv, o[j][1] * inv);
      }
      if (g + 8 < G) {
        __nv_bfloat16* op = a.out + qrow * a.out_stride + (int64_t)(warp * G + g + 8) * kDecHD;
        const float inv = 1.f / L1;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<uint32_t*>(op + j * 8 + 2 * t) = pack_bf16x2(o[j][2] * inv, o[j][3] * inv);
      }
    } else {
      float* ps = a.partials + (int64_t)(blockIdx.x + i) * a.hq * (kDecHD + 2);
      if (g < G) {
        const int h = warp * G + g;
        if (t == 0) {
          ps[h] = m0;
          ps[a.hq + h] = L0;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float2*>(ps + 2 * a.hq + h * kDecHD + j * 8 + 2 * t) = make_float2(o[j][0], o[j][1]);
      }
      if (g + 8 < G) {
        const int h = warp * G + g + 8;
        if (t == 0) {
          ps[h] = m1;
          ps[a.hq + h] = L1;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float2*>(ps + 2 * a.hq + h * kDecHD + j * 8 + 2 * t) = make_float2(o[j][2], o[j][3]);
      }
    }
  };

  int i = locate(gb0);
  int seg_lo = cum[i], seg_hi = cum[i + 1];
  begin_request(i);
  int k = 0;
  for (int gi = gb0; gi < gb1; ++gi, ++k) {
    const int st = k % NST;
    const uint32_t par = (uint32_t)(k / NST) & 1u;
    if (!mbar_wait_bounded(my_bars + st, par, kWaitProbes)) {
      if (lane == 0) raise_flag(a.err, NIE_DEV_ERR_TIMEOUT);
      for (int g2 = gi + 1, k2 = k + 1; g2 < iss; ++g2, ++k2)
        mbar_wait_bounded(my_bars + (k2 % NST), (uint32_t)(k2 / NST) & 1u, kWaitProbes);
      return;
    }
    uint8_t* kt = my_tiles + st * 2 * kTileBytes;
    uint8_t* vt = kt + kTileBytes;
    const int lb = gi - seg_lo;
    const int valid = min(kDecBS, n_tok - lb * kDecBS);
    if (valid < kDecBS) {
      // Rows past the sequence end hold stale cache contents (possibly NaN):
      // zero them so 0-weight columns cannot poison the PV product.
      uint4* vz = reinterpret_cast<uint4*>(vt + valid * 128);
      for (int c = lane; c < (kDecBS - valid) * 8; c += 32) vz[c] = make_uint4(0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
      __syncwarp();
    }

    // S = Q K^T : 2 n-tiles (tokens 0-7, 8-15) x 4 k-steps (head_dim)
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
    const uint32_t kb = smem_u32(kt);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        const int tok = nt * 8 + rr;
        const int chunk = kp * 4 + mi;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, kb + tok * 128 + ((chunk ^ (tok & 7)) << 4));
        mma_bf16_16816(sacc[nt], qa[2 * kp], b0, b1);
        mma_bf16_16816(sacc[nt], qa[2 * kp + 1], b2, b3);
      }
    }

    // online softmax (rows g and g + 8), reference rounding of the scores
    float x[2][4];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = (nt * 8 + 2 * t + e) < valid;
        const float s0 = __bfloat162float(__float2bfloat16_rn(
            __bfloat162float(__float2bfloat16_rn(sacc[nt][e])) * a.scale));
        const float s1 = __bfloat162float(__float2bfloat16_rn(
            __bfloat162float(__float2bfloat16_rn(sacc[nt][2 + e])) * a.scale));
        x[nt][e] = ok ? s0 * kLog2e : -INFINITY;
        x[nt][2 + e] = ok ? s1 * kLog2e : -INFINITY;
        mx0 = fmaxf(mx0, x[nt][e]);
        mx1 = fmaxf(mx1, x[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
    float p[2][4];
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = fast_exp2(x[nt][e] - mn0);
        p[nt][2 + e] = fast_exp2(x[nt][2 + e] - mn1);
        rs0 += p[nt][e];
        rs1 += p[nt][2 + e];
      }
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(p[0][0], p[0][1]);
    pa[1] = pack_bf16x2(p[0][2], p[0][3]);
    pa[2] = pack_bf16x2(p[1][0], p[1][1]);
    pa[3] = pack_bf16x2(p[1][2], p[1][3]);

    // O += P V : 8 n-tiles over head_dim, one k-step of 16 tokens
    const uint32_t vb = smem_u32(vt);
#pragma unroll
    for (int cp = 0; cp < 4; ++cp) {
      const int tok = (mi & 1) * 8 + rr;
      const int chunk = cp * 2 + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3, vb + tok * 128 + ((chunk ^ (tok & 7)) << 4));
      mma_bf16_16816(o[2 * cp], pa, b0, b1);
      mma_bf16_16816(o[2 * cp + 1], pa, b2, b3);
    }
    __syncwarp();
    if (iss < gb1) {
      issue(iss, st);
      ++iss;
    }
    if (gi + 1 == seg_hi || gi + 1 == gb1) {
      finalize(i, seg_lo >= gb0 && seg_hi <= gb1);
      if (gi + 1 < gb1) {
        i = locate(gi + 1);
        seg_lo = cum[i];
        seg_hi = cum[i + 1];
        begin_request(i);
      }
    }
  }
}

// Merge the partials of requests whose blocks were split across CTAs.
// grid = (requests, q_heads), one thread per head-dim element.  A merge is
// latency-bound (a handful of loads per thread, each an L2 round trip that may
// cross the die boundary), so the loads are batched: the split bounds and the
// output row in one round trip, then (m, l, O) of up to CHUNK splits at once;
// the maximum is taken over the loaded values and the weighted sums run in
// split order.  More splits take one more round trip per CHUNK.  CHUNK 16
// needs twice the registers of CHUNK 8, so it is used only while the grid
// still fits on the GPU in one wave.
template <int CHUNK>
__global__ void __launch_bounds__(kDecHD, CHUNK <= 8 ? 14 : 8) decode_combine_kernel(DecodeArgs a) {
  constexpr int kChunk = CHUNK;
  pdl_trigger();  // the projection after the attention may be staged now (it waits for this grid)
  const int i = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int R = a.num_req;
  const int32_t* cum = a.cum_out;
  const int W = cum[R + 1];
  const int lo = cum[i], hi = cum[i + 1];
  const int req = a.req_list ? a.req_list[i] : i;
  if (hi <= lo || W <= 0) return;
  const int c0 = lo / W, c1 = (hi - 1) / W;
  if (c0 == c1) return;
  const int64_t qrow = a.q_rows ? a.q_rows[req] : (int64_t)req;
  const int64_t stride = (int64_t)a.hq * (kDecHD + 2);
  const float* base = a.partials + (int64_t)(c0 + i) * stride;
  const int n = c1 - c0 + 1;
  float mv[kChunk], lv[kChunk], ov[kChunk];
  auto load = [&](int c) {
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const float* ps = base + (int64_t)(c + j) * stride;
      const bool ok = c + j < n;
      mv[j] = ok ? ps[h] : -INFINITY;
      lv[j] = ok ? ps[a.hq + h] : 0.f;
      ov[j] = ok ? ps[2 * a.hq + h * kDecHD + d] : 0.f;
    }
  };
  load(0);
  float M = -INFINITY;
#pragma unroll
  for (int j = 0; j < kChunk; ++j) M = fmaxf(M, mv[j]);
  for (int c = kChunk; c < n; ++c) M = fmaxf(M, base[(int64_t)c * stride + h]);
  float L = 0.f, O = 0.f;
  for (int c = 0;;) {
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      if (c + j < n) {
        const float w = fast_exp2(mv[j] - M);
        L += lv[j] * w;
        O += ov[j] * w;
      }
    }
    c += kChunk;
    if (c >= n) break;
    load(c);
  }
  a.out[qrow * a.out_stride + (int64_t)h * kDecHD + d] = __float2bfloat16_rn(O / L);
}

static size_t ws_header_bytes(int R) { return (((size_t)(R + 2) * sizeof(int32_t)) + 255) & ~size_t(255); }

static size_t ws_bytes(int grid, int R, int hq) {
  return ws_header_bytes(R) + (size_t)(grid + R) * hq * (kDecHD + 2) * sizeof(float);
}

static int decode_stages(int hkv) { return hkv <= 8 ? kDecStages : kDecStagesWide; }

static size_t decode_smem_bytes(int hkv, int R) {
  const int nst = decode_stages(hkv);
  // tiles, barriers, then cum[R + 1], reqs[R] and trows[R]
  return 1024 + (size_t)hkv * nst * 2 * kTileBytes + (size_t)hkv * nst * 8 + (size_t)(3 * R + 1) * 4;
}

// Dynamic shared memory the decode CTA may use: the 227 KiB opt-in limit of
// sm_100 less a margin for the kernel's static shared memory.
constexpr size_t kMaxDynSmem = 232448 - 1024;

}  // namespace nie

using namespace nie;

extern "C" size_t nie_varlen_workspace_size(int32_t num_requests, int32_t max_query_len, int32_t max_seq_len,
                                            int32_t q_heads) {
  return prefill_workspace_bytes(num_requests, max_query_len, max_seq_len, q_heads);
}

extern "C" size_t nie_paged_decode_workspace_size(int device, int32_t R, int32_t q_heads, int32_t head_dim) {
  const int sms = sm_count(device);
  if (sms <= 0 || R <= 0 || q_heads <= 0) return 0;
  (void)head_dim;
  return ws_bytes(sms * kDecCtasPerSm, R, q_heads);
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shared body of nie_paged_decode and nie_paged_decode_overlapped; `overlap`
// lets the split-K kernel start while the kernel before it is still running.
static int paged_decode_impl(const void* q, int64_t q_row_stride, void* out, int64_t out_row_stride,
                             const void* key_cache, const void* value_cache, int32_t dtype, int32_t layer,
                             int64_t num_layers, int64_t num_blocks, int32_t block_size, int32_t kv_heads,
                             int32_t head_dim, int32_t q_heads, const int32_t* block_tables, int64_t table_stride,
                             const int32_t* table_rows, const int32_t* seq_lens, const int64_t* q_rows,
                             const int32_t* req_list, int32_t num_requests, float scale, void* workspace,
                             size_t workspace_bytes, int32_t* err_flag, void* stream, bool overlap) {
  NIE_REQUIRE(dtype_size(dtype) > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(q && out && key_cache && value_cache && block_tables && seq_lens, "null pointer argument");
  NIE_REQUIRE(layer >= 0 && layer < num_layers, "layer %d out of range", layer);
  NIE_REQUIRE(num_blocks > 0 && block_size > 0 && kv_heads > 0 && head_dim > 0 && q_heads > 0, "bad geometry");
  NIE_REQUIRE(q_heads % kv_heads == 0, "q_heads must be divisible by kv_heads");
  NIE_REQUIRE(num_requests >= 0, "num_requests must be non-negative");
  NIE_REQUIRE(table_stride > 0, "table_stride must be positive");
  if (num_requests == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int group = q_heads / kv_heads;
  const int dev = stream_device(s);
  const int sms = sm_count(dev);
  NIE_REQUIRE(sms > 0, "cannot query the SM count of device %d", dev);
  const int grid = sms * kDecCtasPerSm;
  const bool fast = dtype == NIE_DTYPE_BF16 && head_dim == kDecHD && block_size == kDecBS && group <= 16 &&
                    kv_heads <= 16 && num_requests <= kDecMaxReq && workspace != nullptr &&
                    workspace_bytes >= ws_bytes(grid, num_requests, q_heads) && aligned(q, 4) && aligned(out, 4) &&
                    (q_row_stride % 2) == 0 && (out_row_stride % 2) == 0 && aligned(key_cache, 16) &&
                    aligned(value_cache, 16) && aligned(workspace, 256) &&
                    num_blocks * kDecBS < (int64_t(1) << 31) &&
                    decode_smem_bytes(kv_heads, num_requests) <= kMaxDynSmem;
  if (!fast) {
    GenericArgs ga{};
    ga.q = q;
    ga.out = out;
    ga.q_stride = q_row_stride;
    ga.out_stride = out_row_stride;
    ga.kc = key_cache;
    ga.vc = value_cache;
    ga.layer = layer;
    ga.nb = num_blocks;
    ga.bs = block_size;
    ga.hkv = kv_heads;
    ga.hd = head_dim;
    ga.hq = q_heads;
    ga.tables = block_tables;
    ga.tstride = table_stride;
    ga.table_rows = table_rows;
    ga.seq_lens = seq_lens;
    ga.q_rows = q_rows;
    ga.qsl = nullptr;
    ga.req_list = req_list;
    ga.scale = scale;
    ga.err = err_flag;
    return launch_generic(dtype, ga, num_requests, 1, s);
  }

  const int64_t row_bytes = (int64_t)kv_heads * kDecHD * 2;
  const int64_t layer_bytes = num_blocks * kDecBS * row_bytes;
  CUtensorMap kmap, vmap;
  const uint64_t dims[3] = {(uint64_t)kDecHD, (uint64_t)kv_heads, (uint64_t)(num_blocks * kDecBS)};
  const uint64_t strides[2] = {(uint64_t)kDecHD * 2, (uint64_t)row_bytes};
  const uint32_t box[3] = {(uint32_t)kDecHD, 1u, (uint32_t)kDecBS};
  int rc = encode_tiled(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                        (void*)((const char*)key_cache + layer * layer_bytes), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != NIE_OK) return rc;
  rc = encode_tiled(&vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    (void*)((const char*)value_cache + layer * layer_bytes), dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != NIE_OK) return rc;

  DecodeArgs da{};
  da.q = (const __nv_bfloat16*)q;
  da.q_stride = q_row_stride;
  da.out = (__nv_bfloat16*)out;
  da.out_stride = out_row_stride;
  da.nb = num_blocks;
  da.hkv = kv_heads;
  da.hq = q_heads;
  da.group = group;
  da.tables = block_tables;
  da.tstride = table_stride;
  da.table_rows = table_rows;
  da.seq_lens = seq_lens;
  da.q_rows = q_rows;
  da.req_list = req_list;
  da.num_req = num_requests;
  da.scale = scale;
  da.cum_out = (int32_t*)workspace;
  da.partials = (float*)((char*)workspace + ws_header_bytes(num_requests));
  da.err = err_flag;

  const size_t smem = decode_smem_bytes(kv_heads, num_requests);
  const bool wide = decode_stages(kv_heads) != kDecStages;
  auto* kernel = wide ? decode_tma_kernel<kDecStagesWide> : decode_tma_kernel<kDecStages>;
  rc = opt_in_smem(wide ? kSmemDecodeWide : kSmemDecode, (const void*)kernel, smem);
  if (rc != NIE_OK) return rc;
  if (overlap) {
    // dependent launch: the prologue overlaps the kernel before it (the RoPE +
    // KV write), whose outputs are read only after pdl_wait()
    const cudaError_t le = launch_after_trigger(kernel, dim3(grid), dim3(kv_heads * 32), smem, s, kmap, vmap, da);
    if (le != cudaSuccess) return fail(NIE_ERR_CUDA, "decode_tma_kernel launch: %s", cudaGetErrorString(le));
  } else {
    kernel<<<grid, kv_heads * 32, smem, s>>>(kmap, vmap, da);
    rc = check_launch("decode_tma_kernel");
    if (rc != NIE_OK) return rc;
  }
  // 16-split batches while (requests x heads) CTAs of 64 threads at ~128
  // registers fit in one wave (8 per SM), 8-split batches beyond
  const dim3 cgrid((unsigned)num_requests, (unsigned)q_heads);
  if ((int64_t)num_requests * q_heads <= (int64_t)sms * 8)
    decode_combine_kernel<16><<<cgrid, kDecHD, 0, s>>>(da);
  else
    decode_combine_kernel<8><<<cgrid, kDecHD, 0, s>>>(da);
  return check_launch("decode_combine_kernel");
}

extern "C" int nie_paged_decode(const void* q, int64_t q_row_stride, void* out, int64_t out_row_stride,
                                const void* key_cache, const void* value_cache, int32_t dtype, int32_t layer,
                                int64_t num_layers, int64_t num_blocks, int32_t block_size, int32_t kv_heads,
                                int32_t head_dim, int32_t q_heads, const int32_t* block_tables, int64_t table_stride,
                                const int32_t* table_rows, const int32_t* seq_lens, const int64_t* q_rows,
                                const int32_t* req_list, int32_t num_requests, float scale, void* workspace,
                                size_t workspace_bytes, int32_t* err_flag, void* stream) {
  return paged_decode_impl(q, q_row_stride, out, out_row_stride, key_cache, value_cache, dtype, layer, num_layers,
                           num_blocks, block_size, kv_heads, head_dim, q_heads, block_tables, table_stride,
                           table_rows, seq_lens, q_rows, req_list, num_requests, scale, workspace, workspace_bytes,
                           err_flag, stream, false);
}

extern "C" int nie_paged_decode_overlapped(const void* q, int64_t q_row_stride, void* out, int64_t out_row_stride,
                                           const void* key_cache, const void* value_cache, int32_t dtype,
                                           int32_t layer, int64_t num_layers, int64_t num_blocks, int32_t block_size,
                                           int32_t kv_heads, int32_t head_dim, int32_t q_heads,
                                           const int32_t* block_tables, int64_t table_stride,
                                           const int32_t* table_rows, const int32_t* seq_lens, const int64_t* q_rows,
                                           const int32_t* req_list, int32_t num_requests, float scale,
                                           void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream) {
  return paged_decode_impl(q, q_row_stride, out, out_row_stride, key_cache, value_cache, dtype, layer, num_layers,
                           num_blocks, block_size, kv_heads, head_dim, q_heads, block_tables, table_stride,
                           table_rows, seq_lens, q_rows, req_list, num_requests, scale, workspace, workspace_bytes,
                           err_flag, stream, true);
}

extern "C" int nie_varlen_attention(const void* q, void* out, int64_t row_stride, int64_t num_q_rows,
                                    const void* key_cache,
                                    const void* value_cache, int32_t dtype, int32_t layer, int64_t num_layers,
                                    int64_t num_blocks, int32_t block_size, int32_t kv_heads, int32_t head_dim,
                                    int32_t q_heads, const int32_t* block_tables, int64_t table_stride,
                                    const int32_t* table_rows, const int32_t* seq_lens,
                                    const int64_t* query_start_loc, const int32_t* req_list, int32_t num_requests,
                                    int32_t max_query_len, int32_t max_seq_len, float scale, void* workspace,
                                    size_t workspace_bytes, int32_t* err_flag, void* stream) {
  NIE_REQUIRE(dtype_size(dtype) > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(q && out && key_cache && value_cache && block_tables && seq_lens && query_start_loc,
              "null pointer argument");
  NIE_REQUIRE(layer >= 0 && layer < num_layers, "layer %d out of range", layer);
  NIE_REQUIRE(num_blocks > 0 && block_size > 0 && kv_heads > 0 && head_dim > 0 && q_heads > 0, "bad geometry");
  NIE_REQUIRE(q_heads % kv_heads == 0, "q_heads must be divisible by kv_heads");
  NIE_REQUIRE(num_requests >= 0, "num_requests must be non-negative");
  NIE_REQUIRE(num_q_rows >= 0, "num_q_rows must be non-negative");
  if (num_requests == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == NIE_DTYPE_BF16 && head_dim == 64 && block_size == 16 && max_query_len > 0) {
    const int rc = launch_prefill_tc(q, out, row_stride, num_q_rows, key_cache, value_cache, layer, num_blocks,
                                     kv_heads, q_heads, block_tables, table_stride, table_rows, seq_lens,
                                     query_start_loc, req_list, num_requests, max_query_len, max_seq_len, scale,
                                     workspace, workspace_bytes, err_flag, s);
    if (rc != NIE_ERR_UNSUPPORTED) return rc;
  }
  GenericArgs ga{};
  ga.q = q;
  ga.out = out;
  ga.q_stride = row_stride;
  ga.out_stride = row_stride;
  ga.kc = key_cache;
  ga.vc = value_cache;
  ga.layer = layer;
  ga.nb = num_blocks;
  ga.bs = block_size;
  ga.hkv = kv_heads;
  ga.hd = head_dim;
  ga.hq = q_heads;
  ga.tables = block_tables;
  ga.tstride = table_stride;
  ga.table_rows = table_rows;
  ga.seq_lens = seq_lens;
  ga.q_rows = nullptr;
  ga.qsl = query_start_loc;
  ga.req_list = req_list;
  ga.scale = scale;
  ga.err = err_flag;
  return launch_generic(dtype, ga, num_requests, max_query_len, s);
}

// ------------------------------------------------- allocation-free decode
// Scratch of nie_paged_decode_noalloc: a fixed array in device memory that
// every GPU loading this library holds until the process exits.  Host code
// must never hand this symbol to a kernel directly (on the host it is only a
// stand-in, not a device address); the address comes from
// cudaGetSymbolAddress, resolved once per device below.
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[NIE_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
constexpr int kNoallocMaxDevices = NIE_DECODE_NOALLOC_MAX_DEVICES;
void* g_noalloc_ptr[kNoallocMaxDevices] = {nullptr};

// Resolve the device address of the scratch array on `device`, which must be
// the current device.  Runs once per device (the first call on that device).
int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= kNoallocMaxDevices)
    return nie::fail(NIE_ERR_INVALID, "nie_paged_decode_noalloc: device ordinal %d outside 0..%d", device,
                     kNoallocMaxDevices - 1);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return nie::fail(NIE_ERR_CUDA, "cudaGetSymbolAddress(decode scratch) on device %d: %s", device,
                       cudaGetErrorString(e));
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return NIE_OK;
}
}  // namespace

extern "C" size_t nie_paged_decode_noalloc_capacity(void) { return NIE_DECODE_NOALLOC_SCRATCH_BYTES; }

extern "C" int nie_paged_decode_noalloc(const void* q, int64_t q_row_stride, void* out, int64_t out_row_stride,
                                        const void* key_cache, const void* value_cache, int32_t dtype, int32_t layer,
                                        int64_t num_layers, int64_t num_blocks, int32_t block_size, int32_t kv_heads,
                                        int32_t head_dim, int32_t q_heads, const int32_t* block_tables,
                                        int64_t table_stride, const int32_t* table_rows, const int32_t* seq_lens,
                                        const int64_t* q_rows, const int32_t* req_list, int32_t num_requests,
                                        float scale, int32_t* err_flag, void* stream) {
  NIE_REQUIRE(num_requests >= 0 && q_heads > 0, "num_requests must be non-negative and q_heads positive");
  if (num_requests == 0)  // argument checks only: an empty batch never touches (or resolves) the scratch
    return nie_paged_decode(q, q_row_stride, out, out_row_stride, key_cache, value_cache, dtype, layer, num_layers,
                            num_blocks, block_size, kv_heads, head_dim, q_heads, block_tables, table_stride,
                            table_rows, seq_lens, q_rows, req_list, 0, scale, nullptr, 0, err_flag, stream);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int dev = stream_device(s);
  const int sms = sm_count(dev);
  NIE_REQUIRE(sms > 0, "cannot query the SM count of device %d", dev);
  const size_t need = ws_bytes(sms * kDecCtasPerSm, num_requests, q_heads);
  if (need > (size_t)NIE_DECODE_NOALLOC_SCRATCH_BYTES)
    return fail(NIE_ERR_INVALID,
                "nie_paged_decode_noalloc: %d requests x %d query heads need %zu bytes of scratch, above the "
                "fixed %d-byte array; use nie_paged_decode with a caller-provided workspace",
                num_requests, q_heads, need, NIE_DECODE_NOALLOC_SCRATCH_BYTES);
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(NIE_ERR_CUDA, "cudaGetDevice failed");
  if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return fail(NIE_ERR_CUDA, "cudaSetDevice(%d) failed", dev);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(dev, &scratch);
  if (prev != dev) cudaSetDevice(prev);
  if (rc != NIE_OK) return rc;
  return nie_paged_decode(q, q_row_stride, out, out_row_stride, key_cache, value_cache, dtype, layer, num_layers,
                          num_blocks, block_size, kv_heads, head_dim, q_heads, block_tables, table_stride, table_rows,
                          seq_lens, q_rows, req_list, num_requests, scale, scratch,
                          (size_t)NIE_DECODE_NOALLOC_SCRATCH_BYTES, err_flag, stream);
}
