// (d) Varlen causal attention over the paged cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), bf16 / head_dim 64 / block_size 16.
//
// One CTA computes one (128-query tile of one request, one query head):
//
//   warp 4  TMA producer   Q tile once (128 rows x 128 B), then per 128-key
//                          tile 8+8 block loads of K and V rows of the kv
//                          head (2 KiB each, 128-byte swizzle) into a
//                          4-stage ring; blocks past the needed keys are
//                          fetched out of bounds, i.e. as zeros.
//   warp 5  MMA issuer     one thread issues S_j = Q K_j^T (M=128, N=128,
//                          4 x K=16) into TMEM and, once softmax has written
//                          P_j, O_j = P_j V_j (M=128, N=64, 8 x K=16, A = P
//                          read from TMEM, V as an MN-major operand).  S and
//                          O use two TMEM buffers each, so S_{j+1} runs while
//                          softmax works on S_j.
//   warps 0-3 softmax      thread t owns query row t: reads its S row from
//                          TMEM, applies the causal mask and the reference's
//                          rounding (score = bf16(bf16(q.k) * scale)),
//                          online max / sum in fp32, writes P as bf16 pairs
//                          back over the S columns (the A operand of the PV
//                          MMA), and accumulates O_j into fp32 registers with
//                          the running rescale.  Epilogue: O / l -> bf16.
//
// Waits are bounded: a wait that runs out raises NIE_DEV_ERR_TIMEOUT, the
// CTA stops issuing work, drains what is in flight and frees its TMEM.
#include "nie_attn.cuh"

namespace nie {

constexpr int kPfBM = 128;
constexpr int kPfBN = 128;
constexpr int kPfHD = 64;
constexpr int kPfBS = 16;
constexpr int kPfStages = 4;
constexpr int kPfThreads = 192;
constexpr uint32_t kPfTmemCols = 512;
constexpr uint32_t kPfWait = 1u << 22;
constexpr int kPfTile = kPfBN * kPfHD * 2;  // 16 KiB: 128 rows x 128 B
constexpr uint32_t kSCol0 = 0, kSCol1 = 128, kOCol0 = 256, kOCol1 = 320;
constexpr float kPfLog2e = 1.4426950408889634f;

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
  float scale;
  int32_t* err;
};

struct PfBars {
  uint64_t q_full;
  uint64_t kv_full[kPfStages];
  uint64_t kv_empty[kPfStages];
  uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float pf_score(uint32_t raw, float scale) {
  const float s = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(__uint_as_float(raw))) *
                                                       scale));
  return s * kPfLog2e;
}

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

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, PrefillArgs a) {
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm;
  uint8_t* skv = sm + kPfTile;
  PfBars* b = reinterpret_cast<PfBars*>(skv + kPfStages * 2 * kPfTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item (uniform across the CTA, decided before any barrier)
  const int item = blockIdx.x / a.tiles_per_req, tile = blockIdx.x % a.tiles_per_req;
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
  const int n_kt = (n_keys + kPfBN - 1) / kPfBN;
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
      mbar_init(&b->o_full[i], 1);
      mbar_init(&b->o_empty[i], kPfBM);
    }
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
      mbar_arrive_expect_tx(&b->q_full, kPfTile);
      tma_load_3d(sq, &qmap, &b->q_full, 0, h, (int)(qs + q0));
    }
    int issued = 0;
    for (int kt = 0; kt < n_kt; ++kt) {
      const int st = kt % kPfStages;
      if (kt >= kPfStages && !pf_wait(b, &b->kv_empty[st], (uint32_t)((kt - kPfStages) / kPfStages) & 1u, a.err))
        break;
      int coord = (int)(a.nb * kPfBS);  // out of bounds: zero fill
      if (lane < 8) {
        const int lb = kt * 8 + lane;
        if (lb * kPfBS < n_keys) {
          int64_t blk = (lb < a.tstride) ? (int64_t)a.tables[(int64_t)trow * a.tstride + lb] : -1;
          if (blk < 0 || blk >= a.nb) {
            raise_flag(a.err, NIE_DEV_ERR_BLOCK_RANGE);
            blk = 0;
          }
          coord = (int)(blk * kPfBS);
        }
      }
      if (lane == 0) mbar_arrive_expect_tx(&b->kv_full[st], 2 * kPfTile);
      __syncwarp();
      if (lane < 8) {
        uint8_t* dst = skv + st * 2 * kPfTile + lane * (kPfBS * kPfHD * 2);
        tma_load_3d(dst, &kmap, &b->kv_full[st], 0, kvh, coord);
        tma_load_3d(dst + kPfTile, &vmap, &b->kv_full[st], 0, kvh, coord);
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

    auto do_pv = [&](int j) -> bool {
      const int sb = j & 1;
      if (!pf_wait(b, &b->p_full[sb], (uint32_t)(j >> 1) & 1u, a.err)) return false;
      if (j >= 2 && !pf_wait(b, &b->o_empty[sb], (uint32_t)((j - 2) >> 1) & 1u, a.err)) return false;
      const int st = j % kPfStages;
      uint8_t* vt = skv + st * 2 * kPfTile + kPfTile;
      if (tail != 0 && last_lb / 8 == j && last_lb * kPfBS < n_keys) {
        // stale rows past the sequence end (possibly NaN) must not meet P = 0
        uint4* z = reinterpret_cast<uint4*>(vt + (last_lb % 8) * (kPfBS * kPfHD * 2) + tail * (kPfHD * 2));
        for (int c = lane; c < (kPfBS - tail) * 8; c += 32) z[c] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
      }
      __syncwarp();
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(vt);
        const uint32_t d = tbase + (sb ? kOCol1 : kOCol0);
        const uint32_t p = tbase + (sb ? kSCol1 : kSCol0);
#pragma unroll
        for (int k = 0; k < kPfBN / 16; ++k)
          tc_mma_ts(d, p + k * 8, smem_desc_sw128(v_addr + k * 2048, kPfTile, 1024), id_pv, k > 0 ? 1u : 0u);
        tc_commit(&b->o_full[sb]);
        tc_commit(&b->kv_empty[st]);
      }
      __syncwarp();
      return true;
    };

    for (int kt = 0; ok && kt < n_kt; ++kt) {
      const int st = kt % kPfStages, sb = kt & 1;
      if (!pf_wait(b, &b->kv_full[st], (uint32_t)(kt / kPfStages) & 1u, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(skv + st * 2 * kPfTile);
        const uint32_t d = tbase + (sb ? kSCol1 : kSCol0);
#pragma unroll
        for (int k = 0; k < kPfHD / 16; ++k)
          tc_mma_ss(d, smem_desc_sw128(q_addr + k * 32, 16, 1024), smem_desc_sw128(k_addr + k * 32, 16, 1024), id_s,
                    k > 0 ? 1u : 0u);
        tc_commit(&b->s_full[sb]);
      }
      __syncwarp();
      if (kt >= 1 && !do_pv(kt - 1)) ok = false;
    }
    if (ok && n_kt > 0) do_pv(n_kt - 1);
    if (lane == 0) tc_commit(&b->done);
    __syncwarp();
    mbar_wait_bounded(&b->done, 0, kPfWait);
  } else {
    // -------------------------------------------------- softmax warps
    const int t = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int qpos = ctx + q0 + t;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    float acc[kPfHD];
#pragma unroll
    for (int c = 0; c < kPfHD; ++c) acc[c] = 0.f;
    bool ok = true;

    auto finish_o = [&](int j, float alpha) -> bool {
      const int sb = j & 1;
      if (!pf_wait(b, &b->o_full[sb], (uint32_t)(j >> 1) & 1u, a.err)) return false;
      tc_fence_after();
      uint32_t v[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tbase + lane_off + (sb ? kOCol1 : kOCol0) + 32 * half, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[32 * half + c] = acc[32 * half + c] * alpha + __uint_as_float(v[c]);
      }
      tc_fence_before();
      mbar_arrive(&b->o_empty[sb]);
      return true;
    };

    for (int kt = 0; kt < n_kt; ++kt) {
      const int sb = kt & 1;
      if (!pf_wait(b, &b->s_full[sb], (uint32_t)(kt >> 1) & 1u, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tbase + lane_off + (sb ? kSCol1 : kSCol0);
      const int key0 = kt * kPfBN;
      uint32_t v[32];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(s_addr + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float x = (key0 + 32 * c + e <= qpos) ? pf_score(v[e], a.scale) : -INFINITY;
          mx = fmaxf(mx, x);
        }
      }
      const float mn = fmaxf(m, mx);
      const float alpha = fast_exp2(m - mn);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(s_addr + 32 * c, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int k0 = key0 + 32 * c + 2 * e;
          const float x0 = (k0 <= qpos) ? pf_score(v[2 * e], a.scale) : -INFINITY;
          const float x1 = (k0 + 1 <= qpos) ? pf_score(v[2 * e + 1], a.scale) : -INFINITY;
          const float p0 = fast_exp2(x0 - mn), p1 = fast_exp2(x1 - mn);
          rs += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        tmem_st16(s_addr + 16 * c, pk);
      }
      tmem_wait_st();
      l = l * alpha + rs;
      m = mn;
      tc_fence_before();
      mbar_arrive(&b->p_full[sb]);
      if (kt >= 1 && !finish_o(kt - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && n_kt > 0) ok = finish_o(n_kt - 1, alpha_prev);
    if (ok && t < nq) {
      const float inv = 1.f / l;
      __nv_bfloat16* op = a.out + (qs + q0 + t) * a.out_stride + (int64_t)h * kPfHD;
#pragma unroll
      for (int c = 0; c < kPfHD / 8; ++c) {
        uint4 w;
        w.x = pack_bf16x2(acc[8 * c + 0] * inv, acc[8 * c + 1] * inv);
        w.y = pack_bf16x2(acc[8 * c + 2] * inv, acc[8 * c + 3] * inv);
        w.z = pack_bf16x2(acc[8 * c + 4] * inv, acc[8 * c + 5] * inv);
        w.w = pack_bf16x2(acc[8 * c + 6] * inv, acc[8 * c + 7] * inv);
        *reinterpret_cast<uint4*>(op + 8 * c) = w;
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

static size_t prefill_smem_bytes() { return 1024 + kPfTile + (size_t)kPfStages * 2 * kPfTile + sizeof(PfBars); }

// Returns NIE_ERR_UNSUPPORTED when the shape is not the tensor-core one, so
// the caller can use the generic kernel.
int launch_prefill_tc(const void* q, void* out, int64_t row_stride, int64_t num_q_rows, const void* key_cache,
                      const void* value_cache, int32_t layer, int64_t num_blocks, int32_t kv_heads, int32_t q_heads,
                      const int32_t* block_tables, int64_t table_stride, const int32_t* table_rows,
                      const int32_t* seq_lens, const int64_t* qsl, const int32_t* req_list, int32_t num_requests,
                      int32_t max_query_len, float scale, int32_t* err_flag, cudaStream_t s) {
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
  pa.scale = scale;
  pa.err = err_flag;
  const size_t smem = prefill_smem_bytes();
  static thread_local bool s_attr = false;
  if (!s_attr) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NIE_ERR_CUDA, "prefill smem %zu: %s", smem, cudaGetErrorString(e));
    s_attr = true;
  }
  const int64_t gx = (int64_t)num_requests * pa.tiles_per_req;
  if (gx >= (int64_t(1) << 31)) return NIE_ERR_UNSUPPORTED;
  dim3 grid((unsigned)gx, (unsigned)q_heads);
  prefill_tc_kernel<<<grid, kPfThreads, smem, s>>>(qmap, kmap, vmap, pa);
  return check_launch("prefill_tc_kernel");
}

}  // namespace nie
