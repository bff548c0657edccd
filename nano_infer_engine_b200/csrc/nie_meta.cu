// (a) ragged batch packing, (b) paged KV slot write, the paged gather, and
// (e) block copies between paged pools (export / import / NVLink handoff).
// All of these are integer or byte-moving work: the kernels are sized for
// coalesced 16-byte accesses and carry no tensor-core code.
#include "nie_common.cuh"

namespace nie {

// ------------------------------------------------------------------ packing
constexpr int kPackThreads = 256;
constexpr int kPackMaxRequests = 8192;

// Exclusive block-wide scan of `vals` (length n, in shared memory) in place;
// returns the total.  Each thread scans a contiguous chunk, then the chunk
// sums are scanned with warp shuffles.
__device__ int block_exclusive_scan(int* vals, int n, int* warp_tot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kPackThreads - 1) / kPackThreads;
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
    int w = (lane < kPackThreads / 32) ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < kPackThreads / 32) warp_tot[lane] = wi - w;  // exclusive warp offsets
    if (lane == kPackThreads / 32 - 1) warp_tot[kPackThreads / 32] = wi;
  }
  __syncthreads();
  int run = warp_tot[warp] + incl - local;
  for (int i = b; i < e; ++i) {
    int v = vals[i];
    vals[i] = run;
    run += v;
  }
  int total = warp_tot[kPackThreads / 32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kPackThreads) pack_ragged_kernel(
    const int32_t* __restrict__ plan, int R, int64_t T, const int32_t* __restrict__ tables, int64_t stride, int bs,
    int64_t num_blocks, int64_t* __restrict__ qsl, int64_t* __restrict__ positions, int64_t* __restrict__ slots,
    int32_t* __restrict__ seq_lens, int64_t* __restrict__ last_idx, int32_t* __restrict__ tok_req,
    int32_t* __restrict__ dec_list, int32_t* __restrict__ pf_list, int32_t* __restrict__ counts,
    int32_t* __restrict__ err) {
  extern __shared__ int sh[];
  int* start = sh;                 // [R+1] exclusive prefix of query lengths
  int* dpre = sh + (R + 1);        // [R+1] exclusive prefix of (qlen == 1)
  __shared__ int warp_tot[kPackThreads / 32 + 1];

  for (int r = threadIdx.x; r < R; r += kPackThreads) {
    int ql = plan[2 * R + r];
    start[r] = ql;
    dpre[r] = (ql == 1) ? 1 : 0;
  }
  __syncthreads();
  const int total = block_exclusive_scan(start, R, warp_tot);
  const int ndec = block_exclusive_scan(dpre, R, warp_tot);
  if (threadIdx.x == 0) {
    start[R] = total;
    dpre[R] = ndec;
  }
  __syncthreads();

  if (blockIdx.x == 0) {
    for (int r = threadIdx.x; r < R; r += kPackThreads) {
      const int ctx = plan[R + r], ql = plan[2 * R + r];
      qsl[r] = start[r];
      seq_lens[r] = ctx + ql;
      if (last_idx) last_idx[r] = (int64_t)start[r + 1] - 1;
      if (ql == 1) {
        if (dec_list) dec_list[dpre[r]] = r;
      } else {
        if (pf_list) pf_list[r - dpre[r]] = r;
      }
    }
    if (threadIdx.x == 0) {
      qsl[R] = total;
      if (counts) {
        counts[0] = ndec;
        counts[1] = R - ndec;
      }
    }
  }

  const int64_t t = (int64_t)blockIdx.x * kPackThreads + threadIdx.x;
  if (t >= T || t >= total) return;
  // upper_bound(start[0..R], t) - 1
  int lo = 0, hi = R;  // invariant: start[lo] <= t < start[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (start[mid] <= t) lo = mid; else hi = mid;
  }
  const int r = lo;
  const int row = plan[r], ctx = plan[R + r];
  const int64_t pos = (int64_t)ctx + (t - start[r]);
  positions[t] = pos;
  if (tok_req) tok_req[t] = r;
  const int64_t lb = pos / bs;
  int64_t slot = -1;
  if (lb >= stride || row < 0) {
    raise_flag(err, NIE_DEV_ERR_CAPACITY);
  } else {
    const int64_t blk = tables[(int64_t)row * stride + lb];
    if (blk < 0 || blk >= num_blocks) raise_flag(err, NIE_DEV_ERR_BLOCK_RANGE);
    else slot = blk * bs + pos % bs;
  }
  slots[t] = slot;
}

// --------------------------------------------------------------- slot write
// One warp per token row; V is the widest vector type the row size and the
// base pointers allow (16 bytes for the Llama shape: 64 vectors per 1 KiB row).
template <typename V>
__global__ void write_kv_kernel(const V* __restrict__ k, const V* __restrict__ v, V* __restrict__ kc,
                                V* __restrict__ vc, int64_t T, int64_t nvec, int64_t layer_off, int64_t total_slots,
                                const int64_t* __restrict__ slots, int32_t* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    const int64_t s = slots[t];
    if (s < 0) continue;  // packing already flagged it
    if (s >= total_slots) {
      if (lane == 0) raise_flag(err, NIE_DEV_ERR_SLOT_RANGE);
      continue;
    }
    const V* ks = k + t * nvec;
    const V* vs = v + t * nvec;
    V* kd = kc + layer_off + s * nvec;
    V* vd = vc + layer_off + s * nvec;
    for (int64_t i = lane; i < nvec; i += 32) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
}

template <typename V>
__global__ void gather_kv_kernel(const V* __restrict__ kc, const V* __restrict__ vc, V* __restrict__ ok,
                                 V* __restrict__ ov, int64_t T, int64_t nvec, int64_t layer_off, int bs,
                                 int64_t num_blocks, const int32_t* __restrict__ table, int32_t* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    const int64_t blk = table[t / bs];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) raise_flag(err, NIE_DEV_ERR_BLOCK_RANGE);
      continue;
    }
    const int64_t s = blk * bs + t % bs;
    for (int64_t i = lane; i < nvec; i += 32) {
      ok[t * nvec + i] = kc[layer_off + s * nvec + i];
      ov[t * nvec + i] = vc[layer_off + s * nvec + i];
    }
  }
}

// -------------------------------------------------------------- block copy
// grid = (num_copy_blocks, num_layers, 2): one CTA moves one [bs, H, D] block
// of K (z = 0) or V (z = 1).  Rows at or past `tail_valid` of the last block
// are written as zeros.
template <typename V>
__global__ void __launch_bounds__(256) copy_blocks_kernel(
    const V* __restrict__ sk, const V* __restrict__ sv, int64_t src_nb, const int32_t* __restrict__ src_ids,
    V* __restrict__ dk, V* __restrict__ dv, int64_t dst_nb, const int32_t* __restrict__ dst_ids, int64_t n,
    int tail_valid, int bs, int64_t row_vec, int32_t* __restrict__ err) {
  const int64_t j = blockIdx.x;
  const int64_t l = blockIdx.y;
  const V* src = blockIdx.z == 0 ? sk : sv;
  V* dst = blockIdx.z == 0 ? dk : dv;
  const int64_t sb = src_ids ? (int64_t)src_ids[j] : j;
  const int64_t db = dst_ids ? (int64_t)dst_ids[j] : j;
  if (sb < 0 || sb >= src_nb || db < 0 || db >= dst_nb) {
    if (threadIdx.x == 0) raise_flag(err, NIE_DEV_ERR_BLOCK_RANGE);
    return;
  }
  const int64_t blk_vec = (int64_t)bs * row_vec;
  const V* s = src + (l * src_nb + sb) * blk_vec;
  V* d = dst + (l * dst_nb + db) * blk_vec;
  const int64_t zero_from = (j == n - 1 && tail_valid > 0 && tail_valid < bs) ? (int64_t)tail_valid * row_vec : blk_vec;
  for (int64_t i = threadIdx.x; i < blk_vec; i += blockDim.x) {
    V x;
    if (i < zero_from) x = s[i];
    else memset(&x, 0, sizeof(V));
    d[i] = x;
  }
}

static int vec_width(int64_t row_bytes, std::initializer_list<const void*> ptrs) {
  int w = 16;
  while (w > 2) {
    bool ok = (row_bytes % w) == 0;
    for (const void* p : ptrs) ok = ok && ((reinterpret_cast<uintptr_t>(p) % w) == 0);
    if (ok) break;
    w >>= 1;
  }
  return w;
}

}  // namespace nie

using namespace nie;

extern "C" int nie_pack_ragged(const int32_t* plan, int32_t R, int64_t T, const int32_t* block_tables,
                               int64_t table_stride, int32_t block_size, int64_t num_blocks, int64_t* qsl,
                               int64_t* positions, int64_t* slot_mapping, int32_t* seq_lens, int64_t* last_idx,
                               int32_t* tok_req, int32_t* dec_list, int32_t* pf_list, int32_t* counts,
                               int32_t* err_flag, void* stream) {
  NIE_REQUIRE(R > 0 && R <= kPackMaxRequests, "num_requests must be in [1, %d], got %d", kPackMaxRequests, R);
  NIE_REQUIRE(T > 0 && T < (int64_t(1) << 31), "num_tokens out of range: %lld", (long long)T);
  NIE_REQUIRE(plan && block_tables && qsl && positions && slot_mapping && seq_lens, "null pointer argument");
  NIE_REQUIRE(block_size > 0 && num_blocks > 0 && table_stride > 0, "bad cache geometry");
  const int grid = (int)((T + kPackThreads - 1) / kPackThreads);
  const size_t smem = 2 * (size_t)(R + 1) * sizeof(int);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(pack_ragged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  pack_ragged_kernel<<<grid, kPackThreads, smem, s>>>(plan, R, T, block_tables, table_stride, block_size, num_blocks,
                                                       qsl, positions, slot_mapping, seq_lens, last_idx, tok_req,
                                                       dec_list, pf_list, counts, err_flag);
  return check_launch("pack_ragged_kernel");
}

template <typename V>
static void launch_write(const void* k, const void* v, int64_t T, void* kc, void* vc, int64_t row_bytes,
                         int64_t layer_off_bytes, int64_t total_slots, const int64_t* slots, int32_t* err,
                         cudaStream_t s) {
  const int64_t nvec = row_bytes / sizeof(V);
  const int warps_per_cta = 8;
  int64_t grid = (T + warps_per_cta - 1) / warps_per_cta;
  if (grid > 65535 * 8) grid = 65535 * 8;
  write_kv_kernel<V><<<(unsigned)grid, warps_per_cta * 32, 0, s>>>(
      (const V*)k, (const V*)v, (V*)kc, (V*)vc, T, nvec, layer_off_bytes / (int64_t)sizeof(V), total_slots, slots,
      err);
}

extern "C" int nie_write_kv(const void* keys, const void* values, int64_t T, void* key_cache, void* value_cache,
                            int32_t dtype, int32_t layer, int64_t num_layers, int64_t num_blocks, int32_t block_size,
                            int32_t kv_heads, int32_t head_dim, const int64_t* slot_mapping, int32_t* err_flag,
                            void* stream) {
  const int es = dtype_size(dtype);
  NIE_REQUIRE(es > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(T >= 0, "num_tokens must be non-negative");
  NIE_REQUIRE(layer >= 0 && layer < num_layers, "layer %d out of range", layer);
  NIE_REQUIRE(keys && values && key_cache && value_cache && slot_mapping, "null pointer argument");
  NIE_REQUIRE(block_size > 0 && kv_heads > 0 && head_dim > 0 && num_blocks > 0, "bad cache geometry");
  if (T == 0) return NIE_OK;
  const int64_t row_bytes = (int64_t)kv_heads * head_dim * es;
  const int64_t slots_per_layer = num_blocks * block_size;
  const int64_t layer_off = (int64_t)layer * slots_per_layer * row_bytes;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = vec_width(row_bytes, {keys, values, key_cache, value_cache});
  switch (w) {
    case 16: launch_write<uint4>(keys, values, T, key_cache, value_cache, row_bytes, layer_off, slots_per_layer, slot_mapping, err_flag, s); break;
    case 8: launch_write<uint2>(keys, values, T, key_cache, value_cache, row_bytes, layer_off, slots_per_layer, slot_mapping, err_flag, s); break;
    case 4: launch_write<uint32_t>(keys, values, T, key_cache, value_cache, row_bytes, layer_off, slots_per_layer, slot_mapping, err_flag, s); break;
    default: launch_write<uint16_t>(keys, values, T, key_cache, value_cache, row_bytes, layer_off, slots_per_layer, slot_mapping, err_flag, s); break;
  }
  return check_launch("write_kv_kernel");
}

template <typename V>
static void launch_gather(const void* kc, const void* vc, void* ok, void* ov, int64_t T, int64_t row_bytes,
                          int64_t layer_off_bytes, int bs, int64_t nb, const int32_t* table, int32_t* err,
                          cudaStream_t s) {
  const int64_t nvec = row_bytes / sizeof(V);
  int64_t grid = (T + 7) / 8;
  if (grid > 65535 * 8) grid = 65535 * 8;
  gather_kv_kernel<V><<<(unsigned)grid, 256, 0, s>>>((const V*)kc, (const V*)vc, (V*)ok, (V*)ov, T, nvec,
                                                      layer_off_bytes / (int64_t)sizeof(V), bs, nb, table, err);
}

extern "C" int nie_gather_kv(const void* key_cache, const void* value_cache, int32_t dtype, int32_t layer,
                             int64_t num_layers, int64_t num_blocks, int32_t block_size, int32_t kv_heads,
                             int32_t head_dim, const int32_t* block_table, int64_t T, void* out_keys,
                             void* out_values, int32_t* err_flag, void* stream) {
  const int es = dtype_size(dtype);
  NIE_REQUIRE(es > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(layer >= 0 && layer < num_layers, "layer %d out of range", layer);
  NIE_REQUIRE(key_cache && value_cache && block_table && out_keys && out_values, "null pointer argument");
  if (T <= 0) return NIE_OK;
  const int64_t row_bytes = (int64_t)kv_heads * head_dim * es;
  const int64_t layer_off = (int64_t)layer * num_blocks * block_size * row_bytes;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = vec_width(row_bytes, {key_cache, value_cache, out_keys, out_values});
  switch (w) {
    case 16: launch_gather<uint4>(key_cache, value_cache, out_keys, out_values, T, row_bytes, layer_off, block_size, num_blocks, block_table, err_flag, s); break;
    case 8: launch_gather<uint2>(key_cache, value_cache, out_keys, out_values, T, row_bytes, layer_off, block_size, num_blocks, block_table, err_flag, s); break;
    case 4: launch_gather<uint32_t>(key_cache, value_cache, out_keys, out_values, T, row_bytes, layer_off, block_size, num_blocks, block_table, err_flag, s); break;
    default: launch_gather<uint16_t>(key_cache, value_cache, out_keys, out_values, T, row_bytes, layer_off, block_size, num_blocks, block_table, err_flag, s); break;
  }
  return check_launch("gather_kv_kernel");
}

template <typename V>
static void launch_copy(const void* sk, const void* sv, int64_t snb, const int32_t* sids, void* dk, void* dv,
                        int64_t dnb, const int32_t* dids, int64_t n, int tail, int64_t L, int bs, int64_t row_bytes,
                        int32_t* err, cudaStream_t s) {
  dim3 grid((unsigned)n, (unsigned)L, 2);
  copy_blocks_kernel<V><<<grid, 256, 0, s>>>((const V*)sk, (const V*)sv, snb, sids, (V*)dk, (V*)dv, dnb, dids, n,
                                              tail, bs, row_bytes / (int64_t)sizeof(V), err);
}

extern "C" int nie_copy_blocks(const void* src_keys, const void* src_values, int64_t src_num_blocks,
                               const int32_t* src_blocks, void* dst_keys, void* dst_values, int64_t dst_num_blocks,
                               const int32_t* dst_blocks, int64_t n, int32_t tail_valid, int32_t dtype,
                               int64_t num_layers, int32_t block_size, int32_t kv_heads, int32_t head_dim,
                               int32_t* err_flag, void* stream) {
  const int es = dtype_size(dtype);
  NIE_REQUIRE(es > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(src_keys && src_values && dst_keys && dst_values, "null pointer argument");
  NIE_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "num_copy_blocks out of range");
  NIE_REQUIRE(num_layers > 0 && num_layers <= 65535, "num_layers out of range");
  NIE_REQUIRE(tail_valid >= 0 && tail_valid <= block_size, "tail_valid_tokens out of range");
  if (n == 0) return NIE_OK;
  const int64_t row_bytes = (int64_t)kv_heads * head_dim * es;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int w = vec_width(row_bytes, {src_keys, src_values, dst_keys, dst_values});
  switch (w) {
    case 16: launch_copy<uint4>(src_keys, src_values, src_num_blocks, src_blocks, dst_keys, dst_values, dst_num_blocks, dst_blocks, n, tail_valid, num_layers, block_size, row_bytes, err_flag, s); break;
    case 8: launch_copy<uint2>(src_keys, src_values, src_num_blocks, src_blocks, dst_keys, dst_values, dst_num_blocks, dst_blocks, n, tail_valid, num_layers, block_size, row_bytes, err_flag, s); break;
    case 4: launch_copy<uint32_t>(src_keys, src_values, src_num_blocks, src_blocks, dst_keys, dst_values, dst_num_blocks, dst_blocks, n, tail_valid, num_layers, block_size, row_bytes, err_flag, s); break;
    default: launch_copy<uint16_t>(src_keys, src_values, src_num_blocks, src_blocks, dst_keys, dst_values, dst_num_blocks, dst_blocks, n, tail_valid, num_layers, block_size, row_bytes, err_flag, s); break;
  }
  return check_launch("copy_blocks_kernel");
}
