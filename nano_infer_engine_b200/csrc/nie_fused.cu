// Fused elementwise stages of the ragged step.  Each kernel reproduces the
// rounding sequence of the torch op chain it replaces (every intermediate
// the reference materialises in the activation dtype is rounded to it), so
// results match the unfused reference bit for bit except where a reduction
// order differs (the RMSNorm mean).
//
//   add_rmsnorm  : sum = x + residual; out = w * (sum / sqrt(mean(sum^2) + eps))
//                  (reference layers/rms_norm.py:25-31 and the residual adds of
//                  layers/decoder.py:55-74)
//   rope_write_kv: q' = rope(q); k' = rope(k); cache[slot] = k', v
//                  (reference layers/rope.py:6-23 + paged_cache.py:324-382;
//                  the RoPE fusion into the slot write of the build plan)
//   silu_mul     : out = silu(gate) * up  (reference layers/mlp.py:18-22)
#include "nie_common.cuh"

namespace nie {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return Num<T>::to_f(*p);
}

// --------------------------------------------------------- add + RMSNorm
// One CTA per row.  `residual` may be null (plain RMSNorm); `sum_out` may be
// null (the sum is not needed afterwards).
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ residual,
                                                               const T* __restrict__ weight, float eps, int hidden,
                                                               T* __restrict__ sum_out, T* __restrict__ out) {
  using N = Num<T>;
  const int64_t row = blockIdx.x;
  const T* xr = x + row * hidden;
  const T* rr = residual ? residual + row * hidden : nullptr;
  constexpr int kMax = 16;  // hidden <= THREADS * kMax
  float h[kMax];
  float sq = 0.f;
#pragma unroll
  for (int u = 0; u < kMax; ++u) {
    const int i = threadIdx.x + u * THREADS;
    h[u] = 0.f;
    if (i < hidden) {
      float v = N::to_f(xr[i]);
      if (rr) v = N::round_like(v + N::to_f(rr[i]));
      h[u] = v;
      sq += v * v;
    }
  }
  __shared__ float red[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) tot += red[w];
  const float denom = sqrtf(tot / (float)hidden + eps);
  T* so = sum_out ? sum_out + row * hidden : nullptr;
  T* o = out + row * hidden;
#pragma unroll
  for (int u = 0; u < kMax; ++u) {
    const int i = threadIdx.x + u * THREADS;
    if (i < hidden) {
      if (so) so[i] = N::from_f(h[u]);
      o[i] = N::from_f(N::to_f(weight[i]) * (h[u] / denom));
    }
  }
}

// ------------------------------------------------------ RoPE + slot write
// One CTA per token.  q/k/v rows have `*_stride` elements between tokens;
// sin/cos are [T, D/2] in the activation dtype.  The rotated q goes to
// q_out [T, Hq, D]; rotated k and v go to the cache slot (skipped when the
// slot is negative, i.e. the packer already flagged it).
template <typename T>
__global__ void __launch_bounds__(256) rope_write_kernel(
    const T* __restrict__ q, int64_t q_stride, const T* __restrict__ k, int64_t k_stride, const T* __restrict__ v,
    int64_t v_stride, const T* __restrict__ sin, const T* __restrict__ cos, int hq, int hkv, int d,
    T* __restrict__ q_out, T* __restrict__ kc, T* __restrict__ vc, int64_t layer_off, int64_t total_slots,
    const int64_t* __restrict__ slots, int32_t* __restrict__ err) {
  using N = Num<T>;
  const int64_t t = blockIdx.x;
  const int half = d / 2;
  const T* sr = sin + t * half;
  const T* cr = cos + t * half;
  const int64_t slot = slots[t];
  const bool write = slot >= 0 && slot < total_slots;
  if (slot >= total_slots && threadIdx.x == 0) raise_flag(err, NIE_DEV_ERR_SLOT_RANGE);
  const int64_t row_elems = (int64_t)hkv * d;
  T* kd = kc + layer_off + slot * row_elems;
  T* vd = vc + layer_off + slot * row_elems;
  // rotated pairs: (i, i + half) per head; q heads first, then k heads
  const int pairs_q = hq * half, pairs = (hq + hkv) * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const bool is_q = p < pairs_q;
    const int pp = is_q ? p : p - pairs_q;
    const int head = pp / half, i = pp % half;
    const T* src = is_q ? q + t * q_stride + (int64_t)head * d : k + t * k_stride + (int64_t)head * d;
    const float x1 = N::to_f(src[i]), x2 = N::to_f(src[i + half]);
    const float c = N::to_f(cr[i]), s = N::to_f(sr[i]);
    // torch: first * cos - second * sin ; second * cos + first * sin, each
    // product and each sum rounded to the activation dtype (separate
    // kernels in torch, so no fused multiply-add: use the _rn intrinsics)
    const float o1 = N::round_like(__fsub_rn(N::round_like(__fmul_rn(x1, c)), N::round_like(__fmul_rn(x2, s))));
    const float o2 = N::round_like(__fadd_rn(N::round_like(__fmul_rn(x2, c)), N::round_like(__fmul_rn(x1, s))));
    if (is_q) {
      T* dst = q_out + (t * hq + head) * (int64_t)d;
      dst[i] = N::from_f(o1);
      dst[i + half] = N::from_f(o2);
    } else if (write) {
      kd[(int64_t)head * d + i] = N::from_f(o1);
      kd[(int64_t)head * d + i + half] = N::from_f(o2);
    }
  }
  if (write) {
    for (int e = threadIdx.x; e < row_elems; e += blockDim.x) vd[e] = v[t * v_stride + e];
  }
}

// ---------------------------------------------------------------- SiLU * up
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gate, int64_t g_stride, const T* __restrict__ up,
                                int64_t u_stride, T* __restrict__ out, int64_t rows, int cols) {
  using N = Num<T>;
  const int64_t n = rows * cols;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / cols;
    const int c = (int)(idx % cols);
    const float g = N::to_f(gate[r * g_stride + c]);
    // torch silu: x / (1 + exp(-x)) in fp32, rounded; then the bf16 product
    const float sg = N::round_like(g / (1.0f + expf(-g)));
    out[idx] = N::from_f(sg * N::to_f(up[r * u_stride + c]));
  }
}

}  // namespace nie

using namespace nie;

extern "C" int nie_add_rmsnorm(const void* x, const void* residual, const void* weight, float eps, int64_t rows,
                               int32_t hidden, int32_t dtype, void* sum_out, void* out, void* stream) {
  NIE_REQUIRE(x && weight && out, "null pointer argument");
  NIE_REQUIRE(rows >= 0 && rows < (int64_t(1) << 31), "rows out of range");
  NIE_REQUIRE(hidden > 0 && hidden <= 256 * 16, "hidden must be in [1, 4096]");
  if (rows == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NIE_DTYPE_BF16:
      add_rmsnorm_kernel<__nv_bfloat16, 256><<<(unsigned)rows, 256, 0, s>>>(
          (const __nv_bfloat16*)x, (const __nv_bfloat16*)residual, (const __nv_bfloat16*)weight, eps, hidden,
          (__nv_bfloat16*)sum_out, (__nv_bfloat16*)out);
      break;
    case NIE_DTYPE_F32:
      add_rmsnorm_kernel<float, 256><<<(unsigned)rows, 256, 0, s>>>((const float*)x, (const float*)residual,
                                                                     (const float*)weight, eps, hidden,
                                                                     (float*)sum_out, (float*)out);
      break;
    case NIE_DTYPE_F16:
      add_rmsnorm_kernel<__half, 256><<<(unsigned)rows, 256, 0, s>>>((const __half*)x, (const __half*)residual,
                                                                      (const __half*)weight, eps, hidden,
                                                                      (__half*)sum_out, (__half*)out);
      break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("add_rmsnorm_kernel");
}

template <typename T>
static void launch_rope_write(const void* q, int64_t qs, const void* k, int64_t ks, const void* v, int64_t vs,
                              const void* sin, const void* cos, int64_t T_, int hq, int hkv, int d, void* q_out,
                              void* kc, void* vc, int64_t layer_off, int64_t total_slots, const int64_t* slots,
                              int32_t* err, cudaStream_t s) {
  rope_write_kernel<T><<<(unsigned)T_, 256, 0, s>>>((const T*)q, qs, (const T*)k, ks, (const T*)v, vs, (const T*)sin,
                                                    (const T*)cos, hq, hkv, d, (T*)q_out, (T*)kc, (T*)vc, layer_off,
                                                    total_slots, slots, err);
}

extern "C" int nie_rope_write_kv(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                                 int64_t v_stride, const void* sin, const void* cos, int64_t num_tokens,
                                 int32_t q_heads, int32_t kv_heads, int32_t head_dim, void* q_out, void* key_cache,
                                 void* value_cache, int32_t dtype, int32_t layer, int64_t num_layers,
                                 int64_t num_blocks, int32_t block_size, const int64_t* slot_mapping,
                                 int32_t* err_flag, void* stream) {
  NIE_REQUIRE(q && k && v && sin && cos && q_out && key_cache && value_cache && slot_mapping, "null pointer argument");
  NIE_REQUIRE(num_tokens >= 0 && num_tokens < (int64_t(1) << 31), "num_tokens out of range");
  NIE_REQUIRE(head_dim > 0 && head_dim % 2 == 0, "head_dim must be even");
  NIE_REQUIRE(layer >= 0 && layer < num_layers, "layer %d out of range", layer);
  NIE_REQUIRE(q_heads > 0 && kv_heads > 0 && num_blocks > 0 && block_size > 0, "bad geometry");
  if (num_tokens == 0) return NIE_OK;
  const int64_t total_slots = num_blocks * block_size;
  const int64_t layer_off = (int64_t)layer * total_slots * kv_heads * head_dim;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NIE_DTYPE_BF16:
      launch_rope_write<__nv_bfloat16>(q, q_stride, k, k_stride, v, v_stride, sin, cos, num_tokens, q_heads, kv_heads,
                                       head_dim, q_out, key_cache, value_cache, layer_off, total_slots, slot_mapping,
                                       err_flag, s);
      break;
    case NIE_DTYPE_F32:
      launch_rope_write<float>(q, q_stride, k, k_stride, v, v_stride, sin, cos, num_tokens, q_heads, kv_heads,
                               head_dim, q_out, key_cache, value_cache, layer_off, total_slots, slot_mapping,
                               err_flag, s);
      break;
    case NIE_DTYPE_F16:
      launch_rope_write<__half>(q, q_stride, k, k_stride, v, v_stride, sin, cos, num_tokens, q_heads, kv_heads,
                                head_dim, q_out, key_cache, value_cache, layer_off, total_slots, slot_mapping,
                                err_flag, s);
      break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("rope_write_kernel");
}

extern "C" int nie_silu_mul(const void* gate, int64_t gate_stride, const void* up, int64_t up_stride, void* out,
                            int64_t rows, int32_t cols, int32_t dtype, void* stream) {
  NIE_REQUIRE(gate && up && out, "null pointer argument");
  NIE_REQUIRE(rows >= 0 && cols > 0, "bad shape");
  if (rows == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n = rows * cols;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
  switch (dtype) {
    case NIE_DTYPE_BF16:
      silu_mul_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, s>>>(
          (const __nv_bfloat16*)gate, gate_stride, (const __nv_bfloat16*)up, up_stride, (__nv_bfloat16*)out, rows, cols);
      break;
    case NIE_DTYPE_F32:
      silu_mul_kernel<float><<<(unsigned)blocks, threads, 0, s>>>((const float*)gate, gate_stride, (const float*)up,
                                                                  up_stride, (float*)out, rows, cols);
      break;
    case NIE_DTYPE_F16:
      silu_mul_kernel<__half><<<(unsigned)blocks, threads, 0, s>>>((const __half*)gate, gate_stride,
                                                                   (const __half*)up, up_stride, (__half*)out, rows,
                                                                   cols);
      break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("silu_mul_kernel");
}
