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
//                  (reference layers/rope.py:6-23 + paged_cache.py:264-322;
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
  pdl_wait();     // dependent launch: inputs come from the kernel before
  pdl_trigger();  // and the kernel after may be staged now
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
  pdl_wait();     // dependent launch: q/k/v come from the projection before
  pdl_trigger();  // the attention kernel after this one may start its prologue
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
  pdl_wait();     // dependent launch: inputs come from the kernel before
  pdl_trigger();  // and the kernel after may be staged now
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

// ------------------------------------------------ 16-byte vector variants
// Same per-element arithmetic and rounding as the kernels above; every
// thread moves whole 16-byte vectors and issues all of its loads before it
// needs any of them.  Used when rows, strides and pointers are 16-byte aligned.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  float f[N];
  __device__ __forceinline__ void load(const T* p) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Num<T>::to_f(e[i]);
  }
  __device__ __forceinline__ void store(T* p) const {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = Num<T>::from_f(f[i]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};

// add + RMSNorm, one CTA per row, up to MAXV vectors per thread.
template <typename T, int THREADS, int MAXV>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_vec_kernel(const T* __restrict__ x,
                                                                  const T* __restrict__ residual,
                                                                  const T* __restrict__ weight, float eps, int hidden,
                                                                  T* __restrict__ sum_out, T* __restrict__ out) {
  pdl_wait();     // dependent launch: inputs come from the kernel before
  pdl_trigger();  // and the kernel after may be staged now
  using N = Num<T>;
  constexpr int V = Vec16<T>::N;
  const int64_t row = blockIdx.x;
  const int nvec = hidden / V;
  Vec16<T> h[MAXV], w[MAXV];
  float sq = 0.f;
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int iv = threadIdx.x + u * THREADS;
    if (iv < nvec) {
      h[u].load(x + row * hidden + iv * V);
      w[u].load(weight + iv * V);
      if (residual) {
        Vec16<T> r;
        r.load(residual + row * hidden + iv * V);
#pragma unroll
        for (int e = 0; e < V; ++e) h[u].f[e] = N::round_like(h[u].f[e] + r.f[e]);
      }
#pragma unroll
      for (int e = 0; e < V; ++e) sq += h[u].f[e] * h[u].f[e];
    }
  }
  __shared__ float red[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) tot += red[i];
  const float denom = sqrtf(tot / (float)hidden + eps);
#pragma unroll
  for (int u = 0; u < MAXV; ++u) {
    const int iv = threadIdx.x + u * THREADS;
    if (iv < nvec) {
      if (sum_out) h[u].store(sum_out + row * hidden + iv * V);
      Vec16<T> o;
#pragma unroll
      for (int e = 0; e < V; ++e) o.f[e] = w[u].f[e] * (h[u].f[e] / denom);
      o.store(out + row * hidden + iv * V);
    }
  }
}

// SiLU * up over grid (column blocks, rows): no per-element division.
template <typename T>
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(const T* __restrict__ gate, int64_t g_stride,
                                                           const T* __restrict__ up, int64_t u_stride,
                                                           T* __restrict__ out, int cols) {
  pdl_wait();     // dependent launch: inputs come from the kernel before
  pdl_trigger();  // and the kernel after may be staged now
  using N = Num<T>;
  constexpr int V = Vec16<T>::N;
  const int64_t r = blockIdx.y;
  const int c = (blockIdx.x * 256 + threadIdx.x) * V;
  if (c >= cols) return;
  Vec16<T> g, u;
  g.load(gate + r * g_stride + c);
  u.load(up + r * u_stride + c);
#pragma unroll
  for (int e = 0; e < V; ++e) {
    const float sg = N::round_like(g.f[e] / (1.0f + expf(-g.f[e])));
    g.f[e] = sg * u.f[e];
  }
  g.store(out + r * (int64_t)cols + c);
}

// RoPE + slot write, one CTA per token; thread j < (hq + hkv) * half / V
// rotates V pairs (elements i..i+V-1 with i+half..), the rest copy v.
template <typename T>
__global__ void __launch_bounds__(256) rope_write_vec_kernel(
    const T* __restrict__ q, int64_t q_stride, const T* __restrict__ k, int64_t k_stride, const T* __restrict__ v,
    int64_t v_stride, const T* __restrict__ sin, const T* __restrict__ cos, int hq, int hkv, int d,
    T* __restrict__ q_out, T* __restrict__ kc, T* __restrict__ vc, int64_t layer_off, int64_t total_slots,
    const int64_t* __restrict__ slots, int32_t* __restrict__ err) {
  using N = Num<T>;
  pdl_wait();     // dependent launch: q/k/v come from the projection before
  pdl_trigger();  // the attention kernel after this one may start its prologue
  constexpr int V = Vec16<T>::N;
  const int64_t t = blockIdx.x;
  const int half = d / 2;
  const int64_t slot = slots[t];
  const bool write = slot >= 0 && slot < total_slots;
  if (slot >= total_slots && threadIdx.x == 0) raise_flag(err, NIE_DEV_ERR_SLOT_RANGE);
  const int64_t row_elems = (int64_t)hkv * d;
  const int chunks = half / V;                  // vectors per half-head
  const int rot = (hq + hkv) * chunks;          // rotation work items
  const int vcopy = (int)(row_elems / V);       // v copy work items
  for (int j = threadIdx.x; j < rot + vcopy; j += blockDim.x) {
    if (j < rot) {
      const int head_all = j / chunks, i = (j % chunks) * V;
      const bool is_q = head_all < hq;
      const int head = is_q ? head_all : head_all - hq;
      if (!is_q && !write) continue;
      const T* src = is_q ? q + t * q_stride + (int64_t)head * d : k + t * k_stride + (int64_t)head * d;
      Vec16<T> x1, x2, c, s;
      x1.load(src + i);
      x2.load(src + i + half);
      c.load(cos + t * half + i);
      s.load(sin + t * half + i);
      Vec16<T> o1, o2;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        o1.f[e] = N::round_like(__fsub_rn(N::round_like(__fmul_rn(x1.f[e], c.f[e])),
                                          N::round_like(__fmul_rn(x2.f[e], s.f[e]))));
        o2.f[e] = N::round_like(__fadd_rn(N::round_like(__fmul_rn(x2.f[e], c.f[e])),
                                          N::round_like(__fmul_rn(x1.f[e], s.f[e]))));
      }
      T* dst = is_q ? q_out + (t * hq + head) * (int64_t)d : kc + layer_off + slot * row_elems + (int64_t)head * d;
      o1.store(dst + i);
      o2.store(dst + i + half);
    } else if (write) {
      const int e = (j - rot) * V;
      *reinterpret_cast<uint4*>(vc + layer_off + slot * row_elems + e) =
          *reinterpret_cast<const uint4*>(v + t * v_stride + e);
    }
  }
}

__host__ inline bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---------------------------------------------------------- embedding rows
// out[t] = table[ids[t]] (a bit-exact row copy), one CTA per token; an id
// outside [0, vocab) writes a zero row and raises NIE_DEV_ERR_INDEX_RANGE.
__global__ void __launch_bounds__(256) embed_rows_kernel(const int64_t* __restrict__ ids, const uint4* __restrict__ table,
                                                         int64_t vocab, int vecs_per_row, uint4* __restrict__ out,
                                                         int32_t* __restrict__ err) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) raise_flag(err, NIE_DEV_ERR_INDEX_RANGE);
  for (int j = threadIdx.x; j < vecs_per_row; j += blockDim.x)
    out[t * vecs_per_row + j] = ok ? table[id * vecs_per_row + j] : make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------- argmax
// Row-wise argmax with torch.argmax's answer: the first index of the maximum,
// NaN counting as larger than any number.  grid = (kArgChunks, rows): each CTA
// reduces one chunk of a row to (value, index), the last CTA of the row to
// finish merges the chunk results in chunk order and resets the row counter.
constexpr int kArgChunks = 16;
constexpr int kArgMaxRows = 4096;
constexpr size_t kArgCounterBytes = kArgMaxRows * sizeof(int);

struct ArgBest {
  float v;
  int64_t i;
};

// a beats b: larger value (NaN largest), then smaller index
__device__ __forceinline__ bool arg_better(float av, int64_t ai, float bv, int64_t bi) {
  const bool an = av != av, bn = bv != bv;
  if (an || bn) return an && (!bn || ai < bi);
  return av > bv || (av == bv && ai < bi);
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const T* __restrict__ logits, int64_t cols, int64_t stride,
                                                          int64_t* __restrict__ out, int* __restrict__ counters,
                                                          ArgBest* __restrict__ partials) {
  const int64_t r = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t per = (cols + kArgChunks - 1) / kArgChunks;
  const int64_t c0 = chunk * per, c1 = min(cols, c0 + per);
  const T* row = logits + r * stride;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    const float v = Num<T>::to_f(row[c]);
    if (arg_better(v, c, bv, bi)) {
      bv = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (arg_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float sv[8];
  __shared__ int64_t si[8];
  __shared__ int last;
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (arg_better(sv[k], si[k], bv, bi)) {
        bv = sv[k];
        bi = si[k];
      }
    partials[r * kArgChunks + chunk] = ArgBest{bv, bi};
    __threadfence();
    last = atomicAdd(&counters[r], 1) == kArgChunks - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    float mv = -INFINITY;
    int64_t mi = INT64_MAX;
    for (int k = 0; k < kArgChunks; ++k) {
      const float pv = __ldcg(&partials[r * kArgChunks + k].v);
      const int64_t pi = __ldcg(&partials[r * kArgChunks + k].i);
      if (arg_better(pv, pi, mv, mi)) {
        mv = pv;
        mi = pi;
      }
    }
    out[r] = mi == INT64_MAX ? 0 : mi;
    counters[r] = 0;
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
  const int esz = dtype_size(dtype);
  if (esz > 0 && (hidden * esz) % 16 == 0 && hidden * esz <= 256 * 4 * 16 && aligned16(x) && aligned16(residual) &&
      aligned16(weight) && aligned16(sum_out) && aligned16(out)) {
    switch (dtype) {
      case NIE_DTYPE_BF16:
        pdl_launch(add_rmsnorm_vec_kernel<__nv_bfloat16, 256, 4>, dim3((unsigned)rows), dim3(256), s, 
            (const __nv_bfloat16*)x, (const __nv_bfloat16*)residual, (const __nv_bfloat16*)weight, eps, hidden,
            (__nv_bfloat16*)sum_out, (__nv_bfloat16*)out);
        break;
      case NIE_DTYPE_F32:
        pdl_launch(add_rmsnorm_vec_kernel<float, 256, 4>, dim3((unsigned)rows), dim3(256), s, 
            (const float*)x, (const float*)residual, (const float*)weight, eps, hidden, (float*)sum_out, (float*)out);
        break;
      default:
        pdl_launch(add_rmsnorm_vec_kernel<__half, 256, 4>, dim3((unsigned)rows), dim3(256), s, 
            (const __half*)x, (const __half*)residual, (const __half*)weight, eps, hidden, (__half*)sum_out,
            (__half*)out);
        break;
    }
    return check_launch("add_rmsnorm_vec_kernel");
  }
  switch (dtype) {
    case NIE_DTYPE_BF16:
      pdl_launch(add_rmsnorm_kernel<__nv_bfloat16, 256>, dim3((unsigned)rows), dim3(256), s, 
          (const __nv_bfloat16*)x, (const __nv_bfloat16*)residual, (const __nv_bfloat16*)weight, eps, hidden,
          (__nv_bfloat16*)sum_out, (__nv_bfloat16*)out);
      break;
    case NIE_DTYPE_F32:
      pdl_launch(add_rmsnorm_kernel<float, 256>, dim3((unsigned)rows), dim3(256), s, (const float*)x, (const float*)residual,
                                                                     (const float*)weight, eps, hidden,
                                                                     (float*)sum_out, (float*)out);
      break;
    case NIE_DTYPE_F16:
      pdl_launch(add_rmsnorm_kernel<__half, 256>, dim3((unsigned)rows), dim3(256), s, (const __half*)x, (const __half*)residual,
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
  constexpr int V = Vec16<T>::N;
  if ((d / 2) % V == 0 && qs % V == 0 && ks % V == 0 && vs % V == 0 && aligned16(q) && aligned16(k) && aligned16(v) &&
      aligned16(sin) && aligned16(cos) && aligned16(q_out) && aligned16(kc) && aligned16(vc)) {
    pdl_launch(rope_write_vec_kernel<T>, dim3((unsigned)T_), dim3(256), s, (const T*)q, qs, (const T*)k, ks, (const T*)v, vs,
                                                          (const T*)sin, (const T*)cos, hq, hkv, d, (T*)q_out, (T*)kc,
                                                          (T*)vc, layer_off, total_slots, slots, err);
    return;
  }
  pdl_launch(rope_write_kernel<T>, dim3((unsigned)T_), dim3(256), s, (const T*)q, qs, (const T*)k, ks, (const T*)v, vs, (const T*)sin,
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
  const int esz = dtype_size(dtype);
  const int V = esz > 0 ? 16 / esz : 0;
  if (V > 0 && cols % V == 0 && gate_stride % V == 0 && up_stride % V == 0 && aligned16(gate) && aligned16(up) &&
      aligned16(out) && rows <= 65535) {
    const dim3 grid((unsigned)((cols / V + threads - 1) / threads), (unsigned)rows);
    switch (dtype) {
      case NIE_DTYPE_BF16:
        pdl_launch(silu_mul_vec_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), s, (const __nv_bfloat16*)gate, gate_stride,
                                                                    (const __nv_bfloat16*)up, up_stride,
                                                                    (__nv_bfloat16*)out, cols);
        break;
      case NIE_DTYPE_F32:
        pdl_launch(silu_mul_vec_kernel<float>, dim3(grid), dim3(threads), s, (const float*)gate, gate_stride, (const float*)up,
                                                            up_stride, (float*)out, cols);
        break;
      default:
        pdl_launch(silu_mul_vec_kernel<__half>, dim3(grid), dim3(threads), s, (const __half*)gate, gate_stride, (const __half*)up,
                                                             up_stride, (__half*)out, cols);
        break;
    }
    return check_launch("silu_mul_vec_kernel");
  }
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
  switch (dtype) {
    case NIE_DTYPE_BF16:
      pdl_launch(silu_mul_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(threads), s, 
          (const __nv_bfloat16*)gate, gate_stride, (const __nv_bfloat16*)up, up_stride, (__nv_bfloat16*)out, rows, cols);
      break;
    case NIE_DTYPE_F32:
      pdl_launch(silu_mul_kernel<float>, dim3((unsigned)blocks), dim3(threads), s, (const float*)gate, gate_stride, (const float*)up,
                                                                  up_stride, (float*)out, rows, cols);
      break;
    case NIE_DTYPE_F16:
      pdl_launch(silu_mul_kernel<__half>, dim3((unsigned)blocks), dim3(threads), s, (const __half*)gate, gate_stride,
                                                                   (const __half*)up, up_stride, (__half*)out, rows,
                                                                   cols);
      break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("silu_mul_kernel");
}

extern "C" int nie_embed_rows(const int64_t* ids, int64_t num_tokens, const void* table, int64_t vocab,
                              int32_t hidden, int32_t dtype, void* out, int32_t* err_flag, void* stream) {
  NIE_REQUIRE(ids && table && out, "null pointer argument");
  NIE_REQUIRE(num_tokens >= 0 && num_tokens < (int64_t(1) << 31), "num_tokens out of range");
  const int esz = dtype_size(dtype);
  NIE_REQUIRE(esz > 0, "unknown dtype %d", dtype);
  NIE_REQUIRE(hidden > 0 && ((int64_t)hidden * esz) % 16 == 0, "hidden rows must be a multiple of 16 bytes");
  NIE_REQUIRE(aligned16(table) && aligned16(out), "table and out must be 16-byte aligned");
  if (num_tokens == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int vecs = (int)((int64_t)hidden * esz / 16);
  embed_rows_kernel<<<(unsigned)num_tokens, 256, 0, s>>>(ids, (const uint4*)table, vocab, vecs, (uint4*)out, err_flag);
  return check_launch("embed_rows_kernel");
}

extern "C" size_t nie_argmax_workspace_size(void) {
  return kArgCounterBytes + (size_t)kArgMaxRows * kArgChunks * sizeof(ArgBest);
}

extern "C" int nie_argmax_rows(const void* logits, int64_t rows, int64_t cols, int64_t row_stride, int32_t dtype,
                               int64_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  NIE_REQUIRE(logits && out && workspace, "null pointer argument");
  NIE_REQUIRE(rows >= 0 && rows <= kArgMaxRows, "rows must be in [0, %d]", kArgMaxRows);
  NIE_REQUIRE(cols >= 1 && row_stride >= cols, "bad shape");
  NIE_REQUIRE(workspace_bytes >= nie_argmax_workspace_size(), "workspace too small");
  NIE_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  if (rows == 0) return NIE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* counters = static_cast<int*>(workspace);
  ArgBest* partials = reinterpret_cast<ArgBest*>(static_cast<uint8_t*>(workspace) + kArgCounterBytes);
  const dim3 grid(kArgChunks, (unsigned)rows);
  switch (dtype) {
    case NIE_DTYPE_BF16:
      argmax_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)logits, cols, row_stride, out,
                                                             counters, partials);
      break;
    case NIE_DTYPE_F32:
      argmax_rows_kernel<float><<<grid, 256, 0, s>>>((const float*)logits, cols, row_stride, out, counters, partials);
      break;
    case NIE_DTYPE_F16:
      argmax_rows_kernel<__half><<<grid, 256, 0, s>>>((const __half*)logits, cols, row_stride, out, counters,
                                                      partials);
      break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("argmax_rows_kernel");
}
