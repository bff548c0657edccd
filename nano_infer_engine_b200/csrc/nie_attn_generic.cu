// Generic paged attention (any dtype / head_dim <= 256 / block_size / GQA
// group).  It serves the shapes the specialised sm_100a kernels do not cover
// (fp32 caches, the small head dims of unit tests) and restates the
// reference's rounding sequence exactly:
//   s   = round(round(q . k) * scale)                 (bf16 einsum, then *scale)
//   p   = round(exp(s - max) / sum exp(s - max))       (fp32 softmax, cast)
//   out = round(sum p * v)                             (fp32-accumulated matmul)
// following nano_infer_engine/layers/paged_attention.py:95-114 and
// nano_infer_engine/layers/attention.py:400-411.  Two passes over the keys
// (max/sum, then the weighted sum) make the cast of normalised p exact.
#include "nie_attn.cuh"

namespace nie {


constexpr int kGenThreads = 128;
constexpr int kGenMaxPerLane = 8;  // head_dim <= 256
constexpr int kGenWarps = kGenThreads / 32;

template <typename T>
__global__ void __launch_bounds__(kGenThreads) attn_generic_kernel(GenericArgs a) {
  using N = Num<T>;
  const int i = blockIdx.x, j = blockIdx.y, h = blockIdx.z;
  const int r = a.req_list ? a.req_list[i] : i;
  int64_t qrow, npos;
  if (a.qsl) {
    const int64_t q0 = a.qsl[r], q1 = a.qsl[r + 1];
    const int64_t qlen = q1 - q0;
    if (j >= qlen) return;
    qrow = q0 + j;
    npos = (int64_t)a.seq_lens[r] - qlen + j + 1;  // keys [0, position]
  } else {
    if (j > 0) return;
    qrow = a.q_rows ? a.q_rows[r] : r;
    npos = a.seq_lens[r];
  }
  const int trow = a.table_rows ? a.table_rows[r] : r;
  const int group = a.hq / a.hkv;
  const int kvh = h / group;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = kGenWarps;

  const T* qp = reinterpret_cast<const T*>(a.q) + qrow * a.q_stride + (int64_t)h * a.hd;
  float qv[kGenMaxPerLane];
#pragma unroll
  for (int u = 0; u < kGenMaxPerLane; ++u) {
    const int d = lane + 32 * u;
    qv[u] = (d < a.hd) ? N::to_f(qp[d]) : 0.f;
  }
  const T* kc = reinterpret_cast<const T*>(a.kc);
  const T* vc = reinterpret_cast<const T*>(a.vc);
  const int64_t row_elems = (int64_t)a.hkv * a.hd;
  const int64_t layer_off = (int64_t)a.layer * a.nb * a.bs * row_elems;
  const int32_t* table = a.tables + (int64_t)trow * a.tstride;

  auto key_base = [&](int64_t p, bool& ok) -> int64_t {
    const int64_t lb = p / a.bs;
    const int64_t blk = (lb < a.tstride) ? (int64_t)table[lb] : -1;
    ok = blk >= 0 && blk < a.nb;
    return layer_off + (blk * a.bs + p % a.bs) * row_elems + (int64_t)kvh * a.hd;
  };
  auto score = [&](int64_t base) -> float {
    float part = 0.f;
#pragma unroll
    for (int u = 0; u < kGenMaxPerLane; ++u) {
      const int d = lane + 32 * u;
      if (d < a.hd) part += qv[u] * N::to_f(kc[base + d]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    return N::round_like(N::round_like(part) * a.scale);
  };

  // pass 1: running max and sum per warp
  float m = -INFINITY, l = 0.f;
  bool bad = false;
  for (int64_t p = warp; p < npos; p += nwarps) {
    bool ok;
    const int64_t base = key_base(p, ok);
    if (!ok) { bad = true; continue; }
    const float s = score(base);
    const float mn = fmaxf(m, s);
    l = l * expf(m - mn) + expf(s - mn);
    m = mn;
  }
  __shared__ float sm_m[kGenWarps], sm_l[kGenWarps];
  __shared__ float sm_acc[kGenWarps][256];
  if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
  if (bad && lane == 0) raise_flag(a.err, NIE_DEV_ERR_BLOCK_RANGE);
  __syncthreads();
  float gm = -INFINITY;
  for (int w = 0; w < nwarps; ++w) gm = fmaxf(gm, sm_m[w]);
  float gl = 0.f;
  for (int w = 0; w < nwarps; ++w)
    if (sm_m[w] != -INFINITY) gl += sm_l[w] * expf(sm_m[w] - gm);

  // pass 2: normalised, rounded probabilities times V
  float acc[kGenMaxPerLane];
#pragma unroll
  for (int u = 0; u < kGenMaxPerLane; ++u) acc[u] = 0.f;
  for (int64_t p = warp; p < npos; p += nwarps) {
    bool ok;
    const int64_t base = key_base(p, ok);
    if (!ok) continue;
    const float s = score(base);
    const float pr = N::round_like(expf(s - gm) / gl);
#pragma unroll
    for (int u = 0; u < kGenMaxPerLane; ++u) {
      const int d = lane + 32 * u;
      if (d < a.hd) acc[u] += pr * N::to_f(vc[base + d]);
    }
  }
#pragma unroll
  for (int u = 0; u < kGenMaxPerLane; ++u) {
    const int d = lane + 32 * u;
    if (d < a.hd) sm_acc[warp][d] = acc[u];
  }
  __syncthreads();
  T* op = reinterpret_cast<T*>(a.out) + qrow * a.out_stride + (int64_t)h * a.hd;
  for (int d = threadIdx.x; d < a.hd; d += kGenThreads) {
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += sm_acc[w][d];
    op[d] = N::from_f(v);
  }
}

int launch_generic(int dtype, const GenericArgs& a, int num_req, int max_q, cudaStream_t s) {
  if (a.hd > 32 * kGenMaxPerLane) return fail(NIE_ERR_UNSUPPORTED, "head_dim %d > 256", a.hd);
  if (num_req <= 0) return NIE_OK;
  if (max_q <= 0 || max_q > 65535) return fail(NIE_ERR_INVALID, "max_query_len out of range: %d", max_q);
  dim3 grid((unsigned)num_req, (unsigned)max_q, (unsigned)a.hq);
  switch (dtype) {
    case NIE_DTYPE_F32: attn_generic_kernel<float><<<grid, kGenThreads, 0, s>>>(a); break;
    case NIE_DTYPE_BF16: attn_generic_kernel<__nv_bfloat16><<<grid, kGenThreads, 0, s>>>(a); break;
    case NIE_DTYPE_F16: attn_generic_kernel<__half><<<grid, kGenThreads, 0, s>>>(a); break;
    default: return fail(NIE_ERR_INVALID, "unknown dtype %d", dtype);
  }
  return check_launch("attn_generic_kernel");
}

}  // namespace nie
