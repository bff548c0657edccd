// Thin torch C++ extension: the per-layer loop of one ragged step.
//
// models/llama.py runs every decoder layer of a ragged step as
//   add+RMSNorm -> q/k/v GEMM -> RoPE + KV slot write -> decode / varlen
//   attention -> o_proj GEMM -> add+RMSNorm -> gate/up GEMM -> SiLU*up ->
//   down GEMM
// (the reference's models/llama.py:274-325 / 381-391 with layers/decoder.py).
// Driven from Python, each layer costs ~10 wrapper calls of host time, which
// exceeds the GPU time of a 512-token mixed step.  This file issues the same
// launches from C++: the fused kernels through the library's C ABI
// (include/nie_b200.h) with the arguments the Python wrappers pass, and the
// projections through nie_linear (batches of <= 16 rows) or at::linear, the
// same choice and calls as ops.linear, so the results are identical to the
// Python loop's.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <cmath>
#include <vector>

#include "nie_b200.h"

namespace {

void check(int status, const char* what) {
  TORCH_CHECK(status == NIE_OK, what, " failed (status ", status, "): ", nie_last_error());
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return NIE_DTYPE_F32;
    case at::kBFloat16: return NIE_DTYPE_BF16;
    case at::kHalf: return NIE_DTYPE_F16;
    default: TORCH_CHECK(false, "unsupported dtype ", t);
  }
  return -1;
}

// (sum, normed) = add_rmsnorm(x, residual, weight); sum only when wanted
std::pair<at::Tensor, at::Tensor> add_rmsnorm(const at::Tensor& x, const at::Tensor* residual, const at::Tensor& w,
                                              double eps, bool want_sum, void* stream) {
  const int64_t hidden = x.size(-1);
  at::Tensor out = at::empty_like(x);
  at::Tensor sum;
  if (want_sum && residual) sum = at::empty_like(x);
  check(nie_add_rmsnorm(x.data_ptr(), residual ? residual->data_ptr() : nullptr, w.data_ptr(), (float)eps,
                        x.numel() / hidden, (int32_t)hidden, dtype_code(x.scalar_type()),
                        sum.defined() ? sum.data_ptr() : nullptr, out.data_ptr(), stream),
        "nie_add_rmsnorm");
  return {residual ? (sum.defined() ? sum : at::Tensor()) : x, out};
}

// x @ w^T: decode-size bf16 batches with K >= N on nie_linear (the choice the
// Python loop's ops.linear makes), everything else at::linear.
struct Linear {
  bool enabled = false;
  int32_t* err = nullptr;
  void* stream = nullptr;
  int64_t launches = 0;

  // overlap: the kernel that produced x (issued just before) does not write w
  at::Tensor operator()(const at::Tensor& x, const at::Tensor& w, bool overlap = false) {
    const int64_t m = x.size(0), n = w.size(0), k = w.size(1);
    // K >= N only (o_proj, down_proj), where the cluster K split beats cuBLAS
    if (enabled && m >= 1 && m <= 16 && k >= n && x.scalar_type() == at::kBFloat16 &&
        w.scalar_type() == at::kBFloat16 &&
        x.stride(1) == 1 && w.is_contiguous() && x.size(1) == k) {
      at::Tensor y = at::empty({m, n}, x.options());
      const int st = (overlap ? nie_linear_overlapped : nie_linear)(x.data_ptr(), x.stride(0), w.data_ptr(), n, k,
                                                                    m, y.data_ptr(), n, NIE_DTYPE_BF16, err, stream);
      if (st == NIE_OK) {
        ++launches;
        return y;
      }
      TORCH_CHECK(st == NIE_ERR_UNSUPPORTED, "nie_linear failed (status ", st, "): ", nie_last_error());
    }
    return at::linear(x, w);
  }
};

}  // namespace

// Returns the final normed hidden rows (of `logit_rows` when given) and the
// number of library kernels launched.  `weights` holds, per layer, the
// pre-norm weight, fused q/k/v weight, o_proj weight, post-norm weight, fused
// gate/up weight and down_proj weight; `eps` the two norm epsilons per layer.
// The metadata tensors are the fields of one packed ragged step (int64
// slot_mapping and query_start_loc, int32 tables, lengths and request
// lists); dec_ws / var_ws are the decode and varlen scratch buffers sized by
// nie_paged_decode_workspace_size / nie_varlen_workspace_size for this step,
// and decode_launches the number of kernels one decode call launches;
// stream_linear sends projections of <= 16 rows to nie_linear (else cuBLAS).
std::tuple<at::Tensor, int64_t> run_layers(
    const at::Tensor& x, const std::vector<at::Tensor>& weights, const std::vector<double>& eps,
    const at::Tensor& final_w, double final_eps, const at::Tensor& slot_mapping, const at::Tensor& block_tables,
    const at::Tensor& seq_lens, const at::Tensor& qsl, const at::Tensor& table_rows, const at::Tensor& decode_list,
    const at::Tensor& prefill_list, int64_t num_decode, int64_t num_prefill, int64_t max_query_len,
    int64_t max_seq_len, const c10::optional<at::Tensor>& logit_rows, const at::Tensor& keys,
    const at::Tensor& values, const at::Tensor& sin, const at::Tensor& cos, int64_t q_heads, int64_t kv_heads,
    int64_t head_dim, int64_t inner, const at::Tensor& dec_ws, int64_t decode_launches,
    const c10::optional<at::Tensor>& var_ws, bool stream_linear, const at::Tensor& err) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "x must be a contiguous CUDA [T, hidden] tensor");
  TORCH_CHECK(keys.dim() == 5 && keys.is_contiguous() && values.is_contiguous() && keys.sizes() == values.sizes() &&
                  keys.scalar_type() == x.scalar_type() && values.scalar_type() == x.scalar_type(),
              "key/value caches must be contiguous [L, blocks, block_size, kv_heads, head_dim] of x's dtype");
  TORCH_CHECK(keys.size(3) == kv_heads && keys.size(4) == head_dim && q_heads * head_dim == x.size(1),
              "head geometry does not match the caches / hidden size");
  TORCH_CHECK(sin.is_contiguous() && cos.is_contiguous() && sin.size(0) == x.size(0) && sin.size(1) == head_dim / 2 &&
                  cos.sizes() == sin.sizes(),
              "sin/cos must be contiguous [T, head_dim/2]");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kLong && qsl.scalar_type() == at::kLong, "slot_mapping and "
              "query_start_loc must be int64");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.stride(1) == 1 &&
                  seq_lens.scalar_type() == at::kInt && table_rows.scalar_type() == at::kInt &&
                  decode_list.scalar_type() == at::kInt && prefill_list.scalar_type() == at::kInt,
              "block tables, lengths and request lists must be int32");
  const int64_t n_layers = (int64_t)weights.size() / 6;
  TORCH_CHECK((int64_t)weights.size() == 6 * n_layers && (int64_t)eps.size() == 2 * n_layers, "bad weight list");
  void* stream = at::cuda::getCurrentCUDAStream(x.get_device()).stream();
  const int64_t T = x.size(0), hidden = x.size(1);
  const int64_t L = keys.size(0), nb = keys.size(1), bs = keys.size(2);
  const int dt = dtype_code(x.scalar_type());
  const int64_t nq = q_heads * head_dim, nkv = kv_heads * head_dim;
  const float scale = (float)(1.0 / std::sqrt((double)head_dim));
  const size_t var_bytes = var_ws.has_value() ? (size_t)var_ws->numel() : 0;
  int64_t launches = 0;
  Linear linear;
  linear.enabled = stream_linear;
  linear.err = err.data_ptr<int32_t>();
  linear.stream = stream;

  at::Tensor residual = x;
  auto [unused, normed] = add_rmsnorm(x, nullptr, weights[0], eps[0], false, stream);
  (void)unused;
  ++launches;
  at::Tensor out_final;
  for (int64_t li = 0; li < n_layers; ++li) {
    const at::Tensor& qkv_w = weights[6 * li + 1];
    const at::Tensor& o_w = weights[6 * li + 2];
    const at::Tensor& post_w = weights[6 * li + 3];
    const at::Tensor& gu_w = weights[6 * li + 4];
    const at::Tensor& down_w = weights[6 * li + 5];
    // q/k/v, RoPE on q and k, k/v into the cache slots
    at::Tensor qkv = linear(normed, qkv_w);
    at::Tensor q = qkv.narrow(1, 0, nq), k = qkv.narrow(1, nq, nkv), v = qkv.narrow(1, nq + nkv, nkv);
    at::Tensor q_rot = at::empty({T, q_heads, head_dim}, x.options());
    check(nie_rope_write_kv(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                            sin.data_ptr(), cos.data_ptr(), T, (int32_t)q_heads, (int32_t)kv_heads,
                            (int32_t)head_dim, q_rot.data_ptr(), keys.data_ptr(), values.data_ptr(), dt,
                            (int32_t)li, L, nb, (int32_t)bs, slot_mapping.data_ptr<int64_t>(),
                            err.data_ptr<int32_t>(), stream),
          "nie_rope_write_kv");
    ++launches;
    at::Tensor att = at::empty_like(q_rot);
    if (num_decode) {
      // follows the RoPE + KV write; the metadata comes from the packing kernel
      check(nie_paged_decode_overlapped(q_rot.data_ptr(), q_rot.stride(0), att.data_ptr(), att.stride(0),
                             keys.data_ptr(),
                             values.data_ptr(), dt, (int32_t)li, L, nb, (int32_t)bs, (int32_t)kv_heads,
                             (int32_t)head_dim, (int32_t)q_heads, block_tables.data_ptr<int32_t>(),
                             block_tables.stride(0), table_rows.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                             qsl.data_ptr<int64_t>(), decode_list.data_ptr<int32_t>(), (int32_t)num_decode, scale,
                             dec_ws.data_ptr(), (size_t)dec_ws.numel(), err.data_ptr<int32_t>(), stream),
            "nie_paged_decode_overlapped");
      launches += decode_launches;
    }
    if (num_prefill) {
      check(nie_varlen_attention(q_rot.data_ptr(), att.data_ptr(), q_rot.stride(0), T, keys.data_ptr(),
                                 values.data_ptr(), dt, (int32_t)li, L, nb, (int32_t)bs, (int32_t)kv_heads,
                                 (int32_t)head_dim, (int32_t)q_heads, block_tables.data_ptr<int32_t>(),
                                 block_tables.stride(0), table_rows.data_ptr<int32_t>(),
                                 seq_lens.data_ptr<int32_t>(), qsl.data_ptr<int64_t>(),
                                 prefill_list.data_ptr<int32_t>(), (int32_t)num_prefill, (int32_t)max_query_len,
                                 (int32_t)max_seq_len, scale, var_bytes ? var_ws->data_ptr() : nullptr, var_bytes,
                                 err.data_ptr<int32_t>(), stream),
            "nie_varlen_attention");
      launches += 1;
    }
    at::Tensor attn = linear(att.view({T, hidden}), o_w, /*overlap=*/true);  // after the attention kernels
    // h = attn + residual, normed2 = post-norm(h)
    auto [h, normed2] = add_rmsnorm(attn, &residual, post_w, eps[2 * li + 1], true, stream);
    ++launches;
    at::Tensor gate_up = linear(normed2, gu_w);
    at::Tensor gate = gate_up.narrow(1, 0, inner), up = gate_up.narrow(1, inner, inner);
    at::Tensor act = at::empty({T, inner}, x.options());
    check(nie_silu_mul(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0), act.data_ptr(), T,
                       (int32_t)inner, dt, stream),
          "nie_silu_mul");
    ++launches;
    at::Tensor mlp = linear(act, down_w, /*overlap=*/true);  // after SiLU * up
    if (li + 1 < n_layers) {
      auto [sum, nxt] = add_rmsnorm(mlp, &h, weights[6 * (li + 1)], eps[2 * (li + 1)], true, stream);
      ++launches;
      residual = sum;
      normed = nxt;
    } else {
      if (logit_rows.has_value()) {
        mlp = mlp.index_select(0, *logit_rows);
        h = h.index_select(0, *logit_rows);
      }
      auto [unused2, fin] = add_rmsnorm(mlp, &h, final_w, final_eps, false, stream);
      (void)unused2;
      ++launches;
      out_final = fin;
    }
  }
  return {out_final, launches + linear.launches};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "per-layer loop of a ragged step (nano_infer_engine_b200)";
  m.def("run_layers", &run_layers, "all decoder layers of one ragged step");
}
