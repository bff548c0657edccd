// Declarations shared by the attention translation units.
#pragma once

#include "nie_common.cuh"

namespace nie {

// Arguments of the generic (any-shape) paged attention kernel.
struct GenericArgs {
  const void* q;
  void* out;
  int64_t q_stride, out_stride;  // elements between token rows
  const void* kc;
  const void* vc;
  int layer;
  int64_t nb;
  int bs, hkv, hd, hq;
  const int32_t* tables;
  int64_t tstride;
  const int32_t* table_rows;
  const int32_t* seq_lens;
  const int64_t* q_rows;  // decode mode
  const int64_t* qsl;     // varlen mode (non-null selects it)
  const int32_t* req_list;
  float scale;
  int32_t* err;
};

// Launch the generic kernel over grid (num_req, max_q, q_heads).
int launch_generic(int dtype, const GenericArgs& a, int num_req, int max_q, cudaStream_t s);

// tcgen05 varlen kernel (nie_attn_prefill.cu); NIE_ERR_UNSUPPORTED = use the generic one.
int launch_prefill_tc(const void* q, void* out, int64_t row_stride, int64_t num_q_rows, const void* key_cache,
                      const void* value_cache, int32_t layer, int64_t num_blocks, int32_t kv_heads, int32_t q_heads,
                      const int32_t* block_tables, int64_t table_stride, const int32_t* table_rows,
                      const int32_t* seq_lens, const int64_t* qsl, const int32_t* req_list, int32_t num_requests,
                      int32_t max_query_len, int32_t max_seq_len, float scale, void* workspace,
                      size_t workspace_bytes, int32_t* err_flag, cudaStream_t s);

// Scratch bytes the tcgen05 varlen kernel uses to split long key ranges.
size_t prefill_workspace_bytes(int32_t num_requests, int32_t max_query_len, int32_t max_seq_len, int32_t q_heads);

// Build the per-layer 3-D tensor map used by the TMA kernels: dims
// {head_dim, kv_heads, num_blocks * block_size}, box {head_dim, 1, block_size},
// 128-byte swizzle.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

}  // namespace nie
