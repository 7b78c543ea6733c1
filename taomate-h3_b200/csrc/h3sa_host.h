// Host-side helpers shared by the C-ABI translation units (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/h3sa.h"

namespace h3sa {

// Record a message for h3sa_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t e);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda needed),
// 128-byte swizzle, zero fill out of bounds.
int encode_tiled_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                    const uint64_t dims[3], const uint64_t strides_bytes[2], const uint32_t box[3]);

struct AttnLaunch {
  const void* query;  // [rows, heads, 128] bf16 or e4m3
  void* out;          // [rows, heads, 128] bf16
  int rows;
  int heads;
  const void* key_pool;    // [heads, pool_pages * 128, 128]
  const void* value_pool;  // [heads, pool_pages * 128, 128]
  int pool_pages;
  const int32_t* page_table;
  int table_blocks;
  const h3sa_problem* problems;
  int num_problems;
  float softmax_scale;
  const float* q_scale;  // e4m3 path only, [heads]
  const float* k_scale;
  const float* v_scale;
  // segmented e4m3 KV (see AttnParams): per block part | rows << 16, per (part, head) scales
  const int32_t* block_part;
  const float* part_k_scale;
  const float* part_v_scale;
  int n_parts;
  const int32_t* kv_num_blocks;
  const int32_t* kv_indices;
  int q_blocks;
  int kv_stride;
  int32_t* device_error;
  // Output to peers (Ulysses heads -> sequence fused into the epilogue): when set, query row r
  // is written to out_peers[r / out_rows_per_rank] at row r % out_rows_per_rank of a
  // [rows_per_rank, out_heads, 128] tensor, head out_head0 + h. Otherwise to `out`.
  const uint64_t* out_peers;
  int out_ranks;
  int out_rows_per_rank;
  int out_heads;
  int out_head0;
};

int attention_launch(const AttnLaunch& L, bool fp8, cudaStream_t stream);
size_t attention_smem_bytes(bool fp8);

// Per-head e4m3 quantiser over packed [batch, seq, heads, 128] rows or a paged pool.
constexpr int kQuantChunkRows = 256;  // rows per partial-amax slot
constexpr int kQuantMaxBatchHeads = 65535;  // (batch, head) pairs run along gridDim.y

struct QuantSpace {
  const __nv_bfloat16* src;
  uint8_t* dst;
  int paged;
  int batch;
  int seq;  // rows per (batch, head)
  int heads;
  int pool_pages;
  const int* page_table;
  int table_blocks;
};

// Launch amax-partial, finalize and apply; `partial` holds batch * heads * chunks floats,
// every one of which the first kernel writes before the second reads it.
int quantize_launch(const QuantSpace& q, float* scale, float* partial, int chunks, int* err,
                    cudaStream_t stream);

}  // namespace h3sa
