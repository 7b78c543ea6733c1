// C-ABI entry points: argument validation, then the launches in the kernel units.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  return set_error(H3SA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_tiled_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                    const uint64_t dims[3], const uint64_t strides_bytes[2],
                    const uint32_t box[3]) {
  auto fn = encode_fn();
  if (!fn) return set_error(H3SA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(H3SA_ERR_INVALID,
                     "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu", (int)r,
                     (unsigned long long)dims[0], (unsigned long long)dims[1],
                     (unsigned long long)dims[2]);
  return H3SA_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_attention_args(const void* query, void* out, int32_t rows, int32_t heads,
                                int32_t head_dim, const void* key_pool, const void* value_pool,
                                int32_t pool_pages, const int32_t* page_table,
                                int32_t table_blocks, const h3sa_problem* problems,
                                int32_t num_problems, const int32_t* kv_num_blocks,
                                const int32_t* kv_indices, int32_t q_blocks,
                                int32_t kv_index_stride) {
  if (head_dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "attention requires head_dim 128, got %d", head_dim);
  if (rows < 0 || heads <= 0 || pool_pages <= 0 || table_blocks <= 0)
    return set_error(H3SA_ERR_INVALID, "attention: invalid sizes rows=%d heads=%d pages=%d "
                     "table_blocks=%d", rows, heads, pool_pages, table_blocks);
  if (!query || !out || !key_pool || !value_pool || !page_table || !problems)
    return set_error(H3SA_ERR_INVALID, "attention: null pointer argument");
  if (!aligned16(query) || !aligned16(out) || !aligned16(key_pool) || !aligned16(value_pool))
    return set_error(H3SA_ERR_INVALID, "attention: tensors must be 16-byte aligned");
  if (num_problems <= 0 || num_problems > kMaxProblems)
    return set_error(H3SA_ERR_INVALID, "attention: 1..%d problems per launch, got %d",
                     kMaxProblems, num_problems);
  if (static_cast<int64_t>(pool_pages) * kBlockN > INT32_MAX ||
      static_cast<int64_t>(table_blocks) * kBlockN > INT32_MAX)
    return set_error(H3SA_ERR_INVALID, "attention: pool or page table too large");
  for (int i = 0; i < num_problems; ++i) {
    const h3sa_problem& pr = problems[i];
    if (pr.q_lo < 0 || pr.q_hi < pr.q_lo || pr.q_hi > rows)
      return set_error(H3SA_ERR_INVALID, "attention problem %d: query rows [%d, %d) outside "
                       "[0, %d)", i, pr.q_lo, pr.q_hi, rows);
    if (pr.q_hi == pr.q_lo) continue;
    if (pr.kv_lo < 0 || pr.kv_hi <= pr.kv_lo ||
        static_cast<int64_t>(pr.kv_hi) > static_cast<int64_t>(table_blocks) * kBlockN)
      return set_error(H3SA_ERR_INVALID, "attention problem %d: KV rows [%d, %d) invalid for "
                       "%d table blocks", i, pr.kv_lo, pr.kv_hi, table_blocks);
    const int nblocks = (pr.kv_hi + kBlockN - 1) / kBlockN - pr.kv_lo / kBlockN;
    if (pr.sparse) {
      if (!kv_num_blocks || !kv_indices || kv_index_stride <= 0)
        return set_error(H3SA_ERR_INVALID, "attention problem %d: sparse without block lists", i);
      const int tiles = (pr.q_hi - pr.q_lo + kBlockM - 1) / kBlockM;
      if (tiles > q_blocks)
        return set_error(H3SA_ERR_INVALID, "attention problem %d: %d query blocks but lists "
                         "cover %d", i, tiles, q_blocks);
      if (nblocks > kMaxUnionBlocks)
        return set_error(H3SA_ERR_UNSUPPORTED, "attention problem %d: sparse KV range of %d "
                         "blocks exceeds %d", i, nblocks, kMaxUnionBlocks);
    }
  }
  return H3SA_OK;
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_abi_version(void) { return H3SA_ABI_VERSION; }

const char* h3sa_last_error(void) { return g_last_error; }

size_t h3sa_attention_smem_bytes(int fp8) { return attention_smem_bytes(fp8 != 0); }

int h3sa_attention_fwd(const void* query, void* out, int32_t rows, int32_t heads,
                       int32_t head_dim, const void* key_pool, const void* value_pool,
                       int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                       const h3sa_problem* problems, int32_t num_problems, float softmax_scale,
                       const int32_t* kv_num_blocks, const int32_t* kv_indices,
                       int32_t q_blocks, int32_t kv_index_stride, int32_t* device_error,
                       void* stream) {
  int rc = check_attention_args(query, out, rows, heads, head_dim, key_pool, value_pool,
                                pool_pages, page_table, table_blocks, problems, num_problems,
                                kv_num_blocks, kv_indices, q_blocks, kv_index_stride);
  if (rc) return rc;
  AttnLaunch L{};
  L.query = query;
  L.out = out;
  L.rows = rows;
  L.heads = heads;
  L.key_pool = key_pool;
  L.value_pool = value_pool;
  L.pool_pages = pool_pages;
  L.page_table = page_table;
  L.table_blocks = table_blocks;
  L.problems = problems;
  L.num_problems = num_problems;
  L.softmax_scale = softmax_scale;
  L.kv_num_blocks = kv_num_blocks;
  L.kv_indices = kv_indices;
  L.q_blocks = q_blocks;
  L.kv_stride = kv_index_stride;
  L.device_error = device_error;
  return attention_launch(L, false, static_cast<cudaStream_t>(stream));
}

int h3sa_attention_fwd_scatter(const void* query, int32_t rows, int32_t heads, int32_t head_dim,
                               const void* key_pool, const void* value_pool, int32_t pool_pages,
                               const int32_t* page_table, int32_t table_blocks,
                               const h3sa_problem* problems, int32_t num_problems,
                               float softmax_scale, const int32_t* kv_num_blocks,
                               const int32_t* kv_indices, int32_t q_blocks,
                               int32_t kv_index_stride, const uint64_t* out_peers,
                               int32_t out_ranks, int32_t out_rows_per_rank, int32_t out_heads,
                               int32_t out_head0, int32_t* device_error, void* stream) {
  // `out` is not used on this path; the argument check wants a non-null, aligned pointer
  int rc = check_attention_args(query, const_cast<void*>(query), rows, heads, head_dim, key_pool,
                                value_pool,
                                pool_pages, page_table, table_blocks, problems, num_problems,
                                kv_num_blocks, kv_indices, q_blocks, kv_index_stride);
  if (rc) return rc;
  if (!out_peers || out_ranks <= 0 || out_rows_per_rank <= 0 || out_head0 < 0 ||
      out_head0 + heads > out_heads)
    return set_error(H3SA_ERR_INVALID, "attention scatter: invalid output layout (ranks %d, "
                     "rows per rank %d, heads %d + %d of %d)", out_ranks, out_rows_per_rank,
                     out_head0, heads, out_heads);
  if (static_cast<int64_t>(out_ranks) * out_rows_per_rank < rows)
    return set_error(H3SA_ERR_INVALID, "attention scatter: %d ranks x %d rows do not cover %d "
                     "query rows", out_ranks, out_rows_per_rank, rows);
  AttnLaunch L{};
  L.query = query;
  L.out = nullptr;
  L.rows = rows;
  L.heads = heads;
  L.key_pool = key_pool;
  L.value_pool = value_pool;
  L.pool_pages = pool_pages;
  L.page_table = page_table;
  L.table_blocks = table_blocks;
  L.problems = problems;
  L.num_problems = num_problems;
  L.softmax_scale = softmax_scale;
  L.kv_num_blocks = kv_num_blocks;
  L.kv_indices = kv_indices;
  L.q_blocks = q_blocks;
  L.kv_stride = kv_index_stride;
  L.device_error = device_error;
  L.out_peers = out_peers;
  L.out_ranks = out_ranks;
  L.out_rows_per_rank = out_rows_per_rank;
  L.out_heads = out_heads;
  L.out_head0 = out_head0;
  return attention_launch(L, false, static_cast<cudaStream_t>(stream));
}

int h3sa_attention_fwd_fp8(const void* query, void* out, int32_t rows, int32_t heads,
                           int32_t head_dim, const void* key_pool, const void* value_pool,
                           int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                           const h3sa_problem* problems, int32_t num_problems,
                           float softmax_scale, const float* q_scale, const float* k_scale,
                           const float* v_scale, const int32_t* kv_num_blocks,
                           const int32_t* kv_indices, int32_t q_blocks, int32_t kv_index_stride,
                           int32_t* device_error, void* stream) {
  int rc = check_attention_args(query, out, rows, heads, head_dim, key_pool, value_pool,
                                pool_pages, page_table, table_blocks, problems, num_problems,
                                kv_num_blocks, kv_indices, q_blocks, kv_index_stride);
  if (rc) return rc;
  if (!q_scale || !k_scale || !v_scale)
    return set_error(H3SA_ERR_INVALID, "fp8 attention: null scale pointer");
  AttnLaunch L{};
  L.query = query;
  L.out = out;
  L.rows = rows;
  L.heads = heads;
  L.key_pool = key_pool;
  L.value_pool = value_pool;
  L.pool_pages = pool_pages;
  L.page_table = page_table;
  L.table_blocks = table_blocks;
  L.problems = problems;
  L.num_problems = num_problems;
  L.softmax_scale = softmax_scale;
  L.q_scale = q_scale;
  L.k_scale = k_scale;
  L.v_scale = v_scale;
  L.kv_num_blocks = kv_num_blocks;
  L.kv_indices = kv_indices;
  L.q_blocks = q_blocks;
  L.kv_stride = kv_index_stride;
  L.device_error = device_error;
  return attention_launch(L, true, static_cast<cudaStream_t>(stream));
}

int h3sa_attention_fwd_fp8_parts(const void* query, void* out, int32_t rows, int32_t heads,
                                 int32_t head_dim, const void* key_pool, const void* value_pool,
                                 int32_t pool_pages, const int32_t* page_table,
                                 int32_t table_blocks, const h3sa_problem* problems,
                                 int32_t num_problems, float softmax_scale, const float* q_scale,
                                 const int32_t* block_part, int32_t num_parts,
                                 const float* part_k_scale, const float* part_v_scale,
                                 const int32_t* kv_num_blocks, const int32_t* kv_indices,
                                 int32_t q_blocks, int32_t kv_index_stride, int32_t* device_error,
                                 void* stream) {
  int rc = check_attention_args(query, out, rows, heads, head_dim, key_pool, value_pool,
                                pool_pages, page_table, table_blocks, problems, num_problems,
                                kv_num_blocks, kv_indices, q_blocks, kv_index_stride);
  if (rc) return rc;
  if (!q_scale || !block_part || !part_k_scale || !part_v_scale)
    return set_error(H3SA_ERR_INVALID, "fp8 part attention: null scale or part pointer");
  if (num_parts < 1 || num_parts > 0xFFFF)
    return set_error(H3SA_ERR_INVALID, "fp8 part attention: %d parts outside [1, 65535]",
                     num_parts);
  AttnLaunch L{};
  L.query = query;
  L.out = out;
  L.rows = rows;
  L.heads = heads;
  L.key_pool = key_pool;
  L.value_pool = value_pool;
  L.pool_pages = pool_pages;
  L.page_table = page_table;
  L.table_blocks = table_blocks;
  L.problems = problems;
  L.num_problems = num_problems;
  L.softmax_scale = softmax_scale;
  L.q_scale = q_scale;
  L.k_scale = part_k_scale;  // part 0's row; the kernel reads per-block scales instead
  L.v_scale = part_v_scale;
  L.block_part = block_part;
  L.part_k_scale = part_k_scale;
  L.part_v_scale = part_v_scale;
  L.n_parts = num_parts;
  L.kv_num_blocks = kv_num_blocks;
  L.kv_indices = kv_indices;
  L.q_blocks = q_blocks;
  L.kv_stride = kv_index_stride;
  L.device_error = device_error;
  return attention_launch(L, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
