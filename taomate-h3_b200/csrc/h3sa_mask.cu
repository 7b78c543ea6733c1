// 128-token block-sparse mask generator.
//
// Per (head, 128-row query block) it scores KV blocks by mean(Q block) . mean(K block) *
// d^-0.5 and keeps a fixed set plus the best-scoring rest, writing the flex BlockMask
// inputs kv_num_blocks [H, QB] and kv_indices [H, QB, stride] (ascending, zero padded).
//
//   mode 0 (history top-k, F/inference/dynamic_block_sparse.py:50-124): candidates are the
//          full history blocks [0, n_hist / 128); keep max(1, min(full, ceil(full *
//          density))) of them plus every block from the partial history tail on.
//   mode 1 (composite): keep every block pair touching audio, the first `sinks` blocks and
//          the +-`window` band around the query block's timeline position
//          floor((n_hist + 128 j) / 128), then fill a ceil(density * KB) budget by score.
//
// Exact, order-fixed arithmetic: block sums of bf16 values in fp64 (exact), means by one fp64
// division, dot products with separately rounded fp64 multiply and add as eight partial sums
// (terms d = g, g + 8, ... in order, g = 0..7) combined as ((s0 + s1) + (s2 + s3)) +
// ((s4 + s5) + (s6 + s7)), one fp64 multiply by d^-0.5; ties rank the lower block first. A CPU
// restatement of these steps reproduces the selection bit for bit. Eight independent chains
// keep the score loop from waiting on one 128-step chain of dependent additions.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cmath>
#include <cstring>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {

constexpr int kMaskMaxBlocks = 2048;

struct MaskParams {
  const __nv_bfloat16* query;   // packed [rows, heads, d]
  int rows, heads, q_lo, q_hi;
  const __nv_bfloat16* key_pool;  // paged [heads, pages * 128, d]
  int pool_pages;
  const int* page_table;
  int table_blocks;
  int mode;
  int n_hist, n_kv;
  int sinks, window;
  const uint8_t* q_block_audio;   // [QB] (mode 1)
  const uint8_t* kv_block_audio;  // [KB] (mode 1)
  int qb, kb, kb_means;           // query blocks, KV blocks, KV blocks that need means
  int full_hist, keep_count, budget;
  double scale;
  double* q_mean;                 // [H, QB, d]
  double* k_mean;                 // [H, d, kb_means] (d-major: the score loop reads it coalesced)
  int* kv_num_blocks;
  int* kv_indices;
  int stride;
  int* err;
};

// grid (H, QB + kb_means), 256 threads: lane c = tid % 16 owns dims [8c, 8c + 8) of every
// row, row group g = tid / 16 takes rows g, g + 16, ... of the block; all of a thread's rows
// are loaded (16-byte vectors, coalesced) before they are summed. The 16 row groups' fp64
// partial sums are exact, so adding them in shared memory in any order gives the exact
// block sum.
__global__ void __launch_bounds__(256) mask_means_kernel(const MaskParams p) {
  __shared__ double part[16][kHeadDim];
  const int h = blockIdx.x;
  const int blk = blockIdx.y;
  const int c = threadIdx.x & 15;
  const int g = threadIdx.x >> 4;
  const bool is_q = blk < p.qb;
  int r0, r1;
  const __nv_bfloat16* base;  // row 0 of the block for this head, column 0
  size_t row_stride;          // elements between rows
  if (is_q) {
    r0 = p.q_lo + blk * kBlockM;
    r1 = min(r0 + kBlockM, p.q_hi);
    base = p.query + (static_cast<size_t>(r0) * p.heads + h) * kHeadDim;
    row_stride = static_cast<size_t>(p.heads) * kHeadDim;
  } else {
    const int b = blk - p.qb;
    r0 = b * kBlockN;
    r1 = min(r0 + kBlockN, p.mode == 0 ? p.full_hist * kBlockN : p.n_kv);
    const int page = (b < p.table_blocks) ? p.page_table[b] : -1;
    if (page < 0 || page >= p.pool_pages) {
      if (threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadPage);
      return;  // the whole CTA leaves before the barrier below
    }
    base = p.key_pool + ((static_cast<size_t>(h) * p.pool_pages + page) * kBlockN) * kHeadDim;
    row_stride = kHeadDim;
  }
  const int n = r1 - r0;
  uint4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = g + 16 * k;
    v[k] = i < n ? __ldg(reinterpret_cast<const uint4*>(base + i * row_stride) + c)
                 : make_uint4(0u, 0u, 0u, 0u);
  }
  double acc[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[2 * e] += static_cast<double>(__uint_as_float(w[e] << 16));
      acc[2 * e + 1] += static_cast<double>(__uint_as_float(w[e] & 0xFFFF0000u));
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[g][8 * c + e] = acc[e];
  __syncthreads();
  if (threadIdx.x < kHeadDim) {
    const int d = threadIdx.x;
    double sum = 0.0;
#pragma unroll
    for (int k = 0; k < 16; ++k) sum += part[k][d];
    if (is_q)
      p.q_mean[(static_cast<size_t>(h) * p.qb + blk) * kHeadDim + d] = sum / n;
    else
      p.k_mean[(static_cast<size_t>(h) * kHeadDim + d) * p.kb_means + (blk - p.qb)] = sum / n;
  }
}

// grid (H, QB), 256 threads
__global__ void __launch_bounds__(256) mask_select_kernel(const MaskParams p) {
  __shared__ double qm[kHeadDim];
  __shared__ double score[kMaskMaxBlocks];
  __shared__ uint8_t cand[kMaskMaxBlocks];
  __shared__ uint8_t keep[kMaskMaxBlocks];
  __shared__ int warp_count[8];
  const int h = blockIdx.x;
  const int j = blockIdx.y;
  const int tid = threadIdx.x;
  if (tid < kHeadDim) qm[tid] = p.q_mean[(static_cast<size_t>(h) * p.qb + j) * kHeadDim + tid];
  const int qpos = (p.n_hist + kBlockM * j) / kBlockN;
  const bool q_audio = (p.mode == 1) && p.q_block_audio[j];
  for (int b = tid; b < p.kb; b += blockDim.x) {
    bool forced, is_cand;
    if (p.mode == 0) {
      forced = b >= p.full_hist;  // partial history tail and current blocks stay dense
      is_cand = !forced;
    } else {
      const int dist = b > qpos ? b - qpos : qpos - b;
      forced = q_audio || p.kv_block_audio[b] || b < p.sinks || dist <= p.window;
      is_cand = !forced;
    }
    keep[b] = forced ? 1 : 0;
    cand[b] = is_cand ? 1 : 0;
  }
  __syncthreads();
  // forced count -> how many candidates to add
  int forced_n = 0;
  for (int b = tid; b < p.kb; b += blockDim.x) forced_n += keep[b];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) forced_n += __shfl_xor_sync(0xffffffffu, forced_n, o);
  if ((tid & 31) == 0) warp_count[tid >> 5] = forced_n;
  __syncthreads();
  int forced_total = 0;
  for (int w = 0; w < (blockDim.x >> 5); ++w) forced_total += warp_count[w];
  const int take = (p.mode == 0) ? p.keep_count : max(0, p.budget - forced_total);
  // scores of the candidates: sequential fp64 dot over d
  for (int b = tid; b < p.kb; b += blockDim.x) {
    if (!cand[b]) continue;
    const double* km = p.k_mean + static_cast<size_t>(h) * kHeadDim * p.kb_means + b;
    double part[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
#pragma unroll 4
    for (int d0 = 0; d0 < kHeadDim; d0 += 8) {
#pragma unroll
      for (int g = 0; g < 8; ++g)
        part[g] = __dadd_rn(part[g], __dmul_rn(qm[d0 + g], km[static_cast<size_t>(d0 + g) * p.kb_means]));
    }
    const double acc = __dadd_rn(__dadd_rn(__dadd_rn(part[0], part[1]), __dadd_rn(part[2], part[3])),
                                 __dadd_rn(__dadd_rn(part[4], part[5]), __dadd_rn(part[6], part[7])));
    score[b] = __dmul_rn(acc, p.scale);
  }
  __syncthreads();
  // rank each candidate: better score, or equal score and lower index
  for (int b = tid; b < p.kb; b += blockDim.x) {
    if (!cand[b]) continue;
    const double s = score[b];
    int rank = 0;
    for (int c = 0; c < p.kb && rank < take; ++c)
      if (cand[c] && (score[c] > s || (score[c] == s && c < b))) ++rank;
    if (rank < take) keep[b] = 1;
  }
  __syncthreads();
  // ascending compaction by warp 0
  if (tid < 32) {
    const int chunk = (p.kb + 31) / 32;
    const int beg = min(tid * chunk, p.kb);
    const int end = min(beg + chunk, p.kb);
    int cnt = 0;
    for (int b = beg; b < end; ++b) cnt += keep[b];
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += y;
    }
    int pos = incl - cnt;
    int* row = p.kv_indices + (static_cast<size_t>(h) * p.qb + j) * p.stride;
    for (int b = beg; b < end; ++b)
      if (keep[b]) row[pos++] = b;
    if (tid == 31) p.kv_num_blocks[static_cast<size_t>(h) * p.qb + j] = incl;
    __syncwarp();
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    for (int i = total + tid; i < p.stride; i += 32) row[i] = 0;
  }
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_block_mask(const void* query, int32_t rows, int32_t heads, int32_t head_dim,
                    int32_t q_lo, int32_t q_hi, const void* key_pool, int32_t pool_pages,
                    const int32_t* page_table, int32_t table_blocks,
                    const h3sa_mask_policy* policy, int32_t* kv_num_blocks, int32_t* kv_indices,
                    int32_t kv_index_stride, int32_t* device_error, void* stream) {
  if (head_dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "block mask requires head_dim 128, got %d", head_dim);
  if (!query || !key_pool || !page_table || !policy || !kv_num_blocks || !kv_indices)
    return set_error(H3SA_ERR_INVALID, "block mask: null pointer argument");
  if (heads <= 0 || q_lo < 0 || q_hi <= q_lo || q_hi > rows || pool_pages <= 0 ||
      table_blocks <= 0)
    return set_error(H3SA_ERR_INVALID, "block mask: invalid sizes");
  if ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key_pool)) & 15)
    return set_error(H3SA_ERR_INVALID, "block mask: query and key pool must be 16-byte aligned");
  const h3sa_mask_policy& pol = *policy;
  if (pol.mode != 0 && pol.mode != 1)
    return set_error(H3SA_ERR_INVALID, "block mask: unknown policy mode %d", pol.mode);
  if (!(pol.density > 0.0 && pol.density <= 1.0))
    return set_error(H3SA_ERR_INVALID, "dynamic history density must be in (0, 1]");
  if (pol.n_hist < 0 || pol.n_kv <= 0 || pol.n_hist > pol.n_kv ||
      static_cast<int64_t>(pol.n_kv) > static_cast<int64_t>(table_blocks) * kBlockN)
    return set_error(H3SA_ERR_INVALID, "block mask: history %d / KV rows %d invalid", pol.n_hist,
                     pol.n_kv);
  MaskParams p{};
  p.query = static_cast<const __nv_bfloat16*>(query);
  p.rows = rows;
  p.heads = heads;
  p.q_lo = q_lo;
  p.q_hi = q_hi;
  p.key_pool = static_cast<const __nv_bfloat16*>(key_pool);
  p.pool_pages = pool_pages;
  p.page_table = page_table;
  p.table_blocks = table_blocks;
  p.mode = pol.mode;
  p.n_hist = pol.n_hist;
  p.n_kv = pol.n_kv;
  p.sinks = pol.sinks;
  p.window = pol.window;
  p.q_block_audio = pol.q_block_audio;
  p.kv_block_audio = pol.kv_block_audio;
  p.qb = (q_hi - q_lo + kBlockM - 1) / kBlockM;
  p.kb = (pol.n_kv + kBlockN - 1) / kBlockN;
  p.scale = std::pow(static_cast<double>(head_dim), -0.5);
  if (p.kb > kMaskMaxBlocks)
    return set_error(H3SA_ERR_UNSUPPORTED, "block mask: %d KV blocks exceed %d", p.kb,
                     kMaskMaxBlocks);
  if (kv_index_stride < p.kb)
    return set_error(H3SA_ERR_INVALID, "block mask: index stride %d < %d KV blocks",
                     kv_index_stride, p.kb);
  if (pol.mode == 0) {
    p.full_hist = pol.n_hist / kBlockN;
    if (p.full_hist < 1)
      return set_error(H3SA_ERR_INVALID, "dynamic sparse history has no complete K/V block");
    const double want = std::ceil(static_cast<double>(p.full_hist) * pol.density);
    p.keep_count = static_cast<int>(std::max(1.0, std::min(static_cast<double>(p.full_hist), want)));
    p.kb_means = p.full_hist;
  } else {
    if (!pol.q_block_audio || !pol.kv_block_audio)
      return set_error(H3SA_ERR_INVALID, "block mask: composite policy needs audio block flags");
    p.budget = static_cast<int>(std::ceil(pol.density * static_cast<double>(p.kb)));
    p.kb_means = p.kb;
  }
  p.kv_num_blocks = kv_num_blocks;
  p.kv_indices = kv_indices;
  p.stride = kv_index_stride;
  p.err = device_error;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t bytes = (static_cast<size_t>(heads) * p.qb + static_cast<size_t>(heads) * p.kb_means) *
                       kHeadDim * sizeof(double);
  void* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(&scratch, bytes, s);
  if (e != cudaSuccess) return set_cuda_error("cudaMallocAsync(block mask scratch)", e);
  p.q_mean = static_cast<double*>(scratch);
  p.k_mean = p.q_mean + static_cast<size_t>(heads) * p.qb * kHeadDim;
  mask_means_kernel<<<dim3(heads, p.qb + p.kb_means), 256, 0, s>>>(p);
  mask_select_kernel<<<dim3(heads, p.qb), 256, 0, s>>>(p);
  e = cudaGetLastError();
  const cudaError_t ef = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return set_cuda_error("block mask launch", e);
  if (ef != cudaSuccess) return set_cuda_error("cudaFreeAsync(block mask scratch)", ef);
  return H3SA_OK;
}

}  // extern "C"
