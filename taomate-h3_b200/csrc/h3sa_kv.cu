// Paged KV cache row movement and the per-head e4m3 quantiser.
//
// Row copies move 16-byte chunks: consecutive threads cover one (row, head) record, then the
// next head, then the next row, so reads from the packed [rows, heads, d] layout and writes
// into a page's head plane are both full 128-byte lines.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstring>

#include "h3sa_attention.cuh"
#include "h3sa_fp8.cuh"
#include "h3sa_host.h"

namespace h3sa {

struct RowsDev {
  uint8_t* base;
  int paged;
  int extent;
  const int* page_table;
  int table_blocks;
};

struct CopyParams {
  RowsDev src[2];
  RowsDev dst[2];
  int ntensors;
  const int* src_index;
  int src_start;
  const int* dst_index;
  int dst_start;
  int count;
  int heads;
  int row_bytes;
  int* err;
};

__device__ __forceinline__ uint8_t* row_address(const RowsDev& r, int row, int head, int heads,
                                                int row_bytes) {
  if (row < 0) return nullptr;
  if (!r.paged) {
    if (row >= r.extent) return nullptr;
    return r.base + (static_cast<size_t>(row) * heads + head) * row_bytes;
  }
  const int blk = row >> 7;
  if (blk >= r.table_blocks) return nullptr;
  const int page = __ldg(r.page_table + blk);
  if (page < 0 || page >= r.extent) return nullptr;
  return r.base +
         ((static_cast<size_t>(head) * r.extent + page) * kBlockN + (row & 127)) * row_bytes;
}

__global__ void __launch_bounds__(256) kv_copy_kernel(const CopyParams p) {
  const int cpr = p.row_bytes >> 4;
  const long long total = static_cast<long long>(p.count) * p.heads * cpr;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % cpr);
    const long long rh = idx / cpr;
    const int h = static_cast<int>(rh % p.heads);
    const int i = static_cast<int>(rh / p.heads);
    const int sr = p.src_index ? __ldg(p.src_index + i) : p.src_start + i;
    const int dr = p.dst_index ? __ldg(p.dst_index + i) : p.dst_start + i;
    for (int t = 0; t < p.ntensors; ++t) {
      const uint8_t* s = row_address(p.src[t], sr, h, p.heads, p.row_bytes);
      uint8_t* d = row_address(p.dst[t], dr, h, p.heads, p.row_bytes);
      if (!s || !d) {
        if (p.err) atomicOr(p.err, kErrBadIndex);
        continue;
      }
      reinterpret_cast<uint4*>(d)[c] = __ldg(reinterpret_cast<const uint4*>(s) + c);
    }
  }
}

// ------------------------------------------------------------------ e4m3 quantiser
// (kFp8Max, div_by_scale and quant4: h3sa_fp8.cuh)

// Element offset of (b, s, h, 0); -1 when a page lookup fails.
__device__ __forceinline__ long long quant_offset(const QuantSpace& q, int b, int s, int h) {
  if (!q.paged) return ((static_cast<long long>(b) * q.seq + s) * q.heads + h) * kHeadDim;
  const int blk = s >> 7;
  if (blk >= q.table_blocks) return -1;
  const int page = __ldg(q.page_table + blk);
  if (page < 0 || page >= q.pool_pages) return -1;
  return ((static_cast<long long>(h) * q.pool_pages + page) * kBlockN + (s & 127)) * kHeadDim;
}

__device__ __forceinline__ float bf16_bits_abs_max8(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m = fmaxf(m, fabsf(__uint_as_float(w[i] << 16)));
    m = fmaxf(m, fabsf(__uint_as_float(w[i] & 0xFFFF0000u)));
  }
  return m;
}

// grid (chunks, batch*heads): max |x| over kQuantChunkRows rows of one (batch, head). Chunks
// run along x, whose extent has no practical limit; batch*heads along y (at most 65535).
// fmaxf drops a NaN operand, as the reference's GPU quantiser does (Triton's max reduction);
// its CPU fallback (torch amax) would propagate it instead.
__global__ void __launch_bounds__(256) quant_amax_partial_kernel(const QuantSpace q, float* partial,
                                                                 int chunks, int* err) {
  const int bh = blockIdx.y;
  const int b = bh / q.heads;
  const int h = bh - b * q.heads;
  const int chunk = blockIdx.x;
  const int lane16 = threadIdx.x & 15;   // 16-byte column chunk of the 256-byte row
  const int rsub = threadIdx.x >> 4;     // 16 rows per pass
  float m = 0.f;
  const int row_end = min(q.seq, (chunk + 1) * kQuantChunkRows);
  for (int s = chunk * kQuantChunkRows + rsub; s < row_end; s += 16) {
    const long long off = quant_offset(q, b, s, h);
    if (off < 0) {
      if (err) atomicOr(err, kErrBadPage);
      continue;
    }
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(q.src + off) + lane16);
    m = fmaxf(m, bf16_bits_abs_max8(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = red[0];
    for (int i = 1; i < 8; ++i) r = fmaxf(r, red[i]);
    partial[static_cast<size_t>(bh) * chunks + chunk] = r;
  }
}

// grid (batch*heads): scale = max(amax / 448, 1e-12) with IEEE division.
__global__ void __launch_bounds__(256) quant_finalize_kernel(const float* partial, int chunks,
                                                             float* scale) {
  float m = 0.f;
  for (int i = threadIdx.x; i < chunks; i += blockDim.x)
    m = fmaxf(m, partial[static_cast<size_t>(blockIdx.x) * chunks + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = red[0];
    for (int i = 1; i < (blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
    scale[blockIdx.x] = fmaxf(__fdiv_rn(r, kFp8Max), 1.0e-12f);
  }
}

// One thread per 16 input bytes (8 values) -> 8 output bytes.
__global__ void __launch_bounds__(256) quant_apply_kernel(const QuantSpace q, const float* scale,
                                                          int* err) {
  const long long total = static_cast<long long>(q.batch) * q.seq * q.heads * (kHeadDim / 8);
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % (kHeadDim / 8));
    long long r = idx / (kHeadDim / 8);
    int h, s, b;
    if (q.paged) {  // head-major walk keeps page reads contiguous
      s = static_cast<int>(r % q.seq);
      r /= q.seq;
      h = static_cast<int>(r % q.heads);
      b = static_cast<int>(r / q.heads);
    } else {
      h = static_cast<int>(r % q.heads);
      r /= q.heads;
      s = static_cast<int>(r % q.seq);
      b = static_cast<int>(r / q.seq);
    }
    const long long off = quant_offset(q, b, s, h);
    if (off < 0) {
      if (err) atomicOr(err, kErrBadPage);
      continue;
    }
    const float sc = __ldg(scale + b * q.heads + h);
    const float inv = __frcp_rn(sc);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(q.src + off) + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
    uint2 o;
    o.x = quant4(f[0], f[1], f[2], f[3], sc, inv);
    o.y = quant4(f[4], f[5], f[6], f[7], sc, inv);
    reinterpret_cast<uint2*>(q.dst + off)[c] = o;
  }
}


// ------------------------------------------------------------------ per-part e4m3 quantiser
// Rows [src_start, src_start + count) of up to two bf16 row spaces (packed or paged) are
// quantised per head, each tensor with its own scale max(amax / 448, 1e-12), into e4m3 row
// spaces at [dst_start, dst_start + count). With zero_tail, the destination rows after the
// part up to the end of its last 128-row block are set to zero, so a part that starts on a
// block boundary leaves finite keys and values in the block's unused rows.
struct QuantRowsParams {
  RowsDev src[2];
  RowsDev dst[2];
  float* scale[2];      // [heads] per tensor
  unsigned* amax[2];    // [heads] per tensor: max |x| as float bits, zero before the amax pass
  int ntensors;
  int src_start;
  int dst_start;
  int count;
  int tail;             // zero rows after the part (0 without zero_tail)
  int heads;
  int* err;
};

// grid (ceil(count / 256), heads, ntensors): max |x| over 256 rows of one head, merged into
// the head's amax word with an integer atomic (non-negative floats order like their bits).
__global__ void __launch_bounds__(256) quant_rows_amax_kernel(const QuantRowsParams p) {
  const int h = blockIdx.y;
  const int t = blockIdx.z;
  const int c = threadIdx.x & 15;
  float m = 0.f;
  const int end = min(p.count, static_cast<int>(blockIdx.x + 1) * kQuantChunkRows);
  for (int i = blockIdx.x * kQuantChunkRows + (threadIdx.x >> 4); i < end; i += 16) {
    const uint8_t* s = row_address(p.src[t], p.src_start + i, h, p.heads, kHeadDim * 2);
    if (!s) {
      if (p.err) atomicOr(p.err, kErrBadIndex);
      continue;
    }
    m = fmaxf(m, bf16_bits_abs_max8(__ldg(reinterpret_cast<const uint4*>(s) + c)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = red[0];
    for (int i = 1; i < 8; ++i) r = fmaxf(r, red[i]);
    atomicMax(p.amax[t] + h, __float_as_uint(r));
  }
}

// One thread per 8 values of a (tensor, row, head): quantise with the head's scale, or write
// zeros in the tail rows; thread (row 0, head h, chunk 0) also stores the scale.
__global__ void __launch_bounds__(256) quant_rows_apply_kernel(const QuantRowsParams p) {
  const int rows = p.count + p.tail;
  const long long per_tensor = static_cast<long long>(rows) * p.heads * 16;
  const long long total = per_tensor * p.ntensors;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / per_tensor);
    const int rem = static_cast<int>(idx - t * per_tensor);
    const int c = rem & 15;
    const int rh = rem >> 4;
    const int h = rh % p.heads;
    const int i = rh / p.heads;
    uint8_t* d = row_address(p.dst[t], p.dst_start + i, h, p.heads, kHeadDim);
    if (!d) {
      if (p.err) atomicOr(p.err, kErrBadIndex);
      continue;
    }
    if (i >= p.count) {
      reinterpret_cast<uint2*>(d)[c] = make_uint2(0u, 0u);
      continue;
    }
    const float sc = fmaxf(__fdiv_rn(__uint_as_float(__ldcg(p.amax[t] + h)), kFp8Max), 1.0e-12f);
    if (i == 0 && c == 0) p.scale[t][h] = sc;
    const uint8_t* s = row_address(p.src[t], p.src_start + i, h, p.heads, kHeadDim * 2);
    if (!s) continue;  // reported by the amax pass
    const float inv = __frcp_rn(sc);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(s) + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
    uint2 o;
    o.x = quant4(f[0], f[1], f[2], f[3], sc, inv);
    o.y = quant4(f[4], f[5], f[6], f[7], sc, inv);
    reinterpret_cast<uint2*>(d)[c] = o;
  }
}


// ------------------------------------------------------------------ layout permutes
struct PermuteParams {
  const uint8_t* src;
  uint8_t* dst;
  long long dims[4];         // outer index space, row-major
  long long src_stride[4];   // bytes
  long long dst_stride[4];   // bytes
  int row_bytes;             // contiguous inner record, multiple of 16
};

__global__ void __launch_bounds__(256) permute_rows_kernel(const PermuteParams p) {
  const int cpr = p.row_bytes >> 4;
  const long long total = p.dims[0] * p.dims[1] * p.dims[2] * p.dims[3] * cpr;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % cpr);
    long long r = idx / cpr;
    long long so = 0, dof = 0;
#pragma unroll
    for (int k = 3; k >= 0; --k) {
      const long long i = r % p.dims[k];
      r /= p.dims[k];
      so += i * p.src_stride[k];
      dof += i * p.dst_stride[k];
    }
    reinterpret_cast<uint4*>(p.dst + dof)[c] = __ldg(reinterpret_cast<const uint4*>(p.src + so) + c);
  }
}

// ---------------------------------------------------------------- commit-level top-k summaries
// Column means of bf16 rows per (segment, head): the key summary of a committed block
// (F/streaming/cache.py:854, recomputed after retention at :1031-1034) and the media query
// summary (F/streaming/attention_hook.py:1279). Sums are fp64, which holds a sum of up to
// millions of bf16 values exactly at the magnitudes attention sees, so the atomic merge order
// does not change them; the mean is the fp64 quotient rounded to fp32.
constexpr int kSumChunkRows = 256;

struct SegMeansParams {
  RowsDev src;
  const int* segments;  // [n][2]: first logical row, rows
  int heads;
  double* sums;         // [n][heads][128], zero before the sum pass
  float* means;         // [n][heads][128]
  int n;
  int* err;
};

// grid (row chunks, heads, segments), 128 threads: thread d sums column d of its chunk.
__global__ void __launch_bounds__(128) seg_col_sums_kernel(const SegMeansParams p) {
  const int s = blockIdx.z;
  const int h = blockIdx.y;
  const int start = __ldg(p.segments + 2 * s);
  const int rows = __ldg(p.segments + 2 * s + 1);
  const int r0 = blockIdx.x * kSumChunkRows;
  if (r0 >= rows) return;
  const int r1 = min(rows, r0 + kSumChunkRows);
  double acc0 = 0.0, acc1 = 0.0;  // two chains: rows alternate between them
  int i = r0;
  for (; i + 1 < r1; i += 2) {
    const uint8_t* a = row_address(p.src, start + i, h, p.heads, kHeadDim * 2);
    const uint8_t* b = row_address(p.src, start + i + 1, h, p.heads, kHeadDim * 2);
    if (!a || !b) {
      if (p.err) atomicOr(p.err, kErrBadIndex);
      return;
    }
    const unsigned short va = __ldg(reinterpret_cast<const unsigned short*>(a) + threadIdx.x);
    const unsigned short vb = __ldg(reinterpret_cast<const unsigned short*>(b) + threadIdx.x);
    acc0 += static_cast<double>(__uint_as_float(static_cast<unsigned>(va) << 16));
    acc1 += static_cast<double>(__uint_as_float(static_cast<unsigned>(vb) << 16));
  }
  if (i < r1) {
    const uint8_t* a = row_address(p.src, start + i, h, p.heads, kHeadDim * 2);
    if (!a) {
      if (p.err) atomicOr(p.err, kErrBadIndex);
      return;
    }
    const unsigned short va = __ldg(reinterpret_cast<const unsigned short*>(a) + threadIdx.x);
    acc0 += static_cast<double>(__uint_as_float(static_cast<unsigned>(va) << 16));
  }
  atomicAdd(p.sums + (static_cast<size_t>(s) * p.heads + h) * kHeadDim + threadIdx.x, acc0 + acc1);
}

__global__ void __launch_bounds__(256) seg_col_means_kernel(const SegMeansParams p) {
  const long long total = static_cast<long long>(p.n) * p.heads * kHeadDim;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(idx / (static_cast<long long>(p.heads) * kHeadDim));
    const int rows = __ldg(p.segments + 2 * s + 1);
    p.means[idx] = rows > 0 ? __double2float_rn(__ddiv_rn(__ldcg(p.sums + idx), rows)) : 0.f;
  }
}

// score[i] = mean over heads of sum over d of summary[i][h][d] * query_mean[h][d]
// (F/streaming/attention_hook.py:1281-1286), from the fp32 means in fp64 (the products of two
// fp32 values are exact in fp64). One warp per part; fixed summation order.
__global__ void __launch_bounds__(256) commit_scores_kernel(const float* summaries,
                                                            const float* query_mean, int n,
                                                            int heads, double* scores) {
  const int part = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (part >= n) return;
  const float* a = summaries + static_cast<size_t>(part) * heads * kHeadDim;
  const int len = heads * kHeadDim;
  double acc = 0.0;
  for (int j = lane; j < len; j += 32)
    acc = fma(static_cast<double>(__ldg(a + j)), static_cast<double>(__ldg(query_mean + j)), acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) scores[part] = __ddiv_rn(acc, heads);
}

static int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

int quantize_launch(const QuantSpace& q, float* scale, float* partial, int chunks, int* err,
                    cudaStream_t stream) {
  if (q.batch * q.heads > kQuantMaxBatchHeads)
    return set_error(H3SA_ERR_INVALID, "fp8 quantiser: batch * heads = %d exceeds %d",
                     q.batch * q.heads, kQuantMaxBatchHeads);
  quant_amax_partial_kernel<<<dim3(chunks, q.batch * q.heads), 256, 0, stream>>>(q, partial,
                                                                                 chunks, err);
  quant_finalize_kernel<<<q.batch * q.heads, 256, 0, stream>>>(partial, chunks, scale);
  const long long work = static_cast<long long>(q.batch) * q.seq * q.heads * (kHeadDim / 8);
  quant_apply_kernel<<<grid_for(work, 256), 256, 0, stream>>>(q, scale, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("fp8 quantiser launch", e);
  return H3SA_OK;
}

static int quantize_with_scratch(const QuantSpace& q, float* scale, int* err,
                                 cudaStream_t stream) {
  const int chunks = (q.seq + kQuantChunkRows - 1) / kQuantChunkRows;
  const size_t bytes = static_cast<size_t>(q.batch) * q.heads * chunks * sizeof(float);
  void* partial = nullptr;
  cudaError_t e = cudaMallocAsync(&partial, bytes, stream);
  if (e != cudaSuccess) return set_cuda_error("cudaMallocAsync(fp8 amax scratch)", e);
  int rc = quantize_launch(q, scale, static_cast<float*>(partial), chunks, err, stream);
  e = cudaFreeAsync(partial, stream);
  if (rc == H3SA_OK && e != cudaSuccess) return set_cuda_error("cudaFreeAsync", e);
  return rc;
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_kv_copy_rows(const h3sa_rows* src, const h3sa_rows* dst, int32_t num_tensors,
                      const int32_t* src_index, int32_t src_start, const int32_t* dst_index,
                      int32_t dst_start, int32_t count, int32_t heads, int32_t row_bytes,
                      int32_t* device_error, void* stream) {
  if (num_tensors < 1 || num_tensors > 2 || !src || !dst)
    return set_error(H3SA_ERR_INVALID, "kv_copy_rows: 1 or 2 tensor pairs, got %d", num_tensors);
  if (count < 0 || heads <= 0 || row_bytes <= 0 || (row_bytes & 15))
    return set_error(H3SA_ERR_INVALID, "kv_copy_rows: count=%d heads=%d row_bytes=%d", count,
                     heads, row_bytes);
  if (count == 0) return H3SA_OK;
  CopyParams p;
  memset(&p, 0, sizeof(p));
  for (int t = 0; t < num_tensors; ++t) {
    const h3sa_rows* rs[2] = {&src[t], &dst[t]};
    RowsDev* rd[2] = {&p.src[t], &p.dst[t]};
    for (int k = 0; k < 2; ++k) {
      if (!rs[k]->base || (reinterpret_cast<uintptr_t>(rs[k]->base) & 15))
        return set_error(H3SA_ERR_INVALID, "kv_copy_rows: null or unaligned base");
      if (rs[k]->extent <= 0 || (rs[k]->paged && (!rs[k]->page_table || rs[k]->table_blocks <= 0)))
        return set_error(H3SA_ERR_INVALID, "kv_copy_rows: bad row space");
      rd[k]->base = static_cast<uint8_t*>(rs[k]->base);
      rd[k]->paged = rs[k]->paged ? 1 : 0;
      rd[k]->extent = rs[k]->extent;
      rd[k]->page_table = rs[k]->page_table;
      rd[k]->table_blocks = rs[k]->table_blocks;
    }
  }
  p.ntensors = num_tensors;
  p.src_index = src_index;
  p.src_start = src_start;
  p.dst_index = dst_index;
  p.dst_start = dst_start;
  p.count = count;
  p.heads = heads;
  p.row_bytes = row_bytes;
  p.err = device_error;
  const long long work = static_cast<long long>(count) * heads * (row_bytes / 16);
  kv_copy_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("kv_copy_kernel launch", e);
  return H3SA_OK;
}

int h3sa_quantize_fp8_per_head(const void* x, void* y, float* scale, int32_t batch,
                               int32_t seq, int32_t heads, int32_t dim, void* stream) {
  if (dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "quantize_fp8_per_head: dim must be 128, got %d", dim);
  if (batch <= 0 || seq <= 0 || heads <= 0 || !x || !y || !scale)
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_per_head: invalid arguments");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_per_head: tensors must be 16-byte aligned");
  if (static_cast<long long>(batch) * heads > kQuantMaxBatchHeads)
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_per_head: batch * heads = %lld exceeds %d",
                     static_cast<long long>(batch) * heads, kQuantMaxBatchHeads);
  QuantSpace q{};
  q.src = static_cast<const __nv_bfloat16*>(x);
  q.dst = static_cast<uint8_t*>(y);
  q.paged = 0;
  q.batch = batch;
  q.seq = seq;
  q.heads = heads;
  return quantize_with_scratch(q, scale, nullptr, static_cast<cudaStream_t>(stream));
}

int h3sa_quantize_fp8_pool(const void* pool, void* pool_fp8, float* scale, int32_t heads,
                           int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                           int32_t rows, int32_t* device_error, void* stream) {
  if (heads <= 0 || pool_pages <= 0 || rows <= 0 || !pool || !pool_fp8 || !scale || !page_table ||
      table_blocks <= 0 || static_cast<long long>(rows) > static_cast<long long>(table_blocks) * 128)
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_pool: invalid arguments");
  QuantSpace q{};
  q.src = static_cast<const __nv_bfloat16*>(pool);
  q.dst = static_cast<uint8_t*>(pool_fp8);
  q.paged = 1;
  q.batch = 1;
  q.seq = rows;
  q.heads = heads;
  q.pool_pages = pool_pages;
  q.page_table = page_table;
  q.table_blocks = table_blocks;
  return quantize_with_scratch(q, scale, device_error, static_cast<cudaStream_t>(stream));
}

int h3sa_quantize_fp8_rows(const h3sa_rows* src, const h3sa_rows* dst, int32_t num_tensors,
                           int32_t src_start, int32_t dst_start, int32_t count, int32_t heads,
                           float* scale0, float* scale1, uint32_t* amax_workspace,
                           int32_t zero_tail, int32_t* device_error, void* stream) {
  if (num_tensors < 1 || num_tensors > 2 || !src || !dst || !scale0 || !amax_workspace ||
      (num_tensors == 2 && !scale1))
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_rows: invalid tensors or outputs");
  if (count < 0 || heads <= 0 || heads > kQuantMaxBatchHeads || src_start < 0 || dst_start < 0)
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_rows: count=%d heads=%d start=%d/%d", count,
                     heads, src_start, dst_start);
  QuantRowsParams p;
  memset(&p, 0, sizeof(p));
  for (int t = 0; t < num_tensors; ++t) {
    const h3sa_rows* rs[2] = {&src[t], &dst[t]};
    RowsDev* rd[2] = {&p.src[t], &p.dst[t]};
    for (int k = 0; k < 2; ++k) {
      if (!rs[k]->base || (reinterpret_cast<uintptr_t>(rs[k]->base) & 15))
        return set_error(H3SA_ERR_INVALID, "quantize_fp8_rows: null or unaligned base");
      if (rs[k]->extent <= 0 || (rs[k]->paged && (!rs[k]->page_table || rs[k]->table_blocks <= 0)))
        return set_error(H3SA_ERR_INVALID, "quantize_fp8_rows: bad row space");
      rd[k]->base = static_cast<uint8_t*>(rs[k]->base);
      rd[k]->paged = rs[k]->paged ? 1 : 0;
      rd[k]->extent = rs[k]->extent;
      rd[k]->page_table = rs[k]->page_table;
      rd[k]->table_blocks = rs[k]->table_blocks;
    }
    p.amax[t] = reinterpret_cast<unsigned*>(amax_workspace) + t * heads;
  }
  p.scale[0] = scale0;
  p.scale[1] = scale1;
  p.ntensors = num_tensors;
  p.src_start = src_start;
  p.dst_start = dst_start;
  p.count = count;
  p.heads = heads;
  p.err = device_error;
  const int end = dst_start + count;
  p.tail = (zero_tail && dst[0].paged) ? (kBlockN - end % kBlockN) % kBlockN : 0;
  if (count == 0) return H3SA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax_workspace, 0, sizeof(uint32_t) * num_tensors * heads, st);
  if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(amax workspace)", e);
  const int chunks = (count + kQuantChunkRows - 1) / kQuantChunkRows;
  quant_rows_amax_kernel<<<dim3(chunks, heads, num_tensors), 256, 0, st>>>(p);
  const long long work = static_cast<long long>(count + p.tail) * heads * 16 * num_tensors;
  quant_rows_apply_kernel<<<grid_for(work, 256), 256, 0, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("quantize_fp8_rows launch", e);
  return H3SA_OK;
}

int h3sa_permute_rows(const void* src, void* dst, const int64_t* dims, const int64_t* src_strides,
                      const int64_t* dst_strides, int32_t row_bytes, void* stream) {
  if (!src || !dst || !dims || !src_strides || !dst_strides || row_bytes <= 0 || (row_bytes & 15))
    return set_error(H3SA_ERR_INVALID, "permute_rows: invalid arguments");
  if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return set_error(H3SA_ERR_INVALID, "permute_rows: tensors must be 16-byte aligned");
  PermuteParams p;
  p.src = static_cast<const uint8_t*>(src);
  p.dst = static_cast<uint8_t*>(dst);
  long long work = row_bytes / 16;
  for (int k = 0; k < 4; ++k) {
    if (dims[k] < 0 || (src_strides[k] & 15) || (dst_strides[k] & 15))
      return set_error(H3SA_ERR_INVALID, "permute_rows: dims must be >= 0, strides 16-byte multiples");
    p.dims[k] = dims[k];
    p.src_stride[k] = src_strides[k];
    p.dst_stride[k] = dst_strides[k];
    work *= dims[k];
  }
  p.row_bytes = row_bytes;
  if (work == 0) return H3SA_OK;
  permute_rows_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("permute_rows_kernel launch", e);
  return H3SA_OK;
}

int h3sa_segment_row_means(const h3sa_rows* src, const int32_t* segments, int32_t num_segments,
                           int32_t max_rows, int32_t heads, double* workspace, float* means,
                           int32_t* device_error, void* stream) {
  if (!src || !segments || !workspace || !means || num_segments < 0 || max_rows < 0 || heads <= 0 ||
      heads > kQuantMaxBatchHeads || num_segments > 65535)
    return set_error(H3SA_ERR_INVALID, "segment_row_means: invalid arguments (segments=%d, heads=%d)",
                     num_segments, heads);
  if (!src->base || (reinterpret_cast<uintptr_t>(src->base) & 15) || src->extent <= 0 ||
      (src->paged && (!src->page_table || src->table_blocks <= 0)))
    return set_error(H3SA_ERR_INVALID, "segment_row_means: bad row space");
  if (num_segments == 0) return H3SA_OK;
  SegMeansParams p;
  memset(&p, 0, sizeof(p));
  p.src.base = static_cast<uint8_t*>(src->base);
  p.src.paged = src->paged ? 1 : 0;
  p.src.extent = src->extent;
  p.src.page_table = src->page_table;
  p.src.table_blocks = src->table_blocks;
  p.segments = segments;
  p.heads = heads;
  p.sums = workspace;
  p.means = means;
  p.n = num_segments;
  p.err = device_error;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t cells = static_cast<size_t>(num_segments) * heads * kHeadDim;
  cudaError_t e = cudaMemsetAsync(workspace, 0, cells * sizeof(double), st);
  if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(segment sums)", e);
  const int chunks = max_rows > 0 ? (max_rows + kSumChunkRows - 1) / kSumChunkRows : 1;
  seg_col_sums_kernel<<<dim3(chunks, heads, num_segments), 128, 0, st>>>(p);
  seg_col_means_kernel<<<grid_for(static_cast<long long>(cells), 256), 256, 0, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("segment_row_means launch", e);
  return H3SA_OK;
}

int h3sa_commit_scores(const float* summaries, const float* query_mean, int32_t num_parts,
                       int32_t heads, double* scores, void* stream) {
  if (!summaries || !query_mean || !scores || num_parts < 0 || heads <= 0)
    return set_error(H3SA_ERR_INVALID, "commit_scores: invalid arguments");
  if (num_parts == 0) return H3SA_OK;
  commit_scores_kernel<<<(num_parts + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      summaries, query_mean, num_parts, heads, scores);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("commit_scores launch", e);
  return H3SA_OK;
}

}  // extern "C"
