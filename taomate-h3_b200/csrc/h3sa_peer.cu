// Peer memory for the fused Ulysses exchanges over NVLink.
//
// The sequence -> heads exchange before attention and the heads -> sequence exchange after it
// are all-to-alls between the ranks of one node. Instead of NCCL all-to-all plus layout copies
// on both sides, each rank writes straight into the other ranks' buffers through CUDA IPC
// mappings: h3sa_scatter_qkv stores this rank's rows of every head into the attention-ready
// q/k/v planes of the rank that owns the head, and the attention epilogue stores each output
// row into the sequence shard of the rank that owns the row (h3sa_attention_fwd_scatter).
// Plain 16-byte stores to peer memory over NVLink; no bulk or tensor copy touches a peer.
#include <cuda_runtime.h>

#include <cstring>

#include "h3sa_host.h"

namespace h3sa {

constexpr int kPeerHeadDim = 128;

struct ScatterParams {
  const uint4* src;         // [tokens, 3, heads, 128] bf16, this rank's sequence shard
  const uint64_t* peers;    // [world] base of each rank's [3, world * tokens, heads_local, 128]
  int tokens;
  int heads;
  int heads_local;
  int world;
  int rank;
};

// 16-byte chunk c of (token t, plane w, head h) goes to the rank owning h, at plane w, row
// rank * tokens + t, local head h % heads_local. Reads are contiguous; each destination row of
// 256 bytes is written by 16 consecutive threads. Every thread moves kUnroll chunks a grid
// stride apart, loads first, so that that many stores per thread are in flight over NVLink.
constexpr int kScatterUnroll = 4;

__device__ __forceinline__ uint4* scatter_dst(const ScatterParams& p, long long i) {
  constexpr int kChunks = kPeerHeadDim * 2 / 16;
  const int c = static_cast<int>(i % kChunks);
  long long r = i / kChunks;
  const int h = static_cast<int>(r % p.heads);
  r /= p.heads;
  const int w = static_cast<int>(r % 3);
  const long long t = r / 3;
  const int dest = h / p.heads_local;
  const int hl = h - dest * p.heads_local;
  const long long rows_all = static_cast<long long>(p.world) * p.tokens;
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uintptr_t>(__ldg(p.peers + dest)));
  const long long drow =
      (w * rows_all + static_cast<long long>(p.rank) * p.tokens + t) * p.heads_local + hl;
  return dst + drow * kChunks + c;
}

__global__ void scatter_qkv_kernel(const ScatterParams p) {
  constexpr int kChunks = kPeerHeadDim * 2 / 16;  // 16-byte chunks per row
  const long long total = static_cast<long long>(p.tokens) * 3 * p.heads * kChunks;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long base = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       base < total; base += stride * kScatterUnroll) {
    uint4 v[kScatterUnroll];
#pragma unroll
    for (int u = 0; u < kScatterUnroll; ++u) {
      const long long i = base + u * stride;
      if (i < total) v[u] = __ldg(p.src + i);
    }
#pragma unroll
    for (int u = 0; u < kScatterUnroll; ++u) {
      const long long i = base + u * stride;
      if (i < total) *scatter_dst(p, i) = v[u];
    }
  }
  __threadfence_system();
}

// The same exchange with the current chunk's K and V rows stored straight into the owner's
// paged KV pools ([heads_local, pool_pages * 128, 128] per rank) after `dst_start` logical
// rows, through a page table that is the same on every rank (the ranks of a Ulysses group
// commit the same rows, so their caches' tables agree); Q rows go to the owner's
// attention-ready [world * tokens, heads_local, 128] plane. This folds the cache append into
// the exchange.
struct ScatterPagedParams {
  const uint4* src;        // [tokens, 3, heads, 128] bf16, this rank's sequence shard
  const uint64_t* peer_q;  // [world] q planes
  const uint64_t* peer_k;  // [world] key pools
  const uint64_t* peer_v;  // [world] value pools
  const int* page_table;
  int table_blocks;
  int pool_pages;
  int dst_start;
  int tokens;
  int heads;
  int heads_local;
  int world;
  int rank;
  int* err;
};

__device__ __forceinline__ uint4* scatter_paged_dst(const ScatterPagedParams& p, long long i) {
  constexpr int kChunks = kPeerHeadDim * 2 / 16;
  const int c = static_cast<int>(i % kChunks);
  long long r = i / kChunks;
  const int h = static_cast<int>(r % p.heads);
  r /= p.heads;
  const int w = static_cast<int>(r % 3);
  const long long t = r / 3;
  const int dest = h / p.heads_local;
  const int hl = h - dest * p.heads_local;
  const long long row = static_cast<long long>(p.rank) * p.tokens + t;  // row of the chunk
  if (w == 0) {
    uint4* q = reinterpret_cast<uint4*>(static_cast<uintptr_t>(__ldg(p.peer_q + dest)));
    return q + (row * p.heads_local + hl) * kChunks + c;
  }
  const long long logical = p.dst_start + row;
  const int blk = static_cast<int>(logical / 128);
  const int page = blk < p.table_blocks ? __ldg(p.page_table + blk) : -1;
  if (page < 0 || page >= p.pool_pages) return nullptr;
  const uint64_t base = __ldg((w == 1 ? p.peer_k : p.peer_v) + dest);
  const long long pool_row = static_cast<long long>(page) * 128 + logical % 128;
  return reinterpret_cast<uint4*>(static_cast<uintptr_t>(base)) +
         ((static_cast<long long>(hl) * p.pool_pages * 128 + pool_row) * kChunks + c);
}

__global__ void scatter_qkv_paged_kernel(const ScatterPagedParams p) {
  const long long total = static_cast<long long>(p.tokens) * 3 * p.heads * (kPeerHeadDim * 2 / 16);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long base = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       base < total; base += stride * kScatterUnroll) {
    uint4 v[kScatterUnroll];
#pragma unroll
    for (int u = 0; u < kScatterUnroll; ++u) {
      const long long i = base + u * stride;
      if (i < total) v[u] = __ldg(p.src + i);
    }
#pragma unroll
    for (int u = 0; u < kScatterUnroll; ++u) {
      const long long i = base + u * stride;
      if (i < total) {
        uint4* dst = scatter_paged_dst(p, i);
        if (dst) *dst = v[u];
        else if (p.err) atomicOr(p.err, H3SA_DEVERR_BAD_PAGE);
      }
    }
  }
  __threadfence_system();
}

// Barrier over peer memory for the ranks of one node: every rank stores `epoch` into slot
// `rank` of every rank's flag array (release, system scope), then waits until all slots of
// its own array hold at least `epoch` (acquire). One thread per peer. The wait is bounded:
// after `limit_ns` (2 s by default) it sets H3SA_DEVERR_WAIT_TIMEOUT in `err` and returns.
constexpr long long kBarrierSpinNs = 2000000000LL;  // 2 s
constexpr long long kBarrierMaxSpinNs = 60000000000LL;  // longest limit a caller may set

__global__ void peer_barrier_kernel(const uint64_t* flags, int world, int rank,
                                    unsigned int epoch, long long limit_ns, int* err) {
  const int q = threadIdx.x;
  if (q < world) {
    unsigned int* remote =
        reinterpret_cast<unsigned int*>(static_cast<uintptr_t>(flags[q])) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  }
  __syncthreads();
  if (q < world) {
    const unsigned int* mine =
        reinterpret_cast<const unsigned int*>(static_cast<uintptr_t>(flags[rank])) + q;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (static_cast<int>(v - epoch) >= 0) break;
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (static_cast<long long>(t - t0) > limit_ns) {
        if (err) atomicOr(err, H3SA_DEVERR_WAIT_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return set_error(H3SA_ERR_INVALID, "peer_alloc: invalid arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return set_cuda_error("cudaMalloc(peer buffer)", e);
  return H3SA_OK;
}

int h3sa_peer_free(void* ptr) {
  if (!ptr) return H3SA_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_cuda_error("cudaFree(peer buffer)", e);
  return H3SA_OK;
}

int h3sa_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return set_error(H3SA_ERR_INVALID, "ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return set_cuda_error("cudaIpcGetMemHandle", e);
  std::memcpy(handle, &h, sizeof(h));
  return H3SA_OK;
}

int h3sa_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return set_error(H3SA_ERR_INVALID, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_cuda_error("cudaIpcOpenMemHandle", e);
  return H3SA_OK;
}

int h3sa_ipc_close(void* ptr) {
  if (!ptr) return H3SA_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_cuda_error("cudaIpcCloseMemHandle", e);
  return H3SA_OK;
}

int h3sa_scatter_qkv(const void* merged, int32_t tokens, int32_t heads, int32_t head_dim,
                     int32_t world, int32_t rank, const uint64_t* peer_qkv, void* stream) {
  if (head_dim != kPeerHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "scatter_qkv: head_dim must be 128, got %d", head_dim);
  if (!merged || !peer_qkv || tokens <= 0 || heads <= 0 || world <= 0 || rank < 0 ||
      rank >= world)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv: invalid arguments");
  if (heads % world)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv: num_heads=%d not divisible by Ulysses "
                     "world size %d", heads, world);
  if (reinterpret_cast<uintptr_t>(merged) & 15)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv: input must be 16-byte aligned");
  ScatterParams p;
  p.src = static_cast<const uint4*>(merged);
  p.peers = peer_qkv;
  p.tokens = tokens;
  p.heads = heads;
  p.heads_local = heads / world;
  p.world = world;
  p.rank = rank;
  const long long work = static_cast<long long>(tokens) * 3 * heads * (kPeerHeadDim * 2 / 16);
  long long blocks = (work + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  scatter_qkv_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("scatter_qkv_kernel launch", e);
  return H3SA_OK;
}

int h3sa_scatter_qkv_paged(const void* merged, int32_t tokens, int32_t heads, int32_t head_dim,
                           int32_t world, int32_t rank, const uint64_t* peer_q,
                           const uint64_t* peer_key_pool, const uint64_t* peer_value_pool,
                           int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                           int32_t dst_start, int32_t* device_error, void* stream) {
  if (head_dim != kPeerHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "scatter_qkv_paged: head_dim must be 128, got %d",
                     head_dim);
  if (!merged || !peer_q || !peer_key_pool || !peer_value_pool || !page_table || tokens <= 0 ||
      heads <= 0 || world <= 0 || rank < 0 || rank >= world || pool_pages <= 0 ||
      table_blocks <= 0 || dst_start < 0)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv_paged: invalid arguments");
  if (heads % world)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv_paged: num_heads=%d not divisible by "
                     "Ulysses world size %d", heads, world);
  if (static_cast<int64_t>(dst_start) + static_cast<int64_t>(world) * tokens >
      static_cast<int64_t>(table_blocks) * 128)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv_paged: rows [%d, %lld) exceed %d table "
                     "blocks", dst_start,
                     static_cast<long long>(dst_start) + static_cast<long long>(world) * tokens,
                     table_blocks);
  if (reinterpret_cast<uintptr_t>(merged) & 15)
    return set_error(H3SA_ERR_INVALID, "scatter_qkv_paged: input must be 16-byte aligned");
  ScatterPagedParams p;
  p.src = static_cast<const uint4*>(merged);
  p.peer_q = peer_q;
  p.peer_k = peer_key_pool;
  p.peer_v = peer_value_pool;
  p.page_table = page_table;
  p.table_blocks = table_blocks;
  p.pool_pages = pool_pages;
  p.dst_start = dst_start;
  p.tokens = tokens;
  p.heads = heads;
  p.heads_local = heads / world;
  p.world = world;
  p.rank = rank;
  p.err = device_error;
  const long long work = static_cast<long long>(tokens) * 3 * heads * (kPeerHeadDim * 2 / 16);
  long long blocks = (work + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  scatter_qkv_paged_kernel<<<static_cast<int>(blocks), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("scatter_qkv_paged_kernel launch", e);
  return H3SA_OK;
}

int h3sa_peer_barrier_limit(const uint64_t* peer_flags, int32_t world, int32_t rank,
                            uint32_t epoch, int64_t limit_ns, int32_t* device_error,
                            void* stream) {
  if (!peer_flags || world <= 0 || world > 1024 || rank < 0 || rank >= world || epoch == 0)
    return set_error(H3SA_ERR_INVALID, "peer_barrier: invalid arguments");
  if (limit_ns <= 0 || limit_ns > kBarrierMaxSpinNs)
    return set_error(H3SA_ERR_INVALID, "peer_barrier: wait limit %lld ns outside (0, %lld]",
                     static_cast<long long>(limit_ns), kBarrierMaxSpinNs);
  peer_barrier_kernel<<<1, ((world + 31) / 32) * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      peer_flags, world, rank, epoch, static_cast<long long>(limit_ns), device_error);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("peer_barrier_kernel launch", e);
  return H3SA_OK;
}

int h3sa_peer_barrier(const uint64_t* peer_flags, int32_t world, int32_t rank, uint32_t epoch,
                      int32_t* device_error, void* stream) {
  return h3sa_peer_barrier_limit(peer_flags, world, rank, epoch, kBarrierSpinNs, device_error,
                                 stream);
}

}  // extern "C"
