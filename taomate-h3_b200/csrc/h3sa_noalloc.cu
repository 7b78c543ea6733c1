// Allocation-free variant of the per-head e4m3 quantiser.
//
// h3sa_quantize_fp8_per_head takes its partial-amax scratch from the stream-ordered
// allocator on every call. Some callers cannot allocate at all while they run: code that
// executes inside a region where a device allocation would be unsafe or forbidden (an
// allocator that is being torn down or reconfigured, a caller that has handed all device
// memory to its own pool, a real-time loop with a no-allocation rule). This entry point
// serves them: its scratch is a fixed file-scope device array, sized below, and no call
// allocates or frees device memory.
//
// The array is shared by every call on a device and keeps what the last call left in it.
// The quantiser writes every scratch slot it reads (one partial maximum per (batch, head,
// 256-row chunk)) before reading it, so no clearing is needed. Two calls whose device work
// overlaps (different streams with no ordering between them, or different host threads)
// race on the array and may produce wrong scales; callers serialise them.

#include <mutex>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {

// 64 Ki floats = 256 KiB: batch * heads * ceil(seq / 256) partial maxima at most, e.g.
// 24 heads of up to 2730 * 256 = 698,880 rows each (one more chunk would need 65,544 slots).
constexpr int kNoAllocScratchFloats = 65536;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_amax_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_amax_scratch per device, looked up once per device.
static float* g_scratch_ptr[kMaxDevices];
static std::mutex g_scratch_mutex;

static int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(H3SA_ERR_UNSUPPORTED, "quantize_fp8_per_head_noalloc: device %d >= %d", dev,
                     kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_amax_scratch);
    if (e != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(amax scratch)", e);
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return H3SA_OK;
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_quantize_fp8_per_head_noalloc(const void* x, void* y, float* scale, int32_t batch,
                                       int32_t seq, int32_t heads, int32_t dim, void* stream) {
  if (dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED,
                     "quantize_fp8_per_head_noalloc: dim must be 128, got %d", dim);
  if (batch <= 0 || seq <= 0 || heads <= 0 || !x || !y || !scale)
    return set_error(H3SA_ERR_INVALID, "quantize_fp8_per_head_noalloc: invalid arguments");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return set_error(H3SA_ERR_INVALID,
                     "quantize_fp8_per_head_noalloc: tensors must be 16-byte aligned");
  if (static_cast<long long>(batch) * heads > kQuantMaxBatchHeads)
    return set_error(H3SA_ERR_INVALID,
                     "quantize_fp8_per_head_noalloc: batch * heads = %lld exceeds %d",
                     static_cast<long long>(batch) * heads, kQuantMaxBatchHeads);
  const long long chunks = (static_cast<long long>(seq) + kQuantChunkRows - 1) / kQuantChunkRows;
  const long long slots = static_cast<long long>(batch) * heads * chunks;
  if (slots > kNoAllocScratchFloats)
    return set_error(H3SA_ERR_INVALID,
                     "quantize_fp8_per_head_noalloc: batch*heads*ceil(seq/256) = %lld exceeds the "
                     "fixed scratch of %d partial maxima; use h3sa_quantize_fp8_per_head",
                     slots, kNoAllocScratchFloats);
  float* partial = nullptr;
  int rc = noalloc_scratch(&partial);
  if (rc != H3SA_OK) return rc;
  QuantSpace q{};
  q.src = static_cast<const __nv_bfloat16*>(x);
  q.dst = static_cast<uint8_t*>(y);
  q.paged = 0;
  q.batch = batch;
  q.seq = seq;
  q.heads = heads;
  return quantize_launch(q, scale, partial, static_cast<int>(chunks), nullptr,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
