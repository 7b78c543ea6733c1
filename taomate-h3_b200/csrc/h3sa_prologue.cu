// QK-RMSNorm + rotate-half RoPE on merged QKV, optionally written straight into the Ulysses
// send layout.
//
// Arithmetic (the fused prologue of T/inference/fused_kernels.py:413-485):
//   inv  = 1 / sqrt(mean(v^2) + eps)
//   n    = bf16(v * inv * w)                          for every dim
//   rope = bf16(bf16(n * cos) + bf16(rot(n) * sin))   for dims [0, rotary)
// with rot(n)[i] = -n[i + rotary/2] (i < rotary/2), n[i - rotary/2] otherwise. One warp per
// (token, head, q|k) row of 128 values, 4 per lane. The sum of squares is exact (each
// square of a bf16 value is exact in fp32 and the 128 of them sum exactly in fp64), so the
// result does not depend on the reduction order; mean in fp64 rounded to fp32, eps added in
// fp32 (as the reference adds it), reciprocal square root in IEEE fp64 rounded once to fp32.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstring>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {

struct PrologueParams {
  const __nv_bfloat16* src;   // merged [T, 3, H, d]
  __nv_bfloat16* dst;         // in place (== src) or send layout [W, 3, T, H/W, d]
  const __nv_bfloat16* q_weight;
  const __nv_bfloat16* k_weight;
  const __nv_bfloat16* cos_sin;  // [cache_rows, rotary]: cos | sin halves
  const long long* positions;    // [T] rows of cos_sin
  int tokens, heads, rotary, cache_rows, world;
  float eps;
  int* err;
};

__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Destination of (token t, plane j in {q, k, v}, head h): merged in place or send layout.
__device__ __forceinline__ __nv_bfloat16* dst_row(const PrologueParams& p, int t, int j, int h) {
  if (p.world <= 1)
    return p.dst + ((static_cast<size_t>(t) * 3 + j) * p.heads + h) * kHeadDim;
  const int hl = p.heads / p.world;
  const int w = h / hl;
  return p.dst +
         (((static_cast<size_t>(w) * 3 + j) * p.tokens + t) * hl + (h - w * hl)) * kHeadDim;
}

__global__ void __launch_bounds__(256) qkv_norm_rope_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long total = static_cast<long long>(p.tokens) * p.heads * 3;
  const int half = p.rotary >> 1;
  for (long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < total; row += warps) {
    const int j = static_cast<int>(row % 3);          // 0 q, 1 k, 2 v
    const long long th = row / 3;
    const int h = static_cast<int>(th % p.heads);
    const int t = static_cast<int>(th / p.heads);
    const __nv_bfloat16* src = p.src + ((static_cast<size_t>(t) * 3 + j) * p.heads + h) * kHeadDim;
    __nv_bfloat16* dst = dst_row(p, t, j, h);
    const uint2 raw = reinterpret_cast<const uint2*>(src)[lane];
    if (j == 2) {  // V: copied (send layout) or untouched (in place)
      if (dst != src) reinterpret_cast<uint2*>(dst)[lane] = raw;
      continue;
    }
    float v[4];
    v[0] = __uint_as_float(raw.x << 16);
    v[1] = __uint_as_float(raw.x & 0xFFFF0000u);
    v[2] = __uint_as_float(raw.y << 16);
    v[3] = __uint_as_float(raw.y & 0xFFFF0000u);
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += static_cast<double>(v[e] * v[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float var = static_cast<float>(ss / static_cast<double>(kHeadDim));
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(__fadd_rn(var, p.eps))));
    const __nv_bfloat16* wp = (j == 0) ? p.q_weight : p.k_weight;
    float n[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) n[e] = bf16r(__fmul_rn(__fmul_rn(v[e], inv), __bfloat162float(wp[4 * lane + e])));
    // partner values for the rotate-half: lane +- rotary/8 (4 dims per lane)
    const int shift = half >> 2;
    const bool low = 4 * lane < half;
    const int src_lane = low ? lane + shift : lane - shift;
    float pn[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pn[e] = __shfl_sync(0xffffffffu, n[e], src_lane & 31);
    float out[4];
    const long long pos = p.positions[t];
    if (pos < 0 || pos >= p.cache_rows) {
      if (p.err) atomicOr(p.err, kErrBadIndex);
      continue;
    }
    const __nv_bfloat16* cs = p.cos_sin + static_cast<size_t>(pos) * p.rotary;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 4 * lane + e;
      if (d < p.rotary) {
        const int ph = d % half;
        const float c = __bfloat162float(cs[ph]);
        const float s = __bfloat162float(cs[half + ph]);
        const float rot = low ? -pn[e] : pn[e];
        out[e] = bf16r(bf16r(__fmul_rn(n[e], c)) + bf16r(__fmul_rn(rot, s)));
      } else {
        out[e] = n[e];
      }
    }
    uint2 o;
    o.x = (__float_as_uint(out[0]) >> 16) | (__float_as_uint(out[1]) & 0xFFFF0000u);
    o.y = (__float_as_uint(out[2]) >> 16) | (__float_as_uint(out[3]) & 0xFFFF0000u);
    reinterpret_cast<uint2*>(dst)[lane] = o;
  }
}

static int prologue_launch(const PrologueParams& p, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.tokens) * p.heads * 3;
  long long blocks = (rows + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  qkv_norm_rope_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("qkv_norm_rope_kernel launch", e);
  return H3SA_OK;
}

static int check_prologue(const void* qkv, const void* q_weight, const void* k_weight,
                          const void* cos_sin, int32_t cache_rows, int32_t rotary,
                          const int64_t* positions, int32_t tokens, int32_t heads,
                          int32_t head_dim) {
  if (head_dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "qkv prologue requires head_dim 128, got %d", head_dim);
  if (!qkv || !q_weight || !k_weight || !cos_sin || !positions)
    return set_error(H3SA_ERR_INVALID, "qkv prologue: null pointer argument");
  if (tokens < 0 || heads <= 0 || cache_rows <= 0)
    return set_error(H3SA_ERR_INVALID, "qkv prologue: invalid sizes");
  if (rotary <= 0 || rotary > head_dim || (rotary % 8) != 0)
    return set_error(H3SA_ERR_UNSUPPORTED, "qkv prologue: rotary span must be a multiple of 8 "
                     "within the head, got %d", rotary);
  if (reinterpret_cast<uintptr_t>(qkv) & 15)
    return set_error(H3SA_ERR_INVALID, "qkv prologue: tensors must be 16-byte aligned");
  return H3SA_OK;
}

}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_qkv_norm_rope(void* qkv, const void* q_weight, const void* k_weight,
                       const void* cos_sin, int32_t cache_rows, int32_t rotary,
                       const int64_t* positions, int32_t tokens, int32_t heads,
                       int32_t head_dim, float eps, int32_t* device_error, void* stream) {
  int rc = check_prologue(qkv, q_weight, k_weight, cos_sin, cache_rows, rotary, positions, tokens,
                          heads, head_dim);
  if (rc) return rc;
  if (tokens == 0) return H3SA_OK;
  PrologueParams p{};
  p.src = static_cast<const __nv_bfloat16*>(qkv);
  p.dst = static_cast<__nv_bfloat16*>(qkv);
  p.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  p.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
  p.positions = reinterpret_cast<const long long*>(positions);
  p.tokens = tokens;
  p.heads = heads;
  p.rotary = rotary;
  p.cache_rows = cache_rows;
  p.world = 1;
  p.eps = eps;
  p.err = device_error;
  return prologue_launch(p, static_cast<cudaStream_t>(stream));
}

int h3sa_qkv_norm_rope_pack(const void* qkv, void* send, const void* q_weight,
                            const void* k_weight, const void* cos_sin, int32_t cache_rows,
                            int32_t rotary, const int64_t* positions, int32_t tokens,
                            int32_t heads, int32_t head_dim, int32_t world, float eps,
                            int32_t* device_error, void* stream) {
  int rc = check_prologue(qkv, q_weight, k_weight, cos_sin, cache_rows, rotary, positions, tokens,
                          heads, head_dim);
  if (rc) return rc;
  if (!send || (reinterpret_cast<uintptr_t>(send) & 15))
    return set_error(H3SA_ERR_INVALID, "qkv prologue pack: null or unaligned send buffer");
  if (world <= 0 || heads % world)
    return set_error(H3SA_ERR_INVALID, "merged QKV heads are not divisible by Ulysses");
  if (send == qkv)
    return set_error(H3SA_ERR_INVALID, "qkv prologue pack: send buffer must not alias the input");
  if (tokens == 0) return H3SA_OK;
  PrologueParams p{};
  p.src = static_cast<const __nv_bfloat16*>(qkv);
  p.dst = static_cast<__nv_bfloat16*>(send);
  p.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  p.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
  p.positions = reinterpret_cast<const long long*>(positions);
  p.tokens = tokens;
  p.heads = heads;
  p.rotary = rotary;
  p.cache_rows = cache_rows;
  p.world = world;
  p.eps = eps;
  p.err = device_error;
  return prologue_launch(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
