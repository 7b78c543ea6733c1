// QK-RMSNorm + rotate-half RoPE on merged QKV, optionally written straight into the Ulysses
// send layout.
//
// Arithmetic (the fused prologue of T/inference/fused_kernels.py:413-485):
//   inv  = 1 / sqrt(mean(v^2) + eps)
//   n    = bf16(v * inv * w)                          for every dim
//   rope = bf16(bf16(n * cos) + bf16(rot(n) * sin))   for dims [0, rotary)
// with rot(n)[i] = -n[i + rotary/2] (i < rotary/2), n[i - rotary/2] otherwise. Half a warp per
// (token, head, q|k) row of 128 values, 8 per lane. The sum of squares is exact (each
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

// Half a warp per (token, head, plane) row: 16 lanes x 8 values. In place only the Q and K
// planes are visited; the pack variant also copies V.
__global__ void __launch_bounds__(256) qkv_norm_rope_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 15;                 // lane within the row
  const int base_lane = lane & 16;           // first lane of this half-warp
  const unsigned half_mask = 0xFFFFu << base_lane;
  const int planes = (p.world > 1) ? 3 : 2;
  const long long total = static_cast<long long>(p.tokens) * p.heads * planes;
  const long long step = static_cast<long long>(gridDim.x) * (blockDim.x >> 4);
  const int half = p.rotary >> 1;
  // this lane's 8 norm weights of each projection, read once
  float wq[8], wk[8];
  {
    const uint4 a = reinterpret_cast<const uint4*>(p.q_weight)[sub];
    const uint4 b = reinterpret_cast<const uint4*>(p.k_weight)[sub];
    const uint32_t ua[4] = {a.x, a.y, a.z, a.w}, ub[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wq[2 * i] = __uint_as_float(ua[i] << 16);
      wq[2 * i + 1] = __uint_as_float(ua[i] & 0xFFFF0000u);
      wk[2 * i] = __uint_as_float(ub[i] << 16);
      wk[2 * i + 1] = __uint_as_float(ub[i] & 0xFFFF0000u);
    }
  }
  const int d0 = 8 * sub;
  const bool rotating = d0 < p.rotary;
  const bool low = d0 < half;
  const int partner = base_lane + (low ? sub + (half >> 3) : sub - (half >> 3));
  const int phase = rotating ? (low ? d0 : d0 - half) : 0;
  for (long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 4) + (threadIdx.x >> 4);
       row < total; row += step) {
    const int j = static_cast<int>(row % planes);   // 0 q, 1 k, 2 v (pack only)
    const long long th = row / planes;
    const int h = static_cast<int>(th % p.heads);
    const int t = static_cast<int>(th / p.heads);
    const __nv_bfloat16* src = p.src + ((static_cast<size_t>(t) * 3 + j) * p.heads + h) * kHeadDim;
    __nv_bfloat16* dst = dst_row(p, t, j, h);
    const uint4 raw = reinterpret_cast<const uint4*>(src)[sub];
    if (j == 2) {  // V into the send layout, unchanged
      reinterpret_cast<uint4*>(dst)[sub] = raw;
      continue;
    }
    const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(u[i] << 16);
      v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += static_cast<double>(v[e] * v[e]);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(half_mask, ss, o, 16);
    // mean of the exact sum (scaling by 1/128 is exact), eps added in fp32
    const float var = static_cast<float>(ss * (1.0 / kHeadDim));
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(__fadd_rn(var, p.eps))));
    float n[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      n[e] = bf16r(__fmul_rn(__fmul_rn(v[e], inv), j == 0 ? wq[e] : wk[e]));
    float pn[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) pn[e] = __shfl_sync(half_mask, n[e], partner);
    const long long pos = p.positions[t];
    if (pos < 0 || pos >= p.cache_rows) {
      if (p.err && sub == 0) atomicOr(p.err, kErrBadIndex);
      continue;
    }
    float out[8];
    if (rotating) {
      const __nv_bfloat16* cs = p.cos_sin + static_cast<size_t>(pos) * p.rotary;
      const uint4 cr = *reinterpret_cast<const uint4*>(cs + phase);
      const uint4 sr = *reinterpret_cast<const uint4*>(cs + half + phase);
      const uint32_t cu[4] = {cr.x, cr.y, cr.z, cr.w}, su[4] = {sr.x, sr.y, sr.z, sr.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float c0 = __uint_as_float(cu[i] << 16), c1 = __uint_as_float(cu[i] & 0xFFFF0000u);
        const float s0 = __uint_as_float(su[i] << 16), s1 = __uint_as_float(su[i] & 0xFFFF0000u);
        const float r0 = low ? -pn[2 * i] : pn[2 * i];
        const float r1 = low ? -pn[2 * i + 1] : pn[2 * i + 1];
        out[2 * i] = bf16r(bf16r(__fmul_rn(n[2 * i], c0)) + bf16r(__fmul_rn(r0, s0)));
        out[2 * i + 1] = bf16r(bf16r(__fmul_rn(n[2 * i + 1], c1)) + bf16r(__fmul_rn(r1, s1)));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = n[e];
    }
    uint4 o;
    o.x = (__float_as_uint(out[0]) >> 16) | (__float_as_uint(out[1]) & 0xFFFF0000u);
    o.y = (__float_as_uint(out[2]) >> 16) | (__float_as_uint(out[3]) & 0xFFFF0000u);
    o.z = (__float_as_uint(out[4]) >> 16) | (__float_as_uint(out[5]) & 0xFFFF0000u);
    o.w = (__float_as_uint(out[6]) >> 16) | (__float_as_uint(out[7]) & 0xFFFF0000u);
    reinterpret_cast<uint4*>(dst)[sub] = o;
  }
}

static int prologue_launch(const PrologueParams& p, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.tokens) * p.heads * (p.world > 1 ? 3 : 2);
  long long blocks = (rows + 15) / 16;
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
  if (rotary <= 0 || rotary > head_dim || (rotary % 16) != 0)
    return set_error(H3SA_ERR_UNSUPPORTED, "qkv prologue: rotary span must be a multiple of 16 "
                     "within the head, got %d", rotary);
  if ((reinterpret_cast<uintptr_t>(cos_sin) | reinterpret_cast<uintptr_t>(q_weight) |
       reinterpret_cast<uintptr_t>(k_weight)) & 15)
    return set_error(H3SA_ERR_INVALID, "qkv prologue: weights and RoPE cache must be 16-byte aligned");
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
