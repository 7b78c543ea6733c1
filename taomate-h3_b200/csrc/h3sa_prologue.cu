// QK-RMSNorm + rotate-half RoPE on merged QKV, written in place, into the Ulysses send
// layout, or (the fused layer prologue) straight to the ranks that own each head: Q rows into
// their attention-ready planes and K/V rows into their paged KV caches, over NVLink.
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

// Where the rows go.
enum RouteMode : int {
  kRouteInPlace = 0,  // Q and K rewritten in the merged input, V untouched (not read)
  kRoutePack = 1,     // all three planes into the Ulysses send layout [W, 3, T, H/W, d]
  kRoutePeers = 2,    // Q into the owner's [W*T, H/W, d] plane, K/V into the owner's paged pools
};

struct PrologueParams {
  const __nv_bfloat16* src;   // merged [T, 3, H, d]
  __nv_bfloat16* dst;         // kRouteInPlace: == src; kRoutePack: the send layout
  const __nv_bfloat16* q_weight;
  const __nv_bfloat16* k_weight;
  const __nv_bfloat16* cos_sin;  // [cache_rows, rotary]: cos | sin halves
  const long long* positions;    // [T] rows of cos_sin
  int tokens, heads, rotary, cache_rows, world;
  float eps;
  int* err;
  int mode;
  // kRoutePeers: every rank's Q plane and paged pools (device arrays of `world` addresses),
  // the page table shared by the group, and the first logical cache row of this chunk
  int rank;
  const uint64_t* peer_q;
  const uint64_t* peer_k;
  const uint64_t* peer_v;
  const int* page_table;
  int table_blocks;
  int pool_pages;
  int dst_start;
};

__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Destination row (256 bytes) of (token t, plane j in {q, k, v}, head h); nullptr when a page
// lookup fails (reported by the caller).
__device__ __forceinline__ __nv_bfloat16* dst_row(const PrologueParams& p, int t, int j, int h) {
  if (p.mode == kRouteInPlace)
    return p.dst + ((static_cast<size_t>(t) * 3 + j) * p.heads + h) * kHeadDim;
  const int hl = p.heads / p.world;
  const int w = h / hl;
  const int lh = h - w * hl;
  if (p.mode == kRoutePack)
    return p.dst + (((static_cast<size_t>(w) * 3 + j) * p.tokens + t) * hl + lh) * kHeadDim;
  const int row = p.rank * p.tokens + t;  // row of the owner's all-rank sequence
  if (j == 0) {
    __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(static_cast<uintptr_t>(__ldg(p.peer_q + w)));
    return q + (static_cast<size_t>(row) * hl + lh) * kHeadDim;
  }
  const int logical = p.dst_start + row;
  const int blk = logical >> 7;
  const int page = blk < p.table_blocks ? __ldg(p.page_table + blk) : -1;
  if (page < 0 || page >= p.pool_pages) return nullptr;
  __nv_bfloat16* pool = reinterpret_cast<__nv_bfloat16*>(
      static_cast<uintptr_t>(__ldg((j == 1 ? p.peer_k : p.peer_v) + w)));
  return pool + ((static_cast<size_t>(lh) * p.pool_pages + page) * kBlockN + (logical & 127)) *
                    kHeadDim;
}

// RN32(1 / sqrt(x)) as the arithmetic above defines it (square root and division in IEEE fp64,
// one rounding to fp32), without the fp64 square root and division in the common case. Two
// Newton steps y <- y (3/2 - x y^2 / 2) in fp64 from the fp32 hardware estimate leave y within
// a few fp64 ulps of 1/sqrt(x), as is the fp64 expression itself; both then round to the same
// fp32 value unless they lie within 2^-46 (relative) of a midpoint between two fp32 values,
// and in that case the fp64 expression is evaluated (Ziv's rounding test).
__device__ __forceinline__ float rsqrt_rn32(float xf) {
  if (isinf(xf)) return 0.f;
  const double x = xf;
  double y = rsqrtf(xf);
  const double hx = 0.5 * x;
#pragma unroll
  for (int it = 0; it < 2; ++it) y = fma(y, fma(-hx * y, y, 0.5), y);
  const float f = static_cast<float>(y);
  const int bits = __float_as_int(f);
  const double lo = 0.5 * (static_cast<double>(__int_as_float(bits - 1)) + f);
  const double hi = 0.5 * (static_cast<double>(__int_as_float(bits + 1)) + f);
  const double margin = y * 0x1p-46;
  if (fabs(y - lo) < margin || fabs(y - hi) < margin)
    return static_cast<float>(1.0 / sqrt(x));
  return f;
}

// RMSNorm + rotate-half RoPE of one Q or K row held by a half-warp (8 values per lane, lane
// `sub` holds dims [8 sub, 8 sub + 8)). c/sn: this lane's cos/sin values of the token
// (rotating lanes only). Returns the lane's 8 output values packed as bf16.
__device__ __forceinline__ uint4 norm_rope_row(uint4 raw, const float (&w)[8], float eps,
                                               bool rotating, bool low, int partner,
                                               unsigned half_mask, const float (&c)[8],
                                               const float (&sn)[8]) {
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
  const float inv = rsqrt_rn32(__fadd_rn(var, eps));
  float n[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) n[e] = bf16r(__fmul_rn(__fmul_rn(v[e], inv), w[e]));
  float pn[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) pn[e] = __shfl_sync(half_mask, n[e], partner);
  float out[8];
  if (rotating) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float r = low ? -pn[e] : pn[e];
      out[e] = bf16r(bf16r(__fmul_rn(n[e], c[e])) + bf16r(__fmul_rn(r, sn[e])));
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
  return o;
}

__device__ __forceinline__ void unpack8(uint4 a, float (&f)[8]) {
  const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

// Rows of a token handled per half-warp before the next loads are issued.
constexpr int kRouteBatch = 4;

// One CTA per token at a time (grid-stride over tokens); half-warp k of the CTA takes rows
// k, k + 16, ... of the token's [3, H] rows (Q heads, then K, then V; in place only Q and K),
// loading kRouteBatch rows before computing, so each lane has that many 16-byte loads in
// flight. All index arithmetic is 32-bit; the plane of a row comes from two compares.
__global__ void __launch_bounds__(256, 3) qkv_norm_rope_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 15;                 // lane within the row
  const int base_lane = lane & 16;           // first lane of this half-warp
  const unsigned half_mask = 0xFFFFu << base_lane;
  const int hw = threadIdx.x >> 4;           // half-warp of the CTA, 0..15
  const int heads = p.heads;
  const int rows = (p.mode == kRouteInPlace ? 2 : 3) * heads;
  const int half = p.rotary >> 1;
  float wq[8], wk[8];
  unpack8(reinterpret_cast<const uint4*>(p.q_weight)[sub], wq);
  unpack8(reinterpret_cast<const uint4*>(p.k_weight)[sub], wk);
  const int d0 = 8 * sub;
  const bool rotating = d0 < p.rotary;
  const bool low = d0 < half;
  const int partner = base_lane + (low ? sub + (half >> 3) : sub - (half >> 3));
  const int phase = rotating ? (low ? d0 : d0 - half) : 0;
  for (int t = blockIdx.x; t < p.tokens; t += gridDim.x) {
    const long long pos = __ldg(p.positions + t);
    const bool pos_ok = pos >= 0 && pos < p.cache_rows;
    if (!pos_ok && threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadIndex);
    float c[8], sn[8];
    if (rotating && pos_ok) {
      const __nv_bfloat16* cs = p.cos_sin + static_cast<size_t>(pos) * p.rotary;
      unpack8(__ldg(reinterpret_cast<const uint4*>(cs + phase)), c);
      unpack8(__ldg(reinterpret_cast<const uint4*>(cs + half + phase)), sn);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) c[e] = sn[e] = 0.f;
    }
    const uint4* src = reinterpret_cast<const uint4*>(p.src) + static_cast<size_t>(t) * 3 * heads * 16;
    for (int r0 = hw; r0 < rows; r0 += 16 * kRouteBatch) {
      uint4 raw[kRouteBatch];
#pragma unroll
      for (int b = 0; b < kRouteBatch; ++b) {
        const int r = r0 + 16 * b;
        if (r < rows) raw[b] = __ldg(src + r * 16 + sub);
      }
#pragma unroll
      for (int b = 0; b < kRouteBatch; ++b) {
        const int r = r0 + 16 * b;
        if (r >= rows) break;
        const int j = (r >= heads) + (r >= 2 * heads);
        const int h = r - j * heads;
        uint4 o = raw[b];
        if (j < 2) {
          if (!pos_ok) continue;
          o = norm_rope_row(raw[b], j == 0 ? wq : wk, p.eps, rotating, low, partner, half_mask,
                            c, sn);
        }
        __nv_bfloat16* dst = dst_row(p, t, j, h);
        if (dst) reinterpret_cast<uint4*>(dst)[sub] = o;
        else if (sub == 0 && p.err) atomicOr(p.err, kErrBadPage);
      }
    }
  }
  if (p.mode == kRoutePeers) __threadfence_system();
}

static int prologue_launch(const PrologueParams& p, cudaStream_t stream) {
  int blocks = p.tokens < 148 * 8 ? p.tokens : 148 * 8;
  if (blocks < 1) blocks = 1;
  qkv_norm_rope_kernel<<<blocks, 256, 0, stream>>>(p);
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
  p.mode = kRouteInPlace;
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
  p.mode = kRoutePack;
  return prologue_launch(p, static_cast<cudaStream_t>(stream));
}

int h3sa_qkv_norm_rope_scatter_paged(const void* qkv, const void* q_weight, const void* k_weight,
                                     const void* cos_sin, int32_t cache_rows, int32_t rotary,
                                     const int64_t* positions, int32_t tokens, int32_t heads,
                                     int32_t head_dim, int32_t world, int32_t rank,
                                     const uint64_t* peer_q, const uint64_t* peer_key_pool,
                                     const uint64_t* peer_value_pool, int32_t pool_pages,
                                     const int32_t* page_table, int32_t table_blocks,
                                     int32_t dst_start, float eps, int32_t* device_error,
                                     void* stream) {
  int rc = check_prologue(qkv, q_weight, k_weight, cos_sin, cache_rows, rotary, positions, tokens,
                          heads, head_dim);
  if (rc) return rc;
  if (world <= 0 || heads % world)
    return set_error(H3SA_ERR_INVALID, "merged QKV heads are not divisible by Ulysses");
  if (rank < 0 || rank >= world || !peer_q || !peer_key_pool || !peer_value_pool || !page_table ||
      pool_pages <= 0 || table_blocks <= 0 || dst_start < 0)
    return set_error(H3SA_ERR_INVALID, "qkv prologue scatter: invalid peer or page arguments");
  if (static_cast<long long>(dst_start) + static_cast<long long>(world) * tokens >
      static_cast<long long>(table_blocks) * kBlockN)
    return set_error(H3SA_ERR_INVALID, "qkv prologue scatter: rows [%d, %lld) exceed the page "
                     "table's %d blocks", dst_start,
                     static_cast<long long>(dst_start) + static_cast<long long>(world) * tokens,
                     table_blocks);
  if (tokens == 0) return H3SA_OK;
  PrologueParams p{};
  p.src = static_cast<const __nv_bfloat16*>(qkv);
  p.dst = nullptr;
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
  p.mode = kRoutePeers;
  p.rank = rank;
  p.peer_q = peer_q;
  p.peer_k = peer_key_pool;
  p.peer_v = peer_value_pool;
  p.page_table = page_table;
  p.table_blocks = table_blocks;
  p.pool_pages = pool_pages;
  p.dst_start = dst_start;
  return prologue_launch(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
