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
#include "h3sa_fp8.cuh"
#include "h3sa_host.h"

namespace h3sa {

// Where the rows go.
enum RouteMode : int {
  kRouteInPlace = 0,  // Q and K rewritten in the merged input, V untouched (not read)
  kRoutePack = 1,     // all three planes into the Ulysses send layout [W, 3, T, H/W, d]
  kRoutePeers = 2,    // Q into the owner's [W*T, H/W, d] plane, K/V into the owner's paged pools
  kRouteAmax = 3,     // no stores: per-(plane, head) max |x| of the rotated rows (e4m3 pass 1)
  kRoutePeersFp8 = 4, // as kRoutePeers with e4m3 rows at the pass-1 scales (e4m3 pass 2)
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
  int heads_local;  // heads / world
  int hl_recip;     // ceil(65536 / heads_local): h / heads_local = (h * hl_recip) >> 16
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
  // e4m3 passes: per-(plane, head) amax words [3][H] (float bits; pass 1 adds this rank's
  // rows, pass 2 reads the group's maxima), the token rows pass 1 counts ([T] flags, null: all),
  // every rank's e4m3 Q plane and paged pools with their page table, and this rank's scales
  unsigned* amax;
  int amax_sets;             // pass 2: maxima over this many [3][H] sets of words
  const uint8_t* amax_rows;
  int bf16_unflagged_only;   // pass 2: bf16 copies only of the rows amax_rows leaves out
  const uint64_t* peer_q8;
  const uint64_t* peer_k8;
  const uint64_t* peer_v8;
  const int* table8;
  int table8_blocks;
  int pool8_pages;
  int dst8_start;
  float* scale_out[3];  // [H / W] each: this rank's heads
};

__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Destination row (256 bytes) of (token t, plane j in {q, k, v}, head h); nullptr when a page
// lookup fails (reported by the caller).
template <int kMode>
__device__ __forceinline__ __nv_bfloat16* dst_row(const PrologueParams& p, int t, int j, int h) {
  if constexpr (kMode == kRouteInPlace)
    return p.dst + ((static_cast<size_t>(t) * 3 + j) * p.heads + h) * kHeadDim;
  const int hl = p.heads_local;
  const int w = (h * p.hl_recip) >> 16;  // h / hl, exact for h < 256 (host-checked)
  const int lh = h - w * hl;
  if constexpr (kMode == kRoutePack)
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

// e4m3 destination row (128 bytes) of (token t, plane j, head h) for kRoutePeersFp8; nullptr
// when a page lookup fails.
__device__ __forceinline__ uint8_t* dst8_row(const PrologueParams& p, int t, int j, int h) {
  const int hl = p.heads_local;
  const int w = (h * p.hl_recip) >> 16;
  const int lh = h - w * hl;
  const int row = p.rank * p.tokens + t;
  if (j == 0) {
    uint8_t* q = reinterpret_cast<uint8_t*>(static_cast<uintptr_t>(__ldg(p.peer_q8 + w)));
    return q + (static_cast<size_t>(row) * hl + lh) * kHeadDim;
  }
  const int logical = p.dst8_start + row;
  const int blk = logical >> 7;
  const int page = blk < p.table8_blocks ? __ldg(p.table8 + blk) : -1;
  if (page < 0 || page >= p.pool8_pages) return nullptr;
  uint8_t* pool = reinterpret_cast<uint8_t*>(
      static_cast<uintptr_t>(__ldg((j == 1 ? p.peer_k8 : p.peer_v8) + w)));
  return pool + ((static_cast<size_t>(lh) * p.pool8_pages + page) * kBlockN + (logical & 127)) *
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

// RMSNorm + rotate-half RoPE of one Q or K row held by a half-warp (lane `sub` holds dims
// [8 sub, 8 sub + 8) as four bf16 pairs). w2: this lane's norm weights as fp32 pairs; c / sn:
// its cos / sin values of the token as bf16 pairs (rotating lanes only). Every rounding point
// of the arithmetic is kept, in packed form: v * inv * w in fp32 pairs (two roundings), one
// rounding to bf16 per value (cvt.rn.bf16x2), then n * cos and rot(n) * sin as bf16 products
// and their sum as a bf16 sum, each exact before its single rounding to bf16 as the
// reference's fp32 product or sum rounded to bf16 is (a sum of two bf16 values that fp32
// cannot hold exactly is far from any bf16 rounding midpoint). Partners exchange packed pairs.
__device__ __forceinline__ uint4 norm_rope_row(uint4 raw, const uint64_t (&w2)[4], float eps,
                                               bool rotating, bool low, int partner,
                                               unsigned half_mask, const uint32_t (&c)[4],
                                               const uint32_t (&sn)[4]) {
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
  float lo[4], hi[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo[i] = __uint_as_float(u[i] << 16);
    hi[i] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
  // sum of squares: each square of a bf16 value is exact in fp64, and so is the sum
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const double a = lo[i], b = hi[i];
    ss = fma(a, a, ss);
    ss = fma(b, b, ss);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(half_mask, ss, o, 16);
  // mean of the exact sum (scaling by 1/128 is exact), eps added in fp32
  const float var = static_cast<float>(ss * (1.0 / kHeadDim));
  const float inv = rsqrt_rn32(__fadd_rn(var, eps));
  const uint64_t inv2 = f2_pack(inv, inv);
  uint32_t n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float x0, x1;
    f2_unpack(f2_mul(f2_mul(f2_pack(lo[i], hi[i]), inv2), w2[i]), x0, x1);
    n[i] = pack_bf16x2(x0, x1);
  }
  uint32_t pn[4];  // every lane of the half-warp takes part in the exchange
#pragma unroll
  for (int i = 0; i < 4; ++i) pn[i] = __shfl_sync(half_mask, n[i], partner);
  if (!rotating) return make_uint4(n[0], n[1], n[2], n[3]);
  uint32_t out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t r = low ? pn[i] ^ 0x80008000u : pn[i];  // rot(n) = -n[i + rotary/2] first
    out[i] = bf2_add(bf2_mul(n[i], c[i]), bf2_mul(r, sn[i]));
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__device__ __forceinline__ void unpack8(uint4 a, float (&f)[8]) {
  const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

// Staged pipeline, one CTA per contiguous range of tokens. Warp 8 (the producer) streams each
// token into a ring of kPipeStages shared-memory slots with plain bulk copies: the token's
// merged rows (Q and K heads in place, all three planes otherwise; contiguous in the merged
// layout) and its cos / sin row, all completing on the slot's full barrier. Warps 0-7 (16
// half-warps) take the slot's rows k, k + 16, ..., normalise and rotate the Q/K rows from
// shared memory and store every row to its destination, then release the slot. A slot holds
// a whole token (18 KB at 24 heads), so the copies of the next slots are in flight while the
// consumers work: the bytes in flight per SM no longer depend on registers. Every wait is
// bounded.
constexpr int kPipeStages = 4;
constexpr int kPipeConsumerWarps = 8;
constexpr int kPipeThreads = (kPipeConsumerWarps + 1) * 32;

struct PipeSmemLayout {
  int slot_bytes;   // rows of a token, rounded to 128 bytes
  int cs_bytes;     // cos / sin row, rounded to 16 bytes
  int total;        // bytes of dynamic shared memory
};

__host__ __device__ inline PipeSmemLayout pipe_layout(int rows_pt, int rotary, int aux_words = 0) {
  PipeSmemLayout l;
  l.slot_bytes = (rows_pt * kHeadDim * 2 + 127) / 128 * 128;
  l.cs_bytes = (rotary * 2 + 15) / 16 * 16;
  // slots, cos/sin rows, full + empty barriers, per-slot position-valid flags, abort flag,
  // then the e4m3 passes' per-row words (amax, or scale and reciprocal)
  l.total = kPipeStages * (l.slot_bytes + l.cs_bytes) + kPipeStages * 2 * 8 + kPipeStages * 4 + 16 +
            aux_words * 4;
  return l;
}

// aux words of a mode: pass 1 keeps one amax per (plane, head), pass 2 a scale and its
// reciprocal
__host__ __device__ inline int pipe_aux_words(int mode, int heads) {
  return mode == kRouteAmax ? 3 * heads : mode == kRoutePeersFp8 ? 6 * heads : 0;
}

template <int kMode>
__global__ void __launch_bounds__(kPipeThreads, 3) qkv_norm_rope_pipe_kernel(const PrologueParams p,
                                                                             int tokens_per_cta) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int heads = p.heads;
  const int rows_pt = (kMode == kRouteInPlace ? 2 : 3) * heads;
  const PipeSmemLayout L = pipe_layout(rows_pt, p.rotary, pipe_aux_words(kMode, heads));
  uint8_t* slots = smem;
  uint8_t* cs_rows = smem + kPipeStages * L.slot_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(cs_rows + kPipeStages * L.cs_bytes);
  uint64_t* empty = full + kPipeStages;
  int* pos_ok = reinterpret_cast<int*>(empty + kPipeStages);
  volatile int* abort_flag = pos_ok + kPipeStages;
  uint32_t* aux = reinterpret_cast<uint32_t*>(pos_ok + kPipeStages + 4);  // e4m3 passes
  const int t0 = blockIdx.x * tokens_per_cta;
  const int t1 = min(p.tokens, t0 + tokens_per_cta);
  const int n = max(0, t1 - t0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPipeStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), kPipeConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t row_bytes = static_cast<uint32_t>(rows_pt) * kHeadDim * 2;
  if (warp == kPipeConsumerWarps) {
    // ------------------------------------------------------------------ producer
    // positions of 32 tokens at a time, one per lane, handed to lane 0 by shuffles
    int issued = 0;
    for (int c0 = 0; c0 < n && !*abort_flag; c0 += 32) {
      const long long my_pos = c0 + lane < n ? __ldg(p.positions + t0 + c0 + lane) : 0;
      const int m = min(32, n - c0);
      for (int k = 0; k < m; ++k) {
        const long long pos = __shfl_sync(0xffffffffu, my_pos, k);
        if (lane == 0) {
          const int i = c0 + k;
          const int s = i % kPipeStages;
          const bool ok = i < kPipeStages ||
                          mbar_wait(smem_u32(&empty[s]), ((i / kPipeStages) - 1) & 1, abort_flag,
                                    p.err);
          if (ok) {
            const bool pv = pos >= 0 && pos < p.cache_rows;
            pos_ok[s] = pv ? 1 : 0;
            const uint32_t bar = smem_u32(&full[s]);
            mbar_expect_tx(bar, row_bytes + (pv ? 2u * p.rotary : 0u));
            bulk_load(smem_u32(slots + s * L.slot_bytes),
                      p.src + static_cast<size_t>(t0 + i) * 3 * heads * kHeadDim, row_bytes, bar);
            if (pv)
              bulk_load(smem_u32(cs_rows + s * L.cs_bytes),
                        p.cos_sin + static_cast<size_t>(pos) * p.rotary, 2u * p.rotary, bar);
            issued = i + 1;
          }
        }
        __syncwarp();
        if (*abort_flag) break;
      }
    }
    // leave no bulk copy in flight past the end of the CTA: wait for the last slots' data
    if (lane == 0) {
      for (int i = max(0, issued - kPipeStages); i < issued; ++i) {
        const unsigned long long w0 = global_ns();
        while (!mbar_try_wait(smem_u32(&full[i % kPipeStages]), (i / kPipeStages) & 1)) {
          if (global_ns() - w0 > kWaitTimeoutNs) {
            if (p.err) atomicOr(p.err, kErrWaitTimeout);
            break;
          }
        }
      }
    }
    return;
  }
  // -------------------------------------------------------------------- consumers
  const int sub = lane & 15;
  const int base_lane = lane & 16;
  const unsigned half_mask = 0xFFFFu << base_lane;
  const int hw = threadIdx.x >> 4;  // half-warp, 0..15
  const int half = p.rotary >> 1;
  uint64_t wq[4], wk[4];  // this lane's norm weights as fp32 pairs
  {
    float fq[8], fk[8];
    unpack8(reinterpret_cast<const uint4*>(p.q_weight)[sub], fq);
    unpack8(reinterpret_cast<const uint4*>(p.k_weight)[sub], fk);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      wq[i] = f2_pack(fq[2 * i], fq[2 * i + 1]);
      wk[i] = f2_pack(fk[2 * i], fk[2 * i + 1]);
    }
  }
  if constexpr (kMode == kRouteAmax || kMode == kRoutePeersFp8) {
    // per-(plane, head) words for this CTA: zeroed maxima (pass 1), or the group's scales and
    // their reciprocals (pass 2: scale = max(amax / 448, 1e-12) as the e4m3 quantisers set it)
    const int nw = 3 * heads;
    for (int k = threadIdx.x; k < nw; k += kPipeConsumerWarps * 32) {
      if constexpr (kMode == kRouteAmax) {
        aux[k] = 0u;
      } else {
        unsigned a = 0u;
        for (int g = 0; g < p.amax_sets; ++g) a = max(a, __ldcg(p.amax + g * nw + k));
        const float sc = fmaxf(__fdiv_rn(__uint_as_float(a), kFp8Max), 1.0e-12f);
        aux[k] = __float_as_uint(sc);
        aux[nw + k] = __float_as_uint(__frcp_rn(sc));
        const int j = k / heads, h = k - j * heads;
        const int w = (h * p.hl_recip) >> 16;
        if (blockIdx.x == 0 && w == p.rank && p.scale_out[j])
          p.scale_out[j][h - w * p.heads_local] = sc;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kPipeConsumerWarps * 32) : "memory");
  }
  const int d0 = 8 * sub;
  const bool rotating = d0 < p.rotary;
  const bool low = d0 < half;
  const int partner = base_lane + (low ? sub + (half >> 3) : sub - (half >> 3));
  const int phase = rotating ? (low ? d0 : d0 - half) : 0;
  for (int i = 0; i < n; ++i) {
    const int s = i % kPipeStages;
    if (!mbar_wait(smem_u32(&full[s]), (i / kPipeStages) & 1, abort_flag, p.err)) break;
    const int t = t0 + i;
    const bool pv = pos_ok[s] != 0;
    if (!pv && threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadIndex);
    uint32_t c[4] = {0u, 0u, 0u, 0u}, sn[4] = {0u, 0u, 0u, 0u};
    if (pv && rotating) {
      const uint8_t* cs = cs_rows + s * L.cs_bytes;
      const uint4 cr = *reinterpret_cast<const uint4*>(cs + 2 * phase);
      const uint4 sr = *reinterpret_cast<const uint4*>(cs + 2 * (half + phase));
      c[0] = cr.x; c[1] = cr.y; c[2] = cr.z; c[3] = cr.w;
      sn[0] = sr.x; sn[1] = sr.y; sn[2] = sr.z; sn[3] = sr.w;
    }
    const uint4* rows = reinterpret_cast<const uint4*>(slots + s * L.slot_bytes);
    const bool counted = !p.amax_rows || __ldg(p.amax_rows + t) != 0;
    for (int r = hw; r < rows_pt; r += 16) {
      const int j = (r >= heads) + (r >= 2 * heads);
      const int h = r - j * heads;
      uint4 o = rows[r * 16 + sub];
      if (j < 2) {
        if (!pv) continue;
        o = norm_rope_row(o, j == 0 ? wq : wk, p.eps, rotating, low, partner, half_mask, c, sn);
      }
      if constexpr (kMode == kRouteAmax) {
        if (!counted) continue;
        float f[8];
        unpack8(o, f);
        float m = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(f[e]));
#pragma unroll
        for (int x = 8; x > 0; x >>= 1) m = fmaxf(m, __shfl_xor_sync(half_mask, m, x));
        if (sub == 0) atomicMax(aux + j * heads + h, __float_as_uint(m));
        continue;
      } else if constexpr (kMode == kRoutePeersFp8) {
        const int k = j * heads + h;
        const float sc = __uint_as_float(aux[k]);
        const float inv = __uint_as_float(aux[3 * heads + k]);
        float f[8];
        unpack8(o, f);
        const uint2 q8 = make_uint2(quant4(f[0], f[1], f[2], f[3], sc, inv),
                                    quant4(f[4], f[5], f[6], f[7], sc, inv));
        uint8_t* d8 = dst8_row(p, t, j, h);
        if (d8) reinterpret_cast<uint2*>(d8)[sub] = q8;
        else if (sub == 0 && p.err) atomicOr(p.err, kErrBadPage);
        // bf16 rows too where the caller keeps them (Q plane; K/V pools), optionally only the
        // rows the e4m3 scales leave out
        if ((j == 0 ? !p.peer_q : !p.peer_k) || (p.bf16_unflagged_only && counted)) continue;
        __nv_bfloat16* dst = dst_row<kRoutePeers>(p, t, j, h);
        if (dst) reinterpret_cast<uint4*>(dst)[sub] = o;
        else if (sub == 0 && p.err) atomicOr(p.err, kErrBadPage);
      } else {
        __nv_bfloat16* dst = dst_row<kMode>(p, t, j, h);
        if (dst) reinterpret_cast<uint4*>(dst)[sub] = o;
        else if (sub == 0 && p.err) atomicOr(p.err, kErrBadPage);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty[s]));
  }
  if constexpr (kMode == kRouteAmax) {
    // this CTA's maxima into the launch's words (non-negative floats order like their bits)
    asm volatile("bar.sync 1, %0;" ::"n"(kPipeConsumerWarps * 32) : "memory");
    for (int k = threadIdx.x; k < 3 * heads; k += kPipeConsumerWarps * 32)
      if (aux[k]) atomicMax(p.amax + k, aux[k]);
  }
  // stores to other GPUs: visible to them before the kernel is seen as done
  if ((kMode == kRoutePeers || kMode == kRoutePeersFp8) && p.world > 1) __threadfence_system();
}

// CTA t copies `count` words into slot `rank` of rank t's [world][count] slot array (peer
// stores), then makes them visible beyond this GPU before the kernel completes.
__global__ void __launch_bounds__(256) publish_words_kernel(const uint32_t* words,
                                                            const uint64_t* peer_slots, int rank,
                                                            int count) {
  uint32_t* dst = reinterpret_cast<uint32_t*>(static_cast<uintptr_t>(__ldg(peer_slots + blockIdx.x))) +
                  static_cast<size_t>(rank) * count;
  for (int i = threadIdx.x; i < count; i += blockDim.x) dst[i] = __ldcg(words + i);
  __threadfence_system();
}

static int prologue_launch(const PrologueParams& p, cudaStream_t stream) {
  const int rows_pt = (p.mode == kRouteInPlace ? 2 : 3) * p.heads;
  const PipeSmemLayout L = pipe_layout(rows_pt, p.rotary, pipe_aux_words(p.mode, p.heads));
  if (L.total > 227 * 1024)
    return set_error(H3SA_ERR_UNSUPPORTED, "qkv prologue: %d heads need %d bytes of staging",
                     p.heads, L.total);
  auto kernel = p.mode == kRouteInPlace ? qkv_norm_rope_pipe_kernel<kRouteInPlace>
               : p.mode == kRoutePack   ? qkv_norm_rope_pipe_kernel<kRoutePack>
               : p.mode == kRoutePeers  ? qkv_norm_rope_pipe_kernel<kRoutePeers>
               : p.mode == kRouteAmax   ? qkv_norm_rope_pipe_kernel<kRouteAmax>
                                        : qkv_norm_rope_pipe_kernel<kRoutePeersFp8>;
  if (L.total > 48 * 1024) {  // the opt-in applies to the current device
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L.total);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(prologue smem)", e);
  }
  PrologueParams q = p;
  q.heads_local = p.heads / (p.world > 0 ? p.world : 1);
  q.hl_recip = (65536 + q.heads_local - 1) / q.heads_local;
  // as many CTAs per SM as the staging fits (three at 24 heads), one token range each
  const int per_sm = (3 * (L.total + 1024) <= 228 * 1024) ? 3 : (2 * (L.total + 1024) <= 228 * 1024) ? 2 : 1;
  int ctas = 148 * per_sm;
  if (ctas > p.tokens) ctas = p.tokens;
  if (ctas < 1) ctas = 1;
  const int per = (p.tokens + ctas - 1) / ctas;
  ctas = (p.tokens + per - 1) / per;
  kernel<<<ctas, kPipeThreads, L.total, stream>>>(q, per);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("qkv_norm_rope_pipe_kernel launch", e);
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
  if (heads > 255)  // the staging ring holds whole tokens; far above the model's 56 heads
    return set_error(H3SA_ERR_UNSUPPORTED, "qkv prologue: at most 255 heads, got %d", heads);
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


int h3sa_qkv_norm_rope_amax(const void* qkv, const void* q_weight, const void* k_weight,
                            const void* cos_sin, int32_t cache_rows, int32_t rotary,
                            const int64_t* positions, int32_t tokens, int32_t heads,
                            int32_t head_dim, const uint8_t* amax_rows, uint32_t* amax, float eps,
                            int32_t* device_error, void* stream) {
  int rc = check_prologue(qkv, q_weight, k_weight, cos_sin, cache_rows, rotary, positions, tokens,
                          heads, head_dim);
  if (rc) return rc;
  if (!amax) return set_error(H3SA_ERR_INVALID, "qkv prologue amax: null amax words");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(uint32_t) * 3 * heads, st);
  if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(prologue amax)", e);
  if (tokens == 0) return H3SA_OK;
  PrologueParams p{};
  p.src = static_cast<const __nv_bfloat16*>(qkv);
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
  p.mode = kRouteAmax;
  p.amax = amax;
  p.amax_rows = amax_rows;
  return prologue_launch(p, st);
}

int h3sa_publish_words(const uint32_t* words, const uint64_t* peer_slots, int32_t world,
                       int32_t rank, int32_t count, void* stream) {
  if (!words || !peer_slots || world < 1 || rank < 0 || rank >= world || count < 0)
    return set_error(H3SA_ERR_INVALID, "publish_words: invalid arguments");
  if (count == 0) return H3SA_OK;
  publish_words_kernel<<<world, 256, 0, static_cast<cudaStream_t>(stream)>>>(words, peer_slots,
                                                                             rank, count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("publish_words launch", e);
  return H3SA_OK;
}

int h3sa_qkv_norm_rope_scatter_fp8(
    const void* qkv, const void* q_weight, const void* k_weight, const void* cos_sin,
    int32_t cache_rows, int32_t rotary, const int64_t* positions, int32_t tokens, int32_t heads,
    int32_t head_dim, int32_t world, int32_t rank, const uint32_t* amax, int32_t amax_sets,
    const uint8_t* amax_rows, int32_t bf16_unflagged_only, const uint64_t* peer_q8,
    const uint64_t* peer_key_pool8, const uint64_t* peer_value_pool8, int32_t pool8_pages,
    const int32_t* page_table8, int32_t table8_blocks, int32_t dst8_start, float* q_scale,
    float* k_scale, float* v_scale, const uint64_t* peer_q, const uint64_t* peer_key_pool,
    const uint64_t* peer_value_pool, int32_t pool_pages, const int32_t* page_table,
    int32_t table_blocks, int32_t dst_start, float eps, int32_t* device_error, void* stream) {
  int rc = check_prologue(qkv, q_weight, k_weight, cos_sin, cache_rows, rotary, positions, tokens,
                          heads, head_dim);
  if (rc) return rc;
  if (world <= 0 || heads % world)
    return set_error(H3SA_ERR_INVALID, "merged QKV heads are not divisible by Ulysses");
  if (amax_sets < 1 || amax_sets > world)
    return set_error(H3SA_ERR_INVALID, "qkv prologue e4m3 scatter: %d amax sets for %d ranks",
                     amax_sets, world);
  if (bf16_unflagged_only && !amax_rows)
    return set_error(H3SA_ERR_INVALID, "qkv prologue e4m3 scatter: unflagged bf16 rows need flags");
  if (rank < 0 || rank >= world || !amax || !peer_q8 || !peer_key_pool8 || !peer_value_pool8 ||
      !page_table8 || pool8_pages <= 0 || table8_blocks <= 0 || dst8_start < 0)
    return set_error(H3SA_ERR_INVALID, "qkv prologue e4m3 scatter: invalid peer or page arguments");
  const long long end = static_cast<long long>(world) * tokens;
  if (dst8_start + end > static_cast<long long>(table8_blocks) * kBlockN)
    return set_error(H3SA_ERR_INVALID, "qkv prologue e4m3 scatter: rows [%d, %lld) exceed the "
                     "e4m3 page table's %d blocks", dst8_start, dst8_start + end, table8_blocks);
  const bool keep_bf16 = peer_key_pool != nullptr;
  if (keep_bf16 && (!peer_value_pool || !page_table || pool_pages <= 0 || table_blocks <= 0 ||
                    dst_start < 0 || dst_start + end > static_cast<long long>(table_blocks) * kBlockN))
    return set_error(H3SA_ERR_INVALID, "qkv prologue e4m3 scatter: invalid bf16 pool arguments");
  if (tokens == 0) return H3SA_OK;
  PrologueParams p{};
  p.src = static_cast<const __nv_bfloat16*>(qkv);
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
  p.mode = kRoutePeersFp8;
  p.rank = rank;
  p.amax = const_cast<uint32_t*>(amax);
  p.amax_sets = amax_sets;
  p.amax_rows = amax_rows;
  p.bf16_unflagged_only = bf16_unflagged_only ? 1 : 0;
  p.peer_q8 = peer_q8;
  p.peer_k8 = peer_key_pool8;
  p.peer_v8 = peer_value_pool8;
  p.table8 = page_table8;
  p.table8_blocks = table8_blocks;
  p.pool8_pages = pool8_pages;
  p.dst8_start = dst8_start;
  p.scale_out[0] = q_scale;
  p.scale_out[1] = k_scale;
  p.scale_out[2] = v_scale;
  p.peer_q = peer_q;
  p.peer_k = keep_bf16 ? peer_key_pool : nullptr;
  p.peer_v = keep_bf16 ? peer_value_pool : nullptr;
  p.page_table = page_table;
  p.table_blocks = table_blocks;
  p.pool_pages = pool_pages;
  p.dst_start = dst_start;
  return prologue_launch(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
