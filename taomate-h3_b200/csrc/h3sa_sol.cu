// Rectangular SOL-Attn routing for sm_100a (F/inference/sol_attention.py:366-598).
//
// Queries [Nq, H, 128] attend to one packed K/V sequence [Nk, H, 128] cut into 64-row blocks.
// The first ceil(sink / 64) blocks (the sink) and the blocks a query block routes to are
// exact; every other block enters each query row's softmax once, through its centroid: score
// q . k_c, weight = the block's row count, value = the block's V sum. Four launches:
//   1. sol_summaries_kernel   key centroids (mean of the block's K rows) and value sums, bf16
//   2. sol_key_stats_kernel   per head the centroids' mean and population variance (fp32)
//   3. sol_route_kernel       per (64-row query block, head) the threshold
//                             mu + tau * sqrt(var + 1e-6) of the proxy score under a diagonal
//                             covariance, and the exact-block bitmask: sink, or mean proxy
//                             score over the block's query rows above the threshold
//   4. sol_attention_kernel   tcgen05 attention: one CTA per 128 query rows (two query blocks)
//                             and head, walking the approximate centroid chunks (64 centroids
//                             per MMA tile, each half of the rows with its own mask) and the
//                             union of the two query blocks' exact blocks (64 key rows per
//                             tile, masked per half), with one online softmax per row.
// The first three are HBM/L2 work of a few microseconds; the fourth holds the FLOPs.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cmath>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {
namespace {

constexpr int kSolRows = 64;                  // rows of a SOL key / query block
constexpr int kSolMaxKeyBlocks = 4096;        // 262144 key rows
constexpr int kSolMaxChunks = kSolMaxKeyBlocks / 64;
constexpr int kSolMaxItems = kSolMaxKeyBlocks + kSolMaxChunks;
constexpr int kSolStages = 2;                 // K and V rings (two CTAs share an SM)
constexpr int kSolThreads = 256;
constexpr int kSolRouteQBlocks = 8;           // query blocks per routing CTA
constexpr float kSolRescale = 8.0f;           // lazy O rescale threshold (log2 units)
constexpr uint16_t kItemApprox = 0x8000u;

struct SolParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int nq, nk, heads;
  int qb, kb, words;  // query blocks, key blocks, 32-bit mask words per (head, query block)
  float sl2;          // softmax scale * log2(e)
  float tau;
  int sink_blocks;
  __nv_bfloat16* kc;  // [kb, heads, 128] key centroids
  __nv_bfloat16* vs;  // [kb, heads, 128] value sums
  float* stats;       // [heads, 2, 128]: centroid mean, centroid variance
  uint32_t* exact;    // [heads, qb, words]
  unsigned long long* tele;  // [4] selected, exact, routable, candidate (nullable)
  __nv_bfloat16* out;
  int* err;
};

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4 w) {
  acc[0] += __uint_as_float(w.x << 16);
  acc[1] += __uint_as_float(w.x & 0xFFFF0000u);
  acc[2] += __uint_as_float(w.y << 16);
  acc[3] += __uint_as_float(w.y & 0xFFFF0000u);
  acc[4] += __uint_as_float(w.z << 16);
  acc[5] += __uint_as_float(w.z & 0xFFFF0000u);
  acc[6] += __uint_as_float(w.w << 16);
  acc[7] += __uint_as_float(w.w & 0xFFFF0000u);
}

// grid ceil(kb * heads / 8), 128 threads: 16 threads per (key block, head), each summing 8 dims
// (one 16-byte load per row) over the block's rows in row order.
__global__ void __launch_bounds__(128) sol_summaries_kernel(const SolParams p) {
  const int pair = blockIdx.x * 8 + (threadIdx.x >> 4);
  if (pair >= p.kb * p.heads) return;
  const int b = pair / p.heads, h = pair - b * p.heads, c = threadIdx.x & 15;
  const int r0 = b * kSolRows;
  const int n = min(kSolRows, p.nk - r0);
  const size_t stride = static_cast<size_t>(p.heads) * kHeadDim / 8;  // in uint4
  const size_t base = ((static_cast<size_t>(r0) * p.heads + h) * kHeadDim) / 8 + c;
  const uint4* k = reinterpret_cast<const uint4*>(p.k) + base;
  const uint4* v = reinterpret_cast<const uint4*>(p.v) + base;
  float sk[8] = {}, sv[8] = {};
#pragma unroll 8
  for (int r = 0; r < n; ++r) {
    add_bf16x8(sk, __ldg(k + r * stride));
    add_bf16x8(sv, __ldg(v + r * stride));
  }
  const float fn = static_cast<float>(n);
  const size_t o = ((static_cast<size_t>(b) * p.heads + h) * kHeadDim) / 8 + c;
  reinterpret_cast<uint4*>(p.kc)[o] =
      make_uint4(pack_bf16x2(sk[0] / fn, sk[1] / fn), pack_bf16x2(sk[2] / fn, sk[3] / fn),
                 pack_bf16x2(sk[4] / fn, sk[5] / fn), pack_bf16x2(sk[6] / fn, sk[7] / fn));
  reinterpret_cast<uint4*>(p.vs)[o] =
      make_uint4(pack_bf16x2(sv[0], sv[1]), pack_bf16x2(sv[2], sv[3]), pack_bf16x2(sv[4], sv[5]),
                 pack_bf16x2(sv[6], sv[7]));
}

// grid heads, 512 threads: dim d = t % 128, block group g = t / 128 takes blocks g, g + 4, ...;
// the four groups' partial sums are added in group order, first for the mean, then for the
// mean squared deviation.
__global__ void __launch_bounds__(512) sol_key_stats_kernel(const SolParams p) {
  __shared__ float part[4][kHeadDim];
  const int h = blockIdx.x, d = threadIdx.x & (kHeadDim - 1), g = threadIdx.x >> 7;
  const size_t stride = static_cast<size_t>(p.heads) * kHeadDim;
  const __nv_bfloat16* c = p.kc + static_cast<size_t>(h) * kHeadDim + d;
  float s = 0.f;
#pragma unroll 8
  for (int b = g; b < p.kb; b += 4) s += __bfloat162float(c[b * stride]);
  part[g][d] = s;
  __syncthreads();
  const float mean = ((part[0][d] + part[1][d]) + (part[2][d] + part[3][d])) /
                     static_cast<float>(p.kb);
  __syncthreads();
  float s2 = 0.f;
#pragma unroll 8
  for (int b = g; b < p.kb; b += 4) {
    const float x = __bfloat162float(c[b * stride]) - mean;
    s2 += x * x;
  }
  part[g][d] = s2;
  __syncthreads();
  if (g == 0) {
    p.stats[(h * 2 + 0) * kHeadDim + d] = mean;
    p.stats[(h * 2 + 1) * kHeadDim + d] =
        ((part[0][d] + part[1][d]) + (part[2][d] + part[3][d])) / static_cast<float>(p.kb);
  }
}

// grid (ceil(qb / 8), heads), 256 threads. The query blocks' column sums (fp32, row order) go
// to shared memory; warp j computes query block j's threshold from its bf16 centroid; then
// thread t scores key blocks t, t + 256, ... against all the CTA's query blocks (the mean proxy
// score over a block's rows is its column sum . k_c * scale * log2(e) / rows) and each warp
// writes one mask word per query block from a ballot.
__global__ void __launch_bounds__(kSolThreads) sol_route_kernel(const SolParams p) {
  __shared__ __align__(16) float cs[kSolRouteQBlocks][kHeadDim];
  __shared__ float thr[kSolRouteQBlocks];
  __shared__ float inv_len[kSolRouteQBlocks];
  const int h = blockIdx.y;
  const int qb0 = blockIdx.x * kSolRouteQBlocks;
  const int nqb = min(kSolRouteQBlocks, p.qb - qb0);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const size_t stride = static_cast<size_t>(p.heads) * kHeadDim;
  if (t < 16 * kSolRouteQBlocks && (t >> 4) < nqb) {
    // 16 threads per query block, 8 dims each, rows added in order
    const int j = t >> 4, c = t & 15;
    const int r0 = (qb0 + j) * kSolRows;
    const int n = min(kSolRows, p.nq - r0);
    const uint4* src = reinterpret_cast<const uint4*>(p.q) +
                       ((static_cast<size_t>(r0) * p.heads + h) * kHeadDim) / 8 + c;
    float acc[8] = {};
#pragma unroll 8
    for (int r = 0; r < n; ++r) add_bf16x8(acc, __ldg(src + r * (stride / 8)));
    float4* dst = reinterpret_cast<float4*>(&cs[j][8 * c]);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  __syncthreads();
  if (warp < nqb) {
    const int r0 = (qb0 + warp) * kSolRows;
    const float len = static_cast<float>(min(kSolRows, p.nq - r0));
    const float* mean = p.stats + (h * 2 + 0) * kHeadDim;
    const float* var = p.stats + (h * 2 + 1) * kHeadDim;
    float pm = 0.f, pv = 0.f;
    for (int d = lane; d < kHeadDim; d += 32) {
      const float qbar = __bfloat162float(__float2bfloat16_rn(cs[warp][d] / len));
      pm += qbar * __ldg(mean + d);
      pv += qbar * qbar * __ldg(var + d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pm += __shfl_xor_sync(0xffffffffu, pm, o);
      pv += __shfl_xor_sync(0xffffffffu, pv, o);
    }
    if (lane == 0) {
      thr[warp] = pm * p.sl2 + p.tau * sqrtf(fmaxf(pv * (p.sl2 * p.sl2), 0.f) + 1.0e-6f);
      inv_len[warp] = 1.0f / len;
    }
  }
  __syncthreads();
  unsigned long long n_sel = 0, n_exact = 0, n_route = 0, n_cand = 0;
  for (int base = 0; base < p.kb; base += kSolThreads) {
    const int j = base + t;
    const bool valid = j < p.kb;
    float dot[kSolRouteQBlocks];
#pragma unroll
    for (int q = 0; q < kSolRouteQBlocks; ++q) dot[q] = 0.f;
    if (valid) {
      const uint4* row = reinterpret_cast<const uint4*>(p.kc + (static_cast<size_t>(j) * p.heads + h) * kHeadDim);
#pragma unroll 2
      for (int c = 0; c < kHeadDim / 8; ++c) {
        const uint4 w = __ldg(row + c);
        float x[8] = {};
        add_bf16x8(x, w);
#pragma unroll
        for (int q = 0; q < kSolRouteQBlocks; ++q) {
          const float4 a = *reinterpret_cast<const float4*>(&cs[q][8 * c]);
          const float4 b = *reinterpret_cast<const float4*>(&cs[q][8 * c + 4]);
          dot[q] += a.x * x[0] + a.y * x[1] + a.z * x[2] + a.w * x[3] + b.x * x[4] +
                    b.y * x[5] + b.z * x[6] + b.w * x[7];
        }
      }
    }
    const bool sink = j < p.sink_blocks;
    const int word = (base >> 5) + warp;
    const unsigned routable = __ballot_sync(0xffffffffu, valid && !sink);
    const unsigned cand = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int q = 0; q < kSolRouteQBlocks; ++q) {
      if (q >= nqb) break;
      const bool sel = valid && !sink && dot[q] * p.sl2 * inv_len[q] > thr[q];
      const unsigned wsel = __ballot_sync(0xffffffffu, sel);
      const unsigned wex = __ballot_sync(0xffffffffu, sel || (valid && sink));
      if (lane == 0 && word < p.words)
        p.exact[(static_cast<size_t>(h) * p.qb + qb0 + q) * p.words + word] = wex;
      n_sel += __popc(wsel);
      n_exact += __popc(wex);
      n_route += __popc(routable);
      n_cand += __popc(cand);
    }
  }
  if (p.tele && lane == 0 && n_cand) {
    atomicAdd(p.tele + 0, n_sel);
    atomicAdd(p.tele + 1, n_exact);
    atomicAdd(p.tele + 2, n_route);
    atomicAdd(p.tele + 3, n_cand);
  }
}

// ------------------------------------------------------------------ attention
// One CTA = 128 query rows (query blocks 2t and 2t + 1: rows 0-63 and 64-127) x one head.
// Work items (16 bits each), built once in shared memory by warp 2:
//   approximate chunk c (bit 15 set): centroids / value sums of key blocks [64c, 64c + 64),
//     with one 64-bit mask per half of the rows (valid, not exact for that query block);
//   exact key block b (bits 0-11): its 64 K/V rows, bits 12 / 13 = exact for rows 0-63 / 64-127.
// Two CTAs share an SM (107 KB of shared memory and 256 TMEM columns each), so one CTA's
// softmax runs while the other's MMAs do. Warp roles: warp 0 lane 0 TMA (Q once, then per
// item the K tile into a 2-stage ring freed when its S MMA completes, and the V tile into a
// 2-stage ring freed when its P V MMA completes); warp 1 MMA issue (S = Q K^T, M = 128, N = 64, into one of two TMEM S buffers;
// O += P V with P read from TMEM, M = 128, N = 128, K = 64); warps 4-7 softmax, one thread per
// row (TMEM lane), and the epilogue. TMEM: S0 [0, 64), S1 [64, 128), O [128, 256); P(i) is
// stored over the first 32 columns of its S buffer.
struct alignas(1024) SolSmem {
  uint8_t q[2][kBlockM * 128];                  // two 64-column atoms of 128 rows
  uint8_t k[kSolStages][2][kSolRows * 128];     // two atoms of 64 rows
  uint8_t v[kSolStages][2][kSolRows * 128];
  uint16_t items[kSolMaxItems];
  unsigned long long amask[2][kSolMaxChunks];
  uint64_t q_full;
  uint64_t k_full[kSolStages], v_full[kSolStages], k_empty[kSolStages], v_empty[kSolStages];
  uint64_t s_full[2], p_full[2], pv_done, o_done, drain;
  uint32_t tmem_base;
  int abort_flag;
  int n_items;
};
constexpr size_t kSolSmemBytes = sizeof(SolSmem) + 1024;
static_assert(2 * (kSolSmemBytes + 1024) <= 233472, "two SOL attention CTAs exceed an SM's shared memory");

constexpr uint32_t kSolIdescQK = idesc_bf16(kBlockM, kSolRows, false);
constexpr uint32_t kSolIdescPV = idesc_bf16(kBlockM, kHeadDim, true);

// Warp 2: the item list. Lanes take 32 mask words (or chunks) at a time; a warp prefix sum
// places each lane's items, so items stay in ascending order.
__device__ void sol_build_items(const SolParams& p, int head, int tile, SolSmem& sm) {
  const int lane = threadIdx.x & 31;
  const int qa = 2 * tile, qbb = 2 * tile + 1;
  const uint32_t* ex0 = p.exact + (static_cast<size_t>(head) * p.qb + qa) * p.words;
  const uint32_t* ex1 = qbb < p.qb ? p.exact + (static_cast<size_t>(head) * p.qb + qbb) * p.words
                                   : nullptr;
  auto word = [&](const uint32_t* e, int w) -> uint32_t {
    return (e && w < p.words) ? __ldg(e + w) : 0u;
  };
  const int chunks = (p.kb + 63) / 64;
  int n = 0;
  for (int c0 = 0; c0 < chunks; c0 += 32) {
    const int c = c0 + lane;
    bool need = false;
    if (c < chunks) {
      const int nv = min(64, p.kb - 64 * c);
      const unsigned long long valid = nv >= 64 ? ~0ull : ((1ull << nv) - 1ull);
      const unsigned long long e0 =
          word(ex0, 2 * c) | (static_cast<unsigned long long>(word(ex0, 2 * c + 1)) << 32);
      const unsigned long long e1 =
          word(ex1, 2 * c) | (static_cast<unsigned long long>(word(ex1, 2 * c + 1)) << 32);
      const unsigned long long a0 = valid & ~e0;
      const unsigned long long a1 = ex1 ? (valid & ~e1) : 0ull;
      sm.amask[0][c] = a0;
      sm.amask[1][c] = a1;
      need = (a0 | a1) != 0ull;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, need);
    if (need)
      sm.items[n + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(kItemApprox | c);
    n += __popc(bal);
  }
  for (int w0 = 0; w0 < p.words; w0 += 32) {
    const int w = w0 + lane;
    const uint32_t u0 = word(ex0, w), u1 = word(ex1, w);
    uint32_t u = u0 | u1;
    const int cnt = __popc(u);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int at = n + incl - cnt;
    while (u) {
      const int bit = __ffs(u) - 1;
      u &= u - 1;
      const int b = 32 * w + bit;
      sm.items[at++] = static_cast<uint16_t>(b | (((u0 >> bit) & 1u) << 12) |
                                             (((u1 >> bit) & 1u) << 13));
    }
    n += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) sm.n_items = n;
}

__global__ void __launch_bounds__(kSolThreads, 2)
    sol_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV,
                         const __grid_constant__ CUtensorMap tmKC,
                         const __grid_constant__ CUtensorMap tmVS, const SolParams p) {
  extern __shared__ uint8_t smem_raw[];
  SolSmem& sm = *reinterpret_cast<SolSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const int tiles = (p.nq + kBlockM - 1) / kBlockM;
  const int head = static_cast<int>(blockIdx.x) / tiles;
  const int tile = static_cast<int>(blockIdx.x) - head * tiles;
  const int q_row0 = tile * kBlockM;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sm.q_full), 1);
    for (int s = 0; s < kSolStages; ++s) {
      mbar_init(smem_u32(&sm.k_full[s]), 1);
      mbar_init(smem_u32(&sm.v_full[s]), 1);
      mbar_init(smem_u32(&sm.k_empty[s]), 1);
      mbar_init(smem_u32(&sm.v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&sm.s_full[s]), 1);
      mbar_init(smem_u32(&sm.p_full[s]), 128);
    }
    mbar_init(smem_u32(&sm.pv_done), 1);
    mbar_init(smem_u32(&sm.o_done), 1);
    mbar_init(smem_u32(&sm.drain), 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) sol_build_items(p, head, tile, sm);
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  const int n_items = sm.n_items;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint32_t qbar = smem_u32(&sm.q_full);
      mbar_expect_tx(qbar, 2 * kBlockM * 128);
      for (int a = 0; a < 2; ++a)
        tma_load_3d(smem_u32(sm.q[a]), &tmQ, qbar, 64 * a, head, q_row0);
      // K tiles run ahead of V tiles: K(i) needs only S(i - 2) done, V(i) needs PV(i - 2)
      int iv = 0;
      auto load_v = [&](int j) -> bool {
        const int s = j % kSolStages;
        if (!mbar_wait(smem_u32(&sm.v_empty[s]), ((j / kSolStages) & 1) ^ 1, abort_flag, p.err))
          return false;
        const uint16_t it = sm.items[j];
        const bool approx = (it & kItemApprox) != 0;
        const int row = 64 * (it & 0xFFF);
        const uint32_t vb = smem_u32(&sm.v_full[s]);
        mbar_expect_tx(vb, 2 * kSolRows * 128);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(smem_u32(sm.v[s][a]), approx ? &tmVS : &tmV, vb, 64 * a, head, row);
        return true;
      };
      bool ok = true;
      for (int i = 0; ok && i < n_items; ++i) {
        const int s = i % kSolStages;
        if (!mbar_wait(smem_u32(&sm.k_empty[s]), ((i / kSolStages) & 1) ^ 1, abort_flag, p.err))
          break;
        const uint16_t it = sm.items[i];
        const bool approx = (it & kItemApprox) != 0;
        const int row = 64 * (it & 0xFFF);  // centroid row or key row
        const uint32_t kb = smem_u32(&sm.k_full[s]);
        mbar_expect_tx(kb, 2 * kSolRows * 128);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(smem_u32(sm.k[s][a]), approx ? &tmKC : &tmK, kb, 64 * a, head, row);
        // the V tile of the item two behind (its ring slot frees later than a K slot)
        while (ok && iv + 1 < i) ok = load_v(iv++);
      }
      while (ok && iv < n_items) ok = load_v(iv++);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    const uint32_t tO = tbase + 128u;
    const uint32_t qlo = sdesc_lo(smem_u32(sm.q[0]), 16);
    bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sm.q_full), 0, abort_flag, p.err));
    tc_fence_after();
    auto issue_qk = [&](int i) -> bool {
      const int s = i % kSolStages;
      const bool w = mbar_wait(smem_u32(&sm.k_full[s]), (i / kSolStages) & 1, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      const uint32_t tS = tbase + static_cast<uint32_t>(i & 1) * 64u;
      const uint32_t klo = sdesc_lo(smem_u32(sm.k[s][0]), 16);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t qoff = (((kk >> 2) * kBlockM * 128) + (kk & 3) * 32) >> 4;
        const uint32_t koff = (((kk >> 2) * kSolRows * 128) + (kk & 3) * 32) >> 4;
        mma_ss(tS, sdesc_join(qlo + qoff), sdesc_join(klo + koff), kSolIdescQK, kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(&sm.s_full[i & 1]));
      tc_commit(smem_u32(&sm.k_empty[s]));
      return true;
    };
    if (ok && n_items > 0) ok = issue_qk(0);
    if (ok && n_items > 1) ok = issue_qk(1);
    for (int i = 0; ok && i < n_items; ++i) {
      const int s = i % kSolStages;
      bool w = mbar_wait(smem_u32(&sm.v_full[s]), (i / kSolStages) & 1, abort_flag, p.err);
      if (w) w = mbar_wait(smem_u32(&sm.p_full[i & 1]), (i >> 1) & 1, abort_flag, p.err);
      if (!(ok = __all_sync(0xffffffffu, w))) break;
      tc_fence_after();
      const uint32_t tP = tbase + static_cast<uint32_t>(i & 1) * 64u;
      const uint32_t vlo = sdesc_lo(smem_u32(sm.v[s][0]), kSolRows * 128);
#pragma unroll
      for (int kk = 0; kk < kSolRows / 16; ++kk)
        mma_ts(tO, tP + kk * 8u, sdesc_join(vlo + ((kk * 16 * 128) >> 4)), kSolIdescPV,
               (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(smem_u32(&sm.pv_done));
      tc_commit(smem_u32(&sm.v_empty[s]));
      if (i + 2 < n_items) ok = issue_qk(i + 2);
    }
    if (ok) tc_commit(smem_u32(&sm.o_done));
    tc_commit(smem_u32(&sm.drain));
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(smem_u32(&sm.drain), 0)) {
      if (global_ns() - t0 > kWaitTimeoutNs) {
        if (p.err && lane == 0) atomicOr(p.err, kErrWaitTimeout);
        break;
      }
    }
  } else if (warp >= 4) {
    // ================================================================ softmax / epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int half = row >> 6;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tbase + 128u + lane_off;
    const int last_len = p.nk - 64 * (p.kb - 1);  // rows of the last key block
    float m_used = -INFINITY;
    float l_sum = 0.f;
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
      const uint32_t it = sm.items[i];
      const bool approx = (it & kItemApprox) != 0u;
      const int idx = static_cast<int>(it & 0xFFFu);
      unsigned long long vm;
      int jl = -1;  // approximate chunk: the column of the last (partial) key block
      if (approx) {
        vm = sm.amask[half][idx];
        jl = (p.kb - 1) - 64 * idx;
        if (jl >= 64 || last_len == 64) jl = -1;
      } else {
        const int nv = min(64, p.nk - 64 * idx);
        vm = ((it >> (12 + half)) & 1u) ? (nv >= 64 ? ~0ull : ((1ull << nv) - 1ull)) : 0ull;
      }
      if (!(ok = mbar_wait(smem_u32(&sm.s_full[i & 1]), (i >> 1) & 1, abort_flag, p.err))) break;
      tc_fence_after();
      // a warp's 32 rows lie in one half, so `vm` is warp-uniform: a warp whose query block
      // takes nothing from this item only writes zero P
      const bool live = vm != 0ull;
      bool need = false;
      float alpha = 1.0f;
      uint32_t pk[32];
      if (live) {
        const uint32_t tS = tbase + static_cast<uint32_t>(i & 1) * 64u + lane_off;
        uint32_t r[64];
        tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(r));
        tmem_ld32(tS + 32u, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        tmem_wait_ld();
        reg_fence32(*reinterpret_cast<uint32_t(*)[32]>(r));
        reg_fence32(*reinterpret_cast<uint32_t(*)[32]>(r + 32));
        if (vm != ~0ull) {
          const uint32_t vlo = static_cast<uint32_t>(vm), vhi = static_cast<uint32_t>(vm >> 32);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (!((vlo >> j) & 1u)) r[j] = 0xFF800000u;  // -inf
            if (!((vhi >> j) & 1u)) r[32 + j] = 0xFF800000u;
          }
        }
        float m0 = __uint_as_float(r[0]), m1 = __uint_as_float(r[1]);
#pragma unroll
        for (int j = 2; j < 64; j += 4) {
          m0 = fmax3(m0, __uint_as_float(r[j]), __uint_as_float(r[j + 2]));
          m1 = fmax3(m1, __uint_as_float(r[j + 1]), __uint_as_float(r[j + 3]));
        }
        const float mx = fmaxf(m0, m1) * p.sl2;  // the scale is positive
        need = mx > m_used + kSolRescale || (m_used == -INFINITY && mx > -INFINITY);
        const float m_new = need ? mx : m_used;
        alpha = (need && m_used > -INFINITY) ? fast_exp2(m_used - m_new) : 1.0f;
        l_sum *= alpha;
        m_used = m_new;
        const float bias = m_used == -INFINITY ? 0.f : -m_used;
        const uint64_t sl2x2 = f2_pack(p.sl2, p.sl2), bias2 = f2_pack(bias, bias);
        uint64_t sum2 = f2_pack(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), sl2x2, bias2),
                    x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          sum2 = f2_add(sum2, f2_pack(p0, p1));
          pk[j / 2] = pack_bf16x2(p0, p1);
        }
        float sa, sb;
        f2_unpack(sum2, sa, sb);
        float sum = sa + sb;
        if (approx) {  // every block's weight is its row count; only the last may be short
          sum *= 64.0f;
          if (jl >= 0) {
            float rj = -INFINITY;
#pragma unroll
            for (int j = 0; j < 64; ++j)
              if (j == jl) rj = __uint_as_float(r[j]);
            sum += fast_exp2(fmaf(rj, p.sl2, bias)) * static_cast<float>(last_len - 64);
          }
        }
        l_sum += sum;
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) pk[j] = 0u;
      }
      const bool any_need = i > 0 && __any_sync(0xffffffffu, need && alpha != 1.0f);
      if (any_need) {
        // PV(i - 1) has finished (S(i) completed after it); rescale this row's O
        if (!(ok = mbar_wait(smem_u32(&sm.pv_done), (i - 1) & 1, abort_flag, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t o[32];
          tmem_ld32(tO + ch * 32, o);
          tmem_wait_ld();
          reg_fence32(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(tO + ch * 32, o);
        }
      }
      tmem_st32(tbase + static_cast<uint32_t>(i & 1) * 64u + lane_off, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&sm.p_full[i & 1]));
    }
    if (ok) ok = mbar_wait(smem_u32(&sm.o_done), 0, abort_flag, p.err);
    if (ok) {
      tc_fence_after();
      const int qrow = q_row0 + row;
      const float inv = (n_items > 0 && l_sum > 0.f) ? 1.0f / l_sum : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(qrow) * p.heads + head) * kHeadDim);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t o[32];
        tmem_ld32(tO + ch * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (qrow < p.nq) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[j]) * inv, __uint_as_float(o[j + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[j + 2]) * inv, __uint_as_float(o[j + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[j + 4]) * inv, __uint_as_float(o[j + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[j + 6]) * inv, __uint_as_float(o[j + 7]) * inv);
            dst[ch * 4 + j / 8] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

}  // namespace

}  // namespace h3sa

using namespace h3sa;

extern "C" int h3sa_sol_attention(const void* query, int32_t query_tokens, const void* key,
                                  const void* value, int32_t key_tokens, int32_t heads,
                                  int32_t head_dim, float softmax_scale, float tau,
                                  int32_t sink_tokens, void* key_centroids, void* value_sums,
                                  float* key_stats, uint32_t* exact_blocks, int64_t* telemetry,
                                  void* out, int32_t* device_error, void* stream) {
  if (head_dim != kHeadDim)
    return set_error(H3SA_ERR_UNSUPPORTED, "sol attention requires head_dim 128, got %d", head_dim);
  if (query_tokens <= 0 || key_tokens <= 0 || heads <= 0 || heads > 65535 || sink_tokens < 0)
    return set_error(H3SA_ERR_INVALID, "sol attention: invalid sizes queries=%d keys=%d heads=%d "
                     "sink=%d", query_tokens, key_tokens, heads, sink_tokens);
  const int kb = (key_tokens + kSolRows - 1) / kSolRows;
  if (kb > kSolMaxKeyBlocks)
    return set_error(H3SA_ERR_UNSUPPORTED, "sol attention: %d key rows exceed %d", key_tokens,
                     kSolMaxKeyBlocks * kSolRows);
  if (!(softmax_scale > 0.f) || !std::isfinite(tau))
    return set_error(H3SA_ERR_INVALID, "sol attention: scale must be positive, tau finite");
  const void* ptrs[] = {query, key, value, key_centroids, value_sums, key_stats, exact_blocks, out};
  for (const void* q : ptrs) {
    if (!q) return set_error(H3SA_ERR_INVALID, "sol attention: null pointer argument");
    if (reinterpret_cast<uintptr_t>(q) & 15u)
      return set_error(H3SA_ERR_INVALID, "sol attention: tensors must be 16-byte aligned");
  }
  SolParams p{};
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.k = static_cast<const __nv_bfloat16*>(key);
  p.v = static_cast<const __nv_bfloat16*>(value);
  p.nq = query_tokens;
  p.nk = key_tokens;
  p.heads = heads;
  p.qb = (query_tokens + kSolRows - 1) / kSolRows;
  p.kb = kb;
  p.words = (kb + 31) / 32;
  p.sl2 = softmax_scale * 1.4426950408889634f;
  p.tau = tau;
  p.sink_blocks = min((sink_tokens + kSolRows - 1) / kSolRows, kb);
  p.kc = static_cast<__nv_bfloat16*>(key_centroids);
  p.vs = static_cast<__nv_bfloat16*>(value_sums);
  p.stats = key_stats;
  p.exact = exact_blocks;
  p.tele = reinterpret_cast<unsigned long long*>(telemetry);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.err = device_error;

  const uint64_t row_stride[2] = {static_cast<uint64_t>(kHeadDim) * 2,
                                  static_cast<uint64_t>(heads) * kHeadDim * 2};
  CUtensorMap mq, mk, mv, mkc, mvs;
  const uint32_t qbox[3] = {64, 1, kBlockM};
  const uint32_t kbox[3] = {64, 1, kSolRows};
  const uint64_t qdims[3] = {kHeadDim, static_cast<uint64_t>(heads), static_cast<uint64_t>(query_tokens)};
  const uint64_t kdims[3] = {kHeadDim, static_cast<uint64_t>(heads), static_cast<uint64_t>(key_tokens)};
  const uint64_t cdims[3] = {kHeadDim, static_cast<uint64_t>(heads), static_cast<uint64_t>(kb)};
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = encode_tiled_3d(&mq, bf, query, qdims, row_stride, qbox);
  if (!rc) rc = encode_tiled_3d(&mk, bf, key, kdims, row_stride, kbox);
  if (!rc) rc = encode_tiled_3d(&mv, bf, value, kdims, row_stride, kbox);
  if (!rc) rc = encode_tiled_3d(&mkc, bf, key_centroids, cdims, row_stride, kbox);
  if (!rc) rc = encode_tiled_3d(&mvs, bf, value_sums, cdims, row_stride, kbox);
  if (rc) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaFuncSetAttribute(sol_attention_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kSolSmemBytes));
  if (e == cudaSuccess)  // two CTAs per SM need the largest shared-memory carveout
    e = cudaFuncSetAttribute(sol_attention_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             100);
  if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(sol attention)", e);
  sol_summaries_kernel<<<(kb * heads + 7) / 8, 128, 0, st>>>(p);
  sol_key_stats_kernel<<<heads, 512, 0, st>>>(p);
  sol_route_kernel<<<dim3((p.qb + kSolRouteQBlocks - 1) / kSolRouteQBlocks, heads), kSolThreads,
                     0, st>>>(p);
  const int tiles = (query_tokens + kBlockM - 1) / kBlockM;
  sol_attention_kernel<<<tiles * heads, kSolThreads, kSolSmemBytes, st>>>(mq, mk, mv, mkc, mvs, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("sol attention launch", e);
  return H3SA_OK;
}
