// Streaming chunk attention (dense / block-sparse, bf16 / e4m3) for sm_100a.
// Kernel layout and warp roles are described in h3sa_attention.cuh.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "h3sa_attention.cuh"
#include "h3sa_host.h"

namespace h3sa {

// e4m3 P = 2^(x - m_used + boost) stays at most 2^(threshold + boost), which must not pass the
// e4m3 maximum 448 (< 2^9); the boost lifts small P values out of the subnormal range. At the
// 1080p shape with x8 outliers, threshold/boost 2/6, 4/4 and 8/0 measured 1.68 / 1.64 / 1.60 ms
// and 0.96 / 1.29 / 1.74 % relative L2 against attention on the dequantised inputs.
#ifndef H3SA_FP8_RESCALE_THRESHOLD
#define H3SA_FP8_RESCALE_THRESHOLD 4.0f
#endif
#ifndef H3SA_FP8_BOOST
#define H3SA_FP8_BOOST 4.0f
#endif
static_assert(H3SA_FP8_RESCALE_THRESHOLD + H3SA_FP8_BOOST <= 8.5f, "e4m3 P would saturate");

// K and V ring depths. P of each query tile sits in shared memory, which leaves room for two
// K stages and one V stage of bf16 tiles within the 227 KB a CTA can have; e4m3 tiles are half
// the size and keep two V stages.
#ifndef H3SA_K_STAGES
#define H3SA_K_STAGES 2
#endif
#ifndef H3SA_V_STAGES_BF16
#define H3SA_V_STAGES_BF16 1
#endif

// Ping-pong of the exponential phases of the two query tiles of a CTA: the softmax warps of
// tile 0 and tile 1 that share an SM sub-partition take turns on its MUFU, so one computes
// exponentials while the other reads scores, takes row maxima and stores P.
#ifndef H3SA_PINGPONG
#define H3SA_PINGPONG 1
#endif

// Optional per-block timeline of two CTAs (first and middle of the grid), compiled only with
// -DH3SA_TRACE: clock64() at fixed points of the producer, MMA and softmax loops.
#ifndef H3SA_TRACE_QUARTER
#define H3SA_TRACE_QUARTER 0  // one-tile kernel: the row quarter whose softmax warps are traced
#endif
#ifdef H3SA_TRACE
constexpr int kTraceBlocks = 48;
__device__ long long g_h3sa_trace[2][kTraceBlocks][24];
#define H3SA_TRACE_AT(blk, ev)                                                              \
  do {                                                                                     \
    const int slot_ = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x / 2 ? 1 : -1);        \
    if (slot_ >= 0 && (blk) < kTraceBlocks) g_h3sa_trace[slot_][(blk)][(ev)] = clock64();  \
  } while (0)
#else
#define H3SA_TRACE_AT(blk, ev) \
  do {                         \
  } while (0)
#endif

template <bool kFp8>
struct AttnCfg {
  static constexpr int kElem = kFp8 ? 1 : 2;
  static constexpr int kTileBytes = kBlockM * kHeadDim * kElem;  // 32 KB bf16, 16 KB e4m3
  static constexpr int kAtoms = kHeadDim * kElem / 128;          // 128-byte swizzle atoms per row
  static constexpr int kAtomBytes = kBlockM * 128;               // 16 KB
  static constexpr int kKSteps = kFp8 ? 4 : 8;  // MMA K steps over d (QK^T) and over kv (PV)
  static constexpr int kKStepBytes = 32;        // bytes of an operand row per MMA K step
  static constexpr int kPvRowsPerStep = kFp8 ? 32 : 16;  // kv rows per PV MMA step
  static constexpr int kKStages = H3SA_K_STAGES;
  static constexpr int kVStages = kFp8 ? 2 : H3SA_V_STAGES_BF16;
  static constexpr uint32_t kIdescQK = kFp8 ? idesc_e4m3(kBlockM, kBlockN, false)
                                            : idesc_bf16(kBlockM, kBlockN, false);
  // PV: A = P (K-major, shared memory), B = V (rows of kv, so N = d is the contiguous dim)
  static constexpr uint32_t kIdescPV = kFp8 ? idesc_e4m3(kBlockM, kHeadDim, true)
                                            : idesc_bf16(kBlockM, kHeadDim, true);
  static_assert(kBlockN / kPvRowsPerStep == kKSteps, "P is laid out like Q");
};

constexpr int kMaskWords = kMaxUnionBlocks / 32;

template <bool kFp8>
struct alignas(1024) AttnSmem {
  using Cfg = AttnCfg<kFp8>;
  uint8_t q[2][Cfg::kTileBytes];
  uint8_t p[2][Cfg::kTileBytes];  // P of each query tile: the layout of a Q tile (K-major, SW128)
  uint8_t k[Cfg::kKStages][Cfg::kTileBytes];
  uint8_t v[Cfg::kVStages][Cfg::kTileBytes];
  uint64_t q_full;
  uint64_t k_full[Cfg::kKStages], k_empty[Cfg::kKStages];
  uint64_t v_full[Cfg::kVStages], v_empty[Cfg::kVStages];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], o_done[2];
  uint64_t exp_tok[2][4];  // [tile][sub-partition]: that warp finished a round's exponentials
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int n_blocks;
  int split_last;  // split-KV: this CTA finished its pair last and merges the segments
  uint32_t kv_mask[2][kMaskWords];  // block-sparse: bit i = tile t attends to block b_lo + i
};

template <bool kFp8>
constexpr size_t attn_smem_bytes() {
  return sizeof(AttnSmem<kFp8>) + 1024;  // + slack for 1024-byte alignment of the base
}
static_assert(attn_smem_bytes<false>() <= 232448, "bf16 attention needs more than 227 KB");
static_assert(attn_smem_bytes<true>() <= 232448, "e4m3 attention needs more than 227 KB");

// The block-sparse lists of a CTA's two query tiles as bitmaps over [b_lo, b_hi), built by one
// warp; n_out = number of blocks in their union. Indices outside the range set kErrBadIndex
// and abort the CTA.
__device__ void build_masks(const int* A, int na, const int* B, int nb, int b_lo, int b_hi,
                            uint32_t (*mask)[kMaskWords], int* n_out, int* err,
                            volatile int* abort_flag) {
  const int lane = threadIdx.x & 31;
  const int range = b_hi - b_lo;
  if (range > kMaxUnionBlocks) {
    if (lane == 0) {
      if (err) atomicOr(err, kErrBadIndex);
      *abort_flag = 1;
      *n_out = 0;
    }
    return;
  }
  for (int i = lane; i < 2 * kMaskWords; i += 32) mask[i / kMaskWords][i % kMaskWords] = 0u;
  __syncwarp();
  for (int i = lane; i < na; i += 32) {
    const int v = __ldg(A + i) - b_lo;
    if (v >= 0 && v < range) atomicOr(&mask[0][v >> 5], 1u << (v & 31));
    else { if (err) atomicOr(err, kErrBadIndex); *abort_flag = 1; }
  }
  for (int i = lane; i < nb; i += 32) {
    const int v = __ldg(B + i) - b_lo;
    if (v >= 0 && v < range) atomicOr(&mask[1][v >> 5], 1u << (v & 31));
    else { if (err) atomicOr(err, kErrBadIndex); *abort_flag = 1; }
  }
  __syncwarp();
  int cnt = 0;
  for (int w = lane; w < kMaskWords; w += 32) cnt += __popc(mask[0][w] | mask[1][w]);
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) *n_out = cnt;
  __syncwarp();
}

// A CTA's KV blocks in ascending order; every role walks the same sequence with its own
// cursor. Dense problems take every block of [b_lo, b_hi); block-sparse ones the union of the
// two bitmaps. Bit t of m is set when query tile t attends to the block.
struct BlockWalk {
  int next = 0;      // dense: next block offset; block-sparse: next bitmap word
  uint32_t rem = 0;  // block-sparse: blocks of word next - 1 not yet visited
};

__device__ __forceinline__ void walk_next(BlockWalk& s, bool sparse, int b_lo, int dense_mask,
                                          const uint32_t (*mask)[kMaskWords], int& b, int& m) {
  if (!sparse) {
    b = b_lo + s.next++;
    m = dense_mask;
    return;
  }
  while (s.rem == 0u && s.next < kMaskWords) {
    s.rem = mask[0][s.next] | mask[1][s.next];
    ++s.next;
  }
  if (s.rem == 0u) {  // walked past the union (callers stop at n_blocks): attend nothing
    b = b_lo;
    m = 0;
    return;
  }
  const int w = s.next - 1;
  const int bit = __ffs(s.rem) - 1;
  s.rem &= s.rem - 1u;
  b = b_lo + w * 32 + bit;
  m = static_cast<int>(((mask[0][w] >> bit) & 1u) | (((mask[1][w] >> bit) & 1u) << 1));
}

// Skip the first k blocks of the walk (the start of this CTA's split-KV segment).
__device__ __forceinline__ void walk_skip(BlockWalk& s, bool sparse, int k,
                                          const uint32_t (*mask)[kMaskWords]) {
  if (!sparse) {
    s.next += k;
    return;
  }
  while (k > 0) {
    if (s.rem == 0u) {
      if (s.next >= kMaskWords) return;
      s.rem = mask[0][s.next] | mask[1][s.next];
      ++s.next;
      continue;
    }
    const int c = __popc(s.rem);
    if (c <= k) {
      k -= c;
      s.rem = 0u;
    } else {
      for (; k > 0; --k) s.rem &= s.rem - 1u;
    }
  }
}

// Store the 128 output rows of a query tile as bf16. Each warp stages its 32 rows in `stage`
// (32 rows x 128 bytes: half a row at a time, 16-byte chunks XOR-swizzled by row) and stores
// them with 8 lanes per row, so one warp store instruction writes four whole 128-byte lines
// instead of 32 scattered 16-byte pieces (this matters most for rows bound for a peer GPU over
// NVLink). `dst` is this thread's row address (0: no row); `row_values(ch, v)` yields the 32
// scaled fp32 values of column chunk ch (0..3) of this thread's row. Halves [kHalfBegin,
// kHalfEnd) of the row are stored (a warp that owns half of each row stores one half).
template <int kHalfBegin = 0, int kHalfEnd = 2, typename RowValues>
__device__ __forceinline__ void store_tile_rows(uint8_t* stage, int lane, unsigned long long dst,
                                                RowValues&& row_values) {
#pragma unroll
  for (int half = kHalfBegin; half < kHalfEnd; ++half) {
#pragma unroll
    for (int hc = 0; hc < 2; ++hc) {
      float v[32];
      row_values(half * 2 + hc, v);
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int chunk = hc * 4 + j;
        *reinterpret_cast<uint4*>(stage + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
            make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      }
    }
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + (lane >> 3);
      const int chunk = lane & 7;
      const uint4 val =
          *reinterpret_cast<const uint4*>(stage + r * 128 + ((chunk ^ (r & 7)) << 4));
      const unsigned long long d = __shfl_sync(0xffffffffu, dst, r);
      if (d) reinterpret_cast<uint4*>(static_cast<uintptr_t>(d) + half * 128)[chunk] = val;
    }
    __syncwarp();
  }
}

// kParts (e4m3 only): the KV sequence is segmented e4m3 parts with their own scales
// (AttnParams::block_part); a separate instantiation, so the other launches carry none of it.
template <bool kFp8, bool kParts = false>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<kFp8>;
  constexpr int kKS = Cfg::kKStages;
  constexpr int kVS = Cfg::kVStages;
  extern __shared__ uint8_t smem_raw[];
  AttnSmem<kFp8>& sm = *reinterpret_cast<AttnSmem<kFp8>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;

  // ---- locate this CTA's work: problem, head, pair of query tiles
  int pi = 0;
  while (pi + 1 < p.n_prob && static_cast<int>(blockIdx.x) >= p.prob[pi + 1].cta_begin) ++pi;
  const AttnProblemDev pr = p.prob[pi];
  const int local = static_cast<int>(blockIdx.x) - pr.cta_begin;
  const int seg = local % pr.split;  // split-KV segment of this CTA (block-sparse problems)
  const int head = local / pr.split / pr.pairs;
  const int pair = local / pr.split - head * pr.pairs;
  const int n_tiles = min(2, pr.tiles - pair * 2);
  const int q_row0 = pr.q_lo + pair * 2 * kBlockM;
  const int b_lo = pr.kv_lo / kBlockN;
  const int b_hi = (pr.kv_hi + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sm.q_full), 1);
    for (int s = 0; s < kKS; ++s) {
      mbar_init(smem_u32(&sm.k_full[s]), 1);
      mbar_init(smem_u32(&sm.k_empty[s]), n_tiles);  // one release per MMA warp
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(smem_u32(&sm.v_full[s]), 1);
      mbar_init(smem_u32(&sm.v_empty[s]), n_tiles);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&sm.s_full[t]), 1);
      mbar_init(smem_u32(&sm.s_free[t]), 4);    // one per softmax warp of the tile
      mbar_init(smem_u32(&sm.p_full[t]), 128);  // every softmax thread
      mbar_init(smem_u32(&sm.pv_done[t]), 1);
      mbar_init(smem_u32(&sm.o_done[t]), 1);
      for (int q = 0; q < 4; ++q) mbar_init(smem_u32(&sm.exp_tok[t][q]), 1);
    }
    mbar_init(smem_u32(&sm.drain), n_tiles);
    sm.abort_flag = 0;
    sm.n_blocks = b_hi - b_lo;
    fence_mbar_init();
  }
  __syncthreads();
  if (pr.sparse && warp == 2) {
    const int qb = (q_row0 - pr.q_lo) / kBlockM;
    const int* nums = p.kv_num_blocks + static_cast<size_t>(head) * p.q_blocks;
    const int* A = p.kv_indices + (static_cast<size_t>(head) * p.q_blocks + qb) * p.kv_stride;
    const int na = min(__ldg(nums + qb), p.kv_stride);
    const int nb = (n_tiles > 1) ? min(__ldg(nums + qb + 1), p.kv_stride) : 0;
    build_masks(A, na, A + p.kv_stride, nb, b_lo, b_hi, sm.kv_mask, &sm.n_blocks, p.err,
                abort_flag);
  }
  __syncthreads();

  // Split-KV: a union of more than kSplitSegBlocks blocks is cut into up to pr.split equal
  // segments, one per CTA of the pair; each writes unnormalised partial results and the last
  // to finish merges them. CTAs beyond the segments needed leave before taking TMEM.
  const int n_all = sm.n_blocks;
  const int nseg = pr.split > 1 ? max(1, min(pr.split, (n_all + kSplitSegBlocks - 1) / kSplitSegBlocks))
                                : 1;
  if (seg >= nseg) return;
  const int seg_len = (n_all + nseg - 1) / nseg;
  const int seg_lo = min(n_all, seg * seg_len);
  const int nblk = min(n_all, seg_lo + seg_len) - seg_lo;
  const bool split_out = nseg > 1;
  const int gseg = (pr.pair_begin + head * pr.pairs + pair) * pr.split;  // first segment slot

  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tbase = sm.tmem_base;
  const int dense_mask = (n_tiles > 1) ? 3 : 1;
  BlockWalk walk;
  walk_skip(walk, pr.sparse != 0, seg_lo, sm.kv_mask);
  // destination of output row `row` of query tile t; 0 for rows past the problem's range
  auto row_dst = [&](int t, int row) -> unsigned long long {
    const int qrow = q_row0 + t * kBlockM + row;
    if (qrow >= pr.q_hi) return 0ull;
    if (p.out_peers) {
      // heads -> sequence exchange fused into the store: row qrow belongs to the sequence
      // shard of rank qrow / rows_per_rank, which holds all heads of its rows
      const int owner = min(qrow / p.out_rows_per_rank, p.out_ranks - 1);
      const int orow = qrow - owner * p.out_rows_per_rank;
      return p.out_peers[owner] +
             (static_cast<size_t>(orow) * p.out_heads + p.out_head0 + head) * kHeadDim * 2;
    }
    return reinterpret_cast<uintptr_t>(p.out) +
           (static_cast<size_t>(qrow) * p.heads + head) * kHeadDim * 2;
  };
  auto next_block = [&](int& b, int& m) {
    walk_next(walk, pr.sparse != 0, b_lo, dense_mask, sm.kv_mask, b, m);
  };

  // Register split (every warp of a warpgroup executes the same setmaxnreg at the top of its
  // role): the producer/MMA warpgroup gives registers to the two softmax warpgroups.
  if (warp == 0 || warp == 3) {
    // ================================================================ TMA producers
    // Warp 0 loads Q and streams K blocks, warp 3 streams V blocks: K for block i is released
    // by the QK MMAs of block i, V by the PV MMAs, so each stream runs ahead on its own ring.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    const bool is_k = (warp == 0);
    if (lane == 0 && !*abort_flag) {
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      tma_prefetch_desc(map);
      if (is_k) {
        tma_prefetch_desc(&tmQ);
        const uint32_t qbar = smem_u32(&sm.q_full);
        mbar_expect_tx(qbar, n_tiles * Cfg::kTileBytes);
        for (int t = 0; t < n_tiles; ++t)
          for (int a = 0; a < Cfg::kAtoms; ++a)
            tma_load_3d(smem_u32(sm.q[t]) + a * Cfg::kAtomBytes, &tmQ, qbar,
                        a * (128 / Cfg::kElem), head, q_row0 + t * kBlockM);
      }
      for (int i = 0; i < nblk; ++i) {
        const int s = is_k ? i % kKS : i % kVS;
        const uint32_t ph = (is_k ? i / kKS : i / kVS) & 1;
        int b, m;
        next_block(b, m);
        int page = (b >= 0 && b < p.table_blocks) ? __ldg(p.page_table + b) : -1;
        if (page < 0 || page >= p.pool_pages) {
          if (p.err) atomicOr(p.err, kErrBadPage);
          *abort_flag = 1;
          break;
        }
        uint64_t* empty = is_k ? &sm.k_empty[s] : &sm.v_empty[s];
        if (!mbar_wait(smem_u32(empty), ph ^ 1, abort_flag, p.err)) break;
        H3SA_TRACE_AT(i, is_k ? 14 : 15);
        const uint32_t fb = smem_u32(is_k ? &sm.k_full[s] : &sm.v_full[s]);
        mbar_expect_tx(fb, Cfg::kTileBytes);
        const uint32_t dst = smem_u32(is_k ? sm.k[s] : sm.v[s]);
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_3d(dst + a * Cfg::kAtomBytes, map, fb, a * (128 / Cfg::kElem), page * kBlockN,
                      head);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ================================================================ MMA issuers
    // Warp 1 issues the MMAs of query tile 0, warp 2 those of tile 1. A warp stays blocked in
    // tcgen05.mma until the tensor pipe takes the instruction, so one issuer per tile keeps
    // the pipe fed while the other waits on its softmax or on a barrier. Each warp runs its
    // loop converged (all values warp-uniform); one elected lane issues every tcgen05
    // instruction. Shared-memory descriptors advance by constant 32-bit steps.
    //
    // Per block i: QK(i) into S_t as soon as the softmax has read the previous scores out of
    // TMEM (s_free), then PV(i - 1) once that softmax has written P to shared memory (p_full).
    // S and P no longer share TMEM, so the next QK overlaps the current softmax.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    const int mt = warp - 1;  // the query tile this warp serves
    if (mt < n_tiles) {
      const uint32_t tS = tbase + static_cast<uint32_t>(mt) * 128u;
      const uint32_t tO = tbase + 256u + static_cast<uint32_t>(mt) * 128u;
      const uint32_t qlo = sdesc_lo(smem_u32(sm.q[mt]), 16);
      const uint32_t plo = sdesc_lo(smem_u32(sm.p[mt]), 16);
      const uint32_t klo0 = sdesc_lo(smem_u32(sm.k[0]), 16);
      const uint32_t vlo0 = sdesc_lo(smem_u32(sm.v[0]), Cfg::kAtomBytes);
      constexpr uint32_t kTileDesc = Cfg::kTileBytes >> 4;  // descriptor step between stages
      int cnt = 0;        // QK MMAs issued (softmax rounds requested)
      int npv = 0;        // PV rounds issued
      bool pend = false;  // PV for the previous block still to be issued
      int pb = 0;         // block index of the previous block
      bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sm.q_full), 0, abort_flag, p.err));
      tc_fence_after();
      for (int i = 0; ok && i <= nblk; ++i) {
        const bool last = (i == nblk);
        const int sk = i % kKS;
        int b = 0, m = 0;
        bool w = true;
        if (!last) {
          next_block(b, m);
          w = mbar_wait(smem_u32(&sm.k_full[sk]), (i / kKS) & 1, abort_flag, p.err);
        }
        const bool mine = !last && ((m >> mt) & 1);
        // S_t is overwritten only once the softmax has loaded the previous round's scores
        if (w && mine && cnt > 0)
          w = mbar_wait(smem_u32(&sm.s_free[mt]), (cnt - 1) & 1, abort_flag, p.err);
        if (!(ok = __all_sync(0xffffffffu, w))) break;
        H3SA_TRACE_AT(i, mt == 0 ? 10 : 16);
        tc_fence_after();
        if (mine) {
          const uint32_t klo = klo0 + static_cast<uint32_t>(sk) * kTileDesc;
#pragma unroll
          for (int kk = 0; kk < Cfg::kKSteps; ++kk) {
            const uint32_t off = ((kk * Cfg::kKStepBytes / 128) * Cfg::kAtomBytes +
                                  (kk * Cfg::kKStepBytes) % 128) >> 4;
            if constexpr (kFp8)
              mma_ss_f8(tS, sdesc_join(qlo + off), sdesc_join(klo + off), Cfg::kIdescQK,
                        kk > 0 ? 1u : 0u);
            else
              mma_ss(tS, sdesc_join(qlo + off), sdesc_join(klo + off), Cfg::kIdescQK,
                     kk > 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&sm.s_full[mt]));
          ++cnt;
        }
        // this warp's share of the K stage release (the barriers count one per MMA warp)
        if (!last) tc_commit(smem_u32(&sm.k_empty[sk]));
        if (i > 0) {
          const int sv = (i - 1) % kVS;
          // Every warp waits for the previous block's V before releasing its stage, used or
          // not: the release barriers count one arrival per warp and phase, and a warp running
          // ahead (its tile skips blocks) must not arrive twice on one phase.
          w = mbar_wait(smem_u32(&sm.v_full[sv]), ((i - 1) / kVS) & 1, abort_flag, p.err);
          if (w && pend) w = mbar_wait(smem_u32(&sm.p_full[mt]), npv & 1, abort_flag, p.err);
          if (!(ok = __all_sync(0xffffffffu, w))) break;
          H3SA_TRACE_AT(i, 11 + mt);
          tc_fence_after();
          if (pend) {
            // A partial block's P is zero outside its valid rows, but the tensor core still
            // multiplies those zeros with whatever the V rows hold there (rows of the page the
            // problem does not own, possibly never written: a NaN code would poison O). Zero
            // those V rows in shared memory first; both MMA warps may do it, writing the same
            // zeros, and the TMA for this stage has completed (v_full).
            const int col0 = pb * kBlockN;
            const int vlo_row = max(pr.kv_lo - col0, 0);
            const int vhi_row = min(pr.kv_hi - col0, kBlockN);
            if (vlo_row > 0 || vhi_row < kBlockN) {
              uint8_t* vbase = sm.v[sv];
              const int nbad = vlo_row + (kBlockN - vhi_row);
              for (int idx = lane; idx < nbad * Cfg::kAtoms * 8; idx += 32) {
                const int chunk = idx & 7;
                const int rest = idx >> 3;
                const int a = rest % Cfg::kAtoms;
                const int k = rest / Cfg::kAtoms;
                const int r = k < vlo_row ? k : vhi_row + (k - vlo_row);
                reinterpret_cast<uint4*>(vbase + a * Cfg::kAtomBytes + r * 128)[chunk] =
                    make_uint4(0u, 0u, 0u, 0u);
              }
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              __syncwarp();
            }
            const uint32_t vlo = vlo0 + static_cast<uint32_t>(sv) * kTileDesc;
#pragma unroll
            for (int kk = 0; kk < Cfg::kKSteps; ++kk) {
              const uint32_t off = ((kk * Cfg::kKStepBytes / 128) * Cfg::kAtomBytes +
                                    (kk * Cfg::kKStepBytes) % 128) >> 4;
              const uint64_t bdesc =
                  sdesc_join(vlo + ((kk * Cfg::kPvRowsPerStep * 128) >> 4));
              const uint32_t acc = (npv > 0 || kk > 0) ? 1u : 0u;
              if constexpr (kFp8)
                mma_ss_f8(tO, sdesc_join(plo + off), bdesc, Cfg::kIdescPV, acc);
              else
                mma_ss(tO, sdesc_join(plo + off), bdesc, Cfg::kIdescPV, acc);
            }
            tc_commit(smem_u32(&sm.pv_done[mt]));
            ++npv;
          }
          tc_commit(smem_u32(&sm.v_empty[sv]));
        }
        pend = mine;
        pb = b;
        if (mt == 0) H3SA_TRACE_AT(i, 13);
      }
      if (ok) tc_commit(smem_u32(&sm.o_done[mt]));
      // Whatever happened, leave no tensor-core work in flight past the teardown.
      tc_commit(smem_u32(&sm.drain));
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(smem_u32(&sm.drain), 0)) {
        if (global_ns() - t0 > kWaitTimeoutNs) {
          if (p.err && lane == 0) atomicOr(p.err, kErrWaitTimeout);
          break;
        }
      }
    }
  } else {
    // ================================================================ softmax / epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int t = (warp - 4) >> 2;
    if (t < n_tiles) {
      const int row = (warp & 3) * 32 + lane;
      const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
      const uint32_t tS = tbase + static_cast<uint32_t>(t) * 128u + lane_off;
      const uint32_t tO = tbase + 256u + static_cast<uint32_t>(t) * 128u + lane_off;
      uint8_t* const prow = sm.p[t] + row * 128;  // this row in each 16 KB atom of P
      float scale_log2;
      if constexpr (kFp8)
        scale_log2 = __ldg(p.q_scale + head) * __ldg(p.k_scale + head) * p.softmax_scale_log2;
      else
        scale_log2 = p.scale_log2;
      // Lazy rescaling: O and l are rescaled only when a row maximum grows by more than
      // kRescaleThreshold (log2 units); P is then bounded by 2^(threshold + boost).
      constexpr float kRescaleThreshold = kFp8 ? H3SA_FP8_RESCALE_THRESHOLD : 8.0f;
      constexpr float kBoost = kFp8 ? H3SA_FP8_BOOST : 0.0f;  // e4m3 P: bulk above 2^-6
      float m_used = -INFINITY;
      float l_sum = 0.f;
      int c = 0;
      bool ok = true;
      uint64_t scale2 = f2_pack(scale_log2, scale_log2);
      // segmented e4m3 KV: per-block K and V scales (see block_scales)
      constexpr bool parts = kFp8 && kParts;
      float q_sl2 = 0.f;
      float v_cur = 1.f;  // O is accumulated in units of this V scale
      if constexpr (kFp8) {
        v_cur = __ldg(p.v_scale + head);
        if (parts) q_sl2 = __ldg(p.q_scale + head) * p.softmax_scale_log2;
      }
      float sl2 = scale_log2;  // S scale of the current part (log2 units)
      int cur_part = -1;
      // The exponentials of block i of tile 1 follow those of block i of tile 0, and those of
      // block i + 1 of tile 0 follow those of block i of tile 1; a tile that skips a block
      // (block-sparse lists) still takes and passes the turn.
      const bool pingpong = H3SA_PINGPONG && n_tiles == 2;
      const uint32_t tok_wait = smem_u32(&sm.exp_tok[t ^ 1][warp & 3]);
      const uint32_t tok_give = smem_u32(&sm.exp_tok[t][warp & 3]);
      for (int i = 0; i < nblk; ++i) {
        int b, m;
        next_block(b, m);
        const bool turn_wait = pingpong && (t == 1 || i > 0);
        const uint32_t turn_ph = static_cast<uint32_t>(t == 1 ? i : i - 1) & 1u;
        if (!((m >> t) & 1)) {
          if (pingpong) {
            if (turn_wait && !(ok = mbar_wait(tok_wait, turn_ph, abort_flag, p.err))) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(tok_give);
          }
          continue;
        }
        int rows = kBlockN;
        bool v_moved = false;  // O moves into another part's V-scale units at this block
        float vr = 1.0f;
        if (parts) part_step(p, head, b, q_sl2, c > 0, cur_part, rows, sl2, scale2, v_cur, vr,
                             v_moved);
        if (!(ok = mbar_wait(smem_u32(&sm.s_full[t]), c & 1, abort_flag, p.err))) break;
        const bool tr = (warp & 3) == 0 && lane == 0;
        if (tr) H3SA_TRACE_AT(i, 5 * t + 0);
        tc_fence_after();
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(tS + 0, r0);
        tmem_ld32(tS + 32, r1);
        tmem_ld32(tS + 64, r2);
        tmem_ld32(tS + 96, r3);
        tmem_wait_ld();
        reg_fence32(r0);
        reg_fence32(r1);
        reg_fence32(r2);
        reg_fence32(r3);
        // the scores are in registers: the next QK may overwrite S_t
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.s_free[t]));
        if (tr) H3SA_TRACE_AT(i, 5 * t + 1);
        float s[kBlockN];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s[j] = __uint_as_float(r0[j]);
          s[32 + j] = __uint_as_float(r1[j]);
          s[64 + j] = __uint_as_float(r2[j]);
          s[96 + j] = __uint_as_float(r3[j]);
        }
        const int col0 = b * kBlockN;
        const int lo = pr.kv_lo - col0;  // valid columns [lo, hi)
        const int hi = min(pr.kv_hi - col0, rows);
        // Only the first and last block of a problem (or of a segmented e4m3 part) can be
        // partial. The flag goes through an opaque move: otherwise the compiler can see that every per-column condition below
        // implies it, drop the branch and run 2 x 128 compare/selects on every block.
        int partial_i = (lo > 0 || hi < kBlockN) ? 1 : 0;
        asm volatile("" : "+r"(partial_i));
        const bool partial = partial_i != 0;
        if (partial) {
#pragma unroll
          for (int j = 0; j < kBlockN; ++j)
            if (j < lo || j >= hi) s[j] = -INFINITY;
        }
        float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
        for (int j = 4; j < kBlockN; j += 8) {
          mx0 = fmax3(mx0, s[j], s[j + 4]);
          mx1 = fmax3(mx1, s[j + 1], s[j + 5]);
          mx2 = fmax3(mx2, s[j + 2], s[j + 6]);
          mx3 = fmax3(mx3, s[j + 3], s[j + 7]);
        }
        const float mx = fmaxf(fmax3(mx0, mx1, mx2), mx3);
        const float m_blk = mx * sl2;
        const bool need = m_blk > m_used + kRescaleThreshold;
        const float m_new = need ? m_blk : m_used;
        // O is rescaled further down, once the previous PV has completed; l now
        const float alpha = need ? fast_exp2(m_used - m_new) : 1.0f;
        const bool any_need = c > 0 && (__any_sync(0xffffffffu, need) || v_moved);
        const float o_scale = alpha * vr;
        l_sum *= alpha;
        m_used = m_new;
        // x = s * scale_log2 - (m_used - boost) in packed fp32 pairs, then 2^x on the MUFU; P
        // packed for the PV MMA, row sum in fp32.
        const float bias = kBoost - m_used;
        const uint64_t bias2 = f2_pack(bias, bias);
#pragma unroll
        for (int j = 0; j < kBlockN; j += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(s[j], s[j + 1]), scale2, bias2), x0, x1);
          s[j] = x0;
          s[j + 1] = x1;
        }
        if (turn_wait && !(ok = mbar_wait(tok_wait, turn_ph, abort_flag, p.err))) break;
        uint64_t sum2 = f2_pack(0.f, 0.f);
        uint32_t pk[kBlockN / 2];  // bf16: one pair per word; e4m3: two pairs per word
#pragma unroll
        for (int j = 0; j < kBlockN; j += 2) {
          const float p0 = fast_exp2(s[j]);
          const float p1 = fast_exp2(s[j + 1]);
          sum2 = f2_add(sum2, f2_pack(p0, p1));
          if constexpr (kFp8) {
            uint16_t q;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(q) : "f"(p1), "f"(p0));
            if ((j & 2) == 0) pk[j / 4] = q;
            else pk[j / 4] |= static_cast<uint32_t>(q) << 16;
          } else {
            pk[j / 2] = pack_bf16x2(p0, p1);
          }
        }
        if (pingpong) {
          __syncwarp();
          if (lane == 0) mbar_arrive(tok_give);
        }
        float sa, sb;
        f2_unpack(sum2, sa, sb);
        l_sum += sa + sb;
        if (tr) H3SA_TRACE_AT(i, 5 * t + 3);
        // The previous PV has read P out of shared memory and finished accumulating into O.
        if (c > 0 && !(ok = mbar_wait(smem_u32(&sm.pv_done[t]), (c - 1) & 1, abort_flag, p.err)))
          break;
        if (tr) H3SA_TRACE_AT(i, 5 * t + 2);
        if (any_need) {
          tc_fence_after();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t o[32];
            tmem_ld32(tO + ch * 32, o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * o_scale);
            tmem_st32(tO + ch * 32, o);
          }
          tmem_wait_st();
        }
        // P row into shared memory in the 128-byte-swizzled K-major layout the PV MMA reads
        // (16-byte chunk c of a row at position c ^ (row % 8) of its 128-byte line)
        constexpr int kChunks = kBlockN * Cfg::kElem / 16;
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          uint8_t* dst = prow + (ch >> 3) * Cfg::kAtomBytes + (((ch & 7) ^ (row & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) =
              make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        mbar_arrive(smem_u32(&sm.p_full[t]));
        if (tr) H3SA_TRACE_AT(i, 5 * t + 4);
        ++c;
      }
      if (ok) ok = mbar_wait(smem_u32(&sm.o_done[t]), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
        // c == 0: this tile attended no block (of this segment), its rows see no key and are
        // written as zeros (TMEM O was never written)
        const bool any = c > 0;
        if (split_out) {
          // unnormalised partial of this segment: O (fp32, dequantised: times the V scale of
          // its units), the row's running maximum (log2 units of the scaled scores) and its
          // sum of P
          const size_t slot = (static_cast<size_t>(gseg + seg) * 2 + t) * kBlockM + row;
          float4* po = reinterpret_cast<float4*>(p.split_o + slot * kHeadDim);
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            if (any) {
              tmem_ld32(tO + ch * 32, r);
              tmem_wait_ld();
              reg_fence32(r);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) r[j] = 0u;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              po[ch * 8 + j] = make_float4(__uint_as_float(r[4 * j]) * v_cur,
                                           __uint_as_float(r[4 * j + 1]) * v_cur,
                                           __uint_as_float(r[4 * j + 2]) * v_cur,
                                           __uint_as_float(r[4 * j + 3]) * v_cur);
          }
          p.split_ml[slot * 2] = any ? m_used : -INFINITY;
          p.split_ml[slot * 2 + 1] = any ? l_sum : 0.f;
          __threadfence();
        } else {
          float out_scale = any ? 1.0f / l_sum : 0.f;
          if constexpr (kFp8) out_scale *= v_cur;
          store_tile_rows(sm.q[t] + (warp & 3) * (32 * 128), lane, row_dst(t, row),
                          [&](int ch, float (&v)[32]) {
                            uint32_t r[32];
                            if (any) {
                              tmem_ld32(tO + ch * 32, r);
                              tmem_wait_ld();
                              reg_fence32(r);
                            } else {
#pragma unroll
                              for (int j = 0; j < 32; ++j) r[j] = 0u;
                            }
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * out_scale;
                          });
          // peer stores: make them visible system-wide before the kernel is seen as done
          if (p.out_peers) __threadfence_system();
        }
      }
    }
    if (split_out) {
      // Last-arriver merge over the pair's segments (no waiting: the CTA whose increment
      // completes the count merges). Named barrier 1 spans the 256 softmax threads, every one
      // of which reaches it.
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (threadIdx.x == 128) {
        __threadfence();
        const int done = atomicAdd(p.split_count + gseg / pr.split, 1);
        sm.split_last = (done == nseg - 1) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (sm.split_last && t < n_tiles && !*abort_flag) {
        __threadfence();
        const int row = (warp & 3) * 32 + lane;
        float mx = -INFINITY;
        for (int sg = 0; sg < nseg; ++sg) {
          const size_t slot = (static_cast<size_t>(gseg + sg) * 2 + t) * kBlockM + row;
          mx = fmaxf(mx, __ldcg(p.split_ml + slot * 2));
        }
        float acc[kHeadDim];
#pragma unroll
        for (int j = 0; j < kHeadDim; ++j) acc[j] = 0.f;
        float lsum = 0.f;
        if (mx > -INFINITY) {
          for (int sg = 0; sg < nseg; ++sg) {
            const size_t slot = (static_cast<size_t>(gseg + sg) * 2 + t) * kBlockM + row;
            const float ms = __ldcg(p.split_ml + slot * 2);
            const float w = ms > -INFINITY ? fast_exp2(ms - mx) : 0.f;
            lsum += w * __ldcg(p.split_ml + slot * 2 + 1);
            const float4* po = reinterpret_cast<const float4*>(p.split_o + slot * kHeadDim);
#pragma unroll
            for (int j = 0; j < kHeadDim / 4; ++j) {
              const float4 v = __ldcg(po + j);
              acc[4 * j] += w * v.x;
              acc[4 * j + 1] += w * v.y;
              acc[4 * j + 2] += w * v.z;
              acc[4 * j + 3] += w * v.w;
            }
          }
        }
        // the segments' O are already dequantised (see the partial store)
        const float out_scale = lsum > 0.f ? 1.0f / lsum : 0.f;
        store_tile_rows(sm.q[t] + (warp & 3) * (32 * 128), lane, row_dst(t, row),
                        [&](int ch, float (&v)[32]) {
#pragma unroll
                          for (int j = 0; j < 32; ++j) v[j] = acc[ch * 32 + j] * out_scale;
                        });
        if (p.out_peers) __threadfence_system();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ============================================================================ one-tile kernel
// Used for launches with a block-sparse problem. One 128-row query tile per CTA, walking the
// tile's own block list, with S double-buffered in TMEM (S0 [0,128), S1 [128,256)). P goes
// back into TMEM over the S buffer it came from and is read by a TMEM x smem MMA. The MMA warp
// issues PV(i) and then QK(i + 2) into the buffer PV(i) has just read (one thread's
// tcgen05.mma execute in issue order), so the scores of block i + 1 are computed while the
// softmax works on block i. QK(i + 2) still waits for the softmax of block i, through PV(i).
//
// Eight softmax warps: warps 4-7 and 8-11 cover the same 32-row quarters (TMEM lanes
// 32 * (warp % 4)), the first four the left 64 columns of each row and the last four the right
// 64. With kIndep (the default) the two halves are independent online softmaxes, each with its
// own running maximum and sum, its P over its own S columns and its own O accumulator (O0
// [256,384), O1 [384,512)), merged at the end; otherwise they exchange each block's row
// maximum through shared memory and share one O [256,384) with P over S's upper half.
// One-tile kernel: the two column halves of a row run independent online softmaxes with an
// O accumulator each (O0 [256,384), O1 [384,512)), merged at the end (1), or share each
// block's row maximum through shared memory (0). Measured on the 768p SP=8 block-sparse mask:
// 0.236 ms independent, 0.253 ms shared.
#ifndef H3SA_ONE_TILE_INDEP
#define H3SA_ONE_TILE_INDEP 1
#endif

// Dense launches run the two-tile kernel (0) or the one-tile kernel as well (1).
#ifndef H3SA_ONE_TILE_DENSE
#define H3SA_ONE_TILE_DENSE 0
#endif

template <bool kFp8>
struct Attn1Cfg {
  static constexpr int kKStages = kFp8 ? 3 : 2;
  static constexpr int kVStages = kFp8 ? 3 : 2;
};

template <bool kFp8>
struct alignas(1024) Attn1Smem {
  using Cfg = AttnCfg<kFp8>;
  using Cfg1 = Attn1Cfg<kFp8>;
  uint8_t q[Cfg::kTileBytes];
  uint8_t k[Cfg1::kKStages][Cfg::kTileBytes];  // also the epilogue's staging (4 KB per warp)
  uint8_t v[Cfg1::kVStages][Cfg::kTileBytes];
  uint64_t q_full;
  uint64_t k_full[Cfg1::kKStages], k_empty[Cfg1::kKStages];
  uint64_t v_full[Cfg1::kVStages], v_empty[Cfg1::kVStages];
  uint64_t s_full[2], pv_done[2], o_done;  // pv_done: per half (kIndep)
  // P written, per column half (kIndep; otherwise [0] counts both) and block parity: with
  // independent halves one half can run a block ahead, and one barrier per half would then
  // complete twice before the MMA warp waits on it
  uint64_t p_full[2][2];
  uint64_t half_x[4];  // per row quarter: both column halves posted their value
  uint64_t drain;
  float mx_x[2][2][kBlockM];  // [block parity][column half][row]: half-row maxima
  float l_x[2][kBlockM];      // [column half][row]: half-row sums at the end
  uint32_t tmem_base;
  int abort_flag;
  int n_blocks;
  int split_last;
  uint32_t kv_mask[2][kMaskWords];  // block-sparse: the tile's list (second row unused)
};

template <bool kFp8>
constexpr size_t attn1_smem_bytes() {
  return sizeof(Attn1Smem<kFp8>) + 1024;
}
static_assert(attn1_smem_bytes<false>() <= 232448, "bf16 one-tile attention exceeds 227 KB");
static_assert(attn1_smem_bytes<true>() <= 232448, "e4m3 one-tile attention exceeds 227 KB");
static_assert(AttnCfg<false>::kTileBytes * Attn1Cfg<false>::kKStages >= 8 * 32 * 128 &&
                  AttnCfg<true>::kTileBytes * Attn1Cfg<true>::kKStages >= 8 * 32 * 128,
              "the K ring must hold the epilogue staging of eight warps");

template <bool kFp8, bool kIndep, bool kParts = false>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn1_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<kFp8>;
  using Cfg1 = Attn1Cfg<kFp8>;
  constexpr int kKS = Cfg1::kKStages;
  constexpr int kVS = Cfg1::kVStages;
  extern __shared__ uint8_t smem_raw[];
  Attn1Smem<kFp8>& sm = *reinterpret_cast<Attn1Smem<kFp8>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;

  // ---- locate this CTA's work: problem, head, query tile, split-KV segment
  int pi = 0;
  while (pi + 1 < p.n_prob && static_cast<int>(blockIdx.x) >= p.prob[pi + 1].cta_begin) ++pi;
  const AttnProblemDev pr = p.prob[pi];
  const int local = static_cast<int>(blockIdx.x) - pr.cta_begin;
  const int seg = local % pr.split;
  const int unit = local / pr.split;  // `pairs` counts query tiles for this kernel
  const int head = unit / pr.pairs;
  const int tile = unit - head * pr.pairs;
  const int q_row0 = pr.q_lo + tile * kBlockM;
  const int b_lo = pr.kv_lo / kBlockN;
  const int b_hi = (pr.kv_hi + kBlockN - 1) / kBlockN;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&sm.q_full), 1);
    for (int s = 0; s < kKS; ++s) {
      mbar_init(smem_u32(&sm.k_full[s]), 1);
      mbar_init(smem_u32(&sm.k_empty[s]), 1);
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(smem_u32(&sm.v_full[s]), 1);
      mbar_init(smem_u32(&sm.v_empty[s]), 1);
    }
    mbar_init(smem_u32(&sm.s_full[0]), 1);
    mbar_init(smem_u32(&sm.s_full[1]), 1);
    for (int hh = 0; hh < 2; ++hh)
      for (int par = 0; par < 2; ++par)  // every softmax thread (of the half with kIndep)
        mbar_init(smem_u32(&sm.p_full[hh][par]), (kIndep || hh == 1) ? 128 : 256);
    mbar_init(smem_u32(&sm.pv_done[0]), 1);
    mbar_init(smem_u32(&sm.pv_done[1]), 1);
    mbar_init(smem_u32(&sm.o_done), 1);
    for (int q = 0; q < 4; ++q) mbar_init(smem_u32(&sm.half_x[q]), 2);  // one per half warp
    mbar_init(smem_u32(&sm.drain), 1);
    sm.abort_flag = 0;
    sm.n_blocks = b_hi - b_lo;
    fence_mbar_init();
  }
  __syncthreads();
  if (pr.sparse && warp == 2) {
    const int* nums = p.kv_num_blocks + static_cast<size_t>(head) * p.q_blocks;
    const int* A = p.kv_indices + (static_cast<size_t>(head) * p.q_blocks + tile) * p.kv_stride;
    const int na = min(__ldg(nums + tile), p.kv_stride);
    build_masks(A, na, A, 0, b_lo, b_hi, sm.kv_mask, &sm.n_blocks, p.err, abort_flag);
  }
  __syncthreads();

  // split-KV segments, as in attn_fwd_kernel
  const int n_all = sm.n_blocks;
  const int nseg = pr.split > 1 ? max(1, min(pr.split, (n_all + kSplitSegBlocks - 1) / kSplitSegBlocks))
                                : 1;
  if (seg >= nseg) return;
  const int seg_len = (n_all + nseg - 1) / nseg;
  const int seg_lo = min(n_all, seg * seg_len);
  const int nblk = min(n_all, seg_lo + seg_len) - seg_lo;
  const bool split_out = nseg > 1;
  const int gseg = (pr.pair_begin + head * pr.pairs + tile) * pr.split;

  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tbase = sm.tmem_base;
  BlockWalk walk;
  walk_skip(walk, pr.sparse != 0, seg_lo, sm.kv_mask);
  auto next_block = [&](int& b) {
    int m;
    walk_next(walk, pr.sparse != 0, b_lo, 1, sm.kv_mask, b, m);
  };
  auto row_dst = [&](int row) -> unsigned long long {
    const int qrow = q_row0 + row;
    if (qrow >= pr.q_hi) return 0ull;
    if (p.out_peers) {
      const int owner = min(qrow / p.out_rows_per_rank, p.out_ranks - 1);
      const int orow = qrow - owner * p.out_rows_per_rank;
      return p.out_peers[owner] +
             (static_cast<size_t>(orow) * p.out_heads + p.out_head0 + head) * kHeadDim * 2;
    }
    return reinterpret_cast<uintptr_t>(p.out) +
           (static_cast<size_t>(qrow) * p.heads + head) * kHeadDim * 2;
  };

  if (warp == 0 || warp == 3) {
    // ================================================================ TMA producers
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    const bool is_k = (warp == 0);
    if (lane == 0 && !*abort_flag) {
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      tma_prefetch_desc(map);
      if (is_k) {
        tma_prefetch_desc(&tmQ);
        const uint32_t qbar = smem_u32(&sm.q_full);
        mbar_expect_tx(qbar, Cfg::kTileBytes);
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_3d(smem_u32(sm.q) + a * Cfg::kAtomBytes, &tmQ, qbar, a * (128 / Cfg::kElem),
                      head, q_row0);
      }
      for (int i = 0; i < nblk; ++i) {
        const int s = is_k ? i % kKS : i % kVS;
        const uint32_t ph = (is_k ? i / kKS : i / kVS) & 1;
        int b;
        next_block(b);
        int page = (b >= 0 && b < p.table_blocks) ? __ldg(p.page_table + b) : -1;
        if (page < 0 || page >= p.pool_pages) {
          if (p.err) atomicOr(p.err, kErrBadPage);
          *abort_flag = 1;
          break;
        }
        uint64_t* empty = is_k ? &sm.k_empty[s] : &sm.v_empty[s];
        if (!mbar_wait(smem_u32(empty), ph ^ 1, abort_flag, p.err)) break;
        const uint32_t fb = smem_u32(is_k ? &sm.k_full[s] : &sm.v_full[s]);
        mbar_expect_tx(fb, Cfg::kTileBytes);
        const uint32_t dst = smem_u32(is_k ? sm.k[s] : sm.v[s]);
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_3d(dst + a * Cfg::kAtomBytes, map, fb, a * (128 / Cfg::kElem), page * kBlockN,
                      head);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    // QK(0), QK(1), then per block i: PV(i) once P(i) is in TMEM, and QK(i + 2) into the S
    // buffer PV(i) has just read.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    const uint32_t tO = tbase + 256u;
    const uint32_t qlo = sdesc_lo(smem_u32(sm.q), 16);
    const uint32_t klo0 = sdesc_lo(smem_u32(sm.k[0]), 16);
    const uint32_t vlo0 = sdesc_lo(smem_u32(sm.v[0]), Cfg::kAtomBytes);
    constexpr uint32_t kTileDesc = Cfg::kTileBytes >> 4;
    bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sm.q_full), 0, abort_flag, p.err));
    tc_fence_after();
    auto issue_qk = [&](int i) -> bool {
      const int sk = i % kKS;
      const bool w = mbar_wait(smem_u32(&sm.k_full[sk]), (i / kKS) & 1, abort_flag, p.err);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      const uint32_t tS = tbase + static_cast<uint32_t>(i & 1) * 128u;
      const uint32_t klo = klo0 + static_cast<uint32_t>(sk) * kTileDesc;
#pragma unroll
      for (int kk = 0; kk < Cfg::kKSteps; ++kk) {
        const uint32_t off = ((kk * Cfg::kKStepBytes / 128) * Cfg::kAtomBytes +
                              (kk * Cfg::kKStepBytes) % 128) >> 4;
        if constexpr (kFp8)
          mma_ss_f8(tS, sdesc_join(qlo + off), sdesc_join(klo + off), Cfg::kIdescQK,
                    kk > 0 ? 1u : 0u);
        else
          mma_ss(tS, sdesc_join(qlo + off), sdesc_join(klo + off), Cfg::kIdescQK,
                 kk > 0 ? 1u : 0u);
      }
      tc_commit(smem_u32(&sm.s_full[i & 1]));
      tc_commit(smem_u32(&sm.k_empty[sk]));
      return true;
    };
    if (ok && nblk > 0) ok = issue_qk(0);
    if (ok && nblk > 1) ok = issue_qk(1);
    for (int i = 0; ok && i < nblk; ++i) {
      int b;
      next_block(b);
      const int sv = i % kVS;
      bool w = mbar_wait(smem_u32(&sm.v_full[sv]), (i / kVS) & 1, abort_flag, p.err);
      if (w) w = mbar_wait(smem_u32(&sm.p_full[0][i & 1]), (i >> 1) & 1, abort_flag, p.err);
      if (!(ok = __all_sync(0xffffffffu, w))) break;
      if (lane == 0) H3SA_TRACE_AT(i, 12);
      tc_fence_after();
      {
        // V rows of a partial block outside the problem's KV range are zeroed first (they
        // may hold never-written bytes; P is zero there but 0 x NaN is not)
        const int col0 = b * kBlockN;
        const int vlo_row = max(pr.kv_lo - col0, 0);
        const int vhi_row = min(pr.kv_hi - col0, kBlockN);
        if (vlo_row > 0 || vhi_row < kBlockN) {
          uint8_t* vbase = sm.v[sv];
          const int nbad = vlo_row + (kBlockN - vhi_row);
          for (int idx = lane; idx < nbad * Cfg::kAtoms * 8; idx += 32) {
            const int chunk = idx & 7;
            const int rest = idx >> 3;
            const int a = rest % Cfg::kAtoms;
            const int k = rest / Cfg::kAtoms;
            const int r = k < vlo_row ? k : vhi_row + (k - vlo_row);
            reinterpret_cast<uint4*>(vbase + a * Cfg::kAtomBytes + r * 128)[chunk] =
                make_uint4(0u, 0u, 0u, 0u);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
        }
      }
      const uint32_t vlo = vlo0 + static_cast<uint32_t>(sv) * kTileDesc;
      const uint32_t tSb = tbase + static_cast<uint32_t>(i & 1) * 128u;
      if constexpr (kIndep) {
        // each half's P (its 64 KV rows) into its own O: P_h over S columns [64h, 64h + 64)
        constexpr int kSteps = 64 / Cfg::kPvRowsPerStep;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (hh == 1) {
            const bool w1 =
                mbar_wait(smem_u32(&sm.p_full[1][i & 1]), (i >> 1) & 1, abort_flag, p.err);
            if (!(ok = __all_sync(0xffffffffu, w1))) break;
            if (lane == 0) H3SA_TRACE_AT(i, 13);
            tc_fence_after();
          }
#pragma unroll
          for (int kk = 0; kk < kSteps; ++kk) {
            const uint64_t bdesc =
                sdesc_join(vlo + (((64 * hh + kk * Cfg::kPvRowsPerStep) * 128) >> 4));
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            const uint32_t a_tmem = tSb + 64u * hh + kk * 8u;
            if constexpr (kFp8)
              mma_ts_f8(tO + 128u * hh, a_tmem, bdesc, Cfg::kIdescPV, acc);
            else
              mma_ts(tO + 128u * hh, a_tmem, bdesc, Cfg::kIdescPV, acc);
          }
          tc_commit(smem_u32(&sm.pv_done[hh]));
        }
        if (!ok) break;
      } else {
        const uint32_t tP = tSb + 64u;
#pragma unroll
        for (int kk = 0; kk < kBlockN / Cfg::kPvRowsPerStep; ++kk) {
          const uint64_t bdesc = sdesc_join(vlo + ((kk * Cfg::kPvRowsPerStep * 128) >> 4));
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          if constexpr (kFp8)
            mma_ts_f8(tO, tP + kk * 8u, bdesc, Cfg::kIdescPV, acc);
          else
            mma_ts(tO, tP + kk * 8u, bdesc, Cfg::kIdescPV, acc);
        }
        tc_commit(smem_u32(&sm.pv_done[0]));
      }
      tc_commit(smem_u32(&sm.v_empty[sv]));
      if (i + 2 < nblk) ok = issue_qk(i + 2);
      if (lane == 0) H3SA_TRACE_AT(i, 14);
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
  } else if (warp == 2) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  } else {
    // ================================================================ softmax / epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int q = warp & 3;          // row quarter = TMEM lane quarter
    const int h = (warp - 4) >> 2;   // column half of each row
    const int row = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    // this half's O accumulator (kIndep), or the shared one
    const uint32_t tO = tbase + 256u + (kIndep ? 128u * h : 0u) + lane_off;
    const uint32_t xbar = smem_u32(&sm.half_x[q]);
    float scale_log2;
    if constexpr (kFp8)
      scale_log2 = __ldg(p.q_scale + head) * __ldg(p.k_scale + head) * p.softmax_scale_log2;
    else
      scale_log2 = p.scale_log2;
    constexpr float kRescaleThreshold = kFp8 ? H3SA_FP8_RESCALE_THRESHOLD : 8.0f;
    constexpr float kBoost = kFp8 ? H3SA_FP8_BOOST : 0.0f;
    float m_used = -INFINITY;
    float l_sum = 0.f;
    bool ok = true;
    uint64_t scale2 = f2_pack(scale_log2, scale_log2);
    // segmented e4m3 KV: per-block K and V scales (see block_scales)
    constexpr bool parts = kFp8 && kParts;
    float q_sl2 = 0.f;
    float v_cur = 1.f;  // O is accumulated in units of this V scale
    if constexpr (kFp8) {
      v_cur = __ldg(p.v_scale + head);
      if (parts) q_sl2 = __ldg(p.q_scale + head) * p.softmax_scale_log2;
    }
    float sl2 = scale_log2;  // S scale of the current part (log2 units)
    int cur_part = -1;
    int i = 0;
    for (; i < nblk; ++i) {
      int b;
      next_block(b);
      const bool tr = q == H3SA_TRACE_QUARTER && lane == 0;
      int rows = kBlockN;
      bool v_moved = false;  // O moves into another part's V-scale units at this block
      float vr = 1.0f;
      if (parts) part_step(p, head, b, q_sl2, i > 0, cur_part, rows, sl2, scale2, v_cur, vr,
                           v_moved);
      if (!(ok = mbar_wait(smem_u32(&sm.s_full[i & 1]), (i >> 1) & 1, abort_flag, p.err))) break;
      if (tr) H3SA_TRACE_AT(i, 6 * h + 0);
      tc_fence_after();
      const uint32_t tS = tbase + static_cast<uint32_t>(i & 1) * 128u + lane_off;
      uint32_t r0[32], r1[32];
      tmem_ld32(tS + 64u * h, r0);
      tmem_ld32(tS + 64u * h + 32u, r1);
      tmem_wait_ld();
      reg_fence32(r0);
      reg_fence32(r1);
      if (tr) H3SA_TRACE_AT(i, 6 * h + 1);
      float s[64];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        s[j] = __uint_as_float(r0[j]);
        s[32 + j] = __uint_as_float(r1[j]);
      }
      const int col0 = b * kBlockN + 64 * h;
      const int lo = pr.kv_lo - col0;  // valid columns [lo, hi) of this half
      const int hi = min(pr.kv_hi - col0, rows - 64 * h);
      int partial_i = (lo > 0 || hi < 64) ? 1 : 0;
      asm volatile("" : "+r"(partial_i));
      if (partial_i) {
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (j < lo || j >= hi) s[j] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int j = 4; j < 64; j += 8) {
        mx0 = fmax3(mx0, s[j], s[j + 4]);
        mx1 = fmax3(mx1, s[j + 1], s[j + 5]);
        mx2 = fmax3(mx2, s[j + 2], s[j + 6]);
        mx3 = fmax3(mx3, s[j + 3], s[j + 7]);
      }
      const float mh = fmaxf(fmax3(mx0, mx1, mx2), mx3);
      // both halves of the row: post this half's maximum, read the other's (the barrier also
      // orders the other half's TMEM load of S before this half's P store over it)
      float mx = mh;
      if constexpr (!kIndep) {
        sm.mx_x[i & 1][h][row] = mh;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        if (!(ok = mbar_wait(xbar, i & 1, abort_flag, p.err))) break;
        tc_fence_after();
        mx = fmaxf(mh, sm.mx_x[i & 1][h ^ 1][row]);
      }
      const float m_blk = mx * sl2;
      const bool need = m_blk > m_used + kRescaleThreshold;
      const float m_new = need ? m_blk : m_used;
      const float alpha = need ? fast_exp2(m_used - m_new) : 1.0f;
      const bool any_need = i > 0 && (__any_sync(0xffffffffu, need) || v_moved);
      const float o_scale = alpha * vr;
      l_sum *= alpha;
      m_used = m_new;
      // a half that has seen no valid score yet (all its columns outside the KV range so far;
      // possible with independent halves) keeps its P at zero instead of -inf + inf
      const float bias = kBoost - (m_used == -INFINITY ? 0.f : m_used);
      const uint64_t bias2 = f2_pack(bias, bias);
      if (tr) H3SA_TRACE_AT(i, 6 * h + 2);
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(s[j], s[j + 1]), scale2, bias2), x0, x1);
        s[j] = x0;
        s[j + 1] = x1;
      }
      uint64_t sum2 = f2_pack(0.f, 0.f);
      uint32_t pk[32];  // bf16: 32 words of pairs; e4m3: 16 words of quads
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        const float p0 = fast_exp2(s[j]);
        const float p1 = fast_exp2(s[j + 1]);
        sum2 = f2_add(sum2, f2_pack(p0, p1));
        if constexpr (kFp8) {
          uint16_t qq;
          asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(qq) : "f"(p1), "f"(p0));
          if ((j & 2) == 0) pk[j / 4] = qq;
          else pk[j / 4] |= static_cast<uint32_t>(qq) << 16;
        } else {
          pk[j / 2] = pack_bf16x2(p0, p1);
        }
      }
      float sa, sb;
      f2_unpack(sum2, sa, sb);
      l_sum += sa + sb;
      if (tr) H3SA_TRACE_AT(i, 6 * h + 3);
      if (any_need) {
        // PV(i - 1) has finished accumulating; rescale this half's O columns
        if (!(ok = mbar_wait(smem_u32(&sm.pv_done[kIndep ? h : 0]), (i - 1) & 1, abort_flag,
                             p.err)))
          break;
        tc_fence_after();
        // this half's O (kIndep: all 128 columns of its own accumulator; otherwise its 64
        // columns of the shared one)
#pragma unroll
        for (int ch = 0; ch < (kIndep ? 4 : 2); ++ch) {
          const uint32_t addr = kIndep ? tO + ch * 32 : tO + 64u * h + ch * 32;
          uint32_t o[32];
          tmem_ld32(addr, o);
          tmem_wait_ld();
          reg_fence32(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * o_scale);
          tmem_st32(addr, o);
        }
      }
      // P over S: kIndep puts each half's P over its own S columns [64h, ...); otherwise both
      // halves fill the upper half, bf16 columns [64 + 32h, +32), e4m3 [64 + 16h, +16)
      const uint32_t tPst = kIndep ? tS + 64u * h : tS + 64u + (kFp8 ? 16u : 32u) * h;
      if constexpr (kFp8)
        tmem_st16(tPst, pk);
      else
        tmem_st32(tPst, *reinterpret_cast<uint32_t(*)[32]>(pk));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&sm.p_full[kIndep ? h : 0][i & 1]));
      if (tr) H3SA_TRACE_AT(i, 6 * h + 4);
    }
    // combine the two halves' statistics (one more exchange on the same barrier): the row sum
    // (shared maximum), or with kIndep each half's maximum, sum and O weight
    float m_fin = m_used, l_fin = 0.f, w0 = 1.f, w1 = 0.f;
    if (ok) {
      sm.l_x[h][row] = l_sum;
      if constexpr (kIndep) sm.mx_x[0][h][row] = m_used;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      ok = mbar_wait(xbar, (kIndep ? 0 : nblk) & 1, abort_flag, p.err);
      if (ok) {
        const float l_other = sm.l_x[h ^ 1][row];
        if constexpr (kIndep) {
          const float m_other = sm.mx_x[0][h ^ 1][row];
          const float m0 = h == 0 ? m_used : m_other;
          const float m1 = h == 0 ? m_other : m_used;
          const float l0 = h == 0 ? l_sum : l_other;
          const float l1 = h == 0 ? l_other : l_sum;
          m_fin = fmaxf(m0, m1);
          w0 = m0 > -INFINITY ? fast_exp2(m0 - m_fin) : 0.f;
          w1 = m1 > -INFINITY ? fast_exp2(m1 - m_fin) : 0.f;
          l_fin = w0 * l0 + w1 * l1;
        } else {
          l_fin = l_sum + l_other;
        }
      }
    }
    if (ok) ok = mbar_wait(smem_u32(&sm.o_done), 0, abort_flag, p.err);
    if (ok) {
      tc_fence_after();
      const bool any = nblk > 0;
      const uint32_t tO0 = tbase + 256u + lane_off;
      // unnormalised output columns [32 ch, 32 ch + 32) of this row
      auto raw = [&](int ch, float (&v)[32]) {
        if (!any) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
          return;
        }
        uint32_t a[32];
        tmem_ld32(tO0 + ch * 32, a);
        if constexpr (kIndep) {
          uint32_t c2[32];
          tmem_ld32(tO0 + 128u + ch * 32, c2);
          tmem_wait_ld();
          reg_fence32(a);
          reg_fence32(c2);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = w0 * __uint_as_float(a[j]) + w1 * __uint_as_float(c2[j]);
        } else {
          tmem_wait_ld();
          reg_fence32(a);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(a[j]);
        }
      };
      if (split_out) {
        const size_t slot = static_cast<size_t>(gseg + seg) * 2 * kBlockM + row;
        float4* po = reinterpret_cast<float4*>(p.split_o + slot * kHeadDim + 64 * h);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          float v[32];
          raw(2 * h + ch, v);
#pragma unroll
          for (int j = 0; j < 8; ++j)  // dequantised: times the V scale of O's units
            po[ch * 8 + j] = make_float4(v[4 * j] * v_cur, v[4 * j + 1] * v_cur,
                                         v[4 * j + 2] * v_cur, v[4 * j + 3] * v_cur);
        }
        if (h == 0) {
          p.split_ml[slot * 2] = any ? m_fin : -INFINITY;
          p.split_ml[slot * 2 + 1] = any ? l_fin : 0.f;
        }
        __threadfence();
      } else {
        float out_scale = (any && l_fin > 0.f) ? 1.0f / l_fin : 0.f;
        if constexpr (kFp8) out_scale *= v_cur;
        uint8_t* stage = sm.k[0] + (warp - 4) * (32 * 128);
        auto values = [&](int ch, float (&v)[32]) {
          raw(ch, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= out_scale;
        };
        if (h == 0) store_tile_rows<0, 1>(stage, lane, row_dst(row), values);
        else store_tile_rows<1, 2>(stage, lane, row_dst(row), values);
        if (p.out_peers) __threadfence_system();
      }
    }
    if (split_out) {
      // last-arriver merge over the tile's segments (named barrier 1 spans the 256 softmax
      // threads, every one of which reaches it)
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (threadIdx.x == 128) {
        __threadfence();
        const int done = atomicAdd(p.split_count + gseg / pr.split, 1);
        sm.split_last = (done == nseg - 1) ? 1 : 0;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (sm.split_last && !*abort_flag) {
        __threadfence();
        float mx = -INFINITY;
        for (int sg = 0; sg < nseg; ++sg) {
          const size_t slot = static_cast<size_t>(gseg + sg) * 2 * kBlockM + row;
          mx = fmaxf(mx, __ldcg(p.split_ml + slot * 2));
        }
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.f;
        float lsum = 0.f;
        if (mx > -INFINITY) {
          for (int sg = 0; sg < nseg; ++sg) {
            const size_t slot = static_cast<size_t>(gseg + sg) * 2 * kBlockM + row;
            const float ms = __ldcg(p.split_ml + slot * 2);
            const float w = ms > -INFINITY ? fast_exp2(ms - mx) : 0.f;
            lsum += w * __ldcg(p.split_ml + slot * 2 + 1);
            const float4* po = reinterpret_cast<const float4*>(p.split_o + slot * kHeadDim + 64 * h);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 v = __ldcg(po + j);
              acc[4 * j] += w * v.x;
              acc[4 * j + 1] += w * v.y;
              acc[4 * j + 2] += w * v.z;
              acc[4 * j + 3] += w * v.w;
            }
          }
        }
        // the segments' O are already dequantised (see the partial store)
        const float out_scale = lsum > 0.f ? 1.0f / lsum : 0.f;
        uint8_t* stage = sm.k[0] + (warp - 4) * (32 * 128);
        if (h == 0)
          store_tile_rows<0, 1>(stage, lane, row_dst(row), [&](int ch, float (&v)[32]) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = acc[ch * 32 + j] * out_scale;
          });
        else
          store_tile_rows<1, 2>(stage, lane, row_dst(row), [&](int ch, float (&v)[32]) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = acc[(ch - 2) * 32 + j] * out_scale;
          });
        if (p.out_peers) __threadfence_system();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------ host side

// Split-KV workspace of one (device, stream): grown on demand, never shrunk. Growing it waits
// for the device (the old buffer may be in use by launches already queued) and so cannot run
// inside stream capture; a capture needs an earlier call on that stream with at least as many
// split pairs. Launches on one stream are ordered, so they can share the buffer.
struct SplitSpace {
  float* o;
  float* ml;
  int* count;
};

// Guards the split-KV workspaces. The caller holds it from split_workspace() until its kernel
// is enqueued, so a workspace that another host thread grows (after a device synchronisation)
// is never freed between handing out its pointers and the launch that uses them.
static std::mutex g_split_mu;

static int split_workspace(int pairs, cudaStream_t stream, SplitSpace& out) {
  struct Entry {
    int dev;
    cudaStream_t stream;
    int pairs;
    void* base;
  };
  static Entry entries[64];
  static int n_entries = 0;
  const size_t o_floats = static_cast<size_t>(pairs) * kSplitMax * 2 * kBlockM * kHeadDim;
  const size_t ml_floats = static_cast<size_t>(pairs) * kSplitMax * 2 * kBlockM * 2;
  const size_t bytes = (o_floats + ml_floats) * sizeof(float) + static_cast<size_t>(pairs) * 4;
  int dev = 0;
  cudaGetDevice(&dev);
  Entry* e = nullptr;
  for (int i = 0; i < n_entries; ++i)
    if (entries[i].dev == dev && entries[i].stream == stream) e = &entries[i];
  if (!e) {
    if (n_entries == 64)
      return set_error(H3SA_ERR_UNSUPPORTED, "attention: split-KV workspaces for more than 64 "
                       "(device, stream) pairs");
    e = &entries[n_entries++];
    *e = Entry{dev, stream, 0, nullptr};
  }
  if (e->pairs < pairs) {
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return set_cuda_error("split-KV workspace (synchronize)", err);
    if (e->base) cudaFree(e->base);
    e->base = nullptr;
    e->pairs = 0;
    err = cudaMalloc(&e->base, bytes);
    if (err != cudaSuccess) return set_cuda_error("cudaMalloc(split-KV workspace)", err);
    e->pairs = pairs;
  }
  float* base = static_cast<float*>(e->base);
  out.o = base;
  out.ml = base + o_floats;
  out.count = reinterpret_cast<int*>(base + o_floats + ml_floats);
  cudaError_t err = cudaMemsetAsync(out.count, 0, static_cast<size_t>(pairs) * 4, stream);
  if (err != cudaSuccess) return set_cuda_error("cudaMemsetAsync(split-KV counters)", err);
  return H3SA_OK;
}

template <bool kFp8, bool kParts>
static int launch_attention(const AttnLaunch& L, cudaStream_t stream) {
  using Cfg = AttnCfg<kFp8>;
  const CUtensorMapDataType dt =
      kFp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t box_inner = 128 / Cfg::kElem;  // one 128-byte swizzle atom of d
  CUtensorMap tmQ, tmK, tmV;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(L.heads),
                              static_cast<uint64_t>(L.rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim) * Cfg::kElem,
                                 static_cast<uint64_t>(L.heads) * kHeadDim * Cfg::kElem};
    const uint32_t box[3] = {box_inner, 1, static_cast<uint32_t>(kBlockM)};
    int rc = encode_tiled_3d(&tmQ, dt, L.query, dims, strides, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim),
                              static_cast<uint64_t>(L.pool_pages) * kBlockN,
                              static_cast<uint64_t>(L.heads)};
    const uint64_t strides[2] = {
        static_cast<uint64_t>(kHeadDim) * Cfg::kElem,
        static_cast<uint64_t>(L.pool_pages) * kBlockN * kHeadDim * Cfg::kElem};
    const uint32_t box[3] = {box_inner, static_cast<uint32_t>(kBlockN), 1};
    int rc = encode_tiled_3d(&tmK, dt, L.key_pool, dims, strides, box);
    if (rc) return rc;
    rc = encode_tiled_3d(&tmV, dt, L.value_pool, dims, strides, box);
    if (rc) return rc;
  }
  AttnParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.out = L.out;
  prm.rows = L.rows;
  prm.heads = L.heads;
  prm.page_table = L.page_table;
  prm.table_blocks = L.table_blocks;
  prm.pool_pages = L.pool_pages;
  prm.scale_log2 = L.softmax_scale * 1.4426950408889634f;
  prm.softmax_scale_log2 = prm.scale_log2;
  prm.q_scale = L.q_scale;
  prm.k_scale = L.k_scale;
  prm.v_scale = L.v_scale;
  prm.block_part = L.block_part;
  prm.part_k_scale = L.part_k_scale;
  prm.part_v_scale = L.part_v_scale;
  prm.n_parts = L.n_parts;
  prm.kv_num_blocks = L.kv_num_blocks;
  prm.kv_indices = L.kv_indices;
  prm.q_blocks = L.q_blocks;
  prm.kv_stride = L.kv_stride;
  prm.err = L.device_error;
  prm.out_peers = L.out_peers;
  prm.out_ranks = L.out_ranks;
  prm.out_rows_per_rank = L.out_rows_per_rank;
  prm.out_heads = L.out_heads;
  prm.out_head0 = L.out_head0;
  // Launches with a block-sparse problem run the one-tile kernel: each CTA walks its own
  // tile's list (no union of two lists) and the small CTAs balance uneven lists. Dense launches
  // run the two-tile kernel, whose two tiles' softmax phases interleave on each SM.
  bool one_tile = H3SA_ONE_TILE_DENSE != 0;
  for (int i = 0; i < L.num_problems; ++i)
    one_tile = one_tile || (L.problems[i].sparse && L.problems[i].q_hi > L.problems[i].q_lo);
  int ctas = 0;
  int n = 0;
  int split_pairs = 0;
  for (int i = 0; i < L.num_problems; ++i) {
    const auto& src = L.problems[i];
    if (src.q_hi <= src.q_lo) continue;
    AttnProblemDev& d = prm.prob[n++];
    d.q_lo = src.q_lo;
    d.q_hi = src.q_hi;
    d.kv_lo = src.kv_lo;
    d.kv_hi = src.kv_hi;
    d.sparse = src.sparse ? 1 : 0;
    d.tiles = (src.q_hi - src.q_lo + kBlockM - 1) / kBlockM;
    // work units of one CTA: pairs of query tiles, or single tiles for the one-tile kernel
    d.pairs = one_tile ? d.tiles : (d.tiles + 1) / 2;
    // block-sparse lists are uneven (rows that keep every block next to rows that keep a
    // quarter): those pairs get kSplitMax CTAs and decide on the device how many to use
    const int nblocks = (src.kv_hi + kBlockN - 1) / kBlockN - src.kv_lo / kBlockN;
    d.split = (d.sparse && nblocks > kSplitSegBlocks) ? kSplitMax : 1;
    d.pair_begin = split_pairs;
    if (d.split > 1) split_pairs += d.pairs * L.heads;
    d.cta_begin = ctas;
    ctas += d.pairs * L.heads * d.split;
  }
  prm.n_prob = n;
  if (ctas == 0) return H3SA_OK;
  std::unique_lock<std::mutex> ws_lock(g_split_mu, std::defer_lock);
  if (split_pairs > 0) {
    ws_lock.lock();  // held until the launch below is enqueued
    SplitSpace ws;
    int rc = split_workspace(split_pairs, stream, ws);
    if (rc) return rc;
    prm.split_o = ws.o;
    prm.split_ml = ws.ml;
    prm.split_count = ws.count;
  }
  const size_t smem = one_tile ? attn1_smem_bytes<kFp8>() : attn_smem_bytes<kFp8>();
  const auto kernel = one_tile ? attn1_fwd_kernel<kFp8, H3SA_ONE_TILE_INDEP != 0, kParts>
                               : attn_fwd_kernel<kFp8, kParts>;
  // per kernel (two-tile / one-tile) and device: the shared-memory attribute is set once, and
  // setmaxnreg.inc waits until the registers it asks for are free in the block's launch
  // allocation, so a build whose register count cannot fund the split is refused
  static std::mutex mu;
  static bool configured[2][64] = {};
  static bool checked[2] = {};
  const int which = one_tile ? 1 : 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && !configured[which][dev]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute", e);
      configured[which][dev] = true;
    }
    if (!checked[which]) {
      cudaFuncAttributes attr;
      cudaError_t e = cudaFuncGetAttributes(&attr, kernel);
      if (e != cudaSuccess) return set_cuda_error("cudaFuncGetAttributes", e);
      if (attr.numRegs * kAttnThreads < kRegSplitTotal)
        return set_error(H3SA_ERR_UNSUPPORTED, "attention build has %d registers per thread; the "
                         "warp-role register split needs %d", attr.numRegs,
                         (kRegSplitTotal + kAttnThreads - 1) / kAttnThreads);
      checked[which] = true;
    }
  }
  kernel<<<ctas, kAttnThreads, smem, stream>>>(tmQ, tmK, tmV, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("attn_fwd_kernel launch", e);
  return H3SA_OK;
}

int attention_launch(const AttnLaunch& L, bool fp8, cudaStream_t stream) {
  if (!fp8) return launch_attention<false, false>(L, stream);
  return L.block_part ? launch_attention<true, true>(L, stream)
                      : launch_attention<true, false>(L, stream);
}

#ifdef H3SA_TRACE
extern "C" H3SA_API int h3sa_trace_copy(void* host, size_t bytes) {
  if (bytes > sizeof(g_h3sa_trace)) bytes = sizeof(g_h3sa_trace);
  return cudaMemcpyFromSymbol(host, g_h3sa_trace, bytes) == cudaSuccess ? 0 : 3;
}
#endif

size_t attention_smem_bytes(bool fp8) {
  return fp8 ? attn_smem_bytes<true>() : attn_smem_bytes<false>();
}

}  // namespace h3sa
