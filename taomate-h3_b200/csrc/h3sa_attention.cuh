// Streaming chunk attention for sm_100a: O = softmax(Q K^T * scale) V, non-causal, d = 128.
//
// One CTA owns two 128-row query tiles of one head and walks a list of 128-row KV blocks
// taken from a paged, head-major KV pool (page p of head h = rows [128p, 128p+128) of
// that head's plane). Warp roles:
//   warp 0      TMA producer of the Q tiles (once) and of K blocks (2-stage ring).
//   warp 3      TMA producer of V blocks (1 stage for bf16, 2 for e4m3).
//   warp 1, 2   MMA issuers of query tile 0 and tile 1 (warp 1 also owns TMEM), converged
//               warps with one elected lane per tcgen05 instruction:
//               S_t = Q_t K^T (smem x smem) and O_t += P_t V (smem x smem), fp32 in TMEM.
//               Warp 2 builds the block-sparse bitmaps before the roles start.
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1 (one thread per query row;
//               warp w reads TMEM lanes 32*(w%4) .. +31): online max / sum, lazy O rescale,
//               P written to shared memory in the MMA operand layout, and the final
//               normalise + bf16 store.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512). Shared memory: Q0, Q1,
// P0, P1, the K ring and the V ring.
//
// The MMA warp of tile t issues QK_t(i) once the softmax has loaded S_t(i-1) into registers
// (s_free) and PV_t(i-1) once it has written P_t(i-1) (p_full), so QK_t(i) runs while the
// softmax of block i-1 computes its exponentials. The softmax writes P_t(i) only after
// PV_t(i-1) has completed (pv_done), and rescales O_t at that point when its row maximum grew.
//
// Launches with a block-sparse problem use attn1_fwd_kernel instead: one query tile per CTA,
// S double-buffered in TMEM, and the two column halves of each row as independent online
// softmaxes with one O accumulator each (see h3sa_attention.cu).
#pragma once

#include "h3sa_ptx.cuh"

namespace h3sa {

constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kAttnThreads = 384;
// setmaxnreg split: warps 0-3 (producers and MMA issuers) keep kRegsControl registers, the two
// softmax warpgroups get kRegsSoftmax. The sum must fit the launch allocation
// (threads x registers per thread at launch, 168 under these launch bounds).
#ifndef H3SA_REGS_CONTROL
#define H3SA_REGS_CONTROL 48
#endif
#ifndef H3SA_REGS_SOFTMAX
#define H3SA_REGS_SOFTMAX 224
#endif
constexpr int kRegsControl = H3SA_REGS_CONTROL;
constexpr int kRegsSoftmax = H3SA_REGS_SOFTMAX;
constexpr int kRegSplitTotal = 128 * kRegsControl + 256 * kRegsSoftmax;
constexpr int kMaxProblems = 4;
constexpr int kMaxUnionBlocks = 2048;
// Split-KV for block-sparse problems: up to kSplitMax CTAs per work unit (a query tile in the
// one-tile kernel, a query-tile pair with its union list in the two-tile kernel), one segment
// of at least kSplitSegBlocks blocks of the unit's list each.
#ifndef H3SA_SPLIT_SEG_BLOCKS
#define H3SA_SPLIT_SEG_BLOCKS 64
#endif
#ifndef H3SA_SPLIT_MAX
#define H3SA_SPLIT_MAX 4
#endif
constexpr int kSplitMax = H3SA_SPLIT_MAX;
constexpr int kSplitSegBlocks = H3SA_SPLIT_SEG_BLOCKS;

struct AttnProblemDev {
  int q_lo, q_hi;    // query / output rows [q_lo, q_hi) of the packed [rows, heads, d] tensors
  int kv_lo, kv_hi;  // logical KV rows [kv_lo, kv_hi) of the page sequence
  int sparse;        // 1: walk the per-(head, q-block) block lists instead of every block
  int cta_begin;     // first CTA of this problem in the flattened grid
  int tiles;         // ceil((q_hi - q_lo) / 128)
  int pairs;         // ceil(tiles / 2)
  int split;         // CTAs per pair (split-KV segments; 1 = no split)
  int pair_begin;    // index of this problem's first pair among the split problems' pairs
};

struct AttnParams {
  void* out;                 // [rows, heads, d] bf16
  int rows;
  int heads;
  const int* page_table;     // logical block -> physical page
  int table_blocks;          // entries in page_table
  int pool_pages;            // pages per head plane
  AttnProblemDev prob[kMaxProblems];
  int n_prob;
  float scale_log2;          // softmax_scale * log2(e) (bf16 path)
  // FP8 path: S scale = q_scale[h] * k_scale[h] * softmax_scale * log2(e), O scale = v_scale[h].
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  float softmax_scale_log2;
  // Segmented e4m3 KV (null: one K and one V scale per head): block_part[b] of logical KV
  // block b holds its part index (low 16 bits) and its valid rows (high 16 bits, 1..128; parts
  // start on block boundaries); part_k_scale / part_v_scale are [n_parts, heads].
  const int* block_part;
  const float* part_k_scale;
  const float* part_v_scale;
  int n_parts;
  // block-sparse lists in the flex BlockMask layout, used by problems with sparse = 1
  const int* kv_num_blocks;  // [heads, q_blocks]
  const int* kv_indices;     // [heads, q_blocks, kv_stride]
  int q_blocks;
  int kv_stride;
  int* err;                  // device error word (nullable)
  // split-KV workspace (problems with split > 1): per segment slot and tile, 128 rows of
  // unnormalised O [128] and (max, sum); one arrival counter per pair, zero at launch
  float* split_o;
  float* split_ml;
  int* split_count;
  // output rows scattered to peers (see AttnLaunch in h3sa_host.h); null: write `out`
  const uint64_t* out_peers;
  int out_ranks;
  int out_rows_per_rank;
  int out_heads;
  int out_head0;
};

// Segmented e4m3 KV, at block b of the walk (head `head`): the block's valid rows, and on
// entering another part (a few times a row; parts are contiguous runs of blocks and the walk
// ascends) the part's S scale in log2 units and its V scale. P stays unscaled; O is kept in
// units of the current part's V scale, so entering a part with another V scale sets
// vr = v_prev / v_new, by which the softmax rescales O (with a nonzero O: has_o), and
// v_moved. Warp-uniform: every lane of a warp walks the same block of the same head.
__device__ __forceinline__ void part_step(const AttnParams& p, int head, int b, float q_sl2,
                                          bool has_o, int& cur_part, int& rows, float& sl2,
                                          uint64_t& scale2, float& v_cur, float& vr,
                                          bool& v_moved) {
  const int e = __ldg(p.block_part + b);
  rows = e >> 16;
  const int part = e & 0xFFFF;
  if (part == cur_part) return;
  cur_part = part;
  sl2 = q_sl2 * __ldg(p.part_k_scale + part * p.heads + head);
  scale2 = f2_pack(sl2, sl2);
  const float vs = __ldg(p.part_v_scale + part * p.heads + head);
  if (vs == v_cur) return;
  if (has_o) {
    vr = __fdividef(v_cur, vs);
    v_moved = true;
  }
  v_cur = vs;
}

}  // namespace h3sa
