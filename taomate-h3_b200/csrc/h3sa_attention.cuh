// Streaming chunk attention for sm_100a: O = softmax(Q K^T * scale) V, non-causal, d = 128.
//
// One CTA owns two 128-row query tiles of one head and walks a list of 128-row KV blocks
// taken from a paged, head-major KV pool (page p of head h = rows [128p, 128p+128) of
// that head's plane). Warp roles:
//   warp 0      TMA producer: Q tiles once, then K and V blocks through 2-stage rings.
//   warp 1      TMEM owner and MMA issuer (one thread): S_t = Q_t K^T (smem x smem),
//               O_t += P_t V (P from TMEM x V from smem), fp32 accumulators in TMEM.
//   warps 2-3   idle (warp 2 builds the block-sparse union list before the roles start)
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1 (one thread per query row;
//               warp w reads TMEM lanes 32*(w%4) .. +31):
//               online max / sum, lazy O rescale, P written back to TMEM as bf16, and the
//               final normalise + bf16 store.
// TMEM columns: S0 [0,128) with P0 aliased at [64,128), S1 [128,256) with P1 at
// [192,256), O0 [256,384), O1 [384,512).
//
// The MMA issue order per KV block i is PV_t(i-1) then QK_t(i) for each tile t. The QK
// that overwrites S_t (and so P_t) is issued after the PV that reads P_t; tcgen05.mma
// operations issued by one thread execute in issue order, which orders the two.
#pragma once

#include "h3sa_ptx.cuh"

namespace h3sa {

constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kKVStages = 2;
constexpr int kAttnThreads = 384;
// setmaxnreg split: warps 0-3 (producer, MMA, two idle) keep kRegsControl registers, the two
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

struct AttnProblemDev {
  int q_lo, q_hi;    // query / output rows [q_lo, q_hi) of the packed [rows, heads, d] tensors
  int kv_lo, kv_hi;  // logical KV rows [kv_lo, kv_hi) of the page sequence
  int sparse;        // 1: walk the per-(head, q-block) block lists instead of every block
  int cta_begin;     // first CTA of this problem in the flattened grid
  int tiles;         // ceil((q_hi - q_lo) / 128)
  int pairs;         // ceil(tiles / 2)
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
  // block-sparse lists in the flex BlockMask layout, used by problems with sparse = 1
  const int* kv_num_blocks;  // [heads, q_blocks]
  const int* kv_indices;     // [heads, q_blocks, kv_stride]
  int q_blocks;
  int kv_stride;
  int* err;                  // device error word (nullable)
  // output rows scattered to peers (see AttnLaunch in h3sa_host.h); null: write `out`
  const uint64_t* out_peers;
  int out_ranks;
  int out_rows_per_rank;
  int out_heads;
  int out_head0;
};

}  // namespace h3sa
