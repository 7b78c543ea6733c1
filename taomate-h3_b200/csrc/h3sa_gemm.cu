// W8A8 projection GEMM on the sm_100a tensor cores: out[M, N] (bf16) =
//   a_scale[m] * (b_scale[n] * float(sum_k A[m, k] * B[n, k]))
// with A int8 [M, K] (activations, one scale per token row) and B int8 [N, K] (weights, one
// scale per output row), both K-major. This is the arithmetic of the reference's QKV / FC1
// projection (T/inference/w8a8.py:190-221: dynamic per-token int8 activations, per-row int8
// weights, CUTLASS scaled_mm into bf16), written for tcgen05:
//
// * persistent CTAs, one per SM, walking 128 x 256 output tiles;
// * warp 0 streams A and B K-slices (128 bytes of K per row, 128-byte swizzle) by TMA into a
//   4-stage shared-memory ring (3 for bf16);
// * warp 1 issues tcgen05.mma kind::i8 (M 128, N 256, K 32 per instruction) into one of two
//   TMEM accumulators (2 x 256 int32 columns), so the epilogue of one tile overlaps the MMAs
//   of the next;
// * warps 2-5 (one per TMEM lane quadrant) read the int32 accumulators, scale them in the
//   order above and store bf16 rows (the bf16 form stages its 32 rows in shared memory and
//   stores whole 512-byte row segments: full-size packets over NVLink for peer stores).
//
// The same kernel in bf16 (tcgen05 kind::f16, fp32 accumulation) is the row-parallel out_proj
// of the attention (T/model/layers.py:441-443, T/distributed/linear.py:142-198): its epilogue
// can store this TP rank's bf16 partial output straight into slot `rank` of every TP rank's
// partial buffer over NVLink, after which a peer barrier and h3sa_tp_reduce (the slots summed
// in rank order) replace the TP all-reduce.
//
// Every wait is bounded (h3sa_ptx.cuh); a wait that gives up records kErrWaitTimeout in the
// error word and the CTA unwinds.
#include "h3sa_host.h"
#include "h3sa_ptx.cuh"

#include <mutex>

namespace h3sa {
namespace {

constexpr int kGemmBM = 128;
constexpr int kGemmBN = 256;  // 32 16-byte chunks per row: one per lane in the row stores
constexpr int kGemmBK = 128;  // bytes of K per stage (one 128-byte swizzle atom)
constexpr int kGemmThreads = 192;
constexpr int kGemmUmmaK = 32;  // int8 K per tcgen05.mma
constexpr uint32_t kGemmATile = kGemmBM * kGemmBK;  // 16 KB
constexpr uint32_t kGemmBTile = kGemmBN * kGemmBK;  // 32 KB

// int8: 4 stages, each thread stores its own row segments. bf16: 3 stages and a staging area
// through which the epilogue stores whole rows (the peer stores of the fused TP reduce need
// full-size NVLink packets; 4 stages and the staging do not fit together).
template <bool kBf16>
struct GemmCfg {
  static constexpr int kStages = kBf16 ? 3 : 4;
  static constexpr int kStageWarps = kBf16 ? 4 : 1;
  static constexpr int kStageRows = kBf16 ? 32 : 1;
};

template <bool kBf16>
struct GemmSmem {
  using Cfg = GemmCfg<kBf16>;
  uint8_t a[Cfg::kStages][kGemmATile];  // 1024-byte aligned (tile sizes are multiples)
  uint8_t b[Cfg::kStages][kGemmBTile];
  // bf16, per epilogue warp: its 32 rows x kGemmBN bf16 of the tile, 16-byte chunk j of row
  // r at chunk position j ^ r (conflict-free row-wise writes and lane-wise reads)
  uint4 stage[Cfg::kStageWarps][Cfg::kStageRows][kGemmBN / 8];
  float b_scale[2][kGemmBN];
  uint64_t full[Cfg::kStages];
  uint64_t empty[Cfg::kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <bool kBf16>
constexpr size_t gemm_smem_bytes() { return sizeof(GemmSmem<kBf16>) + 1024; }
static_assert(gemm_smem_bytes<false>() <= 232448, "int8 GEMM needs more than 227 KB of smem");
static_assert(gemm_smem_bytes<true>() <= 232448, "bf16 GEMM needs more than 227 KB of smem");

struct GemmParams {
  const float* a_scale;  // [M] (int8 only)
  const float* b_scale;  // [N] (int8 only)
  __nv_bfloat16* out;    // [M, ldo] or null
  const uint64_t* out_peers;  // bf16 only: partial buffers [ranks][M][ldo] of every TP rank
  int out_ranks, out_slot;
  int m, n, k;  // k in elements
  int ldo;
  int tiles_n, tiles;
  int* err;
};

// kind::i8, int32 accumulation, signed A and B, both K-major.
constexpr uint32_t idesc_s8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t" H3SA_ELECT_PRED
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// kBf16: bf16 operands (kind::f16, fp32 accumulators, no scales); else int8 (kind::i8).
template <bool kBf16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmParams p) {
  constexpr int kElemK = kBf16 ? kGemmBK / 2 : kGemmBK;  // K elements per stage
  constexpr int kGemmStages = GemmCfg<kBf16>::kStages;
  extern __shared__ uint8_t smem_raw[];
  GemmSmem<kBf16>& sm = *reinterpret_cast<GemmSmem<kBf16>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const int k_steps = (p.k + kElemK - 1) / kElemK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sm.acc_full[b]), 1);
      mbar_init(smem_u32(&sm.acc_empty[b]), 4);  // one arrival per epilogue warp
    }
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile / p.tiles_n) * kGemmBM;
        const int n0 = (tile % p.tiles_n) * kGemmBN;
        for (int ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % kGemmStages;
          if (!mbar_wait(smem_u32(&sm.empty[s]), ((it / kGemmStages) & 1) ^ 1, abort_flag, p.err))
            break;
          const uint32_t full = smem_u32(&sm.full[s]);
          mbar_expect_tx(full, kGemmATile + kGemmBTile);
          tma_load_3d(smem_u32(sm.a[s]), &tmA, full, ks * kElemK, m0, 0);
          tma_load_3d(smem_u32(sm.b[s]), &tmB, full, ks * kElemK, n0, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp)
    constexpr uint32_t idesc = kBf16 ? idesc_bf16(kGemmBM, kGemmBN, false)
                                     : idesc_s8(kGemmBM, kGemmBN);
    uint32_t it = 0;
    int j = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++j) {
      const int buf = j & 1;
      if (!mbar_wait(smem_u32(&sm.acc_empty[buf]), ((j >> 1) & 1) ^ 1, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t d_tmem = tbase + static_cast<uint32_t>(buf * kGemmBN);
      bool ok = true;
      for (int ks = 0; ks < k_steps; ++ks, ++it) {
        const int s = it % kGemmStages;
        if (!(ok = mbar_wait(smem_u32(&sm.full[s]), (it / kGemmStages) & 1, abort_flag, p.err)))
          break;
        tc_fence_after();
        const uint32_t a_lo = sdesc_lo(smem_u32(sm.a[s]), 16);
        const uint32_t b_lo = sdesc_lo(smem_u32(sm.b[s]), 16);
#pragma unroll
        for (int kk = 0; kk < kGemmBK / kGemmUmmaK; ++kk) {
          // K advance inside the swizzle atom: 32 bytes = 2 in the address field
          if constexpr (kBf16)
            mma_ss(d_tmem, sdesc_join(a_lo + 2 * kk), sdesc_join(b_lo + 2 * kk), idesc,
                   (ks | kk) != 0);
          else
            mma_ss_i8(d_tmem, sdesc_join(a_lo + 2 * kk), sdesc_join(b_lo + 2 * kk), idesc,
                      (ks | kk) != 0);
        }
        tc_commit(smem_u32(&sm.empty[s]));  // the stage is free once these MMAs completed
      }
      if (!ok) break;
      tc_commit(smem_u32(&sm.acc_full[buf]));
    }
  } else {
    // ------------------------------------------------------------ epilogue warps 2..5
    const int quad = warp & 3;  // TMEM lanes 32 * quad .. 32 * quad + 31
    const int ep_thread = threadIdx.x - 64;  // 0..127
    int j = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++j) {
      const int buf = j & 1;
      const int m0 = (tile / p.tiles_n) * kGemmBM;
      const int n0 = (tile % p.tiles_n) * kGemmBN;
      if constexpr (!kBf16) {
        // this tile's column scales into shared memory (the previous tile of this buffer is
        // done: every epilogue warp passed the previous tile's barrier)
        for (int c = ep_thread; c < kGemmBN; c += 128)
          sm.b_scale[buf][c] = n0 + c < p.n ? __ldg(p.b_scale + n0 + c) : 0.f;
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      if (!mbar_wait(smem_u32(&sm.acc_full[buf]), (j >> 1) & 1, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = m0 + quad * 32 + lane;
      const float a_s = (!kBf16 && row < p.m) ? __ldg(p.a_scale + row) : 0.f;
      const uint32_t t_row = tbase + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(buf * kGemmBN);
      if constexpr (kBf16) {
        uint4 (*stage)[kGemmBN / 8] = sm.stage[quad];
#pragma unroll 1
        for (int c = 0; c < kGemmBN; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_row + c, r);
          tmem_wait_ld();
          reg_fence32(r);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = pack_bf16x2(__uint_as_float(r[8 * q + 2 * i]),
                                 __uint_as_float(r[8 * q + 2 * i + 1]));
            stage[lane][(c / 8 + q) ^ lane] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        // the accumulator is in shared memory: the MMAs of tile j + 2 may reuse it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.acc_empty[buf]));
        // rows out, a warp per row: lane l carries 16-byte chunk l
        const size_t slot_off =
            static_cast<size_t>(p.out_slot) * p.m * p.ldo * sizeof(__nv_bfloat16);
        const int chunks = min(kGemmBN, p.n - n0) / 8;  // n is a multiple of 8
        for (int rr = 0; rr < 32; ++rr) {
          const int grow = m0 + quad * 32 + rr;
          if (grow >= p.m) break;
          if (lane < chunks) {
            const uint4 v = stage[rr][lane ^ rr];
            const size_t coff = (static_cast<size_t>(grow) * p.ldo + n0) * sizeof(__nv_bfloat16) +
                                static_cast<size_t>(lane) * 16;
            if (p.out) *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + coff) = v;
            // this rank's partial into its slot of every TP rank's buffer (peer stores)
            for (int t = 0; t < p.out_ranks; ++t)
              *reinterpret_cast<uint4*>(p.out_peers[t] + slot_off + coff) = v;
          }
        }
        __syncwarp();  // the staging rows are read before the next tile overwrites them
      } else {
        __nv_bfloat16* orow = p.out + static_cast<size_t>(row) * p.ldo + n0;
#pragma unroll 1
        for (int c = 0; c < kGemmBN; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_row + c, r);
          tmem_wait_ld();
          reg_fence32(r);
          if (row < p.m && n0 + c < p.n) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float x0 = __fmul_rn(a_s, __fmul_rn(sm.b_scale[buf][c + 2 * i],
                                                        __int2float_rn(static_cast<int>(r[2 * i]))));
              const float x1 = __fmul_rn(
                  a_s, __fmul_rn(sm.b_scale[buf][c + 2 * i + 1],
                                 __int2float_rn(static_cast<int>(r[2 * i + 1]))));
              w[i] = pack_bf16x2(x0, x1);
            }
            // ragged last columns go by 8-column groups (n is a multiple of 8)
            const int groups = n0 + c + 32 <= p.n ? 4 : (p.n - n0 - c) / 8;
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (q < groups) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.acc_empty[buf]));
      }
    }
    // the peer stores are visible to the other GPUs before the barrier that follows
    if (kBf16 && p.out_ranks > 1) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// Per-row int8 quantisation of bf16 rows [rows, cols], one CTA per row:
// mode 0, the activations (dynamic per-token, as vLLM's dynamic_scaled_int8_quant):
//   scale = amax / 127, q = clamp(rint(x * (127 / amax)), -128, 127); an all-zero row gives
//   scale 0 and zeros;
// mode 1, the weights (T/inference/w8a8.py:56-63):
//   scale = max(amax / 127, 1e-12), q = clamp(rint(x / scale), -127, 127).
// rint rounds half to even in both.
constexpr int kQuantRowThreads = 256;
constexpr int kQuantRowCached = 4;  // 16-byte chunks a thread keeps in registers (8192 columns)

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float chunk_amax(const uint4& v, float m) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) m = fmaxf(m, fmaxf(fabsf(bf16_lo(w[i])), fabsf(bf16_hi(w[i]))));
  return m;
}

__device__ __forceinline__ uint2 chunk_quant(const uint4& v, int mode, float sc, float mul,
                                             float lo) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float f = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
    const float t = mode == 0 ? __fmul_rn(f, mul) : __fdiv_rn(f, sc);
    const float r = fminf(fmaxf(rintf(t), lo), 127.f);
    packed[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu) << (8 * (i & 3));
  }
  return make_uint2(packed[0], packed[1]);
}

// Rows of up to kQuantRowThreads * kQuantRowCached * 8 columns are read once (kept in
// registers between the amax and the quantisation); longer rows are read twice.
__global__ void __launch_bounds__(kQuantRowThreads) quantize_int8_rows_kernel(
    const __nv_bfloat16* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
    int cols, int mode) {
  const size_t row = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(x + row * cols);
  const int chunks = cols / 8;
  uint4 cache[kQuantRowCached];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kQuantRowCached; ++i) {
    const int c = threadIdx.x + i * kQuantRowThreads;
    cache[i] = c < chunks ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
    m = chunk_amax(cache[i], m);
  }
  for (int c = threadIdx.x + kQuantRowCached * kQuantRowThreads; c < chunks; c += kQuantRowThreads)
    m = chunk_amax(__ldg(src + c), m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[kQuantRowThreads / 32];
  __shared__ float row_scale, row_mul;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float amax = red[0];
    for (int i = 1; i < kQuantRowThreads / 32; ++i) amax = fmaxf(amax, red[i]);
    if (mode == 0) {
      row_scale = __fdiv_rn(amax, 127.f);
      row_mul = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    } else {
      row_scale = fmaxf(__fdiv_rn(amax, 127.f), 1.0e-12f);
      row_mul = 0.f;
    }
    scale[row] = row_scale;
  }
  __syncthreads();
  const float sc = row_scale, mul = row_mul;
  const float lo = mode == 0 ? -128.f : -127.f;
  uint2* dst = reinterpret_cast<uint2*>(q + row * cols);
#pragma unroll
  for (int i = 0; i < kQuantRowCached; ++i) {
    const int c = threadIdx.x + i * kQuantRowThreads;
    if (c < chunks) dst[c] = chunk_quant(cache[i], mode, sc, mul, lo);
  }
  for (int c = threadIdx.x + kQuantRowCached * kQuantRowThreads; c < chunks; c += kQuantRowThreads)
    dst[c] = chunk_quant(__ldg(src + c), mode, sc, mul, lo);
}

}  // namespace
}  // namespace h3sa

namespace h3sa {
namespace {

// A and B row-major with K contiguous, K a multiple of 16 bytes; tcgen05 kind per kBf16.
template <bool kBf16>
int launch_gemm(const void* a, const void* b, GemmParams prm, cudaStream_t stream) {
  const CUtensorMapDataType dt =
      kBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const uint64_t esize = kBf16 ? 2 : 1;
  const uint32_t box_k = kBf16 ? kGemmBK / 2 : kGemmBK;
  const uint64_t m = prm.m, n = prm.n, k = prm.k;
  CUtensorMap tmA, tmB;
  {
    const uint64_t dims[3] = {k, m, 1};
    const uint64_t strides[2] = {k * esize, k * esize * m};
    const uint32_t box[3] = {box_k, kGemmBM, 1};
    int rc = encode_tiled_3d(&tmA, dt, a, dims, strides, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {k, n, 1};
    const uint64_t strides[2] = {k * esize, k * esize * n};
    const uint32_t box[3] = {box_k, kGemmBN, 1};
    int rc = encode_tiled_3d(&tmB, dt, b, dims, strides, box);
    if (rc) return rc;
  }
  prm.tiles_n = (prm.n + kGemmBN - 1) / kGemmBN;
  prm.tiles = prm.tiles_n * ((prm.m + kGemmBM - 1) / kGemmBM);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static std::mutex mu;
  static bool configured[64] = {};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemm_kernel<kBf16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(gemm_smem_bytes<kBf16>()));
      if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(gemm)", e);
      configured[dev] = true;
    }
  }
  const int grid = prm.tiles < sms ? prm.tiles : sms;
  gemm_kernel<kBf16><<<grid, kGemmThreads, gemm_smem_bytes<kBf16>(), stream>>>(tmA, tmB, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("gemm_kernel launch", e);
  return H3SA_OK;
}

// out[i] = bf16(sum over t of float(slots[t][i])) in rank order t = 0, 1, ...
__global__ void __launch_bounds__(256) tp_reduce_kernel(const __nv_bfloat16* __restrict__ slots,
                                                        __nv_bfloat16* __restrict__ out, int m,
                                                        int n, int ldo, int ranks) {
  const int cpr = n / 8;  // 16-byte chunks per row
  const long long total = static_cast<long long>(m) * cpr;
  const size_t slot = static_cast<size_t>(m) * ldo;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(idx / cpr);
    const int c = static_cast<int>(idx - static_cast<long long>(row) * cpr);
    const size_t off = static_cast<size_t>(row) * ldo + static_cast<size_t>(c) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int t = 0; t < ranks; ++t) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(slots + t * slot + off));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(w[i] << 16);
        acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + off) = o;
  }
}

int check_gemm_args(const void* a, const void* b, const void* out, int32_t m, int32_t n,
                    int32_t k_bytes, int32_t ldo, const char* name) {
  if (!a || !b) return set_error(H3SA_ERR_INVALID, "%s: null operand", name);
  if (m < 0 || n <= 0 || k_bytes <= 0 || (k_bytes % 16) || (n % 8) || ldo < n || (ldo % 8))
    return set_error(H3SA_ERR_INVALID, "%s: m=%d n=%d k bytes=%d ldo=%d (k bytes must be a "
                     "multiple of 16, n and ldo of 8)", name, m, n, k_bytes, ldo);
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(H3SA_ERR_INVALID, "%s: operands must be 16-byte aligned", name);
  return H3SA_OK;
}

}  // namespace
}  // namespace h3sa

using namespace h3sa;

extern "C" {

int h3sa_w8a8_gemm(const void* a, const float* a_scale, const void* b, const float* b_scale,
                   void* out, int32_t m, int32_t n, int32_t k, int32_t ldo, int32_t* device_error,
                   void* stream) {
  if (!a_scale || !b_scale || !out) return set_error(H3SA_ERR_INVALID, "w8a8_gemm: null operand");
  int rc = check_gemm_args(a, b, out, m, n, k, ldo, "w8a8_gemm");
  if (rc) return rc;
  if (m == 0) return H3SA_OK;
  GemmParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.a_scale = a_scale;
  prm.b_scale = b_scale;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.m = m;
  prm.n = n;
  prm.k = k;
  prm.ldo = ldo;
  prm.err = device_error;
  return launch_gemm<false>(a, b, prm, static_cast<cudaStream_t>(stream));
}

int h3sa_gemm_bf16(const void* a, const void* b, void* out, int32_t m, int32_t n, int32_t k,
                   int32_t ldo, const uint64_t* partial_peers, int32_t ranks, int32_t slot,
                   int32_t* device_error, void* stream) {
  if (!out && !partial_peers) return set_error(H3SA_ERR_INVALID, "gemm_bf16: no destination");
  if (partial_peers && (ranks < 1 || slot < 0 || slot >= ranks))
    return set_error(H3SA_ERR_INVALID, "gemm_bf16: slot %d of %d ranks", slot, ranks);
  int rc = check_gemm_args(a, b, out, m, n, 2 * k, ldo, "gemm_bf16");
  if (rc) return rc;
  if (m == 0) return H3SA_OK;
  GemmParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_peers = partial_peers;
  prm.out_ranks = partial_peers ? ranks : 0;
  prm.out_slot = slot;
  prm.m = m;
  prm.n = n;
  prm.k = k;
  prm.ldo = ldo;
  prm.err = device_error;
  return launch_gemm<true>(a, b, prm, static_cast<cudaStream_t>(stream));
}

int h3sa_tp_reduce(const void* slots, void* out, int32_t m, int32_t n, int32_t ldo, int32_t ranks,
                   void* stream) {
  if (!slots || !out || m < 0 || n <= 0 || (n % 8) || ldo < n || (ldo % 8) || ranks < 1)
    return set_error(H3SA_ERR_INVALID, "tp_reduce: m=%d n=%d ldo=%d ranks=%d", m, n, ldo, ranks);
  if ((reinterpret_cast<uintptr_t>(slots) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(H3SA_ERR_INVALID, "tp_reduce: tensors must be 16-byte aligned");
  if (m == 0) return H3SA_OK;
  const long long work = static_cast<long long>(m) * (n / 8);
  long long g = (work + 255) / 256;
  if (g > 148LL * 16) g = 148LL * 16;
  tp_reduce_kernel<<<static_cast<int>(g), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(slots), static_cast<__nv_bfloat16*>(out), m, n, ldo, ranks);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("tp_reduce_kernel launch", e);
  return H3SA_OK;
}

int h3sa_quantize_int8_rows(const void* x, void* q, float* scale, int32_t rows, int32_t cols,
                            int32_t mode, void* stream) {
  if (!x || !q || !scale || rows < 0 || cols <= 0 || (cols % 8) || (mode != 0 && mode != 1))
    return set_error(H3SA_ERR_INVALID, "quantize_int8_rows: rows=%d cols=%d mode=%d (cols must "
                     "be a multiple of 8, mode 0 or 1)", rows, cols, mode);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 7))
    return set_error(H3SA_ERR_INVALID, "quantize_int8_rows: unaligned tensors");
  if (rows == 0) return H3SA_OK;
  quantize_int8_rows_kernel<<<rows, kQuantRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<int8_t*>(q), scale, cols, mode);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("quantize_int8_rows launch", e);
  return H3SA_OK;
}

}  // extern "C"
