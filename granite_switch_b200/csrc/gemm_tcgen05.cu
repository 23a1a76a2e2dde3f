// Switched-LoRA GEMM family for sm_100a (tcgen05 + TMEM + TMA).
//
//   D[M, N] = X[M, K] . W[N, K]^T  (+ per-row LoRA expand)  -> fused epilogue
//
// The reference computes a projection as one cuBLAS GEMM against
// w_ext = [W; A_1; ...; A_n] followed by a Triton expand that adds
// x_ext[:, shrink cols] . B_a^T per row (reference:
// src/granite_switch/vllm/core/lora.py:540-594 and
// src/granite_switch/kernels/switch_lora_kernel.py:171-411). Here the expand is
// folded into the tensor-core mainloop instead: after the K blocks of X.W^T,
// the same TMEM accumulator receives, for every adapter present in the
// 128-row tile, the rank-r product S_a . B_a^T, where S is the row-masked
// shrink output (zero on rows routed to other adapters). The delta therefore
// never makes a global-memory round trip, and tiles whose rows are all base
// skip it through the per-tile adapter bitmask.
//
// Roles (192 threads): warp 0 issues TMA loads into a STAGES-deep shared
// memory ring, warp 1 owns the TMEM allocation and issues tcgen05.mma from
// one thread, warps 2..5 drain the fp32 accumulator with tcgen05.ld and run
// the epilogue (store / residual add / SwiGLU / adapter mask / fp32 logits).
// Every TMA load is a plain single-CTA copy from this GPU's memory, so the
// kernel is safe on every GPU count.
#include "common.cuh"
#include "gemm_common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cstdlib>

namespace gsb {

struct GemmLoraArgs {
  int enabled;            // 0: plain GEMM
  int rank_blocks;        // rank / 32
  int num_adapters;       // adapters in the packed B (kernel-local ids 1..NA)
  int s_ld_slices;        // number of slices in S (column groups of NA*rank)
  int slice_bounds[5];    // output-column starts of each slice, [num_slices+1]
  int num_slices;
  const uint64_t* tile_mask;  // per 128-row tile bitmask of adapters present (bit a-1), or null
};

struct GemmEpiArgs {
  void* out;
  int64_t ldo;              // elements
  const __nv_bfloat16* residual;
  int64_t ldr;
  float scale;
  const int32_t* row_adapter;  // kEpiMaskAdapter: kernel-local adapter id per row
  int mask_rank;               // kEpiMaskAdapter: rank (columns per adapter)
  int mask_num_adapters;
  const uint64_t* skip_mask;   // kEpiMaskAdapter: adapters present per 128-row tile; tiles
                               // whose columns belong only to absent adapters are skipped
};

// Grouped mode (mixture-of-experts): W is a stack [E, N, K] and every 128-row
// tile of X belongs to one expert (tile_expert[mt]; -1 = no rows, skipped).
struct GemmGroupArgs {
  const int32_t* tile_expert;  // null: plain GEMM
  // split-K (decode-sized GEMMs with too few output tiles to fill the GPU): each
  // output tile's K range is cut into `ksplit` equal parts computed by different
  // CTAs; part p stores its fp32 partial sum at ws + p * M * N, and
  // splitk_reduce_kernel adds the parts and applies the epilogue. The LoRA
  // expand blocks run with the last part.
  int ksplit;                  // 1: off
  float* ws;                   // [ksplit, M, N] fp32
};

// A shrink tile is skipped when none of the adapters owning its columns has a
// row in its 128-row tile: the expand never reads those columns for that tile.
template <int BN>
__device__ __forceinline__ bool shrink_tile_skipped(const GemmEpiArgs& epi, int mt, int n0) {
  if (epi.skip_mask == nullptr) return false;
  uint64_t need = 0;
  for (int c = 0; c < BN; c += epi.mask_rank)
    need |= 1ull << (((n0 + c) / epi.mask_rank) % epi.mask_num_adapters);
  return (epi.skip_mask[mt] & need) == 0;
}

template <int BN, int EPI>
__device__ __forceinline__ bool tile_skipped(const GemmEpiArgs& epi, const GemmGroupArgs& grp, int mt, int n0) {
  if (grp.tile_expert != nullptr && grp.tile_expert[mt] < 0) return true;
  return EPI == kEpiMaskAdapter && shrink_tile_skipped<BN>(epi, mt, n0);
}

// Shared memory of the staged epilogue: two 4 KB buffers (32 rows x 64 bf16,
// 128-byte swizzled) per epilogue warp.
constexpr int kEpiStageBytes = 4 * 2 * 4096;

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;     // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;     // BN * 128 B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int TMEM_COLS = 2 * BN;        // two accumulator buffers
  static constexpr int STAGING_OFF = STAGES * STAGE_BYTES;   // epilogue staging (1024-aligned)
  static constexpr int BAR_OFF = STAGING_OFF + kEpiStageBytes;
  static constexpr int SMEM_BYTES = BAR_OFF + 1024 /*align*/ + 256 /*barriers*/;
};

// Tile order: groups of 16 M-tiles, M fastest inside a group, so the CTAs that
// run at the same time share weight tiles (B) in L2 and touch a bounded slice
// of activations (A).
template <int GM = 16>
__device__ __forceinline__ void gemm_tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int group = t / (GM * n_tiles);
  const int first_m = group * GM;
  const int gm = min(GM, m_tiles - first_m);
  const int r = t - group * GM * n_tiles;
  mt = first_m + r % gm;
  nt = r / gm;
}

struct LoraTile {
  uint64_t amask;
  int s_base0, s_base1;
  int blocks;
};

// `m_tile` counts 128-row tiles; a CTA pair covers `span` of them (1 or 2)
// and runs the expand for the union of their adapters.
template <bool SPLIT>
__device__ __forceinline__ LoraTile lora_tile(const GemmLoraArgs& lora, int m_tile, int n0, int span = 1,
                                              int m_tiles128 = 0) {
  LoraTile lt{0, 0, 0, 0};
  if (!lora.enabled) return lt;
  if (lora.tile_mask) {
    lt.amask = lora.tile_mask[m_tile];
    if (span == 2 && m_tile + 1 < m_tiles128) lt.amask |= lora.tile_mask[m_tile + 1];
  } else {
    lt.amask = (lora.num_adapters >= 64) ? ~0ull : ((1ull << lora.num_adapters) - 1);
  }
  const int slice_cols = lora.num_adapters * lora.rank_blocks * 32;
  if (SPLIT) {
    lt.s_base1 = slice_cols;
  } else {
    int s = 0;
    for (int i = 0; i < lora.num_slices; ++i)
      if (n0 >= lora.slice_bounds[i]) s = i;
    lt.s_base0 = s * slice_cols;
  }
  lt.blocks = __popcll(lt.amask) * lora.rank_blocks;
  return lt;
}

// Drains one 128 x BN fp32 accumulator from TMEM and applies the epilogue.
// Called by each of the four epilogue warps: the warp reads TMEM lanes
// [32q, 32q + 32) (`tbase` already points there) and thread `lane` owns output
// row `row`; columns n0 .. n0 + BN - 1.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmEpiArgs& epi, uint32_t tbase, int row, int M, int n0) {
  if (EPI == kEpiSwiGLU) {
    for (int c = 0; c < BN / 2; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld32(tbase + c, g);
      tmem_ld32(tbase + BN / 2 + c, u);
      tmem_wait_ld();
      if (row < M) {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(epi.out) + (int64_t)row * epi.ldo + (n0 / 2) + c;
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          // gate/up pre-activations are rounded to bf16 first, as the
          // unfused path stores them in bf16 before the activation
          const float g0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j])));
          const float g1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j + 1])));
          const float u0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j])));
          const float u1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j + 1])));
          pk[j] = pack_bf16x2(__fdividef(g0, 1.f + __expf(-g0)) * u0, __fdividef(g1, 1.f + __expf(-g1)) * u1);
        }
        uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
        for (int j = 0; j < 4; ++j) o4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
      }
    }
  } else {
    int radapter = 0;
    if (EPI == kEpiMaskAdapter && row < M) radapter = epi.row_adapter[row];
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(tbase + c, r);
      tmem_wait_ld();
      if (row >= M) continue;
      const int col = n0 + c;
      if (EPI == kEpiF32) {
        float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(epi.out) + (int64_t)row * epi.ldo + col);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          o4[j] = make_float4(__uint_as_float(r[4 * j]) * epi.scale, __uint_as_float(r[4 * j + 1]) * epi.scale,
                              __uint_as_float(r[4 * j + 2]) * epi.scale, __uint_as_float(r[4 * j + 3]) * epi.scale);
      } else {
        float v[32];
        if (EPI == kEpiResAdd || (EPI == kEpiMultimemRed && epi.residual != nullptr)) {
          const uint4* r4 = reinterpret_cast<const uint4*>(epi.residual + (int64_t)row * epi.ldr + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 w = r4[j];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
              // the projection is rounded to bf16 before the residual add, as
              // the unfused path materialises it in bf16
              const float2 f = unpack_bf16x2(ww[tt]);
              const float p0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * j + 2 * tt])));
              const float p1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * j + 2 * tt + 1])));
              v[8 * j + 2 * tt] = f.x + p0 * epi.scale;
              v[8 * j + 2 * tt + 1] = f.y + p1 * epi.scale;
            }
          }
        } else if (EPI == kEpiMultimemRed) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j]))) * epi.scale;
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * epi.scale;
          if (EPI == kEpiMaskAdapter) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int a = ((col + j) / epi.mask_rank) % epi.mask_num_adapters + 1;
              if (a != radapter) v[j] = 0.f;
            }
          }
        }
        uint4* o4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(epi.out) + (int64_t)row * epi.ldo + col);
        if (EPI == kEpiMultimemRed) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            multimem_red_add_v4_bf16x2(o4 + j, pack_bf16x2(v[8 * j], v[8 * j + 1]),
                                       pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                                       pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                                       pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            o4[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                               pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
        }
      }
    }
  }
}

// Epilogues whose bf16 output goes out through shared memory and TMA stores
// (output tiles a multiple of 64 columns wide).
__host__ __device__ constexpr bool epi_staged(int epi, int bn) {
  return (epi == kEpiStore || epi == kEpiResAdd || epi == kEpiSwiGLU || epi == kEpiMultimemRed) &&
         ((epi == kEpiSwiGLU ? bn / 2 : bn) % 64 == 0);
}
// Staged epilogues whose output leaves by TMA store (the multimem one leaves by
// row-contiguous multimem reductions instead).
__host__ __device__ constexpr bool epi_tma_store(int epi, int bn) {
  return epi_staged(epi, bn) && epi != kEpiMultimemRed;
}
__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Staged epilogue of one 128 x BN accumulator, 64 output columns at a time.
// Each warp owns 32 rows (TMEM lanes): thread `lane` converts its row's 64
// values to bf16 (after SwiGLU, or adding the residual) and writes them as
// eight 16-byte chunks into a swizzled 32 x 128-byte buffer; lane 0 then
// stores the whole 32 x 64 box with one TMA store, which runs asynchronously
// while the warp moves on to the next buffer. The residual (kEpiResAdd) is
// read with coalesced 16-byte loads (eight threads per 128-byte row) through
// the same buffer. Rows at or past M are dropped by the tensor map bounds.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile_staged(const GemmEpiArgs& epi, const CUtensorMap* tm_out,
                                                     uint32_t tbase, int row0, int M, int n0,
                                                     uint8_t* stage, int& sbuf) {
  const int lane = threadIdx.x & 31;
  constexpr int OUT_COLS = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  const int out_col0 = (EPI == kEpiSwiGLU) ? n0 / 2 : n0;
#pragma unroll 1
  for (int c = 0; c < OUT_COLS; c += 64) {
    uint8_t* buf = stage + sbuf * 4096;
    // the TMA store that last used this buffer must have read it
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    uint32_t pk[32];  // 64 bf16 of this thread's row, chunk-major
    if (EPI == kEpiSwiGLU) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t g[32], u[32];
        tmem_ld32(tbase + c + 32 * h, g);
        tmem_ld32(tbase + BN / 2 + c + 32 * h, u);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          // gate/up pre-activations are rounded to bf16 first, as the
          // unfused path stores them in bf16 before the activation
          const float g0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j])));
          const float g1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j + 1])));
          const float u0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j])));
          const float u1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j + 1])));
          pk[16 * h + j] = pack_bf16x2(__fdividef(g0, 1.f + __expf(-g0)) * u0, __fdividef(g1, 1.f + __expf(-g1)) * u1);
        }
      }
    } else {
      uint32_t r[64];
      tmem_ld32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld32(tbase + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      const bool has_res = (EPI == kEpiResAdd) || (EPI == kEpiMultimemRed && epi.residual != nullptr);
      if (has_res) {
        // coalesced residual read of the warp's 32 x 64 box into the buffer
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int rr = 4 * j + (lane >> 3), ch = lane & 7;
          const int grow = row0 + rr;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (grow < M)
            v = *reinterpret_cast<const uint4*>(epi.residual + (int64_t)grow * epi.ldr + n0 + c + ch * 8);
          *reinterpret_cast<uint4*>(buf + swz128(rr, ch)) = v;
        }
        __syncwarp();
      }
      tmem_wait_ld();
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        if (has_res) {
          const uint4 w = *reinterpret_cast<const uint4*>(buf + swz128(lane, ch));
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            // the projection is rounded to bf16 before the residual add, as
            // the unfused path materialises it in bf16
            const float2 f = unpack_bf16x2(ww[t]);
            const float p0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * ch + 2 * t])));
            const float p1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * ch + 2 * t + 1])));
            pk[4 * ch + t] = pack_bf16x2(f.x + p0 * epi.scale, f.y + p1 * epi.scale);
          }
        } else if (EPI == kEpiMultimemRed) {
          // partial projection rounded to bf16 before scaling, as the unfused path
#pragma unroll
          for (int t = 0; t < 4; ++t)
            pk[4 * ch + t] =
                pack_bf16x2(__bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * ch + 2 * t]))) * epi.scale,
                            __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * ch + 2 * t + 1]))) * epi.scale);
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t)
            pk[4 * ch + t] = pack_bf16x2(__uint_as_float(r[8 * ch + 2 * t]) * epi.scale,
                                         __uint_as_float(r[8 * ch + 2 * t + 1]) * epi.scale);
        }
      }
    }
#pragma unroll
    for (int ch = 0; ch < 8; ++ch)
      *reinterpret_cast<uint4*>(buf + swz128(lane, ch)) =
          make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
    if (EPI == kEpiMultimemRed) {
      // read the box back row-contiguously (eight lanes per 128-byte row, four
      // rows per instruction) and add it into every rank's copy through the
      // multicast address: full-line NVLink transfers instead of 16-byte ones
      __syncwarp();
      __nv_bfloat16* mc = reinterpret_cast<__nv_bfloat16*>(epi.out);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int rr = 4 * j + (lane >> 3), ch = lane & 7;
        if (row0 + rr < M) {
          const uint4 v = *reinterpret_cast<const uint4*>(buf + swz128(rr, ch));
          multimem_red_add_v4_bf16x2(mc + (int64_t)(row0 + rr) * epi.ldo + out_col0 + c + ch * 8, v.x, v.y, v.z, v.w);
        }
      }
      __syncwarp();  // the buffer is rewritten two boxes later
    } else {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < M) {
        tma_store_2d(tm_out, buf, out_col0 + c, row0);
        bulk_commit_group();
      }
    }
    sbuf ^= 1;
  }
}

// Persistent: one CTA per SM walks tiles t = blockIdx.x, +gridDim.x, ...
// TMEM holds two accumulators so the epilogue of tile i overlaps the
// mainloop of tile i+1.
template <int BN, int EPI, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
    switched_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_b,
                         const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_lb,
                         const __grid_constant__ CUtensorMap tm_out, int M, int N, int K,
                         GemmLoraArgs lora, GemmEpiArgs epi, GemmGroupArgs grp, uint32_t* err) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* staging = smem + C::STAGING_OFF;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + C::BM - 1) / C::BM;
  const int n_tiles = N / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int main_blocks = K / C::BK;
  const int ksplit = grp.ksplit > 1 ? grp.ksplit : 1;   // the host keeps main_blocks % ksplit == 0
  const int num_work = num_tiles * ksplit;
  const int part_blocks = main_blocks / ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4);  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (lora.enabled) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_lb);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t kb = 0;  // k-blocks issued by this CTA (ring position)
      bool stop = false;
      for (int t = blockIdx.x; t < num_work && !stop; t += gridDim.x) {
        int mt, nt;
        const int part = t / num_tiles;
        gemm_tile_coords(t - part * num_tiles, m_tiles, n_tiles, mt, nt);
        const int m0 = mt * C::BM, n0 = nt * BN;
        if (tile_skipped<BN, EPI>(epi, grp, mt, n0)) continue;
        const LoraTile lt = (part == ksplit - 1) ? lora_tile<SPLIT>(lora, mt, n0) : LoraTile{0, 0, 0, 0};
        const int kb0 = part * part_blocks;
        const int total = part_blocks + lt.blocks;
        uint64_t rem = lt.amask;
        int a_bit = 0, rb = 0;
        for (int i = 0; i < total; ++i, ++kb) {
          const int s = kb % C::STAGES;
          const uint32_t ph = (kb / C::STAGES) & 1;
          if (*abort_flag || !mbar_wait(&empty_bar[s], ph ^ 1, err, kErrGemmWait)) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          if (i < part_blocks) {
            mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
            tma_load_2d(sa, &tm_a, &full_bar[s], (kb0 + i) * C::BK, m0);
            if (grp.tile_expert != nullptr)
              tma_load_3d(sb, &tm_b, &full_bar[s], (kb0 + i) * C::BK, n0, grp.tile_expert[mt]);
            else
              tma_load_2d(sb, &tm_b, &full_bar[s], (kb0 + i) * C::BK, n0);
          } else {
            if (rb == 0) a_bit = __ffsll((long long)rem) - 1;
            const int kcol = a_bit * lora.rank_blocks * 32 + rb * 32;
            constexpr int nsub = SPLIT ? 2 : 1;
            mbar_arrive_expect_tx(&full_bar[s], nsub * (C::BM * 32 * 2) + BN * 32 * 2);
            tma_load_2d(sa, &tm_s, &full_bar[s], lt.s_base0 + kcol, m0);
            if (SPLIT) tma_load_2d(sa + C::BM * 64, &tm_s, &full_bar[s], lt.s_base1 + kcol, m0);
            tma_load_2d(sb, &tm_lb, &full_bar[s], kcol, n0);
            if (++rb == lora.rank_blocks) {
              rb = 0;
              rem &= rem - 1;
            }
          }
        }
      }
      if (*abort_flag) {
        // drain: no TMA write may still be in flight into our smem at exit
        const uint32_t first = kb > (uint32_t)C::STAGES ? kb - C::STAGES : 0;
        for (uint32_t j = first; j < kb; ++j)
          mbar_wait(&full_bar[j % C::STAGES], (j / C::STAGES) & 1, err, kErrGemmWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_full = umma_idesc_bf16(128, BN);
      const uint32_t idesc_half = umma_idesc_bf16(128, SPLIT ? BN / 2 : BN);
      uint32_t kb = 0;
      int ltile = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < num_work && !stop; t += gridDim.x) {
        int mt, nt;
        const int part = t / num_tiles;
        gemm_tile_coords(t - part * num_tiles, m_tiles, n_tiles, mt, nt);
        if (tile_skipped<BN, EPI>(epi, grp, mt, nt * BN)) continue;
        const LoraTile lt = (part == ksplit - 1) ? lora_tile<SPLIT>(lora, mt, nt * BN) : LoraTile{0, 0, 0, 0};
        const int total = part_blocks + lt.blocks;
        const int acc = ltile & 1;
        if (*abort_flag || !mbar_wait(&tempty_bar[acc], ((ltile >> 1) & 1) ^ 1, err, kErrGemmWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + acc * BN;
        for (int i = 0; i < total; ++i, ++kb) {
          const int s = kb % C::STAGES;
          const uint32_t ph = (kb / C::STAGES) & 1;
          if (*abort_flag || !mbar_wait(&full_bar[s], ph, err, kErrGemmWait)) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
          if (i < part_blocks) {
            const uint64_t ad = umma_desc_sw128(sa);
            const uint64_t bd = umma_desc_sw128(sb);
#pragma unroll
            for (int kk = 0; kk < C::BK / 16; ++kk)
              umma_bf16(tacc, ad + 2 * kk, bd + 2 * kk, idesc_full, (i | kk) != 0);
          } else if (SPLIT) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint64_t ad = umma_desc_sw64(sa + u * C::BM * 64);
              const uint64_t bd = umma_desc_sw64(sb + u * (BN / 2) * 64);
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)
                umma_bf16(tacc + u * (BN / 2), ad + 2 * kk, bd + 2 * kk, idesc_half, 1);
            }
          } else {
            const uint64_t ad = umma_desc_sw64(sa);
            const uint64_t bd = umma_desc_sw64(sb);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) umma_bf16(tacc, ad + 2 * kk, bd + 2 * kk, idesc_full, 1);
          }
          umma_commit(&empty_bar[s]);
        }
        umma_commit(&tfull_bar[acc]);
        ++ltile;  // only tiles that use an accumulator advance the buffer sequence
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int ltile = 0;
    int sbuf = 0;
    for (int t = blockIdx.x; t < num_work; t += gridDim.x) {
      int mt, nt;
      const int part = t / num_tiles;
      gemm_tile_coords(t - part * num_tiles, m_tiles, n_tiles, mt, nt);
      const int m0 = mt * C::BM, n0 = nt * BN;
      if (tile_skipped<BN, EPI>(epi, grp, mt, n0)) continue;
      const int acc = ltile & 1;
      if (*abort_flag || !mbar_wait(&tfull_bar[acc], (ltile >> 1) & 1, err, kErrGemmWait)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if (ksplit > 1) {
        // split-K part: fp32 partial sums; splitk_reduce_kernel applies the epilogue
        GemmEpiArgs pe = epi;
        pe.out = grp.ws + (int64_t)part * M * N;
        pe.ldo = N;
        pe.scale = 1.f;
        epilogue_tile<BN, kEpiF32>(pe, tbase, row, M, n0);
      } else if constexpr (epi_staged(EPI, BN)) {
        epilogue_tile_staged<BN, EPI>(epi, &tm_out, tbase, m0 + q * 32, M, n0, staging + q * 8192, sbuf);
      } else {
        epilogue_tile<BN, EPI>(epi, tbase, row, M, n0);
      }
      if (EPI == kEpiMultimemRed) __threadfence_system();  // this tile's reductions precede the next barrier
      // accumulator drained: hand the TMEM buffer back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      ++ltile;
    }
    if (epi_tma_store(EPI, BN) && lane == 0) bulk_wait_group_all();  // stores done before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a cluster of two CTAs on neighbouring SMs
// computes a 256 x 256 tile. Each CTA stages its own 128 rows of X and its own
// 128 rows of W per K block; the leader CTA's MMA thread issues
// tcgen05.mma.cta_group::2 over both CTAs' shared memory, and each CTA's
// TMEM receives its 128 x 256 accumulator. Per SM this moves half the W bytes
// of the single-CTA 128 x 256 tile through L2 and shared memory for the same
// tensor work. Both CTAs load with plain (non-multicast) TMA copies whose
// completion is counted on the leader's barrier; only the leader sets the
// expected byte count, for both CTAs. MMA completion is signalled to both
// CTAs' barriers by one commit with a two-CTA mask.
// ---------------------------------------------------------------------------
struct PairCfg {
  static constexpr int BM = 128;                   // rows per CTA (tile: 256)
  static constexpr int BN = 256;                   // tile columns (each CTA stages BN/2 rows of W)
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;      // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int TMEM_COLS = 2 * BN;         // two 256-column accumulators = all 512 columns
  static constexpr int STAGING_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STAGING_OFF + kEpiStageBytes;
  static constexpr int SMEM_BYTES = BAR_OFF + 1024 + 256;   // 225.25 KB of the 227 KB a CTA may use
};

template <int EPI, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    switched_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                              const __grid_constant__ CUtensorMap tm_b,
                              const __grid_constant__ CUtensorMap tm_s,
                              const __grid_constant__ CUtensorMap tm_lb,
                              const __grid_constant__ CUtensorMap tm_out, int M, int N, int K,
                              GemmLoraArgs lora, GemmEpiArgs epi, uint32_t* err) {
  using C = PairCfg;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* staging = smem + C::STAGING_OFF;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);  // leader's are used
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;          // [2], leader's are used
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int m_tiles128 = (M + C::BM - 1) / C::BM;
  const int m_tiles = (M + 2 * C::BM - 1) / (2 * C::BM);
  const int n_tiles = N / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int main_blocks = K / C::BK;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 8);  // one arrive per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (lora.enabled) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_lb);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_bar_leader = mapa_shared(smem_u32(full_bar), 0);
  const uint32_t tempty_bar_leader = mapa_shared(smem_u32(tempty_bar), 0);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      uint32_t kb = 0;
      bool stop = false;
      for (int t = cluster_id; t < num_tiles && !stop; t += num_clusters) {
        int mt, nt;
        gemm_tile_coords<8>(t, m_tiles, n_tiles, mt, nt);
        const int m0 = mt * 2 * C::BM + (int)rank * C::BM;  // this CTA's X rows
        const int n0 = nt * BN;
        const LoraTile lt = lora_tile<SPLIT>(lora, 2 * mt, n0, 2, m_tiles128);
        const int total = main_blocks + lt.blocks;
        uint64_t rem = lt.amask;
        int a_bit = 0, rb = 0;
        // The pair expands the union of both CTAs' adapters. With a tile mask,
        // the shrink leaves S columns of adapters absent from a 128-row tile
        // unwritten; for those the CTA loads S rows past M, which TMA fills
        // with zeros (same byte count), so the other adapter's delta is exact.
        const int own_tile = 2 * mt + (int)rank;
        const uint64_t own_mask = (lora.tile_mask == nullptr) ? ~0ull
                                  : (own_tile < m_tiles128 ? lora.tile_mask[own_tile] : 0ull);
        const int zero_row = m_tiles128 * C::BM;  // first row of an all-out-of-bounds box
        for (int i = 0; i < total; ++i, ++kb) {
          const int s = kb % C::STAGES;
          const uint32_t ph = (kb / C::STAGES) & 1;
          if (*abort_flag || !mbar_wait(&empty_bar[s], ph ^ 1, err, kErrGemmWait)) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const uint32_t fb = full_bar_leader + s * 8;
          if (i < main_blocks) {
            if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * C::STAGE_BYTES);
            const int kx = i * C::BK;
            tma_load_2d_pair(sa, &tm_a, fb, kx, m0);
            tma_load_2d_pair(sb, &tm_b, fb, kx, n0 + (int)rank * (BN / 2));
          } else {
            if (rb == 0) a_bit = __ffsll((long long)rem) - 1;
            const int kcol = a_bit * lora.rank_blocks * 32 + rb * 32;
            constexpr int nsub = SPLIT ? 2 : 1;
            // per CTA: nsub S tiles of 128 x 32, and BN/2 rows x 32 of packed B
            if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * (nsub * (C::BM * 32 * 2) + (BN / 2) * 32 * 2));
            const int ys = ((own_mask >> a_bit) & 1ull) ? m0 : zero_row;
            tma_load_2d_pair(sa, &tm_s, fb, lt.s_base0 + kcol, ys);
            if (SPLIT) {
              tma_load_2d_pair(sa + C::BM * 64, &tm_s, fb, lt.s_base1 + kcol, ys);
              // gate rows [n0 + 64r, +64) and up rows [n0 + 128 + 64r, +64): the
              // two N = 128 pair MMAs each take 64 rows from either CTA
              tma_load_2d_pair(sb, &tm_lb, fb, kcol, n0 + (int)rank * 64);
              tma_load_2d_pair(sb + 64 * 64, &tm_lb, fb, kcol, n0 + BN / 2 + (int)rank * 64);
            } else {
              tma_load_2d_pair(sb, &tm_lb, fb, kcol, n0 + (int)rank * (BN / 2));
            }
            if (++rb == lora.rank_blocks) {
              rb = 0;
              rem &= rem - 1;
            }
          }
        }
      }
      // every stage this CTA filled has been released by the pair MMA before
      // the CTA may exit (the release arrives in this CTA's shared memory)
      const uint32_t first = kb > (uint32_t)C::STAGES ? kb - C::STAGES : 0;
      for (uint32_t j = first; j < kb && !*abort_flag; ++j)
        if (!mbar_wait(&empty_bar[j % C::STAGES], (j / C::STAGES) & 1, err, kErrGemmWait)) *abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc_full = umma_idesc_bf16(256, BN);
      const uint32_t idesc_half = umma_idesc_bf16(256, BN / 2);
      uint32_t kb = 0;
      int ltile = 0;
      bool stop = false;
      for (int t = cluster_id; t < num_tiles && !stop; t += num_clusters) {
        int mt, nt;
        gemm_tile_coords<8>(t, m_tiles, n_tiles, mt, nt);
        const LoraTile lt = lora_tile<SPLIT>(lora, 2 * mt, nt * BN, 2, m_tiles128);
        const int total = main_blocks + lt.blocks;
        const int acc = ltile & 1;
        if (*abort_flag || !mbar_wait(&tempty_bar[acc], ((ltile >> 1) & 1) ^ 1, err, kErrGemmWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + acc * BN;
        for (int i = 0; i < total; ++i, ++kb) {
          const int s = kb % C::STAGES;
          const uint32_t ph = (kb / C::STAGES) & 1;
          if (*abort_flag || !mbar_wait(&full_bar[s], ph, err, kErrGemmWait)) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
          if (i < main_blocks) {
            const uint64_t ad = umma_desc_sw128(sa);
            const uint64_t bd = umma_desc_sw128(sb);
#pragma unroll
            for (int kk = 0; kk < C::BK / 16; ++kk)
              umma_bf16_pair(tacc, ad + 2 * kk, bd + 2 * kk, idesc_full, (i | kk) != 0);
          } else if (SPLIT) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint64_t ad = umma_desc_sw64(sa + u * C::BM * 64);
              const uint64_t bd = umma_desc_sw64(sb + u * 64 * 64);
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)
                umma_bf16_pair(tacc + u * (BN / 2), ad + 2 * kk, bd + 2 * kk, idesc_half, 1);
            }
          } else {
            const uint64_t ad = umma_desc_sw64(sa);
            const uint64_t bd = umma_desc_sw64(sb);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) umma_bf16_pair(tacc, ad + 2 * kk, bd + 2 * kk, idesc_full, 1);
          }
          umma_commit_pair(&empty_bar[s], 0x3);
        }
        if (stop) break;
        umma_commit_pair(&tfull_bar[acc], 0x3);
        ++ltile;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;
    int ltile = 0;
    int sbuf = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters) {
      int mt, nt;
      gemm_tile_coords<8>(t, m_tiles, n_tiles, mt, nt);
      const int acc = ltile & 1;
      if (*abort_flag || !mbar_wait(&tfull_bar[acc], (ltile >> 1) & 1, err, kErrGemmWait)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mt * 2 * C::BM + (int)rank * C::BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      if constexpr (epi_staged(EPI, BN))
        epilogue_tile_staged<BN, EPI>(epi, &tm_out, tbase, row - lane, M, nt * BN, staging + q * 8192, sbuf);
      else
        epilogue_tile<BN, EPI>(epi, tbase, row, M, nt * BN);
      if (EPI == kEpiMultimemRed) __threadfence_system();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_bar_leader + acc * 8);
      ++ltile;
    }
    if (epi_tma_store(EPI, BN) && lane == 0) bulk_wait_group_all();
  }

  if (*abort_flag) {
    // error path: give copies that may still be in flight into this CTA's
    // shared memory time to land before the CTA exits (bounded, ~1 ms)
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
static int num_sms_for_current_device() {
  static int cached[64] = {0};
  int dev = 0;
  GSB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  GSB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int BN, int EPI, bool SPLIT>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts,
                        const CUtensorMap& tlb, const CUtensorMap& to, int M, int N, int K, const GemmLoraArgs& lora,
                        const GemmEpiArgs& epi, const GemmGroupArgs& grp, uint32_t* err, cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kfn = switched_gemm_kernel<BN, EPI, SPLIT>;
  static bool configured = false;  // per instantiation; attribute is per-function
  if (!configured) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    configured = true;
  }
  const int tiles = (N / BN) * ((M + C::BM - 1) / C::BM) * (grp.ksplit > 1 ? grp.ksplit : 1);
  const int grid = std::min(tiles, num_sms_for_current_device());
  kfn<<<(::gsb::count_launch(), grid), 192, C::SMEM_BYTES, stream>>>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err);
  GSB_CUDA_CHECK(cudaGetLastError());
}

// Clusters of two that fit at once for the pair kernel (queried once per device).
template <int EPI, bool SPLIT>
static int pair_max_clusters() {
  static int cached[64] = {0};
  int dev = 0;
  GSB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64 && cached[dev]) return cached[dev];
  auto kfn = switched_gemm_pair_kernel<EPI, SPLIT>;
  GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM_BYTES));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 148, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  GSB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kfn, &cfg));
  if (n <= 0) n = num_sms_for_current_device() / 2;
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int EPI, bool SPLIT>
static void launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts,
                             const CUtensorMap& tlb, const CUtensorMap& to, int M, int N, int K,
                             const GemmLoraArgs& lora,
                             const GemmEpiArgs& epi, uint32_t* err, cudaStream_t stream) {
  auto kfn = switched_gemm_pair_kernel<EPI, SPLIT>;
  const int clusters = pair_max_clusters<EPI, SPLIT>();  // also sets the shared-memory attribute
  const int tiles = (N / PairCfg::BN) * ((M + 255) / 256);
  const int grid = 2 * std::min(tiles, clusters);
  kfn<<<(::gsb::count_launch(), grid), 192, PairCfg::SMEM_BYTES, stream>>>(ta, tb, ts, tlb, to, M, N, K, lora, epi, err);
  GSB_CUDA_CHECK(cudaGetLastError());
}

static void dispatch_epi_pair(int epi_kind, const CUtensorMap& ta, const CUtensorMap& tb,
                              const CUtensorMap& ts, const CUtensorMap& tlb, const CUtensorMap& to,
                              int M, int N, int K,
                              const GemmLoraArgs& lora, const GemmEpiArgs& epi, uint32_t* err,
                              cudaStream_t st) {
  switch (epi_kind) {
    case kEpiStore: launch_gemm_pair<kEpiStore, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, err, st); break;
    case kEpiResAdd: launch_gemm_pair<kEpiResAdd, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, err, st); break;
    case kEpiSwiGLU: launch_gemm_pair<kEpiSwiGLU, true>(ta, tb, ts, tlb, to, M, N, K, lora, epi, err, st); break;
    case kEpiMultimemRed: launch_gemm_pair<kEpiMultimemRed, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, err, st); break;
    default: GSB_CHECK(false, "no pair kernel for epilogue kind ", epi_kind);
  }
}

// The pair kernel serves 256-wide tiles of large-M GEMMs: M >= this threshold
// (gemm_pair_min_m() changes it at run time for A/B tests; a negative value
// keeps every GEMM on the single-CTA kernel).
static int g_pair_min_m = 512;

static bool pair_enabled(int M, int bn, int epi_kind) {
  if (g_pair_min_m < 0 || bn != 256 || M < g_pair_min_m) return false;
  return epi_kind == kEpiStore || epi_kind == kEpiResAdd || epi_kind == kEpiSwiGLU || epi_kind == kEpiMultimemRed;
}

template <int BN>
static void dispatch_epi(int epi_kind, const CUtensorMap& ta, const CUtensorMap& tb,
                         const CUtensorMap& ts, const CUtensorMap& tlb, const CUtensorMap& to,
                         int M, int N, int K,
                         const GemmLoraArgs& lora, const GemmEpiArgs& epi, const GemmGroupArgs& grp, uint32_t* err,
                         cudaStream_t st) {
  switch (epi_kind) {
    case kEpiStore: launch_gemm<BN, kEpiStore, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    case kEpiResAdd: launch_gemm<BN, kEpiResAdd, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    case kEpiSwiGLU: launch_gemm<BN, kEpiSwiGLU, true>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    case kEpiMaskAdapter: launch_gemm<BN, kEpiMaskAdapter, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    case kEpiF32: launch_gemm<BN, kEpiF32, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    case kEpiMultimemRed: launch_gemm<BN, kEpiMultimemRed, false>(ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, err, st); break;
    default: GSB_CHECK(false, "unknown epilogue kind ", epi_kind);
  }
}

// Split-K finish: out = epilogue(sum over parts of ws[p]), with the epilogue
// arithmetic of epilogue_tile (bf16 rounding of the projection before a
// residual add; gate / up rounded to bf16 before SwiGLU, whose column tiles of
// `swiglu_tile` hold the gate half then the up half). One thread per two columns.
template <int EPI>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int parts, int M, int N, float scale,
                                     const __nv_bfloat16* __restrict__ res, int64_t ldr, void* __restrict__ out,
                                     int64_t ldo, int swiglu_tile) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int half_n = N / 2;
  if (idx >= (int64_t)M * half_n) return;
  const int row = (int)(idx / half_n);
  const int c = (int)(idx % half_n) * 2;
  const int64_t plane = (int64_t)M * N;
  auto sum2 = [&](int col, float& a0, float& a1) {
    a0 = 0.f;
    a1 = 0.f;
    for (int p = 0; p < parts; ++p) {
      const float2 v = *reinterpret_cast<const float2*>(ws + p * plane + (int64_t)row * N + col);
      a0 += v.x;
      a1 += v.y;
    }
  };
  if (EPI == kEpiSwiGLU) {
    const int t = c / swiglu_tile, j = c % swiglu_tile, h = swiglu_tile / 2;
    if (j >= h) return;  // up columns are read by the thread of their gate columns
    float g0, g1, u0, u1;
    sum2(c, g0, g1);
    sum2(c + h, u0, u1);
    g0 = __bfloat162float(__float2bfloat16_rn(g0));
    g1 = __bfloat162float(__float2bfloat16_rn(g1));
    u0 = __bfloat162float(__float2bfloat16_rn(u0));
    u1 = __bfloat162float(__float2bfloat16_rn(u1));
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)row * ldo + t * h + j) =
        pack_bf16x2(__fdividef(g0, 1.f + __expf(-g0)) * u0, __fdividef(g1, 1.f + __expf(-g1)) * u1);
    return;
  }
  float a0, a1;
  sum2(c, a0, a1);
  if (EPI == kEpiF32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + (int64_t)row * ldo + c) = make_float2(a0 * scale,
                                                                                                    a1 * scale);
    return;
  }
  float v0 = a0 * scale, v1 = a1 * scale;
  if (EPI == kEpiResAdd) {
    const float2 r = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(res + (int64_t)row * ldr + c));
    v0 = r.x + __bfloat162float(__float2bfloat16_rn(a0)) * scale;
    v1 = r.y + __bfloat162float(__float2bfloat16_rn(a1)) * scale;
  }
  *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)row * ldo + c) = pack_bf16x2(v0, v1);
}

// Split-K is used below this many output tiles (half the SMs); 0 turns it off
// (gemm_splitk_max_tiles() changes it at run time for A/B tests).
static int g_splitk_max_tiles = 74;

// Parts for a single-CTA GEMM of `tiles` output tiles and `kblocks` 64-deep K
// blocks: the largest of 4 / 3 / 2 that divides kblocks, leaves at least four
// blocks per part and keeps tiles * parts within one wave; 1 when none does.
static int splitk_parts(int tiles, int kblocks, int nsms) {
  if (tiles >= g_splitk_max_tiles) return 1;
  for (int p = 4; p >= 2; --p)
    if (kblocks % p == 0 && kblocks / p >= 4 && tiles * p <= nsms) return p;
  return 1;
}

}  // namespace gsb

// x [M, K] bf16, w [N, K] bf16 (both row-major, K contiguous).
// LoRA (optional): s [M, Ks] bf16 masked shrink output, lb [N, NA*rank] bf16
// packed expand weights, tile_mask [ceil(M/128)] int64 adapter bitmask.
void gsb_switched_gemm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                       int64_t epi_kind, int64_t bn, const c10::optional<at::Tensor>& residual,
                       double scale, const c10::optional<at::Tensor>& s,
                       const c10::optional<at::Tensor>& lb,
                       const c10::optional<at::Tensor>& tile_mask, int64_t rank,
                       int64_t num_adapters, std::vector<int64_t> slice_bounds,
                       const c10::optional<at::Tensor>& row_adapter, int64_t mask_rank,
                       int64_t mask_num_adapters, const at::Tensor& err, int64_t mc_out,
                       const c10::optional<at::Tensor>& tile_expert) {
  using namespace gsb;
  GSB_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "tensors must be on CUDA");
  GSB_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
            "x and w must be bf16");
  const bool grouped = tile_expert.has_value();
  GSB_CHECK(x.dim() == 2 && w.dim() == (grouped ? 3 : 2) && x.stride(1) == 1 && w.stride(-1) == 1,
            "x must be 2-D and w 2-D (3-D [E, N, K] with tile_expert) with unit inner stride");
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)w.size(grouped ? 1 : 0);
  GSB_CHECK(w.size(-1) == K, "K mismatch");
  GemmGroupArgs grp{};
  grp.tile_expert = nullptr;
  grp.ksplit = 1;
  grp.ws = nullptr;
  if (grouped) {
    GSB_CHECK(w.is_contiguous(), "grouped GEMM: w must be a contiguous [E, N, K] stack");
    GSB_CHECK(tile_expert->scalar_type() == at::kInt && tile_expert->numel() >= (M + 127) / 128,
              "grouped GEMM: tile_expert must be int32 [ceil(M/128)]");
    GSB_CHECK(!s.has_value(), "grouped GEMM: no LoRA operands");
    grp.tile_expert = tile_expert->data_ptr<int32_t>();
  }
  GSB_CHECK(bn == 64 || bn == 128 || bn == 256, "bn must be 64, 128 or 256");
  GSB_CHECK(N % bn == 0, "N=", N, " must be a multiple of bn=", bn);
  GSB_CHECK(K % 64 == 0, "K=", K, " must be a multiple of 64");
  GSB_CHECK(M > 0, "M must be positive");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();

  CUtensorMap ta = make_tmap_bf16_2d(x.data_ptr(), M, K, x.stride(0), 64, 128,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  const bool pair = !grouped && pair_enabled(M, (int)bn, (int)epi_kind);
  // the pair kernel stages half of the 256-row W tile in each CTA
  CUtensorMap tb = grouped ? make_tmap_bf16_3d(w.data_ptr(), w.size(0), N, K, 64, (uint32_t)bn,
                                               CU_TENSOR_MAP_SWIZZLE_128B)
                           : make_tmap_bf16_2d(w.data_ptr(), N, K, w.stride(0), 64, (uint32_t)(pair ? bn / 2 : bn),
                                               CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ts = ta, tlb = tb;  // placeholders when LoRA is off
  GemmLoraArgs lora{};
  lora.enabled = 0;
  if (s.has_value() && lb.has_value() && num_adapters > 0) {
    const auto& S = *s;
    const auto& LB = *lb;
    GSB_CHECK(S.scalar_type() == at::kBFloat16 && LB.scalar_type() == at::kBFloat16,
              "LoRA operands must be bf16");
    GSB_CHECK(rank % 32 == 0 && rank > 0, "padded rank must be a positive multiple of 32");
    GSB_CHECK(S.size(0) == M && S.stride(1) == 1 && LB.stride(1) == 1, "bad LoRA operand layout");
    GSB_CHECK(LB.size(0) == N && LB.size(1) == num_adapters * rank, "lb must be [N, NA*rank]");
    GSB_CHECK(num_adapters <= 64, "at most 64 adapters per module");
    ts = make_tmap_bf16_2d(S.data_ptr(), M, S.size(1), S.stride(0), 32, 128,
                           CU_TENSOR_MAP_SWIZZLE_64B);
    // pair kernel: each CTA stages 128 of the tile's 256 rows of packed B, or
    // (SwiGLU) 64 gate rows and 64 up rows
    const uint32_t lb_rows = pair ? (epi_kind == kEpiSwiGLU ? 64u : 128u) : (uint32_t)bn;
    tlb = make_tmap_bf16_2d(LB.data_ptr(), N, LB.size(1), LB.stride(0), 32, lb_rows,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    lora.enabled = 1;
    lora.rank_blocks = (int)(rank / 32);
    lora.num_adapters = (int)num_adapters;
    GSB_CHECK(slice_bounds.size() >= 2 && slice_bounds.size() <= 5, "1..4 slices");
    lora.num_slices = (int)slice_bounds.size() - 1;
    for (size_t i = 0; i < slice_bounds.size(); ++i) {
      lora.slice_bounds[i] = (int)slice_bounds[i];
      if (i + 1 < slice_bounds.size())
        GSB_CHECK(slice_bounds[i] % bn == 0, "slice start ", slice_bounds[i]
                                                , " not a multiple of bn ", bn);
    }
    lora.s_ld_slices = lora.num_slices;
    GSB_CHECK(S.size(1) >= (int64_t)lora.num_slices * num_adapters * rank, "S too narrow");
    lora.tile_mask = nullptr;
    if (tile_mask.has_value()) {
      GSB_CHECK(tile_mask->scalar_type() == at::kLong && tile_mask->numel() >= (M + 127) / 128,
                "tile_mask must be int64 [ceil(M/128)]");
      lora.tile_mask = reinterpret_cast<const uint64_t*>(tile_mask->data_ptr());
    }
  }
  GemmEpiArgs epi{};
  epi.out = (epi_kind == kEpiMultimemRed && mc_out != 0) ? reinterpret_cast<void*>(mc_out) : out.data_ptr();
  epi.ldo = out.stride(0);
  epi.scale = (float)scale;
  epi.residual = nullptr;
  epi.ldr = 0;
  if (epi_kind == kEpiMultimemRed) {
    GSB_CHECK(mc_out != 0, "multimem epilogue needs the multicast address of the output");
    GSB_CHECK((mc_out & 15) == 0, "multicast address must be 16-byte aligned");
    if (residual.has_value()) {
      epi.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
      epi.ldr = residual->stride(0);
    }
  }
  if (epi_kind == kEpiResAdd) {
    GSB_CHECK(residual.has_value(), "residual required");
    epi.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    epi.ldr = residual->stride(0);
  }
  if (epi_kind == kEpiF32) {
    GSB_CHECK(out.scalar_type() == at::kFloat, "fp32 output expected");
  } else {
    GSB_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output expected");
  }
  if (epi_kind == kEpiSwiGLU) {
    GSB_CHECK(out.size(1) * 2 == N, "SwiGLU output must have N/2 columns");
  } else {
    GSB_CHECK(out.size(1) == N, "output must have N columns");
  }
  GSB_CHECK(out.size(0) == M && out.stride(1) == 1 && (out.stride(0) % 8) == 0,
            "output must be [M, *] with 16-byte aligned rows");
  epi.row_adapter = nullptr;
  if (epi_kind == kEpiMaskAdapter) {
    GSB_CHECK(row_adapter.has_value() && row_adapter->scalar_type() == at::kInt,
              "row_adapter int32 required");
    epi.row_adapter = row_adapter->data_ptr<int32_t>();
    epi.mask_rank = (int)mask_rank;
    epi.mask_num_adapters = (int)mask_num_adapters;
    epi.skip_mask = nullptr;
    if (tile_mask.has_value()) {  // for the shrink, tile_mask selects the tiles to compute
      GSB_CHECK(tile_mask->scalar_type() == at::kLong && tile_mask->numel() >= (M + 127) / 128,
                "tile_mask must be int64 [ceil(M/128)]");
      epi.skip_mask = reinterpret_cast<const uint64_t*>(tile_mask->data_ptr());
      GSB_CHECK(mask_num_adapters <= 64, "at most 64 adapters per module");
    }
    GSB_CHECK(mask_rank > 0 && mask_num_adapters > 0, "mask_rank and mask_num_adapters required");
  }
  uint32_t* errp = reinterpret_cast<uint32_t*>(err.data_ptr());
  if (!grouped) {
    // decode-sized GEMMs: operand-swapped kernel with a cluster split-K (gemm_decode.cu)
    DecodeGemmArgs d{};
    d.x = x.data_ptr();
    d.ldx = x.stride(0);
    d.w = w.data_ptr();
    d.ldw = w.stride(0);
    d.out = epi.out;
    d.ldo = epi.ldo;
    d.M = M;
    d.N = N;
    d.K = K;
    d.epi = (int)epi_kind;
    d.scale = epi.scale;
    d.residual = epi.residual;
    d.ldr = epi.ldr;
    d.swiglu_tile = (int)bn;
    if (lora.enabled) {
      d.s = s->data_ptr();
      d.lds = s->stride(0);
      d.s_cols = (int)s->size(1);
      d.lb = lb->data_ptr();
      d.ldlb = lb->stride(0);
      d.rank = (int)rank;
      d.num_adapters = (int)num_adapters;
      d.num_slices = lora.num_slices;
      for (int i = 0; i <= lora.num_slices; ++i) d.slice_bounds[i] = lora.slice_bounds[i];
      d.tile_mask = lora.tile_mask;
    }
    if (epi_kind == kEpiMaskAdapter) {
      d.row_adapter = epi.row_adapter;
      d.mask_rank = epi.mask_rank;
      d.mask_num_adapters = epi.mask_num_adapters;
      d.skip_mask = epi.skip_mask;
    }
    if (decode_gemm_try(d, errp, stream)) return;
  }
  // staged epilogues store 32-row x 64-column boxes of the bf16 output by TMA
  CUtensorMap to = ta;
  if (epi_tma_store((int)epi_kind, pair ? 256 : (int)bn))
    to = make_tmap_bf16_2d(out.data_ptr(), M, out.size(1), out.stride(0), 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (pair) {
    dispatch_epi_pair((int)epi_kind, ta, tb, ts, tlb, to, M, N, K, lora, epi, errp, stream);
    return;
  }
  // decode-sized GEMMs: split K when the output tiles alone would leave most SMs idle
  const bool split_ok = !grouped && (epi_kind == kEpiStore || epi_kind == kEpiResAdd || epi_kind == kEpiSwiGLU ||
                                     epi_kind == kEpiF32);
  const int tiles = (int)(N / bn) * ((M + 127) / 128);
  const int parts = split_ok ? splitk_parts(tiles, K / 64, num_sms_for_current_device()) : 1;
  at::Tensor ws;
  if (parts > 1) {
    ws = at::empty({parts, M, N}, x.options().dtype(at::kFloat));
    grp.ksplit = parts;
    grp.ws = ws.data_ptr<float>();
  }
  switch (bn) {
    case 64: dispatch_epi<64>((int)epi_kind, ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, errp, stream); break;
    case 128: dispatch_epi<128>((int)epi_kind, ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, errp, stream); break;
    case 256: dispatch_epi<256>((int)epi_kind, ta, tb, ts, tlb, to, M, N, K, lora, epi, grp, errp, stream); break;
  }
  if (parts > 1) {
    const int64_t threads = (int64_t)M * (N / 2);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    const __nv_bfloat16* rp = epi.residual;
    switch (epi_kind) {
      case kEpiStore:
        splitk_reduce_kernel<kEpiStore><<<(::gsb::count_launch(), blocks), 256, 0, stream>>>(grp.ws, parts, M, N, epi.scale, rp, epi.ldr,
                                                                   out.data_ptr(), out.stride(0), (int)bn);
        break;
      case kEpiResAdd:
        splitk_reduce_kernel<kEpiResAdd><<<(::gsb::count_launch(), blocks), 256, 0, stream>>>(grp.ws, parts, M, N, epi.scale, rp, epi.ldr,
                                                                    out.data_ptr(), out.stride(0), (int)bn);
        break;
      case kEpiSwiGLU:
        splitk_reduce_kernel<kEpiSwiGLU><<<(::gsb::count_launch(), blocks), 256, 0, stream>>>(grp.ws, parts, M, N, epi.scale, rp, epi.ldr,
                                                                    out.data_ptr(), out.stride(0), (int)bn);
        break;
      default:
        splitk_reduce_kernel<kEpiF32><<<(::gsb::count_launch(), blocks), 256, 0, stream>>>(grp.ws, parts, M, N, epi.scale, rp, epi.ldr,
                                                                 out.data_ptr(), out.stride(0), (int)bn);
    }
    GSB_CUDA_CHECK(cudaGetLastError());
  }
}

// Sets the largest output-tile count at which single-CTA GEMMs split K (0: never);
// returns the previous value.
int64_t gsb_gemm_splitk_max_tiles(int64_t v) {
  const int64_t old = gsb::g_splitk_max_tiles;
  if (v >= 0) gsb::g_splitk_max_tiles = (int)v;
  return old;
}

// Sets the smallest M served by the CTA-pair kernel (negative: never); returns
// the previous value.
int64_t gsb_gemm_pair_min_m(int64_t m) {
  const int64_t old = gsb::g_pair_min_m;
  gsb::g_pair_min_m = (int)m;
  return old;
}
