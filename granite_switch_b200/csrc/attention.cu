// Paged causal GQA attention over the KV cache, for chunked prefill and decode.
//
// A CTA owns a tile of "rows" of one request and one KV head, where a row is a
// (query token, query head of that KV group) pair: the GQA heads that share a
// KV head are packed into the M dimension, so every K/V page is read once per
// group. A query at absolute position p attends keys [0, p] (the cached prefix
// plus this chunk), so a chunk that hits the prefix cache attends its cached
// context directly.
//
// K/V pages ([num_blocks, Hkv, 16, D] bf16) are fetched by TMA: the cache is
// viewed as a 2-D tensor of 16-token page rows, each page half (64 columns)
// is one [16 x 64] box with 128-byte swizzle, and one producer thread issues
// all boxes of a key tile against an mbarrier. STAGES tiles are in flight.
// The math is mma.sync m16n8k16 (bf16 -> fp32) with the online softmax in
// registers:
//  * prefill layout: WARPS_M warps x 16 rows, every warp walks every key;
//  * decode layout: 16 rows, the four warps split each key tile and merge
//    their softmax states at the end;
//  * nsplit > 1 splits the key range across CTAs (flash-decoding) and a merge
//    kernel combines the partial results by log-sum-exp.
// (reference: attention comes from vLLM's backends, called at
// src/granite_switch/vllm/decoder/lora/decoder.py:146-174.)
#include "common.cuh"
#include <cstdlib>
#include "tma_util.h"

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

namespace attn {

constexpr int PAGE = 16;  // tokens per KV page

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The same with f16 operands (the fp8 cache path: e4m3 -> f16 is one conversion).
__device__ __forceinline__ void mma16816_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `ch` (of D/8) of row `r` in a tile stored as
// [D/64 halves][ROWS][64 bf16] with the TMA 128-byte swizzle (chunk ^ row%8).
template <int ROWS>
__device__ __forceinline__ uint32_t sw(int r, int ch) {
  return (uint32_t)((ch >> 3) * (ROWS * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

// fp8 pages (kv_fp8.cu): K tiles of D-byte rows keep the TMA swizzle of that row
// width (128 B: 16-byte chunk ^ row % 8; 64 B: chunk ^ (row / 2) % 4), so a warp's 32
// fragment words hit 32 banks.
// e4m3 -> f16 is exact (every e4m3 value is an f16 value).
// Four e4m3 values (one 32-bit word) -> two f16x2: the word's 16-bit halves are split by
// a register move, so the pair costs two conversions and nothing else.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
// bf16x2 * s -> f16x2, saturating at the f16 range.
__device__ __forceinline__ uint32_t bf16x2_to_f16x2_scaled(uint32_t v, float s) {
  const float2 f = unpack_bf16x2(v);
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f.y * s), "f"(f.x * s));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace attn

template <int D, int WARPS_M, int KT, int STAGES, bool F8 = false>
struct AttnCfg {
  static constexpr int WARPS = (WARPS_M == 1) ? 4 : WARPS_M;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int ROWS = 16 * WARPS_M;
  static constexpr int WARPS_N = (WARPS_M == 1) ? 4 : 1;
  static constexpr int KPW = KT / WARPS_N;        // keys per warp per tile
  static constexpr int TILE_BYTES = KT * D * (F8 ? 1 : 2);  // one of K or V
  // fp8: the tile's K then V scales, one 128-byte slot per page (a TMA destination in
  // shared memory must start on a 128-byte boundary; a page's 16 scales use 64 bytes)
  static constexpr int SC_SLOT = 128;
  static constexpr int SC_BYTES = F8 ? 2 * (KT / 16) * SC_SLOT : 0;
  static constexpr int TX_BYTES = 2 * TILE_BYTES + (F8 ? 2 * KT * 4 : 0);  // bytes the TMA loads land per stage
  // stages start on 1024-byte boundaries: the swizzled TMA destinations of the K tiles
  // must be aligned to the swizzle pattern (the fp8 scale arrays would break that)
  static constexpr int STAGE_BYTES = (2 * TILE_BYTES + SC_BYTES + 1023) / 1024 * 1024;
  static_assert(STAGE_BYTES % 1024 == 0 && TILE_BYTES % 1024 == 0, "stage alignment");
  static_assert(TX_BYTES % (KT / 16) == 0, "every page's producer expects the same bytes");
  static constexpr int Q_BYTES = ROWS * D * 2;
  // page ids of the CTA's key range, staged in shared memory once (past this
  // many pages the loop falls back to reading the block table in global memory)
  // (the short decode layouts keep 1024 so that three CTAs fit on an SM)
  static constexpr int PT_CAP = (WARPS_M == 1 && STAGES * TILE_BYTES <= 32768) ? 1024 : 2048;
  static constexpr int SMEM = 1024 + Q_BYTES + STAGES * STAGE_BYTES + 256 + PT_CAP * 4;
  // the decode layout merges its key-split warps through the stage ring
  static_assert(WARPS_M != 1 || STAGES * STAGE_BYTES >= (WARPS_N * 16 * (2 + D)) * 4, "merge scratch");
  static_assert(Q_BYTES % 1024 == 0, "the stage ring starts 1024-byte aligned");
};

// Decode layout (16-row tiles): 2 = short rings (2 stages at head_dim 128, 4 at
// 64) and three CTAs per SM; 3 = deep rings (3 / 6 stages) and two CTAs per SM.
// Both keep the same K/V bytes in flight per SM; the short layout has more warps
// to hide each tile's MMA and softmax latency. Measured on B200 (128 requests x
// 4.2k keys, d=128): 5.86 vs 5.05 TB/s, and 16.4 vs 19.0 ms of decode attention
// in an 8B step. attn_decode_stages() switches it at run time for A/B tests.
static int g_decode_stages = 2;

// F8: the cache is the fp8 layout of kv_fp8.cu (K [blocks, Hkv, 16, D] bytes, V
// [blocks, Hkv, D, 16] bytes, fp32 scales [blocks, Hkv, 16] for each); fragments are
// read as 32-bit words and converted to f16 pairs in registers (one conversion per
// pair; bf16 would take three), so these MMAs run on f16 operands: Q is converted
// once per CTA with the softmax scale folded in (saturating at the f16 range), the K
// scales multiply the scores, the V scales the probabilities, which are packed as f16.
template <int D, int WARPS_M, int KT, int STAGES, bool F8 = false>
__global__ void __launch_bounds__(AttnCfg<D, WARPS_M, KT, STAGES, F8>::THREADS)
    paged_attn_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_ks, const __grid_constant__ CUtensorMap tm_vs,
                      const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                      const int32_t* __restrict__ block_table, int bt_stride, int num_blocks,
                      const int32_t* __restrict__ q_start, const int32_t* __restrict__ kv_len_arr,
                      const int32_t* __restrict__ work_seq, const int32_t* __restrict__ work_row0,
                      int Hq, int Hkv, float scale_log2, __nv_bfloat16* __restrict__ out,
                      int64_t out_stride, float* __restrict__ ws_o, float* __restrict__ ws_lse,
                      int nsplit, int T, uint32_t* err) {
  using namespace attn;
  griddep_launch();  // a GEMM launched as a dependent may start its set-up
  using C = AttnCfg<D, WARPS_M, KT, STAGES, F8>;
  constexpr int ROWS = C::ROWS, WARPS_N = C::WARPS_N, KPW = C::KPW, NB = KPW / 8;
  constexpr int DC = D / 8, OB = D / 8, PAGES = KT / PAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::Q_BYTES;  // [STAGES][K tile | V tile (| K, V scales)]
  uint64_t* full = reinterpret_cast<uint64_t*>(sKV + STAGES * C::STAGE_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = (WARPS_M == 1) ? 0 : warp;
  const int wn = (WARPS_M == 1) ? warp : 0;
  const int w = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int seq = work_seq[w];
  const int row0 = work_row0[w];
  const int G = Hq / Hkv;
  const int qs = q_start[seq];
  const int q_len = q_start[seq + 1] - qs;
  const int kv_len = kv_len_arr[seq];
  const int ctx = kv_len - q_len;
  const int n_rows = q_len * G;
  const int32_t* bt = block_table + (int64_t)seq * bt_stride;

  const int last_row = min(row0 + ROWS, n_rows) - 1;
  const int k_limit = max(0, min(kv_len, ctx + last_row / G + 1));
  int per_split = (k_limit + nsplit - 1) / nsplit;
  per_split = (per_split + KT - 1) / KT * KT;
  const int k_begin = split * per_split;
  const int k_end = min(k_limit, k_begin + per_split);
  const int n_tiles = (k_end > k_begin) ? (k_end - k_begin + KT - 1) / KT : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], PAGES);  // one arrival per page's producer
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    if (F8) {
      tma_prefetch_desc(&tm_ks);
      tma_prefetch_desc(&tm_vs);
    }
  }
  // ---- page ids of [k_begin, k_end) into shared memory: the producer thread
  // then issues each tile's page loads without a dependent global read
  int32_t* s_pages = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(full) + 256);
  const int pg0 = k_begin / PAGE;
  const int n_cached = (n_tiles > 0) ? min((k_end + PAGE - 1) / PAGE - pg0, C::PT_CAP) : 0;
  for (int i = threadIdx.x; i < n_cached; i += C::THREADS) s_pages[i] = checked_index(bt[pg0 + i], num_blocks, err, kSitePage);
  // ---- Q tile via cp.async into the swizzled [half][row][64] layout
  for (int c = threadIdx.x; c < ROWS * DC; c += C::THREADS) {
    const int r = c / DC, ch = c % DC;
    const int gr = row0 + r;
    const bool valid = gr < n_rows;
    const int tok = valid ? gr / G : 0;
    const int head = kvh * G + (valid ? gr % G : 0);
    const __nv_bfloat16* src = q + (int64_t)(qs + tok) * q_stride + head * D + ch * 8;
    cp_async16(smem_u32(sQ) + sw<ROWS>(r, ch), valid ? (const void*)src : (const void*)q, valid);
  }
  cp_commit();
  __syncthreads();  // barrier init visible

  // producers: lane 0 of warp p issues page p of every key tile (one arrival with that
  // page's bytes each), so no warp carries the whole tile's copy issue
  static_assert(PAGES <= C::WARPS, "one producer warp per page");
  const int first_page = checked_index(bt[0], num_blocks, err, kSitePage);
  auto issue = [&](int it, int p) {
    const int s = it % STAGES;
    uint8_t* dK = sKV + s * C::STAGE_BYTES;
    uint8_t* dV = dK + C::TILE_BYTES;
    const int tile_start = k_begin + it * KT;
    mbar_arrive_expect_tx(&full[s], C::TX_BYTES / PAGES);
    {
      const int j = tile_start + p * PAGE;
      // pages past the key range still load a valid page (masked later) so no
      // uninitialised smem (possibly NaN) ever meets a zero probability
      const int pi = j / PAGE - pg0;
      const int page = (j < k_end) ? (pi < n_cached ? s_pages[pi] : checked_index(bt[j / PAGE], num_blocks, err,
                                                                                  kSitePage))
                                   : first_page;
      const int row = (page * Hkv + kvh) * PAGE;
      if (F8) {
        uint8_t* dS = dV + C::TILE_BYTES;
        tma_load_2d(dK + p * PAGE * D, &tm_k, &full[s], 0, row);
        // the transposed V page ([D][16] bytes) is contiguous: one box of D / 16 rows of 256 B
        tma_load_2d(dV + p * PAGE * D, &tm_v, &full[s], 0, (page * Hkv + kvh) * (D / 16));
        tma_load_2d(dS + p * C::SC_SLOT, &tm_ks, &full[s], 0, page * Hkv + kvh);
        tma_load_2d(dS + (PAGES + p) * C::SC_SLOT, &tm_vs, &full[s], 0, page * Hkv + kvh);
      } else {
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          tma_load_2d(dK + h * (KT * 128) + p * PAGE * 128, &tm_k, &full[s], h * 64, row);
          tma_load_2d(dV + h * (KT * 128) + p * PAGE * 128, &tm_v, &full[s], h * 64, row);
        }
      }
    }
  };
  const bool producer = lane == 0 && warp < PAGES;
  int issued = 0;  // tiles whose loads were issued (the same on every producer)
  if (producer) {
    for (int it = 0; it < min(n_tiles, STAGES - 1); ++it) issue(it, warp);
    issued = min(n_tiles, STAGES - 1);
  }

  float o[OB][4];
#pragma unroll
  for (int i = 0; i < OB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int g = lane >> 2, t4 = lane & 3;
  const int rA = wm * 16 + g, rB = rA + 8;
  const int posA = ctx + (row0 + rA) / G;
  const int posB = ctx + (row0 + rB) / G;

  cp_wait_all();
  __syncthreads();
  uint32_t qf[D / 16][4];
  {
    const int r = wm * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int ch = kk * 2 + (lane >> 4);
      ldsm_x4(smem_u32(sQ) + sw<ROWS>(r, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      if (F8) {  // f16 operands with the softmax scale (log2 domain) folded into Q
#pragma unroll
        for (int e = 0; e < 4; ++e) qf[kk][e] = bf16x2_to_f16x2_scaled(qf[kk][e], scale_log2);
      }
    }
  }

  bool ok = true;
  int consumed = 0;
  for (int it = 0; it < n_tiles; ++it) {
    const int s = it % STAGES;
    if (producer && it + STAGES - 1 < n_tiles) {
      issue(it + STAGES - 1, warp);
      issued = it + STAGES;
    }
    const bool landed = mbar_wait(&full[s], (it / STAGES) & 1, err, kErrAttnWait);
    const int tile_start = k_begin + it * KT;
    const uint32_t kbase = smem_u32(sKV + s * C::STAGE_BYTES);
    const uint32_t vbase = kbase + C::TILE_BYTES;
    // fp8 fragments are plain shared-memory loads (ordered after the barrier wait above,
    // free to be scheduled ahead of the MMAs)
    const uint8_t* kst = sKV + s * C::STAGE_BYTES;
    const uint8_t* vst = kst + C::TILE_BYTES;
    // scale of tile key kt: slot kt / 16, entry kt % 16 (slots of C::SC_SLOT bytes)
    const float* kss = reinterpret_cast<const float*>(sKV + s * C::STAGE_BYTES + 2 * C::TILE_BYTES);
    const float* vss = kss + PAGES * (C::SC_SLOT / 4);

    float sacc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int nb2 = 0; nb2 < NB / 2; ++nb2) {
        if (F8) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // sw8: row `key` (key % 8 == g), 16-byte chunk kk ^ (swizzle of g): the chunk bits
            // of the lane's base are g's, so the swizzled offset is one XOR with kk
            const int key = wn * KPW + (2 * nb2 + h) * 8 + g;
            const int off = (key * D + 4 * t4 + ((D == 128 ? g : (g >> 1) & 3) << 4)) ^ (kk << 4);
            uint32_t b0, b1;
            e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(kst + off), b0, b1);
            mma16816_f16(sacc[2 * nb2 + h], qf[kk], b0, b1);
          }
        } else {
          const int key = wn * KPW + nb2 * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = kk * 2 + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + sw<KT>(key, ch), b0, b1, b2, b3);
          mma16816(sacc[2 * nb2], qf[kk], b0, b1);
          mma16816(sacc[2 * nb2 + 1], qf[kk], b2, b3);
        }
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
    // a tile inside both the key range and every row's causal limit needs no mask
    // (CTA-uniform: the first row of the CTA has the smallest position)
    const bool edge = tile_start + KT > min(k_end, ctx + row0 / G + 1);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kt = wn * KPW + nb * 8 + 2 * t4 + (e & 1);
        const int j = tile_start + kt;
        const int pos = (e < 2) ? posA : posB;
        float v = sacc[nb][e] * (F8 ? kss[(kt >> 4) * (C::SC_SLOT / 4) + (kt & 15)] : scale_log2);
        if (edge && (j >= k_end || j > pos)) v = -INFINITY;
        sacc[nb][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mnew = fmaxf(m_r[h], mx[h]);
      corr[h] = (mnew == -INFINITY) ? 1.f : exp2f(m_r[h] - mnew);
      m_r[h] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        const float p = (mm == -INFINITY) ? 0.f : exp2f(sacc[nb][e] - mm);
        sacc[nb][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_r[h] = l_r[h] * corr[h] + rs[h];
    }
    if (F8) {  // the V scales fold into the probabilities (the row sums stay unscaled)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kt = wn * KPW + nb * 8 + 2 * t4 + (e & 1);
          sacc[nb][e] *= vss[(kt >> 4) * (C::SC_SLOT / 4) + (kt & 15)];
        }
    }
    // rescale O only when some row's running max grew in this tile (after the first
    // tiles of a long context it rarely does); warp-uniform, so the MMAs stay converged
    if (__any_sync(0xffffffffu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
      for (int i = 0; i < OB; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[0];
        o[i][2] *= corr[1];
        o[i][3] *= corr[1];
      }
    }
#pragma unroll
    for (int kk = 0; kk < KPW / 16; ++kk) {
      uint32_t pa[4];
      if (F8) {
        pa[0] = pack_f16x2(sacc[2 * kk][0], sacc[2 * kk][1]);
        pa[1] = pack_f16x2(sacc[2 * kk][2], sacc[2 * kk][3]);
        pa[2] = pack_f16x2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
        pa[3] = pack_f16x2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      } else {
        pa[0] = pack_bf16x2(sacc[2 * kk][0], sacc[2 * kk][1]);
        pa[1] = pack_bf16x2(sacc[2 * kk][2], sacc[2 * kk][3]);
        pa[2] = pack_bf16x2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      }
#pragma unroll
      for (int db = 0; db < D / 16; ++db) {
        if (F8) {
          // V^T page of the 16 keys: [D][16 bytes]; one word = keys 2t, 2t+1, 2t+8, 2t+9
          const uint8_t* pg = vst + ((wn * KPW + kk * 16) / PAGE) * (PAGE * D) + g * 16 + 4 * t4;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t b0, b1;
            e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(pg + (db * 16 + h * 8) * 16), b0, b1);
            mma16816_f16(o[2 * db + h], pa, b0, b1);
          }
        } else {
          const int key = wn * KPW + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int ch = db * 2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + sw<KT>(key, ch), b0, b1, b2, b3);
          mma16816(o[2 * db], pa, b0, b1);
          mma16816(o[2 * db + 1], pa, b2, b3);
        }
      }
    }
    // every warp is done with stage s before it is refilled; a lost TMA
    // completion in any thread stops every thread at the same point
    if (!__syncthreads_and(landed)) {
      ok = false;
      break;
    }
    consumed = it + 1;
  }
  if (!ok) {
    // drain the copies that may still land in our shared memory, then leave
    if (threadIdx.x == 0)
      for (int it = consumed; it < issued; ++it)
        mbar_wait(&full[it % STAGES], (it / STAGES) & 1, err, kErrAttnWait);
    __syncthreads();
    return;
  }

  // ---- merge the key-split warps (decode layout)
  if (WARPS_N > 1) {
    float* sm = reinterpret_cast<float*>(sKV);
    float* sl = sm + WARPS_N * 16;
    float* so = sl + WARPS_N * 16;  // [WARPS_N][16][D]
    if (t4 == 0) {
      sm[wn * 16 + g] = m_r[0];
      sm[wn * 16 + g + 8] = m_r[1];
      sl[wn * 16 + g] = l_r[0];
      sl[wn * 16 + g + 8] = l_r[1];
    }
    __syncthreads();
    float my[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      float m = -INFINITY;
      for (int k = 0; k < WARPS_N; ++k) m = fmaxf(m, sm[k * 16 + r]);
      my[h] = (m_r[h] == -INFINITY) ? 0.f : exp2f(m_r[h] - m);
    }
#pragma unroll
    for (int i = 0; i < OB; ++i) {
      const int col = i * 8 + 2 * t4;
      so[(wn * 16 + g) * D + col] = o[i][0] * my[0];
      so[(wn * 16 + g) * D + col + 1] = o[i][1] * my[0];
      so[(wn * 16 + g + 8) * D + col] = o[i][2] * my[1];
      so[(wn * 16 + g + 8) * D + col + 1] = o[i][3] * my[1];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * D; idx += C::THREADS) {
      const int r = idx / D, col = idx % D;
      const int gr = row0 + r;
      if (gr >= n_rows) continue;
      float acc = 0.f, m = -INFINITY, l = 0.f;
      for (int k = 0; k < WARPS_N; ++k) {
        acc += so[(k * 16 + r) * D + col];
        m = fmaxf(m, sm[k * 16 + r]);
      }
      for (int k = 0; k < WARPS_N; ++k) {
        const float mk = sm[k * 16 + r];
        l += (mk == -INFINITY) ? 0.f : sl[k * 16 + r] * exp2f(mk - m);
      }
      const int tok = qs + gr / G, head = kvh * G + gr % G;
      const float val = (l > 0.f) ? acc / l : 0.f;
      if (nsplit == 1) {
        out[(int64_t)tok * out_stride + head * D + col] = f2bf(val);
      } else {
        ws_o[(((int64_t)split * T + tok) * Hq + head) * D + col] = val;
        if (col == 0)
          ws_lse[((int64_t)split * T + tok) * Hq + head] = (l > 0.f) ? (m + log2f(l)) : -INFINITY;
      }
    }
    return;
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = wm * 16 + g + 8 * h;
    const int gr = row0 + r;
    if (gr >= n_rows) continue;
    const int tok = qs + gr / G, head = kvh * G + gr % G;
    const float inv = (l_r[h] > 0.f) ? 1.f / l_r[h] : 0.f;
    if (nsplit == 1) {
      __nv_bfloat16* op = out + (int64_t)tok * out_stride + head * D;
#pragma unroll
      for (int i = 0; i < OB; ++i) {
        const int col = i * 8 + 2 * t4;
        *reinterpret_cast<uint32_t*>(op + col) = pack_bf16x2(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
      }
    } else {
      float* wp = ws_o + (((int64_t)split * T + tok) * Hq + head) * D;
#pragma unroll
      for (int i = 0; i < OB; ++i) {
        const int col = i * 8 + 2 * t4;
        wp[col] = o[i][2 * h] * inv;
        wp[col + 1] = o[i][2 * h + 1] * inv;
      }
      if (t4 == 0)
        ws_lse[((int64_t)split * T + tok) * Hq + head] = (l_r[h] > 0.f) ? (m_r[h] + log2f(l_r[h])) : -INFINITY;
    }
  }
}

// Transpose of an 8x8 b16 matrix across the warp: a lane holds row lane / 4, columns
// 2 (lane % 4) and 2 (lane % 4) + 1 before and after.
__device__ __forceinline__ uint32_t attn_movmatrix_t(uint32_t v) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(v));
  return r;
}

// Decode attention over the fp8 cache with the keys on the MMA's 16-row side: S^T =
// K Q^T and O^T = V^T P^T on m16n8k16 (f16 operands, fp32 accumulators), for work tiles
// of at most 8 query rows (rows_per_tile 8: one decode token's query heads of a KV head,
// or two tokens' at 4 heads per KV head). The row-major layout (paged_attn_kernel,
// 16 query rows as M) spends three quarters of its MMAs, exponentials and softmax
// arithmetic on padding rows when a KV head has 4 query heads; here the 8 query
// columns carry 4 of them, so the tensor and softmax work per key halves while every
// K / V byte is still converted once. The stored fp8 layouts fit as they are: a K row's
// 32-bit word at 4 t holds head dims {2t, 2t+1, 2t+8, 2t+9} of its 16-wide group, the
// A fragment of a 16-key x 16-dim block, and the transposed V page row d holds keys in
// the same order, the A fragment of V^T. The probabilities leave the S^T accumulators
// as the B operand of the second MMA through two movmatrix transposes per 16 keys.
// Four warps take 16 keys (one page) of every 64-key tile each and merge their softmax
// states at the end, as the row-major decode layout does; the stage ring, page-id
// staging and TMA issue are the same.
// Shared memory of paged_attn_fp8t_kernel: the stage ring, the barriers and the page ids
// (no Q tile: Q goes from global memory straight into registers), kept small so that
// four CTAs (3 stages) or five (2 stages, then registers limit) share an SM: the kernel
// is bound by latency, not bandwidth, and needs the warps.
template <int D, int STAGES>
struct Fp8tCfg {
  using A = AttnCfg<D, 1, 64, STAGES, true>;
  static constexpr int PT_CAP = 512;  // page ids staged per CTA (8,192 keys; beyond, global reads)
  static constexpr int SMEM = 1024 + STAGES * A::STAGE_BYTES + 256 + PT_CAP * 4;
};

template <int D, int STAGES>
__global__ void __launch_bounds__(128)
    paged_attn_fp8t_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                           const __grid_constant__ CUtensorMap tm_ks, const __grid_constant__ CUtensorMap tm_vs,
                           const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                           const int32_t* __restrict__ block_table, int bt_stride, int num_blocks,
                           const int32_t* __restrict__ q_start, const int32_t* __restrict__ kv_len_arr,
                           const int32_t* __restrict__ work_seq, const int32_t* __restrict__ work_row0,
                           int Hq, int Hkv, float scale_log2, __nv_bfloat16* __restrict__ out,
                           int64_t out_stride, float* __restrict__ ws_o, float* __restrict__ ws_lse,
                           int nsplit, int T, uint32_t* err) {
  using namespace attn;
  griddep_launch();  // a GEMM launched as a dependent may start its set-up
  using C = AttnCfg<D, 1, 64, STAGES, true>;
  constexpr int KT = 64, PAGES = KT / PAGE, NQ = 8, DB = D / 16, PT_CAP = Fp8tCfg<D, STAGES>::PT_CAP;
  static_assert(C::WARPS == 4 && C::KPW == PAGE, "one 16-key page per warp and tile");
  static_assert(STAGES * C::STAGE_BYTES >= (4 * NQ * (2 + D)) * 4, "merge scratch fits the ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sKV = smem;  // [STAGES][K tile | V tile | K, V scales]
  uint64_t* full = reinterpret_cast<uint64_t*>(sKV + STAGES * C::STAGE_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int w = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int seq = work_seq[w];
  const int row0 = work_row0[w];
  const int G = Hq / Hkv;
  const int qs = q_start[seq];
  const int q_len = q_start[seq + 1] - qs;
  const int kv_len = kv_len_arr[seq];
  const int ctx = kv_len - q_len;
  const int n_rows = q_len * G;
  const int32_t* bt = block_table + (int64_t)seq * bt_stride;

  const int last_row = min(row0 + NQ, n_rows) - 1;
  const int k_limit = max(0, min(kv_len, ctx + last_row / G + 1));
  int per_split = (k_limit + nsplit - 1) / nsplit;
  per_split = (per_split + KT - 1) / KT * KT;
  const int k_begin = split * per_split;
  const int k_end = min(k_limit, k_begin + per_split);
  const int n_tiles = (k_end > k_begin) ? (k_end - k_begin + KT - 1) / KT : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], PAGES);  // one arrival per page's producer
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_ks);
    tma_prefetch_desc(&tm_vs);
  }
  int32_t* s_pages = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(full) + 256);
  const int pg0 = k_begin / PAGE;
  const int n_cached = (n_tiles > 0) ? min((k_end + PAGE - 1) / PAGE - pg0, PT_CAP) : 0;
  for (int i = threadIdx.x; i < n_cached; i += C::THREADS) s_pages[i] = checked_index(bt[pg0 + i], num_blocks, err, kSitePage);
  __syncthreads();  // barrier init and page ids visible

  const int first_page = checked_index(bt[0], num_blocks, err, kSitePage);
  auto issue = [&](int it, int p) {
    const int s = it % STAGES;
    uint8_t* dK = sKV + s * C::STAGE_BYTES;
    uint8_t* dV = dK + C::TILE_BYTES;
    uint8_t* dS = dV + C::TILE_BYTES;
    mbar_arrive_expect_tx(&full[s], C::TX_BYTES / PAGES);
    const int j = k_begin + it * KT + p * PAGE;
    // pages past the key range still load a valid page (masked later)
    const int pi = j / PAGE - pg0;
    const int page = (j < k_end) ? (pi < n_cached ? s_pages[pi] : checked_index(bt[j / PAGE], num_blocks, err,
                                                                                kSitePage))
                                 : first_page;
    tma_load_2d(dK + p * PAGE * D, &tm_k, &full[s], 0, (page * Hkv + kvh) * PAGE);
    tma_load_2d(dV + p * PAGE * D, &tm_v, &full[s], 0, (page * Hkv + kvh) * (D / 16));
    tma_load_2d(dS + p * C::SC_SLOT, &tm_ks, &full[s], 0, page * Hkv + kvh);
    tma_load_2d(dS + (PAGES + p) * C::SC_SLOT, &tm_vs, &full[s], 0, page * Hkv + kvh);
  };
  const bool producer = lane == 0;  // lane 0 of warp p issues page p of every tile
  int issued = 0;
  if (producer) {
    for (int it = 0; it < min(n_tiles, STAGES - 1); ++it) issue(it, warp);
    issued = min(n_tiles, STAGES - 1);
  }

  // B fragments of Q^T (query column g of this tile, f16 with the softmax scale folded in):
  // dims 16 kk + 2 t, +1 and 16 kk + 2 t + 8, +9; zero for columns past the tile's rows
  uint32_t qb[DB][2];
  {
    const int r = row0 + g;
    const bool valid = g < NQ && r < n_rows;
    const __nv_bfloat16* src = q + (int64_t)(qs + (valid ? r / G : 0)) * q_stride + (kvh * G + (valid ? r % G : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < DB; ++kk) {
      const uint32_t lo = valid ? *reinterpret_cast<const uint32_t*>(src + 16 * kk + 2 * t4) : 0u;
      const uint32_t hi = valid ? *reinterpret_cast<const uint32_t*>(src + 16 * kk + 2 * t4 + 8) : 0u;
      qb[kk][0] = bf16x2_to_f16x2_scaled(lo, scale_log2);
      qb[kk][1] = bf16x2_to_f16x2_scaled(hi, scale_log2);
    }
  }
  // this thread's two query columns: 2 t and 2 t + 1 of the tile; their positions
  int pos[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) pos[e] = ctx + (row0 + 2 * t4 + e) / G;

  float o[DB][4];  // O^T: rows d = 16 db + g (+ 8), columns 2 t, 2 t + 1
#pragma unroll
  for (int i = 0; i < DB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_c[2] = {-INFINITY, -INFINITY}, l_c[2] = {0.f, 0.f};
  const int key_lo = warp * PAGE + g;  // this thread's keys in the tile: key_lo, key_lo + 8
  // K word of key key_lo in 16-dim group kk: row key_lo, 16-byte chunk swizzled as
  // kv_fp8.cu stores it; key_lo + 8 has the same swizzle
  const int k_off = key_lo * D + 4 * t4 + ((D == 128 ? g : (g >> 1) & 3) << 4);

  bool ok = true;
  int consumed = 0;
  for (int it = 0; it < n_tiles; ++it) {
    const int s = it % STAGES;
    if (producer && it + STAGES - 1 < n_tiles) {
      issue(it + STAGES - 1, warp);
      issued = it + STAGES;
    }
    const bool landed = mbar_wait(&full[s], (it / STAGES) & 1, err, kErrAttnWait);
    const int tile_start = k_begin + it * KT;
    const uint8_t* kst = sKV + s * C::STAGE_BYTES;
    const uint8_t* vst = kst + C::TILE_BYTES;
    const float* kss = reinterpret_cast<const float*>(kst + 2 * C::TILE_BYTES);
    const float* vss = kss + PAGES * (C::SC_SLOT / 4);

    float sc[4] = {0.f, 0.f, 0.f, 0.f};  // S^T: keys key_lo (0, 1), key_lo + 8 (2, 3)
#pragma unroll
    for (int kk = 0; kk < DB; ++kk) {
      uint32_t a[4];
      const int off = k_off ^ (kk << 4);
      e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(kst + off), a[0], a[2]);
      e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(kst + off + 8 * D), a[1], a[3]);
      mma16816_f16(sc, a, qb[kk][0], qb[kk][1]);
    }
    // K scales (the softmax scale is in Q), masks on edge tiles only
    const float ks_lo = kss[warp * (C::SC_SLOT / 4) + g], ks_hi = kss[warp * (C::SC_SLOT / 4) + g + 8];
    const bool edge = tile_start + KT > min(k_end, ctx + row0 / G + 1);
    float mx[2];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = tile_start + key_lo + (e >> 1) * 8;
      float v = sc[e] * ((e < 2) ? ks_lo : ks_hi);
      if (edge && (j >= k_end || j > pos[e & 1])) v = -INFINITY;
      sc[e] = v;
    }
    mx[0] = fmaxf(sc[0], sc[2]);
    mx[1] = fmaxf(sc[1], sc[3]);
    float corr[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
      const float mnew = fmaxf(m_c[e], mx[e]);
      corr[e] = (mnew == -INFINITY) ? 1.f : exp2f(m_c[e] - mnew);
      m_c[e] = mnew;
    }
    float rs[2];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float mm = m_c[e & 1];
      sc[e] = (mm == -INFINITY) ? 0.f : exp2f(sc[e] - mm);
    }
    rs[0] = sc[0] + sc[2];
    rs[1] = sc[1] + sc[3];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 4);
      rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 8);
      rs[e] += __shfl_xor_sync(0xffffffffu, rs[e], 16);
      l_c[e] = l_c[e] * corr[e] + rs[e];
    }
    // the V scales fold into the probabilities (the sums stay unscaled)
    const float vs_lo = vss[warp * (C::SC_SLOT / 4) + g], vs_hi = vss[warp * (C::SC_SLOT / 4) + g + 8];
    const uint32_t pb0 = attn_movmatrix_t(pack_f16x2(sc[0] * vs_lo, sc[1] * vs_lo));  // keys 2 t, 2 t + 1
    const uint32_t pb1 = attn_movmatrix_t(pack_f16x2(sc[2] * vs_hi, sc[3] * vs_hi));  // keys 2 t + 8, + 9
    if (__any_sync(0xffffffffu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
      for (int i = 0; i < DB; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[1];
        o[i][2] *= corr[0];
        o[i][3] *= corr[1];
      }
    }
    // V^T page of this warp's 16 keys: [D][16 bytes], row d's word at 4 t = keys 2t, 2t+1, 2t+8, 2t+9
    const uint8_t* vp = vst + warp * (PAGE * D) + g * 16 + 4 * t4;
#pragma unroll
    for (int db = 0; db < DB; ++db) {
      uint32_t a[4];
      e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(vp + db * 256), a[0], a[2]);
      e4m3x4_to_f16x2x2(*reinterpret_cast<const uint32_t*>(vp + db * 256 + 128), a[1], a[3]);
      mma16816_f16(o[db], a, pb0, pb1);
    }
    // every warp is done with stage s before it is refilled
    if (!__syncthreads_and(landed)) {
      ok = false;
      break;
    }
    consumed = it + 1;
  }
  if (!ok) {
    if (threadIdx.x == 0)
      for (int it = consumed; it < issued; ++it)
        mbar_wait(&full[it % STAGES], (it / STAGES) & 1, err, kErrAttnWait);
    __syncthreads();
    return;
  }

  // ---- merge the four warps' key slices (the ring is free: every tile was consumed)
  float* sm = reinterpret_cast<float*>(sKV);
  float* sl = sm + 4 * NQ;
  float* so = sl + 4 * NQ;  // [4 warps][NQ columns][D]
  if (g == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sm[warp * NQ + 2 * t4 + e] = m_c[e];
      sl[warp * NQ + 2 * t4 + e] = l_c[e];
    }
  }
  __syncthreads();
  float my[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) m = fmaxf(m, sm[k * NQ + 2 * t4 + e]);
    my[e] = (m_c[e] == -INFINITY) ? 0.f : exp2f(m_c[e] - m);
  }
#pragma unroll
  for (int db = 0; db < DB; ++db) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = 2 * t4 + (e & 1), d = 16 * db + g + (e >> 1) * 8;
      so[(warp * NQ + col) * D + d] = o[db][e] * my[e & 1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < NQ * D; idx += C::THREADS) {
    const int r = idx / D, col = idx % D;
    const int gr = row0 + r;
    if (gr >= n_rows) continue;
    float acc = 0.f, m = -INFINITY, l = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      acc += so[(k * NQ + r) * D + col];
      m = fmaxf(m, sm[k * NQ + r]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float mk = sm[k * NQ + r];
      l += (mk == -INFINITY) ? 0.f : sl[k * NQ + r] * exp2f(mk - m);
    }
    const int tok = qs + gr / G, head = kvh * G + gr % G;
    const float val = (l > 0.f) ? acc / l : 0.f;
    if (nsplit == 1) {
      out[(int64_t)tok * out_stride + head * D + col] = f2bf(val);
    } else {
      ws_o[(((int64_t)split * T + tok) * Hq + head) * D + col] = val;
      if (col == 0) ws_lse[((int64_t)split * T + tok) * Hq + head] = (l > 0.f) ? (m + log2f(l)) : -INFINITY;
    }
  }
}

// Merge flash-decoding partials: out = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M),
// for the (token, head) rows owned by this call's work tiles only. The plans of
// one engine step (decode rows, prefill chunks) write disjoint rows of the same
// output and share the split workspaces, so a merge must leave every other
// row untouched. Block (tile w, KV head, group of 8 tile rows); one warp per
// row, each lane D/32 columns (coalesced 128-byte reads of every split).
template <int D>
__global__ void __launch_bounds__(256) attn_merge_kernel(const float* __restrict__ ws_o,
                                                         const float* __restrict__ ws_lse, int nsplit, int T, int Hq,
                                                         int Hkv, const int32_t* __restrict__ q_start,
                                                         const int32_t* __restrict__ work_seq,
                                                         const int32_t* __restrict__ work_row0, int rows_per_tile,
                                                         __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  griddep_launch();  // a GEMM launched as a dependent may start its set-up
  const int w = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.z * 8 + warp;
  const int G = Hq / Hkv;
  const int seq = work_seq[w], row0 = work_row0[w];
  const int qs = q_start[seq];
  const int gr = row0 + r;
  if (r >= rows_per_tile || gr >= (q_start[seq + 1] - qs) * G) return;
  const int tok = qs + gr / G, head = kvh * G + gr % G;
  if (tok >= T) return;
  const int64_t row = (int64_t)tok * Hq + head, split_stride = (int64_t)T * Hq;
  float m = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m = fmaxf(m, ws_lse[s * split_stride + row]);
  float acc[D / 32];
#pragma unroll
  for (int c = 0; c < D / 32; ++c) acc[c] = 0.f;
  float den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float l = ws_lse[s * split_stride + row];
    if (l == -INFINITY) continue;
    const float wgt = exp2f(l - m);
    const float* o = ws_o + (s * split_stride + row) * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) acc[c] += wgt * o[lane + 32 * c];
    den += wgt;
  }
  __nv_bfloat16* op = out + (int64_t)tok * out_stride + head * D;
#pragma unroll
  for (int c = 0; c < D / 32; ++c) op[lane + 32 * c] = f2bf(den > 0.f ? acc[c] / den : 0.f);
}

template <int D>
static void launch_merge(int n_work, int Hkv, cudaStream_t st, const float* wso, const float* wsl, int nsplit, int T,
                         int Hq, const int32_t* q_start, const int32_t* work_seq, const int32_t* work_row0,
                         int rows_per_tile, void* out, int64_t out_stride) {
  attn_merge_kernel<D><<<(::gsb::count_launch(), dim3(n_work, Hkv, (rows_per_tile + 7) / 8)), 256, 0, st>>>(
      wso, wsl, nsplit, T, Hq, Hkv, q_start, work_seq, work_row0, rows_per_tile, reinterpret_cast<__nv_bfloat16*>(out),
      out_stride);
}

void launch_attn_merge(int D, int n_work, int Hkv, cudaStream_t st, const float* wso, const float* wsl, int nsplit,
                       int T, int Hq, const int32_t* q_start, const int32_t* work_seq, const int32_t* work_row0,
                       int rows_per_tile, void* out, int64_t out_stride) {
  auto merge = (D == 128) ? launch_merge<128> : launch_merge<64>;
  merge(n_work, Hkv, st, wso, wsl, nsplit, T, Hq, q_start, work_seq, work_row0, rows_per_tile, out, out_stride);
}

}  // namespace gsb

using namespace gsb;

template <int D, int WM, int KT, int ST, bool F8 = false>
static void launch_attn(dim3 grid, cudaStream_t st, const CUtensorMap& tk, const CUtensorMap& tv,
                        const CUtensorMap& tks, const CUtensorMap& tvs,
                        const at::Tensor& q, const at::Tensor& bt, int num_blocks, const at::Tensor& q_start,
                        const at::Tensor& kv_len,
                        const at::Tensor& work_seq, const at::Tensor& work_row0, int Hq, int Hkv, float scale_log2,
                        const at::Tensor& out, float* wso, float* wsl, int nsplit, int T, uint32_t* err) {
  using C = AttnCfg<D, WM, KT, ST, F8>;
  auto kfn = paged_attn_kernel<D, WM, KT, ST, F8>;
  static bool configured = false;
  if (!configured) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  kfn<<<(::gsb::count_launch(), grid), C::THREADS, C::SMEM, st>>>(
      tk, tv, tks, tvs, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), bt.data_ptr<int32_t>(),
      (int)bt.stride(0), num_blocks, q_start.data_ptr<int32_t>(), kv_len.data_ptr<int32_t>(),
      work_seq.data_ptr<int32_t>(),
      work_row0.data_ptr<int32_t>(), Hq, Hkv, scale_log2, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      out.stride(0), wso, wsl, nsplit, T, err);
  GSB_CUDA_CHECK(cudaGetLastError());
}

template <int D, int ST>
static void launch_attn_fp8t(dim3 grid, cudaStream_t st, const CUtensorMap& tk, const CUtensorMap& tv,
                             const CUtensorMap& tks, const CUtensorMap& tvs, const at::Tensor& q, const at::Tensor& bt,
                             int num_blocks, const at::Tensor& q_start, const at::Tensor& kv_len,
                             const at::Tensor& work_seq, const at::Tensor& work_row0, int Hq, int Hkv,
                             float scale_log2, const at::Tensor& out, float* wso, float* wsl, int nsplit, int T,
                             uint32_t* err) {
  using C = AttnCfg<D, 1, 64, ST, true>;
  constexpr int SMEM = Fp8tCfg<D, ST>::SMEM;
  auto kfn = paged_attn_fp8t_kernel<D, ST>;
  static bool configured = false;
  if (!configured) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    configured = true;
  }
  kfn<<<(::gsb::count_launch(), grid), C::THREADS, SMEM, st>>>(
      tk, tv, tks, tvs, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), bt.data_ptr<int32_t>(),
      (int)bt.stride(0), num_blocks, q_start.data_ptr<int32_t>(), kv_len.data_ptr<int32_t>(),
      work_seq.data_ptr<int32_t>(), work_row0.data_ptr<int32_t>(), Hq, Hkv, scale_log2,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), wso, wsl, nsplit, T, err);
  GSB_CUDA_CHECK(cudaGetLastError());
}

// Stages of the fp8 decode kernel with 8-row tiles: 2 (five CTAs per SM) or 3 (four).
// Measured on B200 (d=128, 8B decode step of 128 rows over 4.5k keys, CUDA-graph
// replay): 13.7 vs 14.1 ms; the kernel needs warps to hide its conversion and MMA
// latencies more than it needs a deeper ring. attn_fp8t_stages() switches it at run
// time for A/B tests.
static int g_fp8t_stages = 2;
int64_t gsb_attn_fp8t_stages(int64_t v) {
  const int64_t old = g_fp8t_stages;
  if (v == 2 || v == 3) g_fp8t_stages = (int)v;
  return old;
}

int64_t gsb_attn_decode_stages(int64_t v) {
  const int64_t old = g_decode_stages;
  if (v == 2 || v == 3) g_decode_stages = (int)v;
  return old;
}

// q: [T, >= Hq*D] bf16 (row stride q.stride(0)); caches [num_blocks, Hkv, 16, D];
// block_table [S, max_blocks] int32; q_start [S+1] int32 (token offsets of each
// request chunk in q); kv_len [S] int32 (cached + new keys); work_seq/work_row0
// [n_work] int32: the (request, first row) of each CTA tile. rows_per_tile
// selects the layout: 128 (prefill, 8 warps), 64 (prefill, 4 warps), 16
// (decode, warps split keys) or, over an fp8 cache only, 8 (decode with the keys on
// the MMA's row side, tiles of at most 8 rows). out [T, Hq*D] bf16.
void gsb_paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                         const at::Tensor& block_table, const at::Tensor& q_start, const at::Tensor& kv_len,
                         const at::Tensor& work_seq, const at::Tensor& work_row0, int64_t rows_per_tile,
                         int64_t num_q_heads, double scale, const at::Tensor& out, int64_t nsplit,
                         const c10::optional<at::Tensor>& ws_o, const c10::optional<at::Tensor>& ws_lse,
                         const at::Tensor& err, const c10::optional<at::Tensor>& k_scale,
                         const c10::optional<at::Tensor>& v_scale) {
  const bool f8 = k_cache.scalar_type() == at::kByte;
  GSB_CHECK(q.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                (k_cache.scalar_type() == at::kBFloat16 || f8) && v_cache.scalar_type() == k_cache.scalar_type(),
            "attention: bf16 q/out and a bf16 or fp8 (uint8) cache required");
  if (f8) {
    GSB_CHECK(k_cache.dim() == 4 && k_cache.size(2) == attn::PAGE && k_cache.is_contiguous() &&
                  v_cache.is_contiguous() && v_cache.dim() == 4 && v_cache.size(0) == k_cache.size(0) &&
                  v_cache.size(1) == k_cache.size(1) && v_cache.size(2) == k_cache.size(3) &&
                  v_cache.size(3) == attn::PAGE,
              "attention: fp8 caches must be K [num_blocks, Hkv, 16, D] and V [num_blocks, Hkv, D, 16]");
    GSB_CHECK(k_scale.has_value() && v_scale.has_value() && k_scale->scalar_type() == at::kFloat &&
                  v_scale->scalar_type() == at::kFloat && k_scale->is_contiguous() && v_scale->is_contiguous() &&
                  k_scale->numel() == k_cache.size(0) * k_cache.size(1) * attn::PAGE &&
                  v_scale->numel() == k_scale->numel(),
              "attention: fp8 caches need fp32 scales [num_blocks, Hkv, 16]");
  } else {
    GSB_CHECK(k_cache.dim() == 4 && k_cache.size(2) == attn::PAGE && k_cache.is_contiguous() &&
                  v_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes(),
              "attention: caches must be contiguous [num_blocks, Hkv, 16, D]");
  }
  GSB_CHECK(block_table.scalar_type() == at::kInt && q_start.scalar_type() == at::kInt &&
                kv_len.scalar_type() == at::kInt && work_seq.scalar_type() == at::kInt &&
                work_row0.scalar_type() == at::kInt,
            "attention: int32 metadata required");
  const int Hkv = (int)k_cache.size(1);
  const int D = (int)k_cache.size(3);
  const int Hq = (int)num_q_heads;
  GSB_CHECK(Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
  GSB_CHECK(q.stride(1) == 1 && (q.stride(0) % 8) == 0 && out.stride(1) == 1 && (out.stride(0) % 2) == 0,
            "attention: q/out rows must be aligned");
  const int n_work = (int)work_seq.numel();
  const int T = (int)q.size(0);
  if (n_work == 0) return;
  GSB_CHECK(nsplit >= 1 && nsplit <= 64, "attention: nsplit out of range");
  float* wso = nullptr;
  float* wsl = nullptr;
  if (nsplit > 1) {
    GSB_CHECK(ws_o.has_value() && ws_lse.has_value(), "attention: workspaces required for nsplit > 1");
    GSB_CHECK(ws_o->numel() >= nsplit * (int64_t)T * Hq * D && ws_lse->numel() >= nsplit * (int64_t)T * Hq,
              "attention: workspaces too small");
    wso = ws_o->data_ptr<float>();
    wsl = ws_lse->data_ptr<float>();
  }
  const int64_t page_rows = k_cache.size(0) * (int64_t)Hkv * attn::PAGE;
  GSB_CHECK(page_rows < (int64_t(1) << 31), "attention: cache too large for 32-bit TMA coordinates");
  c10::cuda::CUDAGuard guard(q.device());
  auto st = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  CUtensorMap tk, tv, tks, tvs;
  if (f8) {
    const CUtensorMapSwizzle swz = D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    tk = make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, page_rows, D, D, D, attn::PAGE, swz);
    // V pages ([D][16] bytes, contiguous) as rows of 256 bytes: D / 16 rows per page
    tv = make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1,
                      (uint64_t)k_cache.size(0) * Hkv * (D / 16), 256, 256, 256, D / 16, CU_TENSOR_MAP_SWIZZLE_NONE);
    tks = make_tmap_2d(k_scale->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k_cache.size(0) * Hkv,
                       attn::PAGE, attn::PAGE, attn::PAGE, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    tvs = make_tmap_2d(v_scale->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k_cache.size(0) * Hkv,
                       attn::PAGE, attn::PAGE, attn::PAGE, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    tk = make_tmap_bf16_2d(k_cache.data_ptr(), page_rows, D, D, 64, attn::PAGE, CU_TENSOR_MAP_SWIZZLE_128B);
    tv = make_tmap_bf16_2d(v_cache.data_ptr(), page_rows, D, D, 64, attn::PAGE, CU_TENSOR_MAP_SWIZZLE_128B);
    tks = tk;
    tvs = tv;
  }
  uint32_t* ep = reinterpret_cast<uint32_t*>(err.data_ptr());
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  dim3 grid(n_work, Hkv, (unsigned)nsplit);
#define GSB_ATTN(DD, WM, KT, ST)                                                                              \
  launch_attn<DD, WM, KT, ST>(grid, st, tk, tv, tks, tvs, q, block_table, (int)k_cache.size(0), q_start, kv_len, \
                              work_seq, work_row0, Hq, Hkv, \
                              scale_log2, out, wso, wsl, (int)nsplit, T, ep)
#define GSB_ATTN8(DD, WM, KT, ST)                                                                             \
  launch_attn<DD, WM, KT, ST, true>(grid, st, tk, tv, tks, tvs, q, block_table, (int)k_cache.size(0), q_start,  \
                                    kv_len, work_seq, work_row0, Hq, Hkv, scale_log2, out, wso, wsl, (int)nsplit, \
                                    T, ep)
  // fp8 pages are half the bytes, so the rings hold twice as many tiles for the same bytes in flight
  // (decode: three CTAs per SM, as the bf16 short-ring layout)
  GSB_CHECK(rows_per_tile != 8 || f8, "attention: 8-row decode tiles read the fp8 cache only");
  if (f8 && rows_per_tile == 8) {
#define GSB_ATTN8T(DD, ST)                                                                                  \
  launch_attn_fp8t<DD, ST>(grid, st, tk, tv, tks, tvs, q, block_table, (int)k_cache.size(0), q_start, kv_len,   \
                           work_seq, work_row0, Hq, Hkv, scale_log2, out, wso, wsl, (int)nsplit, T, ep)
    if (D == 128 && g_fp8t_stages == 3)
      GSB_ATTN8T(128, 3);
    else if (D == 128)
      GSB_ATTN8T(128, 2);
    else if (D == 64 && g_fp8t_stages == 3)
      GSB_ATTN8T(64, 6);
    else if (D == 64)
      GSB_ATTN8T(64, 4);
    else
      GSB_CHECK(false, "attention: head_dim must be 64 or 128, got ", D);
  } else if (f8 && D == 128) {
    if (rows_per_tile == 128) GSB_ATTN8(128, 8, 64, 4);
    else if (rows_per_tile == 64) GSB_ATTN8(128, 4, 64, 4);
    else GSB_ATTN8(128, 1, 64, 3);
  } else if (f8 && D == 64) {
    if (rows_per_tile == 128) GSB_ATTN8(64, 8, 64, 6);
    else if (rows_per_tile == 64) GSB_ATTN8(64, 4, 64, 6);
    else GSB_ATTN8(64, 1, 64, 6);
  } else if (D == 128) {
    if (rows_per_tile == 128) GSB_ATTN(128, 8, 64, 2);
    else if (rows_per_tile == 64) GSB_ATTN(128, 4, 64, 2);
    else if (g_decode_stages == 2) GSB_ATTN(128, 1, 64, 2);
    else GSB_ATTN(128, 1, 64, 3);
  } else if (D == 64) {
    if (rows_per_tile == 128) GSB_ATTN(64, 8, 64, 3);
    else if (rows_per_tile == 64) GSB_ATTN(64, 4, 64, 3);
    else if (g_decode_stages == 2) GSB_ATTN(64, 1, 64, 4);
    else GSB_ATTN(64, 1, 64, 6);
  } else {
    GSB_CHECK(false, "attention: head_dim must be 64 or 128, got ", D);
  }
#undef GSB_ATTN
#undef GSB_ATTN8
#undef GSB_ATTN8T
  if (nsplit > 1) {
    auto merge = (D == 128) ? launch_merge<128> : launch_merge<64>;
    merge(n_work, Hkv, st, wso, wsl, (int)nsplit, T, Hq, q_start.data_ptr<int32_t>(), work_seq.data_ptr<int32_t>(),
          work_row0.data_ptr<int32_t>(), (int)rows_per_tile, out.data_ptr(), out.stride(0));
    GSB_CUDA_CHECK(cudaGetLastError());
  }
}

// ---------------------------------------------------------------------------
// Allocation-free split-KV decode attention (declared in noalloc_attention.h;
// no counterpart in the reference). Same kernels as the nsplit > 1 decode path
// of gsb_paged_attention, but the fp32 partial outputs and log-sum-exps live
// in a fixed static device array instead of caller-allocated workspaces, and
// the entry point takes raw pointers so a caller without PyTorch (or one that
// may not allocate) can use it.
// ---------------------------------------------------------------------------
#include "noalloc_attention.h"

#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace gsb {
namespace noalloc {

constexpr int64_t kScratchFloats = GSB_NOALLOC_SCRATCH_FLOATS;
constexpr int kMaxDevices = 64;

// Shared by every call on a device; see the header for the sharing rules.
static __device__ __align__(256) float g_scratch[kScratchFloats];

__global__ void fill_neg_inf_kernel(float* __restrict__ p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = -INFINITY;
}

struct DeviceState {
  bool ready = false;
  float* scratch = nullptr;
};
static std::mutex g_mu;
static DeviceState g_state[kMaxDevices];

static int fail(char* msg, size_t len, int code, const char* fmt, ...) {
  if (msg != nullptr && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, len, fmt, ap);
    va_end(ap);
  }
  return code;
}

// Once per device, with that device current: the scratch array's address and
// the kernels' shared-memory limits.
static int setup(int dev, float** scratch, char* msg, size_t len) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& s = g_state[dev];
  if (!s.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(msg, len, GSB_NOALLOC_ECUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    // both decode layouts of each head size (the one used follows attn_decode_stages())
    e = cudaFuncSetAttribute(paged_attn_kernel<128, 1, 64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AttnCfg<128, 1, 64, 2>::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_attn_kernel<128, 1, 64, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               AttnCfg<128, 1, 64, 3>::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_attn_kernel<64, 1, 64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               AttnCfg<64, 1, 64, 4>::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_attn_kernel<64, 1, 64, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               AttnCfg<64, 1, 64, 6>::SMEM);
    if (e != cudaSuccess)
      return fail(msg, len, GSB_NOALLOC_ECUDA, "cudaFuncSetAttribute failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    s.scratch = static_cast<float*>(p);
    s.ready = true;
  }
  *scratch = s.scratch;
  return GSB_NOALLOC_OK;
}

template <int D, int ST>
static void launch_decode(dim3 grid, cudaStream_t st, const CUtensorMap& tk, const CUtensorMap& tv, const void* q,
                          int64_t q_stride, const int32_t* bt, int64_t bt_stride, int num_blocks, const int32_t* q_start,
                          const int32_t* kv_len, const int32_t* work_seq, const int32_t* work_row0, int Hq, int Hkv,
                          float scale_log2, void* out, int64_t out_stride, float* wso, float* wsl, int nsplit, int T,
                          uint32_t* err) {
  using C = AttnCfg<D, 1, 64, ST>;
  paged_attn_kernel<D, 1, 64, ST><<<(::gsb::count_launch(), grid), C::THREADS, C::SMEM, st>>>(
      tk, tv, tk, tv, reinterpret_cast<const __nv_bfloat16*>(q), q_stride, bt, (int)bt_stride, num_blocks, q_start, kv_len,
      work_seq, work_row0, Hq, Hkv, scale_log2, reinterpret_cast<__nv_bfloat16*>(out), out_stride, wso, wsl, nsplit,
      T, err);
  if (nsplit > 1)
    launch_merge<D>((int)grid.x, Hkv, st, wso, wsl, nsplit, T, Hq, q_start, work_seq, work_row0, 16, out, out_stride);
}

}  // namespace noalloc
}  // namespace gsb

extern "C" int gsb_decode_attention_noalloc(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                            int64_t num_blocks, int num_kv_heads, int head_dim,
                                            const int32_t* block_table, int64_t block_table_stride,
                                            const int32_t* q_start, const int32_t* kv_len, const int32_t* work_seq,
                                            const int32_t* work_row0, int num_work, int num_tokens, int num_q_heads,
                                            float scale, int nsplit, void* out, int64_t out_stride, uint32_t* err,
                                            cudaStream_t stream, char* msg, size_t msg_len) {
  using namespace gsb::noalloc;
  if (msg != nullptr && msg_len > 0) msg[0] = '\0';
  if (!q || !k_cache || !v_cache || !block_table || !q_start || !kv_len || !work_seq || !work_row0 || !out || !err)
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "null pointer argument");
  const int D = head_dim, Hq = num_q_heads, Hkv = num_kv_heads, T = num_tokens;
  if (D != 64 && D != 128) return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "head_dim must be 64 or 128, got %d", D);
  if (Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0)
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                Hq, Hkv);
  if (num_work < 0 || T <= 0 || num_blocks <= 0 || block_table_stride <= 0)
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "sizes must be positive");
  if (nsplit < 1 || nsplit > 64) return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "nsplit must be in [1, 64], got %d", nsplit);
  if ((reinterpret_cast<uintptr_t>(q) & 15) || q_stride < (int64_t)Hq * D || q_stride % 8 != 0)
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "q must be 16-byte aligned with a row stride >= Hq*D, multiple of 8");
  if ((reinterpret_cast<uintptr_t>(out) & 3) || out_stride < (int64_t)Hq * D || out_stride % 2 != 0)
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "out must be 4-byte aligned with an even row stride >= Hq*D");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "k_cache and v_cache must be 16-byte aligned");
  const int64_t page_rows = num_blocks * (int64_t)Hkv * attn::PAGE;
  if (page_rows >= (int64_t(1) << 31))
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "cache too large for 32-bit TMA coordinates");
  const int64_t o_floats = (int64_t)nsplit * T * Hq * D;
  const int64_t lse_off = (o_floats + 63) / 64 * 64;  // 256-byte aligned LSE region
  const int64_t need = (nsplit > 1) ? lse_off + (int64_t)nsplit * T * Hq : 0;
  if (need > kScratchFloats)
    return fail(msg, msg_len, GSB_NOALLOC_ETOOBIG,
                "split partials need %lld fp32 values (nsplit %d x tokens %d x heads %d x (head_dim %d + 1)), "
                "over the fixed scratch of %lld; lower nsplit or split the batch",
                (long long)need, nsplit, T, Hq, D, (long long)kScratchFloats);
  if (num_work == 0) return GSB_NOALLOC_OK;

  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(msg, msg_len, GSB_NOALLOC_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "device %d out of range", dev);
  float* scratch = nullptr;
  const int rc = setup(dev, &scratch, msg, msg_len);
  if (rc != GSB_NOALLOC_OK) return rc;
  try {
    const CUtensorMap tk = gsb::make_tmap_bf16_2d(k_cache, page_rows, D, D, 64, attn::PAGE, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tv = gsb::make_tmap_bf16_2d(v_cache, page_rows, D, D, 64, attn::PAGE, CU_TENSOR_MAP_SWIZZLE_128B);
    float* wso = (nsplit > 1) ? scratch : nullptr;
    float* wsl = (nsplit > 1) ? scratch + lse_off : nullptr;
    if (nsplit > 1) {
      const int64_t n = (int64_t)nsplit * T * Hq;
      fill_neg_inf_kernel<<<(::gsb::count_launch(), (unsigned)std::min<int64_t>((n + 255) / 256, 148)), 256, 0, stream>>>(wsl, n);
    }
    const float scale_log2 = (float)(scale * 1.4426950408889634);
    const dim3 grid(num_work, Hkv, nsplit);
    // the same layout choice as gsb_paged_attention: short rings (default) or deep rings
    const bool short_ring = g_decode_stages == 2;
#define GSB_NOALLOC_DECODE(DD, ST)                                                                               \
  launch_decode<DD, ST>(grid, stream, tk, tv, q, q_stride, block_table, block_table_stride, (int)num_blocks,    \
                        q_start, kv_len, work_seq, work_row0, Hq, Hkv, scale_log2, out, out_stride, wso, wsl, \
                        nsplit, T, err)
    if (D == 128) {
      if (short_ring) GSB_NOALLOC_DECODE(128, 2);
      else GSB_NOALLOC_DECODE(128, 3);
    } else {
      if (short_ring) GSB_NOALLOC_DECODE(64, 4);
      else GSB_NOALLOC_DECODE(64, 6);
    }
#undef GSB_NOALLOC_DECODE
  } catch (const std::exception& ex) {
    return fail(msg, msg_len, GSB_NOALLOC_EINVAL, "%s", ex.what());
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(msg, msg_len, GSB_NOALLOC_ECUDA, "launch failed: %s", cudaGetErrorString(e));
  return GSB_NOALLOC_OK;
}
