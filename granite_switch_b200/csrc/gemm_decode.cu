// Decode-sized switched-LoRA GEMMs (M <= 256 tokens) on tcgen05.
//
// A decode step multiplies a few hundred token rows by every weight matrix:
// the work is a stream of weight bytes with almost no reuse, so the kernel is
// laid out to read each weight byte once, with every SM streaming its share:
//
// * Operands swapped: the MMA's 128-row side (M) is a tile of 128 weight rows
//   and its N side is all Mp tokens (M rounded up to 16, at most 256), so
//   D^T[128 weight rows, Mp tokens] = W_tile . X^T accumulates in TMEM. One
//   weight tile is read once for every token, whatever M is.
// * Split-K over a thread-block cluster: the ks CTAs of a cluster share one
//   weight tile and take contiguous K ranges, so n_tiles * ks CTAs fill the
//   SMs. Each CTA drains its fp32 partial from TMEM into its own shared
//   memory (token-major), then after a cluster barrier every CTA sums a
//   slice of the tokens over all ks partials through distributed shared
//   memory (ld.shared::cluster, fixed order, so the result is deterministic)
//   and applies the epilogue. No global workspace, no second kernel.
// * The LoRA expand rides in the same accumulator: for every adapter present
//   among the step's tokens, rank/32 extra K blocks multiply B_a (weight rows
//   x rank, the A operand) by the masked shrink output S (tokens x rank, the
//   B operand; zero on tokens of other adapters). Those blocks are spread over
//   the cluster's CTAs round-robin.
// * Epilogues: store, residual add, SwiGLU (a tile holds 64 gate rows and the
//   matching 64 up rows, loaded as two TMA boxes), adapter mask (the LoRA
//   shrink itself) and the NVSwitch multicast reduction for tensor parallelism.
//   Rounding follows the general kernel (gemm_tcgen05.cu) bit for bit.
//
// Launched as a programmatic dependent of the kernel before it (when enabled), a
// CTA sets up its barriers and TMEM and puts its first stages' weight tiles in
// flight while that kernel finishes, then waits for it (griddepcontrol.wait)
// before it touches the step's activations.
//
// Warp roles (192 threads): warp 0 issues TMA loads into a ring of stages,
// warp 1 owns TMEM and issues tcgen05.mma from one thread, warps 2..5 drain
// TMEM; all six warps run the cluster reduction and the epilogue. Every wait
// is bounded; a CTA that gives up still arrives at both cluster barriers, so
// its peers never wait on it. TMA loads are plain single-CTA copies from this
// GPU's memory (no multicast).
#include "common.cuh"
#include "gemm_common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>

#include <algorithm>
#include <utility>
#include <vector>

namespace gsb {
namespace dec {

constexpr int BW = 128;        // weight rows per accumulator (the MMA's M)
constexpr int BK = 64;         // K per main block
constexpr int THREADS = 192;
constexpr int MAX_KS = 8;      // portable cluster size
constexpr int MAX_STAGES = 8;
constexpr int RING = 192 * 1024;                      // operand ring (the partial reuses it)
constexpr int SMEM_BYTES = RING + 512 + 1024;         // + barriers + alignment
constexpr int P_STRIDE = BW;                          // fp32 per token row of a drained partial
// Tokens per CTA of a K-split cluster in the reduction: ceil(M / ks) rounded up to 32,
// so every 32-column chunk of an accumulator belongs to one CTA. The receive buffer of
// one accumulator is ks * rows_per rows of P_STRIDE fp32 (the host keeps it in the ring).
__host__ __device__ constexpr int rows_per_part(int M, int ks) { return ((M + ks - 1) / ks + 31) / 32 * 32; }
__host__ __device__ constexpr bool split_fits(int M, int ks) { return ks * rows_per_part(M, ks) * P_STRIDE * 4 <= RING; }
static_assert(split_fits(256, 1) && split_fits(256, 2) && split_fits(256, 4) && split_fits(256, 8),
              "power-of-two splits of 256 tokens fit the ring");

struct Params {
  int M, N, K, Mp, Mp_pad;
  int rows_per;  // rows_per_part(M, ks)
  int ks;            // K parts per tile = cluster size
  int kblocks;       // K / 64
  int stages;        // ring stages (runtime: stage size follows Mp)
  int stage_bytes;   // ACC * 16 KB of W, then the token rows of the k block
  float scale;
  void* out;
  int64_t ldo;
  const __nv_bfloat16* residual;
  int64_t ldr;
  int swiglu_half;   // kEpiSwiGLU: gate (then up) rows per interleave tile
  int lora;
  int rank_blocks;
  int num_adapters;
  int num_slices;
  int slice_bounds[5];
  const uint64_t* tile_mask;  // adapters present per 128-token tile (expand, or shrink tiles to skip)
  const int32_t* row_adapter;
  int mask_rank, mask_num_adapters;
  // optional phase timestamps (%globaltimer, ns) per CTA: [start, set-up done, first
  // stage landed, accumulator ready, partials shared, epilogue done, end, reduction
  // barrier passed, warp 2's partial pushed, every drain warp's partial pushed]
  uint64_t* trace;
};
constexpr int TRACE_SLOTS = 16;

__device__ __forceinline__ void trace_mark(const Params& p, int slot) {
  if (p.trace != nullptr && threadIdx.x % 32 == 0)
    atomicMax(reinterpret_cast<unsigned long long*>(p.trace + blockIdx.x * TRACE_SLOTS + slot),
              (unsigned long long)globaltimer_ns());
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int OFF>
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0+%2], %1;" ::"r"(addr), "f"(v), "n"(OFF));
}

// r[j] -> the fp32 at byte addr + j * P_STRIDE * 4 of a cluster peer's shared memory
// (one store per value, offsets folded into the instruction).
template <int... J>
__device__ __forceinline__ void push_rows32(uint32_t addr, const uint32_t (&r)[32], std::integer_sequence<int, J...>) {
  (st_dsmem_f32<J * P_STRIDE * 4>(addr, __uint_as_float(r[J])), ...);
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Adapters (bits) present among all M tokens.
__device__ __forceinline__ uint64_t present_adapters(const Params& p) {
  if (p.tile_mask == nullptr) return (p.num_adapters >= 64) ? ~0ull : ((1ull << p.num_adapters) - 1);
  uint64_t m = 0;
  for (int t = 0; t < (p.M + 127) / 128; ++t) m |= p.tile_mask[t];
  return m;
}

// Shrink (kEpiMaskAdapter): the tile's columns belong to adapters none of whose
// tokens is in the step, so nothing reads them; the tile is skipped.
__device__ __forceinline__ bool shrink_skipped(const Params& p, int n0, int rows) {
  if (p.tile_mask == nullptr) return false;
  uint64_t need = 0;
  for (int c = 0; c < rows && n0 + c < p.N; c += p.mask_rank)
    need |= 1ull << (((n0 + c) / p.mask_rank) % p.mask_num_adapters);
  return (present_adapters(p) & need) == 0;
}

// S column offset of the LoRA slice holding weight row `row` (a 128-row
// accumulator lies within one slice; the host checks the bounds).
__device__ __forceinline__ int slice_base(const Params& p, int row) {
  int sl = 0;
  for (int i = 0; i < p.num_slices; ++i)
    if (row >= p.slice_bounds[i]) sl = i;
  return sl * p.num_adapters * p.rank_blocks * 32;
}

// Global inputs of an epilogue item (loaded ahead of the reduction, so their
// latency overlaps it): the residual's 8 values and the row's adapter.
struct EpiIn {
  uint4 res;
  int ra;
};

template <int EPI>
__device__ __forceinline__ EpiIn epilogue_inputs(const Params& p, int m, int col) {
  EpiIn in{make_uint4(0u, 0u, 0u, 0u), 0};
  if (EPI == kEpiResAdd || (EPI == kEpiMultimemRed && p.residual != nullptr))
    in.res = *reinterpret_cast<const uint4*>(p.residual + (int64_t)m * p.ldr + col);
  if (EPI == kEpiMaskAdapter) in.ra = p.row_adapter[m];
  return in;
}

template <int EPI>
__device__ __forceinline__ void epilogue8(const Params& p, int m, int col, const float (&v)[8], const float (&u)[8],
                                          const EpiIn& in) {
  if (EPI == kEpiSwiGLU) {
    uint32_t pk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // gate / up rounded to bf16 first, as the unfused path stores them
      const float g0 = bf16r(v[2 * j]), g1 = bf16r(v[2 * j + 1]);
      const float u0 = bf16r(u[2 * j]), u1 = bf16r(u[2 * j + 1]);
      pk[j] = pack_bf16x2(__fdividef(g0, 1.f + __expf(-g0)) * u0, __fdividef(g1, 1.f + __expf(-g1)) * u1);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)m * p.ldo + col) =
        make_uint4(pk[0], pk[1], pk[2], pk[3]);
    return;
  }
  float o[8];
  const bool has_res = (EPI == kEpiResAdd) || (EPI == kEpiMultimemRed && p.residual != nullptr);
  if (has_res) {
    const uint32_t rr[4] = {in.res.x, in.res.y, in.res.z, in.res.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // the projection is rounded to bf16 before the residual add
      const float2 f = unpack_bf16x2(rr[j]);
      o[2 * j] = f.x + bf16r(v[2 * j]) * p.scale;
      o[2 * j + 1] = f.y + bf16r(v[2 * j + 1]) * p.scale;
    }
  } else if (EPI == kEpiMultimemRed) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = bf16r(v[j]) * p.scale;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = v[j] * p.scale;
    if (EPI == kEpiMaskAdapter) {
      // the 8 columns share one adapter: mask_rank is a multiple of 8 (checked by the host)
      if ((col / p.mask_rank) % p.mask_num_adapters + 1 != in.ra) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
      }
    }
  }
  const uint4 pk = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                              pack_bf16x2(o[6], o[7]));
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)m * p.ldo + col;
  if (EPI == kEpiMultimemRed)
    multimem_red_add_v4_bf16x2(dst, pk.x, pk.y, pk.z, pk.w);
  else
    *reinterpret_cast<uint4*>(dst) = pk;
}

// ACC accumulators of 128 weight rows each share every token tile: a CTA owns
// 128 * ACC weight rows, and the tokens' bytes it reads per weight byte drop by ACC.
template <int ACC, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_lb, const __grid_constant__ CUtensorMap tm_s,
                       const Params p, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + RING);
  uint64_t* empty_bar = full_bar + MAX_STAGES;
  uint64_t* tfull_bar = empty_bar + MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) trace_mark(p, 0);
  const int ks = p.ks, stages = p.stages;
  const int part = ks > 1 ? (int)cluster_ctarank() : 0;
  const int tile = blockIdx.x / ks;
  const int n0 = tile * BW * ACC;  // first row of the tile in the (packed) weight
  if (EPI == kEpiMaskAdapter) {
    // the skip test reads the step's adapter masks, which an earlier kernel writes
    griddep_wait();
    if (shrink_skipped(p, n0, BW * ACC)) return;  // the whole cluster skips alike
  }

  // this CTA's blocks: a contiguous K range, then every ks-th LoRA block (their count
  // depends on the step's adapters, read after the dependency wait below)
  const int kb_lo = part * p.kblocks / ks, kb_hi = (part + 1) * p.kblocks / ks;
  const int n_main = kb_hi - kb_lo;
  const int w_bytes = ACC * BW * BK * 2;
  const int need_cols = ACC * p.Mp_pad;
  const int tcols = need_cols <= 32 ? 32 : (need_cols <= 64 ? 64 : (need_cols <= 128 ? 128 : (need_cols <= 256 ? 256 : 512)));

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
    if (p.lora) {
      tma_prefetch_desc(&tm_lb);
      tma_prefetch_desc(&tm_s);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0) trace_mark(p, 1);
  // The next kernel may start its own set-up now; it waits for this grid's end before
  // it reads anything this grid writes.
  griddep_launch();

  // main block i's weight tiles into stage s (the stage's barrier expects them and
  // the block's token tile)
  auto load_w_main = [&](int i, int s) {
    uint8_t* sa = smem + s * p.stage_bytes;
    const int kx = (kb_lo + i) * BK;
    mbar_arrive_expect_tx(&full_bar[s], w_bytes + p.Mp * BK * 2);
#pragma unroll
    for (int a = 0; a < ACC; ++a) {
      if (EPI == kEpiSwiGLU) {
        // out columns [64 (ACC tile + a), +64): their gate rows, then their up rows
        const int o0 = (tile * ACC + a) * 64, it = o0 / p.swiglu_half, off = o0 % p.swiglu_half;
        const int g0 = it * 2 * p.swiglu_half + off;
        tma_load_2d(sa + a * BW * 128, &tm_w, &full_bar[s], kx, g0);
        tma_load_2d(sa + a * BW * 128 + 64 * 128, &tm_w, &full_bar[s], kx, g0 + p.swiglu_half);
      } else {
        tma_load_2d(sa + a * BW * 128, &tm_w, &full_bar[s], kx, n0 + a * BW);
      }
    }
  };
  auto load_x_main = [&](int i, int s) {
    tma_load_2d(smem + s * p.stage_bytes + w_bytes, &tm_x, &full_bar[s], (kb_lo + i) * BK, 0);
  };
  // Weights are constant: the producer puts the weight tiles of its first ring's worth
  // of main blocks in flight before it waits for the previous kernel (launched as its
  // programmatic dependent, this kernel may start while that one still runs). Every
  // thread waits before it reads the step's activations or adapter masks.
  const int prefetch = (warp == 0 && lane == 0) ? min(stages, n_main) : 0;
  for (int i = 0; i < prefetch; ++i) load_w_main(i, i);  // fresh ring: no empty-slot wait
  griddep_wait();
  const uint64_t amask = (EPI != kEpiMaskAdapter && p.lora) ? present_adapters(p) : 0ull;
  const int n_lora_all = __popcll(amask) * p.rank_blocks;
  const int n_lora = n_lora_all > part ? (n_lora_all - part + ks - 1) / ks : 0;
  const int total = n_main + n_lora;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int i = 0; i < prefetch; ++i) load_x_main(i, i);
      uint32_t issued = (uint32_t)prefetch;
      for (int i = prefetch; i < total; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (*abort_flag || !mbar_wait(&empty_bar[s], ph ^ 1, err, kErrGemmWait)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* sa = smem + s * p.stage_bytes;
        uint8_t* sb = sa + w_bytes;
        if (i < n_main) {
          load_w_main(i, s);
          load_x_main(i, s);
        } else {
          const int j = part + (i - n_main) * ks;  // global LoRA block index
          const int ai = j / p.rank_blocks, rb = j % p.rank_blocks;
          uint64_t rem = amask;
          for (int t = 0; t < ai; ++t) rem &= rem - 1;
          const int a_bit = __ffsll((long long)rem) - 1;
          const int kcol = a_bit * p.rank_blocks * 32 + rb * 32;
          mbar_arrive_expect_tx(&full_bar[s], ACC * (BW * 64 + p.Mp * 64));
#pragma unroll
          for (int a = 0; a < ACC; ++a) {
            tma_load_2d(sa + a * BW * 64, &tm_lb, &full_bar[s], kcol, n0 + a * BW);
            tma_load_2d(sb + a * p.Mp_pad * 64, &tm_s, &full_bar[s], slice_base(p, n0 + a * BW) + kcol, 0);
          }
        }
        ++issued;
      }
      if (*abort_flag) {
        // no TMA write may still be in flight into this CTA's shared memory at exit
        const uint32_t first = issued > (uint32_t)stages ? issued - stages : 0;
        for (uint32_t j = first; j < issued; ++j)
          mbar_wait(&full_bar[j % stages], (j / stages) & 1, err, kErrGemmWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(BW, p.Mp);
      bool ok = true;
      for (int i = 0; i < total; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (*abort_flag || !mbar_wait(&full_bar[s], ph, err, kErrGemmWait)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (i == 0 && p.trace != nullptr)
          p.trace[blockIdx.x * TRACE_SLOTS + 2] = globaltimer_ns();
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * p.stage_bytes);
        const uint32_t sb = sa + w_bytes;
        if (i < n_main) {
          const uint64_t bd = umma_desc_sw128(sb);
#pragma unroll
          for (int a = 0; a < ACC; ++a) {
            const uint64_t ad = umma_desc_sw128(sa + a * BW * 128);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_bf16(tmem_base + a * p.Mp_pad, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0);
          }
        } else {
#pragma unroll
          for (int a = 0; a < ACC; ++a) {
            const uint64_t ad = umma_desc_sw64(sa + a * BW * 64), bd = umma_desc_sw64(sb + a * p.Mp_pad * 64);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) umma_bf16(tmem_base + a * p.Mp_pad, ad + 2 * kk, bd + 2 * kk, idesc, 1);
          }
        }
        umma_commit(&empty_bar[s]);
      }
      if (ok) umma_commit(tfull_bar);
    }
  }
  // Reduction over the cluster, one accumulator at a time. Token m belongs to CTA
  // owner(m) = m / rows_per of the cluster. After every CTA's main loop is done (the
  // shared-memory rings are free), the drain warps push their fp32 partial rows from
  // TMEM straight into the owner's receive buffer R[part][m - owner's first row][128]
  // with remote shared-memory stores, which need no round trip; after a second
  // cluster barrier each CTA sums its rows over the ks parts from its own shared
  // memory, in a fixed order (deterministic), and applies the epilogue.
  bool ready = false;
  if (warp >= 2) {
    ready = !*abort_flag && mbar_wait(tfull_bar, 0, err, kErrGemmWait);
    if (!ready) *abort_flag = 1;
    else tc_fence_after();
    if (warp == 2) trace_mark(p, 3);
  }
  const int rows_per = p.rows_per;
  const uint32_t rbase = smem_u32(smem);
  const float* R = reinterpret_cast<const float*>(smem);
#pragma unroll 1
  for (int a = 0; a < ACC; ++a) {
    __syncthreads();
    if (ks > 1) cluster_sync();  // a == 0: every main loop is done; a > 0: the last sums read R
    if (warp == 2) trace_mark(p, 7);
    if (warp >= 2 && ready) {
      const int q = warp & 3;  // the TMEM lane quarter this warp may read
      const int n = q * 32 + lane;
      // token m goes to row (part * rows_per + m - owner * rows_per) of CTA owner's R,
      // owner = m / rows_per; rows_per is a multiple of 32, so one 32-token chunk has
      // one owner and each value is one store at a fixed offset from the chunk's base
      float* Rw = reinterpret_cast<float*>(smem);
      for (int c = 0, owner = 0, oc = 0; c < p.M; c += 32) {
        if (c - oc >= rows_per) {
          ++owner;
          oc += rows_per;
        }
        uint32_t r[32];
        tmem_ld32(tmem_base + a * p.Mp_pad + c + ((uint32_t)(q * 32) << 16), r);
        tmem_wait_ld();
        const int row = part * rows_per + c - oc;  // rows past M land in the owner's buffer, unread
        if (ks > 1) {
          push_rows32(mapa_shared(rbase + (uint32_t)(row * P_STRIDE + n) * 4u, (uint32_t)owner), r,
                      std::make_integer_sequence<int, 32>{});
        } else {
          float* dst = Rw + row * P_STRIDE + n;
#pragma unroll
          for (int j = 0; j < 32; ++j) dst[j * P_STRIDE] = __uint_as_float(r[j]);
        }
      }
      if (warp == 2) trace_mark(p, 8);
      trace_mark(p, 9);
    }
    __syncthreads();
    if (ks > 1) cluster_sync();  // every partial row has landed in its owner's R
    if (warp == 0) trace_mark(p, 4);
    if (!*abort_flag) {
      const int r0 = part * rows_per, r1 = min(p.M, r0 + rows_per);
      constexpr int GROUPS = (EPI == kEpiSwiGLU) ? 8 : 16;  // 8-column groups per token row
      const int n_items = max(0, r1 - r0) * GROUPS;
      const int row0 = n0 + a * BW;
      for (int it = threadIdx.x; it < n_items; it += THREADS) {
        const int lm = it / GROUPS, c = (it % GROUPS) * 8, m = r0 + lm;
        const int col = (EPI == kEpiSwiGLU) ? (tile * ACC + a) * 64 + c : row0 + c;
        if (EPI != kEpiSwiGLU && col >= p.N) continue;
        const EpiIn ein = epilogue_inputs<EPI>(p, m, col);
        float v[8], u[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = u[j] = 0.f;
#pragma unroll 1
        for (int q = 0; q < ks; ++q) {
          const float* src = R + (q * rows_per + lm) * P_STRIDE + c;
          const float4 a0 = *reinterpret_cast<const float4*>(src), a1 = *reinterpret_cast<const float4*>(src + 4);
          v[0] += a0.x; v[1] += a0.y; v[2] += a0.z; v[3] += a0.w;
          v[4] += a1.x; v[5] += a1.y; v[6] += a1.z; v[7] += a1.w;
          if (EPI == kEpiSwiGLU) {
            const float4 b0 = *reinterpret_cast<const float4*>(src + 64), b1 = *reinterpret_cast<const float4*>(src + 68);
            u[0] += b0.x; u[1] += b0.y; u[2] += b0.z; u[3] += b0.w;
            u[4] += b1.x; u[5] += b1.y; u[6] += b1.z; u[7] += b1.w;
          }
        }
        epilogue8<EPI>(p, m, col, v, u, ein);
      }
    }
    trace_mark(p, 5);
  }
  if (*abort_flag) {
    // error path: MMAs and copies this CTA issued may still be in flight; give them
    // time to finish before the tensor memory is released (bounded, ~1 ms)
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) {
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
  if (warp == 0) trace_mark(p, 6);
}

}  // namespace dec

// Largest M served by the decode kernel (0 turns it off; gemm_decode_max_m()
// changes it at run time for A/B tests).
static int g_decode_max_m = 256;

static int dec_num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  GSB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  GSB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int ACC, int EPI>
static void launch_decode(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tlb,
                          const CUtensorMap& ts, const dec::Params& p, int n_tiles, uint32_t* err,
                          cudaStream_t stream) {
  auto kfn = dec::decode_gemm_kernel<ACC, EPI>;
  static bool configured = false;  // per instantiation
  if (!configured) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::SMEM_BYTES));
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_tiles * p.ks), 1, 1);
  cfg.blockDim = dim3(dec::THREADS, 1, 1);
  cfg.dynamicSmemBytes = dec::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n_attr = 0;
  if (p.ks > 1) {
    attr[n_attr].id = cudaLaunchAttributeClusterDimension;
    attr[n_attr].val.clusterDim.x = (unsigned)p.ks;
    attr[n_attr].val.clusterDim.y = 1;
    attr[n_attr].val.clusterDim.z = 1;
    ++n_attr;
  }
  // a programmatic dependent of the previous kernel (not while tracing: the caller
  // zeroes the trace buffer with a kernel that an early start would race)
  if (pdl_enabled() && p.trace == nullptr) {
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n_attr;
  count_launch();
  GSB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kfn, tw, tx, tlb, ts, p, err));
}

template <int ACC>
static void dispatch_decode(int epi, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tlb,
                            const CUtensorMap& ts, const dec::Params& p, int n_tiles, uint32_t* err,
                            cudaStream_t st) {
  switch (epi) {
    case kEpiStore: launch_decode<ACC, kEpiStore>(tw, tx, tlb, ts, p, n_tiles, err, st); break;
    case kEpiResAdd: launch_decode<ACC, kEpiResAdd>(tw, tx, tlb, ts, p, n_tiles, err, st); break;
    case kEpiSwiGLU: launch_decode<ACC, kEpiSwiGLU>(tw, tx, tlb, ts, p, n_tiles, err, st); break;
    case kEpiMaskAdapter: launch_decode<ACC, kEpiMaskAdapter>(tw, tx, tlb, ts, p, n_tiles, err, st); break;
    case kEpiMultimemRed: launch_decode<ACC, kEpiMultimemRed>(tw, tx, tlb, ts, p, n_tiles, err, st); break;
  }
}

// Clusters of `ks` CTAs of the decode kernel that fit on the GPU at once (queried
// once per device, accumulator count and cluster size; every epilogue variant
// has the same shared memory and block size). Clusters must sit inside one GPC,
// so large clusters leave SMs unused: on B200, 15 clusters of 8 fit (120 CTAs)
// but 33 of 4 (132).
template <int ACC>
static int max_active_clusters(int ks) {
  static int cached[64][dec::MAX_KS + 1] = {{0}};
  int dev = 0;
  GSB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64 && cached[dev][ks]) return cached[dev][ks];
  auto kfn = dec::decode_gemm_kernel<ACC, kEpiStore>;
  GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::SMEM_BYTES));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(ks * dec_num_sms()), 1, 1);
  cfg.blockDim = dim3(dec::THREADS, 1, 1);
  cfg.dynamicSmemBytes = dec::SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = dec_num_sms() / ks;
  }
  if (dev < 64) cached[dev][ks] = n;
  return n;
}

// Split of a call over CTAs: `acc` accumulators (128 * acc weight rows per CTA)
// and `ks` K parts per tile. At a few hundred tokens the tensor work per weight
// byte matches the HBM stream, so every SM has to take part in one wave:
// measured on B200 at M = 222, 96 CTAs with two accumulators ran the 4096-row
// projections 1.3-1.7x slower than 128 CTAs with one, and a second wave of
// clusters doubled the time. The rule: one accumulator and the largest K split
// whose clusters all fit at once (at most one wave, at least four 64-deep K
// blocks per part); when even an unsplit grid of one-accumulator tiles needs a
// second wave, two accumulators per CTA if that fits one wave, else the general
// kernel takes the call (acc = 0).
struct DecodeSplit {
  int acc, ks, n_tiles;
};

// A/B override of the split (gemm_decode_force_split): 0 keeps the rule above.
static int g_force_acc = 0, g_force_ks = 0;
// Phase trace buffer (gemm_decode_trace): uint64 [CTAs][16], or null.
static uint64_t* g_trace = nullptr;

static DecodeSplit choose_split(int N, int M, int kblocks, bool two_ok) {
  if (g_force_acc > 0 && g_force_ks > 0 && (g_force_acc == 1 || two_ok)) {
    int ks = std::min(g_force_ks, std::max(1, kblocks));
    while (ks > 1 && !dec::split_fits(M, ks)) --ks;
    return DecodeSplit{g_force_acc, ks, (N + dec::BW * g_force_acc - 1) / (dec::BW * g_force_acc)};
  }
  const int nsms = dec_num_sms();
  const int t1 = (N + dec::BW - 1) / dec::BW;
  if (t1 <= max_active_clusters<1>(1)) {
    int best = 1;
    for (int ks = 2; ks <= dec::MAX_KS; ++ks) {
      if (kblocks / ks < 4 || t1 * ks > nsms) break;
      if (dec::split_fits(M, ks) && t1 <= max_active_clusters<1>(ks)) best = ks;
    }
    return DecodeSplit{1, best, t1};
  }
  const int t2 = (N + 2 * dec::BW - 1) / (2 * dec::BW);
  if (two_ok && t2 <= max_active_clusters<2>(1)) return DecodeSplit{2, 1, t2};
  return DecodeSplit{0, 0, 0};
}

bool decode_gemm_try(const DecodeGemmArgs& a, uint32_t* err, cudaStream_t stream) {
  const int epi = a.epi;
  if (g_decode_max_m <= 0 || a.M < 1 || a.M > std::min(g_decode_max_m, 256)) return false;
  if (!(epi == kEpiStore || epi == kEpiResAdd || epi == kEpiSwiGLU || epi == kEpiMaskAdapter ||
        epi == kEpiMultimemRed))
    return false;
  if (a.K % 64 != 0 || a.N % 64 != 0) return false;
  const bool lora = a.s != nullptr && a.lb != nullptr && a.num_adapters > 0 && epi != kEpiMaskAdapter;
  if (epi == kEpiSwiGLU && (lora || a.swiglu_tile % 128 != 0 || a.N % a.swiglu_tile != 0)) return false;
  if (epi == kEpiResAdd && a.residual == nullptr) return false;
  if (epi == kEpiMaskAdapter && (a.mask_rank % 8 != 0 || a.mask_rank <= 0 || a.mask_num_adapters <= 0)) return false;
  if (lora) {
    if (a.rank % 32 != 0 || a.num_adapters > 64 || a.num_slices < 1 || a.num_slices > 4) return false;
    for (int i = 0; i < a.num_slices; ++i)
      if (a.slice_bounds[i] % dec::BW != 0) return false;  // a weight tile lies in one slice
  }
  // 16-byte aligned rows for the vector epilogue
  if ((a.ldo % 8) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15) != 0) return false;
  if (a.residual != nullptr && ((a.ldr % 8) != 0 || (reinterpret_cast<uintptr_t>(a.residual) & 15) != 0))
    return false;

  dec::Params p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.Mp = (a.M + 15) / 16 * 16;
  p.Mp_pad = (p.Mp + 31) / 32 * 32;
  p.kblocks = a.K / 64;
  p.scale = a.scale;
  p.out = a.out;
  p.ldo = a.ldo;
  p.residual = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  p.ldr = a.ldr;
  p.swiglu_half = a.swiglu_tile / 2;
  p.trace = g_trace;
  // one or two 128-row accumulators per CTA (two need Mp_pad <= 256 columns each, and
  // for SwiGLU a whole number of 128-column output tiles)
  const bool two_ok = 2 * p.Mp_pad <= 512 && (epi != kEpiSwiGLU || (a.N / 2) % 128 == 0);
  const DecodeSplit sp = choose_split(a.N, a.M, p.kblocks, two_ok);
  if (sp.acc == 0) return false;
  const int acc = sp.acc, n_tiles = sp.n_tiles;
  p.ks = sp.ks;
  p.rows_per = dec::rows_per_part(p.M, p.ks);
  p.stage_bytes = acc * dec::BW * dec::BK * 2 + (p.Mp_pad * dec::BK * 2 + 1023) / 1024 * 1024;
  p.stages = std::min(dec::MAX_STAGES, dec::RING / p.stage_bytes);
  p.lora = lora ? 1 : 0;
  p.tile_mask = nullptr;
  if (lora) {
    p.rank_blocks = a.rank / 32;
    p.num_adapters = a.num_adapters;
    p.num_slices = a.num_slices;
    for (int i = 0; i <= a.num_slices; ++i) p.slice_bounds[i] = a.slice_bounds[i];
    p.tile_mask = a.tile_mask;
  }
  if (epi == kEpiMaskAdapter) {
    p.row_adapter = a.row_adapter;
    p.mask_rank = a.mask_rank;
    p.mask_num_adapters = a.mask_num_adapters;
    p.tile_mask = a.skip_mask;
  }
  const uint32_t mp_box = (uint32_t)p.Mp;
  const CUtensorMap tw = make_tmap_bf16_2d(a.w, (uint64_t)a.N, (uint64_t)a.K, (uint64_t)a.ldw, 64,
                                           epi == kEpiSwiGLU ? 64u : 128u, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tx = make_tmap_bf16_2d(a.x, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.ldx, 64, mp_box,
                                           CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tlb = tw, ts = tx;
  if (lora) {
    tlb = make_tmap_bf16_2d(a.lb, (uint64_t)a.N, (uint64_t)a.num_adapters * a.rank, (uint64_t)a.ldlb, 32, 128,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    ts = make_tmap_bf16_2d(a.s, (uint64_t)a.M, (uint64_t)a.s_cols, (uint64_t)a.lds, 32, mp_box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (acc == 2)
    dispatch_decode<2>(epi, tw, tx, tlb, ts, p, n_tiles, err, stream);
  else
    dispatch_decode<1>(epi, tw, tx, tlb, ts, p, n_tiles, err, stream);
  return true;
}

}  // namespace gsb

// The split the decode kernel would use for an M x N x K call: {accumulators,
// K parts, weight tiles, ring stages}, or {0, 0, 0, 0} when M is out of its range
// (diagnostics and tests).
std::vector<int64_t> gsb_gemm_decode_plan(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t swiglu_tile) {
  using namespace gsb;
  if (M < 1 || M > std::min(g_decode_max_m, 256) || K % 64 != 0) return {0, 0, 0, 0};
  const int Mp = (int)(M + 15) / 16 * 16, Mp_pad = (Mp + 31) / 32 * 32;
  const bool two_ok = 2 * Mp_pad <= 512 && (epi != kEpiSwiGLU || (N / 2) % 128 == 0);
  const DecodeSplit sp = choose_split((int)N, (int)M, (int)(K / 64), two_ok);
  if (sp.acc == 0) return {0, 0, 0, 0};
  const int stage_bytes = sp.acc * dec::BW * dec::BK * 2 + (Mp_pad * dec::BK * 2 + 1023) / 1024 * 1024;
  (void)swiglu_tile;
  return {sp.acc, sp.ks, sp.n_tiles, std::min(dec::MAX_STAGES, dec::RING / stage_bytes)};
}

// Forces the decode kernel's split (accumulators, K parts; 0, 0 restores the rule), for
// A/B measurements.
void gsb_gemm_decode_force_split(int64_t acc, int64_t ks) {
  gsb::g_force_acc = (int)acc;
  gsb::g_force_ks = (int)std::min<int64_t>(ks, gsb::dec::MAX_KS);
}

// Records per-CTA phase timestamps of the following decode-kernel launches into
// `buf` (uint64, 16 per CTA, zeroed by the caller); an empty tensor stops.
void gsb_gemm_decode_trace(const at::Tensor& buf) {
  gsb::g_trace = buf.numel() ? reinterpret_cast<uint64_t*>(buf.data_ptr()) : nullptr;
}

// Sets the largest M served by the decode kernel (0: never); returns the previous value.
int64_t gsb_gemm_decode_max_m(int64_t v) {
  const int64_t old = gsb::g_decode_max_m;
  if (v >= 0) gsb::g_decode_max_m = (int)v;
  return old;
}
