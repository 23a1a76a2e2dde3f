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
// No cluster multicast is used, so the kernel is safe on every GPU count.
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

enum EpiKind : int {
  kEpiStore = 0,     // out(bf16) = acc * scale
  kEpiResAdd = 1,    // out(bf16) = residual + acc * scale  (out may alias residual)
  kEpiSwiGLU = 2,    // out(bf16)[:, n/2] = silu(gate) * up, gate/up interleaved per tile
  kEpiMaskAdapter = 3,  // shrink: keep column j only where row's adapter == (j/r)%NA+1
  kEpiF32 = 4,       // out(fp32) = acc * scale
};

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
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;     // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;     // BN * 128 B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN, int EPI, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
    switched_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_b,
                         const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_lb, int M, int N, int K,
                         GemmLoraArgs lora, GemmEpiArgs epi, uint32_t* err) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tmem_full_bar = empty_bar + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;
  const int n0 = n_tile * BN;
  const int m0 = m_tile * C::BM;

  // ---- LoRA schedule for this tile -------------------------------------------
  uint64_t amask = 0;
  int s_base0 = 0, s_base1 = 0;
  if (lora.enabled) {
    amask = lora.tile_mask ? lora.tile_mask[m_tile]
                           : ((lora.num_adapters >= 64) ? ~0ull
                                                        : ((1ull << lora.num_adapters) - 1));
    const int slice_cols = lora.num_adapters * lora.rank_blocks * 32;
    if (SPLIT) {
      s_base0 = 0;
      s_base1 = slice_cols;
    } else {
      int s = 0;
      for (int i = 0; i < lora.num_slices; ++i)
        if (n0 >= lora.slice_bounds[i]) s = i;
      s_base0 = s * slice_cols;
    }
  }
  const int main_blocks = K / C::BK;
  const int lora_blocks = __popcll(amask) * lora.rank_blocks;
  const int total_blocks = main_blocks + (lora.enabled ? lora_blocks : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tmem_full_bar, 1);
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
      int issued = 0;
      int a_iter = 0, rb_iter = 0;  // LoRA cursor: adapter bit index, rank block
      uint64_t rem = amask;
      for (int i = 0; i < total_blocks; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (*abort_flag || !mbar_wait(&empty_bar[s], ph ^ 1, err, kErrGemmWait)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* sa = smem + s * C::STAGE_BYTES;
        uint8_t* sb = sa + C::A_BYTES;
        if (i < main_blocks) {
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          tma_load_2d(sa, &tm_a, &full_bar[s], i * C::BK, m0);
          tma_load_2d(sb, &tm_b, &full_bar[s], i * C::BK, n0);
        } else {
          if (rb_iter == 0) {
            a_iter = __ffsll((long long)rem) - 1;  // adapter bit (kernel-local id - 1)
          }
          const int kcol = a_iter * lora.rank_blocks * 32 + rb_iter * 32;
          const int nsub = SPLIT ? 2 : 1;
          const uint32_t bytes = nsub * (C::BM * 32 * 2) + BN * 32 * 2;
          mbar_arrive_expect_tx(&full_bar[s], bytes);
          tma_load_2d(sa, &tm_s, &full_bar[s], s_base0 + kcol, m0);
          if (SPLIT) tma_load_2d(sa + C::BM * 64, &tm_s, &full_bar[s], s_base1 + kcol, m0);
          tma_load_2d(sb, &tm_lb, &full_bar[s], kcol, n0);
          if (++rb_iter == lora.rank_blocks) {
            rb_iter = 0;
            rem &= rem - 1;
          }
        }
        ++issued;
      }
      // Drain: make sure no TMA write is still in flight into our smem.
      if (*abort_flag) {
        for (int j = (issued > C::STAGES ? issued - C::STAGES : 0); j < issued; ++j)
          mbar_wait(&full_bar[j % C::STAGES], (j / C::STAGES) & 1, err, kErrGemmWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_full = umma_idesc_bf16(128, BN);
      const uint32_t idesc_half = umma_idesc_bf16(128, SPLIT ? BN / 2 : BN);
      bool ok = true;
      for (int i = 0; i < total_blocks; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (*abort_flag || !mbar_wait(&full_bar[s], ph, err, kErrGemmWait)) {
          *abort_flag = 1;
          ok = false;
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
            umma_bf16(tmem_base, ad + 2 * kk, bd + 2 * kk, idesc_full, (i | kk) != 0);
        } else {
          if (SPLIT) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint64_t ad = umma_desc_sw64(sa + u * C::BM * 64);
              const uint64_t bd = umma_desc_sw64(sb + u * (BN / 2) * 64);
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)
                umma_bf16(tmem_base + u * (BN / 2), ad + 2 * kk, bd + 2 * kk, idesc_half, 1);
            }
          } else {
            const uint64_t ad = umma_desc_sw64(sa);
            const uint64_t bd = umma_desc_sw64(sb);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              umma_bf16(tmem_base, ad + 2 * kk, bd + 2 * kk, idesc_full, 1);
          }
        }
        umma_commit(&empty_bar[s]);
      }
      (void)ok;
      umma_commit(tmem_full_bar);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = m0 + q * 32 + lane;
    const bool ok = mbar_wait(tmem_full_bar, 0, err, kErrGemmWait);
    tc_fence_after();
    if (ok && !*abort_flag) {
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16);
      if (EPI == kEpiSwiGLU) {
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + BN / 2 + c, u);
          tmem_wait_ld();
          if (row < M) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(epi.out) + (int64_t)row * epi.ldo +
                               (n0 / 2) + c;
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // The gate/up pre-activations are rounded to bf16 first, as the
              // unfused path stores them in bf16 before the activation.
              float g0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j]) * epi.scale));
              float g1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[2 * j + 1]) * epi.scale));
              float u0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j]) * epi.scale));
              float u1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[2 * j + 1]) * epi.scale));
              pk[j] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            }
            uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              o4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
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
            float* o = reinterpret_cast<float*>(epi.out) + (int64_t)row * epi.ldo + col;
            float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              o4[j] = make_float4(__uint_as_float(r[4 * j]) * epi.scale,
                                  __uint_as_float(r[4 * j + 1]) * epi.scale,
                                  __uint_as_float(r[4 * j + 2]) * epi.scale,
                                  __uint_as_float(r[4 * j + 3]) * epi.scale);
          } else {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * epi.scale;
            if (EPI == kEpiMaskAdapter) {
              // Columns of this chunk belong to one adapter when rank >= 32;
              // evaluate per column to also cover rank 16 groups.
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int a = ((col + j) / epi.mask_rank) % epi.mask_num_adapters + 1;
                if (a != radapter) v[j] = 0.f;
              }
            }
            if (EPI == kEpiResAdd) {
              const uint4* r4 = reinterpret_cast<const uint4*>(epi.residual +
                                                               (int64_t)row * epi.ldr + col);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint4 w = r4[j];
                uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  // Round the projection to bf16 before the residual add, as
                  // the unfused path materialises it in bf16.
                  float2 f = unpack_bf16x2(ww[t]);
                  float p0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * j + 2 * t])));
                  float p1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * j + 2 * t + 1])));
                  v[8 * j + 2 * t] = f.x + p0 * epi.scale;
                  v[8 * j + 2 * t + 1] = f.y + p1 * epi.scale;
                }
              }
            }
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(epi.out) + (int64_t)row * epi.ldo + col;
            uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              o4[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]),
                                 pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                                 pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                                 pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
template <int BN, int EPI, bool SPLIT>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts,
                        const CUtensorMap& tlb, int M, int N, int K, const GemmLoraArgs& lora,
                        const GemmEpiArgs& epi, uint32_t* err, cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kfn = switched_gemm_kernel<BN, EPI, SPLIT>;
  static bool configured = false;  // per instantiation; attribute is per-function
  if (!configured) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES));
    configured = true;
  }
  dim3 grid(N / BN, (M + C::BM - 1) / C::BM);
  kfn<<<grid, 192, C::SMEM_BYTES, stream>>>(ta, tb, ts, tlb, M, N, K, lora, epi, err);
  GSB_CUDA_CHECK(cudaGetLastError());
}

template <int BN>
static void dispatch_epi(int epi_kind, const CUtensorMap& ta, const CUtensorMap& tb,
                         const CUtensorMap& ts, const CUtensorMap& tlb, int M, int N, int K,
                         const GemmLoraArgs& lora, const GemmEpiArgs& epi, uint32_t* err,
                         cudaStream_t st) {
  switch (epi_kind) {
    case kEpiStore: launch_gemm<BN, kEpiStore, false>(ta, tb, ts, tlb, M, N, K, lora, epi, err, st); break;
    case kEpiResAdd: launch_gemm<BN, kEpiResAdd, false>(ta, tb, ts, tlb, M, N, K, lora, epi, err, st); break;
    case kEpiSwiGLU: launch_gemm<BN, kEpiSwiGLU, true>(ta, tb, ts, tlb, M, N, K, lora, epi, err, st); break;
    case kEpiMaskAdapter: launch_gemm<BN, kEpiMaskAdapter, false>(ta, tb, ts, tlb, M, N, K, lora, epi, err, st); break;
    case kEpiF32: launch_gemm<BN, kEpiF32, false>(ta, tb, ts, tlb, M, N, K, lora, epi, err, st); break;
    default: GSB_CHECK(false, "unknown epilogue kind ", epi_kind);
  }
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
                       int64_t mask_num_adapters, const at::Tensor& err) {
  using namespace gsb;
  GSB_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "tensors must be on CUDA");
  GSB_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
            "x and w must be bf16");
  GSB_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1,
            "x and w must be 2-D with unit inner stride");
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)w.size(0);
  GSB_CHECK(w.size(1) == K, "K mismatch");
  GSB_CHECK(bn == 64 || bn == 128 || bn == 256, "bn must be 64, 128 or 256");
  GSB_CHECK(N % bn == 0, "N=", N, " must be a multiple of bn=", bn);
  GSB_CHECK(K % 64 == 0, "K=", K, " must be a multiple of 64");
  GSB_CHECK(M > 0, "M must be positive");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();

  CUtensorMap ta = make_tmap_bf16_2d(x.data_ptr(), M, K, x.stride(0), 64, 128,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_bf16_2d(w.data_ptr(), N, K, w.stride(0), 64, (uint32_t)bn,
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
    tlb = make_tmap_bf16_2d(LB.data_ptr(), N, LB.size(1), LB.stride(0), 32, (uint32_t)bn,
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
  epi.out = out.data_ptr();
  epi.ldo = out.stride(0);
  epi.scale = (float)scale;
  epi.residual = nullptr;
  epi.ldr = 0;
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
    GSB_CHECK(mask_rank > 0 && mask_num_adapters > 0, "mask_rank and mask_num_adapters required");
  }
  uint32_t* errp = reinterpret_cast<uint32_t*>(err.data_ptr());
  switch (bn) {
    case 64: dispatch_epi<64>((int)epi_kind, ta, tb, ts, tlb, M, N, K, lora, epi, errp, stream); break;
    case 128: dispatch_epi<128>((int)epi_kind, ta, tb, ts, tlb, M, N, K, lora, epi, errp, stream); break;
    case 256: dispatch_epi<256>((int)epi_kind, ta, tb, ts, tlb, M, N, K, lora, epi, errp, stream); break;
  }
}
