// Block-scaled fp8 GEMM with the switched-LoRA expand fused (tcgen05, TMEM, TMA).
//
//   out[M, N] = epi( scale * ( X8 . W8^T  (block-scaled e4m3)  +  S . LB^T  (bf16 LoRA expand) ) )
//
// X8 [M, K] and W8 [N, K] are e4m3 bytes, K-major. Their scales are UE8M0 (powers
// of two): one per (token row, 128-element K block) of X and one per (128-row,
// 128-K) block of W, the 1x128 / 128x128 granularity of block-scaled fp8
// checkpoints. Scales are stored as the 512-byte scale-factor atoms the tensor
// core reads: an atom covers 128 rows x 128 K, and byte 16 (r % 32) + 4 (r / 32) + j
// holds row r's scale for K sub-block j (32 elements); the quantisers write one
// value to all four sub-blocks. Atoms are stored [row tile][K tile][512].
//
// Main loop: per 128-K stage one TMA box of X (128 x 128 B) and of W (256 x 128 B),
// both 128-byte swizzled, and three 512-byte bulk copies of scale atoms. The MMA
// thread copies the stage's atoms from shared memory into tensor memory
// (tcgen05.cp 32x128b, broadcast to the four lane quarters) and issues four
// tcgen05.mma kind::mxf8f6f4.block_scale (K = 32 each, scale_vec::1X) whose
// instruction descriptors pick the K sub-block of the scale words. With LoRA, the
// adapters present in the 128-row tile (bitmask) append rank/32 bf16 K-blocks
// (kind::f16, 64-byte swizzled S and LB tiles) into the same fp32 accumulator, as
// the bf16 switched GEMM does; LoRA stays bf16.
//
// Persistent: one CTA per SM walks 128 x 256 output tiles (token tiles fastest, so
// concurrent CTAs share weight tiles in L2). One 256-column accumulator plus a
// scale-factor ring fill the CTA's tensor memory; the epilogue warps release the
// accumulator right after their last tcgen05.ld, so the next tile's main loop
// overlaps their conversion and stores.
//
// The reference serves fp8 base weights through vLLM's quantised linear methods
// (its decoder passes vLLM's quant_config into every projection, reference:
// src/granite_switch/vllm/decoder/lora/decoder.py:62-152) while its switched-LoRA
// kernels stay bf16 (reference: src/granite_switch/kernels/switch_lora_kernel.py).
#include "common.cuh"
#include "gemm_common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_fp8.h>

#include <vector>

namespace gsb {
namespace f8 {

constexpr int BM = 128, BN = 256, BK = 128;  // BK: fp8 elements (bytes) per stage row
constexpr int THREADS = 192;                 // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int A_BYTES = BM * BK;             // 16 KB
constexpr int B_BYTES = BN * BK;             // 32 KB
constexpr int SFA_OFF = A_BYTES + B_BYTES;   // one 512-byte atom
constexpr int SFB_OFF = SFA_OFF + 512;       // two atoms (256 weight rows)
constexpr int STAGE_BYTES = 50 * 1024;       // keeps every stage's swizzled tiles 1024-byte aligned
constexpr int STAGES = 4;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
constexpr int ACC_COLS = BN;                 // fp32 accumulator columns
constexpr int SF_COLS = 16;                  // per stage: A scales 4 columns, B scales 8
constexpr int TMEM_COLS = 512;
static_assert(SFB_OFF + 1024 <= STAGE_BYTES && STAGE_BYTES % 1024 == 0, "stage layout");
static_assert(ACC_COLS + STAGES * SF_COLS <= TMEM_COLS, "tensor memory budget");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
// LoRA stages reuse the ring: S [128 x 32] bf16 at offset 0, LB [256 x 32] bf16 at A_BYTES
static_assert(BM * 64 <= A_BYTES && BN * 64 <= B_BYTES, "LoRA tiles fit a stage");

struct Params {
  int M, N, K, kblocks;
  int m_tiles, n_tiles, num_tiles;
  const uint8_t* sfa;  // [m_tiles][kblocks][512]
  const uint8_t* sfb;  // [2 n_tiles][kblocks][512]
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* residual;
  int64_t ldr;
  float scale;
  // LoRA expand
  int lora, rank_blocks, num_adapters, num_slices;
  int slice_bounds[5];
  const uint64_t* tile_mask;  // [m_tiles] adapters present per 128-row tile
};

// Instruction descriptor, kind::mxf8f6f4 with block scaling: e4m3 A and B, K-major,
// fp32 accumulator, UE8M0 scale factors; sf_id selects the byte (K sub-block) of
// the 32-bit scale words for A and B.
__host__ __device__ constexpr uint32_t idesc_mxf8(int M, int N, int sf_id) {
  return ((uint32_t)sf_id << 4)          // B scale-factor id
         | (0u << 7) | (0u << 10)        // A, B format: E4M3
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | (1u << 23)                    // scale format: UE8M0
         | ((uint32_t)(M >> 4) << 24)    // M / 16
         | ((uint32_t)sf_id << 29);      // A scale-factor id
}

// Shared-memory descriptor of one scale atom as the tcgen05.cp source: 32 rows of
// 16 bytes, no swizzle, 8-row core matrices 128 bytes apart (SBO), one core matrix
// along K (LBO unused).
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version (sm100); layout SWIZZLE_NONE
  return d;
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void umma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`
// (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ int slice_base(const Params& p, int row) {
  int sl = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)  // constant indices keep the parameter block out of local memory
    if (i < p.num_slices && row >= p.slice_bounds[i]) sl = i;
  return sl * p.num_adapters * p.rank_blocks * 32;
}

__device__ __forceinline__ uint64_t tile_adapters(const Params& p, int mt) {
  if (!p.lora) return 0ull;
  if (p.tile_mask == nullptr) return (p.num_adapters >= 64) ? ~0ull : ((1ull << p.num_adapters) - 1);
  return p.tile_mask[mt];
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_lb,
                    const Params p, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);  // one arrival per epilogue warp
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (p.lora) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_lb);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        const int mt = t % p.m_tiles, nt = t / p.m_tiles;
        const int m0 = mt * BM, n0 = nt * BN;
        const uint64_t amask = tile_adapters(p, mt);
        const int total = p.kblocks + __popcll(amask) * p.rank_blocks;
        const int sbase = p.lora ? slice_base(p, n0) : 0;
        for (int i = 0; i < total; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (*abort_flag || !mbar_wait(&empty_bar[s], ph ^ 1, err, kErrGemmWait)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          if (i < p.kblocks) {
            mbar_arrive_expect_tx(&full_bar[s], A_BYTES + B_BYTES + 3 * 512);
            tma_load_2d(st, &tm_a, &full_bar[s], i * BK, m0);
            tma_load_2d(st + A_BYTES, &tm_b, &full_bar[s], i * BK, n0);
            bulk_load(st + SFA_OFF, p.sfa + ((size_t)mt * p.kblocks + i) * 512, 512, &full_bar[s]);
            bulk_load(st + SFB_OFF, p.sfb + ((size_t)(2 * nt) * p.kblocks + i) * 512, 512, &full_bar[s]);
            bulk_load(st + SFB_OFF + 512, p.sfb + ((size_t)(2 * nt + 1) * p.kblocks + i) * 512, 512, &full_bar[s]);
          } else {
            const int j = i - p.kblocks;
            const int ai = j / p.rank_blocks, rb = j % p.rank_blocks;
            uint64_t rem = amask;
            for (int q = 0; q < ai; ++q) rem &= rem - 1;
            const int a_bit = __ffsll((long long)rem) - 1;
            const int kcol = a_bit * p.rank_blocks * 32 + rb * 32;
            mbar_arrive_expect_tx(&full_bar[s], BM * 64 + BN * 64);
            tma_load_2d(st, &tm_s, &full_bar[s], sbase + kcol, m0);
            tma_load_2d(st + A_BYTES, &tm_lb, &full_bar[s], kcol, n0);
          }
        }
      }
      if (*abort_flag) {
        // no copy may still be landing in this CTA's shared memory at exit
        const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, err, kErrGemmWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_bf = umma_idesc_bf16(BM, BN);
      uint32_t it = 0;
      int tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++tl) {
        const int mt = t % p.m_tiles;
        const int total = p.kblocks + __popcll(tile_adapters(p, mt)) * p.rank_blocks;
        // the epilogue has read the previous tile's accumulator
        if (*abort_flag || !mbar_wait(acc_empty, (tl & 1) ^ 1, err, kErrGemmWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int i = 0; i < total; ++i, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (*abort_flag || !mbar_wait(&full_bar[s], ph, err, kErrGemmWait)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          if (i < p.kblocks) {
            // scale atoms of this stage: A -> 4 columns, B (two atoms) -> 8 columns
            const uint32_t tsf = tmem_base + ACC_COLS + s * SF_COLS;
            tmem_cp_sf(tsf, sf_desc(sa + SFA_OFF));
            tmem_cp_sf(tsf + 4, sf_desc(sa + SFB_OFF));
            tmem_cp_sf(tsf + 8, sf_desc(sa + SFB_OFF + 512));
            const uint64_t ad = umma_desc_sw128(sa), bd = umma_desc_sw128(sb);
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk)
              umma_mxf8(tmem_base, ad + 2 * kk, bd + 2 * kk, idesc_mxf8(BM, BN, kk), tsf, tsf + 4, (i | kk) != 0);
          } else {
            const uint64_t ad = umma_desc_sw64(sa), bd = umma_desc_sw64(sb);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) umma_bf16(tmem_base, ad + 2 * kk, bd + 2 * kk, idesc_bf, 1);
          }
          umma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5: TMEM lane quarter warp % 4) ----------------
    const int q = warp & 3;
    int tl = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++tl) {
      const int m0 = (t % p.m_tiles) * BM, n0 = (t / p.m_tiles) * BN;
      if (*abort_flag || !mbar_wait(acc_full, tl & 1, err, kErrGemmWait)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + c + ((uint32_t)(q * 32) << 16), r);
        tmem_wait_ld();
        if (c == BN - 32) {
          // the accumulator is in registers: the next tile's MMAs may start
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty);
        }
        const int col = n0 + c;
        if (m >= p.M || col >= p.N) continue;
        __nv_bfloat16* dst = p.out + (int64_t)m * p.ldo + col;
        const __nv_bfloat16* res = (EPI == kEpiResAdd) ? p.residual + (int64_t)m * p.ldr + col : nullptr;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t pk[4];
          uint4 rv = make_uint4(0u, 0u, 0u, 0u);
          if (EPI == kEpiResAdd) rv = *reinterpret_cast<const uint4*>(res + v * 8);
          const uint32_t rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a0 = __uint_as_float(r[v * 8 + 2 * j]), a1 = __uint_as_float(r[v * 8 + 2 * j + 1]);
            if (EPI == kEpiResAdd) {
              // the projection is rounded to bf16 before the residual add
              const float2 f = unpack_bf16x2(rr[j]);
              pk[j] = pack_bf16x2(f.x + bf16r(a0) * p.scale, f.y + bf16r(a1) * p.scale);
            } else {
              pk[j] = pack_bf16x2(a0 * p.scale, a1 * p.scale);
            }
          }
          *reinterpret_cast<uint4*>(dst + v * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
  }

  if (*abort_flag) {
    // error path: MMAs and copies this CTA issued may still be in flight; give them
    // time to finish before the tensor memory is released (bounded, ~1 ms)
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Activation quantiser: one warp per (row, 128-element K block). Scale
// 2^e with the smallest e such that max|x| / 2^e <= 448 (e4m3's largest finite
// value); values are stored as e4m3(x / 2^e) (exact power-of-two scaling, round to
// nearest, saturating) and the scale byte (e + 127) goes to all four K sub-blocks of
// the row's word in the atom.
__device__ __forceinline__ int ue8m0_exponent(float amax) {
  const float r = __fdiv_rn(amax, 448.f);
  const uint32_t b = __float_as_uint(r);
  const int f = (int)((b >> 23) & 0xffu);
  if (f == 0) return -127;  // zero or subnormal ratio
  int e = f - 127 + ((b & 0x7fffffu) != 0u ? 1 : 0);
  return max(-127, min(126, e));
}

__global__ void quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M, int kblocks,
                                     uint8_t* __restrict__ x8, int64_t ld8, uint8_t* __restrict__ sfa) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x, kb = blockIdx.y * 8 + warp;
  if (row >= M || kb >= kblocks) return;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + (int64_t)row * ldx + kb * 128 + lane * 4);
  const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
  const float amax = warp_max(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
  const int e = ue8m0_exponent(amax);
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e, e in [-127, 126]
  const uint32_t lo = (uint32_t)(uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a.x * inv, a.y * inv), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = (uint32_t)(uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(b.x * inv, b.y * inv), __NV_SATFINITE, __NV_E4M3);
  *reinterpret_cast<uint32_t*>(x8 + (int64_t)row * ld8 + kb * 128 + lane * 4) = lo | (hi << 16);
  if (lane == 0) {
    const uint32_t byte = (uint32_t)(e + 127);
    const int r = row % 128;
    *reinterpret_cast<uint32_t*>(sfa + ((size_t)(row / 128) * kblocks + kb) * 512 + 16 * (r % 32) + 4 * (r / 32)) =
        byte * 0x01010101u;
  }
}

}  // namespace f8
}  // namespace gsb

using namespace gsb;

// x [M, K] bf16 -> x8 [M, K] e4m3 bytes and sfa [ceil(M / 128), K / 128, 512] scale atoms.
void gsb_quantize_fp8_rows(const at::Tensor& x, const at::Tensor& x8, const at::Tensor& sfa, const at::Tensor& err) {
  (void)err;
  GSB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
            "quantize_fp8_rows: bf16 [M, K] input with unit column stride required");
  const int M = (int)x.size(0), K = (int)x.size(1);
  GSB_CHECK(K % 128 == 0 && x.stride(0) % 4 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 7) == 0,
            "quantize_fp8_rows: K must be a multiple of 128 with 8-byte aligned rows");
  GSB_CHECK(x8.scalar_type() == at::kByte && x8.dim() == 2 && x8.size(0) == M && x8.size(1) == K &&
                x8.stride(1) == 1 && x8.stride(0) % 16 == 0,
            "quantize_fp8_rows: uint8 [M, K] output with 16-byte aligned rows required");
  const int kblocks = K / 128;
  GSB_CHECK(sfa.scalar_type() == at::kByte && sfa.is_contiguous() &&
                sfa.numel() >= (int64_t)((M + 127) / 128) * kblocks * 512,
            "quantize_fp8_rows: sfa must hold ceil(M/128) x K/128 atoms of 512 bytes");
  if (M == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  auto st = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
  dim3 grid((unsigned)M, (unsigned)((kblocks + 7) / 8));
  f8::quantize_rows_kernel<<<(::gsb::count_launch(), grid), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), M, kblocks, x8.data_ptr<uint8_t>(),
      x8.stride(0), sfa.data_ptr<uint8_t>());
  GSB_CUDA_CHECK(cudaGetLastError());
}

static int fp8_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    GSB_CUDA_CHECK(cudaGetDevice(&dev));
    GSB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// out [M, N] bf16 = epi(scale * (x8 . w8^T (block scales sfa, sfb) + s . lb^T)).
// x8 [M, K] / w8 [N, K] e4m3 bytes; sfa [ceil(M/128), K/128, 512], sfb
// [2 ceil(N/256), K/128, 512] scale atoms; epi 0 store, 1 residual add. LoRA (optional):
// s [M, slices * adapters * rank] bf16 (masked shrink output), lb [N, adapters * rank]
// bf16, tile_mask [ceil(M/128)] uint64, slice bounds multiples of 256.
void gsb_fp8_gemm(const at::Tensor& x8, const at::Tensor& sfa, const at::Tensor& w8, const at::Tensor& sfb,
                  const at::Tensor& out, int64_t epi, double scale, const c10::optional<at::Tensor>& residual,
                  const c10::optional<at::Tensor>& s, const c10::optional<at::Tensor>& lb,
                  const c10::optional<at::Tensor>& tile_mask, int64_t rank, int64_t num_adapters,
                  std::vector<int64_t> slice_bounds, const at::Tensor& err) {
  using namespace gsb::f8;
  GSB_CHECK(x8.is_cuda() && w8.is_cuda() && out.is_cuda(), "fp8_gemm: CUDA tensors required");
  GSB_CHECK(x8.scalar_type() == at::kByte && w8.scalar_type() == at::kByte, "fp8_gemm: e4m3 operands as uint8");
  GSB_CHECK(x8.dim() == 2 && w8.dim() == 2 && x8.stride(1) == 1 && w8.stride(1) == 1, "fp8_gemm: 2-D K-major operands");
  const int M = (int)x8.size(0), K = (int)x8.size(1), N = (int)w8.size(0);
  GSB_CHECK(w8.size(1) == K && K % 128 == 0 && K > 0, "fp8_gemm: K must match and be a multiple of 128");
  GSB_CHECK(N % 128 == 0, "fp8_gemm: N must be a multiple of 128");
  GSB_CHECK(x8.stride(0) % 16 == 0 && w8.stride(0) % 16 == 0, "fp8_gemm: 16-byte aligned operand rows");
  const int kblocks = K / 128, m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  GSB_CHECK(sfa.scalar_type() == at::kByte && sfa.is_contiguous() && sfa.numel() >= (int64_t)m_tiles * kblocks * 512,
            "fp8_gemm: sfa must hold ceil(M/128) x K/128 atoms");
  GSB_CHECK(sfb.scalar_type() == at::kByte && sfb.is_contiguous() &&
                sfb.numel() >= (int64_t)2 * n_tiles * kblocks * 512,
            "fp8_gemm: sfb must hold 2 ceil(N/256) x K/128 atoms");
  GSB_CHECK((reinterpret_cast<uintptr_t>(sfa.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(sfb.data_ptr()) & 15) == 0,
            "fp8_gemm: 16-byte aligned scale atoms");
  GSB_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) == M && out.size(1) == N &&
                out.stride(1) == 1 && out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
            "fp8_gemm: bf16 [M, N] output with 16-byte aligned rows");
  GSB_CHECK(epi == kEpiStore || epi == kEpiResAdd, "fp8_gemm: epilogue must be store (0) or residual add (1)");
  if (M == 0) return;

  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.kblocks = kblocks;
  p.m_tiles = m_tiles;
  p.n_tiles = n_tiles;
  p.num_tiles = m_tiles * n_tiles;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.scale = (float)scale;
  if (epi == kEpiResAdd) {
    GSB_CHECK(residual.has_value() && residual->scalar_type() == at::kBFloat16 && residual->size(0) == M &&
                  residual->size(1) == N && residual->stride(1) == 1 && residual->stride(0) % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(residual->data_ptr()) & 15) == 0,
              "fp8_gemm: residual add needs a bf16 [M, N] residual with 16-byte aligned rows");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  CUtensorMap ta = make_tmap_2d(x8.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)M, (uint64_t)K,
                                (uint64_t)x8.stride(0), BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(w8.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)N, (uint64_t)K,
                                (uint64_t)w8.stride(0), BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ts = ta, tlb = tb;
  const bool lora = s.has_value() && lb.has_value() && num_adapters > 0 && rank > 0;
  if (lora) {
    GSB_CHECK(rank % 32 == 0 && num_adapters <= 64, "fp8_gemm: LoRA rank must be a multiple of 32, at most 64 adapters");
    GSB_CHECK(s->scalar_type() == at::kBFloat16 && lb->scalar_type() == at::kBFloat16 && s->size(0) == M &&
                  lb->size(0) == N && lb->size(1) >= num_adapters * rank && s->stride(1) == 1 && lb->stride(1) == 1,
              "fp8_gemm: bf16 s [M, *] and lb [N, adapters * rank] required");
    GSB_CHECK(slice_bounds.size() >= 2 && slice_bounds.size() <= 5 && slice_bounds.front() == 0 &&
                  slice_bounds.back() == N,
              "fp8_gemm: slice bounds must run from 0 to N (at most 4 slices)");
    p.num_slices = (int)slice_bounds.size() - 1;
    for (size_t i = 0; i < slice_bounds.size(); ++i) {
      GSB_CHECK(slice_bounds[i] % BN == 0 || slice_bounds[i] == N, "fp8_gemm: slice bounds must be multiples of 256");
      p.slice_bounds[i] = (int)slice_bounds[i];
    }
    GSB_CHECK(s->size(1) >= (int64_t)p.num_slices * num_adapters * rank, "fp8_gemm: s too narrow for the slices");
    p.lora = 1;
    p.rank_blocks = (int)rank / 32;
    p.num_adapters = (int)num_adapters;
    if (tile_mask.has_value()) {
      GSB_CHECK(tile_mask->scalar_type() == at::kLong && tile_mask->numel() >= m_tiles,
                "fp8_gemm: tile_mask must hold one int64 per 128-row tile");
      p.tile_mask = reinterpret_cast<const uint64_t*>(tile_mask->data_ptr());
    }
    ts = make_tmap_bf16_2d(s->data_ptr(), (uint64_t)M, (uint64_t)s->size(1), (uint64_t)s->stride(0), 32, BM,
                           CU_TENSOR_MAP_SWIZZLE_64B);
    tlb = make_tmap_bf16_2d(lb->data_ptr(), (uint64_t)N, (uint64_t)lb->size(1), (uint64_t)lb->stride(0), 32, BN,
                            CU_TENSOR_MAP_SWIZZLE_64B);
  }
  c10::cuda::CUDAGuard g(x8.device());
  auto st = c10::cuda::getCurrentCUDAStream(x8.device().index()).stream();
  auto* ep = reinterpret_cast<uint32_t*>(err.data_ptr());
  const int grid = std::min(p.num_tiles, fp8_num_sms());
  static bool attr_set = false;  // per process: both instantiations at once
  if (!attr_set) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(fp8_gemm_kernel<kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    GSB_CUDA_CHECK(cudaFuncSetAttribute(fp8_gemm_kernel<kEpiResAdd>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    attr_set = true;
  }
  if (epi == kEpiResAdd)
    fp8_gemm_kernel<kEpiResAdd><<<(::gsb::count_launch(), grid), THREADS, SMEM_BYTES, st>>>(ta, tb, ts, tlb, p, ep);
  else
    fp8_gemm_kernel<kEpiStore><<<(::gsb::count_launch(), grid), THREADS, SMEM_BYTES, st>>>(ta, tb, ts, tlb, p, ep);
  GSB_CUDA_CHECK(cudaGetLastError());
}
