// LoRA shrink for small token counts on CUDA cores.
//
//   S[m, c] = x[m] . A[c]   for the columns c of row m's own adapter (in every slice),
//   S[m, c] = 0             elsewhere,
//
// the same result as the tensor-core shrink with the adapter-mask epilogue
// (gemm_tcgen05.cu, kEpiMaskAdapter). Column c belongs to adapter (c / rank) %
// adapters + 1 of slice c / (adapters * rank). A decode step of a few tokens needs
// only rank dot products per token and slice, a few hundred kilobytes of A in all:
// the tensor-core kernel's fixed cost (set-up, K split across a cluster and its
// reduction) dominates there, while one block per (token, slice) streams its
// adapter's rank rows once.
// (reference: the shrink is the extra rows of the reference's single cuBLAS GEMM
// against [W; A_1..A_n], src/granite_switch/kernels/switch_lora_kernel.py:134-169.)
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

constexpr int SHRINK_THREADS = 256;
constexpr int SHRINK_ROWS = 8;  // adapter rows (dot products) per block

// grid (M, ceil(n / (adapters * rank)), ceil(rank / 8)): row m, slice s (the last one may
// be the zero padding of A), rows [8 z, 8 z + 8) of the adapter. Every thread takes K / 256
// of the row in 16-byte vectors: per vector it first loads x and the 8 rows of A (nine
// independent loads in flight), then accumulates; the 8 sums are reduced over the warp by
// shuffles and over the 8 warps in shared memory. K % 8 == 0, rows 16-byte aligned.
__global__ void __launch_bounds__(SHRINK_THREADS)
    lora_shrink_small_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ a,
                             int64_t lda, const int32_t* __restrict__ row_adapter, __nv_bfloat16* __restrict__ s,
                             int64_t lds, int K, int rank, int num_adapters, int n_cols) {
  __shared__ float part[SHRINK_THREADS / 32][SHRINK_ROWS];
  griddep_launch();  // the projection GEMM (this kernel's dependent) may start its set-up
  griddep_wait();    // launched as a dependent itself: x is the previous kernel's output
  const int m = blockIdx.x, sl = blockIdx.y, z = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cols = num_adapters * rank;  // columns of one slice
  const int c0 = sl * cols;
  const int ra = row_adapter[m];
  __nv_bfloat16* srow = s + (int64_t)m * lds;
  const int own0 = (ra >= 1 && ra <= num_adapters) ? c0 + (ra - 1) * rank : -1;
  if (z == 0) {  // zero the slice's columns of other adapters
    const int c1 = min(n_cols, c0 + cols);
    for (int c = c0 + threadIdx.x; c < c1; c += SHRINK_THREADS)
      if (own0 < 0 || c < own0 || c >= own0 + rank) srow[c] = __float2bfloat16(0.f);
  }
  if (own0 < 0 || own0 >= n_cols) return;  // block-uniform
  const int own_n = min(rank, n_cols - own0);  // A's zero padding may cut the last slice
  const int j0 = z * SHRINK_ROWS;
  if (j0 >= own_n) return;
  // rows past own_n read row own0 (valid memory); their sums are not stored
  const uint4* arow[SHRINK_ROWS];
#pragma unroll
  for (int r = 0; r < SHRINK_ROWS; ++r)
    arow[r] = reinterpret_cast<const uint4*>(a + (int64_t)(own0 + (j0 + r < own_n ? j0 + r : 0)) * lda);
  const uint4* xv = reinterpret_cast<const uint4*>(x + (int64_t)m * ldx);
  const int nvec = K / 8;
  float acc[SHRINK_ROWS];
#pragma unroll
  for (int r = 0; r < SHRINK_ROWS; ++r) acc[r] = 0.f;
  for (int v = threadIdx.x; v < nvec; v += SHRINK_THREADS) {
    uint4 av[SHRINK_ROWS];
    const uint4 xa = __ldg(xv + v);
#pragma unroll
    for (int r = 0; r < SHRINK_ROWS; ++r) av[r] = __ldg(arow[r] + v);
    float xf[8];
    const uint32_t* px = reinterpret_cast<const uint32_t*>(&xa);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(px[e]);
      xf[2 * e] = f.x;
      xf[2 * e + 1] = f.y;
    }
#pragma unroll
    for (int r = 0; r < SHRINK_ROWS; ++r) {
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&av[r]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(pa[e]);
        acc[r] = fmaf(xf[2 * e], f.x, fmaf(xf[2 * e + 1], f.y, acc[r]));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < SHRINK_ROWS; ++r) {
    const float t = warp_sum(acc[r]);
    if (lane == 0) part[warp][r] = t;
  }
  __syncthreads();
  if (threadIdx.x < SHRINK_ROWS && j0 + threadIdx.x < own_n) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < SHRINK_THREADS / 32; ++w) t += part[w][threadIdx.x];
    srow[own0 + j0 + threadIdx.x] = __float2bfloat16(t);
  }
}

}  // namespace gsb

using namespace gsb;

// x [M, K] bf16, a_all [n, K] bf16 (slices x adapters x rank rows, then zero padding),
// row_adapter [M] int32 (0 = base), s [M, n] bf16.
void gsb_lora_shrink_small(const at::Tensor& x, const at::Tensor& a_all, const at::Tensor& row_adapter,
                           const at::Tensor& s, int64_t rank, int64_t num_adapters) {
  GSB_CHECK(x.scalar_type() == at::kBFloat16 && a_all.scalar_type() == at::kBFloat16 &&
                s.scalar_type() == at::kBFloat16 && row_adapter.scalar_type() == at::kInt,
            "lora_shrink_small: bf16 x / a_all / s and int32 row_adapter required");
  GSB_CHECK(x.dim() == 2 && a_all.dim() == 2 && s.dim() == 2 && x.stride(1) == 1 && a_all.stride(1) == 1 &&
                s.stride(1) == 1,
            "lora_shrink_small: 2-D row-major tensors");
  const int M = (int)x.size(0), K = (int)x.size(1), n = (int)a_all.size(0);
  GSB_CHECK(a_all.size(1) == K && s.size(0) == M && s.size(1) >= n && row_adapter.numel() >= M,
            "lora_shrink_small: shape mismatch");
  GSB_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && a_all.stride(0) % 8 == 0 &&
                (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                (reinterpret_cast<uintptr_t>(a_all.data_ptr()) & 15) == 0,
            "lora_shrink_small: 16-byte aligned rows required");
  GSB_CHECK(rank >= 1 && num_adapters >= 1, "lora_shrink_small: rank and adapters must be positive");
  const int64_t num_slices = (n + num_adapters * rank - 1) / (num_adapters * rank);
  if (M == 0 || n == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  auto st = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const dim3 grid((unsigned)M, (unsigned)num_slices, (unsigned)((rank + SHRINK_ROWS - 1) / SHRINK_ROWS));
  launch_dependent(
      lora_shrink_small_kernel, grid, dim3(SHRINK_THREADS), 0, st, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(a_all.data_ptr()), a_all.stride(0), row_adapter.data_ptr<int32_t>(),
      reinterpret_cast<__nv_bfloat16*>(s.data_ptr()), s.stride(0), K, (int)rank, (int)num_adapters, n);
  GSB_CUDA_CHECK(cudaGetLastError());
}
