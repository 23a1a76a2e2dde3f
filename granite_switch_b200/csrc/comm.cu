// Tensor-parallel communication kernels over NVLink / NVSwitch peer memory.
//
// * peer_barrier: every rank stores an epoch into its slot of every peer's
//   signal pad (plain P2P st.release.sys) and waits, with a bounded spin, until
//   all peers' epochs arrived in its own pad (ld.acquire.sys). A wait that runs
//   out sets kErrPeerWait and returns; it never hangs. The epoch is a counter in
//   this rank's device memory that every barrier advances, so barriers replayed
//   from a CUDA graph and eager ones stay in one sequence (an epoch passed as a
//   launch argument would be frozen into the graph at capture).
// * rmsnorm_residual_from: h <- y (the reduced residual stream), x <- RMSNorm(y),
//   y <- 0 ready for the next accumulation - one pass over the row.
// The fused row-parallel GEMM (gemm_tcgen05.cu, kEpiMultimemRed) pushes each
// output tile into the multicast buffer with multimem.red as soon as its
// accumulator is drained, so the transfer overlaps the remaining tiles.
// (reference: the one collective of the reference is
// tensor_model_parallel_all_reduce at src/granite_switch/vllm/core/lora.py:575.)
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// signal pads: uint32 [tp] per rank; slot `src` of rank r's pad holds the last
// epoch rank `src` announced to r.
__global__ void peer_barrier_kernel(const uint64_t* __restrict__ pads, int rank, int tp, uint32_t* __restrict__ ctr,
                                    uint64_t budget_ns, uint32_t* err) {
  const int p = threadIdx.x;
  const uint32_t epoch = *ctr + 1;  // read by every thread before thread 0 advances it
  if (p < tp) {
    __threadfence_system();  // this rank's earlier writes (incl. multimem) before the announce
    uint32_t* peer_pad = reinterpret_cast<uint32_t*>(pads[p]);
    st_release_sys(peer_pad + rank, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(pads[rank]) + p;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
      if (globaltimer_ns() - t0 > budget_ns) {
        raise_error(err, kErrPeerWait);
        break;
      }
    }
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x == 0) *ctr = epoch;
}

// h <- y; x <- rmsnorm(y) * w; y <- 0   (rows of H bf16, H % 8 == 0)
template <int VPT>
__global__ void rmsnorm_residual_from_kernel(__nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ h,
                                             const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ x,
                                             int H, float eps) {
  const int r = blockIdx.x;
  uint4* yv = reinterpret_cast<uint4*>(y + (int64_t)r * H);
  uint4* hv = reinterpret_cast<uint4*>(h + (int64_t)r * H);
  uint4* xv = reinterpret_cast<uint4*>(x + (int64_t)r * H);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const int nvec = H / 8;
  uint4 buf[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      buf[i] = yv[v];
      hv[v] = buf[i];
      yv[v] = make_uint4(0, 0, 0, 0);
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&buf[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(p[j]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&buf[i]);
      const uint4 wq = wv[v];
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wq);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(p[j]);
        const float2 g = unpack_bf16x2(pw[j]);
        const float a = __bfloat162float(__float2bfloat16_rn(f.x * inv));
        const float b = __bfloat162float(__float2bfloat16_rn(f.y * inv));
        o[j] = pack_bf16x2(a * g.x, b * g.y);
      }
      xv[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace gsb

using namespace gsb;

void gsb_peer_barrier(const at::Tensor& pad_ptrs_dev, int64_t rank, int64_t tp, const at::Tensor& epoch_ctr,
                      int64_t budget_ns, const at::Tensor& err) {
  GSB_CHECK(pad_ptrs_dev.is_cuda() && pad_ptrs_dev.numel() >= tp && tp >= 1 && tp <= 64, "barrier: bad pads");
  GSB_CHECK(epoch_ctr.is_cuda() && epoch_ctr.scalar_type() == at::kInt && epoch_ctr.numel() >= 1,
            "barrier: the epoch counter is one int32 on the device");
  c10::cuda::CUDAGuard g(err.device());
  auto st = c10::cuda::getCurrentCUDAStream(err.device().index()).stream();
  peer_barrier_kernel<<<(::gsb::count_launch(), 1), 64, 0, st>>>(reinterpret_cast<const uint64_t*>(pad_ptrs_dev.data_ptr()), (int)rank,
                                        (int)tp, reinterpret_cast<uint32_t*>(epoch_ctr.data_ptr()), (uint64_t)budget_ns,
                                        reinterpret_cast<uint32_t*>(err.data_ptr()));
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_rmsnorm_residual_from(const at::Tensor& y, const at::Tensor& h, const at::Tensor& w, const at::Tensor& x,
                               double eps) {
  GSB_CHECK(y.scalar_type() == at::kBFloat16 && h.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16,
            "rmsnorm_residual_from: bf16 required");
  const int T = (int)h.size(0), H = (int)h.size(1);
  GSB_CHECK(y.is_contiguous() && h.is_contiguous() && x.is_contiguous() && H % 8 == 0 && y.numel() >= (int64_t)T * H,
            "rmsnorm_residual_from: contiguous [T, H] tensors with H % 8 == 0");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(h.device());
  auto st = c10::cuda::getCurrentCUDAStream(h.device().index()).stream();
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto* hp = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  const int vpt = (H / 8 + 255) / 256;
  if (vpt <= 1) rmsnorm_residual_from_kernel<1><<<(::gsb::count_launch(), T), 256, 0, st>>>(yp, hp, wp, xp, H, (float)eps);
  else if (vpt <= 2) rmsnorm_residual_from_kernel<2><<<(::gsb::count_launch(), T), 256, 0, st>>>(yp, hp, wp, xp, H, (float)eps);
  else rmsnorm_residual_from_kernel<4><<<(::gsb::count_launch(), T), 256, 0, st>>>(yp, hp, wp, xp, H, (float)eps);
  GSB_CUDA_CHECK(cudaGetLastError());
}
