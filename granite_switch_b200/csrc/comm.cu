// Tensor-parallel communication kernels over NVLink / NVSwitch peer memory.
//
// * peer_barrier: every rank stores an epoch into its slot of every peer's
//   signal pad (plain P2P st.release.sys) and waits, with a bounded spin, until
//   all peers' epochs arrived in its own pad (ld.acquire.sys). A wait that runs
//   out sets kErrPeerWait and returns; it never hangs.
// * multimem_allreduce_bf16: one-shot all-reduce of a symmetric bf16 buffer
//   through the NVSwitch: each rank reduces a 1/tp slice with
//   multimem.ld_reduce (the switch sums every rank's copy) and multicasts the
//   sum back with multimem.st, so every rank ends up with the full result
//   (reduce-scatter + all-gather in one pass over NVLink).
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
__global__ void peer_barrier_kernel(const uint64_t* __restrict__ pads, int rank, int tp, uint32_t epoch,
                                    uint64_t budget_ns, uint32_t* err) {
  const int p = threadIdx.x;
  if (p >= tp) return;
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

__device__ __forceinline__ void multimem_ld_reduce_v4_bf16x2(const void* mc, uint32_t (&r)[4]) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(mc)
               : "memory");
}
__device__ __forceinline__ void multimem_st_v4(void* mc, const uint32_t (&r)[4]) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// one-shot all-reduce over a multicast mapping: rank r reduces 16-byte vectors
// [r*n/tp, (r+1)*n/tp) and stores the sums to every rank
__global__ void multimem_allreduce_bf16_kernel(uint8_t* __restrict__ mc, int64_t n_vec, int rank, int tp) {
  const int64_t per = (n_vec + tp - 1) / tp;
  const int64_t lo = rank * per, hi = min(n_vec, lo + per);
  for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t r[4];
    multimem_ld_reduce_v4_bf16x2(mc + i * 16, r);
    multimem_st_v4(mc + i * 16, r);
  }
  __threadfence_system();  // the multicast stores precede the barrier that follows this kernel
}

// All-reduce whose result travels by plain peer stores: rank r sums its 1/tp
// slice through the switch (multimem.ld_reduce) and writes the sums into every
// rank's copy with ordinary P2P stores. Completion is then signalled by the P2P
// barrier on the same path as the data (multicast stores followed by a P2P flag
// were observed out of order by a reader that did not synchronise).
__global__ void allreduce_ldreduce_p2p_kernel(const uint8_t* __restrict__ mc, const uint64_t* __restrict__ peers,
                                              int64_t offset, int64_t n_vec, int rank, int tp) {
  const int64_t per = (n_vec + tp - 1) / tp;
  const int64_t lo = rank * per, hi = min(n_vec, lo + per);
  for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t r[4];
    multimem_ld_reduce_v4_bf16x2(mc + offset + i * 16, r);
    const uint4 v = make_uint4(r[0], r[1], r[2], r[3]);
    for (int p = 0; p < tp; ++p)
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peers[p]) + offset + i * 16) = v;
  }
  __threadfence_system();
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

void gsb_peer_barrier(const at::Tensor& pad_ptrs_dev, int64_t rank, int64_t tp, int64_t epoch, int64_t budget_ns,
                      const at::Tensor& err) {
  GSB_CHECK(pad_ptrs_dev.is_cuda() && pad_ptrs_dev.numel() >= tp && tp >= 1 && tp <= 64, "barrier: bad pads");
  c10::cuda::CUDAGuard g(err.device());
  auto st = c10::cuda::getCurrentCUDAStream(err.device().index()).stream();
  peer_barrier_kernel<<<(::gsb::count_launch(), 1), 64, 0, st>>>(reinterpret_cast<const uint64_t*>(pad_ptrs_dev.data_ptr()), (int)rank,
                                        (int)tp, (uint32_t)epoch, (uint64_t)budget_ns,
                                        reinterpret_cast<uint32_t*>(err.data_ptr()));
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_multimem_allreduce_bf16(int64_t mc_ptr, int64_t nbytes, int64_t rank, int64_t tp, const at::Tensor& like) {
  GSB_CHECK(mc_ptr != 0 && nbytes % 16 == 0, "multimem all-reduce: multicast pointer and 16-byte size required");
  c10::cuda::CUDAGuard g(like.device());
  auto st = c10::cuda::getCurrentCUDAStream(like.device().index()).stream();
  const int64_t n_vec = nbytes / 16;
  const int64_t per = (n_vec + tp - 1) / tp;
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>(1, (per + 255) / 256), 132);
  multimem_allreduce_bf16_kernel<<<(::gsb::count_launch(), blocks), 256, 0, st>>>(reinterpret_cast<uint8_t*>(mc_ptr), n_vec, (int)rank,
                                                          (int)tp);
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_allreduce_ldreduce_p2p(int64_t mc_ptr, const at::Tensor& peer_ptrs, int64_t offset, int64_t nbytes,
                                int64_t rank, int64_t tp) {
  GSB_CHECK(mc_ptr != 0 && nbytes % 16 == 0 && offset % 16 == 0,
            "all-reduce: multicast pointer and 16-byte size/offset required");
  GSB_CHECK(peer_ptrs.is_cuda() && peer_ptrs.scalar_type() == at::kLong && peer_ptrs.numel() >= tp,
            "all-reduce: int64 device tensor of peer base pointers required");
  c10::cuda::CUDAGuard g(peer_ptrs.device());
  auto st = c10::cuda::getCurrentCUDAStream(peer_ptrs.device().index()).stream();
  const int64_t n_vec = nbytes / 16;
  const int64_t per = (n_vec + tp - 1) / tp;
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>(1, (per + 255) / 256), 148);
  allreduce_ldreduce_p2p_kernel<<<(::gsb::count_launch(), blocks), 256, 0, st>>>(reinterpret_cast<const uint8_t*>(mc_ptr),
                                                         reinterpret_cast<const uint64_t*>(peer_ptrs.data_ptr()),
                                                         offset, n_vec, (int)rank, (int)tp);
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
