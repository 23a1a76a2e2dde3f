// Temperature / top-k / top-p sampling, one CTA per row of fp32 logits.
//
// The top-k and top-p cut-offs are found as value thresholds by bisection on
// the logit range (each probe is one block-wide count or probability sum), so
// no sort is needed. A token is then drawn by the Gumbel-max rule among the
// survivors, which samples exactly from the renormalised softmax over them;
// the Gumbel noise comes from a counter-based Philox stream keyed by
// (seed, step offset, row, token), so a request's draws are reproducible.
// (reference: the sampler is vLLM's, used by every generate call.)
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <curand_kernel.h>

namespace gsb {

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < THREADS / 32 ? sh[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = warp_sum(t);
  if (threadIdx.x == 0) sh[32] = t;
  __syncthreads();
  const float r = sh[32];
  __syncthreads();
  return r;
}
template <int THREADS>
__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < THREADS / 32 ? sh[threadIdx.x] : -INFINITY;
  if (threadIdx.x < 32) t = warp_max(t);
  if (threadIdx.x == 0) sh[32] = t;
  __syncthreads();
  const float r = sh[32];
  __syncthreads();
  return r;
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS)
    sample_kernel(const float* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temperature,
                  const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
                  const int64_t* __restrict__ seeds, const int64_t* __restrict__ offsets,
                  int64_t* __restrict__ out) {
  __shared__ float sh[33];
  const int r = blockIdx.x;
  const float* row = logits + (int64_t)r * ld;
  const float temp = temperature[r];
  // greedy rows: plain argmax
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += THREADS) mx = fmaxf(mx, row[i]);
  mx = block_max<THREADS>(mx, sh);
  if (!(temp > 0.f)) {
    int best = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += THREADS)
      if (row[i] == mx && i < best) best = i;
    best = (int)-block_max<THREADS>(-(float)best, sh);
    if (threadIdx.x == 0) out[r] = best;
    return;
  }
  const float inv_t = 1.f / temp;
  float mn = INFINITY;
  for (int i = threadIdx.x; i < V; i += THREADS) mn = fminf(mn, row[i]);
  mn = -block_max<THREADS>(-mn, sh);
  // ---- top-k threshold: largest thr with count(l >= thr) >= k
  float thr = -INFINITY;
  const int k = top_k[r];
  if (k > 0 && k < V) {
    float lo = mn, hi = mx;
    for (int it = 0; it < 40; ++it) {
      const float mid = 0.5f * (lo + hi);
      float c = 0.f;
      for (int i = threadIdx.x; i < V; i += THREADS) c += (row[i] >= mid) ? 1.f : 0.f;
      c = block_sum<THREADS>(c, sh);
      if (c >= (float)k) lo = mid; else hi = mid;
    }
    thr = lo;
  }
  // ---- top-p threshold over the survivors' softmax
  const float p = top_p[r];
  if (p < 1.f) {
    float z = 0.f;
    for (int i = threadIdx.x; i < V; i += THREADS)
      if (row[i] >= thr) z += __expf((row[i] - mx) * inv_t);
    z = block_sum<THREADS>(z, sh);
    float lo = fmaxf(thr, mn), hi = mx;
    for (int it = 0; it < 40; ++it) {
      const float mid = 0.5f * (lo + hi);
      float s = 0.f;
      for (int i = threadIdx.x; i < V; i += THREADS)
        if (row[i] >= mid) s += __expf((row[i] - mx) * inv_t);
      s = block_sum<THREADS>(s, sh);
      if (s >= p * z) lo = mid; else hi = mid;
    }
    thr = fmaxf(thr, lo);
  }
  // ---- Gumbel-max among survivors
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  const uint64_t seed = (uint64_t)seeds[r];
  const uint64_t off = (uint64_t)offsets[r];
  for (int i = threadIdx.x; i < V; i += THREADS) {
    const float l = row[i];
    if (l < thr) continue;
    curandStatePhilox4_32_10_t st;
    curand_init(seed, ((uint64_t)i << 20) ^ (uint64_t)r, off, &st);
    const float u = fmaxf(curand_uniform(&st), 1e-20f);
    const float g = -__logf(-__logf(u));
    const float v = l * inv_t + g;
    if (v > best_v || (v == best_v && i < best_i)) {
      best_v = v;
      best_i = i;
    }
  }
  // block argmax of (best_v, best_i)
  __shared__ float sv[THREADS / 32];
  __shared__ int si[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best_v || (ov == best_v && oi < best_i)) {
      best_v = ov;
      best_i = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best_v;
    si[threadIdx.x >> 5] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < THREADS / 32; ++w)
      if (sv[w] > best_v || (sv[w] == best_v && si[w] < best_i)) {
        best_v = sv[w];
        best_i = si[w];
      }
    out[r] = best_i == 0x7fffffff ? 0 : best_i;
  }
}

}  // namespace gsb

using namespace gsb;

void gsb_sample(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                const at::Tensor& top_p, const at::Tensor& seeds, const at::Tensor& offsets, const at::Tensor& out) {
  GSB_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "sample: fp32 logits required");
  GSB_CHECK(temperature.scalar_type() == at::kFloat && top_p.scalar_type() == at::kFloat &&
                top_k.scalar_type() == at::kInt && seeds.scalar_type() == at::kLong &&
                offsets.scalar_type() == at::kLong && out.scalar_type() == at::kLong,
            "sample: parameter dtypes");
  const int B = (int)logits.size(0);
  if (B == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  auto st = c10::cuda::getCurrentCUDAStream(logits.device().index()).stream();
  sample_kernel<512><<<(::gsb::count_launch(), B), 512, 0, st>>>(logits.data_ptr<float>(), logits.stride(0), (int)logits.size(1),
                                        temperature.data_ptr<float>(), top_k.data_ptr<int32_t>(),
                                        top_p.data_ptr<float>(), seeds.data_ptr<int64_t>(),
                                        offsets.data_ptr<int64_t>(), out.data_ptr<int64_t>());
  GSB_CUDA_CHECK(cudaGetLastError());
}
