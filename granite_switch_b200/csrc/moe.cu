// Mixture-of-experts routing, token permutation and combine for frozen expert
// banks (reference: the vLLM FusedMoE the reference's MoE bases run on,
// src/granite_switch/vllm/decoder/lora/decoder.py:257-374; HF semantics in
// src/granite_switch/hf/modeling_granite_switch.py:116-153): router logits ->
// top-k -> softmax over the k logits -> each token's rows go to its experts ->
// per expert y = down(silu(gate) * up) -> weighted sum over the k experts.
//
// The expert GEMMs are the tcgen05 switched GEMM in grouped mode: rows are
// sorted by expert into segments padded to 128 rows, each 128-row tile reads
// its expert's weights through a 3-D tensor map, and tiles past the last
// segment are skipped. Everything stays on the device (no host sync): the
// GEMMs are launched for the worst-case row count and skip empty tiles.
//
//   moe_topk     one warp per token: top-k over E router logits (fp32),
//                softmax of the k values, per-expert counts (atomics)
//   moe_plan     one block: padded segment offsets and the tile -> expert map
//   moe_scatter  one warp per (token, k): slot in its expert's segment,
//                copy of the token's row into the permuted activations
//   moe_combine  one block per token: sum_k w_k * Y[slot(t, k)] (+ shared MLP
//                output), optionally added to the residual stream
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>

namespace gsb {

constexpr int kMoeMaxK = 8;
constexpr int kMoeMaxExperts = 256;

__global__ void moe_topk_kernel(const float* __restrict__ logits, int64_t ldl, int T, int E, int K,
                                int32_t* __restrict__ ids, float* __restrict__ wts, int32_t* __restrict__ counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + (int64_t)warp * ldl;
  constexpr int PER = kMoeMaxExperts / 32;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? row[e] : -INFINITY;
  }
  float top_v[kMoeMaxK];
  int top_e[kMoeMaxK];
  for (int k = 0; k < K; ++k) {
    // warp argmax (lowest expert index wins ties)
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv || (v[i] == bv && e < be)) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    top_v[k] = bv;
    top_e[k] = be;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) v[i] = -INFINITY;
  }
  if (lane == 0) {
    float mx = top_v[0], s = 0.f;
    for (int k = 0; k < K; ++k) s += __expf(top_v[k] - mx);
    for (int k = 0; k < K; ++k) {
      ids[(int64_t)warp * K + k] = top_e[k];
      wts[(int64_t)warp * K + k] = __expf(top_v[k] - mx) / s;
      atomicAdd(&counts[top_e[k]], 1);
    }
  }
}

// counts[E] -> offsets[E] (segments padded to 128 rows), tile_expert[max_tiles]
// (-1 past the last segment), cursor[E] = 0; counts are cleared for the next call.
__global__ void moe_plan_kernel(int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                int32_t* __restrict__ cursor, int32_t* __restrict__ tile_expert, int E,
                                int max_tiles) {
  __shared__ int32_t s_off[kMoeMaxExperts + 1];
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = acc;
      acc += (counts[e] + 127) / 128 * 128;
    }
    s_off[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    offsets[e] = s_off[e];
    cursor[e] = 0;
  }
  const int used = s_off[E] / 128;
  for (int t = threadIdx.x; t < max_tiles; t += blockDim.x) {
    int ex = -1;
    if (t < used) {
      // segment containing row t*128 (segments are whole tiles)
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= t * 128) lo = mid;
        else hi = mid - 1;
      }
      ex = lo;  // the largest such expert is never an empty one
    }
    tile_expert[t] = ex;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = 0;
}

__global__ void moe_scatter_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int T, int K, int H,
                                   const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets,
                                   int32_t* __restrict__ cursor, int32_t* __restrict__ slot,
                                   __nv_bfloat16* __restrict__ xp, int64_t ldp) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * K) return;
  const int t = w / K;
  int pos = 0;
  if (lane == 0) {
    if (cursor != nullptr) {
      const int e = ids[w];
      pos = offsets[e] + atomicAdd(&cursor[e], 1);
      slot[w] = pos;
    } else {
      pos = slot[w];  // slots of an earlier scatter with the same routing
    }
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)pos * ldp);
  for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ yp, int64_t ldy, const int32_t* __restrict__ slot,
                                   const float* __restrict__ wts, int K, int H,
                                   const __nv_bfloat16* __restrict__ shared, int64_t lds,
                                   const __nv_bfloat16* __restrict__ residual, int64_t ldr, float scale,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int t = blockIdx.x;
  int sl[kMoeMaxK];
  float wk[kMoeMaxK];
  for (int k = 0; k < K; ++k) {
    sl[k] = slot[(int64_t)t * K + k];
    wk[k] = wts[(int64_t)t * K + k];
  }
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    float a0 = 0.f, a1 = 0.f;
    for (int k = 0; k < K; ++k) {
      const float2 y = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(yp + (int64_t)sl[k] * ldy + c));
      a0 = fmaf(wk[k], y.x, a0);
      a1 = fmaf(wk[k], y.y, a1);
    }
    // the expert sum is materialised in bf16 before the shared MLP is added,
    // and their sum in bf16 before the residual multiplier, as unfused
    a0 = __bfloat162float(__float2bfloat16_rn(a0));
    a1 = __bfloat162float(__float2bfloat16_rn(a1));
    if (shared != nullptr) {
      const float2 s = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(shared + (int64_t)t * lds + c));
      a0 = __bfloat162float(__float2bfloat16_rn(a0 + s.x));
      a1 = __bfloat162float(__float2bfloat16_rn(a1 + s.y));
    }
    if (residual != nullptr) {
      const float2 r = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(residual + (int64_t)t * ldr + c));
      a0 = r.x + a0 * scale;
      a1 = r.y + a1 * scale;
    }
    *reinterpret_cast<uint32_t*>(out + (int64_t)t * ldo + c) = pack_bf16x2(a0, a1);
  }
}

}  // namespace gsb

static cudaStream_t moe_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// logits [T, >=E] fp32 -> ids [T, K] int32, wts [T, K] fp32; counts [E] int32 (zero on entry,
// accumulated). Then offsets / cursor [E], tile_expert [max_tiles] and counts cleared.
void gsb_moe_route(const at::Tensor& logits, int64_t num_experts, int64_t top_k, const at::Tensor& ids,
                   const at::Tensor& wts, const at::Tensor& counts, const at::Tensor& offsets, const at::Tensor& cursor,
                   const at::Tensor& tile_expert) {
  using namespace gsb;
  const int T = (int)logits.size(0), E = (int)num_experts, K = (int)top_k;
  GSB_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1 && logits.size(1) >= E,
            "moe_route: fp32 logits [T, >=E] required");
  GSB_CHECK(E >= 1 && E <= kMoeMaxExperts && K >= 1 && K <= kMoeMaxK && K <= E, "moe_route: 1 <= k <= 8, E <= 256");
  GSB_CHECK(ids.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat && counts.scalar_type() == at::kInt &&
                offsets.scalar_type() == at::kInt && cursor.scalar_type() == at::kInt &&
                tile_expert.scalar_type() == at::kInt,
            "moe_route: int32 ids/counts/offsets/cursor/tile_expert and fp32 wts required");
  GSB_CHECK(ids.numel() >= (int64_t)T * K && wts.numel() >= (int64_t)T * K && counts.numel() >= E &&
                offsets.numel() >= E && cursor.numel() >= E,
            "moe_route: output buffers too small");
  c10::cuda::CUDAGuard g(logits.device());
  auto st = moe_stream(logits);
  if (T > 0) {
    const int threads = 256;
    moe_topk_kernel<<<(::gsb::count_launch(), (T * 32 + threads - 1) / threads), threads, 0, st>>>(
        logits.data_ptr<float>(), logits.stride(0), T, E, K, ids.data_ptr<int32_t>(), wts.data_ptr<float>(),
        counts.data_ptr<int32_t>());
    GSB_CUDA_CHECK(cudaGetLastError());
  }
  moe_plan_kernel<<<(::gsb::count_launch(), 1), 256, 0, st>>>(counts.data_ptr<int32_t>(), offsets.data_ptr<int32_t>(),
                                     cursor.data_ptr<int32_t>(), tile_expert.data_ptr<int32_t>(), E,
                                     (int)tile_expert.numel());
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_moe_scatter(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& offsets, const at::Tensor& cursor,
                     const at::Tensor& slot, const at::Tensor& xp) {
  using namespace gsb;
  const int T = (int)x.size(0), H = (int)x.size(1), K = (int)(ids.numel() / std::max<int64_t>(T, 1));
  if (T == 0) return;
  GSB_CHECK(x.scalar_type() == at::kBFloat16 && xp.scalar_type() == at::kBFloat16 && H % 8 == 0 &&
                x.stride(0) % 8 == 0 && xp.stride(0) % 8 == 0 && xp.size(1) == H,
            "moe_scatter: bf16 rows of equal, 16-byte aligned width required");
  c10::cuda::CUDAGuard g(x.device());
  const int threads = 256;
  const int64_t warps = (int64_t)T * K;
  moe_scatter_kernel<<<(::gsb::count_launch(), (unsigned)((warps * 32 + threads - 1) / threads)), threads, 0, moe_stream(x)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), T, K, H, ids.data_ptr<int32_t>(),
      offsets.data_ptr<int32_t>(), cursor.data_ptr<int32_t>(), slot.data_ptr<int32_t>(),
      reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()), xp.stride(0));
  GSB_CUDA_CHECK(cudaGetLastError());
}

// Scatter x's rows to the slots an earlier gsb_moe_scatter assigned (same routing,
// another stream of hidden states: the Shadow-Residual adapter stream reuses the
// base stream's expert choice). slot [T*K] int32.
void gsb_moe_scatter_slots(const at::Tensor& x, const at::Tensor& slot, int64_t top_k, const at::Tensor& xp) {
  using namespace gsb;
  const int T = (int)x.size(0), H = (int)x.size(1), K = (int)top_k;
  if (T == 0) return;
  GSB_CHECK(x.scalar_type() == at::kBFloat16 && xp.scalar_type() == at::kBFloat16 && H % 8 == 0 &&
                x.stride(0) % 8 == 0 && xp.stride(0) % 8 == 0 && xp.size(1) == H,
            "moe_scatter_slots: bf16 rows of equal, 16-byte aligned width required");
  GSB_CHECK(slot.scalar_type() == at::kInt && slot.numel() >= (int64_t)T * K && K >= 1 && K <= kMoeMaxK,
            "moe_scatter_slots: int32 slot [T * k] required");
  c10::cuda::CUDAGuard g(x.device());
  const int threads = 256;
  const int64_t warps = (int64_t)T * K;
  moe_scatter_kernel<<<(::gsb::count_launch(), (unsigned)((warps * 32 + threads - 1) / threads)), threads, 0, moe_stream(x)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), T, K, H, nullptr, nullptr, nullptr,
      slot.data_ptr<int32_t>(), reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()), xp.stride(0));
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_moe_combine(const at::Tensor& yp, const at::Tensor& slot, const at::Tensor& wts, int64_t top_k,
                     const c10::optional<at::Tensor>& shared, const c10::optional<at::Tensor>& residual, double scale,
                     const at::Tensor& out) {
  using namespace gsb;
  const int T = (int)out.size(0), H = (int)out.size(1);
  if (T == 0) return;
  GSB_CHECK(yp.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 && H % 2 == 0 &&
                yp.size(1) == H,
            "moe_combine: bf16 [*, H] required");
  GSB_CHECK(top_k >= 1 && top_k <= kMoeMaxK, "moe_combine: 1 <= k <= 8");
  c10::cuda::CUDAGuard g(out.device());
  const __nv_bfloat16* sp = shared ? reinterpret_cast<const __nv_bfloat16*>(shared->data_ptr()) : nullptr;
  const __nv_bfloat16* rp = residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  moe_combine_kernel<<<(::gsb::count_launch(), T), 256, 0, moe_stream(out)>>>(
      reinterpret_cast<const __nv_bfloat16*>(yp.data_ptr()), yp.stride(0), slot.data_ptr<int32_t>(),
      wts.data_ptr<float>(), (int)top_k, H, sp, shared ? shared->stride(0) : 0, rp, residual ? residual->stride(0) : 0,
      (float)scale, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
  GSB_CUDA_CHECK(cudaGetLastError());
}
