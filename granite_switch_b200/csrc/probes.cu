// Probe heads (reference: src/granite_switch/hf/core/probe.py:20-111 and the
// verdict rewrite in src/granite_switch/hf/modeling_granite_switch.py:903-931).
//
// A probe slot is a linear classifier bank weight[slot, L, H], bias[slot, L]
// read at the probe's control token (always the request's last token). Its
// verdict replaces that row's logits: -inf everywhere except the slot's label
// token ids, which receive the L scores.
//
//   probe_verdict: one CTA per marker; warp w computes labels w, w+4, ... as a
//                  dot product over H (16-byte loads), fp32 accumulation.
//   probe_rewrite: one CTA per marker; fills the logit row (this rank's vocab
//                  shard [vocab_lo, vocab_lo + V)) with -inf, then writes the
//                  label scores that fall inside the shard.
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

__global__ void probe_verdict_kernel(const __nv_bfloat16* __restrict__ hidden, int64_t ldh,
                                     const int32_t* __restrict__ rows, const int32_t* __restrict__ slots,
                                     const int32_t* __restrict__ out_rows, const __nv_bfloat16* __restrict__ w,
                                     const float* __restrict__ bias, int L, int H, float* __restrict__ verdict,
                                     int ldv) {
  const int j = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = slots[j] - 1;
  const __nv_bfloat16* x = hidden + (int64_t)rows[j] * ldh;
  for (int l = warp; l < L; l += blockDim.x >> 5) {
    const __nv_bfloat16* wr = w + ((int64_t)slot * L + l) * H;
    float acc = 0.f;
    for (int c = lane * 8; c < H; c += 32 * 8) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + c);
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
      const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 a = unpack_bf16x2(xs[t]), b = unpack_bf16x2(ws[t]);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) verdict[(int64_t)out_rows[j] * ldv + l] = acc + bias[slot * L + l];
  }
}

__global__ void probe_rewrite_kernel(float* __restrict__ logits, int64_t ldl, int V, int64_t vocab_lo,
                                     const int32_t* __restrict__ out_rows, const int32_t* __restrict__ slots,
                                     const int32_t* __restrict__ labels, int L, const float* __restrict__ verdict,
                                     int ldv) {
  const int j = blockIdx.x;
  const int r = out_rows[j];
  float* row = logits + (int64_t)r * ldl;
  const float ninf = __int_as_float(0xff800000u);
  for (int v = threadIdx.x; v < V; v += blockDim.x) row[v] = ninf;
  __syncthreads();
  const int slot = slots[j] - 1;
  for (int l = threadIdx.x; l < L; l += blockDim.x) {
    const int64_t id = labels[slot * L + l];
    if (id >= vocab_lo && id < vocab_lo + V) row[id - vocab_lo] = verdict[(int64_t)r * ldv + l];
  }
}

}  // namespace gsb

// hidden [T, H] bf16; rows / slots / out_rows int32 [n]; w [NA, L, H] bf16;
// bias [NA, L] fp32; verdict [B, L] fp32 (row out_rows[j] receives marker j).
void gsb_probe_verdict(const at::Tensor& hidden, const at::Tensor& rows, const at::Tensor& slots,
                       const at::Tensor& out_rows, const at::Tensor& w, const at::Tensor& bias,
                       const at::Tensor& verdict) {
  using namespace gsb;
  const int n = (int)rows.numel();
  if (n == 0) return;
  GSB_CHECK(hidden.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                bias.scalar_type() == at::kFloat && verdict.scalar_type() == at::kFloat,
            "probe_verdict: bf16 hidden/weight, fp32 bias/verdict required");
  GSB_CHECK(rows.scalar_type() == at::kInt && slots.scalar_type() == at::kInt && out_rows.scalar_type() == at::kInt,
            "probe_verdict: int32 rows/slots/out_rows required");
  GSB_CHECK(w.dim() == 3 && w.is_contiguous() && bias.is_contiguous(), "probe_verdict: w [NA, L, H] contiguous");
  const int L = (int)w.size(1), H = (int)w.size(2);
  GSB_CHECK(hidden.size(1) == H && hidden.stride(1) == 1 && hidden.stride(0) % 8 == 0 && H % 8 == 0,
            "probe_verdict: hidden must be [T, H] with 16-byte rows");
  GSB_CHECK(verdict.size(1) >= L && verdict.stride(1) == 1, "probe_verdict: verdict too narrow");
  c10::cuda::CUDAGuard g(hidden.device());
  auto st = c10::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  probe_verdict_kernel<<<(::gsb::count_launch(), n), 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(hidden.data_ptr()),
                                          hidden.stride(0), rows.data_ptr<int32_t>(), slots.data_ptr<int32_t>(),
                                          out_rows.data_ptr<int32_t>(),
                                          reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                          bias.data_ptr<float>(), L, H, verdict.data_ptr<float>(),
                                          (int)verdict.stride(0));
  GSB_CUDA_CHECK(cudaGetLastError());
}

// logits [B, V] fp32 (this rank's vocab shard starting at vocab_lo); labels
// [NA, L] int32 (-1 padded).
void gsb_probe_rewrite(const at::Tensor& logits, int64_t vocab_lo, const at::Tensor& out_rows,
                       const at::Tensor& slots, const at::Tensor& labels, const at::Tensor& verdict) {
  using namespace gsb;
  const int n = (int)out_rows.numel();
  if (n == 0) return;
  GSB_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "probe_rewrite: fp32 logits required");
  GSB_CHECK(labels.scalar_type() == at::kInt && labels.dim() == 2 && labels.is_contiguous(),
            "probe_rewrite: int32 labels [NA, L] required");
  GSB_CHECK(verdict.scalar_type() == at::kFloat && verdict.size(1) >= labels.size(1),
            "probe_rewrite: verdict too narrow");
  c10::cuda::CUDAGuard g(logits.device());
  auto st = c10::cuda::getCurrentCUDAStream(logits.device().index()).stream();
  probe_rewrite_kernel<<<(::gsb::count_launch(), n), 256, 0, st>>>(logits.data_ptr<float>(), logits.stride(0), (int)logits.size(1), vocab_lo,
                                          out_rows.data_ptr<int32_t>(), slots.data_ptr<int32_t>(),
                                          labels.data_ptr<int32_t>(), (int)labels.size(1),
                                          verdict.data_ptr<float>(), (int)verdict.stride(0));
  GSB_CUDA_CHECK(cudaGetLastError());
}
