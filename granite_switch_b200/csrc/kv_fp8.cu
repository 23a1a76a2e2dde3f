// fp8 (e4m3) paged KV cache: quantised write of a step's new K/V.
//
// Each (token, KV head) row of K and of V gets its own fp32 scale,
// scale = max|x| / 448 (448 is e4m3's largest finite value), and is stored as
// e4m3(x / scale): per-row scales keep the relative error of every element
// within e4m3's 3-bit mantissa whatever the row's magnitude, at 4 bytes of
// scale per 128-byte row. Layout (per layer):
//
//   K  [num_blocks, Hkv, 16 tokens, D]  bytes; inside every group of 16 head
//      dimensions the bytes are stored in the order
//      0 1 8 9 | 2 3 10 11 | 4 5 12 13 | 6 7 14 15, so the four values a thread
//      feeds to one mma.sync m16n8k16 B fragment (dims 2t, 2t+1, 2t+8, 2t+9) are
//      one 32-bit word in shared memory;
//   V  [num_blocks, Hkv, D, 16 tokens]  bytes: the page transposed, tokens in the
//      same 16-element order, so a thread's B fragment of P.V (tokens 2t, 2t+1,
//      2t+8, 2t+9 of one dimension) is one 32-bit word too;
//   scales [num_blocks, Hkv, 16] fp32 for K and for V.
//
// The paged attention kernel (attention.cu) loads these pages by TMA, converts
// the e4m3 pairs exactly to bf16 in registers, and applies the scales to the
// scores (K) and to the probabilities (V). The reference serves fp8 KV through
// vLLM's --kv-cache-dtype fp8 (reference: docs/MULTISWITCH_EXPLAINED.md:559-568);
// here routing never reads the cache, so quantising it cannot disturb routing.
#include "common.cuh"
#include "rope.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_fp8.h>

namespace gsb {

// Position of element i (0..15) of a 16-element group in the stored order.
__host__ __device__ __forceinline__ int fp8_perm16(int i) {
  return (i < 8) ? ((i >> 1) << 2) + (i & 1) : (((i - 8) >> 1) << 2) + 2 + (i & 1);
}

__device__ __forceinline__ uint16_t to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// Quantised write of one (token, KV head) row of K and of V by one warp: lane l holds
// dims [E l, E l + E); `row` is the token's qkv row (K already rotated).
template <int D>
__device__ __forceinline__ void kv_write_fp8_row(const __nv_bfloat16* __restrict__ row, int Hq, int Hkv, int kh,
                                                 int lane, int64_t slot, uint8_t* __restrict__ k8,
                                                 uint8_t* __restrict__ v8, float* __restrict__ ks,
                                                 float* __restrict__ vs) {
  constexpr int E = D / 32;
  const int64_t blk = slot / 16, off = slot % 16;
  const __nv_bfloat16* krow = row + (int64_t)(Hq + kh) * D + lane * E;
  const __nv_bfloat16* vrow = row + (int64_t)(Hq + Hkv + kh) * D + lane * E;
  float kf[E], vf[E];
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(krow + e));
    const float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(vrow + e));
    kf[e] = a.x;
    kf[e + 1] = a.y;
    vf[e] = b.x;
    vf[e + 1] = b.y;
  }
  float km = 0.f, vm = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    km = fmaxf(km, fabsf(kf[e]));
    vm = fmaxf(vm, fabsf(vf[e]));
  }
  km = warp_max(km);
  vm = warp_max(vm);
  const float ksc = km > 0.f ? km / 448.f : 1.f, vsc = vm > 0.f ? vm / 448.f : 1.f;
  const int64_t head_row = blk * Hkv + kh;
  uint8_t* kdst = k8 + (head_row * 16 + off) * D;
  uint8_t* vdst = v8 + head_row * D * 16;
  const int pv = fp8_perm16((int)off);
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    const int d = lane * E + e;  // even: d and d + 1 share a 2-byte slot in the stored order
    *reinterpret_cast<uint16_t*>(kdst + (d & ~15) + fp8_perm16(d & 15)) = to_e4m3x2(kf[e] / ksc, kf[e + 1] / ksc);
    const uint16_t vq = to_e4m3x2(vf[e] / vsc, vf[e + 1] / vsc);
    vdst[(int64_t)d * 16 + pv] = (uint8_t)(vq & 0xff);
    vdst[(int64_t)(d + 1) * 16 + pv] = (uint8_t)(vq >> 8);
  }
  if (lane == 0) {
    ks[head_row * 16 + off] = ksc;
    vs[head_row * 16 + off] = vsc;
  }
}

// One warp per (token, KV head).
template <int D>
__global__ void kv_write_fp8_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int Hq, int Hkv,
                                    const int64_t* __restrict__ slots, int64_t num_slots,
                                    uint8_t* __restrict__ k8, uint8_t* __restrict__ v8, float* __restrict__ ks,
                                    float* __restrict__ vs, uint32_t* err) {
  const int t = blockIdx.x;
  const int kh = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (kh >= Hkv) return;
  const int64_t slot = slots[t];
  if (slot < 0 || slot >= num_slots) {
    if (slot >= num_slots && threadIdx.x == 0) report_bad_index(err, kSiteKvSlot, slot);
    return;
  }
  kv_write_fp8_row<D>(qkv + (int64_t)t * ldq, Hq, Hkv, kh, lane, slot, k8, v8, ks, vs);
}

// RoPE on one token's q and k heads, then the quantised write of its K / V rows: one
// block per token (the rotation over all its threads, then one warp per KV head), so
// the fp8 cache costs one launch per layer like the bf16 one.
template <int D>
__global__ void rope_kv_fp8_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ldq, const int64_t* __restrict__ positions,
                                   const float* __restrict__ cos_sin, int max_pos, const int64_t* __restrict__ slots,
                                   int64_t num_slots, int Hq, int Hkv, uint8_t* __restrict__ k8,
                                   uint8_t* __restrict__ v8, float* __restrict__ ks, float* __restrict__ vs,
                                   uint32_t* err) {
  griddep_wait();  // launched as a dependent of the projection that writes qkv
  const int t = blockIdx.x;
  int64_t pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) report_bad_index(err, kSiteRopePos, pos);
    pos = 0;
  }
  __nv_bfloat16* row = qkv + (int64_t)t * ldq;
  rope_rotate_row<D>(row, cos_sin + pos * D, Hq, Hkv, nullptr, 0);
  __syncthreads();  // the rotated k heads (global stores of this block) before the quantised write
  const int64_t slot = slots[t];
  if (slot < 0 || slot >= num_slots) {
    if (slot >= num_slots && threadIdx.x == 0) report_bad_index(err, kSiteKvSlot, slot);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int kh = warp; kh < Hkv; kh += blockDim.x >> 5)
    kv_write_fp8_row<D>(row, Hq, Hkv, kh, lane, slot, k8, v8, ks, vs);
}

}  // namespace gsb

using namespace gsb;

// qkv [T, (Hq + 2 Hkv) D] bf16 with K already rotated; slots [T] int64;
// k8 [num_blocks, Hkv, 16, D] uint8; v8 [num_blocks, Hkv, D, 16] uint8;
// k_scale / v_scale [num_blocks, Hkv, 16] fp32.
void gsb_kv_write_fp8(const at::Tensor& qkv, const at::Tensor& slots, const at::Tensor& k8, const at::Tensor& v8,
                      const at::Tensor& k_scale, const at::Tensor& v_scale, int64_t num_q_heads,
                      int64_t num_kv_heads, int64_t head_dim, const at::Tensor& err) {
  GSB_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && qkv.stride(0) % 2 == 0,
            "kv_write_fp8: bf16 qkv with even row stride required");
  GSB_CHECK(slots.scalar_type() == at::kLong, "kv_write_fp8: int64 slots required");
  GSB_CHECK(k8.scalar_type() == at::kByte && v8.scalar_type() == at::kByte && k8.is_contiguous() &&
                v8.is_contiguous() && k8.dim() == 4 && v8.dim() == 4,
            "kv_write_fp8: contiguous uint8 caches required");
  const int D = (int)head_dim, Hkv = (int)num_kv_heads;
  GSB_CHECK(k8.size(1) == Hkv && k8.size(2) == 16 && k8.size(3) == D && v8.size(1) == Hkv && v8.size(2) == D &&
                v8.size(3) == 16 && v8.size(0) == k8.size(0),
            "kv_write_fp8: caches must be K [blocks, Hkv, 16, D] and V [blocks, Hkv, D, 16]");
  GSB_CHECK(k_scale.scalar_type() == at::kFloat && v_scale.scalar_type() == at::kFloat && k_scale.is_contiguous() &&
                v_scale.is_contiguous() && k_scale.numel() == k8.size(0) * Hkv * 16 &&
                v_scale.numel() == k_scale.numel(),
            "kv_write_fp8: fp32 scales [blocks, Hkv, 16] required");
  GSB_CHECK(Hkv >= 1 && Hkv <= 32, "kv_write_fp8: 1..32 KV heads");
  GSB_CHECK(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * head_dim, "kv_write_fp8: qkv too narrow");
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.device());
  auto st = c10::cuda::getCurrentCUDAStream(qkv.device().index()).stream();
  const int64_t num_slots = k8.size(0) * 16;
  auto* ep = reinterpret_cast<uint32_t*>(err.data_ptr());
#define GSB_KVW(DD)                                                                                              \
  kv_write_fp8_kernel<DD><<<(::gsb::count_launch(), T), 32 * Hkv, 0, st>>>(                                      \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), (int)num_q_heads, Hkv,              \
      slots.data_ptr<int64_t>(), num_slots, k8.data_ptr<uint8_t>(), v8.data_ptr<uint8_t>(),                      \
      k_scale.data_ptr<float>(), v_scale.data_ptr<float>(), ep)
  if (D == 128) GSB_KVW(128);
  else if (D == 64) GSB_KVW(64);
  else GSB_CHECK(false, "kv_write_fp8: head_dim must be 64 or 128, got ", D);
#undef GSB_KVW
  GSB_CUDA_CHECK(cudaGetLastError());
}

// RoPE + quantised K / V write in one launch: qkv [T, (Hq + 2 Hkv) D] bf16 (q and k rotated
// in place), positions / slots [T] int64, cos_sin [max_pos, D] fp32, caches and scales as
// gsb_kv_write_fp8.
void gsb_rope_kv_fp8(const at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                     const at::Tensor& slots, const at::Tensor& k8, const at::Tensor& v8, const at::Tensor& k_scale,
                     const at::Tensor& v_scale, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                     const at::Tensor& err) {
  GSB_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0 &&
                (reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15) == 0,
            "rope_kv_fp8: bf16 qkv with 16-byte aligned rows required");
  GSB_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong &&
                cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == head_dim,
            "rope_kv_fp8: int64 positions / slots and fp32 cos_sin [max_pos, head_dim] required");
  GSB_CHECK(k8.scalar_type() == at::kByte && v8.scalar_type() == at::kByte && k8.is_contiguous() &&
                v8.is_contiguous() && k8.dim() == 4 && v8.dim() == 4,
            "rope_kv_fp8: contiguous uint8 caches required");
  const int D = (int)head_dim, Hkv = (int)num_kv_heads;
  GSB_CHECK(k8.size(1) == Hkv && k8.size(2) == 16 && k8.size(3) == D && v8.size(1) == Hkv && v8.size(2) == D &&
                v8.size(3) == 16 && v8.size(0) == k8.size(0),
            "rope_kv_fp8: caches must be K [blocks, Hkv, 16, D] and V [blocks, Hkv, D, 16]");
  GSB_CHECK(k_scale.scalar_type() == at::kFloat && v_scale.scalar_type() == at::kFloat && k_scale.is_contiguous() &&
                v_scale.is_contiguous() && k_scale.numel() == k8.size(0) * Hkv * 16 &&
                v_scale.numel() == k_scale.numel(),
            "rope_kv_fp8: fp32 scales [blocks, Hkv, 16] required");
  GSB_CHECK(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * head_dim, "rope_kv_fp8: qkv too narrow");
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.device());
  auto st = c10::cuda::getCurrentCUDAStream(qkv.device().index()).stream();
  const int64_t num_slots = k8.size(0) * 16;
  auto* ep = reinterpret_cast<uint32_t*>(err.data_ptr());
#define GSB_ROPE8(DD)                                                                                           \
  launch_dependent(rope_kv_fp8_kernel<DD>, dim3(T), dim3(256), 0, st, reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), \
                   qkv.stride(0), positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), (int)cos_sin.size(0), \
                   slots.data_ptr<int64_t>(), num_slots, (int)num_q_heads, Hkv, k8.data_ptr<uint8_t>(),          \
                   v8.data_ptr<uint8_t>(), k_scale.data_ptr<float>(), v_scale.data_ptr<float>(), ep)
  if (D == 128) GSB_ROPE8(128);
  else if (D == 64) GSB_ROPE8(64);
  else GSB_CHECK(false, "rope_kv_fp8: head_dim must be 64 or 128, got ", D);
#undef GSB_ROPE8
  GSB_CUDA_CHECK(cudaGetLastError());
}

