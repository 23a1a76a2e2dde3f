// Rotary embedding of one token's q and k heads, shared by the bf16 RoPE + KV write
// (elementwise.cu) and the fused RoPE + fp8 KV write (kv_fp8.cu).
#pragma once

#include "common.cuh"

namespace gsb {

// Rotates the Hq query heads and Hkv key heads of `row` (one token of qkv, head_dim D)
// in place with the cos / sin row `cs` (neox layout: x cos + rotate_half(x) sin, the
// same cos / sin on both halves). The block's threads take 8 pairs (i, i + D/2) each,
// with 16-byte loads and stores. With `k_cache` non-null the rotated key head kh is
// also stored at k_cache + kh * kh_stride (bf16 cache row).
template <int D>
__device__ __forceinline__ void rope_rotate_row(__nv_bfloat16* __restrict__ row, const float* __restrict__ cs, int Hq,
                                                int Hkv, __nv_bfloat16* __restrict__ k_cache, int64_t kh_stride) {
  constexpr int HALF = D / 2;
  constexpr int CH = HALF / 8;  // 8-element (16-byte) chunks per half
  const int nheads = Hq + Hkv;
  for (int idx = threadIdx.x; idx < nheads * CH; idx += blockDim.x) {
    const int h = idx / CH;
    const int i0 = (idx % CH) * 8;
    __nv_bfloat16* hp = row + h * D;
    const uint4 a = *reinterpret_cast<const uint4*>(hp + i0);
    const uint4 b = *reinterpret_cast<const uint4*>(hp + HALF + i0);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x1 = unpack_bf16x2(av[j]), x2 = unpack_bf16x2(bv[j]);
      const float c0 = cs[i0 + 2 * j], c1 = cs[i0 + 2 * j + 1];
      const float s0 = cs[HALF + i0 + 2 * j], s1 = cs[HALF + i0 + 2 * j + 1];
      const float y10 = x1.x * c0 - x2.x * s0, y11 = x1.y * c1 - x2.y * s1;
      const float y20 = x2.x * c0 + x1.x * s0, y21 = x2.y * c1 + x1.y * s1;
      ya[j] = pack_bf16x2(y10, y11);
      yb[j] = pack_bf16x2(y20, y21);
    }
    const uint4 oa = make_uint4(ya[0], ya[1], ya[2], ya[3]), ob = make_uint4(yb[0], yb[1], yb[2], yb[3]);
    *reinterpret_cast<uint4*>(hp + i0) = oa;
    *reinterpret_cast<uint4*>(hp + HALF + i0) = ob;
    if (k_cache != nullptr && h >= Hq) {
      __nv_bfloat16* kc = k_cache + (int64_t)(h - Hq) * kh_stride;
      *reinterpret_cast<uint4*>(kc + i0) = oa;
      *reinterpret_cast<uint4*>(kc + HALF + i0) = ob;
    }
  }
}

}  // namespace gsb
