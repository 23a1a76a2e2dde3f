// Shared by the GEMM kernels (gemm_tcgen05.cu, gemm_decode.cu): epilogue kinds
// and the multicast reduction store.
#pragma once

#include "common.cuh"

#include <cuda_runtime.h>

#include <cstdint>

namespace gsb {

enum EpiKind : int {
  kEpiStore = 0,     // out(bf16) = acc * scale
  kEpiResAdd = 1,    // out(bf16) = residual + acc * scale  (out may alias residual)
  kEpiSwiGLU = 2,    // out(bf16)[:, n/2] = silu(gate) * up, gate/up interleaved per tile
  kEpiMaskAdapter = 3,  // shrink: keep column j only where row's adapter == (j/r)%NA+1
  kEpiF32 = 4,       // out(fp32) = acc * scale
  // out = multicast address of a symmetric bf16 buffer: every rank adds
  // (residual +) acc * scale into all ranks' copies through NVSwitch
  // (multimem.red), tile by tile as accumulators drain
  kEpiMultimemRed = 5,
};

__device__ __forceinline__ void multimem_red_add_v4_bf16x2(void* mc, uint32_t a, uint32_t b, uint32_t c,
                                                           uint32_t d) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

// Decode-sized GEMM path (gemm_decode.cu). Returns false when the call does not
// qualify (the caller then runs the general kernel). Operands as in
// gsb_switched_gemm; `s` and `lb` are null without LoRA.
struct DecodeGemmArgs {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  void* out;            // bf16 output, or the multicast address (kEpiMultimemRed)
  int64_t ldo;
  int M, N, K;
  int epi;
  float scale;
  const void* residual;  // kEpiResAdd / kEpiMultimemRed (rank 0)
  int64_t ldr;
  int swiglu_tile;       // kEpiSwiGLU: rows per gate|up interleave tile
  // LoRA expand (optional)
  const void* s;         // [M, s_cols] masked shrink output
  int64_t lds;
  int s_cols;
  const void* lb;        // [N, NA*rank]
  int64_t ldlb;
  int rank, num_adapters, num_slices;
  int slice_bounds[5];
  const uint64_t* tile_mask;  // [ceil(M/128)] adapters present per 128-row tile
  // kEpiMaskAdapter (the shrink)
  const int32_t* row_adapter;
  int mask_rank, mask_num_adapters;
  const uint64_t* skip_mask;
};
bool decode_gemm_try(const DecodeGemmArgs& a, uint32_t* err, cudaStream_t stream);

}  // namespace gsb
