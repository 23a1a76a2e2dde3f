// Routing + LoRA metadata in one launch.
//
// For a flattened batch of request chunks this computes, per token:
//   adapter index  = expert of the most recent control token at or before it
//                    in the same request (carry-in from earlier chunks), 0 if none;
//   LoRA index     = adapter index, zeroed on probe slots;
//   modified id    = control id replaced by its substitute (token exchange);
// per request the carry-out, and per LoRA module group the kernel-local adapter
// id of every row plus a 64-bit "adapters present" mask per 128-row GEMM tile.
//
// The reference gets the first two from two attention heads over a coded
// memory plus a separate Triton bitmask kernel (reference:
// src/granite_switch/vllm/switch/multi.py:348-525 and
// src/granite_switch/vllm/core/lora_kernel_meta.py:31-91); the latest-wins
// value those heads produce is computed here exactly by a segmented max-scan.
#include "common.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cub/block/block_scan.cuh>

namespace gsb {

struct MaxOp {
  __device__ __forceinline__ int operator()(int a, int b) const { return a > b ? a : b; }
};

template <int THREADS>
__global__ void routing_kernel(const int64_t* __restrict__ ids, const int32_t* __restrict__ seq_starts,
                               const int32_t* __restrict__ carry_in, const int32_t* __restrict__ expert_tbl,
                               int64_t tbl_size, const int64_t* __restrict__ lut, int64_t lut_size,
                               const uint8_t* __restrict__ kind_lut, int num_adapters,
                               const int32_t* __restrict__ remap, int n_maps,
                               int32_t* __restrict__ adapter_idx, int32_t* __restrict__ lora_idx,
                               int64_t* __restrict__ modified_ids, int32_t* __restrict__ carry_out,
                               int32_t* __restrict__ row_adapter, unsigned long long* __restrict__ tile_mask,
                               int T, int n_tiles) {
  using Scan = cub::BlockScan<int, THREADS>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int s_expert[THREADS];
  __shared__ int s_carry;
  const int seq = blockIdx.x;
  const int a = seq_starts[seq], b = seq_starts[seq + 1];
  if (threadIdx.x == 0) s_carry = carry_in ? carry_in[seq] : 0;
  __syncthreads();
  for (int base = a; base < b; base += THREADS) {
    const int t = base + threadIdx.x;
    int e = -1;
    int64_t id = 0;
    if (t < b) {
      id = ids[t];
      if (id >= 0 && id < tbl_size) e = expert_tbl[id];
    }
    s_expert[threadIdx.x] = e;
    int key = (e >= 0) ? (int)threadIdx.x : -1;
    int last;
    Scan(tmp).InclusiveScan(key, last, MaxOp());
    __syncthreads();  // s_expert visible
    const int carry = s_carry;
    int v = (last >= 0) ? s_expert[last] : carry;
    v = v < 0 ? 0 : (v > num_adapters ? num_adapters : v);
    if (t < b) {
      adapter_idx[t] = v;
      const int lv = (kind_lut != nullptr && kind_lut[v]) ? 0 : v;
      lora_idx[t] = lv;
      int64_t mid = id;
      if (lut != nullptr && id >= 0 && id < lut_size) {
        const int64_t s = lut[id];
        if (s >= 0) mid = s;
      }
      modified_ids[t] = mid;
      for (int m = 0; m < n_maps; ++m) {
        const int local = remap[m * (num_adapters + 1) + lv];
        row_adapter[(int64_t)m * T + t] = local;
        if (local > 0) atomicOr(&tile_mask[(int64_t)m * n_tiles + t / 128], 1ull << (local - 1));
      }
    }
    __syncthreads();
    // the last thread of the chunk (or of the sequence) publishes the carry
    const int last_t = min(b, base + THREADS) - 1 - base;
    if ((int)threadIdx.x == last_t) s_carry = v;
    __syncthreads();
  }
  if (threadIdx.x == 0 && carry_out != nullptr) carry_out[seq] = s_carry;
}

}  // namespace gsb

using namespace gsb;

void gsb_routing(const at::Tensor& ids, const at::Tensor& seq_starts, const c10::optional<at::Tensor>& carry_in,
                 const at::Tensor& expert_tbl, const c10::optional<at::Tensor>& lut,
                 const c10::optional<at::Tensor>& kind_lut, int64_t num_adapters,
                 const c10::optional<at::Tensor>& remap, const at::Tensor& adapter_idx,
                 const at::Tensor& lora_idx, const at::Tensor& modified_ids,
                 const c10::optional<at::Tensor>& carry_out, const c10::optional<at::Tensor>& row_adapter,
                 const c10::optional<at::Tensor>& tile_mask) {
  GSB_CHECK(ids.scalar_type() == at::kLong && seq_starts.scalar_type() == at::kInt &&
                expert_tbl.scalar_type() == at::kInt,
            "routing: int64 ids, int32 seq_starts and expert table required");
  const int T = (int)ids.numel();
  const int S = (int)seq_starts.numel() - 1;
  if (S <= 0) return;
  c10::cuda::CUDAGuard g(ids.device());
  auto st = c10::cuda::getCurrentCUDAStream(ids.device().index()).stream();
  int n_maps = 0, n_tiles = (T + 127) / 128;
  const int32_t* rp = nullptr;
  int32_t* rap = nullptr;
  unsigned long long* tmp = nullptr;
  if (remap.has_value()) {
    GSB_CHECK(remap->scalar_type() == at::kInt && remap->size(1) == num_adapters + 1,
              "routing: remap must be int32 [n_maps, NA+1]");
    n_maps = (int)remap->size(0);
    rp = remap->data_ptr<int32_t>();
    GSB_CHECK(row_adapter.has_value() && tile_mask.has_value(), "routing: outputs for remap required");
    GSB_CHECK(row_adapter->numel() >= (int64_t)n_maps * T && tile_mask->numel() >= (int64_t)n_maps * n_tiles,
              "routing: metadata outputs too small");
    rap = row_adapter->data_ptr<int32_t>();
    tmp = reinterpret_cast<unsigned long long*>(tile_mask->data_ptr<int64_t>());
    GSB_CUDA_CHECK(cudaMemsetAsync(tmp, 0, sizeof(int64_t) * (size_t)n_maps * n_tiles, st));
  }
  const uint8_t* kp = nullptr;
  if (kind_lut.has_value()) {
    GSB_CHECK(kind_lut->scalar_type() == at::kBool || kind_lut->scalar_type() == at::kByte,
              "routing: kind_lut must be bool");
    kp = reinterpret_cast<const uint8_t*>(kind_lut->data_ptr());
  }
  routing_kernel<256><<<(::gsb::count_launch(), S), 256, 0, st>>>(
      ids.data_ptr<int64_t>(), seq_starts.data_ptr<int32_t>(),
      carry_in.has_value() ? carry_in->data_ptr<int32_t>() : nullptr, expert_tbl.data_ptr<int32_t>(),
      expert_tbl.numel(), lut.has_value() ? lut->data_ptr<int64_t>() : nullptr,
      lut.has_value() ? lut->numel() : 0, kp, (int)num_adapters, rp, n_maps, adapter_idx.data_ptr<int32_t>(),
      lora_idx.data_ptr<int32_t>(), modified_ids.data_ptr<int64_t>(),
      carry_out.has_value() ? carry_out->data_ptr<int32_t>() : nullptr, rap, tmp, T, n_tiles);
  GSB_CUDA_CHECK(cudaGetLastError());
}
