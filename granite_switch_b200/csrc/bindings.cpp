// Python bindings of the native extension granite_switch_b200._C.
// Every op launches on the current PyTorch CUDA stream of its inputs' device.
#include <torch/extension.h>

#include <vector>

#include "ops.h"

#include <atomic>

namespace gsb {
static std::atomic<int64_t> g_kernel_launches{0};
void count_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }
static std::atomic<bool> g_pdl{false};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
}  // namespace gsb

static bool gsb_set_pdl(bool on) { return gsb::g_pdl.exchange(on); }

static int64_t gsb_kernel_launches() { return gsb::g_kernel_launches.load(std::memory_order_relaxed); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("kernel_launches", &gsb_kernel_launches, "kernels launched by this extension since it was loaded");
  m.def("set_pdl", &gsb_set_pdl,
        "launch the GEMMs as programmatic dependents of the kernel before them (returns the old setting)");
  m.doc() = "granite_switch_b200 sm_100a kernels";
  m.def("switched_gemm", &gsb_switched_gemm, "tcgen05 GEMM with fused switched-LoRA expand");
  m.def("gemm_pair_min_m", &gsb_gemm_pair_min_m, "set the smallest M of the CTA-pair GEMM (returns the old value)");
  m.def("gemm_decode_plan", &gsb_gemm_decode_plan,
        "decode-kernel split for (M, N, K, epilogue, swiglu tile): [accumulators, K parts, tiles, stages]");
  m.def("gemm_decode_force_split", &gsb_gemm_decode_force_split,
        "force the decode kernel's (accumulators, K parts) for A/B tests; (0, 0) restores the rule");
  m.def("gemm_decode_trace", &gsb_gemm_decode_trace,
        "record per-CTA phase timestamps of later decode-GEMM launches into a uint64 [CTAs, 16] tensor");
  m.def("gemm_decode_max_m", &gsb_gemm_decode_max_m,
        "set the largest M of the operand-swapped decode GEMM (0: off; -1 reads; returns the old value)");
  m.def("rmsnorm", &gsb_rmsnorm, "RMSNorm (optionally gathering rows)");
  m.def("embed", &gsb_embed, "embedding gather with token exchange and multiplier");
  m.def("rope_kv", &gsb_rope_kv, "RoPE on q/k fused with the paged KV-cache write");
  m.def("argmax", &gsb_argmax, "greedy argmax over fp32 logits");
  m.def("routing", &gsb_routing, "latest-wins routing, token exchange and LoRA tile metadata");
  m.def("sample", &gsb_sample, "temperature / top-k / top-p sampling (Gumbel-max, Philox)");
  m.def("prefill_attention_tc", &gsb_prefill_attention_tc, "tcgen05/TMEM prefill attention (128-row tiles)");
  m.def("peer_barrier", &gsb_peer_barrier,
        "bounded cross-rank barrier over P2P signal pads; the epoch is an int32 counter on the device it advances");
  m.def("rmsnorm_residual_from", &gsb_rmsnorm_residual_from, "h <- y; x <- rmsnorm(y); y <- 0");
  m.def("probe_verdict", &gsb_probe_verdict, "probe-head scores at marker rows");
  m.def("probe_rewrite", &gsb_probe_rewrite, "replace marker logit rows by the probe verdict");
  m.def("moe_route", &gsb_moe_route, "MoE top-k routing, softmax and per-expert segment plan");
  m.def("moe_scatter", &gsb_moe_scatter, "MoE token rows into their experts' segments");
  m.def("gemm_splitk_max_tiles", &gsb_gemm_splitk_max_tiles,
        "single-CTA GEMMs with fewer output tiles split K (0: never; -1 reads)");
  m.def("attn_fp8t_stages", &gsb_attn_fp8t_stages,
        "stages of the fp8 decode kernel with 8-row tiles: 3 (four CTAs per SM) or 2 (five); other values read");
  m.def("attn_decode_stages", &gsb_attn_decode_stages, "decode attention layout: 2 = short rings, three CTAs per SM; 3 = deep rings, two (other values read)");
  m.def("attn_packed", &gsb_attn_packed, "prefill attention softmax on packed f32x2 math (0/1; -1 reads)");
  m.def("moe_scatter_slots", &gsb_moe_scatter_slots, "MoE rows into the slots of an earlier scatter");
  m.def("moe_combine", &gsb_moe_combine, "MoE weighted sum of expert outputs (+ shared MLP, residual)");
  m.def("residual_axpy", &gsb_residual_axpy, "h <- h + y * scale");
  m.def("paged_attention", &gsb_paged_attention, "paged causal GQA attention (prefill + decode; bf16 or fp8 cache)");
  m.def("lora_shrink_small", &gsb_lora_shrink_small,
        "masked LoRA shrink for a few tokens on CUDA cores (each row's own adapter columns only)");
  m.def("quantize_fp8_rows", &gsb_quantize_fp8_rows,
        "bf16 rows -> e4m3 bytes with one power-of-two scale per (row, 128-K block), as scale atoms");
  m.def("fp8_gemm", &gsb_fp8_gemm, "block-scaled fp8 tcgen05 GEMM with the bf16 switched-LoRA expand fused");
  m.def("rope_kv_fp8", &gsb_rope_kv_fp8, "RoPE on q / k then the quantised fp8 K / V write, one launch");
  m.def("kv_write_fp8", &gsb_kv_write_fp8, "quantised (e4m3, per-row scale) write of a step's K/V into the fp8 cache");
}
