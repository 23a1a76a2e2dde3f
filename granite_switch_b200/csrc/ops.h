// Declarations of the host launchers exported by the native extension.
#pragma once

#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <vector>

void gsb_switched_gemm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                       int64_t epi_kind, int64_t bn, const c10::optional<at::Tensor>& residual,
                       double scale, const c10::optional<at::Tensor>& s,
                       const c10::optional<at::Tensor>& lb,
                       const c10::optional<at::Tensor>& tile_mask, int64_t rank,
                       int64_t num_adapters, std::vector<int64_t> slice_bounds,
                       const c10::optional<at::Tensor>& row_adapter, int64_t mask_rank,
                       int64_t mask_num_adapters, const at::Tensor& err);
