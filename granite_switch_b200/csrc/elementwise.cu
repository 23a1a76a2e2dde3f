// Memory-bound kernels of the decoder step, all with 16-byte vector accesses:
//   * rmsnorm (optionally gathering rows, e.g. the last token of each request)
//   * embedding gather fused with control-token exchange and embedding_multiplier
//   * RoPE (NeoX rotate-half) on q and k fused with the paged KV-cache write
//   * greedy argmax over fp32 logits
// (reference hot path: vLLM RMSNorm / get_rope / VocabParallelEmbedding /
// sampler as called from src/granite_switch/vllm/decoder/lora/decoder.py:136-215
// and src/granite_switch/vllm/granite_switch_model.py:423-433.)
#include "common.cuh"
#include "rope.cuh"
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

// ---------------------------------------------------------------- rmsnorm
// One CTA per output row; H is a multiple of 8. The row is held in registers
// (up to 16 bf16x8 vectors per thread, i.e. H <= 16 * 8 * blockDim).
template <int VPT>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                               int64_t ldo, const int64_t* __restrict__ rows, int H, float eps) {
  griddep_launch();  // a GEMM launched as this kernel's dependent may start its set-up
  griddep_wait();    // launched as a dependent itself: x is the previous kernel's output
  const int r = blockIdx.x;
  const int64_t src = rows ? rows[r] : r;
  const uint4* xv = reinterpret_cast<const uint4*>(x + src * ldx);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4* ov = reinterpret_cast<uint4*>(out + (int64_t)r * ldo);
  const int nvec = H / 8;
  uint4 buf[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      buf[i] = xv[v];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&buf[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = unpack_bf16x2(p[j]);
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
      uint4 wq = wv[v];
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wq);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = unpack_bf16x2(p[j]);
        float2 g = unpack_bf16x2(pw[j]);
        // normalise in fp32, round to bf16, then scale by the weight (Granite RMSNorm)
        float a = __bfloat162float(__float2bfloat16_rn(f.x * inv));
        float b = __bfloat162float(__float2bfloat16_rn(f.y * inv));
        o[j] = pack_bf16x2(a * g.x, b * g.y);
      }
      ov[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ---------------------------------------------------------------- embedding
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             const int64_t* __restrict__ lut, int64_t lut_size, int64_t vocab,
                             float mult, __nv_bfloat16* __restrict__ out, int H, uint32_t* err) {
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (lut != nullptr && id >= 0 && id < lut_size) {
    const int64_t s = lut[id];
    if (s >= 0) id = s;
  }
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report_bad_index(err, kSiteEmbedId, id);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * (int64_t)H);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)t * H);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    uint4 q = src[v];
    uint32_t* p = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16x2(p[j]);
      p[j] = pack_bf16x2(f.x * mult, f.y * mult);
    }
    dst[v] = q;
  }
}

// ---------------------------------------------------------------- rope + kv write
// qkv: [T, (Hq + 2 Hkv) * D] bf16. q heads are rotated in place; k is rotated
// and, with v, written to the paged cache laid out [num_blocks, Hkv, BS, D].
// cos_sin: [max_pos, D] fp32 with cos in [0, D/2) and sin in [D/2, D).
template <int D>
__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ldq,
                               const int64_t* __restrict__ positions,
                               const float* __restrict__ cos_sin, int max_pos,
                               __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                               const int64_t* __restrict__ slots, int Hq, int Hkv, int BS,
                               int64_t num_slots, uint32_t* err) {
  griddep_wait();  // launched as a dependent of the projection that writes qkv
  const int t = blockIdx.x;
  int64_t pos = positions[t];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) report_bad_index(err, kSiteRopePos, pos);
    pos = 0;
  }
  const float* cs = cos_sin + pos * D;
  __nv_bfloat16* row = qkv + (int64_t)t * ldq;
  const int64_t slot = slots ? slots[t] : -1;
  // rotate q and k heads; with a valid slot the rotated k heads also go to the cache
  __nv_bfloat16* kc = nullptr;
  if (slot >= 0 && slot < num_slots) kc = k_cache + ((slot / BS) * Hkv * BS + slot % BS) * D;
  rope_rotate_row<D>(row, cs, Hq, Hkv, kc, (int64_t)BS * D);
  if (slot >= 0 && slot < num_slots) {
    const __nv_bfloat16* vrow = row + (Hq + Hkv) * D;
    const int64_t blk = slot / BS, off = slot % BS;
    for (int v = threadIdx.x; v < Hkv * D / 8; v += blockDim.x) {
      const int kh = (v * 8) / D;
      const int d0 = (v * 8) % D;
      const uint4 q = *reinterpret_cast<const uint4*>(vrow + kh * D + d0);
      *reinterpret_cast<uint4*>(v_cache + ((blk * Hkv + kh) * BS + off) * D + d0) = q;
    }
  } else if (slot >= num_slots && threadIdx.x == 0) {
    report_bad_index(err, kSiteKvSlot, slot);
  }
}

// ---------------------------------------------------------------- argmax
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t ld, int V,
                              int64_t* __restrict__ out) {
  const int r = blockIdx.x;
  const float* row = logits + (int64_t)r * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[r] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

}  // namespace gsb

using namespace gsb;

static cudaStream_t cur_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void gsb_rmsnorm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                 const c10::optional<at::Tensor>& rows, double eps) {
  GSB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                out.scalar_type() == at::kBFloat16,
            "rmsnorm: bf16 CUDA tensors required");
  const int H = (int)x.size(1);
  GSB_CHECK(H % 8 == 0 && x.stride(1) == 1 && out.stride(1) == 1 && w.numel() == H,
            "rmsnorm: H must be a multiple of 8 with contiguous rows");
  GSB_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "rmsnorm: rows must be 16-byte aligned");
  const int n = rows.has_value() ? (int)rows->numel() : (int)x.size(0);
  GSB_CHECK(out.size(0) >= n, "rmsnorm: output too small");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const int threads = 256;
  const int vpt = (H / 8 + threads - 1) / threads;
  const int64_t* rp = rows.has_value() ? rows->data_ptr<int64_t>() : nullptr;
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto st = cur_stream(x);
  if (vpt <= 1)
    launch_dependent(rmsnorm_kernel<1>, dim3(n), dim3(threads), 0, st, xp, x.stride(0), wp, op, out.stride(0), rp, H, (float)eps);
  else if (vpt <= 2)
    launch_dependent(rmsnorm_kernel<2>, dim3(n), dim3(threads), 0, st, xp, x.stride(0), wp, op, out.stride(0), rp, H, (float)eps);
  else if (vpt <= 4)
    launch_dependent(rmsnorm_kernel<4>, dim3(n), dim3(threads), 0, st, xp, x.stride(0), wp, op, out.stride(0), rp, H, (float)eps);
  else {
    GSB_CHECK(vpt <= 8, "rmsnorm: H too large");
    launch_dependent(rmsnorm_kernel<8>, dim3(n), dim3(threads), 0, st, xp, x.stride(0), wp, op, out.stride(0), rp, H, (float)eps);
  }
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_embed(const at::Tensor& ids, const at::Tensor& table, const c10::optional<at::Tensor>& lut,
               double mult, const at::Tensor& out, const at::Tensor& err) {
  GSB_CHECK(ids.scalar_type() == at::kLong && table.scalar_type() == at::kBFloat16 &&
                out.scalar_type() == at::kBFloat16,
            "embed: int64 ids and bf16 table/out required");
  const int T = (int)ids.numel();
  const int H = (int)table.size(1);
  GSB_CHECK(H % 8 == 0 && table.is_contiguous() && out.is_contiguous() && out.size(1) == H,
            "embed: contiguous [*, H] tensors with H % 8 == 0 required");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(ids.device());
  const int64_t* lp = lut.has_value() ? lut->data_ptr<int64_t>() : nullptr;
  const int64_t ls = lut.has_value() ? lut->numel() : 0;
  embed_kernel<<<(::gsb::count_launch(), T), 128, 0, cur_stream(ids)>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), lp, ls,
      table.size(0), (float)mult, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H,
      reinterpret_cast<uint32_t*>(err.data_ptr()));
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_rope_kv(const at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                 const c10::optional<at::Tensor>& k_cache, const c10::optional<at::Tensor>& v_cache,
                 const c10::optional<at::Tensor>& slots, int64_t num_q_heads, int64_t num_kv_heads,
                 int64_t head_dim, const at::Tensor& err) {
  GSB_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1, "rope: bf16 qkv required");
  GSB_CHECK(qkv.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15) == 0,
            "rope: qkv rows must be 16-byte aligned");
  GSB_CHECK(positions.scalar_type() == at::kLong && cos_sin.scalar_type() == at::kFloat,
            "rope: int64 positions and fp32 cos_sin required");
  GSB_CHECK(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * head_dim, "rope: qkv too narrow");
  GSB_CHECK(cos_sin.size(1) == head_dim, "rope: cos_sin must be [max_pos, head_dim]");
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.device());
  __nv_bfloat16* kc = nullptr;
  __nv_bfloat16* vc = nullptr;
  int BS = 16;
  int64_t num_slots = 0;
  const int64_t* sp = nullptr;
  if (slots.has_value()) {
    GSB_CHECK(k_cache.has_value() && v_cache.has_value(), "rope: caches required with slots");
    GSB_CHECK(k_cache->dim() == 4 && k_cache->size(1) == num_kv_heads && k_cache->size(3) == head_dim,
              "rope: cache must be [num_blocks, Hkv, BS, D]");
    GSB_CHECK(k_cache->is_contiguous() && v_cache->is_contiguous(), "rope: contiguous caches required");
    BS = (int)k_cache->size(2);
    num_slots = k_cache->size(0) * BS;
    kc = reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr());
    vc = reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr());
    sp = slots->data_ptr<int64_t>();
  }
  auto* qp = reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr());
  auto* ep = reinterpret_cast<uint32_t*>(err.data_ptr());
  auto st = cur_stream(qkv);
  const int threads = 256;
  switch (head_dim) {
    case 64:
      launch_dependent(rope_kv_kernel<64>, dim3(T), dim3(threads), 0, st, qp, qkv.stride(0), positions.data_ptr<int64_t>(),
                                                cos_sin.data_ptr<float>(), (int)cos_sin.size(0), kc, vc,
                                                sp, (int)num_q_heads, (int)num_kv_heads, BS, num_slots, ep);
      break;
    case 128:
      launch_dependent(rope_kv_kernel<128>, dim3(T), dim3(threads), 0, st, qp, qkv.stride(0), positions.data_ptr<int64_t>(),
                                                 cos_sin.data_ptr<float>(), (int)cos_sin.size(0), kc, vc,
                                                 sp, (int)num_q_heads, (int)num_kv_heads, BS, num_slots, ep);
      break;
    case 16:
      launch_dependent(rope_kv_kernel<16>, dim3(T), dim3(threads), 0, st, qp, qkv.stride(0), positions.data_ptr<int64_t>(),
                                                cos_sin.data_ptr<float>(), (int)cos_sin.size(0), kc, vc,
                                                sp, (int)num_q_heads, (int)num_kv_heads, BS, num_slots, ep);
      break;
    default:
      GSB_CHECK(false, "rope: unsupported head_dim ", head_dim);
  }
  GSB_CUDA_CHECK(cudaGetLastError());
}

void gsb_argmax(const at::Tensor& logits, const at::Tensor& out) {
  GSB_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1 && out.scalar_type() == at::kLong,
            "argmax: fp32 logits and int64 out required");
  const int B = (int)logits.size(0);
  if (B == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  argmax_kernel<<<(::gsb::count_launch(), B), 512, 0, cur_stream(logits)>>>(logits.data_ptr<float>(), logits.stride(0),
                                                   (int)logits.size(1), out.data_ptr<int64_t>());
  GSB_CUDA_CHECK(cudaGetLastError());
}

namespace gsb {
__global__ void residual_axpy_kernel(__nv_bfloat16* __restrict__ h, int64_t ldh, const __nv_bfloat16* __restrict__ y,
                                     int64_t ldy, int H, float scale) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    uint32_t* hp = reinterpret_cast<uint32_t*>(h + (int64_t)t * ldh + c);
    const float2 a = unpack_bf16x2(*hp);
    const float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(y + (int64_t)t * ldy + c));
    *hp = pack_bf16x2(a.x + b.x * scale, a.y + b.y * scale);
  }
}
}  // namespace gsb

// h <- h + y * scale (bf16 rows; the residual add after a reduced MLP output).
void gsb_residual_axpy(const at::Tensor& h, const at::Tensor& y, double scale) {
  using namespace gsb;
  GSB_CHECK(h.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 && h.sizes() == y.sizes() &&
                h.size(1) % 2 == 0 && h.stride(1) == 1 && y.stride(1) == 1,
            "residual_axpy: matching bf16 [T, H] tensors required");
  const int T = (int)h.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(h.device());
  residual_axpy_kernel<<<(::gsb::count_launch(), T), 256, 0, cur_stream(h)>>>(reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), h.stride(0),
                                                     reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
                                                     (int)h.size(1), (float)scale);
  GSB_CUDA_CHECK(cudaGetLastError());
}
