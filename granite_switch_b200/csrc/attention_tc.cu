// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// head_dim 64 or 128.
//
// One CTA owns 128 query rows of one request and one KV head (a row is a
// (query token, query head of the GQA group) pair, as in attention.cu) and
// walks the request's paged K/V in tiles of 64 keys:
//
//   S_j  = Q . K_j^T        tcgen05.mma M=128 N=64 K=D, S_j in TMEM (2 buffers)
//   P_j  = softmax rows      softmax warps: tcgen05.ld one S row per thread,
//                            mask, running max/sum in registers, P_j (bf16,
//                            two per column) tcgen05.st over S_j's columns
//   O   += P_j . V_j         tcgen05.mma M=128 N=D K=64 with A = P_j read from
//                            TMEM, O in TMEM; V is read straight from its
//                            [key][d] tile as an MN-major B
//
// Warp roles (192 threads): warp 0 issues the K/V page boxes by TMA, warp 1
// owns TMEM and issues every MMA from one thread, warps 2..5 run the softmax,
// rescale O in TMEM when a row maximum grows by more than 2^8, and write the
// normalised output. K and V have separate two-stage rings: a K stage is
// released when S_j completes (P never touches shared memory), a V stage when
// P_j . V_j completes, and K runs one tile ahead of V. S_{j+1} is issued
// before P_j . V_j, so the tensor core computes the next scores while the
// softmax of the current tile runs, and two CTAs share an SM so one CTA's
// softmax overlaps the other's MMAs. Work tiles arrive heaviest first.
// Every mbarrier wait is bounded; the error word reports a timeout.
// (reference: attention comes from vLLM's backends, called at
// src/granite_switch/vllm/decoder/lora/decoder.py:146-174.)
#include "common.cuh"
#include <cstdlib>
#include "tma_util.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace gsb {

template <int D, int KT_ = 64>
struct FaCfg {
  static constexpr int BM = 128;
  static constexpr int KT = KT_;
  static constexpr int PAGE = 16;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = KT * D * 2;      // one of K or V
  static constexpr int STAGES = 2;
  static constexpr int PT_CAP = 2048;             // page ids staged in shared memory (32k keys)
  static constexpr int SMEM = 1024 + Q_BYTES + STAGES * 2 * KV_BYTES + 512 + PT_CAP * 4;
  static constexpr int TMEM_COLS = (2 * KT + D) <= 256 ? 256 : 512;  // S0 | S1 | O
  static constexpr int S_COL0 = 0, S_COL1 = KT, O_COL = 2 * KT;
};

// byte offset of 16-byte chunk `ch` of row `r` in a [D/64][rows][64] SW128 tile
template <int ROWS>
__device__ __forceinline__ uint32_t fa_sw(int r, int ch) {
  return (uint32_t)((ch >> 3) * (ROWS * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

template <int D, int KT_, bool PACKED>
__global__ void __launch_bounds__(192, 2)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                             const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                             const int32_t* __restrict__ block_table, int bt_stride, int num_blocks,
                             const int32_t* __restrict__ q_start, const int32_t* __restrict__ kv_len_arr,
                             const int32_t* __restrict__ work_seq, const int32_t* __restrict__ work_row0, int Hq,
                             int Hkv, float scale_log2, __nv_bfloat16* __restrict__ out, int64_t out_stride,
                             float* __restrict__ ws_o, float* __restrict__ ws_lse, int nsplit, int T,
                             uint32_t* err) {
  using C = FaCfg<D, KT_>;
  constexpr int KT = C::KT, BM = C::BM, PAGE = C::PAGE;
  static_assert(KT == 64, "the P store below writes 32 TMEM columns (64 keys)");
  griddep_launch();  // a GEMM launched as a dependent may start its set-up
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;                  // [2][KT x D]
  uint8_t* sV = sK + 2 * C::KV_BYTES;             // [2][KT x D]
  uint64_t* k_full = reinterpret_cast<uint64_t*>(sV + 2 * C::KV_BYTES);
  uint64_t* k_empty = k_full + 2;
  uint64_t* v_full = k_empty + 2;
  uint64_t* v_empty = v_full + 2;
  uint64_t* s_full = v_empty + 2;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_pages = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(k_full) + 512);  // [PT_CAP]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, w = blockIdx.y;
  const int seq = work_seq[w];
  const int row0 = work_row0[w];
  const int G = Hq / Hkv;
  const int qs = q_start[seq];
  const int q_len = q_start[seq + 1] - qs;
  const int kv_len = kv_len_arr[seq];
  const int ctx = kv_len - q_len;
  const int n_rows = q_len * G;
  const int32_t* bt = block_table + (int64_t)seq * bt_stride;
  const int last_row = min(row0 + BM, n_rows) - 1;
  // keys [k_begin, k_end): split blockIdx.z of the tile's causal key range,
  // whole 64-key tiles per split (nsplit 1: the whole range)
  const int split = blockIdx.z;
  const int k_limit = max(0, min(kv_len, ctx + last_row / G + 1));
  const int per_split = ((k_limit + nsplit - 1) / nsplit + KT - 1) / KT * KT;
  const int k_begin = min(k_limit, split * per_split);
  const int k_end = min(k_limit, k_begin + per_split);
  const int n_tiles = (k_end - k_begin + KT - 1) / KT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  // page ids of the key range into shared memory: the producer then issues each
  // tile's boxes without a dependent global read per page
  const int pg0 = k_begin / PAGE;
  const int n_pages = max(0, min((k_end + PAGE - 1) / PAGE - pg0, C::PT_CAP));
  for (int i = threadIdx.x; i < n_pages; i += blockDim.x)
    s_pages[i] = checked_index(bt[pg0 + i], num_blocks, err, kSiteTcPage);
  for (int c = threadIdx.x; c < BM * (D / 8); c += blockDim.x) {
    const int r = c / (D / 8), ch = c % (D / 8);
    const int gr = row0 + r;
    const bool valid = gr < n_rows;
    const int tok = valid ? gr / G : 0;
    const int head = kvh * G + (valid ? gr % G : 0);
    const __nv_bfloat16* src = q + (int64_t)(qs + tok) * q_stride + head * D + ch * 8;
    const uint32_t dst = smem_u32(sQ) + fa_sw<BM>(r, ch);
    const int nbytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
                 "l"(valid ? (const void*)src : (const void*)q), "r"(nbytes)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- K/V producer: K runs one tile ahead of V ----------------
    if (lane == 0 && n_tiles > 0) {
      const int first_page = s_pages[0];
      auto load = [&](uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int j) {
        mbar_arrive_expect_tx(bar, C::KV_BYTES);
#pragma unroll
        for (int p = 0; p < KT / PAGE; ++p) {
          const int key = k_begin + j * KT + p * PAGE;
          const int pi = key / PAGE - pg0;
          const int page = (key < k_end) ? (pi < n_pages ? s_pages[pi] : checked_index(bt[pg0 + pi], num_blocks, err,
                                                                                      kSiteTcPage))
                                         : first_page;
          const int row = (page * Hkv + kvh) * PAGE;
#pragma unroll
          for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * (KT * 128) + p * PAGE * 128, tm, bar, h * 64, row);
        }
      };
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      auto issue_k = [&](int j) {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, err, kErrAttnWait)) return false;
        load(sK + s * C::KV_BYTES, &tm_k, &k_full[s], j);
        k_issued = j + 1;
        return true;
      };
      ok = issue_k(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !(ok = issue_k(j + 1))) break;
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&v_empty[s], ((j >> 1) & 1) ^ 1, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        load(sV + s * C::KV_BYTES, &tm_v, &v_full[s], j);
        v_issued = j + 1;
      }
      if (!ok) {
        *abort_flag = 1;
        // drain this CTA's own copies still in flight before the CTA exits
        for (int j = (k_issued > 2 ? k_issued - 2 : 0); j < k_issued; ++j)
          mbar_wait(&k_full[j & 1], (j >> 1) & 1, err, kErrAttnWait);
        for (int j = (v_issued > 2 ? v_issued - 2 : 0); j < v_issued; ++j)
          mbar_wait(&v_full[j & 1], (j >> 1) & 1, err, kErrAttnWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(128, KT);
      const uint32_t idesc_o = umma_idesc_bf16_bmn(128, D);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&k_full[s], (j >> 1) & 1, err, kErrAttnWait)) return false;
        // S_j reuses the TMEM columns of S_{j-2} / P_{j-2}: P_{j-2} . V_{j-2} must be done
        if (j >= 2 && !mbar_wait(&o_done[s], ((j - 2) >> 1) & 1, err, kErrAttnWait)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * C::KV_BYTES);
        const uint32_t tS = tmem + (s ? C::S_COL1 : C::S_COL0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(q_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32);
          const uint64_t bd = umma_desc_sw128(k_addr + (kk >> 2) * (KT * 128) + (kk & 3) * 32);
          umma_bf16(tS, ad, bd, idesc_s, kk != 0);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        return true;
      };
      bool ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !(ok = issue_s(j + 1))) break;
        const int s = j & 1;
        if (*abort_flag || !mbar_wait(&p_full[s], (j >> 1) & 1, err, kErrAttnWait) ||
            !mbar_wait(&v_full[s], (j >> 1) & 1, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tP = tmem + (s ? C::S_COL1 : C::S_COL0);
        const uint32_t v_addr = smem_u32(sV + s * C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          const uint64_t bd = umma_desc_sw128_mn(v_addr + kk * 2048, KT * 128, 1024);
          umma_bf16_tmem_a(tmem + C::O_COL, tP + kk * 8, bd, idesc_o, (j | kk) != 0);
        }
        umma_commit(&o_done[s]);
        umma_commit(&v_empty[s]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    // Each thread owns one row. The running max m (log2 domain) may lag the
    // true maximum by up to kLazyLog2: P = 2^(s - m) then stays below
    // 2^kLazyLog2, which bf16 P and fp32 O / l represent as well as P <= 1,
    // and O in TMEM is rescaled only when some row's max grows by more than
    // that. Without a rescale the warp never waits for the previous P.V.
    constexpr float kLazyLog2 = 8.f;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int gr = row0 + r;
    const int pos = ctx + gr / G;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j & 1;
      const bool got_s = !*abort_flag && mbar_wait(&s_full[s], (j >> 1) & 1, err, kErrAttnWait);
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + (s ? C::S_COL1 : C::S_COL0);
      uint32_t sv[KT];
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) tmem_ld32(tS + c * 32, reinterpret_cast<uint32_t(&)[32]>(sv[c * 32]));
      tmem_wait_ld();
      const int kbase = k_begin + j * KT;
      if (__any_sync(0xffffffffu, kbase + KT - 1 > pos || kbase + KT > k_end)) {
#pragma unroll
        for (int i = 0; i < KT; ++i) {
          const int key = kbase + i;
          if (key > pos || key >= k_end) sv[i] = 0xff800000u;
        }
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = __uint_as_float(sv[i]);
#pragma unroll
      for (int i = 8; i < KT; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(sv[i]));
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale_log2;
      const bool grow = mt > m + kLazyLog2;
      const bool rescale = grow && m != -INFINITY && j > 0;
      if (__any_sync(0xffffffffu, rescale)) {
        const bool got_o = mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err, kErrAttnWait);
        if (!__all_sync(0xffffffffu, got_o)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = rescale ? ex2_approx(m - mt) : 1.f;
        l *= f;
        const uint32_t tO = tmem + lane_base + C::O_COL;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(tO + c * 32, rr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * f);
          tmem_st32(tO + c * 32, rr);
        }
      }
      if (grow) m = mt;
      const float mb = (m == -INFINITY) ? 0.f : m;
      uint32_t pk[KT / 2];
      if constexpr (PACKED) {
        // the scale-and-shift and the row sum on packed fp32 pairs (one f32x2
        // instruction per two scores): fewer issue slots per score for the
        // softmax warps, which share each SM sub-partition with the other CTA
        const uint64_t sc2 = f32x2_pack(scale_log2, scale_log2), nm2 = f32x2_pack(-mb, -mb);
        uint64_t acc[2] = {0ull, 0ull};
#pragma unroll
        for (int i = 0; i < KT / 2; ++i) {
          const uint64_t y = f32x2_fma(f32x2_pack_bits(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
          const float a = ex2_approx(f32x2_lo(y)), b = ex2_approx(f32x2_hi(y));
          acc[i & 1] = f32x2_add(acc[i & 1], f32x2_pack(a, b));
          pk[i] = pack_bf16x2(a, b);
        }
        const uint64_t t = f32x2_add(acc[0], acc[1]);
        l += f32x2_lo(t) + f32x2_hi(t);
      } else {
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < KT / 2; ++i) {
          const float a = ex2_approx(fmaf(__uint_as_float(sv[2 * i]), scale_log2, -mb));
          const float b = ex2_approx(fmaf(__uint_as_float(sv[2 * i + 1]), scale_log2, -mb));
          rs[i & 3] += a + b;
          pk[i] = pack_bf16x2(a, b);
        }
        l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      }
      tmem_st32(tS, pk);  // P_j over the first 32 columns of S_j
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    const bool go = ok && n_tiles > 0 && !*abort_flag;
    if (__all_sync(0xffffffffu, go)) {
      const int jl = n_tiles - 1;
      if (__all_sync(0xffffffffu, mbar_wait(&o_done[jl & 1], (jl >> 1) & 1, err, kErrAttnWait))) {
        tc_fence_after();
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        const bool valid = gr < n_rows;
        const int tok = qs + (valid ? gr / G : 0);
        const int head = kvh * G + (valid ? gr % G : 0);
        __nv_bfloat16* op = out + (int64_t)tok * out_stride + head * D;
        const uint32_t tO = tmem + lane_base + C::O_COL;
        // split partial: normalised fp32 O and the row's log2-sum-exp, merged
        // afterwards (m lags the row maximum by at most 2^8, l matches it)
        const int64_t ws_row = ((int64_t)split * T + tok) * Hq + head;
        if (nsplit > 1 && valid) ws_lse[ws_row] = (l > 0.f) ? m + log2f(l) : -INFINITY;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(tO + c * 32, rr);
          tmem_wait_ld();
          if (nsplit > 1) {
            if (valid) {
              float4* w4 = reinterpret_cast<float4*>(ws_o + ws_row * D + c * 32);
#pragma unroll
              for (int e = 0; e < 8; ++e)
                w4[e] = make_float4(__uint_as_float(rr[4 * e]) * inv, __uint_as_float(rr[4 * e + 1]) * inv,
                                    __uint_as_float(rr[4 * e + 2]) * inv, __uint_as_float(rr[4 * e + 3]) * inv);
            }
          } else if (valid) {
            uint4* o4 = reinterpret_cast<uint4*>(op + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              o4[e] = make_uint4(pack_bf16x2(__uint_as_float(rr[8 * e]) * inv, __uint_as_float(rr[8 * e + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 2]) * inv, __uint_as_float(rr[8 * e + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 4]) * inv, __uint_as_float(rr[8 * e + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 6]) * inv, __uint_as_float(rr[8 * e + 7]) * inv));
          }
        }
      } else {
        *abort_flag = 1;
      }
    } else if (n_tiles == 0 && gr < n_rows) {
      if (nsplit > 1) {
        ws_lse[((int64_t)split * T + qs + gr / G) * Hq + kvh * G + gr % G] = -INFINITY;  // empty split
      } else {
        __nv_bfloat16* op = out + (int64_t)(qs + gr / G) * out_stride + (kvh * G + gr % G) * D;
        for (int c = 0; c < D; c += 8) *reinterpret_cast<uint4*>(op + c) = make_uint4(0, 0, 0, 0);
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// Two query tiles per CTA ("ping-pong"): 256 rows of one request and KV head,
// 128-key tiles, one CTA per SM.
//
//   TMEM (512 columns): S_A [0,128) | S_B [128,256) | O_A | O_B (D columns each)
//   warp 0: K/V TMA producer, warp 1: TMEM owner + MMA issuer,
//   warps 2..5: softmax of tile A, warps 6..9: softmax of tile B.
//
// Each K/V tile in shared memory serves both query tiles (half the K/V traffic
// per query row of the one-tile kernel), and each S tile holds 128 keys, so a
// softmax pass does twice the work per TMEM round trip. The MMA issuer runs
//   S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) ...
// so the tensor core computes one tile's products while the other tile's
// softmax runs. S_t(j+1) reuses S_t's columns (P_t(j) lives in the first 64
// of them): it is issued after PV_t(j) by the same thread, and tcgen05.mma
// operations from one thread execute in issue order. Every wait is bounded.
template <int D>
struct FaPPCfg {
  static constexpr int BM = 128;            // rows per query tile
  static constexpr int KT = 128;            // keys per tile
  static constexpr int PAGE = 16;
  static constexpr int Q_BYTES = BM * D * 2;  // one query tile
  static constexpr int KV_BYTES = KT * D * 2;  // one K (or V) tile
  static constexpr int STAGES = 2;
  static constexpr int PT_CAP = 4096;             // page ids staged in shared memory (64k keys)
  static constexpr int SMEM = 1024 + 2 * Q_BYTES + STAGES * 2 * KV_BYTES + 512 + PT_CAP * 4;
  static constexpr int TMEM_COLS = 512;
  static constexpr int S_COL = 0;           // + t * KT
  static constexpr int O_COL = 2 * KT;      // + t * D
};

template <int D, bool PACKED>
__global__ void __launch_bounds__(320, 1)
    fa_pingpong_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                       const int32_t* __restrict__ block_table, int bt_stride, int num_blocks,
                       const int32_t* __restrict__ q_start, const int32_t* __restrict__ kv_len_arr,
                       const int32_t* __restrict__ work_seq, const int32_t* __restrict__ work_row0, int Hq,
                       int Hkv, float scale_log2, __nv_bfloat16* __restrict__ out, int64_t out_stride,
                       uint32_t* err) {
  using C = FaPPCfg<D>;
  constexpr int KT = C::KT, BM = C::BM, PAGE = C::PAGE, ST = C::STAGES;
  griddep_launch();  // a GEMM launched as a dependent may start its set-up
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                               // [2][D/64][BM][64]
  uint8_t* sK = sQ + 2 * C::Q_BYTES;                // [ST][D/64][KT][64]
  uint8_t* sV = sK + ST * C::KV_BYTES;              // [ST][D/64][KT][64]
  uint64_t* k_full = reinterpret_cast<uint64_t*>(sV + ST * C::KV_BYTES);
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;   // [2] per query tile
  uint64_t* p_full = s_full + 2;     // [2]
  uint64_t* o_done = p_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_pages = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(k_full) + 512);  // [PT_CAP]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, w = blockIdx.y;
  const int seq = work_seq[w];
  const int row0 = work_row0[w];
  const int G = Hq / Hkv;
  const int qs = q_start[seq];
  const int q_len = q_start[seq + 1] - qs;
  const int kv_len = kv_len_arr[seq];
  const int ctx = kv_len - q_len;
  const int n_rows = q_len * G;
  const int32_t* bt = block_table + (int64_t)seq * bt_stride;
  const int last_row = min(row0 + 2 * BM, n_rows) - 1;
  const int k_end = max(0, min(kv_len, ctx + last_row / G + 1));
  const int n_tiles = (k_end + KT - 1) / KT;
  const int nq = (row0 + BM < n_rows) ? 2 : 1;   // query tiles with any valid row

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  const int n_pages = min((k_end + PAGE - 1) / PAGE, C::PT_CAP);
  for (int i = threadIdx.x; i < n_pages; i += blockDim.x) s_pages[i] = checked_index(bt[i], num_blocks, err, kSiteTcPage);
  for (int c = threadIdx.x; c < 2 * BM * (D / 8); c += blockDim.x) {
    const int rr = c / (D / 8), ch = c % (D / 8);
    const int t = rr / BM, r = rr % BM;
    const int gr = row0 + rr;
    const bool valid = gr < n_rows;
    const int tok = valid ? gr / G : 0;
    const int head = kvh * G + (valid ? gr % G : 0);
    const __nv_bfloat16* src = q + (int64_t)(qs + tok) * q_stride + head * D + ch * 8;
    const uint32_t dst = smem_u32(sQ + t * C::Q_BYTES) + fa_sw<BM>(r, ch);
    const int nbytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
                 "l"(valid ? (const void*)src : (const void*)q), "r"(nbytes)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- K/V producer: K runs one tile ahead of V ----------------
    if (lane == 0 && n_tiles > 0) {
      const int first_page = s_pages[0];
      auto load = [&](uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int j) {
        mbar_arrive_expect_tx(bar, C::KV_BYTES);
#pragma unroll
        for (int p = 0; p < KT / PAGE; ++p) {
          const int key = j * KT + p * PAGE;
          const int pi = key / PAGE;
          const int page = (key < k_end) ? (pi < n_pages ? s_pages[pi] : checked_index(bt[pi], num_blocks, err,
                                                                                      kSiteTcPage))
                                         : first_page;
          const int row = (page * Hkv + kvh) * PAGE;
#pragma unroll
          for (int h = 0; h < D / 64; ++h) tma_load_2d(dst + h * (KT * 128) + p * PAGE * 128, tm, bar, h * 64, row);
        }
      };
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      auto issue_k = [&](int j) {
        const int st = j % ST;
        if (*abort_flag || !mbar_wait(&k_empty[st], ((j / ST) & 1) ^ 1, err, kErrAttnWait)) return false;
        load(sK + st * C::KV_BYTES, &tm_k, &k_full[st], j);
        k_issued = j + 1;
        return true;
      };
      ok = issue_k(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !(ok = issue_k(j + 1))) break;
        const int st = j % ST;
        if (*abort_flag || !mbar_wait(&v_empty[st], ((j / ST) & 1) ^ 1, err, kErrAttnWait)) {
          ok = false;
          break;
        }
        load(sV + st * C::KV_BYTES, &tm_v, &v_full[st], j);
        v_issued = j + 1;
      }
      if (!ok) {
        *abort_flag = 1;
        for (int j = (k_issued > ST ? k_issued - ST : 0); j < k_issued; ++j)
          mbar_wait(&k_full[j % ST], (j / ST) & 1, err, kErrAttnWait);
        for (int j = (v_issued > ST ? v_issued - ST : 0); j < v_issued; ++j)
          mbar_wait(&v_full[j % ST], (j / ST) & 1, err, kErrAttnWait);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(128, KT);
      const uint32_t idesc_o = umma_idesc_bf16_bmn(128, D);
      auto issue_s = [&](int t, int j) -> bool {
        const int st = j % ST;
        if (t == 0 && (*abort_flag || !mbar_wait(&k_full[st], (j / ST) & 1, err, kErrAttnWait))) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + t * C::Q_BYTES);
        const uint32_t k_addr = smem_u32(sK + st * C::KV_BYTES);
        const uint32_t tS = tmem + C::S_COL + t * KT;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(q_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32);
          const uint64_t bd = umma_desc_sw128(k_addr + (kk >> 2) * (KT * 128) + (kk & 3) * 32);
          umma_bf16(tS, ad, bd, idesc_s, kk != 0);
        }
        umma_commit(&s_full[t]);
        if (t == nq - 1) umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        const int st = j % ST;
        if (*abort_flag || (t == 0 && !mbar_wait(&v_full[st], (j / ST) & 1, err, kErrAttnWait)) ||
            !mbar_wait(&p_full[t], j & 1, err, kErrAttnWait))
          return false;
        tc_fence_after();
        const uint32_t tP = tmem + C::S_COL + t * KT;
        const uint32_t v_addr = smem_u32(sV + st * C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          const uint64_t bd = umma_desc_sw128_mn(v_addr + kk * 2048, KT * 128, 1024);
          umma_bf16_tmem_a(tmem + C::O_COL + t * D, tP + kk * 8, bd, idesc_o, (j | kk) != 0);
        }
        umma_commit(&o_done[t]);
        if (t == nq - 1) umma_commit(&v_empty[st]);
        return true;
      };
      bool ok = issue_s(0, 0) && (nq < 2 || issue_s(1, 0));
      for (int j = 0; j < n_tiles && ok; ++j) {
        for (int t = 0; t < nq && ok; ++t) {
          ok = issue_pv(t, j);
          if (ok && j + 1 < n_tiles) ok = issue_s(t, j + 1);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax + epilogue: warps 2..5 tile A, 6..9 tile B ----------------
    constexpr float kLazyLog2 = 8.f;
    const int t = (warp - 2) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int gr = row0 + t * BM + r;
    const int pos = ctx + gr / G;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t tS = tmem + lane_base + C::S_COL + t * KT;
    const uint32_t tO = tmem + lane_base + C::O_COL + t * D;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    const bool live = t < nq;
    for (int j = 0; live && j < n_tiles; ++j) {
      const bool got_s = !*abort_flag && mbar_wait(&s_full[t], j & 1, err, kErrAttnWait);
      if (!__all_sync(0xffffffffu, got_s)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[KT];
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) tmem_ld32(tS + c * 32, reinterpret_cast<uint32_t(&)[32]>(sv[c * 32]));
      tmem_wait_ld();
      const int kbase = j * KT;
      if (__any_sync(0xffffffffu, kbase + KT - 1 > pos || kbase + KT > k_end)) {
#pragma unroll
        for (int i = 0; i < KT; ++i) {
          const int key = kbase + i;
          if (key > pos || key >= k_end) sv[i] = 0xff800000u;
        }
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = __uint_as_float(sv[i]);
#pragma unroll
      for (int i = 8; i < KT; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(sv[i]));
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale_log2;
      const bool grow = mt > m + kLazyLog2;
      const bool rescale = grow && m != -INFINITY && j > 0;
      if (__any_sync(0xffffffffu, rescale)) {
        // O_t must hold P_t(j-1) . V(j-1) before it is scaled
        const bool got_o = mbar_wait(&o_done[t], (j - 1) & 1, err, kErrAttnWait);
        if (!__all_sync(0xffffffffu, got_o)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = rescale ? ex2_approx(m - mt) : 1.f;
        l *= f;
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {  // 16 columns at a time: the 128 scores stay in registers
          uint32_t rr[16];
          tmem_ld16(tO + c * 16, rr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * f);
          tmem_st16(tO + c * 16, rr);
        }
      }
      if (grow) m = mt;
      const float mb = (m == -INFINITY) ? 0.f : m;
      // P_t(j) as bf16 pairs over the first KT/2 columns of S_t. Packed in place:
      // pair i lands in sv[i], whose own score was read by an earlier pair.
      if constexpr (PACKED) {
        const uint64_t sc2 = f32x2_pack(scale_log2, scale_log2), nm2 = f32x2_pack(-mb, -mb);
        uint64_t acc[2] = {0ull, 0ull};
#pragma unroll
        for (int i = 0; i < KT / 2; ++i) {
          const uint64_t y = f32x2_fma(f32x2_pack_bits(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
          const float a = ex2_approx(f32x2_lo(y)), b = ex2_approx(f32x2_hi(y));
          acc[i & 1] = f32x2_add(acc[i & 1], f32x2_pack(a, b));
          sv[i] = pack_bf16x2(a, b);
        }
        const uint64_t tt = f32x2_add(acc[0], acc[1]);
        l += f32x2_lo(tt) + f32x2_hi(tt);
      } else {
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < KT / 2; ++i) {
          const float a = ex2_approx(fmaf(__uint_as_float(sv[2 * i]), scale_log2, -mb));
          const float b = ex2_approx(fmaf(__uint_as_float(sv[2 * i + 1]), scale_log2, -mb));
          rs[i & 3] += a + b;
          sv[i] = pack_bf16x2(a, b);
        }
        l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      }
      tmem_st32(tS, reinterpret_cast<uint32_t(&)[32]>(sv[0]));
      tmem_st32(tS + 32, reinterpret_cast<uint32_t(&)[32]>(sv[32]));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    const bool go = live && ok && n_tiles > 0 && !*abort_flag;
    if (__all_sync(0xffffffffu, go)) {
      const int jl = n_tiles - 1;
      if (__all_sync(0xffffffffu, mbar_wait(&o_done[t], jl & 1, err, kErrAttnWait))) {
        tc_fence_after();
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        const bool valid = gr < n_rows;
        const int tok = qs + (valid ? gr / G : 0);
        const int head = kvh * G + (valid ? gr % G : 0);
        __nv_bfloat16* op = out + (int64_t)tok * out_stride + head * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32(tO + c * 32, rr);
          tmem_wait_ld();
          if (valid) {
            uint4* o4 = reinterpret_cast<uint4*>(op + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              o4[e] = make_uint4(pack_bf16x2(__uint_as_float(rr[8 * e]) * inv, __uint_as_float(rr[8 * e + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 2]) * inv, __uint_as_float(rr[8 * e + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 4]) * inv, __uint_as_float(rr[8 * e + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(rr[8 * e + 6]) * inv, __uint_as_float(rr[8 * e + 7]) * inv));
          }
        }
      }
    } else if (live && n_tiles == 0 && gr < n_rows) {
      __nv_bfloat16* op = out + (int64_t)(qs + gr / G) * out_stride + (kvh * G + gr % G) * D;
      for (int c = 0; c < D; c += 8) *reinterpret_cast<uint4*>(op + c) = make_uint4(0, 0, 0, 0);
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}
}  // namespace gsb

using namespace gsb;

// Softmax arithmetic: 0 = scalar fp32, 1 = packed f32x2 scale-and-shift and row
// sums (attn_packed() switches it at run time for A/B tests). Taking a quarter
// of the exponentials off MUFU with a polynomial was measured slower on B200
// (530 vs 518 TFLOP/s causal 4k), so the exponentials stay on ex2.approx.
static int g_attn_packed = 1;

int64_t gsb_attn_packed(int64_t v) {
  const int64_t old = g_attn_packed;
  if (v >= 0) g_attn_packed = (int)v;
  return old;
}

// Same metadata contract as gsb_paged_attention (rows_per_tile = 128 or 256).
// nsplit > 1 (128-row tiles only) splits each tile's key range over CTAs, as the
// paged kernel's flash-decoding split, with the same workspaces and merge.
void gsb_prefill_attention_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                              const at::Tensor& block_table, const at::Tensor& q_start, const at::Tensor& kv_len,
                              const at::Tensor& work_seq, const at::Tensor& work_row0, int64_t num_q_heads,
                              double scale, const at::Tensor& out, const at::Tensor& err, int64_t rows_per_tile,
                              int64_t nsplit, const c10::optional<at::Tensor>& ws_o,
                              const c10::optional<at::Tensor>& ws_lse) {
  GSB_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                out.scalar_type() == at::kBFloat16,
            "attention_tc: bf16 tensors required");
  GSB_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 16 && k_cache.is_contiguous() && v_cache.is_contiguous(),
            "attention_tc: caches must be contiguous [num_blocks, Hkv, 16, D]");
  const int Hkv = (int)k_cache.size(1), D = (int)k_cache.size(3), Hq = (int)num_q_heads;
  GSB_CHECK(D == 128 || D == 64, "attention_tc: head_dim must be 64 or 128, got ", D);
  GSB_CHECK(Hq % Hkv == 0, "attention_tc: Hq must be a multiple of Hkv");
  GSB_CHECK(q.stride(1) == 1 && (q.stride(0) % 8) == 0 && out.stride(1) == 1 && (out.stride(0) % 8) == 0,
            "attention_tc: q/out rows must be 16-byte aligned");
  const int n_work = (int)work_seq.numel();
  if (n_work == 0) return;
  const int64_t page_rows = k_cache.size(0) * (int64_t)Hkv * 16;
  GSB_CHECK(page_rows < (int64_t(1) << 31), "attention_tc: cache too large for 32-bit TMA coordinates");
  c10::cuda::CUDAGuard guard(q.device());
  auto st = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  CUtensorMap tk = make_tmap_bf16_2d(k_cache.data_ptr(), page_rows, D, D, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = make_tmap_bf16_2d(v_cache.data_ptr(), page_rows, D, D, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  GSB_CHECK(n_work < 65536, "attention_tc: too many work tiles");
  GSB_CHECK(rows_per_tile == 128 || rows_per_tile == 256, "attention_tc: rows_per_tile must be 128 or 256");
  GSB_CHECK(nsplit >= 1 && nsplit <= 64 && (nsplit == 1 || rows_per_tile == 128),
            "attention_tc: nsplit must be in [1, 64], and 1 with 256-row tiles");
  const int T = (int)q.size(0);
  float* wso = nullptr;
  float* wsl = nullptr;
  if (nsplit > 1) {
    GSB_CHECK(ws_o.has_value() && ws_lse.has_value() && ws_o->scalar_type() == at::kFloat &&
                  ws_lse->scalar_type() == at::kFloat && ws_o->is_contiguous() && ws_lse->is_contiguous(),
              "attention_tc: contiguous fp32 workspaces required for nsplit > 1");
    GSB_CHECK(ws_o->numel() >= nsplit * (int64_t)T * Hq * D && ws_lse->numel() >= nsplit * (int64_t)T * Hq,
              "attention_tc: workspaces too small");
    wso = ws_o->data_ptr<float>();
    wsl = ws_lse->data_ptr<float>();
  }
  dim3 grid(Hkv, n_work);
  const bool packed = g_attn_packed != 0;
  if (rows_per_tile == 256) {
    auto kp = (D == 128) ? (packed ? fa_pingpong_kernel<128, true> : fa_pingpong_kernel<128, false>)
                         : (packed ? fa_pingpong_kernel<64, true> : fa_pingpong_kernel<64, false>);
    const int smem_p = (D == 128) ? FaPPCfg<128>::SMEM : FaPPCfg<64>::SMEM;
    static bool configured_p[4] = {false, false, false, false};
    const int vp = (D == 128) * 2 + packed;
    if (!configured_p[vp]) {
      GSB_CUDA_CHECK(cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_p));
      configured_p[vp] = true;
    }
    kp<<<(::gsb::count_launch(), grid), 320, smem_p, st>>>(tk, tv, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0),
                                  block_table.data_ptr<int32_t>(), (int)block_table.stride(0), (int)k_cache.size(0),
                                  q_start.data_ptr<int32_t>(), kv_len.data_ptr<int32_t>(),
                                  work_seq.data_ptr<int32_t>(), work_row0.data_ptr<int32_t>(), Hq, Hkv,
                                  (float)(scale * 1.4426950408889634),
                                  reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
                                  reinterpret_cast<uint32_t*>(err.data_ptr()));
    GSB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  auto kfn = (D == 128) ? (packed ? fa_prefill_kernel<128, 64, true> : fa_prefill_kernel<128, 64, false>)
                        : (packed ? fa_prefill_kernel<64, 64, true> : fa_prefill_kernel<64, 64, false>);
  const int smem = (D == 128) ? FaCfg<128, 64>::SMEM : FaCfg<64, 64>::SMEM;
  static bool configured[4] = {false, false, false, false};
  const int variant = (D == 128) * 2 + packed;
  if (!configured[variant]) {
    GSB_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[variant] = true;
  }
  kfn<<<(::gsb::count_launch(), dim3(Hkv, n_work, (unsigned)nsplit)), 192, smem, st>>>(
      tk, tv, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), block_table.data_ptr<int32_t>(),
      (int)block_table.stride(0), (int)k_cache.size(0), q_start.data_ptr<int32_t>(), kv_len.data_ptr<int32_t>(),
      work_seq.data_ptr<int32_t>(), work_row0.data_ptr<int32_t>(), Hq, Hkv, (float)(scale * 1.4426950408889634),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), wso, wsl, (int)nsplit, T,
      reinterpret_cast<uint32_t*>(err.data_ptr()));
  GSB_CUDA_CHECK(cudaGetLastError());
  if (nsplit > 1) {
    launch_attn_merge(D, n_work, Hkv, st, wso, wsl, (int)nsplit, T, Hq, q_start.data_ptr<int32_t>(),
                      work_seq.data_ptr<int32_t>(), work_row0.data_ptr<int32_t>(), 128, out.data_ptr(), out.stride(0));
    GSB_CUDA_CHECK(cudaGetLastError());
  }
}
