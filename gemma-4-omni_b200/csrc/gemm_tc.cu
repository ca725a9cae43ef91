// Weight x activation GEMM on 5th-generation tensor cores (tcgen05 / UMMA).
//
//   D[t, o] = sum_k X[t, k] * W[o, k]      (X: [tokens, K] bf16, W: [O, K])
//
// This is every dense contraction of the listener step (Conformer FFN, Q/K/V,
// attention post, light-conv start/end, subsampler input projection, output
// projection, embedder and FiLM linears).  It replaces the per-Linear Triton
// kernel of the reference (duplex_kernel/streaming_conformer_kernels.py:27-73,
// launcher :110-168) and the torch Linears of transformers' Gemma4 audio
// modules (models/gemma4/modeling_gemma4.py:128-154).
//
// Design (swap-AB): the UMMA M dimension (128) runs over output features, the
// UMMA N dimension over tokens (TN = 32..256), so a step with 2 tokens streams
// weights through the tensor core exactly like a step with 2048 tokens, only
// with a narrower N.  Operands are staged by TMA (128-byte swizzle, no
// multicast) into a STAGES-deep shared-memory ring; one thread issues
// tcgen05.mma into a TMEM accumulator of 128 lanes x TN fp32 columns; four
// epilogue warps drain TMEM with tcgen05.ld and apply the per-channel int8
// scale, bias, activation and output rounding.
//
// Weight-only int8: W arrives as int8 rows with one fp16 scale per output
// channel.  Four converter warps widen each staged int8 tile to bf16 (exact:
// every int8 value is a bf16 value) directly into the 128-byte-swizzled layout
// UMMA reads; the scale is applied per accumulator lane in the epilogue, which
// equals x . (q * s) up to fp32 summation order.
//
// Split-K: grid.z splits the K loop; splits accumulate with fp32 reductions
// into a zeroed fp32 buffer (out_mode 2) that a finalize pass consumes.
#include "common.cuh"
#include "kernels.h"

#include <cudaTypedefs.h>
#include <cstdio>
#include <mutex>

namespace lb {

namespace {

constexpr int kBlockO = 128;
constexpr int kBlockK = 64;
constexpr uint32_t kABytes = kBlockO * kBlockK * 2;  // bf16 A tile, 16 KB
constexpr uint32_t kRawBytes = kBlockO * kBlockK;    // int8 A tile, 8 KB

template <int TN, bool WINT8>
struct GemmCfg {
  static constexpr int kStages = WINT8 ? (TN >= 256 ? 3 : 4) : (TN >= 256 ? 4 : 6);
  static constexpr uint32_t kBBytes = TN * kBlockK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + (WINT8 ? kRawBytes : 0);
  static constexpr uint32_t kBarBytes = (4 * kStages + 2) * 8 + 16;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;
  static constexpr int kThreads = WINT8 ? 320 : 192;
  static constexpr uint32_t kTmemCols = TN;  // power of two >= 32
};

__device__ __forceinline__ void convert_i8x16_to_bf16(const int4 raw, int4& lo, int4& hi) {
  const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
  __nv_bfloat162 out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    out[i] = __floats2bfloat162_rn(static_cast<float>(b[2 * i]), static_cast<float>(b[2 * i + 1]));
  }
  lo = *reinterpret_cast<int4*>(&out[0]);
  hi = *reinterpret_cast<int4*>(&out[4]);
}

template <int TN, bool WINT8>
__global__ void __launch_bounds__(GemmCfg<TN, WINT8>::kThreads, 1)
    gemm_wx_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const GemmParams p) {
  using Cfg = GemmCfg<TN, WINT8>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));

  const int M = p.m_dev ? *p.m_dev : p.m_static;
  const int t0 = blockIdx.y * TN;
  if (t0 >= M) return;
  const int o0 = blockIdx.x * kBlockO;
  const int total_kb = p.K / kBlockK;
  const int kb_begin = blockIdx.z * p.kb_per_split;
  const int kb_end = min(kb_begin + p.kb_per_split, total_kb);
  if (kb_begin >= kb_end) return;
  const int nkb = kb_end - kb_begin;

  auto stage_a = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto stage_b = [&](int s) { return smem + s * Cfg::kStageBytes + kABytes; };
  auto stage_raw = [&](int s) { return smem + s * Cfg::kStageBytes + kABytes + Cfg::kBBytes; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* conv = bars + 2 * S;
  uint64_t* tmem_full = bars + 4 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (WINT8) mbar_init(&conv[s], 128);
    }
    mbar_init(tmem_full, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t tx = (WINT8 ? kRawBytes : kABytes) + p.b_tx_bytes;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&full[s], tx);
        const int k = (kb_begin + i) * kBlockK;
        tma_load_2d(WINT8 ? stage_raw(s) : stage_a(s), &tm_w, &full[s], k, o0, pol_w);
        tma_load_2d(stage_b(s), &tm_x, &full[s], k, t0, pol_x);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBlockO, TN);
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        ok = mbar_wait(&full[s], ph, p.status);
        if (ok && WINT8) ok = mbar_wait(&conv[s], ph, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint64_t a_desc = smem_desc_k128(smem_u32(stage_a(s)));
        const uint64_t b_desc = smem_desc_k128(smem_u32(stage_b(s)));
#pragma unroll
        for (int j = 0; j < kBlockK / 16; ++j) {
          // advance 16 bf16 = 32 bytes along K inside the swizzled row
          umma_bf16(tmem_base, a_desc + static_cast<uint64_t>(j * 2),
                    b_desc + static_cast<uint64_t>(j * 2), idesc, (i > 0 || j > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tmem_full);
    }
  } else if (warp < 6) {
    // ---------------- epilogue: TMEM -> registers -> global
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int o = o0 + q * 32 + lane;
    const bool ok = mbar_wait(tmem_full, 0, p.status);
    tc_fence_after();
    if (ok) {
      const float scale = WINT8 ? __half2float(p.w_scale[o]) : 1.0f;
      const float bias = (p.bias && blockIdx.z == 0) ? p.bias[o] : 0.0f;  // once across splits
#pragma unroll 1
      for (int c = 0; c < TN; c += 32) {
        float v[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c, v);
        if (t0 + c >= M) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = t0 + c + j;
          if (t < M) {
            float y = v[j] * scale + bias;
            const size_t idx = static_cast<size_t>(t) * p.ld_out + o;
            if (p.out_mode == 0) {
              y = fminf(fmaxf(y, p.out_lo), p.out_hi);
              if (p.act == 1) y = silu_f(bf16_round(y));
              y = fminf(fmaxf(y, p.post_lo), p.post_hi);
              reinterpret_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(y);
            } else if (p.out_mode == 1) {
              reinterpret_cast<float*>(p.out)[idx] = fminf(fmaxf(y, p.out_lo), p.out_hi);
            } else {
              atomicAdd(reinterpret_cast<float*>(p.out) + idx, y);
            }
          }
        }
      }
    }
  } else {
    // ---------------- int8 -> bf16 converters (WINT8 only; warps 6..9)
    if (WINT8) {
      const int ct = threadIdx.x - 192;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&full[s], ph, p.status)) break;
        const uint8_t* raw = stage_raw(s);
        uint8_t* dst = stage_a(s);
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int c = ct + 128 * qd;  // 16-byte chunk id in the 128 x 64 B raw tile
          const int row = c >> 2;
          const int ch = c & 3;
          const int4 r = *reinterpret_cast<const int4*>(raw + row * 64 + ch * 16);
          int4 lo, hi;
          convert_i8x16_to_bf16(r, lo, hi);
          const int sw = row & 7;
          *reinterpret_cast<int4*>(dst + row * 128 + (((2 * ch) ^ sw) << 4)) = lo;
          *reinterpret_cast<int4*>(dst + row * 128 + (((2 * ch + 1) ^ sw) << 4)) = hi;
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

template <int TN, bool WINT8>
cudaError_t launch_gemm_t(const CUtensorMap& tw, const CUtensorMap& tx, const GemmParams& p,
                          int m_cap, int splits, cudaStream_t stream) {
  using Cfg = GemmCfg<TN, WINT8>;
  dim3 grid(p.O / kBlockO, (m_cap + TN - 1) / TN, splits);
  gemm_wx_kernel<TN, WINT8><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tw, tx, p);
  return cudaGetLastError();
}

template <int TN, bool WINT8>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(gemm_wx_kernel<TN, WINT8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(GemmCfg<TN, WINT8>::kSmemBytes));
}

}  // namespace

// Raises the dynamic shared-memory limit of every GEMM instance on the current
// device.  Called once per device before any launch (and before graph capture).
cudaError_t gemm_init_attributes() {
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = set_smem_attr<32, false>();
  if (e == cudaSuccess) e = set_smem_attr<64, false>();
  if (e == cudaSuccess) e = set_smem_attr<128, false>();
  if (e == cudaSuccess) e = set_smem_attr<256, false>();
  if (e == cudaSuccess) e = set_smem_attr<32, true>();
  if (e == cudaSuccess) e = set_smem_attr<64, true>();
  if (e == cudaSuccess) e = set_smem_attr<128, true>();
  if (e == cudaSuccess) e = set_smem_attr<256, true>();
  return e;
}

int make_tensor_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, bool swizzle128) {
  auto enc = tensor_map_encoder();
  if (!enc) return -1;
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int gemm_token_tile(int m_cap) {
  if (m_cap <= 32) return 32;
  if (m_cap <= 64) return 64;
  if (m_cap <= 128) return 128;
  return 256;
}

int gemm_prepare(GemmPlan* plan, const void* w, bool w_int8, int O, int K, const void* x,
                 int x_ld, int m_cap) {
  if (O % kBlockO != 0 || K % kBlockK != 0 || x_ld % 8 != 0) return -3;
  plan->O = O;
  plan->K = K;
  plan->w_int8 = w_int8;
  plan->m_cap = m_cap;
  plan->tn = gemm_token_tile(m_cap);
  int rc;
  if (w_int8) {
    rc = make_tensor_map_2d(&plan->tm_w, w, 1, K, O, static_cast<uint64_t>(K), kBlockK, kBlockO,
                            false);
  } else {
    rc = make_tensor_map_2d(&plan->tm_w, w, 2, K, O, static_cast<uint64_t>(K) * 2, kBlockK,
                            kBlockO, true);
  }
  if (rc) return rc;
  // The activation map covers exactly m_cap rows (TMA zero-fills rows past it).
  // A box may not exceed the tensor extent, so with fewer rows than the token
  // tile the box shrinks to m_cap rows; the tile's remaining shared-memory rows
  // then hold stale data that only reaches output columns t >= m_cap, which the
  // epilogue never stores.
  plan->x_box_rows = m_cap < plan->tn ? m_cap : plan->tn;
  return make_tensor_map_2d(&plan->tm_x, x, 2, K, static_cast<uint64_t>(m_cap),
                            static_cast<uint64_t>(x_ld) * 2, kBlockK,
                            static_cast<uint32_t>(plan->x_box_rows), true);
}

cudaError_t gemm_launch(const GemmPlan& plan, GemmParams p, int splits, cudaStream_t stream) {
  p.O = plan.O;
  p.K = plan.K;
  p.b_tx_bytes = static_cast<uint32_t>(plan.x_box_rows) * kBlockK * 2;
  const int total_kb = plan.K / kBlockK;
  if (splits < 1) splits = 1;
  if (splits > total_kb) splits = total_kb;
  p.kb_per_split = (total_kb + splits - 1) / splits;
  splits = (total_kb + p.kb_per_split - 1) / p.kb_per_split;
  if (splits > 1 && p.out_mode != 2) return cudaErrorInvalidValue;
#define LB_GEMM_CASE(TNV)                                                              \
  case TNV:                                                                            \
    return plan.w_int8 ? launch_gemm_t<TNV, true>(plan.tm_w, plan.tm_x, p, plan.m_cap, \
                                                  splits, stream)                      \
                       : launch_gemm_t<TNV, false>(plan.tm_w, plan.tm_x, p, plan.m_cap, \
                                                   splits, stream);
  switch (plan.tn) {
    LB_GEMM_CASE(32)
    LB_GEMM_CASE(64)
    LB_GEMM_CASE(128)
    LB_GEMM_CASE(256)
    default:
      return cudaErrorInvalidValue;
  }
#undef LB_GEMM_CASE
}

int gemm_pick_splits(const GemmPlan& plan, int num_sms) {
  const int tiles = (plan.O / kBlockO) * ((plan.m_cap + plan.tn - 1) / plan.tn);
  const int total_kb = plan.K / kBlockK;
  if (tiles >= num_sms) return 1;
  int splits = (num_sms + tiles - 1) / tiles;
  // keep at least 4 k-blocks per split so the pipeline fills
  const int max_splits = total_kb / 4 > 0 ? total_kb / 4 : 1;
  if (splits > max_splits) splits = max_splits;
  return splits < 1 ? 1 : splits;
}

}  // namespace lb
