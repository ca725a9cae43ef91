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
// with a narrower N.
//
// Persistent, warp-specialised: one CTA per SM walks a list of work units
// (output tile, token tile, K split), output tiles fastest so concurrently
// running CTAs share the activation tile in L2.
//   warp 0      TMA producer: W and X tiles into a STAGES-deep smem ring
//               (128-byte swizzle; no multicast anywhere)
//   warp 1      UMMA issuer: tcgen05.mma into one of two TMEM accumulators
//               (2 x TN fp32 columns), so the epilogue of one unit overlaps the
//               main loop of the next
//   warps 2..9  epilogue, two groups of four warps draining alternate tiles:
//               tcgen05.ld (double-buffered 32-column loads) -> per-channel
//               int8 scale, bias, clamps, SiLU -> direct coalesced global
//               stores (one token's 32 features per warp instruction) or
//               fp32 reductions for split-K partial sums
//   warps 10..17 int8 only: widen each staged int8 weight tile to fp16 directly
//               in the 128-byte-swizzled layout UMMA reads (exact: every int8
//               is an fp16); the scale is applied per accumulator lane.
// Every wait is bounded (common.cuh); on a timeout the kernel records
// kStatusWaitTimeout and takes its teardown path (TMEM freed).
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

// Weight kinds: bf16 weights (bf16 x bf16 MMA); int8 codes widened to fp16
// in shared memory by converter warps; fp16 weights (int8 codes or bf16 weights
// widened once in HBM), read by TMA like bf16.  The fp16 kinds run fp16 x fp16
// MMAs with fp16 activations and apply the per-channel scale, when there is
// one (int8 codes), in the epilogue.
constexpr int kWBf16 = 0, kWInt8 = 1, kWF16 = 2;

template <int TN, int WK>
struct GemmCfg {
  // TMEM columns (tokens) per epilogue load: the int8 kernel runs 18 warps,
  // which caps it at 96 registers per thread, so it drains 16 columns at a time
  static constexpr int kCols = WK == kWInt8 ? 16 : 32;
  static constexpr uint32_t kBBytes = TN * kBlockK * 2;
  // int8 codes land in their own buffer beside the fp16 tile they widen into
  static constexpr uint32_t kRawStage = WK == kWInt8 ? kRawBytes : 0;
  static constexpr uint32_t kStageBytes = kABytes + kRawStage + kBBytes;
  // operand ring within 224 KB (the 227 KB opt-in limit leaves room for the
  // barriers and the 1 KB alignment slack)
  static constexpr int kStages = (224 * 1024) / kStageBytes > 8 ? 8 : (224 * 1024) / kStageBytes;
  static constexpr uint32_t kBarBytes = (4 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;
  static constexpr int kThreads = WK == kWInt8 ? 576 : 320;
  // double-buffered accumulator: two power-of-two column blocks of >= TN
  static constexpr uint32_t kTmemCols = TN <= 32 ? 64 : TN <= 64 ? 128 : TN <= 128 ? 256 : 512;
  static constexpr int kBufCols = kTmemCols / 2;  // column offset of accumulator 1
  // the two epilogue groups split a tile's columns at kHalf (a kCols multiple)
  static constexpr int kHalf = ((TN / 2 + kCols - 1) / kCols) * kCols;
};

// Widens 16 int8 to 16 fp16 with two byte permutes and two packed fp16
// subtractions per four values: flipping the sign bit maps v to u = v + 128 in
// [0, 255]; the fp16 bit pattern 0x6400 | u is exactly 1024 + u, so
// subtracting 1152 recovers v exactly (every |v| <= 128 is exact in fp16).
__device__ __forceinline__ void convert_i8x16_to_f16(const int4 raw, int4& lo, int4& hi) {
  const uint32_t w[4] = {static_cast<uint32_t>(raw.x) ^ 0x80808080u, static_cast<uint32_t>(raw.y) ^ 0x80808080u,
                         static_cast<uint32_t>(raw.z) ^ 0x80808080u, static_cast<uint32_t>(raw.w) ^ 0x80808080u};
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t p0 = __byte_perm(w[i], 0x64646464u, 0x5140);  // {0x64|u0, 0x64|u1}
    uint32_t p1 = __byte_perm(w[i], 0x64646464u, 0x5342);  // {0x64|u2, 0x64|u3}
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&p0), bias);
    __half2 h1 = __hsub2(*reinterpret_cast<__half2*>(&p1), bias);
    out[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
    out[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
  }
  lo = make_int4(static_cast<int>(out[0]), static_cast<int>(out[1]), static_cast<int>(out[2]), static_cast<int>(out[3]));
  hi = make_int4(static_cast<int>(out[4]), static_cast<int>(out[5]), static_cast<int>(out[6]), static_cast<int>(out[7]));
}

__device__ __forceinline__ void tma_load_2d_nohint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                   int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 32 lanes x NC consecutive fp32 columns per warp, issued without waiting:
// the registers are valid only after tmem_wait_ld on the same array.
__device__ __forceinline__ void tmem_ld_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Waits for this thread's TMEM loads; the array is threaded through the asm so
// no use of the loaded values can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// SiLU(x) = x * sigmoid(x) = h + h * tanh(h) with h = x / 2: one hardware
// tanh (tanh.approx.f32, ~2^-11 relative error) and two FMAs.  The result is
// rounded to bf16 (2^-8) right after.
__device__ __forceinline__ float silu_tanh(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

struct Unit {
  int o0, t0, kb_begin, nkb, split;
};

__device__ __forceinline__ Unit unit_of(int u, int o_tiles, int t_tiles, int TN, int kb_per_split,
                                        int total_kb) {
  Unit r;
  const int per_split = o_tiles * t_tiles;
  r.split = u / per_split;
  const int rem = u - r.split * per_split;
  const int tt = rem / o_tiles;
  r.o0 = (rem - tt * o_tiles) * kBlockO;
  r.t0 = tt * TN;
  r.kb_begin = r.split * kb_per_split;
  const int kb_end = min(r.kb_begin + kb_per_split, total_kb);
  r.nkb = kb_end - r.kb_begin;
  return r;
}

// Epilogue math of NC accumulator columns (tokens) of one output feature:
// int8 scale, bias, output clamp, optional SiLU of the bf16-rounded linear
// output, next-input clamp.  Branch-free over the columns so the NC
// independent chains interleave.
// CLAMP = false when all four bounds are infinite (the clamps are the identity
// then), which halves the instructions per value of a fp32 or bf16 store.
template <bool SILU, bool CLAMP, int NC>
__device__ __forceinline__ void epilogue_math(const uint32_t (&r)[NC], float (&y)[NC], float scale,
                                              float bias, float lo, float hi, float plo, float phi) {
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    float v = fmaf(__uint_as_float(r[j]), scale, bias);
    if (CLAMP) v = fminf(fmaxf(v, lo), hi);
    if (SILU) v = silu_tanh(bf16_round(v));
    y[j] = CLAMP ? fminf(fmaxf(v, plo), phi) : v;
  }
}

template <int TN, int WK>
__global__ void __launch_bounds__(GemmCfg<TN, WK>::kThreads, 1)
    gemm_wx_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const GemmParams p) {
  using Cfg = GemmCfg<TN, WK>;
  constexpr bool WINT8 = WK == kWInt8;   // converter warps widen int8 in shared memory
  constexpr bool SCALED = WK != kWBf16;  // fp16 operands, per-channel scale
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));

  const int M = p.m_dev ? *p.m_dev : p.m_static;
  const int o_tiles = p.O / kBlockO;
  const int t_tiles = (M + TN - 1) / TN;
  const int total_kb = p.K / kBlockK;
  const int splits = (total_kb + p.kb_per_split - 1) / p.kb_per_split;
  const int units = o_tiles * t_tiles * splits;

  auto stage_a = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto stage_b = [&](int s) { return smem + s * Cfg::kStageBytes + kABytes + Cfg::kRawStage; };
  // int8 weights land in the raw buffer after their stage's fp16 A tile
  auto stage_raw = [&](int s) { return smem + s * Cfg::kStageBytes + kABytes; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* full = bars;                    // bf16: W and X tiles; int8: X tile
  uint64_t* empty = bars + S;
  uint64_t* conv = bars + 2 * S;            // int8: W tile widened to fp16
  uint64_t* full_w = bars + 3 * S;          // int8: raw W tile landed
  uint64_t* tmem_full = bars + 4 * S;       // [2]
  uint64_t* tmem_empty = bars + 4 * S + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (WINT8) {
        mbar_init(&conv[s], 8);
        mbar_init(&full_w[s], 1);
      }
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);  // all eight epilogue warps
    }
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
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_x = l2_policy_evict_last();
      // With one token tile every weight tile is read exactly once: stream it
      // evict-first so it does not push the step's activations and caches out
      // of L2.  With several token tiles the later waves re-read the weights
      // from L2, so they keep the default policy.
      const bool w_once = t_tiles == 1;
      const uint64_t pol_w = l2_policy_evict_first();
      auto load_w = [&](void* dst, uint64_t* bar, int k, int o0) {
        if (w_once) {
          tma_load_2d(dst, &tm_w, bar, k, o0, pol_w);
        } else {
          tma_load_2d_nohint(dst, &tm_w, bar, k, o0);
        }
      };
      // int8: the raw weight tile completes on its own barrier, so widening
      // never waits for the activation tile
      const uint32_t tx = WINT8 ? p.b_tx_bytes : kABytes + p.b_tx_bytes;
      // The weights never depend on the previous kernel in the stream, so the
      // first ring's worth of weight tiles (the ring starts empty) is requested
      // before pdl_wait(); the activation tiles, which that kernel produces,
      // follow it.  In the weight-streaming regime (a few tokens) this overlaps
      // most of a GEMM's HBM traffic with the kernel before it.
      int pre = 0;
      for (int u = blockIdx.x; u < units && pre < S; u += gridDim.x) {
        const Unit w = unit_of(u, o_tiles, t_tiles, TN, p.kb_per_split, total_kb);
        for (int i = 0; i < w.nkb && pre < S; ++i, ++pre) {
          const int k = (w.kb_begin + i) * kBlockK;
          if (WINT8) {
            mbar_arrive_expect_tx(&full_w[pre], kRawBytes);
            load_w(stage_raw(pre), &full_w[pre], k, w.o0);
          } else {
            mbar_arrive_expect_tx(&full[pre], tx);  // W now, X after the wait
            load_w(stage_a(pre), &full[pre], k, w.o0);
          }
        }
      }
      pdl_wait();
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, o_tiles, t_tiles, TN, p.kb_per_split, total_kb);
        // stacked parts (Q/K/V) may read their own activation block
        const int x_row = w.t0 + (p.x_part_rows ? (w.o0 / p.part_o) * p.x_part_rows : 0);
        for (int i = 0; i < w.nkb; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          const int k = (w.kb_begin + i) * kBlockK;
          if (it >= pre) {
            if (!mbar_wait(&empty[s], ph ^ 1, p.status)) {
              ok = false;
              break;
            }
            if (WINT8) {
              mbar_arrive_expect_tx(&full_w[s], kRawBytes);
              load_w(stage_raw(s), &full_w[s], k, w.o0);
            }
            mbar_arrive_expect_tx(&full[s], tx);
            if (!WINT8) load_w(stage_a(s), &full[s], k, w.o0);
          } else if (WINT8) {
            mbar_arrive_expect_tx(&full[s], tx);  // the raw W tile is already on its way
          }
          tma_load_2d(stage_b(s), &tm_x, &full[s], k, x_row, pol_x);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer
    if (lane == 0) {
      // int8 weights run with fp16 operands (widened codes, fp16 activations)
      constexpr uint32_t idesc = SCALED ? umma_idesc_f16(kBlockO, TN) : umma_idesc_bf16(kBlockO, TN);
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
        const Unit w = unit_of(u, o_tiles, t_tiles, TN, p.kb_per_split, total_kb);
        const int b = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&tmem_empty[b], aph ^ 1, p.status)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(b * Cfg::kBufCols);
        for (int i = 0; i < w.nkb; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = mbar_wait(&full[s], ph, p.status);
          if (ok && WINT8) ok = mbar_wait(&conv[s], ph, p.status);
          if (!ok) break;
          tc_fence_after();
          const uint64_t a_desc = smem_desc_k128(smem_u32(stage_a(s)));
          const uint64_t b_desc = smem_desc_k128(smem_u32(stage_b(s)));
#pragma unroll
          for (int j = 0; j < kBlockK / 16; ++j) {
            // advance 16 elements = 32 bytes along K inside the swizzled row
            umma_bf16(acc, a_desc + static_cast<uint64_t>(j * 2), b_desc + static_cast<uint64_t>(j * 2),
                      idesc, (i > 0 || j > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tmem_full[b]);
      }
    }
  } else if (warp < 10) {
    // ---------------- epilogue: TMEM -> registers -> global memory.
    // All eight warps drain every tile: group g (four warps, one per TMEM lane
    // quarter) takes columns [g*kHalf, (g+1)*kHalf).  The other accumulator
    // buffer keeps the MMA warp busy meanwhile.
    // Lane = output feature, TMEM column = token: every store instruction
    // writes one token's 32 consecutive features (64 B bf16/fp16, 128 B fp32).
    // TMEM loads (kCols columns) are double-buffered in registers, so the next
    // load is in flight while the current columns are scaled and stored.
    const int g = (warp - 2) >> 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool f16 = p.out_f16 != 0;
    const bool silu = p.out_mode == 0 && p.act == 1;
    // clamps of the linear output (bf16 / fp32 stores) and of the next input
    // (split-K partial sums are clamped by the finalize pass instead)
    const bool clip_out = p.out_mode != 2;
    const bool parts = clip_out && p.part_o > 0;
    const float lo0 = clip_out ? p.out_lo : -INFINITY, hi0 = clip_out ? p.out_hi : INFINITY;
    const float plo = p.out_mode == 0 ? p.post_lo : -INFINITY, phi = p.out_mode == 0 ? p.post_hi : INFINITY;
    bool clamps = isfinite(lo0) || isfinite(hi0) || isfinite(plo) || isfinite(phi);
    if (parts)
#pragma unroll
      for (int j = 0; j < GemmParams::kMaxParts; ++j) clamps = clamps || isfinite(p.part_lo[j]) || isfinite(p.part_hi[j]);
    int local = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
      const Unit w = unit_of(u, o_tiles, t_tiles, TN, p.kb_per_split, total_kb);
      float lo = lo0, hi = hi0;
      if (parts) {  // selects, not a dynamic index into the parameter block
        const int j = w.o0 / p.part_o;
        lo = j == 0 ? p.part_lo[0] : j == 1 ? p.part_lo[1] : p.part_lo[2];
        hi = j == 0 ? p.part_hi[0] : j == 1 ? p.part_hi[1] : p.part_hi[2];
      }
      const int o = w.o0 + q * 32 + lane;
      const float scale = SCALED && p.w_scale ? __half2float(p.w_scale[o]) : 1.0f;
      const float bias = (p.bias && w.split == 0) ? p.bias[o] : 0.0f;
      const int b = local & 1;
      if (!mbar_wait(&tmem_full[b], (local >> 1) & 1, p.status)) break;
      tc_fence_after();
      const int nvalid = min(TN, M - w.t0);  // tokens of this tile below the live count
      const int c_begin = g * Cfg::kHalf;
      const int c_end = min(c_begin + Cfg::kHalf, nvalid);
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * Cfg::kBufCols);
      const size_t ld = static_cast<size_t>(p.ld_out);
      constexpr int NC = Cfg::kCols;
      auto drain = [&](const uint32_t (&r)[NC], int c, float sc, float bi) {
        float y[NC];
        if (clamps) {
          if (silu) {
            epilogue_math<true, true, NC>(r, y, sc, bi, lo, hi, plo, phi);
          } else {
            epilogue_math<false, true, NC>(r, y, sc, bi, lo, hi, plo, phi);
          }
        } else if (silu) {
          epilogue_math<true, false, NC>(r, y, sc, bi, lo, hi, plo, phi);
        } else {
          epilogue_math<false, false, NC>(r, y, sc, bi, lo, hi, plo, phi);
        }
        const size_t base = static_cast<size_t>(w.t0 + c) * ld + o;
        const int n = c_end - c;  // >= 1
        if (p.out_mode == 0) {
          uint16_t* dst = static_cast<uint16_t*>(p.out) + base;
          if (n >= NC) {
#pragma unroll
            for (int j = 0; j < NC; ++j) dst[j * ld] = act_bits(y[j], f16);
          } else {
#pragma unroll
            for (int j = 0; j < NC; ++j)
              if (j < n) dst[j * ld] = act_bits(y[j], f16);
          }
        } else if (p.out_mode == 1) {
          float* dst = static_cast<float*>(p.out) + base;
#pragma unroll
          for (int j = 0; j < NC; ++j)
            if (j < n) dst[j * ld] = y[j];
        } else {
          float* dst = static_cast<float*>(p.out) + base;
#pragma unroll
          for (int j = 0; j < NC; ++j)
            if (j < n) atomicAdd(dst + j * ld, y[j]);  // split-K partial sum
        }
      };
      if (c_begin < c_end) {
        uint32_t ra[NC], rb[NC];
        tmem_ld_async(tbase + static_cast<uint32_t>(c_begin), ra);
        tmem_wait_ld(ra);
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 2 * NC) {
          const bool more_b = c + NC < c_end;
          if (more_b) tmem_ld_async(tbase + static_cast<uint32_t>(c + NC), rb);
          drain(ra, c, scale, bias);
          if (more_b) {
            tmem_wait_ld(rb);
            const bool more_a = c + 2 * NC < c_end;
            if (more_a) tmem_ld_async(tbase + static_cast<uint32_t>(c + 2 * NC), ra);
            drain(rb, c + NC, scale, bias);
            if (more_a) tmem_wait_ld(ra);
          }
        }
      }
      // accumulator drained: hand the TMEM buffer back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
    }
  } else {
    // ---------------- int8 -> fp16 converters (WINT8 only; warps 10..17)
    // The raw int8 tile has its own buffer, so each converter warp widens its
    // rows (8 + 8 of the 128) as soon as the tile lands, with no meeting of the
    // warps: read 2 x 16 codes, widen, store 4 x 16 bytes into the swizzled
    // fp16 tile, one proxy fence, one arrival on conv[s] per warp.
    if (WINT8) {
      const int ct = threadIdx.x - 320;
      int n_it = 0;  // k-blocks this CTA streams, in ring order
      for (int u = blockIdx.x; u < units; u += gridDim.x)
        n_it += unit_of(u, o_tiles, t_tiles, TN, p.kb_per_split, total_kb).nkb;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % S;
        if (!mbar_wait(&full_w[s], (it / S) & 1, p.status)) break;
        const uint8_t* raw = stage_raw(s);
        uint8_t* dst = stage_a(s);
        int4 r[2];
#pragma unroll
        for (int qd = 0; qd < 2; ++qd) {
          const int cidx = ct + 256 * qd;  // 16-byte chunk id in the 128 x 64 B raw tile
          r[qd] = *reinterpret_cast<const int4*>(raw + (cidx >> 2) * 64 + (cidx & 3) * 16);
        }
#pragma unroll
        for (int qd = 0; qd < 2; ++qd) {
          const int cidx = ct + 256 * qd;
          const int row = cidx >> 2;
          const int ch = cidx & 3;
          int4 lo4, hi4;
          convert_i8x16_to_f16(r[qd], lo4, hi4);
          const int sw = row & 7;
          *reinterpret_cast<int4*>(dst + row * 128 + (((2 * ch) ^ sw) << 4)) = lo4;
          *reinterpret_cast<int4*>(dst + row * 128 + (((2 * ch + 1) ^ sw) << 4)) = hi4;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
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

template <int TN, int WK>
cudaError_t launch_gemm_t(const GemmPlan& plan, const GemmParams& p, int splits, int num_sms,
                          cudaStream_t stream, bool pdl) {
  using Cfg = GemmCfg<TN, WK>;
  const int units = (plan.O / kBlockO) * ((plan.m_cap + TN - 1) / TN) * splits;
  const int grid = units < num_sms ? units : num_sms;
  return launch_kernel(pdl, gemm_wx_kernel<TN, WK>, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, stream,
                       plan.tm_w, plan.tm_x, p);
}

template <int TN, int WK>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(gemm_wx_kernel<TN, WK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(GemmCfg<TN, WK>::kSmemBytes));
}

// Widens int8 codes to fp16 (exact), 16 per thread.
__global__ void widen_i8_kernel(const int4* __restrict__ src, int4* __restrict__ dst, size_t n16) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    int4 lo, hi;
    convert_i8x16_to_f16(src[i], lo, hi);
    dst[2 * i] = lo;
    dst[2 * i + 1] = hi;
  }
}

// bf16 -> fp16, 8 per thread (saturating: beyond +/-65504 becomes +/-65504).
__global__ void widen_bf16_kernel(const int4* __restrict__ src, int4* __restrict__ dst, size_t n8) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int4 v = src[i];
    const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y), static_cast<uint32_t>(v.z),
                           static_cast<uint32_t>(v.w)};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xffff0000u);
      o[j] = act_bits2(lo, hi, true);
    }
    dst[i] = make_int4(static_cast<int>(o[0]), static_cast<int>(o[1]), static_cast<int>(o[2]), static_cast<int>(o[3]));
  }
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

// Raises the dynamic shared-memory limit of every GEMM instance on the current
// device.  Called once per device before any launch (and before graph capture).
cudaError_t gemm_init_attributes() {
  cudaError_t e = cudaSuccess;
#define LB_GEMM_ATTR(TNV)                                      \
  if (e == cudaSuccess) e = set_smem_attr<TNV, kWBf16>();      \
  if (e == cudaSuccess) e = set_smem_attr<TNV, kWInt8>();      \
  if (e == cudaSuccess) e = set_smem_attr<TNV, kWF16>();
  LB_GEMM_ATTR(32)
  LB_GEMM_ATTR(64)
  LB_GEMM_ATTR(128)
  LB_GEMM_ATTR(144)
  LB_GEMM_ATTR(160)
  LB_GEMM_ATTR(176)
  LB_GEMM_ATTR(192)
  LB_GEMM_ATTR(208)
  LB_GEMM_ATTR(224)
  LB_GEMM_ATTR(240)
  LB_GEMM_ATTR(256)
#undef LB_GEMM_ATTR
  return e;
}

int make_tensor_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, bool swizzle128, bool f16) {
  auto enc = tensor_map_encoder();
  if (!enc) return -1;
  const CUtensorMapDataType dt = elem_bytes == 2   ? (f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16)
                                 : elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
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

int gemm_token_tile(int O, int m_cap, int num_sms) {
  if (m_cap <= 32) return 32;
  if (m_cap <= 64) return 64;
  if (m_cap <= 128) return 128;
  if (m_cap <= 256) return 256;
  // Several token tiles: pick the width (a multiple of 16 in [128, 256]) that
  // minimises waves x (TN + 32), i.e. whole waves of equal-length units with a
  // per-unit overhead, so e.g. 12 feature tiles x 2048 tokens run as
  // 12 x 12 units of 176 tokens (one full wave) instead of 12 x 8 of 256.
  static constexpr int kCand[] = {256, 240, 224, 208, 192, 176, 160, 144, 128};
  const int o_tiles = O / kBlockO;
  int best = 256;
  long best_cost = -1;
  for (int tn : kCand) {
    const long units = static_cast<long>(o_tiles) * ((m_cap + tn - 1) / tn);
    const long waves = (units + num_sms - 1) / num_sms;
    const long cost = waves * (tn + 32);
    if (best_cost < 0 || cost < best_cost) {
      best = tn;
      best_cost = cost;
    }
  }
  return best;
}

cudaError_t widen_int8_codes(const void* src, void* dst, size_t n, cudaStream_t stream) {
  if (n % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 16)
    return cudaErrorInvalidValue;
  const size_t n16 = n / 16;
  const int blocks = static_cast<int>(n16 / 256 + 1 < 4096 ? n16 / 256 + 1 : 4096);
  widen_i8_kernel<<<blocks, 256, 0, stream>>>(static_cast<const int4*>(src), static_cast<int4*>(dst), n16);
  return cudaGetLastError();
}

cudaError_t widen_bf16_to_f16(const void* src, void* dst, size_t n, cudaStream_t stream) {
  if (n % 8 != 0 || reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 16)
    return cudaErrorInvalidValue;
  const size_t n8 = n / 8;
  const int blocks = static_cast<int>(n8 / 256 + 1 < 4096 ? n8 / 256 + 1 : 4096);
  widen_bf16_kernel<<<blocks, 256, 0, stream>>>(static_cast<const int4*>(src), static_cast<int4*>(dst), n8);
  return cudaGetLastError();
}

int gemm_prepare(GemmPlan* plan, const void* w, int w_kind, int O, int K, const void* x, int x_ld,
                 int m_cap, void* out, int ld_out, int out_mode, bool out_f16, int x_parts,
                 int x_part_rows) {
  if (O % kBlockO != 0 || K % kBlockK != 0 || x_ld % 8 != 0 || ld_out % 8 != 0 || m_cap < 1 ||
      w_kind < kWBf16 || w_kind > kWF16 || x_parts < 1 || x_parts > GemmParams::kMaxParts ||
      (x_parts > 1 && x_part_rows < m_cap))
    return -3;
  const bool w_int8 = w_kind == kWInt8;
  plan->O = O;
  plan->K = K;
  plan->w_kind = w_kind;
  plan->m_cap = m_cap;
  plan->tn = gemm_token_tile(O, m_cap, sm_count());
  plan->out_mode = out_mode;
  plan->out_f16 = out_f16;
  int rc;
  if (w_int8) {
    rc = make_tensor_map_2d(&plan->tm_w, w, 1, K, O, static_cast<uint64_t>(K), kBlockK, kBlockO,
                            false);
  } else {
    rc = make_tensor_map_2d(&plan->tm_w, w, 2, K, O, static_cast<uint64_t>(K) * 2, kBlockK,
                            kBlockO, true, w_kind == kWF16);
  }
  if (rc) return rc;
  // The activation map covers exactly m_cap rows (TMA zero-fills rows past it).
  // A box may not exceed the tensor extent, so with fewer rows than the token
  // tile the box shrinks to m_cap rows; the tile's remaining shared-memory rows
  // then hold stale data that only reaches output columns t >= m_cap, which
  // the epilogue never stores (it stops at the live token count M <= m_cap).
  // Stacked parts: the map spans every part's block; the rows between a part's
  // m_cap and the next part's first row feed only columns t >= m_cap as well.
  plan->x_box_rows = m_cap < plan->tn ? m_cap : plan->tn;
  const uint64_t x_rows = static_cast<uint64_t>(x_parts - 1) * x_part_rows + m_cap;
  // activations are fp16 when the weights are int8 (either kind), bf16 otherwise
  rc = make_tensor_map_2d(&plan->tm_x, x, 2, K, x_rows,
                          static_cast<uint64_t>(x_ld) * 2, kBlockK,
                          static_cast<uint32_t>(plan->x_box_rows), true, w_kind != kWBf16);
  if (rc) return rc;
  // The output [m_cap rows][ld_out] is written with plain stores, clipped at
  // the live token count, so it needs no tensor map.
  (void)out;
  (void)ld_out;
  return 0;
}

cudaError_t gemm_launch(const GemmPlan& plan, GemmParams p, int splits, cudaStream_t stream, bool pdl) {
  p.O = plan.O;
  p.K = plan.K;
  p.b_tx_bytes = static_cast<uint32_t>(plan.x_box_rows) * kBlockK * 2;
  p.out_f16 = plan.out_f16 ? 1 : 0;
  if (p.out_mode != plan.out_mode) return cudaErrorInvalidValue;
  if (p.part_o < 0 || p.x_part_rows < 0 || (p.x_part_rows > 0 && p.part_o == 0) ||
      (p.part_o > 0 && (p.part_o % kBlockO != 0 || p.O % p.part_o != 0 ||
                        p.O / p.part_o > GemmParams::kMaxParts)))
    return cudaErrorInvalidValue;
  const int total_kb = plan.K / kBlockK;
  if (splits < 1) splits = 1;
  if (splits > total_kb) splits = total_kb;
  p.kb_per_split = (total_kb + splits - 1) / splits;
  splits = (total_kb + p.kb_per_split - 1) / p.kb_per_split;
  if (splits > 1 && p.out_mode != 2) return cudaErrorInvalidValue;
  const int sms = sm_count();
#define LB_GEMM_CASE(TNV)                                                                  \
  case TNV:                                                                                \
    return plan.w_kind == kWInt8  ? launch_gemm_t<TNV, kWInt8>(plan, p, splits, sms, stream, pdl) \
           : plan.w_kind == kWF16 ? launch_gemm_t<TNV, kWF16>(plan, p, splits, sms, stream, pdl)  \
                                  : launch_gemm_t<TNV, kWBf16>(plan, p, splits, sms, stream, pdl);
  switch (plan.tn) {
    LB_GEMM_CASE(32)
    LB_GEMM_CASE(64)
    LB_GEMM_CASE(128)
    LB_GEMM_CASE(144)
    LB_GEMM_CASE(160)
    LB_GEMM_CASE(176)
    LB_GEMM_CASE(192)
    LB_GEMM_CASE(208)
    LB_GEMM_CASE(224)
    LB_GEMM_CASE(240)
    LB_GEMM_CASE(256)
    default:
      return cudaErrorInvalidValue;
  }
#undef LB_GEMM_CASE
}

int gemm_pick_splits(int O, int K, int m_cap, int num_sms) {
  const int tn = gemm_token_tile(O, m_cap, num_sms);
  const int tiles = (O / kBlockO) * ((m_cap + tn - 1) / tn);
  const int total_kb = K / kBlockK;
  // Choose the split count that best fills whole waves of SMs: efficiency =
  // units / (waves * SMs).  Each extra split costs an fp32 partial-sum
  // reduction, so a split must gain at least 8% and keep >= 6 k-blocks; with
  // a few tokens (weight streaming, latency-bound) the reductions are tiny and
  // a shorter per-CTA weight stream is what counts, so >= 2 k-blocks there.
  const int min_kb = m_cap <= 128 ? 2 : 6;
  int best = 1;
  double best_eff = static_cast<double>(tiles) / (((tiles + num_sms - 1) / num_sms) * num_sms);
  for (int s = 2; s <= 16; ++s) {
    if (total_kb / s < min_kb) break;
    const int units = tiles * s;
    const double eff = static_cast<double>(units) / (((units + num_sms - 1) / num_sms) * num_sms);
    if (eff > best_eff + 0.08) {
      best = s;
      best_eff = eff;
    }
  }
  return best;
}

}  // namespace lb
