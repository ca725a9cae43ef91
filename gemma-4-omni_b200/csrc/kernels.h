// Internal (host-side) interface between the C-ABI layer and the kernels.
// Nothing here is exported; the public surface is include/listener_b200.h.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

namespace lb {

// ------------------------------------------------------------------ GEMM
struct GemmParams {
  int K = 0;                   // reduction length (multiple of 64)
  int O = 0;                   // output features (multiple of 128)
  const int* m_dev = nullptr;  // device token count; null -> m_static
  int m_static = 0;
  int kb_per_split = 0;
  const __half* w_scale = nullptr;  // per-output-channel scale (int8 weights)
  const float* bias = nullptr;      // per-output-channel bias (fp32) or null
  void* out = nullptr;
  int ld_out = 0;    // elements between consecutive token rows of `out`
  int out_mode = 0;  // 0: bf16 store, 1: fp32 store, 2: fp32 atomic add (split-K)
  int act = 0;       // 0: none, 1: SiLU of the bf16-rounded linear output
  float out_lo = -INFINITY, out_hi = INFINITY;    // linear output clamp (before act)
  float post_lo = -INFINITY, post_hi = INFINITY;  // next linear's input clamp (after act)
  int* status = nullptr;
  uint32_t b_tx_bytes = 0;  // bytes one activation-tile TMA load delivers (set by gemm_launch)
  int out_f16 = 0;          // out_mode 0 stores fp16 instead of bf16 (set by gemm_launch)
  // Stacked linears (the fused Q/K/V weight): output features [j*part_o,
  // (j+1)*part_o) belong to part j (< kMaxParts), which has its own output clamp
  // part_lo[j]/part_hi[j] (replacing out_lo/out_hi) and reads its activations
  // x_part_rows * j rows further down X (0: every part reads the same rows).
  // part_o = 0: one part.  part_o is a multiple of the 128-feature tile.
  static constexpr int kMaxParts = 3;
  int part_o = 0;
  int x_part_rows = 0;
  float part_lo[kMaxParts] = {-INFINITY, -INFINITY, -INFINITY};
  float part_hi[kMaxParts] = {INFINITY, INFINITY, INFINITY};
};

struct GemmPlan {
  CUtensorMap tm_w;
  CUtensorMap tm_x;
  int O = 0, K = 0, m_cap = 0, tn = 0;
  int x_box_rows = 0;    // rows per activation TMA box: min(tn, m_cap)
  int out_mode = 0;
  bool out_f16 = false;
  int w_kind = 0;  // 0 bf16 weights, 1 int8 codes (widened in-kernel), 2 fp16 codes of int8
};

int make_tensor_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, bool swizzle128, bool f16 = false);
// Token tile (UMMA N) for an [m_cap x O] output: 32/64/128/256 up to 256
// tokens, beyond that the multiple of 16 in [128, 256] that fills whole waves.
int gemm_token_tile(int O, int m_cap, int num_sms);
// Encodes the tensor maps for W ([O,K]: bf16, int8 codes or fp16 codes of int8,
// per w_kind) and X ([m_cap,K], row stride x_ld elements; bf16, or fp16 with
// either int8 kind; TMA zero-fills rows past m_cap).  The output [m_cap, ld_out]
// is out_mode 0 bf16 (fp16 with out_f16), else fp32; rows past the live token
// count are never written.  x_parts > 1 stacks that many activation blocks,
// x_part_rows rows apart, in one X map (GemmParams::x_part_rows).
int gemm_prepare(GemmPlan* plan, const void* w, int w_kind, int O, int K, const void* x, int x_ld,
                 int m_cap, void* out, int ld_out, int out_mode, bool out_f16 = false,
                 int x_parts = 1, int x_part_rows = 0);
// dst[i] = fp16(src[i]) for n int8 codes (n % 16 == 0, 16-byte aligned).
cudaError_t widen_int8_codes(const void* src, void* dst, size_t n, cudaStream_t stream);
// dst[i] = fp16(src[i]) for n bf16 values (n % 8 == 0, 16-byte aligned), saturating.
cudaError_t widen_bf16_to_f16(const void* src, void* dst, size_t n, cudaStream_t stream);
// Clamps of the split-K finish pass: output clamp per stacked part (part_o
// features each; part_o = 0: one part, lo[0]/hi[0]) and the next input clamp.
struct FinalizeClip {
  int part_o = 0;
  float lo[3] = {-INFINITY, -INFINITY, -INFINITY}, hi[3] = {INFINITY, INFINITY, INFINITY};
  float plo = -INFINITY, phi = INFINITY;
};
// Finishes a split-K GEMM whose K slices were reduce-added into acc (fp32
// [rows][width], out_mode 2): rows below *m_dev (or m_static when m_dev is
// null) get the output clamp, SiLU (act 1, of the bf16-rounded sum) and the
// next-input clamp and are stored to out ([rows][ld_out]; out_f32: fp32, else
// bf16, or fp16 with f16); the accumulator is zeroed behind the read, so it is
// ready for the next split-K GEMM without a memset.
cudaError_t launch_split_finish(const int* m_dev, int m_static, int m_cap, float* acc, int width, int act,
                                void* out, int ld_out, bool out_f32, bool f16, const FinalizeClip& fc,
                                bool pdl, cudaStream_t s);
// pdl: launch with programmatic stream serialisation (common.cuh pdl_wait).
cudaError_t gemm_launch(const GemmPlan& plan, GemmParams p, int splits, cudaStream_t stream, bool pdl = false);
// K-split count that fills the SMs for an [m_cap x O] output with K reduction.
int gemm_pick_splits(int O, int K, int m_cap, int num_sms);

}  // namespace lb
