// Per-layer non-GEMM kernels of the streaming Conformer step.
//
// All of them are row-parallel over the packed tokens (token 2r+t = tick token
// t of batch row r), read the device row count and exit for rows beyond it, use
// 16/32-byte vector loads and warp-shuffle reductions, and keep the residual
// stream in fp32.
//
//   row_fused_kernel   FFN post-norm + 0.5-scaled residual, attention post-norm
//                      + residual, norm_out, and the RMSNorm that produces the
//                      next GEMM's bf16 input, in one pass
//                      (transformers modeling_gemma4.py:390-408, 513-537;
//                      streaming_conformer.py:777, 853-860)
//   lconv_kernel       GLU -> causal depthwise conv (k=5) over the conv-state
//                      ring -> clamp -> RMSNorm -> SiLU -> bf16; stages the 2 new
//                      GLU rows (streaming_conformer.py:830-852, modeling_gemma4.py:444-482)
//   outputs / film     output_proj + embed_audio tails and the FiLM elementwise
//                      stages (streaming_conformer.py:871-872,
//                      frame_residual_adapter.py:203-234)
#include "common.cuh"
#include "listener.h"

#include <cmath>

namespace lb {
namespace {

// Buckets of at most this many tokens run the per-token row kernels with one
// CTA of G warps per token (or session) instead of one warp: with few tokens
// the step is latency-bound and the shorter per-warp chain is what counts.
constexpr int kSmallBucketTokens = 128;

// Block-wide sum for blocks of up to 32 warps.
__device__ __forceinline__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  return t;
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
// Read-only (non-coherent) forms for data the kernel never writes: the
// compiler may then issue them ahead of the kernel's own stores.
__device__ __forceinline__ void load8_nc(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8_bf16_nc(const __nv_bfloat16* p, float (&v)[8]) {
  const int4 r = __ldg(reinterpret_cast<const int4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float (&v)[8]) {
  const int4 r = *reinterpret_cast<const int4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&v)[8]) {
  int4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<int4*>(p) = r;
}

// RMSNorm of 8-element thread slices over a block row: x * pow(mean(x^2)+eps, -0.5) * w
__device__ __forceinline__ void rms8(float (&v)[8], const float* w, int e0, int d, float eps,
                                     float* sh) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  ss = block_sum(ss, sh);
  const float r = rsqrtf(ss / static_cast<float>(d) + eps);
  if (w) {
    float wv[8];
    load8(w + e0, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * r * wv[i];
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * r;
  }
}

struct RowFusedDev {
  const int* counts;
  int d;
  float eps, clip;
  float* h;
  const float* y;
  const float* post_w;
  float alpha;
  int residual;
  const float* out_w;
  const float* pre_w;
  int pre_norm, pre_clamp;
  float in_lo, in_hi;
  __nv_bfloat16* xa;
  float* dbg;
  bool f16;  // xa holds fp16 (int8-weight GEMM input) instead of bf16
  // stacked Q/K/V inputs with their own clamps: blocks 1 and 2 of xa, at
  // xa_part_stride elements apart, clamped to part_lo/part_hi (0: none)
  int xa_parts;
  size_t xa_part_stride;
  float part_lo[2], part_hi[2];
  // y is a split-K GEMM's partial-sum buffer: finish it here (the linear's
  // output clamp y_lo / y_hi) and zero it behind the read
  int zero_y;
  float y_lo, y_hi;
};

// W = 1: one warp per token, four tokens per 128-thread CTA.  Lane owns G
// groups of 8 elements, e = (g*32 + lane)*8, so each load is a whole-warp
// coalesced 512-byte run and every RMS reduction is five shuffles (no block
// barriers).  All 2G 32-byte loads of h and y are in flight together; at ~128
// registers a thread, 16 warps fit per SM, i.e. a 2048-token step in one wave.
// W = G (small buckets): one token per CTA of G warps, warp w owning group w,
// so a token's dependent load -> reduce -> store chain is G times shorter; the
// three RMS reductions add a shared-memory sum over the warps.
template <int G, int W>
__global__ void __launch_bounds__(W == 1 ? 128 : 32 * W, W == 1 ? 4 : 1) row_fused_kernel(RowFusedDev a) {
  pdl_wait();  // first: nothing of the previous kernel is read or written before it
  pdl_trigger();
  static_assert(W == 1 || W == G, "one warp per token, or one warp per channel group");
  constexpr int GW = G / W;  // channel groups per warp
  __shared__ float red[3][W];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // the grid covers the bucket's tokens exactly: (warps per CTA) / W tokens per
  // CTA, warp w of a token owning channel groups [w*GW, (w+1)*GW)
  const int t = blockIdx.x * ((blockDim.x >> 5) / W) + warp / W;
  const int g0 = (warp % W) * GW;
  constexpr int d = G * 256;
  constexpr float inv_d = 1.0f / static_cast<float>(d);
  const int e_lane = g0 * 256 + lane * 8;  // element of group gg: e_lane + gg * 256
  const size_t base = static_cast<size_t>(t) * d + e_lane;
  const int n_tok = a.counts[1];
  // sum over the token's d elements (a CTA-uniform call when W > 1)
  auto row_sum = [&](float v, int k) {
    v = warp_sum(v);
    if (W == 1) return v;
    if (lane == 0) red[k][warp % W] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) r += red[k][i];
    return r;
  };
  float h[GW][8], y[GW][8];
#pragma unroll
  for (int g = 0; g < GW; ++g) {
    load8(a.h + base + g * 256, h[g]);
    if (a.y) load8(a.y + base + g * 256, y[g]);
  }
  if (t >= n_tok) return;  // CTA-uniform when W > 1 (launched with one token per CTA)
  if (a.zero_y) {
    const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int g = 0; g < GW; ++g) {
      store8(const_cast<float*>(a.y) + base + g * 256, z);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[g][i] = fminf(fmaxf(y[g][i], a.y_lo), a.y_hi);
    }
  }
  if (a.y) {
    if (a.post_w) {
      float ss = 0.f;
#pragma unroll
      for (int g = 0; g < GW; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          y[g][i] = fminf(fmaxf(y[g][i], -a.clip), a.clip);
          ss = fmaf(y[g][i], y[g][i], ss);
        }
      const float r = rsqrtf(row_sum(ss, 0) * inv_d + a.eps);
#pragma unroll
      for (int g = 0; g < GW; ++g) {
        float w8[8];
        load8_nc(a.post_w + e_lane + g * 256, w8);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[g][i] = y[g][i] * r * w8[i];
      }
    }
#pragma unroll
    for (int g = 0; g < GW; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) h[g][i] = a.residual ? fmaf(y[g][i], a.alpha, h[g][i]) : y[g][i] * a.alpha;
  }
  if (a.out_w) {
    float ss = 0.f;
#pragma unroll
    for (int g = 0; g < GW; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        h[g][i] = fminf(fmaxf(h[g][i], -a.clip), a.clip);
        ss = fmaf(h[g][i], h[g][i], ss);
      }
    const float r = rsqrtf(row_sum(ss, 1) * inv_d + a.eps);
#pragma unroll
    for (int g = 0; g < GW; ++g) {
      float w8[8];
      load8_nc(a.out_w + e_lane + g * 256, w8);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[g][i] = h[g][i] * r * w8[i];
    }
  }
#pragma unroll
  for (int g = 0; g < GW; ++g) {
    store8(a.h + base + g * 256, h[g]);
    if (a.dbg) store8(a.dbg + base + g * 256, h[g]);
  }
  if (a.xa) {
    float ss = 0.f;
#pragma unroll
    for (int g = 0; g < GW; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (a.pre_clamp) h[g][i] = fminf(fmaxf(h[g][i], -a.clip), a.clip);
        ss = fmaf(h[g][i], h[g][i], ss);
      }
    const float r = a.pre_norm ? rsqrtf(row_sum(ss, 2) * inv_d + a.eps) : 1.0f;
#pragma unroll
    for (int g = 0; g < GW; ++g) {
      float w8[8];
      if (a.pre_norm && a.pre_w) {
        load8_nc(a.pre_w + e_lane + g * 256, w8);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) w8[i] = 1.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) h[g][i] = h[g][i] * r * w8[i];
      if (a.xa_parts > 1) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = fminf(fmaxf(h[g][i], a.part_lo[j]), a.part_hi[j]);
          store8_act(a.xa + (j + 1) * a.xa_part_stride + base + g * 256, v, a.f16);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) h[g][i] = fminf(fmaxf(h[g][i], a.in_lo), a.in_hi);
      store8_act(a.xa + base + g * 256, h[g], a.f16);
    }
  }
}

// ---------------------------------------------------------------- lconv
struct LconvDev {
  const int* counts;
  const int* row_slot;
  const SlotMeta* row_meta;
  const __nv_bfloat16* gl;   // [tok][2d]
  __nv_bfloat16* ring;       // [S][L][8][d]
  const float* dw;           // [5][d] tap-major
  const float* norm_w;       // [d]
  __nv_bfloat16* xa;         // [tok][d]
  int layer, layers, d, slots, rows_cap;
  float eps, clip, in_lo, in_hi;
  bool f16;  // xa holds fp16 (int8-weight GEMM input) instead of bf16
};

// W warps per session (both tick tokens; W = G in small buckets, one session
// per CTA); warp w of a session owns channel
// groups [w*G/W, (w+1)*G/W), lane its 8 channels e = (g*32 + lane)*8 of each,
// so every load is a whole-warp coalesced 512-byte run.  The two RMS
// reductions are warp shuffles, then (W > 1) a sum over the session's warps in
// shared memory.  Splitting a session over two warps halves each warp's
// dependent load chain and doubles the warps per SM, with 1024 sessions still
// in one wave of 256-thread CTAs.
template <int G, int W>
__global__ void __launch_bounds__(256) lconv_kernel(LconvDev a) {
  pdl_wait();  // first: nothing of the previous kernel is read or written before it
  pdl_trigger();
  constexpr int GW = G / W;  // channel groups per warp
  static_assert(G % W == 0, "channel groups must split evenly over the session's warps");
  __shared__ float2 part[8];  // per warp: (sum sq token 0, sum sq token 1)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sess = warp / W, w = warp % W;
  const int row = blockIdx.x * ((blockDim.x >> 5) / W) + sess;
  const int n_rows = a.counts[0];
  const int rl = min(row, a.rows_cap - 1);  // the grid rounds the bucket up to whole CTAs
  const int slot = a.row_slot[rl];
  const SlotMeta m = a.row_meta[rl];
  const bool live = row < n_rows;
  const int d = G * 256;
  const size_t rb = ring_base(slot, a.layer, a.slots, kConvRing, d);
  const int first_real = 4 - min(m.fill, 4);  // ring rows written since the last reset
  float cv[2][GW][8];
  float ss0 = 0.f, ss1 = 0.f;
  if (live) {
#pragma unroll
    for (int gg = 0; gg < GW; ++gg) {
      const int e0 = ((w * GW + gg) * 32 + lane) * 8;
      float win[6][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j >= first_real) {  // canonical rows: read-only here (the step writes only staged rows)
          load8_bf16_nc(a.ring + rb + static_cast<size_t>((m.pos + j) & (kConvRing - 1)) * d + e0, win[j]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) win[j][i] = 0.f;
        }
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        float av[8], bv[8];
        const __nv_bfloat16* gp = a.gl + (static_cast<size_t>(row) * 2 + t) * 2 * d;
        load8_bf16_nc(gp + e0, av);
        load8_bf16_nc(gp + d + e0, bv);
#pragma unroll
        for (int i = 0; i < 8; ++i) win[4 + t][i] = bf16_round(__fdividef(av[i], 1.0f + __expf(-bv[i])));  // GLU
        store8_bf16(a.ring + rb + static_cast<size_t>((m.pos + 4 + t) & (kConvRing - 1)) * d + e0, win[4 + t]);
      }
      float w5t[5][8];  // tap-major weights: 2 vector loads per tap
#pragma unroll
      for (int k = 0; k < 5; ++k) load8_nc(a.dw + static_cast<size_t>(k) * d + e0, w5t[k]);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 5; ++k) acc = fmaf(w5t[k][i], win[t + k][i], acc);
          acc = fminf(fmaxf(acc, -a.clip), a.clip);
          cv[t][gg][i] = acc;
          if (t == 0) ss0 = fmaf(acc, acc, ss0);
          else ss1 = fmaf(acc, acc, ss1);
        }
    }
  }
  ss0 = warp_sum(ss0);
  ss1 = warp_sum(ss1);
  if (W > 1) {
    if (lane == 0) part[warp] = make_float2(ss0, ss1);
    __syncthreads();
    ss0 = ss1 = 0.f;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const float2 v = part[sess * W + k];
      ss0 += v.x;
      ss1 += v.y;
    }
  }
  if (!live) return;
  const float r0 = rsqrtf(ss0 / static_cast<float>(d) + a.eps);
  const float r1 = rsqrtf(ss1 / static_cast<float>(d) + a.eps);
#pragma unroll
  for (int gg = 0; gg < GW; ++gg) {
    const int e0 = ((w * GW + gg) * 32 + lane) * 8;
    float wv[8];
    load8_nc(a.norm_w + e0, wv);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = fminf(fmaxf(silu_f(cv[t][gg][i] * (t == 0 ? r0 : r1) * wv[i]), a.in_lo), a.in_hi);
      store8_act(a.xa + (static_cast<size_t>(row) * 2 + t) * d + e0, o, a.f16);
    }
  }
}

// --------------------------------------------------------- split-K finish
__global__ void split_finish_kernel(const int* m_dev, int m_static, float* acc, int width, int act, void* out,
                                    int ld_out, int out_f32, FinalizeClip fc, bool f16) {
  pdl_wait();  // the GEMM's partial sums are complete
  pdl_trigger();
  const int t = blockIdx.y;
  if (t >= (m_dev ? *m_dev : m_static)) return;
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (o >= width) return;
  // stacked parts: 8 consecutive features never straddle a part (part_o % 128 == 0)
  const int j = fc.part_o ? o / fc.part_o : 0;
  const float lo = j == 0 ? fc.lo[0] : j == 1 ? fc.lo[1] : fc.lo[2];
  const float hi = j == 0 ? fc.hi[0] : j == 1 ? fc.hi[1] : fc.hi[2];
  float* a = acc + static_cast<size_t>(t) * width + o;
  float v[8];
  load8(a, v);
  const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  store8(a, z);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float y = fminf(fmaxf(v[i], lo), hi);
    if (act == 1) y = silu_f(bf16_round(y));
    v[i] = fminf(fmaxf(y, fc.plo), fc.phi);
  }
  if (out_f32) {
    store8(static_cast<float*>(out) + static_cast<size_t>(t) * ld_out + o, v);
  } else {
    store8_act(static_cast<__nv_bfloat16*>(out) + static_cast<size_t>(t) * ld_out + o, v, f16);
  }
}

// ----------------------------------------------------------- output tails
// stage 0: y = output_proj(h) fp32 -> raw bf16, embed input bf16(RMS(raw)) (no scale)
// stage 1: y = embed(...) fp32 -> soft bf16
__global__ void __launch_bounds__(256) outputs_kernel(const int* counts, const float* y, int width,
                                                     int stage, __nv_bfloat16* out,
                                                     __nv_bfloat16* next_in, float eps, bool f16) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sh[32];
  const int t = blockIdx.x;
  if (t >= counts[1]) return;
  const int e0 = threadIdx.x * 8;
  float v[8];
  load8(y + static_cast<size_t>(t) * width + e0, v);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = bf16_round(v[i]);
  store8_bf16(out + static_cast<size_t>(t) * width + e0, v);
  if (stage == 0) {
    rms8(v, nullptr, e0, width, eps, sh);
    store8_act(next_in + static_cast<size_t>(t) * width + e0, v, f16);
  }
}

// FiLM stage 0: LayerNorm(query) and LayerNorm(soft) -> bf16 GEMM inputs, RMS(query) -> amp
__global__ void __launch_bounds__(256) film_norm_kernel(const int* counts, const __nv_bfloat16* query,
                                                       int qdim, const __nv_bfloat16* soft, int hdim,
                                                       const float* qw, const float* qb,
                                                       const float* hw, const float* hb,
                                                       __nv_bfloat16* xq, __nv_bfloat16* xr,
                                                       float* amp, bool f16) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sh[32];
  const int t = blockIdx.x;
  if (t >= counts[1]) return;
  // a row of up to kHeld * 8 * blockDim elements stays in registers between the
  // statistics and the normalisation (one read); longer rows re-read the rest
  constexpr int kHeld = 4;
  const int step = blockDim.x * 8;
  for (int pass = 0; pass < 2; ++pass) {
    const int dim = pass == 0 ? qdim : hdim;
    const __nv_bfloat16* src = (pass == 0 ? query : soft) + static_cast<size_t>(t) * dim;
    const float* w = pass == 0 ? qw : hw;
    const float* b = pass == 0 ? qb : hb;
    __nv_bfloat16* dst = (pass == 0 ? xq : xr) + static_cast<size_t>(t) * dim;
    float held[kHeld][8];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const int e = threadIdx.x * 8 + j * step;
      if (e < dim) {
        load8_bf16(src + e, held[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          s += held[j][i];
          ss += held[j][i] * held[j][i];
        }
      }
    }
    for (int e = threadIdx.x * 8 + kHeld * step; e < dim; e += step) {
      float v[8];
      load8_bf16(src + e, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s += v[i];
        ss += v[i] * v[i];
      }
    }
    s = block_sum(s, sh);
    ss = block_sum(ss, sh);
    const float mean = s / dim;
    const float var = fmaxf(ss / dim - mean * mean, 0.f);
    const float rstd = rsqrtf(var + 1e-5f);
    if (pass == 0 && threadIdx.x == 0) amp[t] = sqrtf(ss / dim);
    auto finish = [&](int e, float (&v)[8]) {
      float wv[8], bv[8];
      load8(w + e, wv);
      load8(b + e, bv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (v[i] - mean) * rstd * wv[i] + bv[i];
      store8_act(dst + e, v, f16);
    };
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const int e = threadIdx.x * 8 + j * step;
      if (e < dim) finish(e, held[j]);
    }
    for (int e = threadIdx.x * 8 + kHeld * step; e < dim; e += step) {
      float v[8];
      load8_bf16(src + e, v);
      finish(e, v);
    }
  }
}

// FiLM stage 1: fused = SiLU(qd * (1 + tanh(gamma)) + beta) -> bf16
__global__ void film_fuse_kernel(const int* counts, const float* qd, const float* gb, int bdim,
                                 __nv_bfloat16* fused, bool f16) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  if (t >= counts[1]) return;
  for (int e = threadIdx.x; e < bdim; e += blockDim.x) {
    const float g = gb[static_cast<size_t>(t) * 2 * bdim + e];
    const float b = gb[static_cast<size_t>(t) * 2 * bdim + bdim + e];
    const float v = qd[static_cast<size_t>(t) * bdim + e] * (1.0f + tanhf(g)) + b;
    reinterpret_cast<uint16_t*>(fused)[static_cast<size_t>(t) * bdim + e] = act_bits(silu_f(v), f16);
  }
}

// FiLM stage 2: out = query + tanh(mapped) * scale * RMS(query)
__global__ void film_out_kernel(const int* counts, const float* mapped, const __nv_bfloat16* query,
                                const float* amp, int qdim, float scale, __nv_bfloat16* out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  if (t >= counts[1]) return;
  const int e = (blockIdx.x * blockDim.x + threadIdx.x) * 8;  // qdim is a multiple of 256
  if (e >= qdim) return;
  const size_t i = static_cast<size_t>(t) * qdim + e;
  float m[8], q[8];
  load8(mapped + i, m);
  load8_bf16(query + i, q);
  const float a = scale * amp[t];
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = q[k] + tanhf(m[k]) * a;
  store8_bf16(out + i, q);
}

}  // namespace

cudaError_t launch_row_fused(Ctx& c, int tok_cap, const RowFusedArgs& r, cudaStream_t s) {
  RowFusedDev a;
  a.counts = c.dev_counts;
  a.d = c.cfg.hidden;
  a.eps = c.cfg.rms_eps;
  a.clip = c.cfg.gradient_clipping;
  a.h = c.h;
  a.y = r.y;
  a.post_w = r.post_w;
  a.alpha = r.alpha;
  a.residual = r.residual ? 1 : 0;
  a.out_w = r.out_w;
  a.pre_w = r.pre_w;
  a.pre_norm = r.pre_norm ? 1 : 0;
  a.pre_clamp = r.pre_clamp ? 1 : 0;
  a.in_lo = r.in_lo;
  a.in_hi = r.in_hi;
  a.xa = r.xa;
  a.dbg = r.dbg;
  a.f16 = c.f16_acts != 0;
  a.zero_y = r.zero_y ? 1 : 0;
  a.y_lo = r.y_lo;
  a.y_hi = r.y_hi;
  a.xa_parts = r.xa_parts;
  a.xa_part_stride = static_cast<size_t>(2) * c.cfg.max_rows * c.cfg.hidden;
  for (int j = 0; j < 2; ++j) {
    a.part_lo[j] = r.part_lo[j];
    a.part_hi[j] = r.part_hi[j];
  }
  if (r.xa_parts != 1 && (r.xa_parts != 3 || r.xa != c.xa)) return cudaErrorInvalidValue;
  // small buckets: one token per CTA of G warps; otherwise four tokens (warps)
  // per CTA (tok_cap is a multiple of 32)
  const bool wide = tok_cap <= kSmallBucketTokens;
  const int grid = wide ? tok_cap : tok_cap / 4;
#define LB_ROW_CASE(GV)                                                                                    \
  case GV:                                                                                                 \
    if (wide)                                                                                              \
      launch_kernel(c.pdl_all, row_fused_kernel<GV, GV>, dim3(grid), dim3(32 * GV), 0, s, a);              \
    else                                                                                                   \
      launch_kernel(c.pdl_all, row_fused_kernel<GV, 1>, dim3(grid), dim3(128), 0, s, a);                   \
    break;
  switch (c.cfg.hidden / 256) {
    LB_ROW_CASE(1)
    LB_ROW_CASE(2)
    LB_ROW_CASE(3)
    LB_ROW_CASE(4)
    LB_ROW_CASE(5)
    LB_ROW_CASE(6)
    LB_ROW_CASE(8)
    default: return cudaErrorInvalidValue;
  }
#undef LB_ROW_CASE
  return cudaGetLastError();
}

cudaError_t launch_lconv(Ctx& c, int layer, int rows_cap, cudaStream_t s) {
  LconvDev a;
  a.counts = c.dev_counts;
  a.row_slot = c.row_slot;
  a.row_meta = c.row_meta;
  a.gl = c.gl;
  a.ring = c.conv_ring;
  a.dw = c.w.layers[layer].lc_dw;
  a.norm_w = c.w.layers[layer].lc_norm;
  a.xa = c.xa;
  a.layer = layer;
  a.layers = c.cfg.layers;
  a.d = c.cfg.hidden;
  a.slots = c.cfg.max_sessions;
  a.rows_cap = rows_cap;
  a.eps = c.cfg.rms_eps;
  a.clip = c.cfg.gradient_clipping;
  a.in_lo = c.w.layers[layer].clip[7][0];  // linear_end input bounds
  a.in_hi = c.w.layers[layer].clip[7][1];
  a.f16 = c.f16_acts != 0;
  // 256-thread CTAs: 8 sessions of one warp (odd G) or 4 sessions of two warps
  // (even G); small buckets: one session per CTA of G warps (one per group)
  const int g = c.cfg.hidden / 256;
  const bool wide = 2 * rows_cap <= kSmallBucketTokens;
  const int per_cta = wide ? 1 : g % 2 == 0 ? 4 : 8;
  const int grid = (rows_cap + per_cta - 1) / per_cta;
#define LB_LCONV_CASE(GV, WV)                                                                            \
  case GV:                                                                                               \
    if (wide)                                                                                            \
      launch_kernel(c.pdl_all, lconv_kernel<GV, GV>, dim3(grid), dim3(32 * GV), 0, s, a);                \
    else                                                                                                 \
      launch_kernel(c.pdl_all, lconv_kernel<GV, WV>, dim3(grid), dim3(256), 0, s, a);                    \
    break;
  switch (g) {
    LB_LCONV_CASE(1, 1)
    LB_LCONV_CASE(2, 2)
    LB_LCONV_CASE(3, 1)
    LB_LCONV_CASE(4, 2)
    LB_LCONV_CASE(5, 1)
    LB_LCONV_CASE(6, 2)
    LB_LCONV_CASE(8, 2)
    default: return cudaErrorInvalidValue;
  }
#undef LB_LCONV_CASE
  return cudaGetLastError();
}

cudaError_t launch_split_finish(const int* m_dev, int m_static, int m_cap, float* acc, int width, int act,
                                void* out, int ld_out, bool out_f32, bool f16, const FinalizeClip& fc,
                                bool pdl, cudaStream_t s) {
  if (width % 8 || ld_out % 8 || fc.part_o < 0 || (fc.part_o && (fc.part_o % 128 || width / fc.part_o > 3)))
    return cudaErrorInvalidValue;
  const int per_block = 128 * 8;
  dim3 grid((width + per_block - 1) / per_block, m_cap);
  launch_kernel(pdl, split_finish_kernel, grid, dim3(128), 0, s, m_dev, m_static, acc, width, act, out, ld_out,
                out_f32 ? 1 : 0, fc, f16);
  return cudaGetLastError();
}

cudaError_t launch_outputs(Ctx& c, int tok_cap, int stage, cudaStream_t s) {
  const int width = stage == 0 ? c.cfg.output_dims : c.cfg.text_hidden;
  launch_kernel(c.pdl_all, outputs_kernel, dim3(tok_cap), dim3(width / 8), 0, s, c.dev_counts, c.y, width, stage,
                                               stage == 0 ? c.out_raw : c.out_soft, c.xe,
                                               c.cfg.rms_eps, c.f16_acts != 0);
  return cudaGetLastError();
}

// Talker placement of the FiLM adapter (apply_response_state_residual,
// duplex_kernel/frame_residual_adapter.py:38-71): row i takes response state
// min(step, n_states - 1) of its [max_states][hdim] response hidden (the
// Qwen text cursor; the last state is held once the text is exhausted) and
// its query into the FiLM inputs, and sets the FiLM token count to n.
__global__ void __launch_bounds__(256) film_talker_gather_kernel(
    int n, const __nv_bfloat16* hidden, int max_states, const int* n_states, const int* steps,
    const __nv_bfloat16* query, int hdim, int qdim, __nv_bfloat16* soft, __nv_bfloat16* in_query, int* counts,
    int* status) {
  const int i = blockIdx.x;
  if (i == 0 && threadIdx.x == 0) counts[1] = n;
  const int ns = n_states[i], st = steps[i];
  if (ns < 1 || ns > max_states || st < 0) {
    if (threadIdx.x == 0) atomicOr(status, kStatusBadRowCount);
    return;
  }
  const int idx = min(st, ns - 1);
  const int4* src = reinterpret_cast<const int4*>(hidden + (static_cast<size_t>(i) * max_states + idx) * hdim);
  int4* dst = reinterpret_cast<int4*>(soft + static_cast<size_t>(i) * hdim);
  for (int e = threadIdx.x; e < hdim / 8; e += blockDim.x) dst[e] = src[e];
  const int4* qs = reinterpret_cast<const int4*>(query + static_cast<size_t>(i) * qdim);
  int4* qd = reinterpret_cast<int4*>(in_query + static_cast<size_t>(i) * qdim);
  for (int e = threadIdx.x; e < qdim / 8; e += blockDim.x) qd[e] = qs[e];
}

// out = query at the first generation step (the query FiLM adapter's
// preserve_frame0), the conditioned query otherwise.
__global__ void __launch_bounds__(256) film_talker_finish_kernel(int n, const int* steps, const __nv_bfloat16* query,
                                                                 const __nv_bfloat16* film, int qdim,
                                                                 __nv_bfloat16* out) {
  const int i = blockIdx.x;
  const bool keep = steps[i] == 0;
  const int4* src = reinterpret_cast<const int4*>((keep ? query : film) + static_cast<size_t>(i) * qdim);
  int4* dst = reinterpret_cast<int4*>(out + static_cast<size_t>(i) * qdim);
  for (int e = threadIdx.x; e < qdim / 8; e += blockDim.x) dst[e] = src[e];
}

cudaError_t launch_film_talker(Ctx& c, int n, const __nv_bfloat16* hidden, int max_states, const int* n_states,
                               const int* steps, const __nv_bfloat16* query, __nv_bfloat16* out, int stage,
                               cudaStream_t s) {
  const int Q = c.cfg.film_query_dim, T = c.cfg.text_hidden;
  if (stage == 0)
    film_talker_gather_kernel<<<n, 256, 0, s>>>(n, hidden, max_states, n_states, steps, query, T, Q, c.out_soft,
                                                 c.in_query, c.dev_counts, c.status);
  else
    film_talker_finish_kernel<<<n, 256, 0, s>>>(n, steps, query, c.out_film, Q, out);
  return cudaGetLastError();
}

cudaError_t launch_film(Ctx& c, int tok_cap, int stage, cudaStream_t s) {
  const int Q = c.cfg.film_query_dim, B = c.cfg.film_bottleneck, T = c.cfg.text_hidden;
  if (stage == 0) {
    launch_kernel(c.pdl_all, film_norm_kernel, dim3(tok_cap), dim3(128), 0, s, c.dev_counts, c.in_query, Q, c.out_soft, T,
                                             c.w.fq_norm_w, c.w.fq_norm_b, c.w.fr_norm_w,
                                             c.w.fr_norm_b, c.film_xq, c.film_xr, c.film_amp,
                                             c.f16_acts != 0);
  } else if (stage == 1) {
    launch_kernel(c.pdl_all, film_fuse_kernel, dim3(tok_cap), dim3(128), 0, s, c.dev_counts, c.film_qd, c.film_gb, B, c.film_fused,
                                             c.f16_acts != 0);
  } else {
    dim3 grid((Q / 8 + 255) / 256, tok_cap);  // eight elements per thread
    launch_kernel(c.pdl_all, film_out_kernel, dim3(grid), dim3(256), 0, s, c.dev_counts, c.film_map, c.in_query, c.film_amp, Q,
                                         c.w.film_scale, c.out_film);
  }
  return cudaGetLastError();
}

}  // namespace lb
