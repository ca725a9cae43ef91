// Chunked local attention of the streaming Conformer step, reading each
// session's K/V ring in place (no gather, no window copy).
//
// Restates the Q2 attention of StreamingConformerAudioTower._compute_step
// (duplex_kernel/streaming_conformer.py:778-829) over transformers'
// Gemma4AudioAttention (models/gemma4/modeling_gemma4.py:209-314):
//   q = q_proj(x) * (hd^-0.5 / ln 2) * softplus(per_dim_scale)
//   k = k_proj(x) * ln(1+e)/ln 2;  keys = 13 cached + the 2 new tokens
//   logit = q.k + q.relK[12 - clamp(dist, 0, 12)]          (dist = query - key position)
//   logit = 50 tanh(logit / 50); masked to -1e9 outside 0 <= dist < 12 or for
//   invalid tokens; fp32 softmax; out = sum p_j v_j.
//
// Layout: one CTA per batch row (session), one warp per head.  Lanes own head
// dimensions for every load, so K rows, V rows and relative-key rows are read
// with whole-warp coalesced accesses; each lane forms partial dot products for
// the 13 reachable keys and the 12 window distances, and a padded shared-memory
// transpose sums them.  Lanes then own (query, key) pairs -- lanes 0..14 query
// 0, lanes 16..30 query 1 -- for the logits and the softmax, which reduces
// within each 16-lane half.  Cached keys 0 and 1 lie outside both windows and
// invalid keys are masked, so neither is loaded.  If every key of a query is
// masked, all logits equal the invalid value and the softmax is uniform over
// the 15 keys, exactly as in the reference; values are loaded only for keys
// with a non-zero weight.
#include "common.cuh"
#include "listener.h"

#include <cmath>

namespace lb {
namespace {

struct AttnDev {
  const int* counts;
  const int *row_slot, *row_mask;
  const SlotMeta* row_meta;
  const __nv_bfloat16* qkv;  // [tok][3d]
  __nv_bfloat16 *kc, *vc;    // [S][L][16][d]
  __nv_bfloat16* out;        // [tok][d]
  const float* q_mult;       // [hd]
  const float* rel;          // [13][d]
  int layer, layers, d;
  float k_scale, softcap, invalid;
  float in_lo, in_hi;  // attention.post input clamp
  bool f16;            // out holds fp16 (int8-weight GEMM input) instead of bf16
};

template <int HD>
__global__ void __launch_bounds__(512) attention_kernel(AttnDev a) {
  constexpr int NP = HD / 64;  // bf16 pairs per lane (lanes own head dimensions)
  // per warp: 52 partial sums x 33 (padded) + 52 totals
  constexpr int kParts = 52, kPad = 33;
  extern __shared__ float smem_att[];
  const int row = blockIdx.x;
  if (row >= a.counts[0]) return;
  const int head = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = a.row_slot[row];
  const SlotMeta m = a.row_meta[row];
  const int mask = a.row_mask[row];
  const int d = a.d;
  const size_t ring_base = (static_cast<size_t>(slot) * a.layers + a.layer) * kRing * d;
  const int hoff = head * HD;
  const __nv_bfloat16* qkv0 = a.qkv + static_cast<size_t>(row) * 2 * 3 * d;
  float* part = smem_att + head * (kParts * kPad + kParts);
  float* tot = part + kParts * kPad;

  // scaled queries (registers), lane dims e = 2*lane + 64*r
  float q[2][2 * NP];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const int e = 2 * lane + 64 * r;
      const float2 qv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qkv0 + t * 3 * d + hoff + e));
      q[t][2 * r] = qv.x * a.q_mult[e];
      q[t][2 * r + 1] = qv.y * a.q_mult[e + 1];
    }
  // ---- partial dot products, all loads coalesced across the warp.
  // part[2*i + t]       : q_t . k_{2+i}            keys j = 2..14 (i = 0..12)
  // part[26 + 2*dist + t]: q_t . relK[12 - dist]    dist = 0..11
  // Cached keys 0 and 1 lie outside both windows; invalid cached keys are
  // masked whatever their logit, so neither is loaded.
#pragma unroll
  for (int i = 0; i < 13; ++i) {
    const int j = 2 + i;
    float s0 = 0.f, s1 = 0.f;
    bool need;
    const __nv_bfloat16* krow;
    if (j < kCached) {
      const int idx = (m.pos + j) & (kRing - 1);
      need = (m.valid_bits >> idx) & 1;
      krow = a.kc + ring_base + static_cast<size_t>(idx) * d + hoff;
    } else {
      need = (mask >> (4 * (j - kCached))) & 1;
      krow = qkv0 + (j - kCached) * 3 * d + d + hoff;
    }
    if (need) {
#pragma unroll
      for (int r = 0; r < NP; ++r) {
        const float2 k = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(krow + 2 * lane + 64 * r));
        s0 = fmaf(q[0][2 * r], k.x, fmaf(q[0][2 * r + 1], k.y, s0));
        s1 = fmaf(q[1][2 * r], k.x, fmaf(q[1][2 * r + 1], k.y, s1));
      }
    }
    part[(2 * i) * kPad + lane] = s0;
    part[(2 * i + 1) * kPad + lane] = s1;
  }
#pragma unroll
  for (int dist = 0; dist < 12; ++dist) {
    const float* rrow = a.rel + static_cast<size_t>(12 - dist) * d + hoff;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const float2 rv = __ldg(reinterpret_cast<const float2*>(rrow + 2 * lane + 64 * r));
      s0 = fmaf(q[0][2 * r], rv.x, fmaf(q[0][2 * r + 1], rv.y, s0));
      s1 = fmaf(q[1][2 * r], rv.x, fmaf(q[1][2 * r + 1], rv.y, s1));
    }
    part[(26 + 2 * dist) * kPad + lane] = s0;
    part[(26 + 2 * dist + 1) * kPad + lane] = s1;
  }
  __syncwarp();
  // transpose-reduce: lane l totals rows l and l + 32
  for (int rr = lane; rr < 50; rr += 32) {
    float s = 0.f;
#pragma unroll 8
    for (int c = 0; c < 32; ++c) s += part[rr * kPad + c];
    tot[rr] = s;
  }
  __syncwarp();

  // ---- logits: lane -> (query t, key j); lanes 15 and 31 hold no key
  const int t = lane >> 4;
  const int j = lane & 15;
  float logit = -INFINITY;
  if (j < 15) {
    const int dist = j < kCached ? (kCached - j + t) : (t - (j - kCached));
    bool ok = dist >= 0 && dist < 12;
    if (j < kCached) {
      ok = ok && ((m.valid_bits >> ((m.pos + j) & (kRing - 1))) & 1);
    } else {
      ok = ok && ((mask >> (4 * (j - kCached))) & 1);
    }
    logit = a.invalid;
    if (ok) {  // ok implies j >= 2 and 0 <= dist < 12
      const float acc = fmaf(tot[2 * (j - 2) + t], a.k_scale, tot[26 + 2 * dist + t]);
      logit = tanhf(acc / a.softcap) * a.softcap;
    }
  }
  // ---- softmax within each 16-lane half (one query per half).  If every key of
  // a query is masked, all 15 logits equal the invalid value: uniform weights.
  float mx = logit;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float p = (j < 15) ? expf(logit - mx) : 0.f;
  float sum = p;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  p = p / sum;

  // ---- weighted values: lanes own head dimensions again
  float o0[2 * NP], o1[2 * NP];
#pragma unroll
  for (int i = 0; i < 2 * NP; ++i) o0[i] = o1[i] = 0.f;
  const int first_real = kCached - m.fill;  // cached entries before this were never written (zero)
#pragma unroll
  for (int jj = 0; jj < 15; ++jj) {
    const float p0 = __shfl_sync(0xffffffffu, p, jj);
    const float p1 = __shfl_sync(0xffffffffu, p, 16 + jj);
    if (p0 == 0.f && p1 == 0.f) continue;  // warp-uniform
    if (jj < kCached && jj < first_real) continue;  // a zero value row adds nothing
    const __nv_bfloat16* vrow =
        jj < kCached ? a.vc + ring_base + static_cast<size_t>((m.pos + jj) & (kRing - 1)) * d + hoff
                     : qkv0 + (jj - kCached) * 3 * d + 2 * d + hoff;
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vrow + 2 * lane + 64 * r));
      o0[2 * r] = fmaf(p0, v.x, o0[2 * r]);
      o0[2 * r + 1] = fmaf(p0, v.y, o0[2 * r + 1]);
      o1[2 * r] = fmaf(p1, v.x, o1[2 * r]);
      o1[2 * r + 1] = fmaf(p1, v.y, o1[2 * r + 1]);
    }
  }
  __nv_bfloat16* dst0 = a.out + static_cast<size_t>(row) * 2 * d + hoff;
#pragma unroll
  for (int r = 0; r < NP; ++r) {
    const int e = 2 * lane + 64 * r;
    *reinterpret_cast<uint32_t*>(dst0 + e) =
        act_bits2(fminf(fmaxf(o0[2 * r], a.in_lo), a.in_hi), fminf(fmaxf(o0[2 * r + 1], a.in_lo), a.in_hi), a.f16);
    *reinterpret_cast<uint32_t*>(dst0 + d + e) =
        act_bits2(fminf(fmaxf(o1[2 * r], a.in_lo), a.in_hi), fminf(fmaxf(o1[2 * r + 1], a.in_lo), a.in_hi), a.f16);
  }
  // ---- stage the two new K/V entries at ring positions pos+13, pos+14
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    const size_t idx = static_cast<size_t>((m.pos + kCached + tt) & (kRing - 1));
    const __nv_bfloat16* src = qkv0 + tt * 3 * d + hoff;
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const int e = 2 * lane + 64 * r;
      *reinterpret_cast<__nv_bfloat162*>(a.kc + ring_base + idx * d + hoff + e) =
          *reinterpret_cast<const __nv_bfloat162*>(src + d + e);
      *reinterpret_cast<__nv_bfloat162*>(a.vc + ring_base + idx * d + hoff + e) =
          *reinterpret_cast<const __nv_bfloat162*>(src + 2 * d + e);
    }
  }
}

size_t attention_smem_bytes(int heads) { return static_cast<size_t>(heads) * (52 * 33 + 52) * sizeof(float); }

}  // namespace

// Dynamic shared memory above 48 KB must be enabled per kernel instance, once
// per device and before any graph capture.
cudaError_t attention_init_attributes() {
  const int bytes = static_cast<int>(attention_smem_bytes(16));
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<192>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e;
}

cudaError_t launch_attention(Ctx& c, int layer, int rows_cap, cudaStream_t s) {
  AttnDev a;
  a.counts = c.dev_counts;
  a.row_slot = c.row_slot;
  a.row_mask = c.row_mask;
  a.row_meta = c.row_meta;
  a.qkv = c.qkv;
  a.kc = c.kv_k;
  a.vc = c.kv_v;
  a.out = c.att;
  a.q_mult = c.w.layers[layer].q_mult;
  a.rel = c.w.layers[layer].rel_keys;
  a.layer = layer;
  a.layers = c.cfg.layers;
  a.d = c.cfg.hidden;
  a.k_scale = static_cast<float>(std::log1p(std::exp(1.0)) / std::log(2.0));
  a.softcap = c.cfg.softcap;
  a.invalid = c.cfg.invalid_logit;
  a.in_lo = c.w.layers[layer].clip[5][0];
  a.in_hi = c.w.layers[layer].clip[5][1];
  a.f16 = c.weight_int8 != 0;
  const int threads = 32 * c.cfg.heads;
  const size_t smem = attention_smem_bytes(c.cfg.heads);
  switch (c.hd) {
    case 64: attention_kernel<64><<<rows_cap, threads, smem, s>>>(a); break;
    case 128: attention_kernel<128><<<rows_cap, threads, smem, s>>>(a); break;
    case 192: attention_kernel<192><<<rows_cap, threads, smem, s>>>(a); break;
    case 256: attention_kernel<256><<<rows_cap, threads, smem, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace lb
