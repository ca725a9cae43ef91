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
// Layout: one CTA per batch row (session), one warp per head.  For the logits
// a lane owns one (query, key) pair -- lanes 0..14 query 0, lanes 16..30 query
// 1 -- and computes its dot product privately from its own K row (16-byte
// loads, all independent), so no per-key warp reduction is needed.  Keys that
// are outside the window of the lane's query are never loaded (cached keys 0
// and 1 are outside both windows).  The softmax reduces within each 16-lane
// half; then lanes switch to owning head dimensions and accumulate p_j * v_j,
// loading only values with a non-zero weight.  If every key of a query is
// masked, all logits equal the invalid value and the softmax is uniform over
// the 15 keys, exactly as in the reference.
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
};

template <int HD>
__global__ void __launch_bounds__(512) attention_kernel(AttnDev a) {
  constexpr int NP = HD / 64;  // bf16 pairs per lane when lanes own dimensions
  extern __shared__ float qs[];  // [heads][2][HD]
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
  float* q_smem = qs + head * 2 * HD;

  // scaled queries of this head into shared memory
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const int e = 2 * lane + 64 * r;
      const float2 qv = __bfloat1622float2(
          *reinterpret_cast<const __nv_bfloat162*>(qkv0 + t * 3 * d + hoff + e));
      q_smem[t * HD + e] = qv.x * a.q_mult[e];
      q_smem[t * HD + e + 1] = qv.y * a.q_mult[e + 1];
    }
  __syncwarp();

  // ---- logits: lane -> (query t, key j)
  const int t = lane >> 4;
  const int j = lane & 15;
  float logit = -INFINITY;  // lanes 15 and 31 hold no key
  if (j < 15) {
    const int dist = j < kCached ? (kCached - j + t) : (t - (j - kCached));
    bool ok = dist >= 0 && dist < 12;
    if (j < kCached) {
      ok = ok && ((m.valid_bits >> ((m.pos + j) & (kRing - 1))) & 1);
    } else {
      ok = ok && ((mask >> (4 * (j - kCached))) & 1);
    }
    logit = a.invalid;
    if (ok) {
      const __nv_bfloat16* krow =
          j < kCached ? a.kc + ring_base + static_cast<size_t>((m.pos + j) & (kRing - 1)) * d + hoff
                      : qkv0 + (j - kCached) * 3 * d + d + hoff;
      const float* rel = a.rel + static_cast<size_t>(12 - min(max(dist, 0), 12)) * d + hoff;
      const float* qrow = q_smem + t * HD;
      float acc = 0.f;
#pragma unroll 4
      for (int e = 0; e < HD; e += 8) {
        const int4 kr = *reinterpret_cast<const int4*>(krow + e);
        const __nv_bfloat162* kp = reinterpret_cast<const __nv_bfloat162*>(&kr);
        const float4 r0 = __ldg(reinterpret_cast<const float4*>(rel + e));
        const float4 r1 = __ldg(reinterpret_cast<const float4*>(rel + e + 4));
        const float4 q0 = *reinterpret_cast<const float4*>(qrow + e);
        const float4 q1 = *reinterpret_cast<const float4*>(qrow + e + 4);
        const float2 k0 = __bfloat1622float2(kp[0]), k1 = __bfloat1622float2(kp[1]);
        const float2 k2 = __bfloat1622float2(kp[2]), k3 = __bfloat1622float2(kp[3]);
        acc = fmaf(q0.x, fmaf(k0.x, a.k_scale, r0.x), acc);
        acc = fmaf(q0.y, fmaf(k0.y, a.k_scale, r0.y), acc);
        acc = fmaf(q0.z, fmaf(k1.x, a.k_scale, r0.z), acc);
        acc = fmaf(q0.w, fmaf(k1.y, a.k_scale, r0.w), acc);
        acc = fmaf(q1.x, fmaf(k2.x, a.k_scale, r1.x), acc);
        acc = fmaf(q1.y, fmaf(k2.y, a.k_scale, r1.y), acc);
        acc = fmaf(q1.z, fmaf(k3.x, a.k_scale, r1.z), acc);
        acc = fmaf(q1.w, fmaf(k3.y, a.k_scale, r1.w), acc);
      }
      logit = tanhf(acc / a.softcap) * a.softcap;
    }
  }
  // ---- softmax within each 16-lane half (one query per half)
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
    *reinterpret_cast<__nv_bfloat162*>(dst0 + e) =
        __floats2bfloat162_rn(fminf(fmaxf(o0[2 * r], a.in_lo), a.in_hi), fminf(fmaxf(o0[2 * r + 1], a.in_lo), a.in_hi));
    *reinterpret_cast<__nv_bfloat162*>(dst0 + d + e) =
        __floats2bfloat162_rn(fminf(fmaxf(o1[2 * r], a.in_lo), a.in_hi), fminf(fmaxf(o1[2 * r + 1], a.in_lo), a.in_hi));
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

}  // namespace

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
  const int threads = 32 * c.cfg.heads;
  const size_t smem = static_cast<size_t>(c.cfg.heads) * 2 * c.hd * sizeof(float);
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
