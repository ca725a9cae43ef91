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
// Layout: one CTA per batch row (session), one warp per head.  Each warp first
// requests every K and V row its keys need with bulk asynchronous copies into
// its shared-memory slice (one mbarrier, one memory round trip), so the loads
// of a whole window are in flight together.  The 2 x 13 query-key and the
// 2 x 13 query-relative-key dot products then run on the tensor cores:
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) with the two queries as rows
// 0-1 of A (the scaled query rounded to bf16, as the reference's bf16 tower
// holds it), the shared-memory K rows (ldmatrix) and the bf16 relative keys as
// two B n-tiles each, over hd/16 k-steps.  Lanes then own (query, key) pairs --
// lanes 0..14 query 0, lanes 16..30 query 1 -- for the logits and the fp32
// softmax, which reduces within each 16-lane half.  Out-of-window keys (cached
// keys 0 and 1) and invalid keys are masked and not copied.  If every key of a
// query is masked, all logits equal the invalid value and the softmax is
// uniform over the 15 keys, exactly as in the reference; the value rows that
// were not copied are then read directly.  The value sum runs on the SIMT
// cores with lanes owning head dimensions.
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
  const __nv_bfloat16* rel_bf16;  // [13][d] relative keys, bf16
  int* status;
  int layer, layers, d, slots;
  float k_scale, softcap, invalid;
  float in_lo, in_hi;  // attention.post input clamp
  bool f16;            // out holds fp16 (int8-weight GEMM input) instead of bf16
};

__device__ __forceinline__ void mma_bf16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                                  uint32_t b1) {
  // A rows 8..15 are zero (only the two queries are real)
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float x, float y) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// Shared memory of one warp: 16 K rows (padded by 16 bytes so the 8 rows an
// ldmatrix reads fall in distinct banks), 15 V rows, the mbarrier, and the
// 2 x 2 x 16 logit partials.
template <int HD>
struct AttnSmem {
  static constexpr int kKStride = HD * 2 + 16;
  static constexpr int kK = 0;
  static constexpr int kV = 16 * kKStride;
  static constexpr int kBar = kV + 15 * HD * 2;
  static constexpr int kLogit = kBar + 16;
  static constexpr int kBytes = kLogit + 64 * 4;
};

template <int HD>
__global__ void __launch_bounds__(512) attention_kernel(AttnDev a) {
  pdl_wait();  // first: nothing of the previous kernel is read or written before it
  pdl_trigger();
  using L = AttnSmem<HD>;
  constexpr int NP = HD / 64;  // bf16 pairs per lane in the value sum (lanes own dimensions)
  constexpr int KS = HD / 16;  // MMA k-steps over the head dimension
  extern __shared__ __align__(128) unsigned char smem_att[];
  const int row = blockIdx.x;
  // the row tables are read together with the live row count (one round trip);
  // they are in bounds for every row of the bucket, and a row past the count
  // uses none of them
  const int n_rows = a.counts[0];
  const int slot = a.row_slot[row];
  const SlotMeta m = a.row_meta[row];
  const int mask = a.row_mask[row];
  if (row >= n_rows) return;
  const int head = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;  // MMA fragment coordinates
  unsigned char* ws = smem_att + head * L::kBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ws + L::kBar);
  float* sl = reinterpret_cast<float*>(ws + L::kLogit);
  const int d = a.d;
  const size_t ring_off = ring_base(slot, a.layer, a.slots, kRing, d);
  const int hoff = head * HD;
  const __nv_bfloat16* qkv0 = a.qkv + static_cast<size_t>(row) * 2 * 3 * d;

  // ---- key j (0..14) of this lane: ring entry (m.pos + j) or new token j - 13.
  // Lane j copies key j's K row, lane 16 + j its V row (keys 2..14 that are valid).
  const int kj = lane & 15;
  bool need = false;
  const __nv_bfloat16* krow = qkv0;
  if (kj >= 2 && kj < kCached) {
    const int idx = (m.pos + kj) & (kRing - 1);
    need = (m.valid_bits >> idx) & 1;
    krow = a.kc + ring_off + static_cast<size_t>(idx) * d + hoff;
  } else if (kj >= kCached && kj < kCached + 2) {
    need = (mask >> (4 * (kj - kCached))) & 1;
    krow = qkv0 + (kj - kCached) * 3 * d + d + hoff;
  }
  const __nv_bfloat16* src = lane < 16 ? krow
                             : kj < kCached ? a.vc + (krow - a.kc)  // same ring position in V
                                            : krow + d;              // V follows K in the qkv row
  const uint32_t loaded = __ballot_sync(0xffffffffu, need) & 0xffffu;  // key bits (K == V set)
  if (lane == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  if (lane == 0) mbar_arrive_expect_tx(bar, 2u * __popc(loaded) * HD * 2);
  __syncwarp();
  if (need) {
    void* dst = lane < 16 ? static_cast<void*>(ws + L::kK + kj * L::kKStride)
                          : static_cast<void*>(ws + L::kV + kj * HD * 2);
    bulk_copy_g2s(dst, src, HD * 2, bar);
  }

  // ---- the two new K/V rows this head stages into the ring (positions pos+13,
  // pos+14) are read now and stored at the end: interleaving those loads with
  // the ring stores would serialise one memory round trip per pair
  uint32_t stage_k[2][NP], stage_v[2][NP];
#pragma unroll
  for (int tt = 0; tt < 2; ++tt)
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const __nv_bfloat16* srcq = qkv0 + tt * 3 * d + hoff + 2 * lane + 64 * r;
      stage_k[tt][r] = *reinterpret_cast<const uint32_t*>(srcq + d);
      stage_v[tt][r] = *reinterpret_cast<const uint32_t*>(srcq + 2 * d);
    }

  // ---- every remaining global load of the logit phase is issued before any
  // use: the queries (lanes 0..7, rows 0 and 1 of A) with their scale, and the
  // relative-key B fragments r = nt*8 + g (rows 0..12 of the bf16 copy; 13..15
  // padding, zero)
  uint32_t qraw[KS][2];
  float2 qmul[KS][2];
  uint32_t rb[2][KS][2];
  const __nv_bfloat16* qrow = qkv0 + (g & 1) * 3 * d + hoff;
#pragma unroll
  for (int s = 0; s < KS; ++s)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 16 * s + 8 * h + 2 * c;
      qraw[s][h] = g < 2 ? *reinterpret_cast<const uint32_t*>(qrow + e) : 0u;
      qmul[s][h] = g < 2 ? __ldg(reinterpret_cast<const float2*>(a.q_mult + e)) : make_float2(0.f, 0.f);
    }
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int r = nt * 8 + g;
    const __nv_bfloat16* rrow = a.rel_bf16 + static_cast<size_t>(r <= 12 ? r : 0) * d + hoff;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int e0 = 16 * s + 2 * c;
      rb[nt][s][0] = r <= 12 ? __ldg(reinterpret_cast<const unsigned int*>(rrow + e0)) : 0u;
      rb[nt][s][1] = r <= 12 ? __ldg(reinterpret_cast<const unsigned int*>(rrow + e0 + 8)) : 0u;
    }
  }
  uint32_t qa[KS][2];
#pragma unroll
  for (int s = 0; s < KS; ++s)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 qv = unpack_bf16x2(qraw[s][h]);
      qa[s][h] = pack_bf16x2(qv.x * qmul[s][h].x, qv.y * qmul[s][h].y);  // zero for lanes 8..31
    }
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    mma_bf16_m16n8k16(acc[2], qa[s][0], qa[s][1], rb[0][s][0], rb[0][s][1]);
    mma_bf16_m16n8k16(acc[3], qa[s][0], qa[s][1], rb[1][s][0], rb[1][s][1]);
  }
  // ---- K rows have landed: query-key products from shared memory
  const bool landed = mbar_wait(bar, 0, a.status);
  if (landed) {
    const int mi = lane >> 3;
    const uint32_t kaddr = smem_u32(ws + L::kK + ((mi >> 1) * 8 + (lane & 7)) * L::kKStride + (mi & 1) * 16);
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      uint32_t b00, b01, b10, b11;
      ldmatrix_x4(kaddr + s * 32, b00, b01, b10, b11);
      mma_bf16_m16n8k16(acc[0], qa[s][0], qa[s][1], b00, b01);
      mma_bf16_m16n8k16(acc[1], qa[s][0], qa[s][1], b10, b11);
    }
  } else if (!mbar_wait(bar, 0, a.status)) {
    return;  // status already records the timeout; the copies had a second bound to land
  }
  // C fragments: lanes 0..7 hold row (query) g, columns nt*8 + 2c + {0, 1}
  if (g < 2) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      *reinterpret_cast<float2*>(sl + g * 16 + nt * 8 + 2 * c) = make_float2(acc[nt][0], acc[nt][1]);
      *reinterpret_cast<float2*>(sl + 32 + g * 16 + nt * 8 + 2 * c) = make_float2(acc[2 + nt][0], acc[2 + nt][1]);
    }
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
      const float s = fmaf(sl[t * 16 + j], a.k_scale, sl[32 + t * 16 + (12 - dist)]);
      logit = tanhf(s / a.softcap) * a.softcap;
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

  // ---- weighted values from the shared-memory V rows; lanes own dimensions
  float2 o0[NP], o1[NP];
#pragma unroll
  for (int r = 0; r < NP; ++r) o0[r] = o1[r] = make_float2(0.f, 0.f);
  const unsigned char* vs = ws + L::kV;
#pragma unroll
  for (int jj = 2; jj < 15; ++jj) {
    const float w0 = __shfl_sync(0xffffffffu, p, jj), w1 = __shfl_sync(0xffffffffu, p, 16 + jj);
    if (!((loaded >> jj) & 1)) continue;  // warp-uniform; not copied (masked: weight 0 unless uniform)
    const float2 p0 = make_float2(w0, w0), p1 = make_float2(w1, w1);
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(vs + jj * HD * 2 + (2 * lane + 64 * r) * 2));
      o0[r] = __ffma2_rn(p0, v, o0[r]);
      o1[r] = __ffma2_rn(p1, v, o1[r]);
    }
  }
  // rare: a query with every key masked weights all 15 keys; add the rows not copied
  const int first_real = kCached - m.fill;  // cached entries before this were never written (zero)
  const bool extra = j < 15 && p != 0.f && !((loaded >> j) & 1) && (j >= kCached || j >= first_real);
  if (__any_sync(0xffffffffu, extra)) {
    for (int jj = 0; jj < 15; ++jj) {
      if ((loaded >> jj) & 1) continue;
      if (jj < kCached && jj < first_real) continue;
      const float w0 = __shfl_sync(0xffffffffu, p, jj), w1 = __shfl_sync(0xffffffffu, p, 16 + jj);
      if (w0 == 0.f && w1 == 0.f) continue;
      const __nv_bfloat16* vrow =
          jj < kCached ? a.vc + ring_off + static_cast<size_t>((m.pos + jj) & (kRing - 1)) * d + hoff
                       : qkv0 + (jj - kCached) * 3 * d + 2 * d + hoff;
      const float2 p0 = make_float2(w0, w0), p1 = make_float2(w1, w1);
#pragma unroll
      for (int r = 0; r < NP; ++r) {
        const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(vrow + 2 * lane + 64 * r));
        o0[r] = __ffma2_rn(p0, v, o0[r]);
        o1[r] = __ffma2_rn(p1, v, o1[r]);
      }
    }
  }
  __nv_bfloat16* dst0 = a.out + static_cast<size_t>(row) * 2 * d + hoff;
#pragma unroll
  for (int r = 0; r < NP; ++r) {
    const int e = 2 * lane + 64 * r;
    *reinterpret_cast<uint32_t*>(dst0 + e) =
        act_bits2(fminf(fmaxf(o0[r].x, a.in_lo), a.in_hi), fminf(fmaxf(o0[r].y, a.in_lo), a.in_hi), a.f16);
    *reinterpret_cast<uint32_t*>(dst0 + d + e) =
        act_bits2(fminf(fmaxf(o1[r].x, a.in_lo), a.in_hi), fminf(fmaxf(o1[r].y, a.in_lo), a.in_hi), a.f16);
  }
  // ---- stage the two new K/V entries at ring positions pos+13, pos+14
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    const size_t idx = static_cast<size_t>((m.pos + kCached + tt) & (kRing - 1));
#pragma unroll
    for (int r = 0; r < NP; ++r) {
      const int e = 2 * lane + 64 * r;
      *reinterpret_cast<uint32_t*>(a.kc + ring_off + idx * d + hoff + e) = stage_k[tt][r];
      *reinterpret_cast<uint32_t*>(a.vc + ring_off + idx * d + hoff + e) = stage_v[tt][r];
    }
  }
}

__global__ void rel_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

size_t attention_smem_bytes(int heads, int hd) {
  switch (hd) {
    case 64: return static_cast<size_t>(heads) * AttnSmem<64>::kBytes;
    case 128: return static_cast<size_t>(heads) * AttnSmem<128>::kBytes;
    case 192: return static_cast<size_t>(heads) * AttnSmem<192>::kBytes;
    default: return static_cast<size_t>(heads) * AttnSmem<256>::kBytes;
  }
}

}  // namespace

// Dynamic shared memory above 48 KB must be enabled per kernel instance, once
// per device and before any graph capture.
cudaError_t attention_init_attributes() {
  // the largest CTA each instance can get: d <= 2048, so heads <= 2048 / hd (and <= 16)
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(attention_smem_bytes(16, 64)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(attention_smem_bytes(16, 128)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_kernel<192>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(attention_smem_bytes(10, 192)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(attention_smem_bytes(8, 256)));
  return e;
}

cudaError_t attention_prepare(Ctx& c, cudaStream_t s) {
  const int n = 13 * c.cfg.hidden;
  for (int l = 0; l < c.cfg.layers; ++l) {
    LayerW& L = c.w.layers[l];
    L.rel_bf16 = c.rel_bf16_arena + static_cast<size_t>(l) * n;
    rel_to_bf16_kernel<<<(n + 255) / 256, 256, 0, s>>>(L.rel_keys, L.rel_bf16, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
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
  a.rel_bf16 = c.w.layers[layer].rel_bf16;
  a.status = c.status;
  a.layer = layer;
  a.layers = c.cfg.layers;
  a.d = c.cfg.hidden;
  a.slots = c.cfg.max_sessions;
  a.k_scale = static_cast<float>(std::log1p(std::exp(1.0)) / std::log(2.0));
  a.softcap = c.cfg.softcap;
  a.invalid = c.cfg.invalid_logit;
  a.in_lo = c.w.layers[layer].clip[5][0];
  a.in_hi = c.w.layers[layer].clip[5][1];
  a.f16 = c.f16_acts != 0;
  const int threads = 32 * c.cfg.heads;
  const size_t smem = attention_smem_bytes(c.cfg.heads, c.hd);
  switch (c.hd) {
    case 64: launch_kernel(c.pdl_all, attention_kernel<64>, dim3(rows_cap), dim3(threads), smem, s, a); break;
    case 128: launch_kernel(c.pdl_all, attention_kernel<128>, dim3(rows_cap), dim3(threads), smem, s, a); break;
    case 192: launch_kernel(c.pdl_all, attention_kernel<192>, dim3(rows_cap), dim3(threads), smem, s, a); break;
    case 256: launch_kernel(c.pdl_all, attention_kernel<256>, dim3(rows_cap), dim3(threads), smem, s, a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace lb
