// Frontend kernels of the listener step: PCM -> log-mel, and the streaming
// 2x(3x3, stride 2) convolutional subsampler.
//
// mel_kernel restates GemmaAudioTowerBackend._extract_single_frame
// (duplex_kernel/listener.py:1807-1850): [160-sample tail | 1280 PCM | 0] ->
// eight 320-sample frames at hop 160, times the periodic Hann window (the
// product is formed in fp32 exactly as the reference's float32 NumPy does),
// 512-point real DFT magnitude (a 256-point complex FFT and the real-input
// split, exact twiddles from a 512-entry table), HTK mel filterbank,
// log(x + 1e-3).  One CTA per session.
//
// subsample_kernel restates the streaming subsampler
// (duplex_kernel/streaming_conformer.py:741-761, _stream_subsample_layer
// :1055-1068; transformers Gemma4AudioSubSampleConvProjectionLayer,
// models/gemma4/modeling_gemma4.py:317-372): conv0 (1 -> 128 channels) +
// LayerNorm(128) + ReLU over [cached mel row | 8 new rows], then conv1
// (128 -> C1) + LayerNorm(C1) + ReLU over [cached conv0 row | 4 new rows].
// conv0 is [256 positions x 16 (9) taps] x [16 x 128] on mma.sync fp16 tiles;
// conv1 is an implicit GEMM [64 positions x 1152] x [1152 x C1] on mma.sync
// bf16 tiles; both accumulate in fp32.  The output is the bf16 input of the input projection.
#include "common.cuh"
#include "listener.h"

namespace lb {
namespace {

constexpr int kFrames = 8;
constexpr int kWin = 320;
constexpr int kBins = 257;

struct MelArgs {
  const int* counts;
  const int *row_slot, *row_reason;
  const SlotMeta* row_meta;
  const float* pcm;    // [rows][1280]
  float* tail;         // [S][2][160]
  float* mel;          // [rows][8][128]
  const float *window, *cos_tab, *sin_tab, *filters;  // [320], [512], [512], [257][128]
  const int2* filter_range;                          // [128] (k_lo, k_hi)
  // Stand-alone form (counts == nullptr): n_static rows, each with its own
  // caller-held tail [rows][160] (ext_tail_in, nullptr = a fresh stream) and
  // the new tails written to ext_tail_out; no slot state is touched.
  int n_static;
  const float* ext_tail_in;
  float* ext_tail_out;
};

// One complex multiply-free radix-4 DFT in place: (x0, x1, x2, x3) ->
// (X0, X1, X2, X3) with W4 = exp(-2 pi i / 4) = -i.
__device__ __forceinline__ void dft4(float& r0, float& i0, float& r1, float& i1, float& r2, float& i2, float& r3,
                                     float& i3) {
  const float t0r = r0 + r2, t0i = i0 + i2, t1r = r0 - r2, t1i = i0 - i2;
  const float t2r = r1 + r3, t2i = i1 + i3, t3r = r1 - r3, t3i = i1 - i3;
  r0 = t0r + t2r;
  i0 = t0i + t2i;
  r2 = t0r - t2r;
  i2 = t0i - t2i;
  r1 = t1r + t3i;  // t1 - i t3
  i1 = t1i - t3r;
  r3 = t1r - t3i;  // t1 + i t3
  i3 = t1i + t3r;
}

// 16-point DFT in registers, natural order in and out, as 4 x 4: radix-4 DFTs
// over n1 of x[4 n1 + n2], twiddles W16^(n2 k1), radix-4 DFTs over n2.
// Twiddles W16^j = W512^(32 j) come from the exact 512-entry table.
__device__ __forceinline__ void dft16(float (&re)[16], float (&im)[16], const float* __restrict__ ct,
                                      const float* __restrict__ st) {
#pragma unroll
  for (int n2 = 0; n2 < 4; ++n2) dft4(re[n2], im[n2], re[4 + n2], im[4 + n2], re[8 + n2], im[8 + n2], re[12 + n2], im[12 + n2]);
  // element 4 k1 + n2 now holds A[n2][k1]
#pragma unroll
  for (int n2 = 1; n2 < 4; ++n2)
#pragma unroll
    for (int k1 = 1; k1 < 4; ++k1) {
      const int j = n2 * k1;  // 1..9
      const float wr = __ldg(ct + 32 * j), wi = -__ldg(st + 32 * j);
      const float ar = re[4 * k1 + n2], ai = im[4 * k1 + n2];
      re[4 * k1 + n2] = ar * wr - ai * wi;
      im[4 * k1 + n2] = ar * wi + ai * wr;
    }
  float orr[16], oi[16];
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) {
    float a0 = re[4 * k1], b0 = im[4 * k1], a1 = re[4 * k1 + 1], b1 = im[4 * k1 + 1];
    float a2 = re[4 * k1 + 2], b2 = im[4 * k1 + 2], a3 = re[4 * k1 + 3], b3 = im[4 * k1 + 3];
    dft4(a0, b0, a1, b1, a2, b2, a3, b3);  // over n2 -> k2
    orr[k1] = a0, oi[k1] = b0;
    orr[k1 + 4] = a1, oi[k1 + 4] = b1;
    orr[k1 + 8] = a2, oi[k1 + 8] = b2;
    orr[k1 + 12] = a3, oi[k1 + 12] = b3;
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    re[k] = orr[k];
    im[k] = oi[k];
  }
}

// |X[k]|, k = 0..256, of the 512-point real DFT of each frame (zero-padded from
// 320 samples), computed as a 256-point complex FFT of z[m] = x[2m] + i x[2m+1]
// followed by the real-input split X[k] = E[k] + W^k O[k] with
// E = (Z[k] + conj Z[256-k]) / 2, O = (Z[k] - conj Z[256-k]) / 2i and
// W = exp(-2 pi i / 512).  The 256-point FFT is the four-step 16 x 16 form:
// with m = 16 a + b and k = k1 + 16 k2,
//   Z[k1 + 16 k2] = sum_b W16^(b k2) W256^(b k1) sum_a z[16 a + b] W16^(a k1),
// i.e. 16-point DFTs in registers (one thread per frame and column), a twiddle,
// one padded shared-memory transpose, and 16-point DFTs again.  Exact twiddles
// cos/sin(2 pi j / 512) from the table; fp32 throughout.
__global__ void __launch_bounds__(256) mel_kernel(MelArgs a) {
  pdl_wait();  // first: nothing of the previous kernel is read or written before it
  pdl_trigger();
  const int row = blockIdx.x;
  constexpr int kSig = kTail + kPcm;                // padded signal [tail | pcm]
  __shared__ __align__(16) float sig[kSig];         // phases 0-1
  __shared__ float yr[kFrames][16][17], yi[kFrames][16][17];  // after the first DFTs
  __shared__ float zr[kFrames][256], zi[kFrames][256];        // natural-order spectrum
  float (*mag)[kBins + 3] = reinterpret_cast<float (*)[kBins + 3]>(&yr[0][0][0]);  // reuses yr/yi
  static_assert(sizeof(yr) + sizeof(yi) >= sizeof(float) * kFrames * (kBins + 3), "mag fits in yr/yi");
  // row tables (in bounds for every row of the bucket) read with the live count
  const bool ext = a.counts == nullptr;
  const int n_rows = ext ? a.n_static : a.counts[0];
  const int slot = ext ? 0 : a.row_slot[row];
  const int parity = ext ? 0 : (a.row_meta[row].pos >> 1) & 1;
  const int reason = ext ? 0 : a.row_reason[row];
  if (row >= n_rows) return;
  // A new session or identity (identity_reset) and an explicit reset start
  // from a zero tail; across a cursor gap the session keeps its tail, as the
  // reference frontend keeps it in the session state.
  const bool fresh = ext ? a.ext_tail_in == nullptr : (reason == 3 || reason == 1);
  const float* tail_in = ext ? (a.ext_tail_in ? a.ext_tail_in + static_cast<size_t>(row) * kTail : nullptr)
                             : a.tail + (static_cast<size_t>(slot) * 2 + parity) * kTail;
  const float* pcm = a.pcm + static_cast<size_t>(row) * kPcm;
  const int tid = threadIdx.x;
  // ---- phase 0: [tail | pcm] into shared memory (16-byte loads), new tail out
  for (int i = tid; i < kSig / 4; i += blockDim.x) {
    float4 v;
    if (i < kTail / 4) {
      v = fresh ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(reinterpret_cast<const float4*>(tail_in) + i);
    } else {
      v = __ldg(reinterpret_cast<const float4*>(pcm) + (i - kTail / 4));
    }
    reinterpret_cast<float4*>(sig)[i] = v;
  }
  float* tail_out = ext ? a.ext_tail_out + static_cast<size_t>(row) * kTail
                       : a.tail + (static_cast<size_t>(slot) * 2 + (parity ^ 1)) * kTail;
  for (int i = tid; i < kTail / 4; i += blockDim.x)
    reinterpret_cast<float4*>(tail_out)[i] = __ldg(reinterpret_cast<const float4*>(pcm) + (kPcm - kTail) / 4 + i);
  __syncthreads();
  // ---- phase 1: thread (f, b) -> Y[k1] = sum_a z[16 a + b] W16^(a k1), times
  // W256^(b k1); z[m] = 0 for m >= 160 (samples past the 320-sample window).
  // The windowed product is formed in fp32 as the reference's float32 NumPy does.
  if (tid < kFrames * 16) {
    const int f = tid >> 4, b = tid & 15;
    float re[16], im[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      if (q < 10) {
        const int n = 32 * q + 2 * b;  // < 320
        re[q] = sig[f * 160 + n] * __ldg(a.window + n);
        im[q] = sig[f * 160 + n + 1] * __ldg(a.window + n + 1);
      } else {
        re[q] = 0.f;
        im[q] = 0.f;
      }
    }
    dft16(re, im, a.cos_tab, a.sin_tab);
#pragma unroll
    for (int k1 = 0; k1 < 16; ++k1) {
      const int j = 2 * b * k1;  // W256^(b k1) = W512^(2 b k1), 2 b k1 <= 450
      const float wr = __ldg(a.cos_tab + j), wi = -__ldg(a.sin_tab + j);
      yr[f][k1][b] = re[k1] * wr - im[k1] * wi;
      yi[f][k1][b] = re[k1] * wi + im[k1] * wr;
    }
  }
  __syncthreads();
  // ---- phase 2: thread (f, k1) -> Z[k1 + 16 k2] = sum_b Y'[b][k1] W16^(b k2)
  if (tid < kFrames * 16) {
    const int f = tid >> 4, k1 = tid & 15;
    float re[16], im[16];
#pragma unroll
    for (int bb = 0; bb < 16; ++bb) {
      re[bb] = yr[f][k1][bb];
      im[bb] = yi[f][k1][bb];
    }
    dft16(re, im, a.cos_tab, a.sin_tab);
#pragma unroll
    for (int k2 = 0; k2 < 16; ++k2) {
      zr[f][k1 + 16 * k2] = re[k2];
      zi[f][k1 + 16 * k2] = im[k2];
    }
  }
  __syncthreads();
  // ---- real-input split -> magnitudes of bins 0..256 (mag reuses yr/yi)
  for (int o = tid; o < kFrames * kBins; o += blockDim.x) {
    const int f = o / kBins, k = o % kBins;
    const int k1 = k & 255, k2 = (256 - k) & 255;
    const float zkr = zr[f][k1], zki = zi[f][k1];
    const float ckr = zr[f][k2], cki = -zi[f][k2];  // conj Z[256 - k]
    const float er = 0.5f * (zkr + ckr), ei = 0.5f * (zki + cki);
    const float orr = 0.5f * (zki - cki), oi = -0.5f * (zkr - ckr);  // (Z - conj Z') / 2i
    const float wr = __ldg(a.cos_tab + k), wi = -__ldg(a.sin_tab + k);  // exp(-2 pi i k / 512)
    const float xr = er + (orr * wr - oi * wi), xi = ei + (orr * wi + oi * wr);
    mag[f][k] = sqrtf(xr * xr + xi * xi);
  }
  __syncthreads();
  // mel filterbank (sparse row ranges) + log
  float* out = a.mel + static_cast<size_t>(row) * kFrames * kMelBins;
  for (int o = tid; o < kFrames * kMelBins; o += blockDim.x) {
    const int f = o / kMelBins, m = o % kMelBins;
    const int2 r = a.filter_range[m];
    float acc = 0.0f;
    for (int k = r.x; k < r.y; ++k) acc = fmaf(mag[f][k], a.filters[k * kMelBins + m], acc);
    out[o] = logf(acc + 1e-3f);
  }
}

// ------------------------------------------------------------ subsampler
constexpr int kF0 = 64;        // conv0 output frequencies
constexpr int kCiPad = 136;    // channel stride of the conv1 input tile (16-byte rows for ldmatrix)
constexpr int kK1 = 9 * 128;   // conv1 reduction length
constexpr int kK1Pad = kK1 + 8;
constexpr int kSubThreads = 256;

struct SubArgs {
  const int* counts;
  const int *row_slot, *row_mask;
  const SlotMeta* row_meta;
  const float* mel;             // [rows][8][128]
  float* mel_prev;              // [S][2][128]
  __nv_bfloat16* sub_prev;      // [S][2][64][128]
  const float *w0, *ln0;        // [128][9], [128]
  const __nv_bfloat16* w1;      // [C1][kK1Pad]
  const float* ln1;             // [C1]
  __nv_bfloat16* sub_in;        // [tok][32 * C1]  index f * C1 + c
  float eps;
  int c1;                       // conv1 output channels (32)
  bool f16;                     // sub_in holds fp16 (int8-weight GEMM input) instead of bf16
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_f16x2(float x, float y) {
  const __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// C1 = 32 output channels (validated at create): 8 warps = 4 position tiles x 2 channel halves.
__global__ void __launch_bounds__(kSubThreads, 1) subsample_kernel(SubArgs a) {
  pdl_wait();  // first: nothing of the previous kernel is read or written before it
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sp = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                           ~static_cast<uintptr_t>(127));
  __nv_bfloat16* w1s = reinterpret_cast<__nv_bfloat16*>(sp);           // [32][kK1Pad]
  __nv_bfloat16* xin = w1s + 32 * kK1Pad;                              // [5][66][kCiPad]
  float* w0s = reinterpret_cast<float*>(xin + 5 * 66 * kCiPad);        // [128][12] (unused)
  float* ln0s = w0s + 128 * 12;                                        // [128]
  float* mels = ln0s + 128;                                            // [9][130]
  float* c1out = mels + 9 * 130;                                       // [64][33]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * kK1Pad / 8; i += blockDim.x)
    reinterpret_cast<int4*>(w1s)[i] = reinterpret_cast<const int4*>(a.w1)[i];
  for (int i = tid; i < 128; i += blockDim.x) ln0s[i] = a.ln0[i];
  // zero the frequency padding columns of the conv1 input once (never written)
  for (int i = tid; i < 5 * 2 * kCiPad; i += blockDim.x) {
    const int r = i / (2 * kCiPad), side = (i / kCiPad) & 1, c = i % kCiPad;
    xin[(r * 66 + (side ? 65 : 0)) * kCiPad + c] = __float2bfloat16_rn(0.0f);
  }
  // conv0 weights as m16n8k16 B fragments (taps 9..15 zero), held for every row:
  // n-tile nt covers channels nt*8 .. +7; this lane's column is channel nt*8 + g
  uint32_t w0b[16][2];
  {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float* wr = a.w0 + (nt * 8 + g) * 9;
      auto tap = [&](int k) { return k < 9 ? wr[k] : 0.0f; };
      w0b[nt][0] = pack_f16x2(tap(2 * tq), tap(2 * tq + 1));
      w0b[nt][1] = pack_f16x2(tap(2 * tq + 8), tap(2 * tq + 9));
    }
  }
  // the frequency padding columns of the mel tile are zero for every row
  for (int i = tid; i < 9 * 2; i += blockDim.x) mels[(i >> 1) * 130 + ((i & 1) ? 129 : 0)] = 0.0f;
  const int n_rows = a.counts[0];
  // row tables of this CTA's first row; each iteration fetches the next row's
  // with its own data loads, so a row costs one memory round trip
  int row = blockIdx.x;
  int slot = 0, mask = 0;
  SlotMeta m{};
  if (row < n_rows) {
    slot = a.row_slot[row];
    m = a.row_meta[row];
    mask = a.row_mask[row];
  }
  for (; row < n_rows; row += gridDim.x) {
    __syncthreads();
    const int parity = (m.pos >> 1) & 1;
    const bool mel_prev_ok = (m.flags & 1) != 0;
    const bool sub_prev_ok = (m.flags & 2) != 0;
    const float* mel_in = a.mel + static_cast<size_t>(row) * 8 * kMelBins;
    const float* mp_in = a.mel_prev + (static_cast<size_t>(slot) * 2 + parity) * kMelBins;
    float* mp_out = a.mel_prev + (static_cast<size_t>(slot) * 2 + (parity ^ 1)) * kMelBins;
    const __nv_bfloat16* sp_in = a.sub_prev + (static_cast<size_t>(slot) * 2 + parity) * kF0 * 128;
    // ---- every global load of this row in flight together: the 8 new mel rows
    // (4 floats per thread), the cached mel row (threads 0..31), the cached
    // conv0 row (16 KB: four 16-byte chunks per thread) and the next row's tables
    float4 mv = __ldg(reinterpret_cast<const float4*>(mel_in) + tid);  // 256 x 4 = 8 x 128
    float4 pv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < 32 && mel_prev_ok) pv = __ldg(reinterpret_cast<const float4*>(mp_in) + tid);
    int4 sv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      sv[q] = sub_prev_ok ? __ldg(reinterpret_cast<const int4*>(sp_in) + tid + q * kSubThreads)
                          : make_int4(0, 0, 0, 0);
    }
    const int next = row + gridDim.x;
    int n_slot = slot, n_mask = mask;
    SlotMeta n_m = m;
    if (next < n_rows) {
      n_slot = a.row_slot[next];
      n_m = a.row_meta[next];
      n_mask = a.row_mask[next];
    }
    // masked mel rows (row 0 = cached row), frequency-padded by one zero each side
    {
      const int r = tid >> 5, f4 = (tid & 31) * 4;  // new mel row r (0..7), frequencies f4..f4+3
      const bool keep = (mask >> r) & 1;
      float* dst = mels + (r + 1) * 130 + 1 + f4;
      dst[0] = keep ? mv.x : 0.f;
      dst[1] = keep ? mv.y : 0.f;
      dst[2] = keep ? mv.z : 0.f;
      dst[3] = keep ? mv.w : 0.f;
      if (tid < 32) {
        float* d0 = mels + 1 + tid * 4;
        d0[0] = pv.x;
        d0[1] = pv.y;
        d0[2] = pv.z;
        d0[3] = pv.w;
      }
      // staged mel_prev = last mel row (unmasked)
      if (r == 7) *reinterpret_cast<float4*>(mp_out + f4) = mv;
    }
    // cached conv0 row -> conv1 input row 0 (16-byte chunk c = 8 channels of one frequency)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = tid + q * kSubThreads;
      const int fq = c >> 4, c8 = (c & 15) * 8;
      uint2* dst = reinterpret_cast<uint2*>(xin + (0 * 66 + fq + 1) * kCiPad + c8);
      dst[0] = make_uint2(static_cast<uint32_t>(sv[q].x), static_cast<uint32_t>(sv[q].y));
      dst[1] = make_uint2(static_cast<uint32_t>(sv[q].z), static_cast<uint32_t>(sv[q].w));
    }
    __syncthreads();
    // ---- conv0 + LN(128) + ReLU on the tensor cores: D[pos][ch] = sum_tap A[pos][tap] W0[ch][tap]
    // as one m16n8k16 per (16 positions, 8 channels) -- the 9 taps padded to 16,
    // fp16 operands (the mel rounded to fp16; the bf16-valued weights exactly),
    // fp32 accumulation.  Warp w owns time row t = w/2 and frequencies
    // (w&1)*32 .. +31 (two 16-position m-tiles); each position's 128 channels
    // sit in one lane quad, so the LayerNorm statistics are two quad shuffles.
    __nv_bfloat16* sp_out = a.sub_prev + (static_cast<size_t>(slot) * 2 + (parity ^ 1)) * kF0 * 128;
    {
      const int t = warp >> 1;
      const int g = lane >> 2, tq = lane & 3;
      const bool keep = (mask >> (2 * t)) & 1;  // mask0 = mask[::2]
      // mel value feeding tap k of position (t, f): rows 2t..2t+2, padded columns 2f..2f+2
      auto xval = [&](int f, int k) {
        return k < 9 ? mels[(2 * t + k / 3) * 130 + 2 * f + k % 3] : 0.0f;
      };
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const int f0 = (warp & 1) * 32 + half * 16;
        const int fa = f0 + g, fb = fa + 8;
        const uint32_t a0 = pack_f16x2(xval(fa, 2 * tq), xval(fa, 2 * tq + 1));
        const uint32_t a1 = pack_f16x2(xval(fb, 2 * tq), xval(fb, 2 * tq + 1));
        const uint32_t a2 = pack_f16x2(xval(fa, 2 * tq + 8), xval(fa, 2 * tq + 9));
        const uint32_t a3 = pack_f16x2(xval(fb, 2 * tq + 8), xval(fb, 2 * tq + 9));
        float acc[16][4];
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
          mma_f16_16816(acc[nt], a0, a1, a2, a3, w0b[nt][0], w0b[nt][1]);
        }
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          sa += acc[nt][0] + acc[nt][1];
          sb += acc[nt][2] + acc[nt][3];
        }
        sa += __shfl_xor_sync(0xffffffffu, sa, 1);
        sa += __shfl_xor_sync(0xffffffffu, sa, 2);
        sb += __shfl_xor_sync(0xffffffffu, sb, 1);
        sb += __shfl_xor_sync(0xffffffffu, sb, 2);
        const float ma = sa * (1.0f / 128.0f), mb = sb * (1.0f / 128.0f);
        float va = 0.f, vb = 0.f;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          va = fmaf(acc[nt][0] - ma, acc[nt][0] - ma, fmaf(acc[nt][1] - ma, acc[nt][1] - ma, va));
          vb = fmaf(acc[nt][2] - mb, acc[nt][2] - mb, fmaf(acc[nt][3] - mb, acc[nt][3] - mb, vb));
        }
        va += __shfl_xor_sync(0xffffffffu, va, 1);
        va += __shfl_xor_sync(0xffffffffu, va, 2);
        vb += __shfl_xor_sync(0xffffffffu, vb, 1);
        vb += __shfl_xor_sync(0xffffffffu, vb, 2);
        const float ra = rsqrtf(va * (1.0f / 128.0f) + a.eps), rbv = rsqrtf(vb * (1.0f / 128.0f) + a.eps);
        __nv_bfloat16* xa_row = xin + ((1 + t) * 66 + fa + 1) * kCiPad;
        __nv_bfloat16* xb_row = xin + ((1 + t) * 66 + fb + 1) * kCiPad;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          const int ch = nt * 8 + 2 * tq;
          const float2 lw = *reinterpret_cast<const float2*>(ln0s + ch);
          const __nv_bfloat162 oa = __floats2bfloat162_rn(fmaxf((acc[nt][0] - ma) * ra * lw.x, 0.0f),
                                                          fmaxf((acc[nt][1] - ma) * ra * lw.y, 0.0f));
          const __nv_bfloat162 ob = __floats2bfloat162_rn(fmaxf((acc[nt][2] - mb) * rbv * lw.x, 0.0f),
                                                          fmaxf((acc[nt][3] - mb) * rbv * lw.y, 0.0f));
          const __nv_bfloat162 z = __floats2bfloat162_rn(0.f, 0.f);
          *reinterpret_cast<__nv_bfloat162*>(xa_row + ch) = keep ? oa : z;
          *reinterpret_cast<__nv_bfloat162*>(xb_row + ch) = keep ? ob : z;
          if (t == 3) {
            *reinterpret_cast<__nv_bfloat162*>(sp_out + fa * 128 + ch) = oa;
            *reinterpret_cast<__nv_bfloat162*>(sp_out + fb * 128 + ch) = ob;
          }
        }
      }
    }
    __syncthreads();
    // ---- conv1 as implicit GEMM on mma.sync: D[pos][co] = sum_k A[pos][k] W1[co][k]
    {
      const int pt = warp & 3;          // position tile: 16 positions
      const int ch = warp >> 2;         // channel half: 16 channels = 2 n-tiles
      const int g = lane >> 2, tq = lane & 3;
      float acc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
      const int p_lo = pt * 16 + g, p_hi = p_lo + 8;
      // ldmatrix.x4 row addresses: lane L feeds row L%8 of matrix L/8.  A: the
      // 16 positions of this tile (matrices 0/1: positions +0..7 / +8..15 at
      // k 0..7, matrices 2/3: the same at k 8..15); B: output channels
      // ch*16 + 0..7 (matrices 0/1: k 0..7 / 8..15) and + 8..15 (matrices 2/3).
      // Per k-step only the tap / channel-chunk offset changes (an immediate).
      const int mi = lane >> 3, mr = lane & 7;
      const int pa = pt * 16 + mr + (mi & 1) * 8;
      const uint32_t a_lane = smem_u32(xin + ((2 * (pa >> 5)) * 66 + 2 * (pa & 31)) * kCiPad + (mi >> 1) * 8);
      const uint32_t b_lane = smem_u32(w1s + (ch * 16 + (mi >> 1) * 8 + mr) * kK1Pad + (mi & 1) * 8);
#pragma unroll
      for (int ks = 0; ks < kK1 / 16; ++ks) {
        const int tap = ks >> 3, ci0 = (ks & 7) * 16;
        const int i = tap / 3, j = tap % 3;
        uint32_t af[4], bf[4];
        ldsm_x4(a_lane + ((i * 66 + j) * kCiPad + ci0) * 2, af[0], af[1], af[2], af[3]);
        ldsm_x4(b_lane + ks * 32, bf[0], bf[1], bf[2], bf[3]);
        mma_bf16_16816(acc[0], af, bf[0], bf[1]);
        mma_bf16_16816(acc[1], af, bf[2], bf[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int co = ch * 16 + nt * 8 + 2 * tq;
        c1out[p_lo * 33 + co] = acc[nt][0];
        c1out[p_lo * 33 + co + 1] = acc[nt][1];
        c1out[p_hi * 33 + co] = acc[nt][2];
        c1out[p_hi * 33 + co + 1] = acc[nt][3];
      }
    }
    __syncthreads();
    // ---- LN(C1) + ReLU, write [token t][f * C1 + c] bf16
    if (tid < 64) {
      const int p = tid, t = p >> 5, fq = p & 31;
      float mean = 0.f;
      for (int c = 0; c < 32; ++c) mean += c1out[p * 33 + c];
      mean *= (1.0f / 32.0f);
      float var = 0.f;
      for (int c = 0; c < 32; ++c) {
        const float dv = c1out[p * 33 + c] - mean;
        var += dv * dv;
      }
      const float rstd = rsqrtf(var * (1.0f / 32.0f) + a.eps);
      __nv_bfloat16* o = a.sub_in + (static_cast<size_t>(row) * 2 + t) * (32 * 32) + fq * 32;
      for (int c = 0; c < 32; c += 2) {
        const float y0 = fmaxf((c1out[p * 33 + c] - mean) * rstd * a.ln1[c], 0.f);
        const float y1 = fmaxf((c1out[p * 33 + c + 1] - mean) * rstd * a.ln1[c + 1], 0.f);
        *reinterpret_cast<uint32_t*>(o + c) = act_bits2(y0, y1, a.f16);
      }
    }
    slot = n_slot;
    m = n_m;
    mask = n_mask;
  }
}

constexpr size_t kSubSmem = 128 + 32 * kK1Pad * 2 + 5 * 66 * kCiPad * 2 + 128 * 12 * 4 + 128 * 4 +
                            9 * 130 * 4 + 64 * 33 * 4;

}  // namespace

cudaError_t launch_mel(Ctx& c, int rows_cap, int input_kind, cudaStream_t s) {
  if (input_kind != LB_INPUT_PCM) return cudaSuccess;  // mel supplied by the caller
  MelArgs a = {};
  a.counts = c.dev_counts;
  a.row_slot = c.row_slot;
  a.row_reason = c.row_reason;
  a.row_meta = c.row_meta;
  a.pcm = c.in_pcm;
  a.tail = c.pcm_tail;
  a.mel = c.in_mel;
  a.window = c.fe_window;
  a.cos_tab = c.fe_cos;
  a.sin_tab = c.fe_sin;
  a.filters = c.fe_filters;
  a.filter_range = c.fe_range;
  launch_kernel(c.pdl_all, mel_kernel, dim3(rows_cap), dim3(256), 0, s, a);
  return cudaGetLastError();
}

cudaError_t launch_mel_standalone(Ctx& c, int n, const float* pcm, const float* tail_in, float* tail_out,
                                  float* mel, cudaStream_t s) {
  MelArgs a = {};
  a.counts = nullptr;
  a.n_static = n;
  a.pcm = pcm;
  a.ext_tail_in = tail_in;
  a.ext_tail_out = tail_out;
  a.mel = mel;
  a.window = c.fe_window;
  a.cos_tab = c.fe_cos;
  a.sin_tab = c.fe_sin;
  a.filters = c.fe_filters;
  a.filter_range = c.fe_range;
  mel_kernel<<<n, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t frontend_init_attributes() {
  return cudaFuncSetAttribute(subsample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSubSmem));
}

cudaError_t launch_subsample(Ctx& c, int rows_cap, cudaStream_t s) {
  SubArgs a;
  a.counts = c.dev_counts;
  a.row_slot = c.row_slot;
  a.row_mask = c.row_mask;
  a.row_meta = c.row_meta;
  a.mel = c.in_mel;
  a.mel_prev = c.mel_prev;
  a.sub_prev = c.sub_prev;
  a.w0 = c.w.conv0;
  a.ln0 = c.w.ln0;
  a.w1 = c.w.conv1;
  a.ln1 = c.w.ln1;
  a.sub_in = c.sub_in;
  a.f16 = c.f16_acts != 0;
  a.eps = c.cfg.rms_eps;
  a.c1 = c.cfg.sub_ch1;
  int grid = rows_cap < c.num_sms ? rows_cap : c.num_sms;
  launch_kernel(c.pdl_all, subsample_kernel, dim3(grid), dim3(kSubThreads), kSubSmem, s, a);
  return cudaGetLastError();
}

size_t subsample_smem_bytes() { return kSubSmem; }

}  // namespace lb
