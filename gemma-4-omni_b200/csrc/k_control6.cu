// Batched Control6 policy head over native listener hidden rows.
//
// Restates the tensor part of GemmaNativeControl6BatchPolicy.step_batch
// (duplex_kernel/gemma_native_control6_batch_policy.py:853-893) over
// NativeControl6LoRA.forward (training/duplex_qlora/native_control6.py:157-197):
//   base   = bf16(base_rows . bf16(h))                  (6 tied LM-head rows, bf16 product)
//   delta  = scaling * B (A [h ; phase])                (rank-r LoRA in fp32, phase: 4 values)
//   logits = base + delta                               (fp32)
//   raw = argmax logits; selected = argmax over the row's legal actions;
//   confidence = softmax(legal logits)[selected]; finite = all logits finite.
// One CTA per row: the row's 1536 + 4 inputs are staged in shared memory, each
// warp reduces a share of the 6 + r dot products, and one thread finishes the
// row (the rank-r product, the argmaxes and the softmax).  Argmax ties go to
// the lowest index, as torch.argmax does.
#include <cmath>

#include "../../include/listener_b200.h"
#include "common.cuh"

namespace {

constexpr int kActions = 6;
constexpr int kHidden = 1536;
constexpr int kPhase = 4;
constexpr int kMaxRank = 64;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) control6_kernel(int n, const __nv_bfloat16* __restrict__ hidden,
                                                             int hidden_ld, const float* __restrict__ phase,
                                                             const uint8_t* __restrict__ legal,
                                                             const __nv_bfloat16* __restrict__ base_rows,
                                                             const float* __restrict__ lora_a,
                                                             const float* __restrict__ lora_b, int rank,
                                                             float scaling, float* __restrict__ logits_out,
                                                             float* __restrict__ packet_out) {
  __shared__ float x[kHidden + kPhase];
  __shared__ float dots[kActions + kMaxRank];
  const int row = blockIdx.x;
  if (row >= n) return;
  const __nv_bfloat16* h = hidden + static_cast<size_t>(row) * hidden_ld;
  for (int e = threadIdx.x; e < kHidden; e += blockDim.x) x[e] = __bfloat162float(h[e]);
  if (threadIdx.x < kPhase) x[kHidden + threadIdx.x] = phase ? phase[row * kPhase + threadIdx.x] : 0.0f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out = kActions + rank;
  for (int j = warp; j < n_out; j += kThreads / 32) {
    float acc = 0.0f;
    if (j < kActions) {
      const __nv_bfloat16* w = base_rows + static_cast<size_t>(j) * kHidden;
      for (int e = lane; e < kHidden; e += 32) acc = fmaf(__bfloat162float(w[e]), x[e], acc);
    } else {
      const float* w = lora_a + static_cast<size_t>(j - kActions) * (kHidden + kPhase);
      for (int e = lane; e < kHidden + kPhase; e += 32) acc = fmaf(w[e], x[e], acc);
    }
    acc = lb::warp_sum(acc);
    if (lane == 0) dots[j] = acc;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float logit[kActions];
  bool finite = true;
  for (int a = 0; a < kActions; ++a) {
    float d = 0.0f;
    for (int r = 0; r < rank; ++r) d = fmaf(lora_b[a * rank + r], dots[kActions + r], d);
    // the frozen rows' product is a bf16 tensor in the reference, then widened
    logit[a] = __bfloat162float(__float2bfloat16_rn(dots[a])) + d * scaling;
    finite = finite && isfinite(logit[a]);
    logits_out[row * kActions + a] = logit[a];
  }
  const int mask = legal ? legal[row] : 0x3F;
  int raw = 0, sel = 0;
  float sel_max = (mask & 1) ? logit[0] : -INFINITY;
  for (int a = 1; a < kActions; ++a) {
    if (logit[a] > logit[raw]) raw = a;
    const float v = ((mask >> a) & 1) ? logit[a] : -INFINITY;
    if (v > sel_max) {
      sel_max = v;
      sel = a;
    }
  }
  // softmax of the legal logits (illegal ones are -inf); an all-illegal row
  // gives NaN, as the reference's torch.softmax does
  float sum = 0.0f;
  for (int a = 0; a < kActions; ++a) sum += ((mask >> a) & 1) ? expf(logit[a] - sel_max) : 0.0f;
  const float conf = (((mask >> sel) & 1) ? expf(logit[sel] - sel_max) : 0.0f) / sum;
  float* pk = packet_out + row * 4;
  pk[0] = finite ? 1.0f : 0.0f;
  pk[1] = static_cast<float>(raw);
  pk[2] = static_cast<float>(sel);
  pk[3] = conf;
}

}  // namespace

extern "C" int lb_op_control6_head(int n, const void* hidden, int hidden_ld, const float* phase,
                                   const uint8_t* legal, const void* base_rows, const float* lora_a,
                                   const float* lora_b, int rank, float scaling, float* logits_out,
                                   float* packet_out, void* stream) {
  if (n < 0 || rank < 1 || rank > kMaxRank || hidden_ld < kHidden) return LB_ERR_INVALID_ARGUMENT;
  if (n == 0) return LB_OK;
  if (!hidden || !base_rows || !lora_a || !lora_b || !logits_out || !packet_out) return LB_ERR_INVALID_ARGUMENT;
  if (!std::isfinite(scaling)) return LB_ERR_INVALID_ARGUMENT;
  control6_kernel<<<n, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      n, static_cast<const __nv_bfloat16*>(hidden), hidden_ld, phase, legal,
      static_cast<const __nv_bfloat16*>(base_rows), lora_a, lora_b, rank, scaling, logits_out, packet_out);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}
