// lb_op_gemm_splitk_scratch: the tcgen05 split-K GEMM with a bf16 output whose
// fp32 partial sums live in a fixed device array declared in this file, so a
// call allocates no device memory and the caller passes no accumulator.
//
// Scratch: g_splitk_scratch, kScratchFloats fp32 values (8 MiB) per device,
// one copy per device (the array is part of the library's device module).
// Its device address is resolved once per device with cudaGetSymbolAddress on
// the first call made while that device is current; that first call also
// raises the GEMM kernels' shared-memory limit, so it belongs before any
// stream capture.  Every call zeroes the [m, out_features] prefix it uses
// (the split-K partial sums are reduce-added into it), so calls that overlap
// on the GPU -- on two streams, or from two threads -- race on the one array.
#include <mutex>

#include "../../include/listener_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace lb;

namespace lb {
cudaError_t gemm_init_attributes();
}

namespace {

constexpr size_t kScratchFloats = size_t(1) << 21;  // 8 MiB of fp32 partial sums
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_splitk_scratch[kScratchFloats];

float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Once per device (that device current): the scratch array's address and the
// GEMM's shared-memory attribute.  Later calls only read the cached pointer.
int scratch_setup(int dev, float** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_splitk_scratch);
    if (e != cudaSuccess || p == nullptr) return LB_ERR_CUDA;
    e = gemm_init_attributes();
    if (e != cudaSuccess) return LB_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return LB_OK;
}

// out[t, o..o+7] = bf16(acc) (act 1: bf16(SiLU(bf16(acc)))), 8 outputs per thread.
// Writes nothing when the GEMM recorded an error (its sums are then partial).
__global__ void scratch_finalize_kernel(const float* __restrict__ acc, int m, int width,
                                        int ld_out, int act, const int* status,
                                        __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.y;
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (t >= m || o >= width) return;
  if (status && *status != 0) return;
  const float4* src = reinterpret_cast<const float4*>(acc + static_cast<size_t>(t) * width + o);
  const float4 a = src[0], b = src[1];
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = act == 1 ? silu_f(bf16_round(v[i])) : v[i];
  store8_act(out + static_cast<size_t>(t) * ld_out + o, v, false);
}

}  // namespace

extern "C" {

int lb_op_gemm_splitk_scratch(const void* x, int x_ld, int m, const void* w, int w_int8,
                              const void* w_scale, const float* bias, int out_features, int k,
                              void* out, int ld_out, int act, int splits, int* status_dev,
                              void* stream) {
  if (!x || !w || !out || m <= 0 || out_features <= 0 || k <= 0) return LB_ERR_INVALID_ARGUMENT;
  if (w_int8 < 0 || w_int8 > 2 || (w_int8 && !w_scale)) return LB_ERR_INVALID_ARGUMENT;
  if (act < 0 || act > 1 || splits < 1 || ld_out < out_features || ld_out % 8 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return LB_ERR_INVALID_ARGUMENT;
  // the activation and weight maps start on 16-byte boundaries and rows do not overlap
  if (x_ld < k || reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0)
    return LB_ERR_INVALID_ARGUMENT;
  if (out_features % 128 != 0 || k % 64 != 0) return LB_ERR_INVALID_ARGUMENT;
  const size_t need = static_cast<size_t>(m) * static_cast<size_t>(out_features);
  if (need > kScratchFloats) return LB_ERR_CAPACITY;  // m * out_features > 2^21
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LB_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return LB_ERR_INVALID_ARGUMENT;
  float* acc = nullptr;
  int rc = scratch_setup(dev, &acc);
  if (rc != LB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  GemmPlan plan;
  rc = gemm_prepare(&plan, w, w_int8, out_features, k, x, x_ld, m, acc, out_features, 2);
  if (rc) return rc == -3 ? LB_ERR_INVALID_ARGUMENT : LB_ERR_CUDA;
  GemmParams p;
  p.m_static = m;
  p.w_scale = static_cast<const __half*>(w_scale);
  p.bias = bias;
  p.out = acc;
  p.ld_out = out_features;
  p.out_mode = 2;  // fp32 reduce-add of each K split's partial product
  p.act = 0;       // SiLU needs the whole sum: applied by the finalize kernel
  p.status = status_dev;

  cudaError_t e = cudaMemsetAsync(acc, 0, need * sizeof(float), s);
  if (e == cudaSuccess) e = gemm_launch(plan, p, splits, s);
  if (e == cudaSuccess) {
    const int per_block = 128 * 8;
    dim3 grid((out_features + per_block - 1) / per_block, m);
    scratch_finalize_kernel<<<grid, 128, 0, s>>>(acc, m, out_features, ld_out, act, status_dev,
                                                 static_cast<__nv_bfloat16*>(out));
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

}  // extern "C"
