// Per-kernel C-ABI entry points ("ops").  Each runs exactly one kernel of the
// listener step on caller-owned device buffers so the parity tests can check
// every kernel against the CPU oracle in isolation.  The step-level API that a
// serving process binds lives in api_step.cu.
#include "../../include/listener_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace lb;

namespace lb {
cudaError_t gemm_init_attributes();
}

namespace {
// The GEMM kernels need their shared-memory limit raised once per device.
cudaError_t ensure_gemm_attributes() {
  static unsigned long long done = 0;  // bit per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && (done >> dev) & 1ull) return cudaSuccess;
  e = gemm_init_attributes();
  if (e == cudaSuccess && dev < 64) done |= 1ull << dev;
  return e;
}
}  // namespace

extern "C" {

int lb_op_gemm(const void* x, int x_ld, int m, const void* w, int w_int8, const void* w_scale,
               const float* bias, int out_features, int k, void* out, int ld_out, int out_mode,
               int act, int splits, int* status_dev, void* stream) {
  if (!x || !w || !out || m <= 0) return LB_ERR_INVALID_ARGUMENT;
  if (w_int8 < 0 || w_int8 > 2 || (w_int8 && !w_scale)) return LB_ERR_INVALID_ARGUMENT;
  if (out_mode < 0 || out_mode > 2 || act < 0 || act > 1) return LB_ERR_INVALID_ARGUMENT;
  if (splits > 1 && out_mode != 2) return LB_ERR_INVALID_ARGUMENT;
  if (ensure_gemm_attributes() != cudaSuccess) return LB_ERR_CUDA;
  GemmPlan plan;
  int rc = gemm_prepare(&plan, w, w_int8, out_features, k, x, x_ld, m, out, ld_out, out_mode);
  if (rc) return rc == -3 ? LB_ERR_INVALID_ARGUMENT : LB_ERR_CUDA;
  GemmParams p;
  p.m_static = m;
  p.w_scale = static_cast<const __half*>(w_scale);
  p.bias = bias;
  p.out = out;
  p.ld_out = ld_out;
  p.out_mode = out_mode;
  p.act = act;
  p.status = status_dev;
  cudaError_t e = gemm_launch(plan, p, splits, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

}  // extern "C"
