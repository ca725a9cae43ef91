// Per-kernel C-ABI entry points ("ops").  Each runs exactly one kernel of the
// listener step on caller-owned device buffers so the parity tests can check
// every kernel against the CPU oracle in isolation.  The step-level API that a
// serving process binds lives in api_step.cu.
#include <atomic>
#include <cmath>
#include <cstdint>

#include "../../include/listener_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace lb;

namespace lb {
cudaError_t gemm_init_attributes();
}

namespace {
constexpr int kMaxDevices = 64;
std::atomic<unsigned long long> g_attr_done{0};  // bit per device ordinal

// The GEMM kernels need their shared-memory limit raised once per device.  Two
// threads may both run the (idempotent) set-up; the bit is published with an
// atomic OR.
cudaError_t ensure_gemm_attributes(int dev) {
  if ((g_attr_done.load(std::memory_order_acquire) >> dev) & 1ull) return cudaSuccess;
  cudaError_t e = gemm_init_attributes();
  if (e == cudaSuccess) g_attr_done.fetch_or(1ull << dev, std::memory_order_acq_rel);
  return e;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }
}  // namespace

extern "C" {

int lb_op_gemm_clipped(const void* x, int x_ld, int m, int x_part_rows, const void* w, int w_int8,
                       const void* w_scale, const float* bias, int out_features, int k, void* out,
                       int ld_out, int out_mode, int act, int splits, int parts,
                       const float* out_bounds, const float* post_bounds, float* split_acc,
                       int* status_dev, void* stream) {
  if (!x || !w || !out || m <= 0 || out_features <= 0 || k <= 0) return LB_ERR_INVALID_ARGUMENT;
  if (w_int8 < 0 || w_int8 > 2 || (w_int8 && !w_scale)) return LB_ERR_INVALID_ARGUMENT;
  if (out_mode < 0 || out_mode > 2 || act < 0 || act > 1 || splits < 1) return LB_ERR_INVALID_ARGUMENT;
  // a split-K bf16 / fp32 output reduces through the caller's zeroed fp32
  // workspace and a finish pass (which leaves it zeroed)
  const bool split_ws = splits > 1 && out_mode != 2;
  if (split_ws && !split_acc) return LB_ERR_INVALID_ARGUMENT;
  // the activation and weight maps start on 16-byte boundaries and rows do not overlap
  if (x_ld < k || !aligned16(x) || !aligned16(w) || ld_out < out_features) return LB_ERR_INVALID_ARGUMENT;
  if (parts < 1 || parts > GemmParams::kMaxParts || out_features % (128 * parts) != 0 || x_part_rows < 0 ||
      (x_part_rows > 0 && (parts == 1 || x_part_rows < m)))
    return LB_ERR_INVALID_ARGUMENT;
  GemmParams p;
  bool finite = false;
  if (out_bounds) {
    for (int j = 0; j < parts; ++j) {
      p.part_lo[j] = out_bounds[2 * j];
      p.part_hi[j] = out_bounds[2 * j + 1];
      finite = finite || std::isfinite(p.part_lo[j]) || std::isfinite(p.part_hi[j]);
    }
    p.out_lo = p.part_lo[0];
    p.out_hi = p.part_hi[0];
  }
  if (post_bounds) {
    p.post_lo = post_bounds[0];
    p.post_hi = post_bounds[1];
    // the next-input clamp follows the activation of a bf16 output only
    if (out_mode != 0 && (std::isfinite(p.post_lo) || std::isfinite(p.post_hi))) return LB_ERR_INVALID_ARGUMENT;
  }
  // atomically accumulated partial sums cannot be clamped before they are summed
  if (out_mode == 2 && finite) return LB_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LB_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return LB_ERR_INVALID_ARGUMENT;
  if (ensure_gemm_attributes(dev) != cudaSuccess) return LB_ERR_CUDA;
  GemmPlan plan;
  int rc = gemm_prepare(&plan, w, w_int8, out_features, k, x, x_ld, m, split_ws ? split_acc : out,
                        split_ws ? out_features : ld_out, split_ws ? 2 : out_mode, false,
                        x_part_rows > 0 ? parts : 1, x_part_rows);
  if (rc) return rc == -3 ? LB_ERR_INVALID_ARGUMENT : LB_ERR_CUDA;
  p.m_static = m;
  p.w_scale = static_cast<const __half*>(w_scale);
  p.bias = bias;
  p.out = split_ws ? static_cast<void*>(split_acc) : out;
  p.ld_out = split_ws ? out_features : ld_out;
  p.out_mode = split_ws ? 2 : out_mode;
  p.act = act;
  p.status = status_dev;
  if (parts > 1) {
    p.part_o = out_features / parts;
    p.x_part_rows = x_part_rows;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = gemm_launch(plan, p, splits, s);
  if (e == cudaSuccess && split_ws) {
    FinalizeClip fc;
    fc.part_o = p.part_o;
    for (int j = 0; j < 3; ++j) {
      fc.lo[j] = parts > 1 ? p.part_lo[j] : p.out_lo;
      fc.hi[j] = parts > 1 ? p.part_hi[j] : p.out_hi;
    }
    fc.plo = p.post_lo;
    fc.phi = p.post_hi;
    e = launch_split_finish(nullptr, m, m, split_acc, out_features, act, out, ld_out, out_mode == 1, false, fc,
                            false, s);
  }
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int lb_op_gemm(const void* x, int x_ld, int m, const void* w, int w_int8, const void* w_scale,
               const float* bias, int out_features, int k, void* out, int ld_out, int out_mode,
               int act, int splits, int* status_dev, void* stream) {
  if (splits > 1 && out_mode != 2) return LB_ERR_INVALID_ARGUMENT;
  return lb_op_gemm_clipped(x, x_ld, m, 0, w, w_int8, w_scale, bias, out_features, k, out, ld_out,
                            out_mode, act, splits < 1 ? 1 : splits, 1, nullptr, nullptr, nullptr, status_dev,
                            stream);
}

}  // extern "C"
