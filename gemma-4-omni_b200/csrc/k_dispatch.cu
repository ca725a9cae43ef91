// Tick-level row selection and ordering on the GPU (the two integer policies in
// front of the packer), restated from the reference, not translated:
//
//   snapshot: SharedListenerTickDispatcher._snapshot_ready_rows
//             (duplex_kernel/shared_listener_scheduler.py:486-535)
//     Walk the registered sessions in registration order; skip paused ones;
//     take the session's deferred frame if it has one, else the head of its
//     ingress queue; a frame enqueued after the tick deadline is kept as the
//     session's deferred frame for the next tick; every other frame becomes a
//     row.  Rows keep registration order.
//   order:    ListenerMicrobatchCoordinator._candidate_heads_locked /
//             _take_ready_locked (duplex_kernel/listener_microbatch.py:170-201)
//     Candidate heads (queue heads of sessions not in flight) with
//     ready_at <= now, sorted by (ready_at_ns, submission_order, session_id); a
//     single ready head waits until ready_at + coalesce window; the dispatch
//     reason is batch_full (every registered session ready), multiple_ready
//     (>= 2) or coalesce_deadline (one, after its window).
//
// Both run as one CTA of 1024 threads.  The snapshot is a block-wide prefix sum
// over per-session "emits a row" flags (registration order is the scan order).
// The order is a bitonic sort in shared memory on the key
// (ready_at_ns, submission_order, session_rank) with not-yet-ready heads keyed
// +inf; session_rank is the host's rank of the session id in string order, so
// the comparison equals the reference's tuple order.
#include "../../include/listener_b200.h"
#include "common.cuh"

namespace lb {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxSortHeads = 8192;  // 8192 x (8 + 8 + 4 + 4) B = 192 KB of shared memory

__device__ int scan_exclusive(int v, int* total, int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < (blockDim.x >> 5)) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;
  }
  __syncthreads();
  const int warp_prefix = warp > 0 ? sh[warp - 1] : 0;
  *total = sh[(blockDim.x >> 5) - 1];
  __syncthreads();
  return warp_prefix + x - v;
}

struct SnapshotArgs {
  int n;
  const uint8_t* paused;
  uint8_t* deferred_valid;
  long long *deferred_frame, *deferred_enqueue;
  const uint8_t* head_valid;
  const long long *head_frame, *head_enqueue;
  long long deadline;
  int* rows;             // registration index of each row
  long long* row_frame;  // its frame id
  uint8_t* popped;       // 1: the session's ingress head was consumed this tick
  int* n_rows;
};

__global__ void __launch_bounds__(kThreads) snapshot_kernel(SnapshotArgs a) {
  __shared__ int sh[32];
  int base = 0;
  for (int c0 = 0; c0 < a.n; c0 += kThreads) {
    const int i = c0 + threadIdx.x;
    int emit = 0;
    long long frame = 0;
    if (i < a.n) {
      uint8_t pop = 0;
      if (!a.paused[i]) {
        bool have = false;
        long long enq = 0;
        if (a.deferred_valid[i]) {
          have = true;
          frame = a.deferred_frame[i];
          enq = a.deferred_enqueue[i];
          a.deferred_valid[i] = 0;
        } else if (a.head_valid[i]) {
          have = true;
          pop = 1;
          frame = a.head_frame[i];
          enq = a.head_enqueue[i];
        }
        if (have) {
          if (enq > a.deadline) {  // consumed after the deadline: next tick's frame
            a.deferred_valid[i] = 1;
            a.deferred_frame[i] = frame;
            a.deferred_enqueue[i] = enq;
          } else {
            emit = 1;
          }
        }
      }
      a.popped[i] = pop;
    }
    int total = 0;
    const int r = scan_exclusive(emit, &total, sh);
    if (emit) {
      a.rows[base + r] = i;
      a.row_frame[base + r] = frame;
    }
    base += total;
  }
  if (threadIdx.x == 0) *a.n_rows = base;
}

struct OrderArgs {
  int n;
  const long long *ready_at, *order;
  const int* rank;
  long long now, coalesce;
  int registered;
  int *perm, *count, *reason;
};

__device__ __forceinline__ bool key_less(long long ra, long long oa, int ka, long long rb, long long ob,
                                         int kb) {
  if (ra != rb) return ra < rb;
  if (oa != ob) return oa < ob;
  return ka < kb;
}

__global__ void __launch_bounds__(kThreads) order_kernel(OrderArgs a) {
  extern __shared__ __align__(16) unsigned char smem_order[];
  int padded = 1;
  while (padded < a.n) padded <<= 1;
  long long* sr = reinterpret_cast<long long*>(smem_order);
  long long* so = sr + padded;
  int* sk = reinterpret_cast<int*>(so + padded);
  int* si = sk + padded;
  __shared__ int sh[32];
  constexpr long long kInf = 0x7fffffffffffffffll;
  int ready = 0;
  for (int i = threadIdx.x; i < padded; i += kThreads) {
    const bool live = i < a.n && a.ready_at[i] <= a.now;
    sr[i] = live ? a.ready_at[i] : kInf;
    so[i] = live ? a.order[i] : kInf;
    sk[i] = live ? a.rank[i] : 0x7fffffff;
    si[i] = i;
    ready += live ? 1 : 0;
  }
  // number of ready heads
  int total = 0;
  scan_exclusive(ready, &total, sh);
  // bitonic sort, ascending
  for (int k = 2; k <= padded; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < padded; i += kThreads) {
        const int p = i ^ j;
        if (p > i) {
          const bool up = (i & k) == 0;
          const bool gt = key_less(sr[p], so[p], sk[p], sr[i], so[i], sk[i]);  // [i] > [p]
          if (gt == up) {
            long long t = sr[i]; sr[i] = sr[p]; sr[p] = t;
            t = so[i]; so[i] = so[p]; so[p] = t;
            int u = sk[i]; sk[i] = sk[p]; sk[p] = u;
            u = si[i]; si[i] = si[p]; si[p] = u;
          }
        }
      }
      __syncthreads();
    }
  }
  // coalesce rule and dispatch reason (0: nothing dispatched)
  int count = total, reason = 0;
  if (total == 1 && a.now < sr[0] + a.coalesce) count = 0;
  if (count > 0) reason = total == a.registered ? 1 : total >= 2 ? 2 : 3;
  for (int i = threadIdx.x; i < count; i += kThreads) a.perm[i] = si[i];
  if (threadIdx.x == 0) {
    *a.count = count;
    *a.reason = reason;
  }
}

size_t order_smem_bytes(int n) {
  int padded = 1;
  while (padded < n) padded <<= 1;
  return static_cast<size_t>(padded) * (8 + 8 + 4 + 4);
}

cudaError_t ensure_order_attribute() {
  static unsigned long long done = 0;  // bit per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && (done >> dev) & 1ull) return cudaSuccess;
  e = cudaFuncSetAttribute(order_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(order_smem_bytes(kMaxSortHeads)));
  if (e == cudaSuccess && dev < 64) done |= 1ull << dev;
  return e;
}

}  // namespace
}  // namespace lb

extern "C" {

int lb_snapshot_ready_rows(int n_registered, const uint8_t* paused, uint8_t* deferred_valid,
                           int64_t* deferred_frame_id, int64_t* deferred_enqueue_ns,
                           const uint8_t* head_valid, const int64_t* head_frame_id,
                           const int64_t* head_enqueue_ns, int64_t deadline_ns, int32_t* rows_out,
                           int64_t* row_frame_id_out, uint8_t* popped_out, int32_t* n_rows_out,
                           void* stream) {
  if (n_registered < 0 || !n_rows_out) return LB_ERR_INVALID_ARGUMENT;
  if (n_registered > 0 && (!paused || !deferred_valid || !deferred_frame_id || !deferred_enqueue_ns ||
                           !head_valid || !head_frame_id || !head_enqueue_ns || !rows_out ||
                           !row_frame_id_out || !popped_out))
    return LB_ERR_INVALID_ARGUMENT;
  lb::SnapshotArgs a;
  a.n = n_registered;
  a.paused = paused;
  a.deferred_valid = deferred_valid;
  a.deferred_frame = reinterpret_cast<long long*>(deferred_frame_id);
  a.deferred_enqueue = reinterpret_cast<long long*>(deferred_enqueue_ns);
  a.head_valid = head_valid;
  a.head_frame = reinterpret_cast<const long long*>(head_frame_id);
  a.head_enqueue = reinterpret_cast<const long long*>(head_enqueue_ns);
  a.deadline = deadline_ns;
  a.rows = rows_out;
  a.row_frame = reinterpret_cast<long long*>(row_frame_id_out);
  a.popped = popped_out;
  a.n_rows = n_rows_out;
  lb::snapshot_kernel<<<1, lb::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int lb_order_ready_heads(int n_heads, const int64_t* ready_at_ns, const int64_t* submission_order,
                         const int32_t* session_rank, int64_t now_ns, int64_t coalesce_ns,
                         int n_registered, int32_t* perm_out, int32_t* count_out, int32_t* reason_out,
                         void* stream) {
  if (n_heads < 0 || n_heads > lb::kMaxSortHeads || !count_out || !reason_out)
    return n_heads > lb::kMaxSortHeads ? LB_ERR_CAPACITY : LB_ERR_INVALID_ARGUMENT;
  if (n_heads > 0 && (!ready_at_ns || !submission_order || !session_rank || !perm_out))
    return LB_ERR_INVALID_ARGUMENT;
  if (lb::ensure_order_attribute() != cudaSuccess) return LB_ERR_CUDA;
  lb::OrderArgs a;
  a.n = n_heads;
  a.ready_at = reinterpret_cast<const long long*>(ready_at_ns);
  a.order = reinterpret_cast<const long long*>(submission_order);
  a.rank = session_rank;
  a.now = now_ns;
  a.coalesce = coalesce_ns;
  a.registered = n_registered;
  a.perm = perm_out;
  a.count = count_out;
  a.reason = reason_out;
  lb::order_kernel<<<1, lb::kThreads, lb::order_smem_bytes(n_heads), static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

}  // extern "C"
