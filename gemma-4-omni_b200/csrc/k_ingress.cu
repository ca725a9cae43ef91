// GPU-resident listener ingress: per-session PCM rings on the device, the
// tick's row snapshot and the rows' PCM gather, with session join / leave /
// pause / resume applied as device-side events.
//
// It restates, for device-resident queues, the fixed-grid dispatcher's row
// selection (SharedListenerTickDispatcher._snapshot_ready_rows,
// duplex_kernel/shared_listener_scheduler.py:486-535) and its session
// bookkeeping (register_session / pause / unregister, :80-480): sessions are
// walked in registration order, paused ones are skipped, the oldest queued
// frame of each session becomes a row unless it was enqueued after the tick
// deadline, in which case it stays queued for the next tick (the reference
// moves it to its per-session "deferred" slot, which is taken before the
// queue on the next tick -- the same frame order).  Rows keep registration
// order.
//
// Device state (ring of R frames per session index s):
//   pcm [S][R][1280] f32, frame_id / enqueue_ns [S][R] i64, head / tail
//   counters, paused / active flags, the session's directory handle, and the
//   registration order (order[0 .. n_reg)).
// The host assigns session indices; an index released by a leave is not
// reused within the same event batch.  Each push carries at most one frame per
// session (a per-session stamp detects a second one); a frame that finds its
// session's ring full is refused with LB_DEV_INGRESS_OVERFLOW -- the ring is
// the bounded stand-in for the reference's unbounded queue, sized by the
// caller.  A tick emits at most max_rows rows; ready frames past that stay
// queued (registration order decides who waits).
#include <cstdio>
#include <vector>

#include "../../include/listener_b200.h"
#include "common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kPcm = 1280;
constexpr int kMaxEvents = 1024;

struct IngressDev {
  int S, R, max_rows;
  float* pcm;            // [S][R][kPcm]
  long long* frame_id;   // [S][R]
  long long* enqueue;    // [S][R]
  unsigned* head;        // [S] frames consumed
  unsigned* tail;        // [S] frames pushed
  unsigned char* paused; // [S]
  unsigned char* active; // [S]
  unsigned char* gone;   // [S] left in the current event batch
  int* handle;           // [S]
  long long* stamp;      // [S] last push call that wrote the session
  int* order;            // [S] registration order
  int* order_tmp;        // [S]
  int* n_reg;            // [1]
  int* status;           // [1]
  int* row_src;          // [max_rows] ring slot of each emitted row (s * R + idx)
};

__device__ int block_scan_excl(int v, int* total, int* sh) {
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
    int w = lane < (blockDim.x >> 5) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;
  }
  __syncthreads();
  const int prefix = warp > 0 ? sh[warp - 1] : 0;
  *total = sh[(blockDim.x >> 5) - 1];
  __syncthreads();
  return prefix + x - v;
}

// Events in order (one thread: a handful per tick), then the registration
// list is compacted (sessions that left) and the joins are appended in event
// order.
__global__ void __launch_bounds__(kThreads) ingress_events_kernel(IngressDev d, int n, const int* kind,
                                                                  const int* sess, const int* arg) {
  __shared__ int joins[kMaxEvents];
  __shared__ int n_joins;
  __shared__ int sh[32];
  if (threadIdx.x == 0) {
    int nj = 0;
    for (int e = 0; e < n; ++e) {
      const int s = sess[e];
      if (s < 0 || s >= d.S) {
        atomicOr(d.status, LB_DEV_BAD_HANDLE);
        continue;
      }
      switch (kind[e]) {
        case LB_INGRESS_JOIN:
          if (d.active[s] || d.gone[s]) {  // already registered, or its index was released in this batch
            atomicOr(d.status, LB_DEV_BAD_HANDLE);
            break;
          }
          d.active[s] = 1;
          d.paused[s] = 0;
          d.head[s] = d.tail[s] = 0;
          d.handle[s] = arg[e];
          joins[nj++] = s;
          break;
        case LB_INGRESS_LEAVE:
          if (!d.active[s]) {
            atomicOr(d.status, LB_DEV_BAD_HANDLE);
            break;
          }
          d.active[s] = 0;
          d.gone[s] = 1;
          d.head[s] = d.tail[s] = 0;  // queued frames are dropped with the session
          break;
        case LB_INGRESS_PAUSE:
          d.paused[s] = 1;
          break;
        case LB_INGRESS_RESUME:
          d.paused[s] = 0;
          break;
        default:
          atomicOr(d.status, LB_DEV_BAD_HANDLE);
      }
    }
    n_joins = nj;
  }
  __syncthreads();
  const int n_reg = *d.n_reg;
  int kept = 0;
  for (int base = 0; base < n_reg; base += blockDim.x) {
    const int k = base + threadIdx.x;
    int s = -1, keep = 0;
    if (k < n_reg) {
      s = d.order[k];
      keep = d.active[s] && !d.gone[s];
      // a session that joined in this batch is appended below, not kept here
      if (!d.active[s] || d.gone[s]) d.gone[s] = 0;
    }
    int tot;
    const int p = block_scan_excl(keep, &tot, sh);
    if (keep) d.order_tmp[kept + p] = s;
    kept += tot;
  }
  __syncthreads();
  for (int k = threadIdx.x; k < kept; k += blockDim.x) d.order[k] = d.order_tmp[k];
  __syncthreads();
  if (threadIdx.x == 0) {
    int m = kept;
    for (int j = 0; j < n_joins; ++j) {
      const int s = joins[j];
      if (d.active[s]) d.order[m++] = s;  // joined and still registered
      d.gone[s] = 0;
    }
    *d.n_reg = m;
  }
}

// One CTA per arrival: claim the session's next ring slot and copy the frame in.
__global__ void __launch_bounds__(256) ingress_push_kernel(IngressDev d, long long call, const int* sess,
                                                          const long long* frame_id, const long long* enqueue,
                                                          const float* pcm) {
  __shared__ int slot;
  const int i = blockIdx.x;
  const int s = sess[i];
  if (threadIdx.x == 0) {
    slot = -1;
    if (s < 0 || s >= d.S || !d.active[s]) {
      atomicOr(d.status, LB_DEV_BAD_HANDLE);
    } else if (static_cast<long long>(atomicExch(reinterpret_cast<unsigned long long*>(d.stamp + s),
                                                 static_cast<unsigned long long>(call))) == call) {
      atomicOr(d.status, LB_DEV_DUPLICATE_ROW);  // two frames of one session in one push
    } else if (d.tail[s] - d.head[s] >= static_cast<unsigned>(d.R)) {
      atomicOr(d.status, LB_DEV_INGRESS_OVERFLOW);
    } else {
      const int idx = static_cast<int>(d.tail[s] % static_cast<unsigned>(d.R));
      d.frame_id[static_cast<size_t>(s) * d.R + idx] = frame_id[i];
      d.enqueue[static_cast<size_t>(s) * d.R + idx] = enqueue[i];
      d.tail[s] += 1;
      slot = s * d.R + idx;
    }
  }
  __syncthreads();
  if (slot < 0) return;
  const float4* src = reinterpret_cast<const float4*>(pcm + static_cast<size_t>(i) * kPcm);
  float4* dst = reinterpret_cast<float4*>(d.pcm + static_cast<size_t>(slot) * kPcm);
  for (int e = threadIdx.x; e < kPcm / 4; e += blockDim.x) dst[e] = src[e];
}

// The tick's rows in registration order; emitted frames are consumed.
__global__ void __launch_bounds__(kThreads) ingress_tick_kernel(IngressDev d, long long deadline, int* row_session,
                                                                int* row_handle, long long* row_frame,
                                                                int* n_rows_out) {
  __shared__ int sh[32];
  const int n_reg = *d.n_reg;
  int emitted = 0;
  for (int base = 0; base < n_reg; base += blockDim.x) {
    const int k = base + threadIdx.x;
    int s = -1, idx = 0, ready = 0;
    if (k < n_reg) {
      s = d.order[k];
      if (!d.paused[s] && d.tail[s] != d.head[s]) {
        idx = static_cast<int>(d.head[s] % static_cast<unsigned>(d.R));
        ready = d.enqueue[static_cast<size_t>(s) * d.R + idx] <= deadline;
      }
    }
    int tot;
    const int p = emitted + block_scan_excl(ready, &tot, sh);
    if (ready && p < d.max_rows) {
      row_session[p] = s;
      row_handle[p] = d.handle[s];
      row_frame[p] = d.frame_id[static_cast<size_t>(s) * d.R + idx];
      d.row_src[p] = s * d.R + idx;
      d.head[s] += 1;
    }
    emitted += tot;
  }
  if (threadIdx.x == 0) *n_rows_out = emitted < d.max_rows ? emitted : d.max_rows;
}

__global__ void __launch_bounds__(256) ingress_gather_kernel(IngressDev d, const int* n_rows, float* row_pcm) {
  const int i = blockIdx.x;
  if (i >= *n_rows) return;
  const float4* src = reinterpret_cast<const float4*>(d.pcm + static_cast<size_t>(d.row_src[i]) * kPcm);
  float4* dst = reinterpret_cast<float4*>(row_pcm + static_cast<size_t>(i) * kPcm);
  for (int e = threadIdx.x; e < kPcm / 4; e += blockDim.x) dst[e] = src[e];
}

}  // namespace

struct lb_ingress {
  IngressDev d{};
  int device = 0;
  long long calls = 0;
  void* arena = nullptr;
};

extern "C" {

int lb_ingress_create(int max_sessions, int ring_frames, int max_rows, lb_ingress** out) {
  if (!out) return LB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (max_sessions < 1 || max_sessions > (1 << 20) || ring_frames < 1 || ring_frames > 256 || max_rows < 1)
    return LB_ERR_INVALID_ARGUMENT;
  lb_ingress* g = new lb_ingress();
  cudaGetDevice(&g->device);
  const size_t S = max_sessions, R = ring_frames, M = max_rows;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_pcm = take(S * R * kPcm * 4), o_fid = take(S * R * 8), o_enq = take(S * R * 8);
  const size_t o_head = take(S * 4), o_tail = take(S * 4), o_p = take(S), o_a = take(S), o_g = take(S);
  const size_t o_h = take(S * 4), o_st = take(S * 8), o_ord = take(S * 4), o_ordt = take(S * 4);
  const size_t o_nreg = take(4), o_stat = take(4), o_src = take(M * 4);
  if (cudaMalloc(&g->arena, off) != cudaSuccess) {
    delete g;
    return LB_ERR_CAPACITY;
  }
  cudaMemset(g->arena, 0, off);
  char* b = static_cast<char*>(g->arena);
  IngressDev& d = g->d;
  d.S = max_sessions;
  d.R = ring_frames;
  d.max_rows = max_rows;
  d.pcm = reinterpret_cast<float*>(b + o_pcm);
  d.frame_id = reinterpret_cast<long long*>(b + o_fid);
  d.enqueue = reinterpret_cast<long long*>(b + o_enq);
  d.head = reinterpret_cast<unsigned*>(b + o_head);
  d.tail = reinterpret_cast<unsigned*>(b + o_tail);
  d.paused = reinterpret_cast<unsigned char*>(b + o_p);
  d.active = reinterpret_cast<unsigned char*>(b + o_a);
  d.gone = reinterpret_cast<unsigned char*>(b + o_g);
  d.handle = reinterpret_cast<int*>(b + o_h);
  d.stamp = reinterpret_cast<long long*>(b + o_st);
  d.order = reinterpret_cast<int*>(b + o_ord);
  d.order_tmp = reinterpret_cast<int*>(b + o_ordt);
  d.n_reg = reinterpret_cast<int*>(b + o_nreg);
  d.status = reinterpret_cast<int*>(b + o_stat);
  d.row_src = reinterpret_cast<int*>(b + o_src);
  cudaMemset(d.stamp, 0xFF, S * 8);  // no push call has id -1
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(g->arena);
    delete g;
    return LB_ERR_CUDA;
  }
  *out = g;
  return LB_OK;
}

int lb_ingress_destroy(lb_ingress* g) {
  if (!g) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(g->device);
  cudaDeviceSynchronize();
  cudaFree(g->arena);
  delete g;
  return LB_OK;
}

int lb_ingress_events_async(lb_ingress* g, int n, const int32_t* kind, const int32_t* session, const int32_t* arg,
                            void* stream) {
  if (!g || n < 0 || n > kMaxEvents || (n > 0 && (!kind || !session || !arg))) return LB_ERR_INVALID_ARGUMENT;
  if (n == 0) return LB_OK;
  cudaSetDevice(g->device);
  ingress_events_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(g->d, n, kind, session, arg);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int lb_ingress_push_async(lb_ingress* g, int n, const int32_t* session, const int64_t* frame_id,
                          const int64_t* enqueue_ns, const float* pcm, void* stream) {
  if (!g || n < 0 || (n > 0 && (!session || !frame_id || !enqueue_ns || !pcm))) return LB_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(pcm) % 16) return LB_ERR_INVALID_ARGUMENT;
  if (n == 0) return LB_OK;
  cudaSetDevice(g->device);
  g->calls += 1;
  ingress_push_kernel<<<n, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      g->d, g->calls, session, reinterpret_cast<const long long*>(frame_id),
      reinterpret_cast<const long long*>(enqueue_ns), pcm);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int lb_ingress_tick_async(lb_ingress* g, int64_t deadline_ns, int32_t* row_session, int32_t* row_handle,
                          int64_t* row_frame, float* row_pcm, int32_t* n_rows, void* stream) {
  if (!g || !row_session || !row_handle || !row_frame || !row_pcm || !n_rows) return LB_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(row_pcm) % 16) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(g->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ingress_tick_kernel<<<1, kThreads, 0, s>>>(g->d, deadline_ns, row_session, row_handle,
                                            reinterpret_cast<long long*>(row_frame), n_rows);
  ingress_gather_kernel<<<g->d.max_rows, 256, 0, s>>>(g->d, n_rows, row_pcm);
  return cudaGetLastError() == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int lb_ingress_get_status(lb_ingress* g, int32_t* out, void* stream) {
  if (!g || !out) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(g->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, g->d.status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

}  // extern "C"
