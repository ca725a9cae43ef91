// GPU packer: per-step row -> persistent slot mapping, reset flags and staged
// ring heads, plus the commit / rollback / reset transactions.
//
// Reference policy (restated, not translated):
//   StreamingConformerAudioTower.prepare_batch slot mapping
//     duplex_kernel/streaming_conformer.py:571-606
//   _commit (all-or-nothing cursor check, install)            :904-958
//   _rollback / _restore_entries                              :960-984
//   reset / reset_session                                     :418-451
//
// The host keeps sessions as dense integer handles; the device directory holds,
// per handle, its slot, identity key and expected next cursor, and per slot its
// owner.  One CTA of 1024 threads packs a step: rows are resolved in parallel,
// then a block-wide prefix sum ranks the rows that need a new slot (in row
// order) and another ranks the free slots (in slot order), so row k of the
// "new" rows receives the k-th lowest free slot -- exactly the sequential
// "lowest free slot not yet taken" rule of the reference.
#include "common.cuh"
#include "listener.h"

namespace lb {
namespace {

constexpr int kPackThreads = 1024;

// Block-wide exclusive scan of one int per thread; returns the prefix and the total.
__device__ int block_exclusive_scan(int v, int* total, int* sh) {
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
    sh[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int warp_prefix = warp > 0 ? sh[warp - 1] : 0;
  *total = sh[(blockDim.x >> 5) - 1];
  __syncthreads();
  return warp_prefix + x - v;
}

struct PackArgs {
  int n_rows;
  long long step_id;
  int max_sessions, max_handles;
  const int* row_handle;
  const long long *row_key, *row_frame, *row_seq;
  const uint8_t* row_mask_in;
  int* row_mask;
  int* handle_slot;
  long long *handle_key, *handle_exp_frame, *handle_exp_seq, *handle_stamp;
  int* slot_owner;
  SlotMeta *meta_canon, *meta_stage, *row_meta;
  int *row_slot, *row_reason, *row_reset, *row_replacing;
  long long *row_exp_frame, *row_exp_seq;
  int* free_list;
  int* counts;
  int* status;
  unsigned long long* ctr;
};

// Adds this warp's active lanes' votes for `pred` to *dst with one atomic.
__device__ __forceinline__ void warp_count(bool pred, unsigned long long* dst) {
  const unsigned am = __activemask();
  const unsigned votes = __ballot_sync(am, pred);
  if ((threadIdx.x & 31) == __ffs(am) - 1 && votes) atomicAdd(dst, static_cast<unsigned long long>(__popc(votes)));
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(PackArgs a) {
  __shared__ int sh[32];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  const int n = a.n_rows;
  // ---- phase 1: resolve rows against the directory
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = a.row_handle[i];
    if (h < 0 || h >= a.max_handles) {
      atomicOr(a.status, kStatusBadHandle);
      bad = 1;
      a.row_slot[i] = -1;
      continue;
    }
    const unsigned long long prev = atomicExch(
        reinterpret_cast<unsigned long long*>(&a.handle_stamp[h]),
        static_cast<unsigned long long>(a.step_id));
    if (static_cast<long long>(prev) == a.step_id) {
      atomicOr(a.status, kStatusDuplicateRow);
      bad = 1;
    }
    const int s = a.handle_slot[h];
    const long long key = a.row_key[i];
    int slot = -2, reason = 3, replacing = 0;
    long long ef = -1, es = -1;
    if (s >= 0 && a.handle_key[h] == key) {
      slot = s;
      ef = a.handle_exp_frame[h];
      es = a.handle_exp_seq[h];
      if (ef < 0) {
        reason = 1;  // reset: identity known but no expected cursor
      } else if (ef == a.row_frame[i] && es == a.row_seq[i]) {
        reason = 0;  // continue
      } else {
        reason = 2;  // gap_or_cursor_mismatch
      }
    } else if (s >= 0) {
      slot = s;  // same session, new generation/epoch: reuse its slot
      reason = 3;
      replacing = 1;
    }
    a.row_slot[i] = slot;
    a.row_reason[i] = reason;
    a.row_replacing[i] = replacing;
    a.row_exp_frame[i] = ef;
    a.row_exp_seq[i] = es;
  }
  __syncthreads();
  // ---- phase 2: free slots in slot order
  int n_free = 0;
  for (int base = 0; base < a.max_sessions; base += blockDim.x) {
    const int s = base + threadIdx.x;
    const int f = (s < a.max_sessions && a.slot_owner[s] < 0) ? 1 : 0;
    int tot;
    const int r = block_exclusive_scan(f, &tot, sh);
    if (f) a.free_list[n_free + r] = s;
    n_free += tot;
  }
  __syncthreads();
  // ---- phase 3: rows needing a new slot, in row order
  int taken = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int f = (i < n && a.row_slot[i] == -2) ? 1 : 0;
    int tot;
    const int r = block_exclusive_scan(f, &tot, sh);
    if (f) {
      const int k = taken + r;
      if (k < n_free) {
        a.row_slot[i] = a.free_list[k];
      } else {
        a.row_slot[i] = -1;
        atomicOr(a.status, kStatusSlotExhausted);
        bad = 1;
      }
    }
    taken += tot;
  }
  __syncthreads();
  // ---- phase 4: effective canonical meta and staged meta per row
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int slot = a.row_slot[i];
    const int reason = a.row_reason[i];
    const int reset = reason != 0;
    a.row_reset[i] = reset;
#pragma unroll
    for (int r = 0; r < 4; ++r) warp_count(reason == r, a.ctr + r);
    if (slot < 0) continue;
    SlotMeta m = a.meta_canon[slot];
    if (reset) {
      m.fill = 0;
      m.valid_bits = 0;
      m.flags = 0;
    }
    a.row_meta[i] = m;
    const int mask = a.row_mask_in ? static_cast<int>(a.row_mask_in[i]) : 0xFF;
    a.row_mask[i] = mask;
    SlotMeta st;
    st.pos = (m.pos + 2) & 0xFFFF;
    st.fill = min(m.fill + 2, kCached);
    const int b0 = (m.pos + kCached) & (kRing - 1);
    const int b1 = (m.pos + kCached + 1) & (kRing - 1);
    int vb = m.valid_bits & ~((1 << b0) | (1 << b1));
    if (mask & 0x01) vb |= 1 << b0;  // token 0 valid = mel row 0 valid (mask[::2][::2])
    if (mask & 0x10) vb |= 1 << b1;  // token 1 valid = mel row 4 valid
    st.valid_bits = vb;
    st.flags = ((mask >> 7) & 1) | (((mask >> 6) & 1) << 1);  // last mel row / last conv0 row
    a.meta_stage[slot] = st;
  }
  if (threadIdx.x == 0) {
    a.counts[0] = bad ? 0 : n;  // a failed pack runs no rows
    a.counts[1] = bad ? 0 : 2 * n;
    a.counts[3] = bad ? 0 : 1;
  }
}

struct CommitArgs {
  const int* counts;
  int* counts_w;
  const int *row_handle, *row_slot;
  const long long *row_key, *row_frame, *row_seq, *row_exp_frame, *row_exp_seq;
  int* handle_slot;
  long long *handle_key, *handle_exp_frame, *handle_exp_seq;
  int* slot_owner;
  SlotMeta *meta_canon, *meta_stage, *meta_backup;
  int* bk_handle_slot;
  long long *bk_handle_key, *bk_handle_exp_frame, *bk_handle_exp_seq;
  int* bk_slot_owner;
  int* status;
  unsigned long long* ctr;
};

__global__ void __launch_bounds__(kPackThreads) commit_kernel(CommitArgs a) {
  __shared__ int stale;
  if (threadIdx.x == 0) stale = (a.counts[3] == 0) ? 1 : 0;
  __syncthreads();
  const int n = a.counts[0];
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = a.row_handle[i];
    const bool known = a.handle_slot[h] >= 0 && a.handle_key[h] == a.row_key[i];
    const long long ef = known ? a.handle_exp_frame[h] : -1;
    const long long es = known ? a.handle_exp_seq[h] : -1;
    if (ef != a.row_exp_frame[i] || es != a.row_exp_seq[i]) stale = 1;
  }
  __syncthreads();
  if (stale) {
    if (threadIdx.x == 0) {
      if (a.counts[3]) {
        atomicOr(a.status, kStatusStaleCommit);
        a.ctr[5] += 1;
      }
      a.counts_w[2] = 0;
      a.counts_w[3] = 0;
    }
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = a.row_handle[i];
    const int s = a.row_slot[i];
    a.bk_handle_slot[i] = a.handle_slot[h];
    a.bk_handle_key[i] = a.handle_key[h];
    a.bk_handle_exp_frame[i] = a.handle_exp_frame[h];
    a.bk_handle_exp_seq[i] = a.handle_exp_seq[h];
    a.bk_slot_owner[i] = a.slot_owner[s];
    a.meta_backup[s] = a.meta_canon[s];
    a.handle_slot[h] = s;
    a.handle_key[h] = a.row_key[i];
    a.handle_exp_frame[h] = a.row_frame[i] + 1;
    a.handle_exp_seq[h] = a.row_seq[i] + 1;
    a.slot_owner[s] = h;
    a.meta_canon[s] = a.meta_stage[s];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.counts_w[2] = n;
    a.counts_w[3] = 0;  // the packed rows are consumed
    a.ctr[4] += static_cast<unsigned long long>(n);
  }
}

__global__ void __launch_bounds__(kPackThreads) rollback_kernel(CommitArgs a) {
  const int n = a.counts[2];
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = a.row_handle[i];
    const int s = a.row_slot[i];
    a.handle_slot[h] = a.bk_handle_slot[i];
    a.handle_key[h] = a.bk_handle_key[i];
    a.handle_exp_frame[h] = a.bk_handle_exp_frame[i];
    a.handle_exp_seq[h] = a.bk_handle_exp_seq[i];
    a.slot_owner[s] = a.bk_slot_owner[i];
    a.meta_canon[s] = a.meta_backup[s];
  }
  __syncthreads();
  if (threadIdx.x == 0) a.counts_w[2] = 0;
}

__global__ void reset_kernel(int handle, int slot, int* handle_slot, long long* handle_key,
                             long long* handle_exp_frame, long long* handle_exp_seq,
                             int* slot_owner, SlotMeta* meta_canon) {
  if (threadIdx.x != 0) return;
  if (handle >= 0) slot = handle_slot[handle];
  if (slot >= 0 && handle < 0) handle = slot_owner[slot];
  if (handle >= 0) {
    handle_slot[handle] = -1;
    handle_key[handle] = -1;
    handle_exp_frame[handle] = -1;
    handle_exp_seq[handle] = -1;
  }
  if (slot >= 0) {
    slot_owner[slot] = -1;
    SlotMeta z{0, 0, 0, 0};
    meta_canon[slot] = z;
  }
}

CommitArgs commit_args(Ctx& c) {
  CommitArgs a;
  a.counts = c.dev_counts;
  a.counts_w = c.dev_counts;
  a.row_handle = c.row_handle;
  a.row_slot = c.row_slot;
  a.row_key = c.row_key;
  a.row_frame = c.row_frame;
  a.row_seq = c.row_seq;
  a.row_exp_frame = c.row_exp_frame;
  a.row_exp_seq = c.row_exp_seq;
  a.handle_slot = c.handle_slot;
  a.handle_key = c.handle_key;
  a.handle_exp_frame = c.handle_exp_frame;
  a.handle_exp_seq = c.handle_exp_seq;
  a.slot_owner = c.slot_owner;
  a.meta_canon = c.meta_canon;
  a.meta_stage = c.meta_stage;
  a.meta_backup = c.meta_backup;
  a.bk_handle_slot = c.bk_handle_slot;
  a.bk_handle_key = c.bk_handle_key;
  a.bk_handle_exp_frame = c.bk_handle_exp_frame;
  a.bk_handle_exp_seq = c.bk_handle_exp_seq;
  a.bk_slot_owner = c.bk_slot_owner;
  a.status = c.status;
  a.ctr = c.dev_ctr;
  return a;
}

// Releases n handles at once (sessions that left this tick): each handle's
// slot is freed and its directory entry cleared, as reset_kernel does for one.
// Handles are distinct in a well-formed call; an out-of-range one sets
// kStatusBadHandle and is skipped.
__global__ void reset_many_kernel(const int* handles, int n, int max_handles, int* handle_slot,
                                  long long* handle_key, long long* handle_exp_frame,
                                  long long* handle_exp_seq, int* slot_owner, SlotMeta* meta_canon,
                                  int* status) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int h = handles[i];
    if (h < 0 || h >= max_handles) {
      atomicOr(status, kStatusBadHandle);
      continue;
    }
    const int slot = handle_slot[h];
    handle_slot[h] = -1;
    handle_key[h] = -1;
    handle_exp_frame[h] = -1;
    handle_exp_seq[h] = -1;
    if (slot >= 0) {
      slot_owner[slot] = -1;
      meta_canon[slot] = SlotMeta{0, 0, 0, 0};
    }
  }
}

// status[1] |= status[0]; status[0] = 0 (the history keeps every cleared error)
__global__ void clear_status_kernel(int* status) {
  if (threadIdx.x == 0) {
    status[1] |= status[0];
    status[0] = 0;
  }
}

}  // namespace

cudaError_t launch_pack(Ctx& c, int n_rows, long long step_id, cudaStream_t s) {
  PackArgs a;
  a.n_rows = n_rows;
  a.step_id = step_id;
  a.max_sessions = c.cfg.max_sessions;
  a.max_handles = c.max_handles;
  a.row_handle = c.row_handle;
  a.row_key = c.row_key;
  a.row_frame = c.row_frame;
  a.row_seq = c.row_seq;
  a.row_mask_in = c.row_mask_in;
  a.row_mask = c.row_mask;
  a.handle_slot = c.handle_slot;
  a.handle_key = c.handle_key;
  a.handle_exp_frame = c.handle_exp_frame;
  a.handle_exp_seq = c.handle_exp_seq;
  a.handle_stamp = c.handle_stamp;
  a.slot_owner = c.slot_owner;
  a.meta_canon = c.meta_canon;
  a.meta_stage = c.meta_stage;
  a.row_meta = c.row_meta;
  a.row_slot = c.row_slot;
  a.row_reason = c.row_reason;
  a.row_reset = c.row_reset;
  a.row_replacing = c.row_replacing;
  a.row_exp_frame = c.row_exp_frame;
  a.row_exp_seq = c.row_exp_seq;
  a.free_list = c.free_list;
  a.counts = c.dev_counts;
  a.status = c.status;
  a.ctr = c.dev_ctr;
  pack_kernel<<<1, kPackThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_reset_many(Ctx& c, const int* handles, int n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int blocks = (n + 255) / 256 < 64 ? (n + 255) / 256 : 64;
  reset_many_kernel<<<blocks, 256, 0, s>>>(handles, n, c.max_handles, c.handle_slot, c.handle_key,
                                           c.handle_exp_frame, c.handle_exp_seq, c.slot_owner,
                                           c.meta_canon, c.status);
  return cudaGetLastError();
}

cudaError_t launch_clear_status(Ctx& c, cudaStream_t s) {
  clear_status_kernel<<<1, 32, 0, s>>>(c.status);
  return cudaGetLastError();
}

cudaError_t launch_commit(Ctx& c, cudaStream_t s) {
  commit_kernel<<<1, kPackThreads, 0, s>>>(commit_args(c));
  return cudaGetLastError();
}

cudaError_t launch_rollback(Ctx& c, cudaStream_t s) {
  rollback_kernel<<<1, kPackThreads, 0, s>>>(commit_args(c));
  return cudaGetLastError();
}

cudaError_t launch_reset(Ctx& c, int handle, int slot, cudaStream_t s) {
  reset_kernel<<<1, 32, 0, s>>>(handle, slot, c.handle_slot, c.handle_key, c.handle_exp_frame,
                                c.handle_exp_seq, c.slot_owner, c.meta_canon);
  return cudaGetLastError();
}

}  // namespace lb
