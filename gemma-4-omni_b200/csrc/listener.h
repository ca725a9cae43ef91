// Internal context of a listener step instance (one per GPU / process).
//
// Device memory layout (all owned by the context, allocated at lb_create):
//
//   weights   one arena; GEMM weights bf16 [O,K] or int8 [O,K] + fp16 scale[O];
//             norms / conv / biases fp32 (bf16-rounded values).  With int8
//             weights and buckets of >= 128 tokens, a second arena holds the
//             int8 codes widened to fp16 (exact): from there on the in-kernel
//             widening costs more than the extra weight bytes.
//   sessions  persistent per-slot state, S = max_sessions slots:
//               kv_k, kv_v  bf16 [L][S][16][d] (+pad per slot, ring_base) ring of the
//                           last 13 projected keys / values (pre-scale, exactly
//                           the bf16 linear outputs) plus 2 staged + 1 spare
//               conv_ring   bf16 [L][S][8][d] (+pad)  last 4 GLU rows + 2 staged
//               sub_prev    bf16 [S][2][128][64] last conv0 output row, double-buffered
//               mel_prev    f32  [S][2][128]     last mel row, double-buffered
//               pcm_tail    f32  [S][2][160]     last 160 PCM samples, double-buffered
//               meta        int4 [S] x3          canonical / staged / rollback backup
//                           {pos, fill, valid_bits, flags}
//             A step writes only staged ring entries and the staged meta; commit
//             copies staged meta -> canonical (the "ring head swap"), so no cache
//             window is ever copied (reference: full-window index_copy_ staging,
//             duplex_kernel/streaming_conformer.py:682-697, 904-958).
//   tables    session-handle directory for the packer (handle -> slot / key /
//             expected cursor) and slot -> owner.
//   rows      per-step row tables written by the packer (row -> slot, reset,
//             reason) and the device row count read by every kernel.
//   acts      activation buffers sized for 2*max_rows tokens.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/listener_b200.h"
#include "kernels.h"

namespace lb {

constexpr int kRing = 16;      // K/V ring entries per slot per layer
constexpr int kConvRing = 8;   // conv-state ring entries
constexpr int kCached = 13;    // CACHED_PAST_TOKENS
constexpr int kMelBins = 128;
constexpr int kPcm = 1280;
constexpr int kTail = 160;

// Ring storage is layer-major: for each layer, the slots' rings follow one
// another at a stride of (entries * d + kRingPad) elements.  Concurrent CTAs
// (one per session) read the same layer and ring entry of different slots; the
// 128-byte pad keeps those rows from sharing the low address bits that a
// power-of-two-multiple stride would give them, which spreads them over the
// DRAM channels.
constexpr int kRingPad = 64;  // bf16 elements
__host__ __device__ inline size_t ring_base(int slot, int layer, int slots, int entries, int d) {
  return (static_cast<size_t>(layer) * slots + slot) * (static_cast<size_t>(entries) * d + kRingPad);
}

struct SlotMeta {
  int pos;         // ring base: canonical entries are (pos + j) mod ring
  int fill;        // tokens written since the last reset (saturates at 13)
  int valid_bits;  // token-valid bit per K/V ring entry
  int flags;       // bit0: mel_prev valid, bit1: sub_prev valid
};

struct LayerW {
  float *ffn_pre[2], *ffn_post[2];
  void *w_ffn1[2], *w_ffn2[2];
  __half *s_ffn1[2], *s_ffn2[2];
  float *norm_pre_attn, *norm_post_attn, *norm_out;
  void* w_qkv;
  __half* s_qkv;
  void* w_post;
  __half* s_post;
  float* q_mult;    // [hd] q_scale * softplus(per_dim_scale)
  float* rel_keys;  // [13][d] relative keys, fp32
  __nv_bfloat16* rel_bf16;  // [13][d] the same, bf16 (attention MMA operand; set at finalize)
  float *lc_pre, *lc_norm;
  float* lc_dw;     // [5][d] tap-major (transposed from [d][1][5] on upload)
  void *w_lstart, *w_lend;
  __half *s_lstart, *s_lend;
  float clip[8][4];  // per linear: in_lo, in_hi, out_lo, out_hi (Q/K/V: the q_proj bounds)
  float qkv_clip[3][4];  // q_proj, k_proj, v_proj bounds
  bool qkv_split_in = false;   // their input bounds differ: stacked inputs
  bool qkv_split_out = false;  // their output bounds differ: per-part output clamps
};

struct Weights {
  float* conv0;    // [128][9]
  float* ln0;      // [128]
  __nv_bfloat16* conv1;  // [C1][9*128 (+pad)] k = (i*3+j)*128 + ci
  float* ln1;      // [C1]
  void* w_in;
  __half* s_in;
  std::vector<LayerW> layers;
  void* w_out;
  __half* s_out;
  float* b_out;
  void* w_embed;
  __half* s_embed;
  // FiLM
  float *fq_norm_w, *fq_norm_b, *fr_norm_w, *fr_norm_b;
  void *w_qdown, *w_rdown, *w_film, *w_fout;
  __half *s_qdown, *s_rdown, *s_film, *s_fout;
  float *b_qdown, *b_rdown, *b_film, *b_fout;
  float film_scale;  // 0.25 * sigmoid(scale_logit), set from the host
};

struct TensorSlot {
  void* dst;
  int dtype;
  int64_t numel;
  bool set = false;
  bool gemm = false;  // GEMM weight (bf16, or int8 with ":scale" companion)
  int qkv_part = -1;
  float* clip_dst = nullptr;  // for clip bound scalars
};

struct Ctx;

// One GEMM of the step at one token tile size.
struct GemmOp {
  GemmPlan plan;
  GemmParams params;
  int splits = 1;
  bool final_f16 = false;  // output feeds another GEMM in fp16 (int8 weights)
  bool pdl = false;        // launched with programmatic stream serialisation
  int out_kind = 0;        // 0: bf16 / fp16 tensor, 1: fp32 (the split-K finish pass's store)
  void* out = nullptr;     // the op's output (a split-K GEMM itself writes wide_acc)
  bool consumer_finishes = false;  // split-K: the row kernel after it reads wide_acc and finishes it
};

struct Bucket {
  int rows_cap = 0;   // sessions
  int tok_cap = 0;    // 2 * rows_cap
  cudaGraphExec_t graph = nullptr;
  bool graph_ready = false;
};

struct Ctx {
  lb_config cfg{};
  int device = 0;
  int num_sms = 148;
  int hd = 0;
  int weight_int8 = 0;
  // GEMM operands are fp16: int8 codes and bf16 weights are both widened to
  // fp16 exactly, and every activation that feeds a GEMM is stored as fp16
  // (saturated at +/-65504), 3 more mantissa bits than bf16
  int f16_acts = 1;
  // Programmatic dependent launch of the step's kernels (common.cuh pdl_wait).
  // pdl: GEMMs launch while the kernel before them drains and stream their
  // first weight tiles meanwhile; pdl_all: every other step kernel launches
  // early too.  LB_PDL=0 / 1 / 2: off / GEMMs only / all kernels.
  bool pdl = true;
  bool pdl_all = false;
  // int8 weights: buckets of at least this many tokens read the fp16-widened
  // codes (kept resident beside the int8 arena), smaller ones widen the int8
  // codes inside the GEMM.  LB_WIDE_MIN_TOKENS overrides it.
  int wide_min_tokens = 128;

  // arenas
  void* weight_arena = nullptr;
  size_t weight_bytes = 0;
  // int8 weights: the whole weight arena widened byte-for-byte to fp16, so the
  // fp16 codes of an int8 tensor at arena offset b sit at byte offset 2b here
  // (null when not built).  Large buckets read these instead of the int8 codes.
  void* wide_arena = nullptr;
  __nv_bfloat16* rel_bf16_arena = nullptr;  // [L][13][d] bf16 relative keys
  void* state_arena = nullptr;
  size_t state_bytes = 0;
  void* act_arena = nullptr;
  size_t act_bytes = 0;

  Weights w{};
  std::map<std::string, TensorSlot> tensors;
  bool weights_final = false;

  // persistent session state
  __nv_bfloat16 *kv_k = nullptr, *kv_v = nullptr, *conv_ring = nullptr, *sub_prev = nullptr;
  float *mel_prev = nullptr, *pcm_tail = nullptr;
  SlotMeta *meta_canon = nullptr, *meta_stage = nullptr, *meta_backup = nullptr;
  // handle directory
  int max_handles = 0;
  int *handle_slot = nullptr, *slot_owner = nullptr;
  long long *handle_key = nullptr, *handle_exp_frame = nullptr, *handle_exp_seq = nullptr;
  long long* handle_stamp = nullptr;
  // rollback record of the last committed batch
  int* bk_handle_slot = nullptr;
  long long *bk_handle_key = nullptr, *bk_handle_exp_frame = nullptr, *bk_handle_exp_seq = nullptr;
  int* bk_slot_owner = nullptr;  // previous owner of each committed row's slot
  int* bk_prev_handle_slot = nullptr;
  // per-step rows
  int* dev_counts = nullptr;  // [0] n_rows, [1] n_tok, [2] committed rows, [3] packed flag
  int* status = nullptr;      // device status word; status[1]: OR of every cleared status
  // running device counters (lb_get_counters): [0..3] packed rows per reset
  // reason (continue, reset, gap_or_cursor_mismatch, identity_reset), [4] rows
  // installed by commits, [5] commits refused by the cursor check
  unsigned long long* dev_ctr = nullptr;
  int *row_handle = nullptr, *row_slot = nullptr, *row_reason = nullptr, *row_reset = nullptr;
  int *row_mask = nullptr, *row_replacing = nullptr;
  uint8_t* row_mask_in = nullptr;  // caller's uint8 masks (copied per step)
  SlotMeta* row_meta = nullptr;    // effective canonical meta per row (reset applied)
  long long *row_key = nullptr, *row_frame = nullptr, *row_seq = nullptr;
  long long *row_exp_frame = nullptr, *row_exp_seq = nullptr;
  int* free_list = nullptr;
  long long step_id = 0;
  int packed_rows = 0;  // host copy of the last pack's row count
  int state = 0;        // 0 idle, 1 packed, 2 stepped, 3 committed(rollback-able)
  int last_commit_rows = 0;

  // activations [tok_cap]
  float* in_pcm = nullptr;    // [rows][1280]
  float* in_mel = nullptr;    // [rows][8][128]
  __nv_bfloat16* in_query = nullptr;  // [tok][Q]
  __nv_bfloat16* sub_in = nullptr;    // [tok][C1*F1]
  float* h = nullptr;                 // [tok][d]
  float* y = nullptr;                 // [tok][max(d, out, text)] narrow fp32 outputs
  __nv_bfloat16* xa = nullptr;        // [tok][d]  GEMM input
  __nv_bfloat16* xf = nullptr;        // [tok][F]  FFN mid
  __nv_bfloat16* qkv = nullptr;       // [tok][3d]
  __nv_bfloat16* att = nullptr;       // [tok][d]
  __nv_bfloat16* gl = nullptr;        // [tok][2d] linear_start output
  float* wide_acc = nullptr;          // [tok][max(F,3d,2d)] split-K partial sums (kept zero)
  int wide_width = 0;                 // row width of wide_acc
  __nv_bfloat16* out_raw = nullptr;   // [tok][out]
  __nv_bfloat16* out_soft = nullptr;  // [tok][text]
  __nv_bfloat16* out_film = nullptr;  // [tok][Q]
  __nv_bfloat16* film_xq = nullptr;   // [tok][Q] LN(query)
  __nv_bfloat16* film_xr = nullptr;   // [tok][text] LN(soft)
  float* film_qd = nullptr;           // [tok][B]
  float* film_rd = nullptr;           // [tok][B]
  __nv_bfloat16* film_rd_bf = nullptr;  // [tok][B]
  float* film_gb = nullptr;           // [tok][2B]
  __nv_bfloat16* film_fused = nullptr;  // [tok][B]
  float* film_map = nullptr;          // [tok][Q]
  float* film_amp = nullptr;          // [tok] RMS(query)
  __nv_bfloat16* xe = nullptr;        // [tok][out] embedder input
  // optional per-layer debug outputs (null in serving)
  float* dbg_sub = nullptr;
  float* dbg_layers = nullptr;
  int dbg_stop_layer = -1;  // eager diagnostics: stop after (layer, stage)
  int dbg_stop_stage = -1;

  // frontend tables: periodic Hann window [320], DFT twiddles [512] x2,
  // mel filterbank [257][128] and its non-zero row range per mel bin
  float *fe_window = nullptr, *fe_cos = nullptr, *fe_sin = nullptr, *fe_filters = nullptr;
  int2* fe_range = nullptr;

  std::vector<Bucket> buckets;
  cudaStream_t capture_stream = nullptr;
};

// --------------------------------------------------------- kernel launchers
cudaError_t launch_mel(Ctx& c, int rows_cap, int input_kind, cudaStream_t s);
// The log-mel of n caller rows with caller-held tails (no session state).
cudaError_t launch_mel_standalone(Ctx& c, int n, const float* pcm, const float* tail_in, float* tail_out,
                                  float* mel, cudaStream_t s);
cudaError_t launch_subsample(Ctx& c, int rows_cap, cudaStream_t s);
cudaError_t launch_pack(Ctx& c, int n_rows, long long step_id, cudaStream_t s);
cudaError_t launch_commit(Ctx& c, cudaStream_t s);
cudaError_t launch_rollback(Ctx& c, cudaStream_t s);
cudaError_t launch_reset(Ctx& c, int handle, int slot, cudaStream_t s);
cudaError_t launch_clear_status(Ctx& c, cudaStream_t s);
cudaError_t launch_reset_many(Ctx& c, const int* handles, int n, cudaStream_t s);
cudaError_t run_layers(Ctx& c, const Bucket& b, cudaStream_t s);

struct RowFusedArgs {
  const float* y = nullptr;   // GEMM fp32 output (or null: no addend)
  const float* post_w = nullptr;  // RMSNorm weight applied to clamp(y) (null: none)
  float alpha = 1.0f;
  bool residual = true;           // h = alpha * post(y) + h   (else h = alpha * post(y))
  const float* out_w = nullptr;   // norm_out RMSNorm of clamp(h) (null: none)
  const float* pre_w = nullptr;   // RMSNorm weight for the next GEMM input
  bool pre_norm = true;           // false: xa = bf16(h) without normalisation
  bool pre_clamp = true;          // clamp(h, +/-clip) before the pre-norm
  float in_lo = -INFINITY, in_hi = INFINITY;  // next linear's input clamp
  __nv_bfloat16* xa = nullptr;
  float* dbg = nullptr;           // optional copy of the new h
  // 3: also write blocks 1 and 2 of the stacked Q/K/V input (xa must be the
  // context's xa; blocks are 2 * max_rows tokens apart), clamped to
  // part_lo/part_hi (the K and V input bounds); block 0 gets in_lo/in_hi
  int xa_parts = 1;
  float part_lo[2] = {-INFINITY, -INFINITY}, part_hi[2] = {INFINITY, INFINITY};
  // y is the split-K partial-sum buffer of the GEMM before: clamp it to the
  // linear's output bounds and zero it after reading (its finish pass)
  bool zero_y = false;
  float y_lo = -INFINITY, y_hi = INFINITY;
};
cudaError_t launch_row_fused(Ctx& c, int tok_cap, const RowFusedArgs& a, cudaStream_t s);
cudaError_t launch_attention(Ctx& c, int layer, int rows_cap, cudaStream_t s);
// bf16 copies of every layer's relative keys (after the weights are uploaded).
cudaError_t attention_prepare(Ctx& c, cudaStream_t s);
cudaError_t launch_lconv(Ctx& c, int layer, int rows_cap, cudaStream_t s);
cudaError_t launch_outputs(Ctx& c, int tok_cap, int stage, cudaStream_t s);
cudaError_t launch_film(Ctx& c, int tok_cap, int stage, cudaStream_t s);
// stage 0: gather the cursor-selected response states and queries into the
// FiLM inputs; stage 1: write the outputs (frame 0 preserved)
cudaError_t launch_film_talker(Ctx& c, int n, const __nv_bfloat16* hidden, int max_states, const int* n_states,
                               const int* steps, const __nv_bfloat16* query, __nv_bfloat16* out, int stage,
                               cudaStream_t s);

}  // namespace lb
