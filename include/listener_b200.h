/*
 * listener_b200.h — C ABI of the B200-native streaming listener step.
 *
 * One call of lb_step_async() runs, for every active session of a step, the
 * reference's per-80 ms listener hot path:
 *   PCM frame -> log-mel (duplex_kernel/listener.py:1807-1850)
 *   -> causal chunked-attention Gemma 4 audio Conformer with per-session
 *      K/V, conv and subsampler caches (duplex_kernel/streaming_conformer.py:700-888)
 *   -> output_proj + embed_audio soft tokens (streaming_conformer.py:871-872)
 *   -> optional FrameResidualQueryFiLM residual (duplex_kernel/frame_residual_adapter.py:203-237).
 *
 * Conventions (mirroring the reference's native batch ABI,
 * native/gemma4_listener_microbatch/gemma4_listener_microbatch.h:206-480):
 *   - every function returns an int status: 0 = ok, negative = error;
 *   - configuration structs carry struct_size and api_version;
 *   - contexts are opaque; all device work is enqueued on the caller's
 *     cudaStream_t (passed as void*) and nothing synchronises the host except
 *     lb_get_status / lb_read_* helpers, which say so;
 *   - pointers are plain device pointers unless a name says "host".
 */
#ifndef LISTENER_B200_H_
#define LISTENER_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LB_API_VERSION 1

enum lb_status_code {
  LB_OK = 0,
  LB_ERR_INVALID_ARGUMENT = -1,
  LB_ERR_CUDA = -2,
  LB_ERR_STATE = -3,        /* call not valid in the context's current state */
  LB_ERR_CAPACITY = -4,     /* session bank exhausted / size beyond capacity */
  LB_ERR_VERSION = -5,      /* struct_size / api_version mismatch */
  LB_ERR_DEVICE_STATUS = -6 /* device status word is non-zero (see lb_get_status) */
};

/* Device status bits reported by lb_get_status(). */
enum lb_device_status_bits {
  LB_DEV_WAIT_TIMEOUT = 1 << 0,
  LB_DEV_SLOT_EXHAUSTED = 1 << 1,
  LB_DEV_DUPLICATE_ROW = 1 << 2,
  LB_DEV_BAD_HANDLE = 1 << 3,
  LB_DEV_STALE_COMMIT = 1 << 4,
  LB_DEV_BAD_ROW_COUNT = 1 << 5,
  LB_DEV_INGRESS_OVERFLOW = 1 << 6 /* a frame found its session's ingress ring full (refused) */
};

/* Session events of the GPU ingress (lb_ingress_events_async). */
enum lb_ingress_event {
  LB_INGRESS_JOIN = 0,  /* register (appended to the registration order); arg = directory handle */
  LB_INGRESS_LEAVE = 1, /* unregister; its queued frames are dropped */
  LB_INGRESS_PAUSE = 2,
  LB_INGRESS_RESUME = 3
};

/* Tensor element types for lb_set_tensor. */
enum lb_dtype { LB_F32 = 0, LB_BF16 = 1, LB_I8 = 2, LB_F16 = 3 };

/* Weight formats of the dense contractions. */
enum lb_weight_format {
  LB_WEIGHTS_BF16 = 0,
  LB_WEIGHTS_INT8 = 1 /* int8 rows + one fp16 scale per output channel */
};

/* Step input kinds for lb_step_async. */
enum lb_input_kind {
  LB_INPUT_PCM = 0, /* float32 [n_rows][1280] 16 kHz PCM; log-mel runs on the GPU */
  LB_INPUT_MEL = 1  /* float32 [n_rows][8][128] log-mel tick (tower-only form) */
};

/* Row reasons written by lb_pack_async (streaming_conformer.py:571-606). */
enum lb_row_reason {
  LB_REASON_CONTINUE = 0,
  LB_REASON_RESET = 1,
  LB_REASON_GAP_OR_CURSOR_MISMATCH = 2,
  LB_REASON_IDENTITY_RESET = 3
};

/* Context configuration.  The model shape is that of transformers'
 * Gemma4AudioConfig (models/gemma4/configuration_gemma4.py:27-80) plus the
 * FiLM adapter (frame_residual_adapter.py:164-197). */
typedef struct lb_config {
  uint32_t struct_size; /* sizeof(lb_config) */
  uint32_t api_version; /* LB_API_VERSION */
  int32_t max_sessions; /* persistent cache slots (StreamingConformerAudioTower max_sessions) */
  int32_t max_handles;  /* session-handle table size (>= max_sessions) */
  int32_t max_rows;     /* largest batch of one step */
  int32_t hidden, layers, heads, ffn;
  int32_t sub_ch0, sub_ch1;
  int32_t output_dims, text_hidden;
  int32_t conv_kernel; /* must be 5 */
  int32_t weight_format;
  int32_t film_enabled;
  int32_t film_query_dim, film_bottleneck;
  float rms_eps, softcap, invalid_logit, gradient_clipping, residual_weight;
  float film_max_scale;
} lb_config;

typedef struct lb_ctx lb_ctx;

/* Creates a context on the current CUDA device: allocates the weight arena,
 * the per-slot session state (zeroed) and the activation buffers.
 * Replaces StreamingConformerAudioTower.__init__ (streaming_conformer.py:138-294)
 * and the native batch create call (gemma4_listener_microbatch.h). */
int lb_create(const lb_config* cfg, lb_ctx** out_ctx);
int lb_destroy(lb_ctx* ctx);

/* Uploads one named parameter (transformers Gemma4AudioModel state_dict names;
 * the embedder under "embed.", the FiLM adapter under "film.", precomputed
 * "layers.<i>.self_attn.relative_keys" [13*hidden] f32 and
 * "layers.<i>.self_attn.query_scale" [head_dim] f32).  GEMM weights are LB_BF16,
 * or LB_I8 with a companion "<name>:scale" LB_F16 [rows] tensor.  Synchronous. */
int lb_set_tensor(lb_ctx* ctx, const char* name, const void* host_data, int dtype, int64_t numel);
/* Checks that every required parameter was uploaded.  Must precede stepping,
 * and follow any later lb_set_tensor (which un-finalizes the context).  With
 * int8 weights and max_rows >= 256 it also builds the fp16-widened copy of
 * the int8 codes that buckets of >= 512 tokens read (synchronous). */
int lb_finalize_weights(lb_ctx* ctx);
/* Number of parameter names the context expects, and the i-th name. */
int lb_tensor_count(lb_ctx* ctx);
const char* lb_tensor_name(lb_ctx* ctx, int index);

/* Packs one step: maps rows to persistent slots on the GPU with the reference
 * slot policy (streaming_conformer.py:571-615: existing identity -> its slot,
 * "continue" iff the cursor equals the expected one; same session with a new
 * generation/epoch -> its slot, "identity_reset"; new session -> lowest free
 * slot in row order) and builds the row -> slot / reset / mask tables.
 * handles: int32 [n] session handles in [0, max_handles); keys: int64 [n]
 * identity (generation, epoch) tokens; frames / seqs: int64 [n] cursors;
 * masks: uint8 [n] bit r = mel row r valid (NULL = all valid).  Device
 * pointers.  Errors that only the device can see (exhausted bank, duplicate
 * handle) set lb_get_status bits and leave session state untouched. */
int lb_pack_async(lb_ctx* ctx, int n_rows, const int32_t* handles, const int64_t* keys,
                  const int64_t* frames, const int64_t* seqs, const uint8_t* masks,
                  void* stream);

/* Runs the packed step: (PCM -> log-mel ->) Conformer -> raw / soft tokens
 * (-> FiLM).  input: LB_INPUT_PCM float32 [n][1280] or LB_INPUT_MEL float32
 * [n][8][128]; query: bf16 [n][2][film_query_dim] or NULL (no FiLM output);
 * out_raw bf16 [n][2][output_dims], out_soft bf16 [n][2][text_hidden],
 * out_film bf16 [n][2][film_query_dim] (any output may be NULL).  Writes only
 * staged session state; canonical state advances on lb_commit_async. */
int lb_step_async(lb_ctx* ctx, int input_kind, const void* input, const void* query,
                  void* out_raw, void* out_soft, void* out_film, void* stream);

/* Same step with HOST buffers: copies inputs in, runs pack + step, copies the
 * outputs back and synchronises the stream before returning (end-to-end
 * form of one serving tick).  Row arrays as in lb_pack_async, host memory.
 * Page-locked (pinned) buffers are transferred by DMA directly; pageable ones
 * pass through the context's pinned staging area (one extra host copy).  The
 * FiLM query is copied in on a context-owned copy stream while the tower runs,
 * and raw/soft tokens are copied out on it while FiLM runs; that stream is
 * joined back into `stream` before the call returns. */
int lb_step_host(lb_ctx* ctx, int n_rows, const int32_t* handles, const int64_t* keys,
                 const int64_t* frames, const int64_t* seqs, const uint8_t* masks,
                 int input_kind, const void* input, const void* query, void* out_raw,
                 void* out_soft, void* out_film, int commit, void* stream);

/* Optional diagnostics for the next lb_step_async (forces eager launches):
 * subsampled float32 [n][2][hidden], layers float32 [layers][n][2][hidden]. */
int lb_set_debug_outputs(lb_ctx* ctx, float* subsampled, float* layers);

/* Commits the packed+stepped rows: checks that no cursor changed since pack
 * (all-or-nothing, streaming_conformer.py:904-958), then installs the staged
 * ring heads and cursors.  A stale cursor sets LB_DEV_STALE_COMMIT. */
int lb_commit_async(lb_ctx* ctx, void* stream);
/* Drops the packed step without touching session state (streaming_conformer.py:986-990). */
int lb_abort(lb_ctx* ctx);
/* Restores the state before the last commit (streaming_conformer.py:960-967).
 * Valid only until the next lb_pack_async. */
int lb_rollback_async(lb_ctx* ctx, void* stream);
/* Releases one session handle (its slot becomes free, state logically zero).
 * StreamingConformerAudioTower.reset (streaming_conformer.py:418-434). */
int lb_reset_handle_async(lb_ctx* ctx, int32_t handle, void* stream);
/* Releases n distinct handles (int32 device array) in one launch: the
 * sessions that left this tick (close_session -> reset for each,
 * listener_microbatch_frontend.py:363-377, streaming_conformer.py:418-434).
 * An out-of-range handle sets LB_DEV_BAD_HANDLE and is skipped. */
int lb_reset_handles_async(lb_ctx* ctx, int n, const int32_t* handles, void* stream);
/* Releases one slot (StreamingConformerAudioTower.reset_session, :436-451). */
int lb_reset_slot_async(lb_ctx* ctx, int32_t slot, void* stream);

/* Kernels launched by the CUDA graph of the last lb_step_async (0 if eager). */
int lb_step_kernel_count(lb_ctx* ctx);

/* The reference's incremental log-mel (_extract_single_frame,
 * duplex_kernel/listener.py:1807-1850) for n PCM frames of any streams whose
 * tails the caller holds, outside the session state: e.g. the assistant
 * (reference) audio the frontend turns into mel per row
 * (listener_microbatch_frontend.py:792-809).  pcm f32 [n][1280]; tail_in f32
 * [n][160] (NULL: every stream starts fresh); tail_out f32 [n][160] receives
 * each frame's last 160 samples (must not alias tail_in); mel_out f32
 * [n][8][128].  Device pointers; asynchronous on `stream`. */
int lb_mel_async(lb_ctx* ctx, int n, const float* pcm, const float* tail_in, float* tail_out,
                 float* mel_out, void* stream);

/* The FrameResidualQueryFiLM adapter at its Talker call site, batched over n
 * sessions: apply_response_state_residual
 * (duplex_kernel/frame_residual_adapter.py:38-71, called at engine.py:6757).
 * Row i selects response state min(steps[i], n_states[i] - 1) of its response
 * hidden (bf16 [max_states][text_hidden], rows max_states apart) -- the Qwen
 * text cursor, holding the last state once the text is exhausted -- and
 * conditions its Qwen Q1 query (bf16 [film_query_dim]); at steps[i] == 0 the
 * query is returned unchanged (the adapter's preserve_frame0).  out bf16
 * [n][film_query_dim].  n_states / steps: int32 device arrays.  n <= 2 *
 * max_rows.  Not valid between lb_pack_async and its commit / abort; an
 * invalid n_states or step sets LB_DEV_BAD_ROW_COUNT. */
int lb_film_talker_async(lb_ctx* ctx, int n, const void* response_hidden, int max_states,
                         const int32_t* n_states, const int32_t* steps, const void* query, void* out,
                         void* stream);

/* The batched Control6 policy head over native listener hidden rows: the
 * tensor part of GemmaNativeControl6BatchPolicy.step_batch
 * (duplex_kernel/gemma_native_control6_batch_policy.py:853-893) over
 * NativeControl6LoRA.forward (training/duplex_qlora/native_control6.py:157-197),
 * one launch for n rows.  hidden bf16 [n][hidden_ld] (the final-normalised
 * 1536-wide state; hidden_ld >= 1536, e.g. 3072 for the first token of
 * [n][2][1536]); phase f32 [n][4] or NULL (zeros); legal uint8 [n], bit a =
 * action a legal, or NULL (all legal); base_rows bf16 [6][1536] (the tied
 * LM-head rows); lora_a f32 [rank][1540]; lora_b f32 [6][rank]; 1 <= rank <= 64.
 * logits_out f32 [n][6] = bf16(base_rows . h) + scaling * B(A [h; phase]);
 * packet_out f32 [n][4] = (all six logits finite, argmax, argmax over the legal
 * actions, softmax probability of that action among the legal ones); argmax
 * ties resolve to the lowest action index.  Device pointers; asynchronous. */
int lb_op_control6_head(int n, const void* hidden, int hidden_ld, const float* phase,
                        const uint8_t* legal, const void* base_rows, const float* lora_a,
                        const float* lora_b, int rank, float scaling, float* logits_out,
                        float* packet_out, void* stream);

/* ------------------------------------------------------------------
 * GPU-resident ingress: the fixed-grid dispatcher's per-session queues and its
 * row snapshot on the device (SharedListenerTickDispatcher, register_session /
 * pause / unregister and _snapshot_ready_rows,
 * duplex_kernel/shared_listener_scheduler.py:80-535).  Every session index
 * (chosen by the caller, < max_sessions) owns a ring of ring_frames PCM frames
 * with their frame ids and enqueue times.  Per tick the caller enqueues the
 * session events, pushes the frames that arrived (one H2D copy of the batch)
 * and runs the tick, which emits -- in registration order, skipping paused
 * sessions -- each session's oldest queued frame enqueued no later than the
 * deadline (a later one stays queued: the reference's deferral), consumes it,
 * and gathers the rows' PCM into a [max_rows][1280] buffer ready for
 * lb_step_async.  At most max_rows rows per tick; ready frames past that stay
 * queued.  The ring is bounded: a push that finds it full is refused with
 * LB_DEV_INGRESS_OVERFLOW.  Device pointers; asynchronous on `stream`.
 * ------------------------------------------------------------------ */
typedef struct lb_ingress lb_ingress;
int lb_ingress_create(int max_sessions, int ring_frames, int max_rows, lb_ingress** out);
int lb_ingress_destroy(lb_ingress* ing);
/* n <= 1024 events applied in order: kind (lb_ingress_event), session index,
 * arg (the session's directory handle for LB_INGRESS_JOIN).  An index released
 * by LEAVE must not JOIN again in the same call. */
int lb_ingress_events_async(lb_ingress* ing, int n, const int32_t* kind, const int32_t* session,
                            const int32_t* arg, void* stream);
/* n arrived frames, at most one per session per call: session index, frame
 * id, enqueue time (ns) and PCM f32 [n][1280] (16-byte aligned). */
int lb_ingress_push_async(lb_ingress* ing, int n, const int32_t* session, const int64_t* frame_id,
                          const int64_t* enqueue_ns, const float* pcm, void* stream);
/* One tick: row_session / row_handle int32 [max_rows], row_frame int64
 * [max_rows], row_pcm f32 [max_rows][1280], *n_rows (device int32). */
int lb_ingress_tick_async(lb_ingress* ing, int64_t deadline_ns, int32_t* row_session, int32_t* row_handle,
                          int64_t* row_frame, float* row_pcm, int32_t* n_rows, void* stream);
/* Ingress status bits (LB_DEV_*; synchronises `stream`). */
int lb_ingress_get_status(lb_ingress* ing, int32_t* status_out, void* stream);

/* Synchronous reads (they synchronise the given stream). */
int lb_get_status(lb_ctx* ctx, int32_t* status_out, void* stream);
/* Asynchronous: clears the status word, keeping its bits in the history
 * that lb_get_counters reports. */
int lb_clear_status(lb_ctx* ctx, void* stream);

/* Running per-context counters (the native batch ABI's get_counters,
 * native/gemma4_listener_microbatch/gemma4_listener_microbatch.h:206-480).
 * Call counts are kept on the host; the per-reason row counts (every row a
 * pack resolved, by lb_row_reason), committed rows and refused commits are
 * kept on the device by the packer / commit kernels.  Set struct_size and
 * api_version before the call; synchronises `stream`. */
typedef struct lb_counters {
  uint32_t struct_size;
  uint32_t api_version;
  uint64_t packs, steps, commits, aborts, rollbacks, resets;
  uint64_t rows_stepped;                 /* sum of the row counts of every step */
  uint64_t rows_continue, rows_reset, rows_gap_or_cursor_mismatch, rows_identity_reset;
  uint64_t rows_committed;               /* rows installed by successful commits */
  uint64_t stale_commits;                /* commits refused by the cursor check */
  int32_t status;                        /* current device status word */
  int32_t status_history;                /* OR of every status word since creation */
  int32_t graphs_captured;               /* CUDA graphs instantiated so far */
  int32_t reserved;
} lb_counters;
int lb_get_counters(lb_ctx* ctx, lb_counters* out, void* stream);
/* Last packed rows: slot ids and reasons (lb_row_reason). */
int lb_read_rows(lb_ctx* ctx, int32_t* slots_host, int32_t* reasons_host, int n, void* stream);
/* Directory dump: per handle slot (-1 = none), key, expected frame / seq. */
int lb_read_handles(lb_ctx* ctx, int32_t* slot_host, int64_t* key_host, int64_t* exp_frame_host,
                    int64_t* exp_seq_host, void* stream);
/* Test hook: overwrite one handle's expected cursor (cursor-tamper case). */
int lb_debug_set_expected(lb_ctx* ctx, int32_t handle, int64_t frame, int64_t seq, void* stream);
/* Diagnostics: make the next lb_step_async run eagerly and stop after stage
 * `stage` (0..12) of layer `layer` (-1 disables); lb_debug_read_buffer copies
 * an internal activation ("h", "y", "xa", "xf", "qkv", "att", "gl", "mel",
 * "sub_in") to host memory (synchronous).  GEMM-input buffers ("xa", "xf",
 * "att", "sub_in") hold fp16 instead of bf16 when the weights are int8. */
int lb_debug_set_stop(lb_ctx* ctx, int layer, int stage);
int lb_debug_read_buffer(lb_ctx* ctx, const char* name, void* host_dst, size_t bytes, void* stream);

/* ----------------------------------------------------------------------
 * Per-kernel entry points (one kernel each, caller-owned device buffers).
 * ---------------------------------------------------------------------- */

/* D[t,o] = sum_k X[t,k] W[o,k] (+bias[o]) on tcgen05 tensor cores.
 * Replaces Gemma4ClippableLinear.forward / the reference Triton clipped
 * linear (duplex_kernel/streaming_conformer_kernels.py:27-76, 110-168).
 * w_int8 selects the weight format of w [out_features, k]: 0 = bf16;
 * 1 = int8 codes, widened to fp16 inside the kernel; 2 = the same codes
 * already widened to fp16 (exact), read directly.  With 1 or 2, w_scale is
 * the fp16 per-output-channel scale and x is fp16 (the product runs as an
 * fp16 x fp16 MMA); with 0, x is bf16.  x: [m, x_ld] (K-contiguous,
 * x_ld % 8 == 0); out_mode 0 = bf16, 1 = fp32,
 * 2 = fp32 atomic accumulate (caller zeroes out; required when splits > 1);
 * act 1 = SiLU of the bf16-rounded product (bf16 output only).
 * out_features % 128 == 0, k % 64 == 0, x_ld >= k, ld_out >= out_features,
 * x and w 16-byte aligned (else LB_ERR_INVALID_ARGUMENT). */
int lb_op_gemm(const void* x, int x_ld, int m, const void* w, int w_int8, const void* w_scale,
               const float* bias, int out_features, int k, void* out, int ld_out, int out_mode,
               int act, int splits, int* status_dev, void* stream);

/* lb_op_gemm with the clip bounds of Gemma4ClippableLinear
 * (transformers models/gemma4/modeling_gemma4.py:128-154, whose output clamp
 * the reference's Triton linear fuses, streaming_conformer_kernels.py:27-73).
 * The weight is `parts` stacked linears of out_features/parts features each
 * (3: the fused q/k/v projections; out_features % (128*parts) == 0):
 * out_bounds[2j], out_bounds[2j+1] clamp part j's linear output before the
 * activation; post_bounds[0..1] clamp after it (the next linear's input
 * clamp; bf16 output only).  A null array means +/-inf.  x_part_rows > 0
 * (parts > 1, >= m): part j reads its activations from x rows
 * [j*x_part_rows, j*x_part_rows + m) (per-part input clamps applied by the
 * producer of x); 0: every part reads rows [0, m).  Finite bounds need
 * out_mode 0 or 1 (out_mode 2 accumulates unclamped partial sums).
 * splits > 1 with out_mode 0 or 1: the K slices reduce-add into split_acc
 * (fp32 [m][out_features], zero on entry), then a finish pass applies the
 * bounds / SiLU, stores `out` and zeroes split_acc again -- how the listener
 * step runs its small-batch GEMMs.  split_acc may be NULL when splits == 1 or
 * out_mode == 2. */
int lb_op_gemm_clipped(const void* x, int x_ld, int m, int x_part_rows, const void* w, int w_int8,
                       const void* w_scale, const float* bias, int out_features, int k, void* out,
                       int ld_out, int out_mode, int act, int splits, int parts,
                       const float* out_bounds, const float* post_bounds, float* split_acc,
                       int* status_dev, void* stream);

/* ----------------------------------------------------------------------
 * Tick-level row selection (device arrays, asynchronous on `stream`).
 * ---------------------------------------------------------------------- */

/* One tick's rows over n_registered sessions in registration order.
 * Replaces SharedListenerTickDispatcher._snapshot_ready_rows
 * (duplex_kernel/shared_listener_scheduler.py:486-535): paused sessions are
 * skipped; a session's deferred frame is taken before its ingress head; a frame
 * enqueued after deadline_ns becomes (or stays) the deferred frame; every
 * other frame is a row.  Per session: paused, deferred_valid/_frame_id/
 * _enqueue_ns (updated in place), head_valid/_frame_id/_enqueue_ns (the
 * ingress queue head).  Outputs: rows_out[k] = registration index of row k
 * (registration order), row_frame_id_out[k], popped_out[i] = 1 when session
 * i's ingress head was consumed (the host pops it), *n_rows_out. */
int lb_snapshot_ready_rows(int n_registered, const uint8_t* paused, uint8_t* deferred_valid,
                           int64_t* deferred_frame_id, int64_t* deferred_enqueue_ns,
                           const uint8_t* head_valid, const int64_t* head_frame_id,
                           const int64_t* head_enqueue_ns, int64_t deadline_ns, int32_t* rows_out,
                           int64_t* row_frame_id_out, uint8_t* popped_out, int32_t* n_rows_out,
                           void* stream);

/* Dispatch order of the candidate heads (queue heads of sessions not in
 * flight).  Replaces ListenerMicrobatchCoordinator._candidate_heads_locked /
 * _take_ready_locked (duplex_kernel/listener_microbatch.py:170-201): heads with
 * ready_at_ns <= now_ns sorted by (ready_at_ns, submission_order, session id),
 * session_rank being the rank of the session id in string order; a single
 * ready head waits until ready_at + coalesce_ns.  Outputs perm_out[0..count)
 * (indices into the inputs), *count_out (0 = nothing dispatched) and
 * *reason_out: 0 none, 1 batch_full (count == n_registered), 2 multiple_ready,
 * 3 coalesce_deadline.  n_heads <= 8192 (else LB_ERR_CAPACITY). */
int lb_order_ready_heads(int n_heads, const int64_t* ready_at_ns, const int64_t* submission_order,
                         const int32_t* session_rank, int64_t now_ns, int64_t coalesce_ns,
                         int n_registered, int32_t* perm_out, int32_t* count_out, int32_t* reason_out,
                         void* stream);

/* lb_op_gemm's split-K form with a bf16 output [m, ld_out] and no
 * caller-supplied accumulator: the fp32 partial sums of the `splits` K slices
 * are reduce-added into a fixed device array inside the library (8 MiB, i.e.
 * m * out_features <= 2097152 fp32 values; larger sizes return
 * LB_ERR_CAPACITY), then rounded to bf16 (act 1: SiLU of the bf16-rounded sum).
 * Nothing is allocated by any call.  The first call on a device (that device
 * current) resolves the array's address and sets the GEMM kernel attributes,
 * so make it before any stream capture.  There is one array per device:
 * calls that overlap on the GPU race.  x / w / w_scale / bias as lb_op_gemm.
 * `out` is undefined whenever *status_dev != 0 after the call (the GEMM gave
 * up on a bounded wait): the rounding pass then leaves it unwritten.
 * No counterpart in the reference: it exists for callers that must not
 * allocate device memory per call. */
int lb_op_gemm_splitk_scratch(const void* x, int x_ld, int m, const void* w, int w_int8,
                              const void* w_scale, const float* bias, int out_features, int k,
                              void* out, int ld_out, int act, int splits, int* status_dev,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LISTENER_B200_H_ */
