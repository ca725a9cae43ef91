// Step-level C ABI: context lifetime, weight upload, pack / step / commit.
//
// One lb_step_async runs the whole listener step for the packed rows.  The
// kernel sequence of a step is captured once per (row bucket, input kind,
// FiLM on/off) into a CUDA graph and replayed; every kernel reads the row
// count from device memory, so one graph serves every batch size up to its
// bucket (buckets are powers of two up to max_rows).  This replaces the
// reference's one-graph-per-N capture (streaming_conformer.py:453-532) and its
// fixed N in {1,2,4} coalescing.
#include "common.cuh"
#include "listener.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>

struct lb_ctx {
  lb::Ctx c;
  // per-bucket, per-variant GEMM plans and graphs
  struct LayerOps {
    lb::GemmOp ffn1[2], ffn2[2], qkv, post, lstart, lend;
  };
  struct Plans {
    bool built = false;
    lb::GemmOp in_proj, out_proj, embed, qdown, rdown, film, fout;
    std::vector<LayerOps> layers;
    // graph[0], graph[1]: the tower (PCM / mel input) through the soft tokens;
    // graph[2]: the FiLM chain, launched after the query has landed
    cudaGraphExec_t graph[3] = {nullptr, nullptr, nullptr};
    int graph_kernels[3] = {0, 0, 0};
  };
  int last_graph_kernels = 0;
  // side stream for the copies that need not sit on the step's critical path
  // (query H2D under the tower, soft/raw D2H under FiLM), joined back into the
  // caller's stream at the end of every step
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_begin = nullptr, ev_query = nullptr, ev_tower = nullptr, ev_copies = nullptr;
  std::vector<Plans> plans;
  // pinned staging for lb_step_host
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  std::vector<std::string> names;
  float qkv_bounds[64][3][4];
  // host-side call counters (lb_get_counters)
  unsigned long long n_pack = 0, n_step = 0, n_commit = 0, n_abort = 0, n_rollback = 0, n_reset = 0;
  unsigned long long rows_stepped = 0;
};

using namespace lb;

namespace lb {
cudaError_t gemm_init_attributes();
cudaError_t frontend_init_attributes();
cudaError_t attention_init_attributes();
}  // namespace lb

namespace {

constexpr int kLinFfn1a = 0, kLinFfn1b = 1, kLinFfn2a = 2, kLinFfn2b = 3, kLinQkv = 4,
              kLinPost = 5, kLinStart = 6, kLinEnd = 7;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Arena {
  size_t off = 0;
  char* base = nullptr;
  template <typename T>
  T* take(size_t count, size_t align = 256) {
    off = align_up(off, align);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

bool check_cfg(const lb_config* cfg) {
  if (!cfg) return false;
  const int d = cfg->hidden;
  if (cfg->max_sessions < 2 || cfg->max_rows < 1 || cfg->max_rows > cfg->max_sessions) return false;
  if (cfg->max_handles < cfg->max_sessions) return false;
  if (d <= 0 || cfg->heads <= 0 || d % cfg->heads) return false;
  const int hd = d / cfg->heads;
  if (hd % 64 || hd > 256 || cfg->heads > 16) return false;
  if (d % 256 || cfg->ffn % 128 || cfg->output_dims % 256 || cfg->text_hidden % 256) return false;
  if (d > 2048 || d / 256 == 7) return false;  // row kernels are instantiated for d/256 in {1..6, 8}
  if (cfg->sub_ch0 != 128 || cfg->sub_ch1 != 32 || cfg->conv_kernel != 5) return false;
  if (cfg->layers < 1 || cfg->layers > 64) return false;
  if (cfg->weight_format != LB_WEIGHTS_BF16 && cfg->weight_format != LB_WEIGHTS_INT8) return false;
  if (cfg->film_enabled && (cfg->film_query_dim % 256 || cfg->film_bottleneck % 128)) return false;
  return true;
}

// Registers one GEMM weight [rows, cols]: bf16 data or int8 + fp16 scale.
void reg_gemm(lb_ctx* x, Arena& a, const std::string& name, int rows, int cols, void** data,
              __half** scale, bool assign, int qkv_part = -1, void* qkv_base = nullptr,
              __half* qkv_scale = nullptr) {
  Ctx& c = x->c;
  const bool i8 = c.weight_int8 != 0;
  TensorSlot t;
  t.gemm = true;
  t.qkv_part = qkv_part;
  t.dtype = i8 ? LB_I8 : LB_BF16;
  t.numel = static_cast<int64_t>(rows) * cols;
  TensorSlot s;
  s.dtype = LB_F16;
  s.numel = rows;
  if (qkv_part >= 0) {
    const size_t off = static_cast<size_t>(qkv_part) * rows * cols;
    t.dst = assign ? static_cast<char*>(qkv_base) + off * (i8 ? 1 : 2) : nullptr;
    s.dst = assign && i8 ? qkv_scale + static_cast<size_t>(qkv_part) * rows : nullptr;
  } else {
    void* p = i8 ? static_cast<void*>(a.take<int8_t>(t.numel, 1024))
                 : static_cast<void*>(a.take<__nv_bfloat16>(t.numel, 1024));
    __half* sp = i8 ? a.take<__half>(rows) : nullptr;
    if (assign) {
      *data = p;
      *scale = sp;
    }
    t.dst = p;
    s.dst = sp;
  }
  if (assign) {
    c.tensors[name] = t;
    if (i8) c.tensors[name + ":scale"] = s;
  }
}

float* reg_f32(lb_ctx* x, Arena& a, const std::string& name, int64_t numel, bool assign) {
  float* p = a.take<float>(numel);
  if (assign) {
    TensorSlot t;
    t.dst = p;
    t.dtype = LB_F32;
    t.numel = numel;
    x->c.tensors[name] = t;
  }
  return p;
}

void reg_clip(lb_ctx* x, const std::string& prefix, float* dst4) {
  static const char* kNames[4] = {"input_min", "input_max", "output_min", "output_max"};
  for (int i = 0; i < 4; ++i) {
    dst4[i] = (i % 2 == 0) ? -INFINITY : INFINITY;  // unclipped unless uploaded
    TensorSlot t;
    t.dst = nullptr;
    t.dtype = LB_F32;
    t.numel = 1;
    t.clip_dst = dst4 + i;
    t.set = true;  // optional: defaults to +/-inf
    x->c.tensors[prefix + "." + kNames[i]] = t;
  }
}

// Lays out (assign=false: sizes only) or assigns every weight slot.
size_t layout_weights(lb_ctx* x, char* base, bool assign) {
  Ctx& c = x->c;
  const lb_config& g = c.cfg;
  const int d = g.hidden, F = g.ffn, hd = d / g.heads;
  Arena a;
  a.base = base;
  Weights& w = c.w;
  if (assign) w.layers.resize(g.layers);
  const std::string s = "subsample_conv_projection";
  float* conv0 = reg_f32(x, a, s + ".layer0.conv.weight", 128 * 9, assign);
  float* ln0 = reg_f32(x, a, s + ".layer0.norm.weight", 128, assign);
  __nv_bfloat16* conv1 = a.take<__nv_bfloat16>(static_cast<size_t>(g.sub_ch1) * (9 * 128 + 8));
  float* ln1 = reg_f32(x, a, s + ".layer1.norm.weight", g.sub_ch1, assign);
  if (assign) {
    w.conv0 = conv0;
    w.ln0 = ln0;
    w.conv1 = conv1;
    w.ln1 = ln1;
    TensorSlot t;  // converted on upload: [C1][128][3][3] f32 -> [C1][(i*3+j)*128+ci] bf16
    t.dst = conv1;
    t.dtype = LB_F32;
    t.numel = static_cast<int64_t>(g.sub_ch1) * 128 * 9;
    c.tensors[s + ".layer1.conv.weight"] = t;
  }
  reg_gemm(x, a, s + ".input_proj_linear.weight", d, g.sub_ch1 * 32, &w.w_in, &w.s_in, assign);
  for (int i = 0; i < g.layers; ++i) {
    const std::string p = "layers." + std::to_string(i);
    LayerW dummy{};
    LayerW& L = assign ? w.layers[i] : dummy;
    for (int f = 0; f < 2; ++f) {
      const std::string ff = p + (f == 0 ? ".feed_forward1" : ".feed_forward2");
      reg_gemm(x, a, ff + ".ffw_layer_1.linear.weight", F, d, &L.w_ffn1[f], &L.s_ffn1[f], assign);
      reg_gemm(x, a, ff + ".ffw_layer_2.linear.weight", d, F, &L.w_ffn2[f], &L.s_ffn2[f], assign);
      float* pre = reg_f32(x, a, ff + ".pre_layer_norm.weight", d, assign);
      float* post = reg_f32(x, a, ff + ".post_layer_norm.weight", d, assign);
      if (assign) {
        L.ffn_pre[f] = pre;
        L.ffn_post[f] = post;
        reg_clip(x, ff + ".ffw_layer_1", L.clip[f == 0 ? kLinFfn1a : kLinFfn2a]);
        reg_clip(x, ff + ".ffw_layer_2", L.clip[f == 0 ? kLinFfn1b : kLinFfn2b]);
      }
    }
    // fused Q/K/V weight [3d, d]
    const bool i8 = c.weight_int8 != 0;
    void* qkv = i8 ? static_cast<void*>(a.take<int8_t>(static_cast<size_t>(3) * d * d, 1024))
                   : static_cast<void*>(a.take<__nv_bfloat16>(static_cast<size_t>(3) * d * d, 1024));
    __half* qkv_s = i8 ? a.take<__half>(3 * d) : nullptr;
    if (assign) {
      L.w_qkv = qkv;
      L.s_qkv = qkv_s;
      const char* parts[3] = {"q_proj", "k_proj", "v_proj"};
      for (int q = 0; q < 3; ++q) {
        const std::string n = p + ".self_attn." + parts[q];
        reg_gemm(x, a, n + ".linear.weight", d, d, nullptr, nullptr, true, q, qkv, qkv_s);
        for (int k = 0; k < 4; ++k) x->qkv_bounds[i][q][k] = (k % 2 == 0) ? -INFINITY : INFINITY;
        reg_clip(x, n, x->qkv_bounds[i][q]);
      }
    }
    reg_gemm(x, a, p + ".self_attn.post.linear.weight", d, d, &L.w_post, &L.s_post, assign);
    float* rel = reg_f32(x, a, p + ".self_attn.relative_keys", 13 * d, assign);
    float* qm = reg_f32(x, a, p + ".self_attn.query_scale", hd, assign);
    reg_gemm(x, a, p + ".lconv1d.linear_start.linear.weight", 2 * d, d, &L.w_lstart, &L.s_lstart, assign);
    reg_gemm(x, a, p + ".lconv1d.linear_end.linear.weight", d, d, &L.w_lend, &L.s_lend, assign);
    float* dw = reg_f32(x, a, p + ".lconv1d.depthwise_conv1d.weight", d * 5, assign);
    float* lpre = reg_f32(x, a, p + ".lconv1d.pre_layer_norm.weight", d, assign);
    float* lnorm = reg_f32(x, a, p + ".lconv1d.conv_norm.weight", d, assign);
    float* npa = reg_f32(x, a, p + ".norm_pre_attn.weight", d, assign);
    float* npo = reg_f32(x, a, p + ".norm_post_attn.weight", d, assign);
    float* nout = reg_f32(x, a, p + ".norm_out.weight", d, assign);
    if (assign) {
      L.rel_keys = rel;
      L.q_mult = qm;
      L.lc_dw = dw;
      L.lc_pre = lpre;
      L.lc_norm = lnorm;
      L.norm_pre_attn = npa;
      L.norm_post_attn = npo;
      L.norm_out = nout;
      reg_clip(x, p + ".self_attn.post", L.clip[kLinPost]);
      reg_clip(x, p + ".lconv1d.linear_start", L.clip[kLinStart]);
      reg_clip(x, p + ".lconv1d.linear_end", L.clip[kLinEnd]);
      for (int k = 0; k < 8; ++k)
        if (k != kLinQkv) { /* filled by reg_clip or defaults below */ }
    }
  }
  reg_gemm(x, a, "output_proj.weight", g.output_dims, d, &w.w_out, &w.s_out, assign);
  float* bout = reg_f32(x, a, "output_proj.bias", g.output_dims, assign);
  reg_gemm(x, a, "embed.embedding_projection.weight", g.text_hidden, g.output_dims, &w.w_embed,
           &w.s_embed, assign);
  if (assign) w.b_out = bout;
  if (g.film_enabled) {
    const int Q = g.film_query_dim, B = g.film_bottleneck, T = g.text_hidden;
    float* qw = reg_f32(x, a, "film.query_norm.weight", Q, assign);
    float* qb = reg_f32(x, a, "film.query_norm.bias", Q, assign);
    float* rw = reg_f32(x, a, "film.response_norm.weight", T, assign);
    float* rb = reg_f32(x, a, "film.response_norm.bias", T, assign);
    reg_gemm(x, a, "film.query_down.weight", B, Q, &w.w_qdown, &w.s_qdown, assign);
    reg_gemm(x, a, "film.response_down.weight", B, T, &w.w_rdown, &w.s_rdown, assign);
    reg_gemm(x, a, "film.film.weight", 2 * B, B, &w.w_film, &w.s_film, assign);
    reg_gemm(x, a, "film.output.weight", Q, B, &w.w_fout, &w.s_fout, assign);
    float* bqd = reg_f32(x, a, "film.query_down.bias", B, assign);
    float* brd = reg_f32(x, a, "film.response_down.bias", B, assign);
    float* bf = reg_f32(x, a, "film.film.bias", 2 * B, assign);
    float* bo = reg_f32(x, a, "film.output.bias", Q, assign);
    if (assign) {
      w.fq_norm_w = qw;
      w.fq_norm_b = qb;
      w.fr_norm_w = rw;
      w.fr_norm_b = rb;
      w.b_qdown = bqd;
      w.b_rdown = brd;
      w.b_film = bf;
      w.b_fout = bo;
      TensorSlot t;
      t.dst = nullptr;
      t.dtype = LB_F32;
      t.numel = 1;
      t.clip_dst = &w.film_scale;  // host scalar; converted from scale_logit on upload
      c.tensors["film.scale_logit"] = t;
    }
  }
  // frontend tables
  float* win = reg_f32(x, a, "frontend.window", 320, assign);
  float* filt = reg_f32(x, a, "frontend.mel_filters", 257 * 128, assign);
  float* ct = a.take<float>(512);
  float* st = a.take<float>(512);
  int2* rng = a.take<int2>(128);
  if (assign) {
    c.fe_window = win;
    c.fe_filters = filt;
    c.fe_cos = ct;
    c.fe_sin = st;
    c.fe_range = rng;
  }
  return align_up(a.off, 4096);
}

size_t layout_state(Ctx& c, char* base) {
  const lb_config& g = c.cfg;
  const size_t S = g.max_sessions, L = g.layers, d = g.hidden, H = c.max_handles;
  const size_t R = g.max_rows, T = 2 * R;
  Arena a;
  a.base = base;
  auto kk = a.take<__nv_bfloat16>(S * L * (kRing * d + kRingPad), 4096);
  auto vv = a.take<__nv_bfloat16>(S * L * (kRing * d + kRingPad), 4096);
  auto cr = a.take<__nv_bfloat16>(S * L * (kConvRing * d + kRingPad), 4096);
  auto sp = a.take<__nv_bfloat16>(S * 2 * 64 * 128);
  auto mp = a.take<float>(S * 2 * kMelBins);
  auto pt = a.take<float>(S * 2 * kTail);
  auto m0 = a.take<SlotMeta>(S);
  auto m1 = a.take<SlotMeta>(S);
  auto m2 = a.take<SlotMeta>(S);
  auto hs = a.take<int>(H);
  auto so = a.take<int>(S);
  auto hk = a.take<long long>(H);
  auto hf = a.take<long long>(H);
  auto hq = a.take<long long>(H);
  auto hst = a.take<long long>(H);
  auto bhs = a.take<int>(R);
  auto bhk = a.take<long long>(R);
  auto bhf = a.take<long long>(R);
  auto bhq = a.take<long long>(R);
  auto bso = a.take<int>(R);
  auto cnt = a.take<int>(8);
  auto sta = a.take<int>(8);
  auto ctr = a.take<unsigned long long>(8);
  auto rh = a.take<int>(R);
  auto rs = a.take<int>(R);
  auto rr = a.take<int>(R);
  auto rst = a.take<int>(R);
  auto rm = a.take<int>(R);
  auto rrep = a.take<int>(R);
  auto rmi = a.take<uint8_t>(R);
  auto rme = a.take<SlotMeta>(R);
  auto rk = a.take<long long>(R);
  auto rf = a.take<long long>(R);
  auto rq = a.take<long long>(R);
  auto ref = a.take<long long>(R);
  auto req = a.take<long long>(R);
  auto fl = a.take<int>(S);
  if (base) {
    c.kv_k = kk; c.kv_v = vv; c.conv_ring = cr; c.sub_prev = sp; c.mel_prev = mp; c.pcm_tail = pt;
    c.meta_canon = m0; c.meta_stage = m1; c.meta_backup = m2;
    c.handle_slot = hs; c.slot_owner = so; c.handle_key = hk; c.handle_exp_frame = hf;
    c.handle_exp_seq = hq; c.handle_stamp = hst;
    c.bk_handle_slot = bhs; c.bk_handle_key = bhk; c.bk_handle_exp_frame = bhf;
    c.bk_handle_exp_seq = bhq; c.bk_slot_owner = bso;
    c.dev_counts = cnt; c.status = sta; c.dev_ctr = ctr;
    c.row_handle = rh; c.row_slot = rs; c.row_reason = rr; c.row_reset = rst; c.row_mask = rm;
    c.row_replacing = rrep; c.row_mask_in = rmi; c.row_meta = rme; c.row_key = rk; c.row_frame = rf;
    c.row_seq = rq; c.row_exp_frame = ref; c.row_exp_seq = req; c.free_list = fl;
  }
  (void)T;
  return align_up(a.off, 4096);
}

size_t layout_acts(Ctx& c, char* base) {
  const lb_config& g = c.cfg;
  const size_t R = g.max_rows, T = 2 * R, d = g.hidden, F = g.ffn;
  const size_t O = g.output_dims, TX = g.text_hidden, Q = g.film_query_dim, B = g.film_bottleneck;
  const size_t wide = std::max({F, 3 * d, 2 * d, B});
  const size_t narrow = std::max({d, O, TX, Q, 2 * B});
  Arena a;
  a.base = base;
  auto pcm = a.take<float>(R * kPcm);
  auto mel = a.take<float>(R * 8 * kMelBins);
  auto qry = a.take<__nv_bfloat16>(T * Q);
  auto sub = a.take<__nv_bfloat16>(T * 32 * 32);
  auto h = a.take<float>(T * d);
  auto y = a.take<float>(T * narrow);
  auto xa = a.take<__nv_bfloat16>(3 * T * d);  // [3][T][d]: blocks 1, 2 only for split Q/K/V inputs
  auto xf = a.take<__nv_bfloat16>(T * F);
  auto qkv = a.take<__nv_bfloat16>(T * 3 * d);
  auto att = a.take<__nv_bfloat16>(T * d);
  auto gl = a.take<__nv_bfloat16>(T * 2 * d);
  auto wa = a.take<float>(T * wide);
  auto oraw = a.take<__nv_bfloat16>(T * O);
  auto osoft = a.take<__nv_bfloat16>(T * TX);
  auto ofilm = a.take<__nv_bfloat16>(T * Q);
  auto fxq = a.take<__nv_bfloat16>(T * Q);
  auto fxr = a.take<__nv_bfloat16>(T * TX);
  auto fqd = a.take<float>(T * B);
  auto frb = a.take<__nv_bfloat16>(T * B);
  auto fgb = a.take<float>(T * 2 * B);
  auto ffu = a.take<__nv_bfloat16>(T * B);
  auto fmap = a.take<float>(T * Q);
  auto famp = a.take<float>(T);
  auto xe = a.take<__nv_bfloat16>(T * O);
  if (base) {
    c.in_pcm = pcm; c.in_mel = mel; c.in_query = qry; c.sub_in = sub; c.h = h; c.y = y; c.xa = xa;
    c.xf = xf; c.qkv = qkv; c.att = att; c.gl = gl; c.wide_acc = wa; c.out_raw = oraw;
    c.wide_width = static_cast<int>(wide);
    c.out_soft = osoft; c.out_film = ofilm; c.film_xq = fxq; c.film_xr = fxr; c.film_qd = fqd;
    c.film_rd_bf = frb; c.film_gb = fgb; c.film_fused = ffu; c.film_map = fmap; c.film_amp = famp;
    c.xe = xe;
  }
  return align_up(a.off, 4096);
}

// ------------------------------------------------------------- GEMM plans
int make_op(Ctx& c, GemmOp& op, void* w, const __half* scale, int O, int K, const void* x, int tok_cap,
            const float* bias, void* out, int out_kind, int act, const float* clip4,
            float post_lo = -INFINITY, float post_hi = INFINITY, const LayerW* qkv = nullptr,
            bool consumer_finishes = false) {
  // out_kind: 0 = bf16 tensor, 1 = fp32, 2 = activation that feeds another GEMM
  // (bf16, or fp16 when the weights are int8)
  op.final_f16 = out_kind == 2 && c.f16_acts;
  // int8 weights: buckets of >= wide_min_tokens tokens read the fp16 codes
  // bf16 weights: every bucket reads their exact fp16 copy (same offsets), no scale
  int w_kind = 0;
  if (c.weight_int8) {
    w_kind = 1;
    if (c.wide_arena && tok_cap >= c.wide_min_tokens) {
      w_kind = 2;
      w = static_cast<char*>(c.wide_arena) +
          2 * (static_cast<char*>(w) - static_cast<char*>(c.weight_arena));
    }
  } else if (c.wide_arena) {
    w_kind = 2;
    w = static_cast<char*>(c.wide_arena) + (static_cast<char*>(w) - static_cast<char*>(c.weight_arena));
    scale = nullptr;
  }
  if (out_kind == 2) out_kind = 0;
  op.pdl = c.pdl;
  GemmParams& p = op.params;
  p = GemmParams();
  p.m_dev = c.dev_counts + 1;
  p.w_scale = scale;
  p.bias = bias;
  p.act = act;
  p.status = c.status;
  p.ld_out = O;
  if (clip4) {
    p.out_lo = clip4[2];
    p.out_hi = clip4[3];
  }
  p.post_lo = post_lo;
  p.post_hi = post_hi;
  // the fused Q/K/V linear: three stacked parts of O/3 features, each with its
  // own output clamp and, when their input clamps differ, its own input block
  int x_parts = 1;
  bool finite_out = std::isfinite(p.out_lo) || std::isfinite(p.out_hi);
  if (qkv && (qkv->qkv_split_out || qkv->qkv_split_in)) {
    p.part_o = O / 3;
    for (int j = 0; j < 3; ++j) {
      p.part_lo[j] = qkv->qkv_clip[j][2];
      p.part_hi[j] = qkv->qkv_clip[j][3];
      finite_out = finite_out || std::isfinite(p.part_lo[j]) || std::isfinite(p.part_hi[j]);
    }
    if (qkv->qkv_split_in) {
      x_parts = 3;
      p.x_part_rows = 2 * c.cfg.max_rows;
    }
  }
  (void)finite_out;  // the finish pass of a split-K op clamps
  op.splits = gemm_pick_splits(O, K, tok_cap, c.num_sms);
  const int tn = gemm_token_tile(O, tok_cap, c.num_sms);
  const int tiles = (O / 128) * ((tok_cap + tn - 1) / tn);
  // A split output goes through the fp32 partial-sum buffer and one finish
  // pass; worth it only while the tiles cannot fill half of the SMs.
  if (tiles * 2 >= c.num_sms || O > c.wide_width) op.splits = 1;
  op.out_kind = out_kind;
  op.out = out;
  op.consumer_finishes = false;
  if (op.splits > 1) {
    // K slices reduce-add into the context's partial-sum buffer (kept zero:
    // every finish pass zeroes what it read), then the finish pass (run_op)
    // or the consuming row kernel
    op.consumer_finishes = consumer_finishes;
    p.out_mode = 2;
    p.out = c.wide_acc;
    p.ld_out = O;
  } else {
    p.out_mode = out_kind == 0 ? 0 : 1;
    p.out = out;
  }
  return gemm_prepare(&op.plan, w, w_kind, O, K, x, K, tok_cap, p.out, O, p.out_mode,
                      op.final_f16, x_parts, p.x_part_rows);
}

// One GEMM launch, plus the finish pass of a split-K op (clamps, SiLU, the
// output store and the re-zeroing of the partial-sum buffer).  No memset: the
// partial-sum buffer is zero at creation and after every finish pass.
cudaError_t run_op(Ctx& c, const GemmOp& op, int tok_cap, cudaStream_t s) {
  cudaError_t e = gemm_launch(op.plan, op.params, op.splits, s, op.pdl);
  if (e != cudaSuccess || op.splits <= 1 || op.consumer_finishes) return e;
  FinalizeClip fc;
  fc.part_o = op.params.part_o;
  for (int j = 0; j < 3; ++j) {
    fc.lo[j] = fc.part_o ? op.params.part_lo[j] : op.params.out_lo;
    fc.hi[j] = fc.part_o ? op.params.part_hi[j] : op.params.out_hi;
  }
  fc.plo = op.params.post_lo;
  fc.phi = op.params.post_hi;
  return launch_split_finish(c.dev_counts + 1, 0, tok_cap, c.wide_acc, op.plan.O, op.params.act, op.out,
                             op.plan.O, op.out_kind == 1, op.final_f16, fc, c.pdl_all, s);
}

int build_plans(lb_ctx* x, int bi) {
  Ctx& c = x->c;
  lb_ctx::Plans& P = x->plans[bi];
  if (P.built) return 0;
  const lb_config& g = c.cfg;
  const int d = g.hidden, F = g.ffn, tc = c.buckets[bi].tok_cap;
  const float inf = INFINITY;
  int rc = 0;
  rc |= make_op(c, P.in_proj, c.w.w_in, c.w.s_in, d, g.sub_ch1 * 32, c.sub_in, tc, nullptr, c.h, 1, 0, nullptr);
  P.layers.resize(g.layers);
  for (int i = 0; i < g.layers; ++i) {
    LayerW& L = c.w.layers[i];
    lb_ctx::LayerOps& o = P.layers[i];
    for (int f = 0; f < 2; ++f) {
      const float* c1 = L.clip[f == 0 ? kLinFfn1a : kLinFfn2a];
      const float* c2 = L.clip[f == 0 ? kLinFfn1b : kLinFfn2b];
      GemmOp& a1 = f == 0 ? o.ffn1[0] : o.ffn2[0];
      GemmOp& a2 = f == 0 ? o.ffn1[1] : o.ffn2[1];
      rc |= make_op(c, a1, L.w_ffn1[f], L.s_ffn1[f], F, d, c.xa, tc, nullptr, c.xf, 2, 1, c1, c2[0], c2[1]);
      rc |= make_op(c, a2, L.w_ffn2[f], L.s_ffn2[f], d, F, c.xf, tc, nullptr, c.y, 1, 0, c2, -INFINITY, INFINITY,
                    nullptr, true);
    }
    rc |= make_op(c, o.qkv, L.w_qkv, L.s_qkv, 3 * d, d, c.xa, tc, nullptr, c.qkv, 0, 0, L.clip[kLinQkv],
                  -INFINITY, INFINITY, &L);
    rc |= make_op(c, o.post, L.w_post, L.s_post, d, d, c.att, tc, nullptr, c.y, 1, 0, L.clip[kLinPost], -INFINITY,
                  INFINITY, nullptr, true);
    rc |= make_op(c, o.lstart, L.w_lstart, L.s_lstart, 2 * d, d, c.xa, tc, nullptr, c.gl, 0, 0, L.clip[kLinStart]);
    rc |= make_op(c, o.lend, L.w_lend, L.s_lend, d, d, c.xa, tc, nullptr, c.y, 1, 0, L.clip[kLinEnd], -INFINITY,
                  INFINITY, nullptr, true);
  }
  rc |= make_op(c, P.out_proj, c.w.w_out, c.w.s_out, g.output_dims, d, c.xa, tc, c.w.b_out, c.y, 1, 0, nullptr);
  rc |= make_op(c, P.embed, c.w.w_embed, c.w.s_embed, g.text_hidden, g.output_dims, c.xe, tc, nullptr, c.y, 1, 0, nullptr);
  if (g.film_enabled) {
    const int Q = g.film_query_dim, B = g.film_bottleneck, T = g.text_hidden;
    rc |= make_op(c, P.qdown, c.w.w_qdown, c.w.s_qdown, B, Q, c.film_xq, tc, c.w.b_qdown, c.film_qd, 1, 0, nullptr);
    rc |= make_op(c, P.rdown, c.w.w_rdown, c.w.s_rdown, B, T, c.film_xr, tc, c.w.b_rdown, c.film_rd_bf, 2, 1, nullptr);
    rc |= make_op(c, P.film, c.w.w_film, c.w.s_film, 2 * B, B, c.film_rd_bf, tc, c.w.b_film, c.film_gb, 1, 0, nullptr);
    rc |= make_op(c, P.fout, c.w.w_fout, c.w.s_fout, Q, B, c.film_fused, tc, c.w.b_fout, c.film_map, 1, 0, nullptr);
  }
  (void)inf;
  if (rc) return LB_ERR_CUDA;
  P.built = true;
  return 0;
}

// The row kernel after an op that writes y: from y itself, or from the
// split-K partial sums, which it then finishes (output clamp) and re-zeroes.
void bind_y(Ctx& c, const GemmOp& op, RowFusedArgs& r) {
  if (op.splits > 1 && op.consumer_finishes) {
    r.y = c.wide_acc;
    r.zero_y = true;
    r.y_lo = op.params.out_lo;
    r.y_hi = op.params.out_hi;
  } else {
    r.y = c.y;
  }
}

// Diagnostics only (eager runs): return after stage `k` of layer `i`.
#define LB_STOP(i, k)                                                        \
  do {                                                                       \
    if (c.dbg_stop_layer == (i) && c.dbg_stop_stage == (k)) return cudaSuccess; \
  } while (0)

#define LB_TRY(expr)                         \
  do {                                       \
    cudaError_t _e = (expr);                 \
    if (_e != cudaSuccess) return _e;        \
  } while (0)

// The tower: frontend, Conformer, output projection and embedder (soft tokens).
cudaError_t run_tower(lb_ctx* x, int bi, int input_kind, cudaStream_t s) {
  Ctx& c = x->c;
  lb_ctx::Plans& P = x->plans[bi];
  const Bucket& b = c.buckets[bi];
  const lb_config& g = c.cfg;
  const int tc = b.tok_cap, rc = b.rows_cap, d = g.hidden;
  LB_TRY(launch_mel(c, rc, input_kind, s));
  LB_TRY(launch_subsample(c, rc, s));
  LB_TRY(run_op(c, P.in_proj, tc, s));
  {
    RowFusedArgs r;
    r.pre_w = c.w.layers[0].ffn_pre[0];
    r.in_lo = c.w.layers[0].clip[kLinFfn1a][0];
    r.in_hi = c.w.layers[0].clip[kLinFfn1a][1];
    r.xa = c.xa;
    r.dbg = c.dbg_sub;
    LB_TRY(launch_row_fused(c, tc, r, s));
  }
  const size_t layer_stride = static_cast<size_t>(c.packed_rows) * 2 * d;
  for (int i = 0; i < g.layers; ++i) {
    LayerW& L = c.w.layers[i];
    lb_ctx::LayerOps& o = P.layers[i];
    // FFN1
    LB_TRY(run_op(c, o.ffn1[0], tc, s));
    LB_STOP(i, 0);
    LB_TRY(run_op(c, o.ffn1[1], tc, s));
    LB_STOP(i, 1);
    {
      RowFusedArgs r;
      bind_y(c, o.ffn1[1], r);
      r.post_w = L.ffn_post[0];
      r.alpha = g.residual_weight;
      r.pre_w = L.norm_pre_attn;
      r.in_lo = L.clip[kLinQkv][0];
      r.in_hi = L.clip[kLinQkv][1];
      if (L.qkv_split_in) {  // k_proj / v_proj inputs in blocks 1 and 2
        r.xa_parts = 3;
        for (int j = 0; j < 2; ++j) {
          r.part_lo[j] = L.qkv_clip[j + 1][0];
          r.part_hi[j] = L.qkv_clip[j + 1][1];
        }
      }
      r.xa = c.xa;
      LB_TRY(launch_row_fused(c, tc, r, s));
    }
    LB_STOP(i, 2);
    // attention
    LB_TRY(run_op(c, o.qkv, tc, s));
    LB_STOP(i, 3);
    LB_TRY(launch_attention(c, i, rc, s));
    LB_STOP(i, 4);
    LB_TRY(run_op(c, o.post, tc, s));
    LB_STOP(i, 5);
    {
      RowFusedArgs r;
      bind_y(c, o.post, r);
      r.post_w = L.norm_post_attn;
      r.pre_w = L.lc_pre;
      r.pre_clamp = false;
      r.in_lo = L.clip[kLinStart][0];
      r.in_hi = L.clip[kLinStart][1];
      r.xa = c.xa;
      LB_TRY(launch_row_fused(c, tc, r, s));
    }
    LB_STOP(i, 6);
    // light conv
    LB_TRY(run_op(c, o.lstart, tc, s));
    LB_STOP(i, 7);
    LB_TRY(launch_lconv(c, i, rc, s));
    LB_STOP(i, 8);
    LB_TRY(run_op(c, o.lend, tc, s));
    LB_STOP(i, 9);
    {
      RowFusedArgs r;
      bind_y(c, o.lend, r);
      r.pre_w = L.ffn_pre[1];
      r.in_lo = L.clip[kLinFfn2a][0];
      r.in_hi = L.clip[kLinFfn2a][1];
      r.xa = c.xa;
      LB_TRY(launch_row_fused(c, tc, r, s));
    }
    LB_STOP(i, 10);
    // FFN2 + norm_out (+ next layer's FFN1 pre-norm, or plain bf16 for output_proj)
    LB_TRY(run_op(c, o.ffn2[0], tc, s));
    LB_STOP(i, 11);
    LB_TRY(run_op(c, o.ffn2[1], tc, s));
    LB_STOP(i, 12);
    {
      RowFusedArgs r;
      bind_y(c, o.ffn2[1], r);
      r.post_w = L.ffn_post[1];
      r.alpha = g.residual_weight;
      r.out_w = L.norm_out;
      if (i + 1 < g.layers) {
        r.pre_w = c.w.layers[i + 1].ffn_pre[0];
        r.in_lo = c.w.layers[i + 1].clip[kLinFfn1a][0];
        r.in_hi = c.w.layers[i + 1].clip[kLinFfn1a][1];
      } else {
        r.pre_norm = false;
        r.pre_clamp = false;
      }
      r.xa = c.xa;
      r.dbg = c.dbg_layers ? c.dbg_layers + i * layer_stride : nullptr;
      LB_TRY(launch_row_fused(c, tc, r, s));
    }
  }
  LB_TRY(run_op(c, P.out_proj, tc, s));
  LB_TRY(launch_outputs(c, tc, 0, s));
  LB_TRY(run_op(c, P.embed, tc, s));
  LB_TRY(launch_outputs(c, tc, 1, s));
  return cudaSuccess;
}

// The FiLM adapter over the soft tokens and the query.
cudaError_t run_film(lb_ctx* x, int bi, cudaStream_t s) {
  Ctx& c = x->c;
  lb_ctx::Plans& P = x->plans[bi];
  const int tc = c.buckets[bi].tok_cap;
  LB_TRY(launch_film(c, tc, 0, s));
  LB_TRY(run_op(c, P.qdown, tc, s));
  LB_TRY(run_op(c, P.rdown, tc, s));
  LB_TRY(run_op(c, P.film, tc, s));
  LB_TRY(launch_film(c, tc, 1, s));
  LB_TRY(run_op(c, P.fout, tc, s));
  LB_TRY(launch_film(c, tc, 2, s));
  return cudaSuccess;
}

// Captures `part` (0/1: the tower for that input kind, 2: FiLM) of bucket bi once.
int ensure_graph(lb_ctx* x, int bi, int part) {
  Ctx& c = x->c;
  lb_ctx::Plans& P = x->plans[bi];
  if (P.graph[part]) return LB_OK;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(c.capture_stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return LB_ERR_CUDA;
  cudaError_t e_run = part == 2 ? run_film(x, bi, c.capture_stream) : run_tower(x, bi, part, c.capture_stream);
  e = cudaStreamEndCapture(c.capture_stream, &graph);
  if (e_run != cudaSuccess || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return LB_ERR_CUDA;
  }
  size_t num_nodes = 0;
  cudaGraphGetNodes(graph, nullptr, &num_nodes);
  std::vector<cudaGraphNode_t> nodes(num_nodes);
  cudaGraphGetNodes(graph, nodes.data(), &num_nodes);
  int kernels = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
  }
  P.graph_kernels[part] = kernels;
  e = cudaGraphInstantiate(&P.graph[part], graph, 0);
  cudaGraphDestroy(graph);
  return e == cudaSuccess ? LB_OK : LB_ERR_CUDA;
}

int pick_bucket(Ctx& c, int n) {
  for (size_t i = 0; i < c.buckets.size(); ++i)
    if (c.buckets[i].rows_cap >= n) return static_cast<int>(i);
  return -1;
}

int err_of(cudaError_t e) { return e == cudaSuccess ? LB_OK : LB_ERR_CUDA; }

}  // namespace

// =====================================================================
extern "C" {

int lb_create(const lb_config* cfg, lb_ctx** out_ctx) {
  if (!out_ctx) return LB_ERR_INVALID_ARGUMENT;
  *out_ctx = nullptr;
  if (!cfg) return LB_ERR_INVALID_ARGUMENT;
  if (cfg->struct_size != sizeof(lb_config) || cfg->api_version != LB_API_VERSION) return LB_ERR_VERSION;
  if (!check_cfg(cfg)) return LB_ERR_INVALID_ARGUMENT;
  std::unique_ptr<lb_ctx> x(new lb_ctx());
  Ctx& c = x->c;
  c.cfg = *cfg;
  c.hd = cfg->hidden / cfg->heads;
  c.weight_int8 = cfg->weight_format == LB_WEIGHTS_INT8;
  {
    const char* pdl_env = std::getenv("LB_PDL");
    const int mode = pdl_env ? std::atoi(pdl_env) : 1;
    c.pdl = mode >= 1;
    c.pdl_all = mode >= 2;
    const char* wide_env = std::getenv("LB_WIDE_MIN_TOKENS");
    if (wide_env) c.wide_min_tokens = std::max(0, std::atoi(wide_env));
  }
  c.max_handles = cfg->max_handles;
  if (cudaGetDevice(&c.device) != cudaSuccess) return LB_ERR_CUDA;
  cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, c.device);
  if (gemm_init_attributes() != cudaSuccess || frontend_init_attributes() != cudaSuccess ||
      attention_init_attributes() != cudaSuccess)
    return LB_ERR_CUDA;
  // weights
  c.weight_bytes = layout_weights(x.get(), nullptr, false);
  if (cudaMalloc(&c.weight_arena, c.weight_bytes) != cudaSuccess) return LB_ERR_CAPACITY;
  cudaMemset(c.weight_arena, 0, c.weight_bytes);
  layout_weights(x.get(), static_cast<char*>(c.weight_arena), true);
  // state
  c.state_bytes = layout_state(c, nullptr);
  if (cudaMalloc(&c.state_arena, c.state_bytes) != cudaSuccess) {
    cudaFree(c.weight_arena);
    return LB_ERR_CAPACITY;
  }
  cudaMemset(c.state_arena, 0, c.state_bytes);
  layout_state(c, static_cast<char*>(c.state_arena));
  cudaMemset(c.handle_slot, 0xFF, sizeof(int) * c.max_handles);
  cudaMemset(c.slot_owner, 0xFF, sizeof(int) * cfg->max_sessions);
  cudaMemset(c.handle_key, 0xFF, sizeof(long long) * c.max_handles);
  cudaMemset(c.handle_exp_frame, 0xFF, sizeof(long long) * c.max_handles);
  cudaMemset(c.handle_exp_seq, 0xFF, sizeof(long long) * c.max_handles);
  cudaMemset(c.handle_stamp, 0xFF, sizeof(long long) * c.max_handles);
  // activations
  c.act_bytes = layout_acts(c, nullptr);
  if (cudaMalloc(&c.act_arena, c.act_bytes) != cudaSuccess) {
    cudaFree(c.weight_arena);
    cudaFree(c.state_arena);
    return LB_ERR_CAPACITY;
  }
  cudaMemset(c.act_arena, 0, c.act_bytes);
  layout_acts(c, static_cast<char*>(c.act_arena));
  // DFT twiddles (exact to fp32 rounding of double-precision cos/sin)
  {
    std::vector<float> ct(512), st(512);
    for (int i = 0; i < 512; ++i) {
      const double ang = 2.0 * M_PI * i / 512.0;
      ct[i] = static_cast<float>(std::cos(ang));
      st[i] = static_cast<float>(std::sin(ang));
    }
    cudaMemcpy(c.fe_cos, ct.data(), 512 * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(c.fe_sin, st.data(), 512 * 4, cudaMemcpyHostToDevice);
  }
  // row buckets: powers of two from 16 rows, last = max_rows
  for (int r = 16;; r *= 2) {
    Bucket b;
    b.rows_cap = std::min(r, cfg->max_rows);
    b.tok_cap = 2 * b.rows_cap;
    c.buckets.push_back(b);
    if (b.rows_cap >= cfg->max_rows) break;
  }
  x->plans.resize(c.buckets.size());
  // from here on a failure hands the partly built context to lb_destroy, which
  // frees the arenas and whatever streams, events and staging already exist
  bool ok = cudaStreamCreateWithFlags(&c.capture_stream, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&x->copy_stream, cudaStreamNonBlocking) == cudaSuccess;
  for (cudaEvent_t* ev : {&x->ev_begin, &x->ev_query, &x->ev_tower, &x->ev_copies})
    ok = ok && cudaEventCreateWithFlags(ev, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    lb_destroy(x.release());
    return LB_ERR_CUDA;
  }
  x->pinned_bytes = static_cast<size_t>(cfg->max_rows) *
                    (4 + 8 * 3 + 1 + kPcm * 4 + 2 * (cfg->film_query_dim + cfg->output_dims +
                                                      cfg->text_hidden + cfg->film_query_dim) * 2) +
                    4096;
  if (cudaMallocHost(&x->pinned, x->pinned_bytes) != cudaSuccess) x->pinned = nullptr;
  for (auto& kv : c.tensors) x->names.push_back(kv.first);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    lb_destroy(x.release());
    return LB_ERR_CUDA;
  }
  *out_ctx = x.release();
  return LB_OK;
}

int lb_destroy(lb_ctx* x) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaDeviceSynchronize();
  for (auto& p : x->plans)
    for (auto& gph : p.graph)
      if (gph) cudaGraphExecDestroy(gph);
  if (c.capture_stream) cudaStreamDestroy(c.capture_stream);
  if (x->copy_stream) cudaStreamDestroy(x->copy_stream);
  for (cudaEvent_t ev : {x->ev_begin, x->ev_query, x->ev_tower, x->ev_copies})
    if (ev) cudaEventDestroy(ev);
  if (x->pinned) cudaFreeHost(x->pinned);
  cudaFree(c.weight_arena);
  if (c.wide_arena) cudaFree(c.wide_arena);
  if (c.rel_bf16_arena) cudaFree(c.rel_bf16_arena);
  cudaFree(c.state_arena);
  cudaFree(c.act_arena);
  delete x;
  return LB_OK;
}

int lb_tensor_count(lb_ctx* x) { return x ? static_cast<int>(x->names.size()) : 0; }
const char* lb_tensor_name(lb_ctx* x, int i) {
  if (!x || i < 0 || i >= static_cast<int>(x->names.size())) return nullptr;
  return x->names[i].c_str();
}

int lb_set_tensor(lb_ctx* x, const char* name, const void* host, int dtype, int64_t numel) {
  if (!x || !name || !host) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  auto it = c.tensors.find(name);
  if (it == c.tensors.end()) return LB_ERR_INVALID_ARGUMENT;
  TensorSlot& t = it->second;
  if (t.dtype != dtype || t.numel != numel) return LB_ERR_INVALID_ARGUMENT;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;  // a packed batch is outstanding
  c.weights_final = false;  // derived copies are rebuilt by lb_finalize_weights
  const std::string n(name);
  if (t.clip_dst) {
    float v = *static_cast<const float*>(host);
    if (n == "film.scale_logit") v = c.cfg.film_max_scale / (1.0f + std::exp(-v));
    *t.clip_dst = v;
    t.set = true;
    return LB_OK;
  }
  if (n == "subsample_conv_projection.layer1.conv.weight") {
    const float* w = static_cast<const float*>(host);
    const int C1 = c.cfg.sub_ch1, KP = 9 * 128 + 8;
    std::vector<__nv_bfloat16> out(static_cast<size_t>(C1) * KP, __float2bfloat16(0.f));
    for (int co = 0; co < C1; ++co)
      for (int ci = 0; ci < 128; ++ci)
        for (int i = 0; i < 3; ++i)
          for (int j = 0; j < 3; ++j)
            out[static_cast<size_t>(co) * KP + (i * 3 + j) * 128 + ci] =
                __float2bfloat16(w[((co * 128 + ci) * 3 + i) * 3 + j]);
    if (cudaMemcpy(t.dst, out.data(), out.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
      return LB_ERR_CUDA;
    t.set = true;
    return LB_OK;
  }
  const std::string dw_suffix = ".lconv1d.depthwise_conv1d.weight";
  if (n.size() > dw_suffix.size() && n.compare(n.size() - dw_suffix.size(), dw_suffix.size(), dw_suffix) == 0) {
    // [d][1][5] -> tap-major [5][d] so the conv kernel loads each tap as vectors
    const float* w = static_cast<const float*>(host);
    const int d = c.cfg.hidden;
    std::vector<float> tr(static_cast<size_t>(d) * 5);
    for (int e = 0; e < d; ++e)
      for (int k = 0; k < 5; ++k) tr[static_cast<size_t>(k) * d + e] = w[e * 5 + k];
    if (cudaMemcpy(t.dst, tr.data(), tr.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return LB_ERR_CUDA;
    t.set = true;
    return LB_OK;
  }
  size_t esize = dtype == LB_F32 ? 4 : dtype == LB_I8 ? 1 : 2;
  if (cudaMemcpy(t.dst, host, static_cast<size_t>(numel) * esize, cudaMemcpyHostToDevice) != cudaSuccess)
    return LB_ERR_CUDA;
  if (n == "frontend.mel_filters") {
    const float* f = static_cast<const float*>(host);
    std::vector<int2> rng(128);
    for (int m = 0; m < 128; ++m) {
      int lo = 257, hi = 0;
      for (int k = 0; k < 257; ++k)
        if (f[k * 128 + m] != 0.0f) {
          lo = std::min(lo, k);
          hi = std::max(hi, k + 1);
        }
      if (hi <= lo) lo = hi = 0;
      rng[m] = make_int2(lo, hi);
    }
    cudaMemcpy(c.fe_range, rng.data(), sizeof(int2) * 128, cudaMemcpyHostToDevice);
  }
  t.set = true;
  return LB_OK;
}

int lb_finalize_weights(lb_ctx* x) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  for (auto& kv : c.tensors)
    if (!kv.second.set) {
      fprintf(stderr, "listener_b200: weight %s was not uploaded\n", kv.first.c_str());
      return LB_ERR_STATE;
    }
  // Q/K/V bounds: one fused GEMM serves the three projections; where their
  // bounds differ it clamps per stacked part (outputs) and reads per-part
  // clamped input blocks (inputs)
  for (int i = 0; i < c.cfg.layers; ++i) {
    LayerW& L = c.w.layers[i];
    L.qkv_split_in = L.qkv_split_out = false;
    for (int q = 0; q < 3; ++q)
      for (int k = 0; k < 4; ++k) {
        const float b = x->qkv_bounds[i][q][k];
        L.qkv_clip[q][k] = b;
        if (b != x->qkv_bounds[i][0][k]) (k < 2 ? L.qkv_split_in : L.qkv_split_out) = true;
      }
    for (int k = 0; k < 4; ++k) L.clip[kLinQkv][k] = x->qkv_bounds[i][0][k];
  }
  cudaSetDevice(c.device);
  // plans and graphs bake in clip bounds and weight pointers: rebuild them
  // after every (re)upload
  if (cudaDeviceSynchronize() != cudaSuccess) return LB_ERR_CUDA;
  for (auto& pl : x->plans) {
    for (auto& gph : pl.graph)
      if (gph) {
        cudaGraphExecDestroy(gph);
        gph = nullptr;
      }
    pl.built = false;
    pl.layers.clear();
  }
  if (!c.rel_bf16_arena &&
      cudaMalloc(&c.rel_bf16_arena, static_cast<size_t>(c.cfg.layers) * 13 * c.cfg.hidden * 2) != cudaSuccess) {
    c.rel_bf16_arena = nullptr;
    return LB_ERR_CUDA;
  }
  if (attention_prepare(c, nullptr) != cudaSuccess || cudaStreamSynchronize(nullptr) != cudaSuccess)
    return LB_ERR_CUDA;
  const char* env = std::getenv("LB_INT8_WIDE");
  if (c.weight_int8 && 2 * c.cfg.max_rows >= c.wide_min_tokens && !(env && env[0] == '0')) {
    {
      cudaSetDevice(c.device);
      const size_t n = c.weight_bytes & ~static_cast<size_t>(15);
      cudaError_t e = c.wide_arena ? cudaSuccess : cudaMalloc(&c.wide_arena, 2 * n);
      if (e == cudaSuccess) e = widen_int8_codes(c.weight_arena, c.wide_arena, n, nullptr);
      if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
      if (e != cudaSuccess) {
        if (c.wide_arena) cudaFree(c.wide_arena);
        c.wide_arena = nullptr;
        return LB_ERR_CUDA;
      }
    }
  }
  if (!c.weight_int8) {
    // fp16 copy of the bf16 weights (exact for every weight of magnitude >= 2^-14;
    // the non-GEMM regions of the arena are converted too and never read)
    const size_t n = c.weight_bytes & ~static_cast<size_t>(15);
    cudaError_t e = c.wide_arena ? cudaSuccess : cudaMalloc(&c.wide_arena, n);
    if (e == cudaSuccess) e = widen_bf16_to_f16(c.weight_arena, c.wide_arena, n / 2, nullptr);
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) {
      if (c.wide_arena) cudaFree(c.wide_arena);
      c.wide_arena = nullptr;
      return LB_ERR_CUDA;
    }
  }
  c.weights_final = true;
  return LB_OK;
}

int lb_pack_async(lb_ctx* x, int n, const int32_t* handles, const int64_t* keys, const int64_t* frames,
                  const int64_t* seqs, const uint8_t* masks, void* stream) {
  if (!x || n <= 0 || !handles || !keys || !frames || !seqs) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (!c.weights_final) return LB_ERR_STATE;
  if (n > c.cfg.max_rows) return LB_ERR_CAPACITY;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;  // previous batch not committed / aborted
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  e = cudaMemcpyAsync(c.row_handle, handles, 4ull * n, cudaMemcpyDefault, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c.row_key, keys, 8ull * n, cudaMemcpyDefault, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c.row_frame, frames, 8ull * n, cudaMemcpyDefault, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c.row_seq, seqs, 8ull * n, cudaMemcpyDefault, s);
  if (e == cudaSuccess) {
    if (masks) e = cudaMemcpyAsync(c.row_mask_in, masks, n, cudaMemcpyDefault, s);
    else e = cudaMemsetAsync(c.row_mask_in, 0xFF, n, s);
  }
  if (e != cudaSuccess) return LB_ERR_CUDA;
  c.step_id += 1;
  e = launch_pack(c, n, c.step_id, s);
  if (e != cudaSuccess) return LB_ERR_CUDA;
  c.packed_rows = n;
  c.state = 1;
  x->n_pack += 1;
  return LB_OK;
}

int lb_set_debug_outputs(lb_ctx* x, float* subsampled, float* layers) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  x->c.dbg_sub = subsampled;
  x->c.dbg_layers = layers;
  return LB_OK;
}

namespace {
int step_enqueue(lb_ctx* x, int kind, const void* input, const void* query, void* out_raw, void* out_soft,
                 void* out_film, void* stream, bool overlap);
}

int lb_step_async(lb_ctx* x, int kind, const void* input, const void* query, void* out_raw,
                  void* out_soft, void* out_film, void* stream) {
  return step_enqueue(x, kind, input, query, out_raw, out_soft, out_film, stream, false);
}

namespace {
// overlap: the query H2D and the raw/soft D2H run on the context's copy stream
// under the compute (host buffers); otherwise every copy stays on `stream`.
int step_enqueue(lb_ctx* x, int kind, const void* input, const void* query, void* out_raw, void* out_soft,
                 void* out_film, void* stream, bool overlap) {
  if (!x || !input) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (c.state != 1) return LB_ERR_STATE;
  if (kind != LB_INPUT_PCM && kind != LB_INPUT_MEL) return LB_ERR_INVALID_ARGUMENT;
  const bool film = query != nullptr;
  if (film && !c.cfg.film_enabled) return LB_ERR_INVALID_ARGUMENT;
  if (out_film && !film) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = c.packed_rows;
  const int bi = pick_bucket(c, n);
  if (bi < 0) return LB_ERR_CAPACITY;
  int rc = build_plans(x, bi);
  if (rc) return rc;
  // The query is only read by FiLM after the tower, so its H2D runs on the
  // context's copy stream meanwhile (ordered after everything the caller
  // enqueued before this step, the previous step's FiLM included); the raw and
  // soft tokens are final once the tower ends, so their D2H overlaps FiLM.
  // The copy stream is joined back into `s` at the end of the step.
  cudaStream_t cs = overlap ? x->copy_stream : s;
  cudaError_t e = cudaSuccess;
  if (overlap) {
    e = cudaEventRecord(x->ev_begin, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, x->ev_begin, 0);
  }
  if (e == cudaSuccess && film) {
    e = cudaMemcpyAsync(c.in_query, query, 2ull * n * 2 * c.cfg.film_query_dim, cudaMemcpyDefault, cs);
    if (e == cudaSuccess && overlap) e = cudaEventRecord(x->ev_query, cs);
  }
  if (e == cudaSuccess) {
    if (kind == LB_INPUT_PCM) e = cudaMemcpyAsync(c.in_pcm, input, 4ull * n * kPcm, cudaMemcpyDefault, s);
    else e = cudaMemcpyAsync(c.in_mel, input, 4ull * n * 8 * kMelBins, cudaMemcpyDefault, s);
  }
  if (e != cudaSuccess) return LB_ERR_CUDA;
  const bool eager = c.dbg_sub || c.dbg_layers || c.dbg_stop_layer >= 0;
  lb_ctx::Plans& P = x->plans[bi];
  if (eager) {
    e = run_tower(x, bi, kind, s);
  } else {
    rc = ensure_graph(x, bi, kind);
    if (rc == LB_OK && film) rc = ensure_graph(x, bi, 2);
    if (rc) return rc;
    x->last_graph_kernels = P.graph_kernels[kind] + (film ? P.graph_kernels[2] : 0);
    e = cudaGraphLaunch(P.graph[kind], s);
  }
  if (e != cudaSuccess) return LB_ERR_CUDA;
  const size_t toks = 2ull * n;
  if (overlap) {
    e = cudaEventRecord(x->ev_tower, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, x->ev_tower, 0);
  }
  if (e == cudaSuccess && out_raw)
    e = cudaMemcpyAsync(out_raw, c.out_raw, toks * c.cfg.output_dims * 2, cudaMemcpyDefault, cs);
  if (e == cudaSuccess && out_soft)
    e = cudaMemcpyAsync(out_soft, c.out_soft, toks * c.cfg.text_hidden * 2, cudaMemcpyDefault, cs);
  if (e == cudaSuccess && film) {
    if (overlap) e = cudaStreamWaitEvent(s, x->ev_query, 0);
    if (e == cudaSuccess) e = eager ? run_film(x, bi, s) : cudaGraphLaunch(P.graph[2], s);
    if (e == cudaSuccess && out_film)
      e = cudaMemcpyAsync(out_film, c.out_film, toks * c.cfg.film_query_dim * 2, cudaMemcpyDefault, s);
  }
  if (e == cudaSuccess && overlap) {
    e = cudaEventRecord(x->ev_copies, cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, x->ev_copies, 0);
  }
  if (e != cudaSuccess) return LB_ERR_CUDA;
  c.state = 2;
  x->n_step += 1;
  x->rows_stepped += static_cast<unsigned long long>(n);
  return LB_OK;
}
}  // namespace

int lb_commit_async(lb_ctx* x, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (c.state != 2) return LB_ERR_STATE;
  cudaSetDevice(c.device);
  cudaError_t e = launch_commit(c, static_cast<cudaStream_t>(stream));
  c.state = 3;
  x->n_commit += 1;
  return err_of(e);
}

int lb_abort(lb_ctx* x) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (c.state != 1 && c.state != 2) return LB_ERR_STATE;
  c.state = 0;
  x->n_abort += 1;
  return LB_OK;
}

int lb_rollback_async(lb_ctx* x, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (c.state != 3) return LB_ERR_STATE;
  cudaSetDevice(c.device);
  cudaError_t e = launch_rollback(c, static_cast<cudaStream_t>(stream));
  c.state = 0;
  x->n_rollback += 1;
  return err_of(e);
}

int lb_reset_handle_async(lb_ctx* x, int32_t handle, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (handle < 0 || handle >= c.max_handles) return LB_ERR_INVALID_ARGUMENT;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;
  cudaSetDevice(c.device);
  c.state = 0;
  x->n_reset += 1;
  return err_of(launch_reset(c, handle, -1, static_cast<cudaStream_t>(stream)));
}

int lb_reset_handles_async(lb_ctx* x, int n, const int32_t* handles, void* stream) {
  if (!x || n < 0 || (n > 0 && !handles)) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (n > c.max_handles) return LB_ERR_INVALID_ARGUMENT;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;
  cudaSetDevice(c.device);
  c.state = 0;
  x->n_reset += static_cast<unsigned long long>(n);
  return err_of(launch_reset_many(c, handles, n, static_cast<cudaStream_t>(stream)));
}

int lb_reset_slot_async(lb_ctx* x, int32_t slot, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (slot < 0 || slot >= c.cfg.max_sessions) return LB_ERR_INVALID_ARGUMENT;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;
  cudaSetDevice(c.device);
  c.state = 0;
  x->n_reset += 1;
  return err_of(launch_reset(c, -1, slot, static_cast<cudaStream_t>(stream)));
}

int lb_get_status(lb_ctx* x, int32_t* out, void* stream) {
  if (!x || !out) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, c.status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return err_of(e);
}

int lb_clear_status(lb_ctx* x, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(x->c.device);
  return err_of(launch_clear_status(x->c, static_cast<cudaStream_t>(stream)));
}

int lb_mel_async(lb_ctx* x, int n, const float* pcm, const float* tail_in, float* tail_out, float* mel_out,
                 void* stream) {
  if (!x || n < 0 || (n > 0 && (!pcm || !tail_out || !mel_out))) return LB_ERR_INVALID_ARGUMENT;
  if (tail_in && tail_in == tail_out) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (!c.weights_final) return LB_ERR_STATE;  // the window and filterbank are weights
  if (n == 0) return LB_OK;
  cudaSetDevice(c.device);
  return err_of(launch_mel_standalone(c, n, pcm, tail_in, tail_out, mel_out, static_cast<cudaStream_t>(stream)));
}

int lb_film_talker_async(lb_ctx* x, int n, const void* response_hidden, int max_states, const int32_t* n_states,
                         const int32_t* steps, const void* query, void* out, void* stream) {
  if (!x || n < 0 || max_states < 1) return LB_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!response_hidden || !n_states || !steps || !query || !out)) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (!c.cfg.film_enabled) return LB_ERR_INVALID_ARGUMENT;
  if (!c.weights_final) return LB_ERR_STATE;
  if (c.state == 1 || c.state == 2) return LB_ERR_STATE;  // the FiLM buffers belong to a packed step
  if (n == 0) return LB_OK;
  // FiLM runs over "tokens": one per talker row; the bucket holding n tokens
  int bi = -1;
  for (size_t i = 0; i < c.buckets.size(); ++i)
    if (c.buckets[i].tok_cap >= n) {
      bi = static_cast<int>(i);
      break;
    }
  if (bi < 0) return LB_ERR_CAPACITY;
  cudaSetDevice(c.device);
  int rc = build_plans(x, bi);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* hid = static_cast<const __nv_bfloat16*>(response_hidden);
  const auto* q = static_cast<const __nv_bfloat16*>(query);
  cudaError_t e = launch_film_talker(c, n, hid, max_states, n_states, steps, q, nullptr, 0, s);
  if (e == cudaSuccess) {
    const bool eager = c.dbg_sub || c.dbg_layers || c.dbg_stop_layer >= 0;
    if (eager) {
      e = run_film(x, bi, s);
    } else {
      rc = ensure_graph(x, bi, 2);
      if (rc) return rc;
      e = cudaGraphLaunch(x->plans[bi].graph[2], s);
    }
  }
  if (e == cudaSuccess) e = launch_film_talker(c, n, hid, max_states, n_states, steps, q,
                                               static_cast<__nv_bfloat16*>(out), 1, s);
  return err_of(e);
}

int lb_get_counters(lb_ctx* x, lb_counters* out, void* stream) {
  if (!x || !out) return LB_ERR_INVALID_ARGUMENT;
  if (out->struct_size != sizeof(lb_counters) || out->api_version != LB_API_VERSION) return LB_ERR_VERSION;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned long long dev[8] = {};
  int32_t st[2] = {0, 0};
  cudaError_t e = cudaMemcpyAsync(dev, c.dev_ctr, sizeof(dev), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(st, c.status, sizeof(st), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return LB_ERR_CUDA;
  out->packs = x->n_pack;
  out->steps = x->n_step;
  out->commits = x->n_commit;
  out->aborts = x->n_abort;
  out->rollbacks = x->n_rollback;
  out->resets = x->n_reset;
  out->rows_stepped = x->rows_stepped;
  out->rows_continue = dev[0];
  out->rows_reset = dev[1];
  out->rows_gap_or_cursor_mismatch = dev[2];
  out->rows_identity_reset = dev[3];
  out->rows_committed = dev[4];
  out->stale_commits = dev[5];
  out->status = st[0];
  out->status_history = st[0] | st[1];
  int graphs = 0;
  for (auto& p : x->plans)
    for (auto g : p.graph) graphs += g != nullptr;
  out->graphs_captured = graphs;
  return LB_OK;
}

int lb_read_rows(lb_ctx* x, int32_t* slots, int32_t* reasons, int n, void* stream) {
  if (!x || n < 0 || n > x->c.cfg.max_rows) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (slots) e = cudaMemcpyAsync(slots, c.row_slot, 4ull * n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && reasons) e = cudaMemcpyAsync(reasons, c.row_reason, 4ull * n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return err_of(e);
}

int lb_read_handles(lb_ctx* x, int32_t* slot, int64_t* key, int64_t* ef, int64_t* es, void* stream) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t H = c.max_handles;
  cudaError_t e = cudaSuccess;
  if (slot) e = cudaMemcpyAsync(slot, c.handle_slot, 4 * H, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && key) e = cudaMemcpyAsync(key, c.handle_key, 8 * H, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && ef) e = cudaMemcpyAsync(ef, c.handle_exp_frame, 8 * H, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && es) e = cudaMemcpyAsync(es, c.handle_exp_seq, 8 * H, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return err_of(e);
}

int lb_debug_set_expected(lb_ctx* x, int32_t handle, int64_t frame, int64_t seq, void* stream) {
  if (!x || handle < 0 || handle >= x->c.max_handles) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  long long f = frame, q = seq;
  cudaError_t e = cudaMemcpyAsync(c.handle_exp_frame + handle, &f, 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(c.handle_exp_seq + handle, &q, 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return err_of(e);
}

int lb_step_kernel_count(lb_ctx* x) { return x ? x->last_graph_kernels : 0; }

int lb_debug_set_stop(lb_ctx* x, int layer, int stage) {
  if (!x) return LB_ERR_INVALID_ARGUMENT;
  x->c.dbg_stop_layer = layer;
  x->c.dbg_stop_stage = stage;
  return LB_OK;
}

int lb_debug_read_buffer(lb_ctx* x, const char* name, void* dst, size_t bytes, void* stream) {
  if (!x || !name || !dst) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  const std::string n(name);
  const void* src = n == "h" ? static_cast<const void*>(c.h) : n == "y" ? static_cast<const void*>(c.y)
                  : n == "xa" ? static_cast<const void*>(c.xa) : n == "xf" ? static_cast<const void*>(c.xf)
                  : n == "qkv" ? static_cast<const void*>(c.qkv) : n == "att" ? static_cast<const void*>(c.att)
                  : n == "gl" ? static_cast<const void*>(c.gl) : n == "mel" ? static_cast<const void*>(c.in_mel)
                  : n == "sub_in" ? static_cast<const void*>(c.sub_in) : nullptr;
  if (!src) return LB_ERR_INVALID_ARGUMENT;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return err_of(e);
}

int lb_step_host(lb_ctx* x, int n, const int32_t* handles, const int64_t* keys, const int64_t* frames,
                 const int64_t* seqs, const uint8_t* masks, int kind, const void* input, const void* query,
                 void* out_raw, void* out_soft, void* out_film, int commit, void* stream) {
  if (!x || !x->pinned || n <= 0 || !input) return LB_ERR_INVALID_ARGUMENT;
  Ctx& c = x->c;
  if (n > c.cfg.max_rows) return LB_ERR_CAPACITY;
  cudaSetDevice(c.device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* p = static_cast<char*>(x->pinned);
  // page-locked caller buffers are copied by DMA directly; pageable ones go
  // through the context's pinned staging area
  auto pinned = [](const void* ptr) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return at.type == cudaMemoryTypeHost;
  };
  auto stage = [&](const void* src, size_t bytes) -> void* {
    if (!src) return nullptr;
    if (pinned(src)) return const_cast<void*>(src);
    char* dst = p;
    std::memcpy(dst, src, bytes);
    p += align_up(bytes, 256);
    return dst;
  };
  const size_t in_bytes = kind == LB_INPUT_PCM ? 4ull * n * kPcm : 4ull * n * 8 * kMelBins;
  if (in_bytes > 4ull * c.cfg.max_rows * kPcm) return LB_ERR_CAPACITY;
  void* ph = stage(handles, 4ull * n);
  void* pk = stage(keys, 8ull * n);
  void* pf = stage(frames, 8ull * n);
  void* pq = stage(seqs, 8ull * n);
  void* pm = stage(masks, n);
  void* pin = stage(input, in_bytes);
  void* pqry = stage(query, 2ull * n * 2 * c.cfg.film_query_dim);
  char* outs = p;
  const size_t raw_b = 4ull * n * c.cfg.output_dims, soft_b = 4ull * n * c.cfg.text_hidden;
  const size_t film_b = 4ull * n * c.cfg.film_query_dim;
  char* o_raw = outs;
  char* o_soft = o_raw + align_up(raw_b, 256);
  char* o_film = o_soft + align_up(soft_b, 256);
  if (static_cast<size_t>(o_film + film_b - static_cast<char*>(x->pinned)) > x->pinned_bytes)
    return LB_ERR_CAPACITY;
  const bool raw_direct = out_raw && pinned(out_raw);
  const bool soft_direct = out_soft && pinned(out_soft);
  const bool film_direct = out_film && pinned(out_film);
  if (raw_direct) o_raw = static_cast<char*>(out_raw);
  if (soft_direct) o_soft = static_cast<char*>(out_soft);
  if (film_direct) o_film = static_cast<char*>(out_film);
  int rc = lb_pack_async(x, n, static_cast<int32_t*>(ph), static_cast<int64_t*>(pk),
                         static_cast<int64_t*>(pf), static_cast<int64_t*>(pq),
                         static_cast<uint8_t*>(pm), stream);
  if (rc) return rc;
  rc = step_enqueue(x, kind, pin, pqry, out_raw ? o_raw : nullptr, out_soft ? o_soft : nullptr,
                    out_film ? o_film : nullptr, stream, true);
  if (rc) return rc;
  if (commit) {
    rc = lb_commit_async(x, stream);
    if (rc) return rc;
  }
  if (cudaStreamSynchronize(s) != cudaSuccess) return LB_ERR_CUDA;
  if (out_raw && !raw_direct) std::memcpy(out_raw, o_raw, raw_b);
  if (out_soft && !soft_direct) std::memcpy(out_soft, o_soft, soft_b);
  if (out_film && !film_direct) std::memcpy(out_film, o_film, film_b);
  return LB_OK;
}

}  // extern "C"
