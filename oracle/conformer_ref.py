"""fp32 CPU restatement of the exact streaming Q2 Conformer step (test oracle).

Follows ``StreamingConformerAudioTower._compute_step``
(duplex_kernel/streaming_conformer.py:700-888) and the transformers 5.5.0
Gemma 4 audio modules it calls (TF = transformers/models/gemma4/):

- subsampler: streaming_conformer.py:741-761, _stream_subsample_layer :1055-1068,
  TF modeling_gemma4.py:317-372
- feed-forward: TF modeling_gemma4.py:375-408
- attention: streaming_conformer.py:778-829, TF modeling_gemma4.py:209-314,
  relative positions TF :178-206, precompute streaming_conformer.py:260-279
- light conv: streaming_conformer.py:830-852, TF modeling_gemma4.py:444-482
- layer output: streaming_conformer.py:853-860
- output projection and embedder: streaming_conformer.py:865-872,
  TF modeling_gemma4.py:1928-1953
- state shift: streaming_conformer.py:815-822, 834-836, 865-887

State is explicit per session (no slot banks); ``reset`` zeroes a session's
state exactly like the ``torch.where(reset_rows, 0, ...)`` block at
streaming_conformer.py:721-740.  TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

MEL_TICK_ROWS = 8
MEL_BINS = 128
Q2 = 2
MAX_PAST = 12
CACHED = 13


@dataclass(frozen=True)
class OracleConfig:
    hidden: int
    layers: int
    heads: int
    ffn: int
    sub_ch0: int = 128
    sub_ch1: int = 32
    output_dims: int = 1536
    text_hidden: int = 1536
    conv_kernel: int = 5
    rms_eps: float = 1e-6
    softcap: float = 50.0
    invalid_logit: float = -1.0e9
    gradient_clipping: float = 1e10
    residual_weight: float = 0.5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def _rms(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    # TF modeling_gemma4.py:157-175 (fp32: x * pow(mean(x^2) + eps, -0.5) * w)
    y = x * torch.pow(x.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    return y * w if w is not None else y


def _clip_linear(x, W, bounds):
    # TF modeling_gemma4.py:145-154: clamp(in) -> x W^T -> clamp(out)
    in_lo, in_hi, out_lo, out_hi = bounds
    y = torch.clamp(x, in_lo, in_hi) @ W.t()
    return torch.clamp(y, out_lo, out_hi)


def relative_position_keys(weights: dict, cfg: OracleConfig) -> list[torch.Tensor]:
    """Per-layer relative keys [13, H, hd] (streaming_conformer.py:260-279)."""
    d = cfg.hidden
    nts = d // 2
    inc = math.log(10000.0) / max(nts - 1, 1)
    inv = torch.exp(torch.arange(nts, dtype=torch.float32) * -inc)
    pos = torch.arange(12, -1, -1, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat([torch.sin(pos), torch.cos(pos)], dim=-1)  # TF :200-206
    out = []
    for i in range(cfg.layers):
        W = weights[f"layers.{i}.self_attn.relative_k_proj.weight"]
        out.append((emb @ W.t()).view(-1, cfg.heads, cfg.head_dim))
    return out


def _bounds(weights: dict, prefix: str):
    get = lambda n, default: float(weights.get(f"{prefix}.{n}", torch.tensor(default)))
    return (get("input_min", -math.inf), get("input_max", math.inf),
            get("output_min", -math.inf), get("output_max", math.inf))


def zero_state(cfg: OracleConfig, n: int) -> dict[str, torch.Tensor]:
    d, L, H, hd = cfg.hidden, cfg.layers, cfg.heads, cfg.head_dim
    f0 = (MEL_BINS + 1) // 2
    return {
        "mel": torch.zeros(n, 1, 1, MEL_BINS),
        "mel_mask": torch.zeros(n, 1, dtype=torch.bool),
        "sub": torch.zeros(n, cfg.sub_ch0, 1, f0),
        "sub_mask": torch.zeros(n, 1, dtype=torch.bool),
        "keys": torch.zeros(n, L, CACHED, H, hd),
        "values": torch.zeros(n, L, CACHED, H, hd),
        "conv": torch.zeros(n, L, cfg.conv_kernel - 1, d),
        "valid": torch.zeros(n, CACHED, dtype=torch.bool),
    }


class OracleConformer:
    """Batched fp32 streaming step over explicit per-session state."""

    def __init__(self, weights: dict[str, torch.Tensor], cfg: OracleConfig):
        self.w = {k: v.float() for k, v in weights.items()}
        self.cfg = cfg
        self.rel_keys = relative_position_keys(self.w, cfg)
        q = torch.arange(Q2)[:, None]
        k = torch.arange(CACHED + Q2)[None, :]
        cached = CACHED - k[:, :CACHED] + q
        current = q - (k[:, CACHED:] - CACHED)
        dist = torch.cat((cached, current), dim=1)
        self.window = (dist >= 0) & (dist < MAX_PAST)
        self.rel_index = MAX_PAST - dist.clamp(0, MAX_PAST)

    def _sub_layer(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        # streaming_conformer.py:1055-1068: conv (pad (0,1)) -> LN(channels) -> ReLU
        h = F.conv2d(x, self.w[f"{prefix}.conv.weight"], None, stride=2, padding=(0, 1))
        h = F.layer_norm(h.permute(0, 2, 3, 1), (h.shape[1],), self.w[f"{prefix}.norm.weight"],
                         None, self.cfg.rms_eps)
        return torch.relu(h).permute(0, 3, 1, 2).contiguous()

    def _ffn(self, p: str, x: torch.Tensor) -> torch.Tensor:
        # TF modeling_gemma4.py:390-408
        c = min(self.cfg.gradient_clipping, torch.finfo(torch.float32).max)
        h = _rms(torch.clamp(x, -c, c), self.w[f"{p}.pre_layer_norm.weight"], self.cfg.rms_eps)
        h = _clip_linear(h, self.w[f"{p}.ffw_layer_1.linear.weight"], _bounds(self.w, f"{p}.ffw_layer_1"))
        h = F.silu(h)
        h = _clip_linear(h, self.w[f"{p}.ffw_layer_2.linear.weight"], _bounds(self.w, f"{p}.ffw_layer_2"))
        h = _rms(torch.clamp(h, -c, c), self.w[f"{p}.post_layer_norm.weight"], self.cfg.rms_eps)
        return h * self.cfg.residual_weight + x

    @torch.no_grad()
    def step(self, mel: torch.Tensor, mask: torch.Tensor, state: dict, reset: torch.Tensor):
        """One Q2 tick.  Returns (raw, soft, subsampled, layer_rows, next_state)."""
        cfg, w = self.cfg, self.w
        n = mel.shape[0]
        d, H, hd = cfg.hidden, cfg.heads, cfg.head_dim
        r = reset.bool()
        st = {k: torch.where(r.view(-1, *([1] * (v.ndim - 1))), torch.zeros_like(v), v)
              for k, v in state.items()}
        mel = mel.float()
        mask = mask.bool()
        # ---- subsampler (streaming_conformer.py:741-761)
        prev = st["mel"] * st["mel_mask"][:, None, :, None].float()
        cur = mel.unsqueeze(1) * mask[:, None, :, None].float()
        hidden0 = self._sub_layer("subsample_conv_projection.layer0", torch.cat((prev, cur), dim=2))
        mask0 = mask[:, ::2]
        h1_in = torch.cat((st["sub"] * st["sub_mask"][:, None, :, None].float(),
                           hidden0 * mask0[:, None, :, None].float()), dim=2)
        hidden1 = self._sub_layer("subsample_conv_projection.layer1", h1_in)
        mask1 = mask0[:, ::2]
        b, ch, t, fr = hidden1.shape
        sub = hidden1.permute(0, 2, 3, 1).reshape(b, t, ch * fr) @ \
            w["subsample_conv_projection.input_proj_linear.weight"].t()

        h = sub
        valid_now = mask1
        layers_out, next_k, next_v, next_c = [], [], [], []
        c = min(cfg.gradient_clipping, torch.finfo(torch.float32).max)
        q_scale = (hd ** -0.5) / math.log(2)
        k_scale = math.log(1 + math.e) / math.log(2)
        for li in range(cfg.layers):
            p = f"layers.{li}"
            h = self._ffn(f"{p}.feed_forward1", h)
            residual = h
            x = _rms(torch.clamp(h, -c, c), w[f"{p}.norm_pre_attn.weight"], cfg.rms_eps)
            shape = (n, Q2, H, hd)
            q = _clip_linear(x, w[f"{p}.self_attn.q_proj.linear.weight"], _bounds(w, f"{p}.self_attn.q_proj")).view(shape)
            k = _clip_linear(x, w[f"{p}.self_attn.k_proj.linear.weight"], _bounds(w, f"{p}.self_attn.k_proj")).view(shape)
            v = _clip_linear(x, w[f"{p}.self_attn.v_proj.linear.weight"], _bounds(w, f"{p}.self_attn.v_proj")).view(shape)
            q = q * q_scale * F.softplus(w[f"{p}.self_attn.per_dim_scale"])
            k = k * k_scale
            all_k = torch.cat((st["keys"][:, li], k), dim=1)
            all_v = torch.cat((st["values"][:, li], v), dim=1)
            qh = q.permute(0, 2, 1, 3)
            ac = qh @ all_k.permute(0, 2, 3, 1)
            pk = self.rel_keys[li][self.rel_index].permute(2, 0, 3, 1).unsqueeze(0)
            bd = (qh.unsqueeze(-2) @ pk).squeeze(-2)
            logits = torch.tanh((ac + bd) / cfg.softcap) * cfg.softcap
            key_valid = torch.cat((st["valid"], valid_now), dim=1)
            ok = self.window[None] & key_valid[:, None, :]
            logits = logits.masked_fill(~ok[:, None], cfg.invalid_logit)
            att = F.softmax(logits, dim=-1) @ all_v.permute(0, 2, 1, 3)
            att = att.permute(0, 2, 1, 3).reshape(n, Q2, d)
            att = _clip_linear(att, w[f"{p}.self_attn.post.linear.weight"], _bounds(w, f"{p}.self_attn.post"))
            next_k.append(torch.cat((st["keys"][:, li, Q2:], k), dim=1)[:, -CACHED:])
            next_v.append(torch.cat((st["values"][:, li, Q2:], v), dim=1)[:, -CACHED:])
            h = _rms(torch.clamp(att, -c, c), w[f"{p}.norm_post_attn.weight"], cfg.rms_eps) + residual
            # light conv
            lp = f"{p}.lconv1d"
            residual = h
            x = _rms(h, w[f"{lp}.pre_layer_norm.weight"], cfg.rms_eps)
            g = _clip_linear(x, w[f"{lp}.linear_start.linear.weight"], _bounds(w, f"{lp}.linear_start"))
            g = F.glu(g, dim=-1)
            window = torch.cat((st["conv"][:, li], g), dim=1)
            next_c.append(window[:, -(cfg.conv_kernel - 1):])
            conv = F.conv1d(window.transpose(1, 2), w[f"{lp}.depthwise_conv1d.weight"], None,
                            groups=d).transpose(1, 2)
            conv = _rms(torch.clamp(conv, -c, c), w[f"{lp}.conv_norm.weight"], cfg.rms_eps)
            h = _clip_linear(F.silu(conv), w[f"{lp}.linear_end.linear.weight"], _bounds(w, f"{lp}.linear_end")) + residual
            h = self._ffn(f"{p}.feed_forward2", h)
            h = _rms(torch.clamp(h, -c, c), w[f"{p}.norm_out.weight"], cfg.rms_eps)
            layers_out.append(h)

        raw = h @ w["output_proj.weight"].t() + w["output_proj.bias"]
        soft = _rms(raw, None, cfg.rms_eps) @ w["embed.embedding_projection.weight"].t()
        nxt = {
            "mel": mel[:, -1:, :].unsqueeze(1),
            "mel_mask": mask[:, -1:].clone(),
            "sub": hidden0[:, :, -1:, :].clone(),
            "sub_mask": mask0[:, -1:].clone(),
            "keys": torch.stack(next_k, dim=1),
            "values": torch.stack(next_v, dim=1),
            "conv": torch.stack(next_c, dim=1),
            "valid": torch.cat((st["valid"][:, Q2:], valid_now), dim=1)[:, -CACHED:],
        }
        return raw, soft, sub, layers_out, nxt


def gather_state(states: list[dict], rows: list[int]) -> dict:
    return {k: torch.stack([states[i][k] for i in rows]) for k in states[rows[0]]}


class OracleSessions:
    """Per-session state store driven by (session, reset) rows -- a test helper."""

    def __init__(self, model: OracleConformer):
        self.model = model
        self.state: dict = {}

    def step(self, sessions, mel, mask, resets):
        n = len(sessions)
        zero = zero_state(self.model.cfg, 1)
        st = {k: torch.cat([self.state.get(s, {kk: vv[0] for kk, vv in zero.items()})[k][None]
                            for s in sessions]) for k in zero}
        out = self.model.step(mel, mask, st, torch.as_tensor(resets, dtype=torch.bool))
        nxt = out[4]
        for i, s in enumerate(sessions):
            self.state[s] = {k: v[i] for k, v in nxt.items()}
        return out
