"""Host-side weight preparation for the listener context.

Converts a transformers-style state dict (``Gemma4AudioModel`` names, the
embedder under ``embed.``, the FiLM adapter under ``film.``) into the tensors
the C ABI uploads, and returns the *effective* fp32 weights -- exactly the
values the GPU computes with -- so a checker can run the same model.

- bf16 format: every parameter is rounded to bf16 (as in the reference's bf16
  tower); GEMM weights upload as bf16.
- int8 format: GEMM weights are quantised per output channel
  (scale = fp16(max|w| / 127), q = clip(rint(w / scale), -127, 127)); the
  effective weight is q * scale.  Non-GEMM parameters stay bf16-rounded.
- precomputed: relative keys per layer, relative_k_proj(sinusoid positions
  12..0) in fp32 (streaming_conformer.py:260-279, modeling_gemma4.py:178-206),
  and the query scale (hd^-0.5 / ln 2) * softplus(per_dim_scale)
  (modeling_gemma4.py:220, 287).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from .config import ListenerConfig
from .frontend_tables import hann_window, mel_filterbank


def is_gemm_weight(name: str) -> bool:
    if name.startswith("film."):
        return name.endswith(".weight") and any(
            k in name for k in ("query_down", "response_down", "film.film", "film.output"))
    return name.endswith("linear.weight") or name in (
        "subsample_conv_projection.input_proj_linear.weight", "output_proj.weight",
        "embed.embedding_projection.weight")


def bf16_round(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def bf16_bits(a: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def quantize_int8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-channel symmetric int8: returns (q int8 [O,K], scale fp16 [O])."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    scale = (amax / np.float32(127.0)).astype(np.float16)
    scale[scale == 0] = np.float16(1.0)
    s = scale.astype(np.float32)[:, None]
    q = np.clip(np.rint(w / s), -127, 127).astype(np.int8)
    return q, scale


def dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    return q.astype(np.float32) * scale.astype(np.float32)[:, None]


def relative_keys(rel_w: np.ndarray, hidden: int) -> np.ndarray:
    """[13, hidden] fp32 relative keys for positions 12..0."""
    nts = hidden // 2
    inc = math.log(10000.0) / max(nts - 1, 1)
    inv = np.exp(np.arange(nts, dtype=np.float32) * np.float32(-inc)).astype(np.float32)
    pos = np.arange(12, -1, -1, dtype=np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([np.sin(pos), np.cos(pos)], axis=-1).astype(np.float32)
    return (torch.from_numpy(emb) @ torch.from_numpy(np.ascontiguousarray(rel_w, np.float32)).t()).numpy()


def query_scale(per_dim_scale: np.ndarray, head_dim: int) -> np.ndarray:
    q = (head_dim ** -0.5) / math.log(2)
    return (np.float32(q) * torch.nn.functional.softplus(
        torch.from_numpy(np.asarray(per_dim_scale, np.float32))).numpy()).astype(np.float32)


def prepare(cfg: ListenerConfig, tower: dict[str, np.ndarray], film: dict[str, np.ndarray] | None,
            weight_format: int) -> tuple[list[tuple[str, np.ndarray, int]], dict[str, np.ndarray]]:
    """Returns (uploads [(name, array, lb dtype)], effective fp32 weights by name)."""
    uploads: list[tuple[str, np.ndarray, int]] = []
    eff: dict[str, np.ndarray] = {}
    items = list(tower.items())
    if film is not None:
        items += [(f"film.{k}", v) for k, v in film.items()]
    for name, w in items:
        w = np.asarray(w, dtype=np.float32)
        if is_gemm_weight(name):
            if weight_format == 1:
                q, s = quantize_int8(w)
                uploads.append((name, q, _lib.LB_I8))
                uploads.append((name + ":scale", s, _lib.LB_F16))
                eff[name] = dequantize(q, s)
            else:
                uploads.append((name, bf16_bits(w), _lib.LB_BF16))
                eff[name] = bf16_round(w)
            continue
        e = bf16_round(w)
        eff[name] = e
        if name.endswith("relative_k_proj.weight"):
            layer = name.split(".")[1]
            uploads.append((f"layers.{layer}.self_attn.relative_keys",
                            relative_keys(e, cfg.hidden).reshape(-1), _lib.LB_F32))
            continue
        if name.endswith("per_dim_scale"):
            layer = name.split(".")[1]
            uploads.append((f"layers.{layer}.self_attn.query_scale",
                            query_scale(e, cfg.head_dim), _lib.LB_F32))
            continue
        if name.endswith(("input_min", "input_max", "output_min", "output_max")):
            # the bf16-rounded bound, like every non-GEMM parameter (a bf16 tower's
            # clip buffers are bf16); +/-inf stays infinite
            uploads.append((name, np.asarray(e, np.float32).reshape(1), _lib.LB_F32))
            continue
        uploads.append((name, np.ascontiguousarray(e.reshape(-1)), _lib.LB_F32))
    uploads.append(("frontend.window", hann_window(), _lib.LB_F32))
    uploads.append(("frontend.mel_filters", mel_filterbank().astype(np.float32).reshape(-1), _lib.LB_F32))
    return uploads, eff
