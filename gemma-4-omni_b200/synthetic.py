"""Seeded synthetic weights, audio and session arrival processes.

There are no checkpoints, WAVs or recorded sessions for this path in the
reference (its benchmark WAV and the Gemma 4 checkpoint are not shipped), so
every benchmark and parity case runs on seeded stand-ins with the shapes and
distributions of the reference workload:

- weights: every Linear / Conv weight ~ N(0, 0.02) (transformers
  ``_init_weights`` with initializer_range 0.02), norm weights 1,
  ``per_dim_scale`` 0, clip bounds +/-inf, ``output_proj`` bias 0.  The FiLM
  adapter uses the same init, its ``output`` layer randomised N(0, 1e-3) (as
  tests/kernel/test_frame_residual_query_film_v2.py:32-35 does, otherwise it is
  an exact identity) and ``scale_logit`` such that 0.25*sigmoid = 0.0513.
- audio: 16 kHz, 0.05 * N(0,1) white noise plus a 0.1-amplitude sawtooth whose
  pitch glides linearly between two U[150, 300] Hz endpoints over the session.
- arrivals: start offsets U{0..400} steps, lengths Geometric(1/300) (mean 300).

``nontrivial=True`` (parity runs) perturbs every parameter that the default
init leaves at an identity value, as a real checkpoint would: norm and
LayerNorm weights ~ N(1, 0.1), ``per_dim_scale`` ~ N(0, 0.5), the
``output_proj`` bias and the FiLM LayerNorm biases ~ N(0, 0.05), and finite
clip bounds on every ``Gemma4ClippableLinear`` (transformers
models/gemma4/modeling_gemma4.py:128-154): input and output bounds, each
side drawn separately, so that they bind on a small fraction of the
elements.  The default-init draws come first and are unchanged, and every
value of a nontrivial set is then rounded to bf16, as in a bf16 checkpoint
(the format Gemma 4 weights ship in), so the reference run on them in fp32 is
the exact target of a bf16-weight step and no weight rounding separates the two.
"""
from __future__ import annotations

import numpy as np

from .config import FILM_SCALE_LOGIT, MEL_BINS, PCM_SAMPLES_PER_FRAME, SAMPLE_RATE_HZ, ListenerConfig


def tower_weight_shapes(cfg: ListenerConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) for every audio-tower + embedder parameter, in a fixed order.

    Names are the transformers Gemma4AudioModel state_dict names; the embedder
    (Gemma4MultimodalEmbedder) is prefixed ``embed.``.
    init: 'normal' N(0,0.02), 'ones', 'zeros'.
    """
    d, F, hd = cfg.hidden, cfg.ffn, cfg.head_dim
    s = "subsample_conv_projection"
    out = [
        (f"{s}.layer0.conv.weight", (cfg.sub_ch0, 1, 3, 3), "normal"),
        (f"{s}.layer0.norm.weight", (cfg.sub_ch0,), "ones"),
        (f"{s}.layer1.conv.weight", (cfg.sub_ch1, cfg.sub_ch0, 3, 3), "normal"),
        (f"{s}.layer1.norm.weight", (cfg.sub_ch1,), "ones"),
        (f"{s}.input_proj_linear.weight", (d, cfg.sub_proj_in), "normal"),
    ]
    for i in range(cfg.layers):
        p = f"layers.{i}"
        for ff in ("feed_forward1", "feed_forward2"):
            out += [
                (f"{p}.{ff}.ffw_layer_1.linear.weight", (F, d), "normal"),
                (f"{p}.{ff}.ffw_layer_2.linear.weight", (d, F), "normal"),
                (f"{p}.{ff}.pre_layer_norm.weight", (d,), "ones"),
                (f"{p}.{ff}.post_layer_norm.weight", (d,), "ones"),
            ]
        for proj in ("q_proj", "k_proj", "v_proj", "post"):
            out.append((f"{p}.self_attn.{proj}.linear.weight", (d, d), "normal"))
        out += [
            (f"{p}.self_attn.relative_k_proj.weight", (d, d), "normal"),
            (f"{p}.self_attn.per_dim_scale", (hd,), "zeros"),
            (f"{p}.lconv1d.linear_start.linear.weight", (2 * d, d), "normal"),
            (f"{p}.lconv1d.linear_end.linear.weight", (d, d), "normal"),
            (f"{p}.lconv1d.depthwise_conv1d.weight", (d, 1, cfg.conv_kernel), "normal"),
            (f"{p}.lconv1d.pre_layer_norm.weight", (d,), "ones"),
            (f"{p}.lconv1d.conv_norm.weight", (d,), "ones"),
            (f"{p}.norm_pre_attn.weight", (d,), "ones"),
            (f"{p}.norm_post_attn.weight", (d,), "ones"),
            (f"{p}.norm_out.weight", (d,), "ones"),
        ]
    out += [
        ("output_proj.weight", (cfg.output_dims, d), "normal"),
        ("output_proj.bias", (cfg.output_dims,), "zeros"),
        ("embed.embedding_projection.weight", (cfg.text_hidden, cfg.output_dims), "normal"),
    ]
    return out


def film_weight_shapes(cfg: ListenerConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """FrameResidualQueryFiLMAdapter state_dict (frame_residual_adapter.py:185-197)."""
    q, h, b = cfg.film_query_dim, cfg.text_hidden, cfg.film_bottleneck
    return [
        ("query_norm.weight", (q,), "ones"),
        ("query_norm.bias", (q,), "zeros"),
        ("query_down.weight", (b, q), "normal"),
        ("query_down.bias", (b,), "normal"),
        ("response_norm.weight", (h,), "ones"),
        ("response_norm.bias", (h,), "zeros"),
        ("response_down.weight", (b, h), "normal"),
        ("response_down.bias", (b,), "normal"),
        ("film.weight", (2 * b, b), "normal"),
        ("film.bias", (2 * b,), "normal"),
        ("output.weight", (q, b), "output"),
        ("output.bias", (q,), "output"),
        ("scale_logit", (), "scale_logit"),
    ]


def _draw(rng: np.random.Generator, shape, init: str) -> np.ndarray:
    if init == "normal":
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if init == "output":
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(1e-3)).astype(np.float32)
    if init == "ones":
        return np.ones(shape, dtype=np.float32)
    if init == "zeros":
        return np.zeros(shape, dtype=np.float32)
    if init == "scale_logit":
        return np.asarray(FILM_SCALE_LOGIT, dtype=np.float32)
    raise ValueError(init)


def _bf16_representable(x: float) -> np.ndarray:
    """0-d float32 array rounded toward zero to 8 significant bits, so the bound
    is the same in bf16 and fp32 (clip bounds are 0-d buffers in the module)."""
    v = np.asarray([x], np.float32).view(np.uint32) & np.uint32(0xFFFF0000)
    return np.asarray(v.view(np.float32)[0], dtype=np.float32)


def clippable_linears(cfg: ListenerConfig) -> list[tuple[str, float]]:
    """(prefix, typical |input| scale) of every Gemma4ClippableLinear of the tower.

    The scale is the standard deviation the default init gives the linear's
    input: RMS-normalised rows have unit scale, the FFN's second linear reads
    SiLU of the first one's output (std 0.02*sqrt(d)), the attention ``post``
    reads an average of values and ``linear_end`` SiLU of a normalised row.
    """
    d = cfg.hidden
    first = 0.02 * np.sqrt(d)
    out = []
    for i in range(cfg.layers):
        p = f"layers.{i}"
        for ff in ("feed_forward1", "feed_forward2"):
            out += [(f"{p}.{ff}.ffw_layer_1", 1.0), (f"{p}.{ff}.ffw_layer_2", 0.5 * first)]
        out += [(f"{p}.self_attn.{proj}", 1.0) for proj in ("q_proj", "k_proj", "v_proj")]
        out += [(f"{p}.self_attn.post", first), (f"{p}.lconv1d.linear_start", 1.0),
                (f"{p}.lconv1d.linear_end", 0.6)]
    return out


def _nontrivial_tower(cfg: ListenerConfig, w: dict[str, np.ndarray], seed: int) -> None:
    rng = np.random.default_rng([seed, 0x6E6F6E74])
    for name, shape, init in tower_weight_shapes(cfg):
        if init == "ones":
            w[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        elif name.endswith("per_dim_scale"):
            w[name] = (0.5 * rng.standard_normal(shape)).astype(np.float32)
        elif name == "output_proj.bias":
            w[name] = (0.05 * rng.standard_normal(shape)).astype(np.float32)
    shapes = {name: shape for name, shape, _ in tower_weight_shapes(cfg)}
    for prefix, in_scale in clippable_linears(cfg):
        k_in = shapes[prefix + ".linear.weight"][1]
        out_scale = 0.02 * np.sqrt(k_in) * in_scale
        c = rng.uniform(2.0, 3.0, size=4)
        w[prefix + ".input_min"] = _bf16_representable(-c[0] * in_scale)
        w[prefix + ".input_max"] = _bf16_representable(c[1] * in_scale)
        w[prefix + ".output_min"] = _bf16_representable(-c[2] * out_scale)
        w[prefix + ".output_max"] = _bf16_representable(c[3] * out_scale)


def _round_bf16(w: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Rounds every array to the nearest bf16 value (ties to even), kept as float32."""
    out = {}
    for k, v in w.items():
        shape = np.shape(v)
        a = np.array(v, dtype=np.float32).reshape(-1)
        u = a.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16).astype(np.uint32)
        out[k] = np.where(np.isfinite(a), r.view(np.float32), a).astype(np.float32).reshape(shape)
    return out


def synthetic_tower_weights(cfg: ListenerConfig, seed: int = 1234, nontrivial: bool = False) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    w = {name: _draw(rng, shape, init) for name, shape, init in tower_weight_shapes(cfg)}
    if nontrivial:
        _nontrivial_tower(cfg, w, seed)
        w = _round_bf16(w)
    return w


def synthetic_film_weights(cfg: ListenerConfig, seed: int = 4321, nontrivial: bool = False) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    w = {name: _draw(rng, shape, init) for name, shape, init in film_weight_shapes(cfg)}
    if nontrivial:
        r2 = np.random.default_rng([seed, 0x6E6F6E74])
        for name, shape, init in film_weight_shapes(cfg):
            if init == "ones":
                w[name] = (1.0 + 0.1 * r2.standard_normal(shape)).astype(np.float32)
            elif init == "zeros":
                w[name] = (0.05 * r2.standard_normal(shape)).astype(np.float32)
        w = _round_bf16(w)
    return w


def session_audio(seed: int, session: int, n_frames: int, first_frame: int = 0,
                  total_frames: int | None = None) -> np.ndarray:
    """[n_frames, 1280] float32 PCM for one session (frames first_frame.. of it)."""
    rng = np.random.default_rng([seed, session])
    f0, f1 = rng.uniform(150.0, 300.0, size=2)
    total = max(total_frames or (first_frame + n_frames), 1)
    n = n_frames * PCM_SAMPLES_PER_FRAME
    start = first_frame * PCM_SAMPLES_PER_FRAME
    t = (start + np.arange(n, dtype=np.float64)) / SAMPLE_RATE_HZ
    dur = total * PCM_SAMPLES_PER_FRAME / SAMPLE_RATE_HZ
    # instantaneous frequency glides f0 -> f1; phase = integral of frequency
    phase = f0 * t + 0.5 * (f1 - f0) * t * t / dur
    saw = 2.0 * (phase - np.floor(phase + 0.5))
    noise_rng = np.random.default_rng([seed, session, first_frame])
    pcm = 0.05 * noise_rng.standard_normal(n) + 0.1 * saw
    return pcm.astype(np.float32).reshape(n_frames, PCM_SAMPLES_PER_FRAME)


def seeded_mel(seed: int, n: int) -> np.ndarray:
    """[n, 8, 128] standard-normal mel ticks (for tower-only parity cases)."""
    return np.random.default_rng(seed).standard_normal((n, 8, MEL_BINS), dtype=np.float32)


class ArrivalProcess:
    """Ragged session arrivals.

    ``pool`` mode (configs 2): ``num_sessions`` sessions, start ~ U{0..start_max},
    length ~ Geometric(1/mean_len).  ``lanes`` mode (configs 3-4): each of
    ``num_sessions`` lanes runs sessions back to back, so the number of
    concurrent sessions stays at ``num_sessions`` while sessions join and leave
    every step with differing cache positions.
    """

    def __init__(self, num_sessions: int, seed: int = 7, mean_len: float = 300.0,
                 start_max: int = 400, mode: str = "lanes"):
        self.rng = np.random.default_rng(seed)
        self.mode = mode
        self.mean_len = mean_len
        self.num = num_sessions
        p = 1.0 / mean_len
        if mode == "pool":
            self.start = self.rng.integers(0, start_max + 1, size=num_sessions)
            self.length = self.rng.geometric(p, size=num_sessions)
            self.session_id = np.arange(num_sessions, dtype=np.int64)
            self.pos = np.zeros(num_sessions, dtype=np.int64)
        else:
            self.start = np.zeros(num_sessions, dtype=np.int64)
            # start in the stationary state of back-to-back geometric sessions:
            # both the age and the remaining life of a live session are geometric,
            # so cache positions differ from step 0 and ~num/mean_len join per step
            self.pos = self.rng.geometric(p, size=num_sessions).astype(np.int64) - 1
            self.length = self.pos + self.rng.geometric(p, size=num_sessions)
            self.session_id = np.arange(num_sessions, dtype=np.int64)
            self._next_id = num_sessions
        self.step_index = 0

    def step(self) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        """Advance one tick.  Returns (lane, session_id, frame_id, is_new) of active rows."""
        t = self.step_index
        self.step_index += 1
        if self.mode == "pool":
            active = (self.start <= t) & (t < self.start + self.length)
            lanes = np.nonzero(active)[0]
            frame = t - self.start[lanes]
            return lanes, self.session_id[lanes], frame.astype(np.int64), frame == 0
        ended = self.pos >= self.length
        if ended.any():
            k = int(ended.sum())
            self.session_id[ended] = np.arange(self._next_id, self._next_id + k)
            self._next_id += k
            self.length[ended] = self.rng.geometric(1.0 / self.mean_len, size=k)
            self.pos[ended] = 0
        lanes = np.arange(self.num)
        frame = self.pos.copy()
        self.pos += 1
        return lanes, self.session_id.copy(), frame, frame == 0
