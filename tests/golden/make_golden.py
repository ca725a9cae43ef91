"""Generates the golden fixtures under tests/golden/ by running the REFERENCE.

Run in the build container, where the reference checkout and its pinned
dependency (transformers 5.5.0) are importable:

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py <reference checkout>

It imports the reference's own classes and records their outputs on seeded
synthetic inputs (the reference ships no weights, WAVs or fixtures for this
path).  Weights are regenerated from seeds by the package's
``synthetic_*_weights`` (numpy PCG64, platform independent), so the fixtures
store only inputs that are cheap to regenerate and the reference outputs.

Fixtures:
  mel.npz            GemmaAudioTowerBackend._extract_single_frame over seeded PCM
  tower_tiny.npz     StreamingConformerAudioTower (hidden 32, the reference test's
                     tiny config) over a 2-session trace with reorder, reset, gap,
                     epoch change and input masks
  tower_small.npz    same at the SMALL config (d=256) used by the GPU parity tests
  tower_full.npz     the BASELINE config-0 tower (d=1536, 12 layers), 1 session x 4 ticks
  tower_small_nt.npz the SMALL trace with non-identity parameters (synthetic
                     ``nontrivial=True``: norm weights, per_dim_scale, output_proj
                     bias and finite clip bounds on every clippable linear)
  tower_full_nt.npz  the config-0 tower with non-identity parameters over the
                     first 18 ticks of the 3-session trace (reorder, cursor gap,
                     epoch change, input masks)
  pcm_tower_nt.npz   PCM -> _extract_single_frame -> StreamingConformerAudioTower
                     (SMALL, non-identity parameters), 3 sessions x 12 ticks
  control6.npz       NativeControl6LoRA (rank 16) + the batch policy's selection
                     over 24 seeded rows, with and without phase_t
  film.npz           FrameResidualQueryFiLMAdapter (1536/2048/256 and the SMALL dims),
                     default and non-identity LayerNorm parameters
  packer.npz         slot ids / reasons / committed positions of the tower's slot
                     policy (``events``), the tick dispatcher's snapshot order
                     (``dispatch``), and the ListenerMicrobatchCoordinator's
                     dispatched rows and reasons on a seeded enqueue/take trace
                     (``coordinator``)
"""
from __future__ import annotations

import importlib.util
import json
import queue
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def load_pkg():
    pkg_dir = ROOT / "gemma-4-omni_b200"
    spec = importlib.util.spec_from_file_location("gemma4_omni_b200", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["gemma4_omni_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def build_reference_tower(cfg, tower_w):
    """transformers Gemma4AudioModel + Gemma4MultimodalEmbedder loaded with tower_w."""
    from transformers.models.gemma4 import modeling_gemma4
    from transformers.models.gemma4.configuration_gemma4 import Gemma4AudioConfig, Gemma4TextConfig

    audio_config = Gemma4AudioConfig(
        hidden_size=cfg.hidden, num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
        subsampling_conv_channels=(cfg.sub_ch0, cfg.sub_ch1), conv_kernel_size=5,
        attention_chunk_size=12, attention_context_left=13, attention_context_right=0,
        output_proj_dims=cfg.output_dims, rms_norm_eps=1e-6, use_clipped_linears=True)
    text_config = Gemma4TextConfig(
        hidden_size=cfg.text_hidden, num_hidden_layers=1, num_attention_heads=2,
        layer_types=["full_attention"],
        rope_parameters={"rope_type": "proportional", "partial_rotary_factor": 0.25,
                         "rope_theta": 1_000_000.0})
    tower = modeling_gemma4.Gemma4AudioModel(audio_config).eval()
    embed = modeling_gemma4.Gemma4MultimodalEmbedder(audio_config, text_config).eval()
    assert audio_config.intermediate_size if hasattr(audio_config, "intermediate_size") else True
    t_sd = {k: torch.from_numpy(v) for k, v in tower_w.items() if not k.startswith("embed.")}
    e_sd = {k[len("embed."):]: torch.from_numpy(v) for k, v in tower_w.items() if k.startswith("embed.")}
    missing, unexpected = tower.load_state_dict(t_sd, strict=False)
    assert not unexpected, unexpected
    # the remaining buffers are the clip bounds (+/-inf) and the rel-pos inv_timescales
    assert all(k.endswith(("input_min", "input_max", "output_min", "output_max")) for k in missing), missing
    embed.load_state_dict(e_sd, strict=True)
    return tower, embed


def tiny_config(pkg):
    from gemma4_omni_b200.config import ListenerConfig
    # the reference test's tiny tower (tests/kernel/test_streaming_conformer_q2.py:28-56)
    return ListenerConfig(hidden=32, layers=3, heads=4, ffn=128, sub_ch0=128, sub_ch1=4,
                          output_dims=24, text_hidden=24, film_enabled=False)


def tower_trace(cfg, seed: int, kind: str):
    """A 2-session event trace: (cursors, mel, mask) per tick, as the reference test mixes them."""
    rng = np.random.default_rng(seed)
    ticks = []
    # 4 aligned ticks, one reordered tick, reset of A (gap cursor), gap, epoch change, masked ticks
    plan = [
        [("A", 0, "e0", 0), ("B", 0, "e0", 0)],
        [("A", 0, "e0", 1), ("B", 0, "e0", 1)],
        [("A", 0, "e0", 2), ("B", 0, "e0", 2)],
        [("B", 0, "e0", 3), ("A", 0, "e0", 3)],
        [("B", 0, "e0", 4), ("A", 0, "e0", 20)],      # A gap -> gap_or_cursor_mismatch
        [("A", 0, "e0", 21), ("B", 0, "e0", 5)],
        [("A", 1, "e1", 0)],                          # epoch change -> identity_reset
        [("A", 1, "e1", 1), ("B", 0, "e0", 6), ("C", 0, "e0", 0)],
    ]
    for k in range(8, 30 if kind != "full" else 8):
        plan.append([("A", 1, "e1", k - 6), ("B", 0, "e0", k - 1), ("C", 0, "e0", k - 7)])
    if kind == "full":
        plan = [[("A", 0, "e0", i)] for i in range(4)]
    if kind == "full_nt":
        plan = plan[:18]
    for t, rows in enumerate(plan):
        mel = rng.standard_normal((len(rows), 8, 128), dtype=np.float32)
        mask = np.ones((len(rows), 8), dtype=bool)
        if kind != "full" and t in (2, 9, 10):
            mask[0, rng.integers(0, 8, size=3)] = False
        ticks.append((rows, mel, mask))
    return ticks


def run_tower(pkg, cfg, seed_w: int, seed_trace: int, kind: str, nontrivial: bool = False):
    from duplex_kernel.streaming_conformer import AudioStreamCursor, StreamingConformerAudioTower
    from gemma4_omni_b200.synthetic import synthetic_tower_weights

    tower_w = synthetic_tower_weights(cfg, seed_w, nontrivial=nontrivial)
    tower, embed = build_reference_tower(cfg, tower_w)
    st = StreamingConformerAudioTower(tower, embed, device="cpu", dtype=torch.float32, max_sessions=6)
    out = {"seed_w": seed_w, "seed_trace": seed_trace, "nontrivial": np.bool_(nontrivial)}
    rows_meta, raws, softs, subs, layers, slots, reasons = [], [], [], [], [], [], []
    mels, masks = [], []
    with torch.inference_mode():
        for rows, mel, mask in tower_trace(cfg, seed_trace, kind):
            cursors = tuple(AudioStreamCursor(s, g, e, f, f) for s, g, e, f in rows)
            p = st.prepare_batch(torch.from_numpy(mel), cursors, input_mask=torch.from_numpy(mask))
            raws.append(p.raw_tokens.numpy().copy())
            softs.append(p.soft_tokens.numpy().copy())
            subs.append(p.subsampled.numpy().copy())
            layers.append(np.stack([x.numpy() for x in p.layer_tokens]))
            slots.append(np.asarray(p.slot_ids))
            reasons.append(list(p.reset_reasons))
            rows_meta.append(rows)
            mels.append(mel)
            masks.append(mask)
            p.commit()
    n = [len(r) for r in rows_meta]
    out.update(
        rows=json.dumps(rows_meta), reasons=json.dumps(reasons), counts=np.asarray(n),
        mel=np.concatenate(mels), mask=np.concatenate(masks), raw=np.concatenate(raws),
        soft=np.concatenate(softs), sub=np.concatenate(subs), slots=np.concatenate(slots),
        layers=np.concatenate(layers, axis=1))
    return out


def make_pcm_tower(pkg):
    """PCM -> the reference's incremental mel (_extract_single_frame, tail carried
    per session) -> StreamingConformerAudioTower (SMALL, non-identity bf16
    parameters), 3 sessions over 12 ticks with a late join and a reorder."""
    from transformers.models.gemma4.feature_extraction_gemma4 import Gemma4AudioFeatureExtractor
    from duplex_kernel.listener import GemmaAudioTowerBackend
    from duplex_kernel.streaming_conformer import AudioStreamCursor, StreamingConformerAudioTower
    from gemma4_omni_b200.config import SMALL
    from gemma4_omni_b200.synthetic import session_audio, synthetic_tower_weights

    shim = SimpleNamespace(feature_extractor=Gemma4AudioFeatureExtractor())
    tower, embed = build_reference_tower(SMALL, synthetic_tower_weights(SMALL, 35, nontrivial=True))
    st = StreamingConformerAudioTower(tower, embed, device="cpu", dtype=torch.float32, max_sessions=4)
    audio = {s: session_audio(11, i, 12, total_frames=12) for i, s in enumerate(("u", "v", "w"))}
    tails, frames = {}, {"u": 0, "v": 0, "w": 0}
    rows_meta, pcms, softs, raws = [], [], [], []
    with torch.inference_mode():
        for t in range(12):
            sids = ["u", "v"] if t < 3 else (["w", "u", "v"] if t % 2 else ["u", "v", "w"])
            pcm = np.stack([audio[s][frames[s]] for s in sids])
            mels = []
            for i, s in enumerate(sids):
                m, tails[s] = GemmaAudioTowerBackend._extract_single_frame(shim, pcm[i], tails.get(s))
                mels.append(m)
            cursors = tuple(AudioStreamCursor(s, 0, "e0", frames[s], frames[s]) for s in sids)
            p = st.prepare_batch(torch.from_numpy(np.stack(mels)), cursors)
            raws.append(p.raw_tokens.numpy().copy())
            softs.append(p.soft_tokens.numpy().copy())
            p.commit()
            rows_meta.append([[s, 0, "e0", frames[s]] for s in sids])
            pcms.append(pcm)
            for s in sids:
                frames[s] += 1
    return {"seed_w": 35, "nontrivial": np.bool_(True), "rows": json.dumps(rows_meta),
            "pcm": np.concatenate(pcms), "raw": np.concatenate(raws), "soft": np.concatenate(softs)}


def make_control6(pkg):
    """NativeControl6LoRA.forward on bf16 tied rows + the batch policy's per-row
    selection (gemma_native_control6_batch_policy.py:878-893) on seeded inputs:
    ties, restricted and single-action legal sets, phase_t on and off."""
    from training.duplex_qlora.native_control6 import NativeControl6LoRA

    g = torch.Generator().manual_seed(606)
    base_rows = (torch.randn(6, 1536, generator=g) * 0.05).to(torch.bfloat16)
    torch.manual_seed(607)
    ad = NativeControl6LoRA(base_rows, rank=16, alpha=32.0).eval()
    with torch.no_grad():
        ad.lora_B.copy_(torch.randn(6, 16, generator=g) * 0.05)
    n = 24
    hidden = torch.randn(n, 1536, generator=g).to(torch.bfloat16)
    hidden[5] = hidden[4]  # identical rows
    phase = torch.randn(n, 4, generator=g)
    legal = torch.rand(n, 6, generator=g) < 0.6
    legal[0] = True
    legal[1] = False
    legal[1, 3] = True  # a single legal action
    legal[legal.sum(1) == 0, 0] = True
    out = {}
    with torch.inference_mode():
        for tag, ph in (("phase", phase), ("nophase", None)):
            logits = ad(hidden, phase_t=ph).float()
            finite = torch.isfinite(logits).all(dim=1).float()
            raw = logits.argmax(dim=1)
            selected_logits = logits.masked_fill(~legal, -torch.inf)
            sel = selected_logits.argmax(dim=1)
            conf = torch.softmax(selected_logits, dim=1).gather(1, sel.unsqueeze(1)).squeeze(1)
            out[f"{tag}_logits"] = logits.numpy()
            out[f"{tag}_packet"] = torch.stack((finite, raw.float(), sel.float(), conf), dim=1).numpy()
    out.update(hidden=hidden.float().numpy(), phase=phase.numpy(), legal=legal.numpy(),
               base_rows=base_rows.float().numpy(), lora_a=ad.lora_A.detach().numpy(),
               lora_b=ad.lora_B.detach().numpy(), scaling=np.float32(ad.scaling))
    return out


def make_mel(pkg):
    from transformers.models.gemma4.feature_extraction_gemma4 import Gemma4AudioFeatureExtractor
    from duplex_kernel.listener import GemmaAudioTowerBackend
    from gemma4_omni_b200.synthetic import session_audio

    fe = Gemma4AudioFeatureExtractor()
    shim = SimpleNamespace(feature_extractor=fe)
    pcm = np.concatenate([session_audio(3, s, 6, total_frames=6) for s in range(3)])  # [18, 1280]
    pcm[5] = 0.0  # a silent frame
    mels, tails = [], []
    for s in range(3):
        tail = None
        for f in range(6):
            m, tail = GemmaAudioTowerBackend._extract_single_frame(shim, pcm[s * 6 + f], tail)
            mels.append(m)
            tails.append(tail)
    return dict(pcm=pcm, mel=np.stack(mels), tail=np.stack(tails))


def make_film(pkg):
    from duplex_kernel.frame_residual_adapter import FrameResidualQueryFiLMAdapter
    from gemma4_omni_b200.config import FULL, SMALL
    from gemma4_omni_b200.synthetic import synthetic_film_weights

    out = {}
    for tag, cfg, nt in (("full", FULL, False), ("small", SMALL, False), ("full_nt", FULL, True),
                         ("small_nt", SMALL, True)):
        w = synthetic_film_weights(cfg, 77, nontrivial=nt)
        w["output.weight"] = w["output.weight"] * 300.0  # make the residual clearly non-trivial
        ad = FrameResidualQueryFiLMAdapter(cfg.text_hidden, cfg.film_query_dim, cfg.film_bottleneck).eval()
        ad.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in w.items()}, strict=True)
        g = torch.Generator().manual_seed(78)
        hidden = torch.randn(3, 2, cfg.text_hidden, generator=g)
        query = torch.randn(3, 2, cfg.film_query_dim, generator=g)
        with torch.no_grad():
            y = ad(hidden, query)
        out[f"{tag}_hidden"] = hidden.numpy()
        out[f"{tag}_query"] = query.numpy()
        out[f"{tag}_out"] = y.numpy()
        out[f"{tag}_output_weight_scale"] = np.float32(300.0)
    return out


def make_packer(pkg):
    """Slot policy, dispatcher snapshot and coordinator order on seeded traces."""
    from duplex_kernel.streaming_conformer import AudioStreamCursor, StreamingConformerAudioTower
    from duplex_kernel.shared_listener_scheduler import SharedListenerTickDispatcher
    from duplex_kernel.scheduler import AudioFrame
    from gemma4_omni_b200.synthetic import synthetic_tower_weights

    cfg = tiny_config(pkg)
    tower, embed = build_reference_tower(cfg, synthetic_tower_weights(cfg, 5))
    S = 6
    st = StreamingConformerAudioTower(tower, embed, device="cpu", dtype=torch.float32, max_sessions=S)
    rng = np.random.default_rng(2024)
    sessions = [f"s{i}" for i in range(9)]
    gen = {s: 0 for s in sessions}
    nxt = {s: 0 for s in sessions}
    events = []  # per step: dict(rows=[(sid,gen,epoch,frame,seq)], op=..., slots, reasons, committed, error)
    for step in range(60):
        op = {"kind": "step"}
        r = rng.random()
        if r < 0.08:
            sid = sessions[rng.integers(0, len(sessions))]
            st.reset(sid)
            events.append({"kind": "reset", "sid": sid, "committed": st.committed_positions})
            continue
        if r < 0.12:
            bound = sorted(set(st._slots_by_key.values()))  # noqa: SLF001
            slot = int(bound[rng.integers(0, len(bound))]) if bound else 0
            st.reset_session(slot)
            events.append({"kind": "reset_session", "slot": slot, "committed": st.committed_positions})
            continue
        n = int(rng.integers(1, 6))
        chosen = [sessions[i] for i in rng.choice(len(sessions), size=n, replace=False)]
        rows = []
        for sid in chosen:
            u = rng.random()
            if u < 0.1:
                gen[sid] += 1
                nxt[sid] = 0
            elif u < 0.18:
                nxt[sid] += int(rng.integers(2, 5))  # cursor gap
            rows.append((sid, gen[sid], f"ep{gen[sid]}", nxt[sid], nxt[sid]))
        cursors = tuple(AudioStreamCursor(*row) for row in rows)
        mel = torch.zeros((n, 8, 128))
        try:
            p = st.prepare_batch(mel, cursors)
        except RuntimeError as exc:
            events.append({"kind": "step", "rows": rows, "error": str(exc), "committed": st.committed_positions})
            continue
        action = "commit" if rng.random() < 0.85 else "abort"
        rec = {"kind": "step", "rows": rows, "slots": list(p.slot_ids), "reasons": list(p.reset_reasons),
               "action": action}
        if action == "commit":
            p.commit()
            for sid, g, e, f, q in rows:
                nxt[sid] = f + 1
        else:
            p.abort()
        rec["committed"] = st.committed_positions
        events.append(rec)
    # dispatcher snapshot order (registration order, paused, deferral after deadline)
    disp = SharedListenerTickDispatcher(lambda rows: {})
    queues = {}
    for i, sid in enumerate(["d0", "d1", "d2", "d3", "d4"]):
        queues[sid] = queue.Queue()
        disp.register_session(sid, queues[sid])
    disp._paused_sessions.add("d3")  # noqa: SLF001
    deadline = 1_000_000
    frames_in = [("d0", 0, 10), ("d1", 0, 2_000_000), ("d2", 0, 5), ("d3", 0, 7), ("d4", 0, 999_999),
                 ("d1", 1, 2_000_001), ("d2", 1, 1_500_000)]
    for sid, fid, enq in frames_in:
        queues[sid].put(AudioFrame(frame_id=fid, pcm=np.zeros(1280, np.float32), capture_start_ns=0,
                                   capture_end_ns=0, enqueue_ns=enq))
    tick0 = [r.session_id for r in disp._snapshot_ready_rows(0, deadline, deadline)]  # noqa: SLF001
    deferred0 = sorted(disp._deferred)  # noqa: SLF001
    tick1 = [r.session_id for r in disp._snapshot_ready_rows(1, 3_000_000, 3_000_000)]  # noqa: SLF001
    dispatch = {"frames": frames_in, "paused": ["d3"], "registrations": ["d0", "d1", "d2", "d3", "d4"],
                "tick0": tick0, "deferred0": deferred0, "tick1": tick1, "deadline0": deadline,
                "deadline1": 3_000_000}
    return {"events": json.dumps(events), "max_sessions": np.int64(S), "dispatch": json.dumps(dispatch),
            "coordinator": json.dumps(make_coordinator())}


def make_coordinator():
    """ListenerMicrobatchCoordinator.take_ready on a seeded enqueue/take trace.

    Sessions are registered in a shuffled order; frames arrive with jittered
    ready times (ties included, so submission order and session id break
    them); take_ready runs at times that hit the 2 ms singleton coalesce window
    on both sides; a batch stays in flight for a random number of takes (no
    further batch while one is active) before ``complete``.  Records every
    take's dispatched (session, frame) rows in order and its reason.
    """
    from duplex_kernel.listener_microbatch import ListenerMicrobatchCoordinator
    from duplex_kernel.microbatch_contract import (ListenerFrame, ListenerSessionState, NativeBatchCapability,
                                                   RowStateUpdate, RuntimeSignature)

    sig = RuntimeSignature(model_id="google/gemma-4-E2B-it", model_config_sha256="a" * 64,
                           checkpoint_sha256="b" * 64, topology_sha256="c" * 64,
                           native_library_sha256="d" * 64, native_abi_version=3, batch_api_version=2,
                           attention_backend_id=3, rmsnorm_backend_id=2, max_seq_len=16_384, stream_q_len=2)
    cap = NativeBatchCapability(api_version=2, native_abi_version=3, attention_backend_id=3,
                                rmsnorm_backend_id=2, max_seq_len=16_384, stream_q_len=2,
                                supports_arbitrary_batch_size=True, stream_priority=-1,
                                stream_identity="listener-stream")
    coord = ListenerMicrobatchCoordinator(sig, cap)
    rng = np.random.default_rng(4242)
    sessions = [f"c{i:02d}" for i in rng.permutation(6)]
    for i, sid in enumerate(sessions):
        coord.register_session(ListenerSessionState(
            session_id=sid, generation_id=1, state_epoch_id=f"ep-{sid}", runtime_signature=sig,
            next_frame_id=0, state_version=0, sequence_position=0, cache_position=34,
            valid_history_tokens=34, native_context_id=20_000 + i))
    next_frame = {sid: 0 for sid in sessions}
    events = []
    now = 1_000_000
    active = None
    hold = 0
    for step in range(160):
        now += int(rng.choice([0, 300_000, 1_000_000, 1_999_999, 2_000_000, 2_500_000, 80_000_000]))
        for _ in range(int(rng.choice([0, 0, 1, 1, 1, 2, 4, 6]))):
            sid = sessions[int(rng.integers(0, len(sessions)))]
            ready = now + int(rng.choice([-3_000_000, -2_000_000, -500_000, 0, 0, 700_000, 4_000_000]))
            ready = max(ready, 0)
            coord.enqueue(ListenerFrame(session_id=sid, generation_id=1, state_epoch_id=f"ep-{sid}",
                                        frame_id=next_frame[sid], ready_at_ns=ready,
                                        pcm=np.zeros(1280, np.float32)))
            events.append({"kind": "enqueue", "sid": sid, "frame": next_frame[sid], "ready_at": ready})
            next_frame[sid] += 1
        if active is not None:
            if hold > 0:
                hold -= 1
                events.append({"kind": "take", "now": now, "rows": None, "reason": None, "active": True})
                assert coord.take_ready(now) is None
                continue
            coord.complete(active, tuple(RowStateUpdate(session_id=r.session_id, frame_id=r.frame_id,
                                                        cache_position=r.cache_position + 2,
                                                        valid_history_tokens=r.cache_position + 2)
                                         for r in active.manifest.rows))
            events.append({"kind": "complete"})
            active = None
        batch = coord.take_ready(now)
        if batch is None:
            events.append({"kind": "take", "now": now, "rows": None, "reason": None, "active": False})
            continue
        rows = [[r.session_id, r.frame_id] for r in batch.manifest.rows]
        events.append({"kind": "take", "now": now, "rows": rows, "reason": batch.manifest.dispatch_reason,
                       "active": False})
        active = batch
        hold = int(rng.integers(0, 3))
    return {"registrations": sessions, "coalesce_ns": coord.coalesce_window_ns, "events": events}


def main() -> None:
    """``make_golden.py <reference checkout> [fixture ...]``: writes every
    fixture, or only the named ones (file stems, e.g. ``tower_full_nt``)."""
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "/nonexistent")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    only = set(sys.argv[2:])
    torch.set_num_threads(4)
    pkg = load_pkg()
    from gemma4_omni_b200.config import FULL, SMALL

    def full_tower(seed_w, seed_trace, kind, nontrivial=False):
        out = run_tower(pkg, FULL, seed_w, seed_trace, kind, nontrivial=nontrivial)
        out.pop("layers")  # keep the fixture small: raw/soft/sub only
        return out

    makers = {
        "mel": lambda: make_mel(pkg),
        "film": lambda: make_film(pkg),
        "packer": lambda: make_packer(pkg),
        "tower_tiny": lambda: run_tower(pkg, tiny_config(pkg), 23, 9917, "tiny"),
        "tower_small": lambda: run_tower(pkg, SMALL, 31, 712, "small"),
        "tower_full": lambda: full_tower(41, 125, "full"),
        "tower_small_nt": lambda: run_tower(pkg, SMALL, 33, 713, "small", nontrivial=True),
        "tower_full_nt": lambda: full_tower(43, 126, "full_nt", nontrivial=True),
        "pcm_tower_nt": lambda: make_pcm_tower(pkg),
        "control6": lambda: make_control6(pkg),
    }
    unknown = only - set(makers)
    if unknown:
        raise SystemExit(f"unknown fixtures: {sorted(unknown)}")
    for name, make in makers.items():
        if not only or name in only:
            np.savez_compressed(HERE / f"{name}.npz", **make())
            print("wrote", HERE / f"{name}.npz")


if __name__ == "__main__":
    main()
