"""Pins the CPU oracle against golden vectors produced by the reference itself.

tests/golden/make_golden.py ran the reference's StreamingConformerAudioTower,
_extract_single_frame, FrameResidualQueryFiLMAdapter, tick dispatcher and slot
policy on seeded inputs; these tests check that the oracle restatement
reproduces them (fp32 vs fp32: the reference's own parity tolerance
rtol 2e-5 / atol 2e-6, tests/kernel/test_streaming_conformer_q2.py:261-268).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import conformer_ref, film_ref, mel_ref, packer_ref

GOLD = Path(__file__).resolve().parent / "golden"


def _ocfg(cfg):
    return conformer_ref.OracleConfig(hidden=cfg.hidden, layers=cfg.layers, heads=cfg.heads, ffn=cfg.ffn,
                                      sub_ch0=cfg.sub_ch0, sub_ch1=cfg.sub_ch1, output_dims=cfg.output_dims,
                                      text_hidden=cfg.text_hidden)


def replay_tower(pkg, cfg, g):
    """Drives the oracle through a golden trace; returns (raw, soft, sub, layers) stacked like the golden."""
    from gemma4_omni_b200.synthetic import synthetic_tower_weights
    from helpers import replay_oracle_trace

    nontrivial = bool(g["nontrivial"]) if "nontrivial" in g.files else False
    w = {k: torch.from_numpy(np.asarray(v))
         for k, v in synthetic_tower_weights(cfg, int(g["seed_w"]), nontrivial=nontrivial).items()}
    return replay_oracle_trace(conformer_ref.OracleConformer(w, _ocfg(cfg)), g)


@pytest.mark.parametrize("fixture", ["tower_tiny", "tower_small", "tower_small_nt"])
def test_oracle_tower_matches_reference_trace(pkg, fixture):
    from gemma4_omni_b200.config import SMALL, ListenerConfig

    g = np.load(GOLD / f"{fixture}.npz")
    cfg = SMALL if fixture.startswith("tower_small") else ListenerConfig(
        hidden=32, layers=3, heads=4, ffn=128, sub_ch1=4, output_dims=24, text_hidden=24, film_enabled=False)
    raw, soft, sub, layers = replay_tower(pkg, cfg, g)
    torch.testing.assert_close(sub, torch.from_numpy(g["sub"]), rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(layers, torch.from_numpy(g["layers"]), rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(raw, torch.from_numpy(g["raw"]), rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(soft, torch.from_numpy(g["soft"]), rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("fixture", ["tower_full", "tower_full_nt"])
def test_oracle_full_config_tower_matches_reference(pkg, fixture):
    from gemma4_omni_b200.config import FULL

    g = np.load(GOLD / f"{fixture}.npz")
    raw, soft, sub, _ = replay_tower(pkg, FULL, g)
    torch.testing.assert_close(sub, torch.from_numpy(g["sub"]), rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(raw, torch.from_numpy(g["raw"]), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(soft, torch.from_numpy(g["soft"]), rtol=1e-4, atol=1e-4)


def test_oracle_mel_matches_reference_extractor():
    g = np.load(GOLD / "mel.npz")
    pcm = g["pcm"]
    mels, tails = [], []
    for s in range(3):
        tail = None
        for f in range(6):
            m, tail = mel_ref.extract_single_frame(pcm[s * 6 + f], tail)
            mels.append(m)
            tails.append(tail)
    np.testing.assert_array_equal(np.stack(mels), g["mel"])
    np.testing.assert_array_equal(np.stack(tails), g["tail"])


@pytest.mark.parametrize("tag", ["full", "small", "full_nt", "small_nt"])
def test_oracle_film_matches_reference_adapter(pkg, tag):
    from gemma4_omni_b200.config import FULL, SMALL
    from gemma4_omni_b200.synthetic import synthetic_film_weights

    g = np.load(GOLD / "film.npz")
    cfg = FULL if tag.startswith("full") else SMALL
    w = {k: torch.from_numpy(np.asarray(v))
         for k, v in synthetic_film_weights(cfg, 77, nontrivial=tag.endswith("_nt")).items()}
    w["output.weight"] = w["output.weight"] * float(g[f"{tag}_output_weight_scale"])
    y = film_ref.film_forward(w, torch.from_numpy(g[f"{tag}_hidden"]), torch.from_numpy(g[f"{tag}_query"]))
    ref = torch.from_numpy(g[f"{tag}_out"])
    torch.testing.assert_close(y, ref, rtol=2e-5, atol=2e-5)
    # the residual is clearly non-trivial (otherwise the check would be vacuous)
    assert (ref - torch.from_numpy(g[f"{tag}_query"])).abs().max() > 1e-2


def test_oracle_slot_policy_replays_reference_trace():
    g = np.load(GOLD / "packer.npz")
    pol = packer_ref.SlotPolicy(int(g["max_sessions"]))
    for ev in json.loads(str(g["events"])):
        if ev["kind"] == "reset":
            pol.reset(ev["sid"])
        elif ev["kind"] == "reset_session":
            pol.reset_session(ev["slot"])
        else:
            rows = [tuple(r) for r in ev["rows"]]
            if "error" in ev:
                with pytest.raises(RuntimeError):
                    pol.prepare(rows)
            else:
                p = pol.prepare(rows)
                assert p.slots == ev["slots"]
                assert p.reasons == ev["reasons"]
                pol.commit() if ev["action"] == "commit" else pol.abort()
        assert [list(x) for x in pol.committed_positions] == [list(x) for x in ev["committed"]]


def test_oracle_dispatch_snapshot_matches_reference():
    d = json.loads(str(np.load(GOLD / "packer.npz")["dispatch"]))
    ingress: dict[str, list] = {}
    for sid, fid, enq in d["frames"]:
        ingress.setdefault(sid, []).append(packer_ref.TickFrame(sid, fid, enq))
    deferred: dict = {}
    paused = set(d["paused"])
    t0 = packer_ref.snapshot_ready_rows(d["registrations"], paused, ingress, deferred, d["deadline0"])
    assert [f.session_id for f in t0] == d["tick0"]
    assert sorted(deferred) == d["deferred0"]
    t1 = packer_ref.snapshot_ready_rows(d["registrations"], paused, ingress, deferred, d["deadline1"])
    assert [f.session_id for f in t1] == d["tick1"]


def test_oracle_coordinator_order_matches_reference():
    """order_ready_heads vs the reference coordinator's take_ready on a seeded
    enqueue/take trace with every dispatch reason (listener_microbatch.py:170-279)."""
    from helpers import replay_coordinator

    g = json.loads(str(np.load(GOLD / "packer.npz")["coordinator"]))
    reasons = {ev["reason"] for ev in g["events"] if ev["kind"] == "take"}
    assert {"batch_full", "multiple_ready", "coalesce_deadline", None} <= reasons
    assert replay_coordinator(g, packer_ref.order_ready_heads) > 50


def test_oracle_control6_head_matches_reference():
    """The Control6 head restatement vs NativeControl6LoRA + the batch policy's
    selection (tests/golden/control6.npz)."""
    from oracle import control6_ref

    g = np.load(GOLD / "control6.npz")
    args = (torch.from_numpy(g["legal"]), torch.from_numpy(g["base_rows"]).to(torch.bfloat16),
            torch.from_numpy(g["lora_a"]), torch.from_numpy(g["lora_b"]), float(g["scaling"]))
    hidden = torch.from_numpy(g["hidden"]).to(torch.bfloat16)
    for tag, phase in (("phase", torch.from_numpy(g["phase"])), ("nophase", None)):
        logits, packet = control6_ref.control6_head(hidden, phase, *args)
        torch.testing.assert_close(logits, torch.from_numpy(g[f"{tag}_logits"]), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(packet, torch.from_numpy(g[f"{tag}_packet"]), rtol=1e-5, atol=1e-6)
