"""Drop-in StreamingConformerAudioTower API on the GPU, modeled on the reference's
tests/kernel/test_streaming_conformer_q2.py (reorder/reset/gap/epoch isolation
:300-364, abort/retry and stale-cursor commit :367-390, slot release/reuse
:461-491), with the transformers Gemma4 audio modules as the weight source."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_parity
from oracle import conformer_ref

pytestmark = pytest.mark.gpu


def hf_modules(cfg, seed, nontrivial=True):
    from gemma4_omni_b200.synthetic import synthetic_tower_weights
    from transformers.models.gemma4 import modeling_gemma4
    from transformers.models.gemma4.configuration_gemma4 import Gemma4AudioConfig, Gemma4TextConfig

    ac = Gemma4AudioConfig(hidden_size=cfg.hidden, num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                           subsampling_conv_channels=(cfg.sub_ch0, cfg.sub_ch1), output_proj_dims=cfg.output_dims)
    tc = Gemma4TextConfig(hidden_size=cfg.text_hidden, num_hidden_layers=1, num_attention_heads=2,
                          layer_types=["full_attention"],
                          rope_parameters={"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                           "rope_theta": 1_000_000.0})
    tower = modeling_gemma4.Gemma4AudioModel(ac).eval()
    embed = modeling_gemma4.Gemma4MultimodalEmbedder(ac, tc).eval()
    w = synthetic_tower_weights(cfg, seed, nontrivial=nontrivial)
    missing, _ = tower.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in w.items()
                                        if not k.startswith("embed.")}, strict=False)
    if nontrivial:  # every clip bound is set; only the rel-pos timescales are derived
        assert all("inv_timescales" in k for k in missing), missing
    embed.load_state_dict({k[6:]: torch.from_numpy(v) for k, v in w.items() if k.startswith("embed.")})
    # the reference tower requires its modules on the serving device and dtype already
    return tower.to("cuda", torch.bfloat16), embed.to("cuda", torch.bfloat16), w


@pytest.fixture(scope="module")
def modules(pkg):
    from gemma4_omni_b200.config import SMALL
    return hf_modules(SMALL, 41)


def tower(modules, max_sessions=8, layers=False):
    from gemma4_omni_b200.streaming_conformer import StreamingConformerAudioTower
    t, e, _ = modules
    return StreamingConformerAudioTower(t, e, device="cuda", dtype=torch.bfloat16, max_sessions=max_sessions,
                                        return_layer_tokens=layers)


def cursor(session, frame, generation=0, epoch="epoch-0"):
    from gemma4_omni_b200.streaming_conformer import AudioStreamCursor
    return AudioStreamCursor(session, generation, epoch, frame, frame)


def commit_tick(st, mel, cursors):
    p = st.prepare_batch(mel.cuda(), cursors)
    out = (p.raw_tokens.float().cpu(), p.soft_tokens.float().cpu())
    p.commit()
    return out


# The same session computed in another batch: a state mix-up between sessions
# would break the cosine bound; the relative bound allows a few bf16 ulps (2^-8
# each), since split-K partial sums reduce in a run-dependent fp32 order.
SAME_REL = 2e-2


def test_reorder_reset_gap_and_epoch_do_not_cross_contaminate(modules):
    chunks = torch.randn((9, 8, 128), generator=torch.Generator().manual_seed(125))
    shared, sep_a, sep_b = tower(modules), tower(modules), tower(modules)
    for f in range(4):
        pair = chunks[f:f + 1].expand(2, -1, -1).clone()
        got = commit_tick(shared, pair, (cursor("A", f), cursor("B", f)))[0]
        ra = commit_tick(sep_a, chunks[f:f + 1], (cursor("A", f),))[0]
        rb = commit_tick(sep_b, chunks[f:f + 1], (cursor("B", f),))[0]
        assert_parity(got[0:1], ra, "A", 0.99999, SAME_REL)
        assert_parity(got[1:2], rb, "B", 0.99999, SAME_REL)
    ba = commit_tick(shared, chunks[4:5].expand(2, -1, -1).clone(), (cursor("B", 4), cursor("A", 4)))[0]
    assert_parity(ba[0:1], commit_tick(sep_b, chunks[4:5], (cursor("B", 4),))[0], "B reordered", 0.99999, SAME_REL)
    assert_parity(ba[1:2], commit_tick(sep_a, chunks[4:5], (cursor("A", 4),))[0], "A reordered", 0.99999, SAME_REL)
    shared.reset("A", 0, "epoch-0")
    p = shared.prepare_batch(torch.cat((chunks[5:6], chunks[6:7])).cuda(), (cursor("B", 5), cursor("A", 20)))
    assert p.reset_reasons == ("continue", "identity_reset")
    reset_a = p.raw_tokens.float().cpu()[1:2]
    p.commit()
    fresh = tower(modules)
    assert_parity(reset_a, commit_tick(fresh, chunks[6:7], (cursor("A", 20),))[0], "reset A", 0.99999, SAME_REL)
    p = shared.prepare_batch(chunks[7:8].cuda(), (cursor("A", 22),))
    assert p.reset_reasons == ("gap_or_cursor_mismatch",)
    p.commit()
    p = shared.prepare_batch(chunks[8:9].cuda(), (cursor("A", 0, generation=1, epoch="epoch-1"),))
    assert p.reset_reasons == ("identity_reset",)
    epoch = p.raw_tokens.float().cpu()
    p.commit()
    fresh2 = tower(modules)
    ref = commit_tick(fresh2, chunks[8:9], (cursor("A", 0, generation=1, epoch="epoch-1"),))[0]
    assert_parity(epoch, ref, "epoch change", 0.99999, SAME_REL)
    assert shared.committed_positions == (("A", 1, "epoch-1", 1, 1), ("B", 0, "epoch-0", 6, 6))
    for t in (shared, sep_a, sep_b, fresh, fresh2):
        t.close()


def test_aborted_prepare_is_retryable_and_stale_cursor_prevents_commit(modules):
    st = tower(modules, 4)
    chunks = torch.randn((2, 8, 128), generator=torch.Generator().manual_seed(63)).cuda()
    first = st.prepare_batch(chunks, (cursor("A", 0), cursor("B", 0)))
    discarded = first.raw_tokens.clone()
    first.abort()
    retry = st.prepare_batch(chunks, (cursor("A", 0), cursor("B", 0)))
    assert_parity(retry.raw_tokens, discarded, "retry", 0.99999, 1e-2)
    retry.commit()
    pending = st.prepare_batch(chunks, (cursor("A", 1), cursor("B", 1)))
    before = pending.raw_tokens.clone()
    st._engine.debug_set_expected(st._handles["B"], 99, 99)
    with pytest.raises(RuntimeError, match="cursor changed before streaming commit"):
        pending.commit()
    st._engine.debug_set_expected(st._handles["B"], 1, 1)
    rerun = st.prepare_batch(chunks, (cursor("A", 1), cursor("B", 1)))
    assert_parity(rerun.raw_tokens, before, "rerun", 0.99999, 1e-2)
    rerun.abort()
    st.close()


def test_reset_session_releases_only_requested_slot_and_reuses_it(modules):
    st = tower(modules, 3)
    chunks = torch.randn((2, 8, 128), generator=torch.Generator().manual_seed(68)).cuda()
    p = st.prepare_batch(chunks, (cursor("slot-A", 0), cursor("slot-B", 0)))
    slot_a, slot_b = p.slot_ids
    assert slot_a != slot_b
    p.commit()
    pending = st.prepare_batch(chunks[:1], (cursor("slot-A", 1),))
    before = st.committed_positions
    with pytest.raises(RuntimeError, match="while a batch is prepared"):
        st.reset_session(slot_b)
    assert st.committed_positions == before
    pending.abort()
    with pytest.raises(IndexError):
        st.reset_session(3)
    with pytest.raises(TypeError):
        st.reset_session(True)
    st.reset_session(slot_a)
    assert st.committed_positions == (("slot-B", 0, "epoch-0", 1, 1),)
    reused = st.prepare_batch(chunks[:1], (cursor("slot-C", 0),))
    assert reused.slot_ids == (slot_a,)
    reused.commit()
    st.close()


def test_bank_exhaustion_and_contract_errors(modules):
    st = tower(modules, 2)
    x = torch.zeros((3, 8, 128), device="cuda")
    with pytest.raises(RuntimeError, match="exhausted"):
        st.prepare_batch(x, (cursor("a", 0), cursor("b", 0), cursor("c", 0)))
    with pytest.raises(ValueError, match="distinct"):
        st.prepare_batch(x[:2], (cursor("a", 0), cursor("a", 0)))
    with pytest.raises(ValueError):
        st.prepare_batch(x[:, :4], (cursor("a", 0),))
    p = st.prepare_batch(x[:2], (cursor("a", 0), cursor("b", 0)))
    with pytest.raises(RuntimeError, match="has not committed"):
        st.prepare_batch(x[:1], (cursor("a", 1),))
    p.commit()
    with pytest.raises(RuntimeError, match="already committed"):
        p.commit()
    p.rollback_committed()
    assert st.committed_positions == ()
    st.close()
    with pytest.raises(RuntimeError, match="closed"):
        st.prepare_batch(x[:1], (cursor("a", 0),))


def test_layer_tokens_match_oracle_with_masks(modules, pkg):
    from gemma4_omni_b200.config import SMALL
    from gemma4_omni_b200.weights import bf16_round
    from helpers import oracle_config

    st = tower(modules, 4, layers=True)
    _, _, w = modules
    eff = {k: torch.from_numpy(bf16_round(np.asarray(v))) for k, v in w.items()}
    model = conformer_ref.OracleConformer(eff, oracle_config(SMALL))
    state = conformer_ref.zero_state(model.cfg, 1)
    g = torch.Generator().manual_seed(712)
    for f in range(7):
        mel = torch.randn((1, 8, 128), generator=g)
        mask = torch.ones((1, 8), dtype=torch.bool)
        if f in (1, 4):
            mask[0, (0, 3, 6)] = False
        p = st.prepare_batch(mel.cuda(), (cursor("m", f),), input_mask=mask.cuda())
        raw, _, sub, layers, state = model.step(mel, mask, state, torch.tensor([f == 0]))
        assert_parity(p.subsampled, sub, f"sub {f}")
        for i, lay in enumerate(layers):
            assert_parity(p.layer_tokens[i], lay, f"layer {i} tick {f}")
        assert_parity(p.raw_tokens, raw, f"raw {f}")
        p.commit()
    st.close()


def test_validation_matches_reference_contract(modules):
    """Device, dtype, eval-mode and subsampler-geometry checks of the reference
    (streaming_conformer.py:375-407)."""
    from gemma4_omni_b200.streaming_conformer import StreamingConformerAudioTower
    t, e, _ = modules
    with pytest.raises(ValueError, match="requested dtype"):
        StreamingConformerAudioTower(t, e, device="cuda", dtype=torch.float32, max_sessions=4)
    with pytest.raises(ValueError, match="CUDA only"):
        StreamingConformerAudioTower(t, e, device="cpu", dtype=torch.bfloat16, max_sessions=4)
    conv = t.subsample_conv_projection.layer1.conv
    old = conv.stride
    conv.stride = (1, 1)
    try:
        with pytest.raises(ValueError, match="stride 2"):
            StreamingConformerAudioTower(t, e, device="cuda", dtype=torch.bfloat16, max_sessions=4)
    finally:
        conv.stride = old
    t.train()
    try:
        with pytest.raises(ValueError, match="eval mode"):
            StreamingConformerAudioTower(t, e, device="cuda", dtype=torch.bfloat16, max_sessions=4)
    finally:
        t.eval()


def test_session_churn_recycles_handles_and_matches_oracle(modules, pkg):
    """More than 10x max_handles distinct sessions through one tower: sessions
    join and leave every tick (leaving = close_session -> reset), abort and
    rollback release the handles they introduced, and every tick's raw tokens
    match the oracle."""
    from gemma4_omni_b200.config import SMALL
    from gemma4_omni_b200.weights import bf16_round
    from helpers import oracle_config

    st = tower(modules, 8)
    max_handles = st._engine.max_handles
    _, _, w = modules
    model = conformer_ref.OracleConformer({k: torch.from_numpy(bf16_round(np.asarray(v))) for k, v in w.items()},
                                          oracle_config(SMALL))
    zero = {k: v[0] for k, v in conformer_ref.zero_state(model.cfg, 1).items()}
    rng = np.random.default_rng(99)
    g = torch.Generator().manual_seed(98)
    live: dict[str, int] = {}  # session -> next frame
    states: dict[str, dict] = {}
    next_id = 0
    total = 0
    tick = 0
    while next_id < 10 * max_handles + 40:
        for sid in [s for s in live if rng.random() < 0.25]:  # leavers
            st.reset(sid)
            live.pop(sid)
            states.pop(sid, None)
        while len(live) < 8 and rng.random() < 0.9:  # joiners
            live[f"churn-{next_id}"] = 0
            next_id += 1
        if not live:
            continue
        sids = list(live)
        rng.shuffle(sids)
        n = len(sids)
        mel = torch.randn((n, 8, 128), generator=g)
        p = st.prepare_batch(mel.cuda(), tuple(cursor(s, live[s]) for s in sids))
        action = rng.random()
        if action < 0.08:
            p.abort()
            continue
        raw = p.raw_tokens.float().cpu()
        p.commit()
        if action < 0.12:
            p.rollback_committed()
            continue
        state = {k: torch.stack([states.get(s, zero)[k] for s in sids]) for k in zero}
        reset = torch.tensor([s not in states for s in sids])
        ref, _, _, _, nxt = model.step(mel, torch.ones(n, 8, dtype=torch.bool), state, reset)
        assert_parity(raw, ref, f"churn tick {tick}")
        for i, s in enumerate(sids):
            states[s] = {k: v[i] for k, v in nxt.items()}
            live[s] += 1
        total += n
        tick += 1
    assert next_id > 10 * max_handles and len(st._handles) <= 8
    assert len(st._free_handles) + len(st._handles) == max_handles
    assert st._engine.status() == 0
    st.close()


def test_pcm_entry_matches_cpu_mel_through_prepare_batch(modules):
    """prepare_batch_pcm (GPU log-mel with the tail in the slot) equals
    prepare_batch on the reference extractor's mel, across ticks, a reset and
    a session that joins late."""
    from gemma4_omni_b200 import synthetic
    from oracle import mel_ref

    a, b = tower(modules, 4), tower(modules, 4)
    tails = {}
    plan = [["p", "q"], ["p", "q"], ["q", "p", "r"], ["p", "r"], ["q", "r", "p"]]
    frames = {"p": 0, "q": 0, "r": 0}
    for t, sids in enumerate(plan):
        if t == 3:  # q leaves and comes back later with a fresh state
            a.reset("q")
            b.reset("q")
            frames["q"] = 0
            tails.pop("q", None)
        pcm = np.stack([synthetic.session_audio(5, {"p": 1, "q": 2, "r": 3}[s], 1, first_frame=frames[s], total_frames=8)[0]
                        for s in sids])
        mels = []
        for i, s in enumerate(sids):
            m, tails[s] = mel_ref.extract_single_frame(pcm[i], tails.get(s))
            mels.append(m)
        cur = tuple(cursor(s, frames[s]) for s in sids)
        pa = a.prepare_batch_pcm(torch.from_numpy(pcm).cuda(), cur)
        pb = b.prepare_batch(torch.from_numpy(np.stack(mels)).cuda(), cur)
        assert pa.reset_reasons == pb.reset_reasons
        assert_parity(pa.soft_tokens, pb.soft_tokens.float(), f"pcm vs mel tick {t}", 0.9999, 1e-2)
        pa.commit()
        pb.commit()
        for s in sids:
            frames[s] += 1
    a.close()
    b.close()


def _listener_batch(manifest_id, rows, pcm):
    """Stand-ins with the attribute layout of the reference's ListenerBatch /
    BatchRowDescriptor / ListenerFrame / ListenerSessionState
    (duplex_kernel/microbatch_contract.py)."""
    from types import SimpleNamespace as NS
    descs = tuple(NS(session_id=s, session_generation=g, state_epoch_id=e, frame_id=f, sequence_position=f)
                  for s, g, e, f in rows)
    frames = tuple(NS(session_id=s, frame_id=f, pcm=pcm[i]) for i, (s, _, _, f) in enumerate(rows))
    manifest = NS(manifest_id=manifest_id, batch_size=len(rows), rows=descs)
    states = tuple(NS(session_id=s) for s, _, _, _ in rows)
    return NS(manifest=manifest, frames=frames), states


def test_frontend_encode_batch_matches_reference_pcm_golden(pkg):
    """ListenerMicrobatchAudioFrontend.encode_batch from PCM (GPU mel) against
    the reference's PCM -> _extract_single_frame -> streaming tower run
    (tests/golden/pcm_tower_nt.npz), at the parity gate."""
    import json
    from pathlib import Path

    from gemma4_omni_b200.config import SMALL
    from gemma4_omni_b200.listener_frontend import ListenerMicrobatchAudioFrontend
    from gemma4_omni_b200.streaming_conformer import StreamingConformerAudioTower

    g = np.load(Path(__file__).resolve().parent / "golden" / "pcm_tower_nt.npz")
    t, e, _ = hf_modules(SMALL, int(g["seed_w"]))
    st = StreamingConformerAudioTower(t, e, device="cuda", dtype=torch.bfloat16, max_sessions=4)
    fe = ListenerMicrobatchAudioFrontend(None, None, device="cuda", dtype=torch.bfloat16, streaming_audio_tower=st)
    off = 0
    for k, rows in enumerate(json.loads(str(g["rows"]))):
        n = len(rows)
        batch, states = _listener_batch(f"m{k}", rows, g["pcm"][off:off + n])
        prepared = fe.encode_batch(batch, states)
        assert prepared.streaming_audio_input_shape == (n, 8, 128)
        assert [c.session_id for c in prepared.audio_stream_cursors] == [r[0] for r in rows]
        soft = torch.stack(prepared.audio_soft_tokens)
        assert soft.dtype == torch.bfloat16 and tuple(soft.shape) == (n, 2, SMALL.text_hidden)
        assert_parity(soft, torch.from_numpy(g["soft"][off:off + n]), f"soft tick {k}")
        assert_parity(torch.stack(prepared.audio_tower_raw_tokens), torch.from_numpy(g["raw"][off:off + n]),
                      f"raw tick {k}")
        prepared.commit()
        torch.cuda.synchronize()
        copy_ms, _, tower_ms = prepared.cuda_phase_timings_after_completion()
        assert copy_ms is not None and tower_ms is not None and tower_ms > 0
        off += n
    fe.close()


def test_frontend_assistant_mel_matches_reference_extractor(modules):
    """The assistant (reference) audio of each row becomes mel on the GPU with
    its tail carried per session across committed ticks; rows without
    reference audio use silence (listener_microbatch_frontend.py:792-809)."""
    from gemma4_omni_b200 import synthetic
    from gemma4_omni_b200.listener_frontend import ListenerMicrobatchAudioFrontend
    from oracle import mel_ref

    fe = ListenerMicrobatchAudioFrontend(None, None, device="cuda", dtype=torch.bfloat16,
                                         streaming_audio_tower=tower(modules, 4))
    tails = {}
    for t in range(4):
        sids = ["a", "b"] if t < 2 else ["b", "a", "c"]
        rows = [(s, 0, "e", t if s != "c" else t - 2) for s in sids]
        pcm = np.zeros((len(sids), 1280), np.float32)
        batch, states = _listener_batch(f"x{t}", rows, pcm)
        refs = []
        for i, (s, _, _, f) in enumerate(rows):
            ref = None if (s == "b" and t == 1) else synthetic.session_audio(8, ord(s), 1, first_frame=f,
                                                                              total_frames=4)[0]
            batch.frames[i].reference_pcm = ref
            refs.append(np.zeros(1280, np.float32) if ref is None else ref)
        p = fe.encode_batch(batch, states)
        want = []
        for s, ref in zip(sids, refs):
            m, tails[s] = mel_ref.extract_single_frame(ref, tails.get(s))
            want.append(m)
        np.testing.assert_allclose(p.assistant_mels.cpu().numpy(), np.stack(want), rtol=0, atol=2e-4)
        p.commit()
    fe.close()


def test_frontend_transaction_rules(modules):
    """One active manifest, single owner thread, poisoning after an abort."""
    import threading

    from gemma4_omni_b200.listener_frontend import ListenerMicrobatchAudioFrontend

    fe = ListenerMicrobatchAudioFrontend(None, None, device="cuda", dtype=torch.bfloat16,
                                         streaming_audio_tower=tower(modules, 4))
    pcm = np.zeros((2, 1280), np.float32)
    batch, states = _listener_batch("a", [("x", 0, "e", 0), ("y", 0, "e", 0)], pcm)
    p = fe.encode_batch(batch, states)
    with pytest.raises(RuntimeError, match="has not committed"):
        fe.encode_batch(*_listener_batch("b", [("x", 0, "e", 1)], pcm[:1]))
    with pytest.raises(RuntimeError, match="while a batch is prepared"):
        fe.close_session("x")
    errors = []

    def commit_elsewhere():
        try:
            p.commit()
            errors.append("committed from another thread")
        except RuntimeError as exc:
            errors.append(str(exc))

    th = threading.Thread(target=commit_elsewhere)
    th.start()
    th.join()
    assert errors and "single owner thread" in errors[0], errors
    p.commit()
    fe.close_session("x")
    p2 = fe.encode_batch(*_listener_batch("c", [("y", 0, "e", 1)], pcm[:1]))
    p2.abort()
    with pytest.raises(RuntimeError, match="poisoned"):
        fe.encode_batch(*_listener_batch("d", [("y", 0, "e", 1)], pcm[:1]))
    fe.close()
