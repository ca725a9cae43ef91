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


def hf_modules(cfg, seed):
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
    w = synthetic_tower_weights(cfg, seed)
    tower.load_state_dict({k: torch.from_numpy(v) for k, v in w.items() if not k.startswith("embed.")}, strict=False)
    embed.load_state_dict({k[6:]: torch.from_numpy(v) for k, v in w.items() if k.startswith("embed.")})
    return tower, embed, w


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


def test_reorder_reset_gap_and_epoch_do_not_cross_contaminate(modules):
    chunks = torch.randn((9, 8, 128), generator=torch.Generator().manual_seed(125))
    shared, sep_a, sep_b = tower(modules), tower(modules), tower(modules)
    for f in range(4):
        pair = chunks[f:f + 1].expand(2, -1, -1).clone()
        got = commit_tick(shared, pair, (cursor("A", f), cursor("B", f)))[0]
        ra = commit_tick(sep_a, chunks[f:f + 1], (cursor("A", f),))[0]
        rb = commit_tick(sep_b, chunks[f:f + 1], (cursor("B", f),))[0]
        assert_parity(got[0:1], ra, "A", 0.99999, 5e-3)
        assert_parity(got[1:2], rb, "B", 0.99999, 5e-3)
    ba = commit_tick(shared, chunks[4:5].expand(2, -1, -1).clone(), (cursor("B", 4), cursor("A", 4)))[0]
    assert_parity(ba[0:1], commit_tick(sep_b, chunks[4:5], (cursor("B", 4),))[0], "B reordered", 0.99999, 5e-3)
    assert_parity(ba[1:2], commit_tick(sep_a, chunks[4:5], (cursor("A", 4),))[0], "A reordered", 0.99999, 5e-3)
    shared.reset("A", 0, "epoch-0")
    p = shared.prepare_batch(torch.cat((chunks[5:6], chunks[6:7])).cuda(), (cursor("B", 5), cursor("A", 20)))
    assert p.reset_reasons == ("continue", "identity_reset")
    reset_a = p.raw_tokens.float().cpu()[1:2]
    p.commit()
    fresh = tower(modules)
    assert_parity(reset_a, commit_tick(fresh, chunks[6:7], (cursor("A", 20),))[0], "reset A", 0.99999, 5e-3)
    p = shared.prepare_batch(chunks[7:8].cuda(), (cursor("A", 22),))
    assert p.reset_reasons == ("gap_or_cursor_mismatch",)
    p.commit()
    p = shared.prepare_batch(chunks[8:9].cuda(), (cursor("A", 0, generation=1, epoch="epoch-1"),))
    assert p.reset_reasons == ("identity_reset",)
    epoch = p.raw_tokens.float().cpu()
    p.commit()
    fresh2 = tower(modules)
    ref = commit_tick(fresh2, chunks[8:9], (cursor("A", 0, generation=1, epoch="epoch-1"),))[0]
    assert_parity(epoch, ref, "epoch change", 0.99999, 5e-3)
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
    eff = {k: torch.from_numpy(bf16_round(v)) for k, v in w.items()}
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
