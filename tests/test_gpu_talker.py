"""The two listener pieces next to the step: the stand-alone log-mel
(lb_mel_async, e.g. the assistant reference audio the reference frontend turns
into mel per row, listener_microbatch_frontend.py:792-809) and the FiLM adapter
at its Talker call site (lb_film_talker_async: apply_response_state_residual,
frame_residual_adapter.py:38-71), against the reference goldens and the CPU
oracle."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_parity, film_weights_from_engine
from oracle import film_ref

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def engine(cfg, nontrivial=True, rows=16):
    from gemma4_omni_b200 import runtime, synthetic
    eng = runtime.ListenerEngine(cfg, max_sessions=rows, max_rows=rows, weight_format=0)
    fw = synthetic.synthetic_film_weights(cfg, 12, nontrivial=nontrivial)
    fw["output.weight"] = fw["output.weight"] * 300.0  # a clearly non-trivial residual
    eng.load_weights(synthetic.synthetic_tower_weights(cfg, 11, nontrivial=nontrivial), fw)
    return eng


def test_standalone_mel_matches_reference_extractor(pkg):
    """3 streams x 6 frames, tails carried by the caller (first frame fresh)."""
    from gemma4_omni_b200.config import SMALL

    g = np.load(GOLD / "mel.npz")
    eng = engine(SMALL)
    pcm = torch.from_numpy(g["pcm"].reshape(3, 6, 1280)).cuda()
    tails = [torch.empty(3, 160, device="cuda") for _ in range(2)]
    mel = torch.empty(3, 8, 128, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    got = []
    for f in range(6):
        cur = pcm[:, f].contiguous()
        tin = None if f == 0 else tails[f % 2].data_ptr()
        assert eng.lib.lb_mel_async(eng._ctx, 3, cur.data_ptr(), tin, tails[(f + 1) % 2].data_ptr(),
                                    mel.data_ptr(), s) == 0
        got.append(mel.cpu().numpy().copy())
        np.testing.assert_array_equal(tails[(f + 1) % 2].cpu().numpy(), g["pcm"].reshape(3, 6, 1280)[:, f, -160:])
    got = np.stack(got, axis=1).reshape(18, 8, 128)
    np.testing.assert_allclose(got, g["mel"], rtol=0, atol=2e-4)
    assert np.abs(got - g["mel"]).mean() < 2e-5
    # aliasing the tails is refused
    t = tails[0].data_ptr()
    assert eng.lib.lb_mel_async(eng._ctx, 3, pcm.data_ptr(), t, t, mel.data_ptr(), s) == -1
    eng.close()


@pytest.mark.parametrize("cfg_name", ["SMALL", "FULL"])
def test_film_talker_placement_matches_reference_rule(pkg, cfg_name):
    """Cursor-selected response state (held at the last one past the text), the
    query untouched at generation step 0, the FiLM residual otherwise."""
    from gemma4_omni_b200 import config

    cfg = getattr(config, cfg_name)
    eng = engine(cfg)
    fw = film_weights_from_engine(eng)
    rng = torch.Generator().manual_seed(3)
    n, max_states = 21, 9
    hidden = torch.randn(n, max_states, cfg.text_hidden, generator=rng).to(torch.bfloat16)
    query = torch.randn(n, cfg.film_query_dim, generator=rng).to(torch.bfloat16)
    n_states = torch.randint(1, max_states + 1, (n,), generator=rng, dtype=torch.int32)
    steps = torch.randint(0, 14, (n,), generator=rng, dtype=torch.int32)
    steps[:3] = 0
    steps[3] = 50  # far past the text: the last state is held
    out = torch.empty(n, cfg.film_query_dim, dtype=torch.bfloat16, device="cuda")
    dev = [t.cuda() for t in (hidden, n_states, steps, query)]
    rc = eng.lib.lb_film_talker_async(eng._ctx, n, dev[0].data_ptr(), max_states, dev[1].data_ptr(),
                                      dev[2].data_ptr(), dev[3].data_ptr(), out.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert eng.status() == 0
    idx = torch.minimum(steps.long(), n_states.long() - 1)
    local = hidden[torch.arange(n), idx].float()
    ref = film_ref.film_forward(fw, local[:, None], query.float()[:, None])[:, 0]
    got = out.float().cpu()
    keep = steps == 0
    assert torch.equal(got[keep], query.float()[keep])
    assert_parity(got[~keep], ref[~keep], "talker film", 0.9999, 1e-2)
    # the residual is non-trivial, so the check is not vacuous
    assert (ref[~keep] - query.float()[~keep]).abs().max() > 1e-2
    # an invalid state count is flagged on the device
    bad = dev[1].clone()
    bad[0] = 0
    assert eng.lib.lb_film_talker_async(eng._ctx, n, dev[0].data_ptr(), max_states, bad.data_ptr(),
                                        dev[2].data_ptr(), dev[3].data_ptr(), out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream) == 0
    assert eng.status() & 32  # LB_DEV_BAD_ROW_COUNT
    eng.close()


def test_film_talker_is_refused_while_a_step_is_packed(pkg):
    from gemma4_omni_b200.config import SMALL

    eng = engine(SMALL)
    h = torch.zeros(2, dtype=torch.int32, device="cuda")
    z = torch.zeros(2, dtype=torch.int64, device="cuda")
    eng.pack(h.clone().copy_(torch.arange(2, dtype=torch.int32)), z, z, z)
    x = torch.zeros(2, 1, SMALL.text_hidden, dtype=torch.bfloat16, device="cuda")
    q = torch.zeros(2, SMALL.film_query_dim, dtype=torch.bfloat16, device="cuda")
    one = torch.ones(2, dtype=torch.int32, device="cuda")
    rc = eng.lib.lb_film_talker_async(eng._ctx, 2, x.data_ptr(), 1, one.data_ptr(), one.data_ptr(), q.data_ptr(),
                                      q.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == -3  # LB_ERR_STATE
    eng.abort()
    eng.close()


def _control6(lib, hidden, hidden_ld, phase, legal_bits, base, lora_a, lora_b, scaling):
    n = hidden.shape[0]
    logits = torch.empty(n, 6, device="cuda")
    packet = torch.empty(n, 4, device="cuda")
    rc = lib.lb_op_control6_head(n, hidden.data_ptr(), hidden_ld, None if phase is None else phase.data_ptr(),
                                 None if legal_bits is None else legal_bits.data_ptr(), base.data_ptr(),
                                 lora_a.data_ptr(), lora_b.data_ptr(), lora_a.shape[0], scaling,
                                 logits.data_ptr(), packet.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return logits.cpu(), packet.cpu()


def _bits(legal: torch.Tensor) -> torch.Tensor:
    return (legal.to(torch.uint8) << torch.arange(6, dtype=torch.uint8)).sum(1).to(torch.uint8).cuda()


def check_selection(logits, packet, ref_logits, ref_packet):
    # logits: fp32 sums in another order, and the bf16 product of the frozen
    # rows may round to the neighbouring bf16 value
    tol = 2 ** -7 * ref_logits.abs() + 1e-5
    assert bool(((logits - ref_logits).abs() <= tol).all()), (logits - ref_logits).abs().max()
    assert torch.equal(packet[:, 0], ref_packet[:, 0])
    # indices are exact unless two logits are within the tolerance of each other
    for i in range(len(packet)):
        for col in (1, 2):
            a, b = int(packet[i, col]), int(ref_packet[i, col])
            if a != b:
                assert abs(float(ref_logits[i, a] - ref_logits[i, b])) <= float(tol[i].max()) * 2, (i, col)
    torch.testing.assert_close(packet[:, 3], ref_packet[:, 3], rtol=1e-3, atol=1e-4)


def test_control6_head_matches_reference_golden(pkg):
    from gemma4_omni_b200 import _lib

    lib = _lib.load()
    g = np.load(GOLD / "control6.npz")
    hidden = torch.from_numpy(g["hidden"]).to(torch.bfloat16)
    # the rows sit as the first token of [n, 2, 1536] listener outputs (row stride 3072)
    pair = torch.zeros(hidden.shape[0], 2, 1536, dtype=torch.bfloat16)
    pair[:, 0] = hidden
    pair[:, 1] = -7.0
    base = torch.from_numpy(g["base_rows"]).to(torch.bfloat16).cuda()
    lora_a, lora_b = torch.from_numpy(g["lora_a"]).cuda(), torch.from_numpy(g["lora_b"]).cuda()
    legal = torch.from_numpy(g["legal"])
    for tag, phase in (("phase", torch.from_numpy(g["phase"]).cuda()), ("nophase", None)):
        logits, packet = _control6(lib, pair.cuda(), 3072, phase, _bits(legal), base, lora_a, lora_b,
                                   float(g["scaling"]))
        check_selection(logits, packet, torch.from_numpy(g[f"{tag}_logits"]), torch.from_numpy(g[f"{tag}_packet"]))


@pytest.mark.parametrize("n,rank", [(1, 16), (300, 16), (4096, 8), (33, 64)])
def test_control6_head_matches_oracle(pkg, n, rank):
    from gemma4_omni_b200 import _lib
    from oracle import control6_ref

    lib = _lib.load()
    g = torch.Generator().manual_seed(n + rank)
    hidden = torch.randn(n, 1536, generator=g).to(torch.bfloat16)
    phase = torch.randn(n, 4, generator=g)
    legal = torch.rand(n, 6, generator=g) < 0.5
    legal[legal.sum(1) == 0, 2] = True
    base = (torch.randn(6, 1536, generator=g) * 0.05).to(torch.bfloat16)
    lora_a = torch.randn(rank, 1540, generator=g) * 0.02
    lora_b = torch.randn(6, rank, generator=g) * 0.05
    ref_logits, ref_packet = control6_ref.control6_head(hidden, phase, legal, base, lora_a, lora_b, 2.0)
    logits, packet = _control6(lib, hidden.cuda(), 1536, phase.cuda(), _bits(legal), base.cuda(), lora_a.cuda(),
                               lora_b.cuda(), 2.0)
    check_selection(logits, packet, ref_logits, ref_packet)
