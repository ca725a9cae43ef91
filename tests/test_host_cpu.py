"""CPU-only checks: the C-ABI library loads and exports what the header declares,
and the host-side logic (tables, weight preparation, synthetic workloads)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def header_functions() -> list[str]:
    text = (ROOT / "include" / "listener_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def built_lib(pkg):
    from gemma4_omni_b200 import build
    return build.build_library()


def test_library_loads_and_exports_every_declared_symbol(built_lib, pkg):
    from gemma4_omni_b200 import _lib
    lib = ctypes.CDLL(str(built_lib))
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers the same surface
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_config_struct_matches_header(pkg):
    from gemma4_omni_b200 import _lib
    text = (ROOT / "include" / "listener_b200.h").read_text()
    body = text[text.index("typedef struct lb_config {"):text.index("} lb_config;")]
    fields = re.findall(r"\b([a-z_0-9]+)\s*[,;]", re.sub(r"/\*.*?\*/", "", body, flags=re.S))
    assert fields == [f for f, _ in _lib.LbConfig._fields_]


def test_frontend_tables_match_transformers(pkg):
    from gemma4_omni_b200.frontend_tables import hann_window, mel_filterbank
    from transformers.models.gemma4.feature_extraction_gemma4 import Gemma4AudioFeatureExtractor
    fe = Gemma4AudioFeatureExtractor()
    np.testing.assert_array_equal(hann_window(), fe.window.astype(np.float32))
    np.testing.assert_allclose(mel_filterbank(), fe.mel_filters, rtol=0, atol=1e-15)


def test_int8_quantisation_is_per_channel_and_bounded(pkg):
    from gemma4_omni_b200.weights import dequantize, quantize_int8
    rng = np.random.default_rng(0)
    w = rng.standard_normal((256, 512)).astype(np.float32) * 0.02
    w[3] = 0.0
    q, s = quantize_int8(w)
    assert q.dtype == np.int8 and s.dtype == np.float16 and s.shape == (256,)
    assert np.abs(q).max() <= 127
    err = np.abs(dequantize(q, s) - w)
    assert (err <= s.astype(np.float32)[:, None] * 0.5 + 1e-7).all()
    assert np.all(dequantize(q, s)[3] == 0)


def test_prepare_uploads_cover_the_context_tensor_table(pkg):
    from gemma4_omni_b200 import synthetic, weights
    from gemma4_omni_b200.config import SMALL
    up, eff = weights.prepare(SMALL, synthetic.synthetic_tower_weights(SMALL, 1),
                              synthetic.synthetic_film_weights(SMALL, 2), 1)
    names = {n for n, _, _ in up}
    assert "layers.0.self_attn.relative_keys" in names
    assert "layers.1.self_attn.query_scale" in names
    assert "film.output.weight:scale" in names
    assert "frontend.mel_filters" in names
    # effective int8 weights are exactly the dequantised uploads
    q = dict((n, a) for n, a, _ in up)
    np.testing.assert_array_equal(
        eff["output_proj.weight"],
        weights.dequantize(q["output_proj.weight"], q["output_proj.weight:scale"]))


def test_relative_keys_match_the_reference_rel_pos_encoding(pkg):
    from gemma4_omni_b200.weights import relative_keys
    from transformers.models.gemma4.configuration_gemma4 import Gemma4AudioConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4AudioRelPositionalEncoding
    cfg = Gemma4AudioConfig(hidden_size=256, num_attention_heads=2)
    enc = Gemma4AudioRelPositionalEncoding(cfg)
    emb = enc(torch.zeros(1, 2, 256))
    w = np.random.default_rng(1).standard_normal((256, 256)).astype(np.float32) * 0.02
    ref = (emb.float().reshape(13, 256) @ torch.from_numpy(w).t()).numpy()
    np.testing.assert_allclose(relative_keys(w, 256), ref, rtol=1e-5, atol=1e-6)


def test_synthetic_workloads_are_seeded_and_shaped(pkg):
    from gemma4_omni_b200 import synthetic
    a = synthetic.session_audio(1, 2, 3)
    b = synthetic.session_audio(1, 2, 3)
    assert a.shape == (3, 1280) and a.dtype == np.float32
    np.testing.assert_array_equal(a, b)
    assert 0.05 < a.std() < 0.2
    ar = synthetic.ArrivalProcess(1024, seed=7)
    counts = []
    joins = []
    for _ in range(50):
        lanes, sids, frames, new = ar.step()
        counts.append(len(lanes))
        joins.append(int(new.sum()))
    assert set(counts) == {1024}  # lanes keep the concurrency fixed
    assert 1.0 < np.mean(joins) < 8.0  # about 1024/300 sessions join (and leave) per step
    pool = synthetic.ArrivalProcess(256, seed=7, mode="pool")
    sizes = [len(pool.step()[0]) for _ in range(600)]
    assert max(sizes) <= 256 and min(sizes[1:400]) >= 1


def test_config_validation_rejects_unsupported_shapes(pkg):
    from gemma4_omni_b200.config import FULL, SMALL, ListenerConfig
    FULL.validate()
    SMALL.validate()
    with pytest.raises(ValueError):
        ListenerConfig(hidden=1000).validate()
    with pytest.raises(ValueError):
        ListenerConfig(conv_kernel=3).validate()


def test_nontrivial_weights_cover_every_identity_parameter(pkg):
    """The parity weight set: norm weights != 1, per_dim_scale != 0, biases != 0,
    finite and distinct q/k/v clip bounds on every clippable linear, and every
    value exactly representable in bf16 (a bf16 checkpoint)."""
    import numpy as np
    import torch
    from gemma4_omni_b200 import synthetic
    from gemma4_omni_b200.config import SMALL

    w = synthetic.synthetic_tower_weights(SMALL, 9, nontrivial=True)
    base = synthetic.synthetic_tower_weights(SMALL, 9)
    for name, shape, init in synthetic.tower_weight_shapes(SMALL):
        if init == "normal":  # the default draws are kept (then rounded to bf16)
            np.testing.assert_allclose(w[name], base[name], rtol=2 ** -8, atol=0)
        else:
            assert not np.array_equal(w[name], base[name]), name
    for prefix, _ in synthetic.clippable_linears(SMALL):
        b = [float(w[f"{prefix}.{k}"]) for k in ("input_min", "input_max", "output_min", "output_max")]
        assert all(np.isfinite(b)) and b[0] < 0 < b[1] and b[2] < 0 < b[3], prefix
    qb = [float(w[f"layers.0.self_attn.{p}.input_max"]) for p in ("q_proj", "k_proj", "v_proj")]
    assert len(set(qb)) == 3
    for k, v in w.items():
        t = torch.from_numpy(np.array(v, dtype=np.float32))
        assert torch.equal(t.to(torch.bfloat16).float(), t), k
    f = synthetic.synthetic_film_weights(SMALL, 9, nontrivial=True)
    assert not np.allclose(f["query_norm.bias"], 0) and not np.allclose(f["response_norm.weight"], 1)
