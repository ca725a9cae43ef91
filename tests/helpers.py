"""Test helpers: engine construction, golden-trace replay and parity metrics."""
from __future__ import annotations

import json

import numpy as np
import torch

from oracle import conformer_ref

# Parity gate of the listener step (bf16 GPU vs fp32 reference):
# per-frame cosine >= 0.999 and max|a-b| / max|b| <= 2e-2.
COS_MIN = 0.999
REL_MAX = 2e-2


def frame_cos(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    a = a.double().reshape(-1, a.shape[-1])
    b = b.double().reshape(-1, b.shape[-1])
    return torch.nn.functional.cosine_similarity(a, b, dim=-1)


def frame_rel(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    a = a.double().reshape(-1, a.shape[-1])
    b = b.double().reshape(-1, b.shape[-1])
    return (a - b).abs().amax(-1) / b.abs().amax(-1)


def assert_parity(gpu: torch.Tensor, ref: torch.Tensor, what: str, cos_min=COS_MIN, rel_max=REL_MAX):
    c = frame_cos(gpu.float().cpu(), ref.float().cpu())
    r = frame_rel(gpu.float().cpu(), ref.float().cpu())
    assert c.min().item() >= cos_min, f"{what}: min cosine {c.min().item():.6f} < {cos_min}"
    assert r.max().item() <= rel_max, f"{what}: max rel error {r.max().item():.3e} > {rel_max}"
    return c.min().item(), r.max().item()


def oracle_config(cfg) -> conformer_ref.OracleConfig:
    return conformer_ref.OracleConfig(hidden=cfg.hidden, layers=cfg.layers, heads=cfg.heads, ffn=cfg.ffn,
                                      sub_ch0=cfg.sub_ch0, sub_ch1=cfg.sub_ch1, output_dims=cfg.output_dims,
                                      text_hidden=cfg.text_hidden)


def oracle_from_engine(engine) -> conformer_ref.OracleConformer:
    w = {k: torch.from_numpy(v) for k, v in engine.effective_weights.items() if not k.startswith("film.")}
    return conformer_ref.OracleConformer(w, oracle_config(engine.cfg))


def film_weights_from_engine(engine) -> dict:
    return {k[5:]: torch.from_numpy(v) for k, v in engine.effective_weights.items() if k.startswith("film.")}


class HandleBook:
    """Maps session ids to dense handles and (generation, epoch) to int64 keys."""

    def __init__(self):
        self.handles: dict[str, int] = {}
        self.keys: dict[tuple, int] = {}

    def handle(self, sid: str) -> int:
        return self.handles.setdefault(sid, len(self.handles))

    def key(self, gen, epoch) -> int:
        return self.keys.setdefault((gen, epoch), len(self.keys))

    def arrays(self, rows, device="cuda"):
        h = torch.tensor([self.handle(r[0]) for r in rows], dtype=torch.int32, device=device)
        k = torch.tensor([self.key(r[1], r[2]) for r in rows], dtype=torch.int64, device=device)
        f = torch.tensor([r[3] for r in rows], dtype=torch.int64, device=device)
        q = torch.tensor([r[4] if len(r) > 4 else r[3] for r in rows], dtype=torch.int64, device=device)
        return h, k, f, q


def mask_bits(mask: np.ndarray) -> torch.Tensor:
    bits = (mask.astype(np.uint8) << np.arange(8, dtype=np.uint8)[None, :]).sum(axis=1).astype(np.uint8)
    return torch.from_numpy(bits).cuda()


def golden_rows(g):
    return json.loads(str(g["rows"])), json.loads(str(g["reasons"]))


def replay_coordinator(golden: dict, order_fn) -> int:
    """Replays the reference ListenerMicrobatchCoordinator golden trace
    (listener_microbatch.py:144-279) through ``order_fn(heads, now_ns,
    coalesce_ns, registered) -> (rows, reason)``: per-session FIFO queues with a
    global submission counter, the head of every queue as a candidate, no take
    while a batch is in flight.  Asserts every take's rows and reason; returns
    the number of takes checked."""
    from collections import deque

    queues = {sid: deque() for sid in golden["registrations"]}
    order = 0
    in_flight = False
    checked = 0
    for ev in golden["events"]:
        if ev["kind"] == "enqueue":
            queues[ev["sid"]].append((ev["ready_at"], order, ev["sid"], ev["frame"]))
            order += 1
        elif ev["kind"] == "complete":
            assert in_flight
            in_flight = False
        else:
            if ev["active"]:
                assert in_flight and ev["rows"] is None
                continue
            assert not in_flight
            heads = [q[0][:3] for q in queues.values() if q]
            rows, reason = order_fn(heads, ev["now"], golden["coalesce_ns"], len(golden["registrations"]))
            if ev["rows"] is None:
                assert (rows, reason) == ([], None), (ev, rows, reason)
            else:
                got = []
                for h in rows:
                    ready_at, sub, sid, frame = queues[h[2]].popleft()
                    assert (ready_at, sub) == (h[0], h[1])
                    got.append([sid, frame])
                assert got == ev["rows"] and reason == ev["reason"], (ev, got, reason)
                in_flight = True
            checked += 1
    return checked


def replay_oracle_trace(model, g):
    """Drives the CPU oracle through a golden tower trace (rows, reasons, slots,
    mel, mask); returns (raw, soft, sub, layers) stacked like the golden."""
    rows = json.loads(str(g["rows"]))
    reasons = json.loads(str(g["reasons"]))
    slots = g["slots"]
    state: dict[int, dict] = {}
    zero = {k: v[0] for k, v in conformer_ref.zero_state(model.cfg, 1).items()}
    raws, softs, subs, layers = [], [], [], []
    off = 0
    for tick_rows, tick_reasons in zip(rows, reasons):
        n = len(tick_rows)
        sl = [int(s) for s in slots[off:off + n]]
        st = {k: torch.stack([state.get(s, zero)[k] for s in sl]) for k in zero}
        reset = torch.tensor([r != "continue" for r in tick_reasons])
        mel = torch.from_numpy(g["mel"][off:off + n])
        mask = torch.from_numpy(g["mask"][off:off + n])
        raw, soft, sub, lay, nxt = model.step(mel, mask, st, reset)
        for i, s in enumerate(sl):
            state[s] = {k: v[i] for k, v in nxt.items()}
        raws.append(raw)
        softs.append(soft)
        subs.append(sub)
        layers.append(torch.stack(lay))
        off += n
    return torch.cat(raws), torch.cat(softs), torch.cat(subs), torch.cat(layers, dim=1)
